"""ctypes binding of the CPU oracle (TEST INFRASTRUCTURE ONLY).

The oracle (furnace_oracle.cpp in this folder) restates the furnace reference's
CPU decode path -- src/quant.rs, src/tensor.rs, src/model.rs, src/sampler.rs and
src/generate.rs -- and is the checker the CUDA path is compared against.  Only
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this
module; the product never does.

Parity is pinned by tests/test_oracle_golden.py: the reference's own
known-answer tests (quant.rs, tensor.rs, model.rs, sampler.rs, generate.rs,
gguf.rs) and gguf-py 0.19.0 dequantization golden vectors under tests/golden/.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")

F32, F16, Q5_0, Q8_0, Q4_K, Q6_K = 0, 1, 6, 8, 12, 14
BLOCK = {F32: (1, 4), F16: (1, 2), Q8_0: (32, 34), Q5_0: (32, 22), Q4_K: (256, 144), Q6_K: (256, 210)}

_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        P, S, U32, U64, F, I = C.c_void_p, C.c_size_t, C.c_uint32, C.c_uint64, C.c_float, C.c_int
        fp = C.POINTER(C.c_float)
        u32p = C.POINTER(C.c_uint32)
        sig = {
            "orc_last_error": (C.c_char_p, []),
            "orc_set_threads": (None, [I]),
            "orc_threads": (I, []),
            "orc_f16_to_f32": (F, [C.c_uint16]),
            "orc_dequantize": (I, [U32, P, S, S, fp]),
            "orc_matmul_quant": (I, [fp, S, P, S, S, S, U32, fp]),
            "orc_matmul_f32": (None, [fp, S, fp, S, S, fp]),
            "orc_dot": (F, [fp, fp, S]),
            "orc_rmsnorm": (None, [fp, S, S, fp, F, fp]),
            "orc_softmax": (None, [fp, S, S]),
            "orc_silu": (None, [fp, S, fp]),
            "orc_swiglu": (None, [fp, fp, S, fp]),
            "orc_rope": (None, [fp, S, S, S, F, S]),
            "orc_attention": (None, [fp, fp, fp, S, S, S, S, fp]),
            "orc_argmax": (U32, [fp, S]),
            "orc_gguf_parse_bytes": (I, [P, S, u32p, C.POINTER(S), C.POINTER(S), C.POINTER(S)]),
            "orc_model_open": (P, [C.c_char_p, I]),
            "orc_model_close": (None, [P]),
            "orc_model_config": (None, [P, u32p, fp]),
            "orc_model_truncate": (None, [P, U32]),
            "orc_kv_new": (P, [P, S]),
            "orc_kv_free": (None, [P]),
            "orc_kv_set_f16": (None, [P, I]),
            "orc_float_to_half": (C.c_uint16, [F]),
            "orc_kv_len": (S, [P]),
            "orc_kv_set_len": (None, [P, S]),
            "orc_kv_read": (I, [P, S, I, S, fp]),
            "orc_kv_write": (I, [P, S, I, S, fp]),
            "orc_forward_cached": (I, [P, P, u32p, S, fp]),
            "orc_forward_last": (I, [P, u32p, S, fp]),
            "orc_embed": (I, [P, u32p, S, fp]),
            "orc_layer_forward": (I, [P, P, S, fp, S, S, fp]),
            "orc_tensor": (I, [P, C.c_char_p, u32p, C.POINTER(U64), u32p, C.POINTER(C.c_void_p), C.POINTER(S)]),
            "orc_sampler_new": (P, [F, S, F, F, U64]),
            "orc_sampler_free": (None, [P]),
            "orc_sampler_sample": (U32, [P, fp, S, u32p, S]),
            "orc_sampler_draws": (U64, [P]),
            "orc_sampler_filtered": (S, [P, fp, S, u32p, fp]),
            "orc_repeat_penalty": (None, [fp, u32p, S, F]),
            "orc_generate": (I, [P, u32p, S, S, u32p, S, P, S, u32p, C.POINTER(S), fp,
                                 C.POINTER(C.c_double), C.POINTER(C.c_double)]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _fp(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _u32p(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint32))


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _err():
    return lib().orc_last_error().decode()


class OracleError(RuntimeError):
    pass


def set_threads(n: int):
    lib().orc_set_threads(int(n))


def threads() -> int:
    return lib().orc_threads()


def float_to_half(f: float) -> int:
    """binary32 -> binary16 bits, round to nearest even."""
    return lib().orc_float_to_half(f)


def f16_to_f32(h: int) -> float:
    return lib().orc_f16_to_f32(h)


def dequantize(dtype: int, raw: bytes, n: int) -> np.ndarray:
    """quant::dequantize (src/quant.rs:261-281)."""
    buf = np.frombuffer(bytes(raw), dtype=np.uint8)
    out = np.zeros(n, dtype=np.float32)
    if lib().orc_dequantize(dtype, buf.ctypes.data, buf.size, n, _fp(out)) != 0:
        raise OracleError(_err())
    return out


def matmul_quant(a: np.ndarray, raw: bytes, d_out: int, d_in: int, dtype: int) -> np.ndarray:
    """quant::matmul_quant (src/quant.rs:170-193): a [seq, in] x W[out, in]^T."""
    a = _f32(a).reshape(-1, d_in)
    buf = np.frombuffer(bytes(raw), dtype=np.uint8)
    out = np.zeros((a.shape[0], d_out), dtype=np.float32)
    if lib().orc_matmul_quant(_fp(a), a.shape[0], buf.ctypes.data, buf.size, d_out, d_in, dtype, _fp(out)) != 0:
        raise OracleError(_err())
    return out


def matmul(a: np.ndarray, w: np.ndarray) -> np.ndarray:
    """tensor::matmul (src/tensor.rs:74-80)."""
    a, w = _f32(a), _f32(w)
    out = np.zeros((a.shape[0], w.shape[0]), dtype=np.float32)
    lib().orc_matmul_f32(_fp(a), a.shape[0], _fp(w), w.shape[0], w.shape[1], _fp(out))
    return out


def dot(a, b) -> float:
    a, b = _f32(a), _f32(b)
    return lib().orc_dot(_fp(a), _fp(b), a.size)


def rmsnorm(x, w, eps) -> np.ndarray:
    x, w = _f32(x), _f32(w)
    cols = w.size
    out = np.zeros_like(x)
    lib().orc_rmsnorm(_fp(x), x.size // cols, cols, _fp(w), eps, _fp(out))
    return out


def softmax(x) -> np.ndarray:
    x = _f32(x).copy()
    cols = x.shape[-1]
    lib().orc_softmax(_fp(x), x.size // cols, cols)
    return x


def silu(x) -> np.ndarray:
    x = _f32(x)
    out = np.zeros_like(x)
    lib().orc_silu(_fp(x), x.size, _fp(out))
    return out


def swiglu(g, u) -> np.ndarray:
    g, u = _f32(g), _f32(u)
    out = np.zeros_like(g)
    lib().orc_swiglu(_fp(g), _fp(u), g.size, _fp(out))
    return out


def rope(x, n_heads, head_dim, theta, start_pos) -> np.ndarray:
    x = _f32(x).copy()
    seq = x.size // (n_heads * head_dim)
    lib().orc_rope(_fp(x), seq, n_heads, head_dim, theta, start_pos)
    return x


def attention(q, k, v, n_heads, n_kv_heads, head_dim) -> np.ndarray:
    """attention_scores + attention_apply, uncached (src/model.rs:224-290)."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    seq = q.size // (n_heads * head_dim)
    out = np.zeros((seq, n_heads * head_dim), dtype=np.float32)
    lib().orc_attention(_fp(q), _fp(k), _fp(v), seq, n_heads, n_kv_heads, head_dim, _fp(out))
    return out


def argmax(x) -> int:
    x = _f32(x)
    return int(lib().orc_argmax(_fp(x), x.size))


def parse_gguf_bytes(data: bytes):
    """Returns (version, n_tensors, n_meta, data_start) or raises OracleError."""
    buf = np.frombuffer(bytes(data), dtype=np.uint8) if len(data) else np.zeros(1, np.uint8)
    v = C.c_uint32()
    nt, nm, ds = C.c_size_t(), C.c_size_t(), C.c_size_t()
    if lib().orc_gguf_parse_bytes(buf.ctypes.data, len(data), C.byref(v), C.byref(nt), C.byref(nm), C.byref(ds)) != 0:
        raise OracleError(_err())
    return v.value, nt.value, nm.value, ds.value


class Model:
    """Model::load + forward_cached / forward_last (src/model.rs:511-601)."""

    def __init__(self, path: str, use_f32: bool = False):
        self._h = lib().orc_model_open(path.encode(), int(use_f32))
        if not self._h:
            raise OracleError(_err())
        u = np.zeros(8, np.uint32)
        f = np.zeros(2, np.float32)
        lib().orc_model_config(self._h, _u32p(u), _fp(f))
        (self.n_layers, self.n_heads, self.n_kv_heads, self.hidden, self.ffn, self.head_dim, self.vocab,
         self.context_length) = (int(x) for x in u)
        self.rope_theta, self.rms_eps = float(f[0]), float(f[1])

    def close(self):
        if self._h:
            lib().orc_model_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def truncate(self, n_layers: int):
        lib().orc_model_truncate(self._h, n_layers)
        self.n_layers = min(self.n_layers, n_layers)

    def kv_new(self, max_ctx: int, kv_dtype: int = 0) -> "KvCache":
        return KvCache(self, max_ctx, kv_dtype)

    def forward_cached(self, tokens, cache: "KvCache") -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.zeros(self.vocab, np.float32)
        if lib().orc_forward_cached(self._h, cache._h, _u32p(t), t.size, _fp(out)) != 0:
            raise OracleError(_err())
        return out

    def forward_last(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.zeros(self.vocab, np.float32)
        if lib().orc_forward_last(self._h, _u32p(t), t.size, _fp(out)) != 0:
            raise OracleError(_err())
        return out

    def embed(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.zeros((t.size, self.hidden), np.float32)
        if lib().orc_embed(self._h, _u32p(t), t.size, _fp(out)) != 0:
            raise OracleError(_err())
        return out

    def layer_forward(self, cache, layer: int, x, start_pos: int) -> np.ndarray:
        x = _f32(x).reshape(-1, self.hidden)
        out = np.zeros_like(x)
        h = cache._h if cache is not None else None
        if lib().orc_layer_forward(self._h, h, layer, _fp(x), x.shape[0], start_pos, _fp(out)) != 0:
            raise OracleError(_err())
        return out

    def tensor(self, name: str):
        """(dtype, dims in ggml order, raw bytes) of a GGUF tensor."""
        dt, nd = C.c_uint32(), C.c_uint32()
        dims = (C.c_uint64 * 4)()
        raw, nb = C.c_void_p(), C.c_size_t()
        if lib().orc_tensor(self._h, name.encode(), C.byref(dt), dims, C.byref(nd), C.byref(raw), C.byref(nb)) != 0:
            raise OracleError(_err())
        return dt.value, [dims[i] for i in range(nd.value)], C.string_at(raw.value, nb.value)

    def generate(self, prompt, max_new: int, stop_ids=(), sampler: "Sampler" = None, max_ctx: int = None,
                 keep_logits: bool = False):
        """generate (src/generate.rs:83-157).  Returns (ids, step_logits|None,
        prefill_seconds, decode_seconds)."""
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        st = np.ascontiguousarray(list(stop_ids) or [0], dtype=np.uint32)
        sampler = sampler or Sampler(0.0, 1, 1.0, 1.0, 0)
        max_ctx = max_ctx or (p.size + max_new)
        ids = np.zeros(max(1, max_new), np.uint32)
        n_out = C.c_size_t()
        logits = np.zeros((max(1, max_new), self.vocab), np.float32) if keep_logits else None
        pf, dc = C.c_double(), C.c_double()
        lp = _fp(logits) if keep_logits else C.cast(None, C.POINTER(C.c_float))
        rc = lib().orc_generate(self._h, _u32p(p), p.size, max_new, _u32p(st), len(stop_ids), sampler._h, max_ctx,
                                _u32p(ids), C.byref(n_out), lp, C.byref(pf), C.byref(dc))
        if rc != 0:
            raise OracleError(_err())
        n = n_out.value
        return ids[:n].copy(), (logits[:n] if keep_logits else None), pf.value, dc.value


class KvCache:
    """KvCache (src/model.rs:321-363)."""

    def __init__(self, model: Model, max_ctx: int, kv_dtype: int = 0):
        """kv_dtype 1: elements kept as IEEE binary16, rounded to nearest even
        when appended (the device's FZ_KV_F16 cache); 0: f32 (the reference)."""
        self.model = model
        self.max_ctx = max_ctx
        self._h = lib().orc_kv_new(model._h, max_ctx)
        if kv_dtype:
            lib().orc_kv_set_f16(self._h, 1)

    def __del__(self):
        try:
            if self._h:
                lib().orc_kv_free(self._h)
        except Exception:
            pass

    @property
    def len(self) -> int:
        return lib().orc_kv_len(self._h)

    @len.setter
    def len(self, n: int):
        lib().orc_kv_set_len(self._h, n)

    def read(self, layer: int, which_v: bool, n: int) -> np.ndarray:
        kvd = self.model.n_kv_heads * self.model.head_dim
        out = np.zeros((n, kvd), np.float32)
        if lib().orc_kv_read(self._h, layer, int(which_v), n, _fp(out)) != 0:
            raise OracleError(_err())
        return out

    def fill_synthetic(self, n: int, seed: int = 0, scale: float = 1.0):
        """Rows [0, n) of every layer's K and V set to seeded N(0, scale^2)
        values and len = n: a long context for timing decode steps (their
        cost does not depend on the cached values)."""
        kvd = self.model.n_kv_heads * self.model.head_dim
        rng = np.random.default_rng(seed)
        for layer in range(self.model.n_layers):
            for which in (0, 1):
                rows = np.ascontiguousarray((rng.standard_normal((n, kvd)) * scale).astype(np.float32))
                if lib().orc_kv_write(self._h, layer, which, n, _fp(rows)) != 0:
                    raise OracleError(_err())
        self.len = n


class Sampler:
    """Sampler (src/sampler.rs:57-155)."""

    def __init__(self, temperature, top_k, top_p, repeat_penalty, seed):
        self._h = lib().orc_sampler_new(temperature, top_k, top_p, repeat_penalty, seed)

    def __del__(self):
        try:
            lib().orc_sampler_free(self._h)
        except Exception:
            pass

    def sample(self, logits, recent=()) -> int:
        lg = _f32(logits)
        r = np.ascontiguousarray(list(recent) or [0], dtype=np.uint32)
        return int(lib().orc_sampler_sample(self._h, _fp(lg), lg.size, _u32p(r), len(recent)))

    def draws(self) -> int:
        return int(lib().orc_sampler_draws(self._h))

    def filtered(self, logits):
        lg = _f32(logits)
        ids = np.zeros(lg.size, np.uint32)
        pr = np.zeros(lg.size, np.float32)
        n = lib().orc_sampler_filtered(self._h, _fp(lg), lg.size, _u32p(ids), _fp(pr))
        return [(int(ids[i]), float(pr[i])) for i in range(n)]


def repeat_penalty(logits, recent, penalty) -> np.ndarray:
    lg = _f32(logits).copy()
    r = np.ascontiguousarray(list(recent) or [0], dtype=np.uint32)
    lib().orc_repeat_penalty(_fp(lg), _u32p(r), len(recent), penalty)
    return lg
