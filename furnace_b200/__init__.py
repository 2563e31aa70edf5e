"""furnace-b200: the furnace decode token loop on B200 (sm_100a).

Python mirror of the reference's internal API (the reference is a Rust
binary crate; these names follow its modules), bound to libfurnace_cuda.so
through its C ABI (include/furnace.h):

    GgufFile.open(path)                      src/gguf.rs:366
    GgufFile.tensor(name)                    src/gguf.rs:412
    Config.from_gguf(file)                   src/model.rs:41
    Model.load(file)                         src/model.rs:520
    KvCache(model, max_ctx)                  src/model.rs:330
    Model.forward_cached(tokens, cache)      src/model.rs:579
    quant.dequantize / quant.matmul_quant    src/quant.rs:261, :170
    generate(model, prompt, max_new, ...)    src/generate.rs:83 (greedy)

Errors raise FurnaceError carrying the library's status code and message.
There is no CPU fallback: when the CUDA library cannot be loaded or a call
needs a GPU that is absent, the call raises.
"""

from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

from . import build as _build

F32, F16, Q5_0, Q8_0, Q4_K, Q6_K = 0, 1, 6, 8, 12, 14
BLOCK = {F32: (1, 4), F16: (1, 2), Q8_0: (32, 34), Q5_0: (32, 22), Q4_K: (256, 144), Q6_K: (256, 210)}
TYPE_NAMES = {F32: "F32", F16: "F16", Q5_0: "Q5_0", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K"}

FZ_OK, FZ_EINVAL, FZ_EFORMAT, FZ_EIO, FZ_ECUDA, FZ_ENOMEM, FZ_ETIMEOUT, FZ_ESPACE = range(8)
FZ_KV_F32, FZ_KV_F16 = 0, 1  # KV cache element types

# Every symbol include/furnace.h declares.
EXPORTS = [
    "fz_last_error", "fz_version", "fz_open", "fz_open_bytes", "fz_file_free", "fz_file_info", "fz_tensor_at",
    "fz_tensor", "fz_meta_u32", "fz_meta_f32", "fz_meta_str", "fz_meta_array_len", "fz_config_from_gguf",
    "fz_model_load", "fz_model_free", "fz_model_config", "fz_model_bytes", "fz_kv_new", "fz_kv_free", "fz_kv_len",
    "fz_kv_set_len", "fz_kv_reset", "fz_kv_bytes", "fz_kv_read", "fz_forward", "fz_forward_last", "fz_decode_greedy",
    "fz_dequant", "fz_matmul_quant", "fz_gemv", "fz_weight_upload", "fz_weight_free", "fz_matmul_quant_dev",
    "fz_step_profile", "fz_model_stream", "fz_dequant_dev_noalloc", "fz_tp_slice_of", "fz_tp_unique_id",
    "fz_model_load_tp", "fz_sampler_new", "fz_sampler_free", "fz_sampler_draws", "fz_sample_logits", "fz_sample",
    "fz_generate", "fz_tokenizer_from_gguf", "fz_tokenizer_new", "fz_tokenizer_free", "fz_tokenizer_vocab_size",
    "fz_tokenizer_encode", "fz_tokenizer_decode", "fz_tokenizer_token_bytes", "fz_pretokenize", "fz_chat_template",
    "fz_utf8_stream_new", "fz_utf8_stream_free", "fz_utf8_stream_push", "fz_utf8_stream_flush",
    "fz_selftest_exchange_timeout",
]

OPS = ["embed", "qkv", "rope_append", "attention", "o_proj", "gate_up", "down", "lm_head", "finalize"]


class FurnaceError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class _Config(C.Structure):
    _fields_ = [("n_layers", C.c_uint32), ("n_heads", C.c_uint32), ("n_kv_heads", C.c_uint32),
                ("hidden", C.c_uint32), ("ffn", C.c_uint32), ("head_dim", C.c_uint32), ("rope_theta", C.c_float),
                ("rms_eps", C.c_float), ("vocab", C.c_uint32), ("context_length", C.c_uint32)]


class _TpSlice(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("q_head0", "q_heads", "kv_head0", "kv_heads", "o_col0", "o_cols", "ffn0",
                                          "ffn_n", "vocab0", "vocab_n", "vocab_pad")]


class _TensorInfo(C.Structure):
    _fields_ = [("name", C.c_char_p), ("dtype", C.c_uint32), ("n_dims", C.c_uint32), ("dims", C.c_uint64 * 4),
                ("offset", C.c_uint64), ("nbytes", C.c_uint64)]


_lib = None


def lib_path() -> str:
    return os.environ.get("FURNACE_B200_LIB") or _build.LIB


def load_library(build_if_missing: bool = True):
    """Load libfurnace_cuda.so (building it in-tree first if needed)."""
    global _lib
    if _lib is not None:
        return _lib
    path = os.environ.get("FURNACE_B200_LIB") or _build.LIB
    if not os.path.exists(path):
        if not build_if_missing:
            raise FurnaceError(FZ_ECUDA, f"CUDA library missing: {path}")
        _build.build_cuda()
    L = C.CDLL(path)
    P, S, U32, U64, I = C.c_void_p, C.c_size_t, C.c_uint32, C.c_uint64, C.c_int
    fp, u32p = C.POINTER(C.c_float), C.POINTER(C.c_uint32)
    pp = C.POINTER(C.c_void_p)
    sig = {
        "fz_last_error": (C.c_char_p, []),
        "fz_version": (C.c_char_p, []),
        "fz_selftest_exchange_timeout": (I, [I, U32]),
        "fz_open": (I, [C.c_char_p, pp]),
        "fz_open_bytes": (I, [P, S, pp]),
        "fz_file_free": (None, [P]),
        "fz_file_info": (I, [P, u32p, C.POINTER(S), C.POINTER(S), C.POINTER(S)]),
        "fz_tensor_at": (I, [P, S, C.POINTER(_TensorInfo)]),
        "fz_tensor": (I, [P, C.c_char_p, C.POINTER(_TensorInfo), pp]),
        "fz_meta_u32": (I, [P, C.c_char_p, u32p]),
        "fz_meta_f32": (I, [P, C.c_char_p, fp]),
        "fz_meta_str": (I, [P, C.c_char_p, C.POINTER(C.c_char_p)]),
        "fz_meta_array_len": (I, [P, C.c_char_p, C.POINTER(S)]),
        "fz_config_from_gguf": (I, [P, C.POINTER(_Config)]),
        "fz_model_load": (I, [P, I, C.POINTER(I), pp]),
        "fz_model_free": (None, [P]),
        "fz_model_config": (I, [P, C.POINTER(_Config)]),
        "fz_model_bytes": (I, [P, C.POINTER(U64), C.POINTER(U64)]),
        "fz_kv_new": (I, [P, U32, I, pp]),
        "fz_kv_free": (None, [P]),
        "fz_kv_len": (I, [P, u32p]),
        "fz_kv_set_len": (I, [P, U32]),
        "fz_kv_read": (I, [P, U32, I, U32, fp]),
        "fz_forward": (I, [P, P, u32p, U32, fp, u32p]),
        "fz_forward_last": (I, [P, u32p, U32, fp, u32p]),
        "fz_decode_greedy": (I, [P, P, U32, U32, u32p, U32, u32p, fp, u32p]),
        "fz_dequant": (I, [U32, P, S, S, fp]),
        "fz_gemv": (I, [U32, P, U32, U32, fp, fp]),
        "fz_kv_reset": (I, [P]),
        "fz_kv_bytes": (I, [P, C.POINTER(U64)]),
        "fz_matmul_quant": (I, [fp, U32, P, S, U32, U32, U32, fp]),
        "fz_weight_upload": (I, [U32, P, S, U32, U32, pp]),
        "fz_weight_free": (None, [P]),
        "fz_matmul_quant_dev": (I, [P, P, U32, P, P]),
        "fz_dequant_dev_noalloc": (I, [U32, P, S, S, P, P]),
        "fz_tp_slice_of": (I, [P, I, I, P]),
        "fz_tp_unique_id": (I, [P, S]),
        "fz_model_load_tp": (I, [P, I, I, P, S, I, pp]),
        "fz_sampler_new": (I, [C.c_float, U32, C.c_float, C.c_float, U64, pp]),
        "fz_sampler_free": (None, [P]),
        "fz_sampler_draws": (I, [P, C.POINTER(U64)]),
        "fz_sample_logits": (I, [P, fp, S, u32p, S, u32p]),
        "fz_sample": (I, [P, P, u32p, U32, u32p]),
        "fz_generate": (I, [P, P, P, u32p, U32, U32, u32p, U32, u32p, u32p]),
        "fz_model_stream": (I, [P, pp, C.POINTER(I)]),
        "fz_step_profile": (I, [P, P, U32, U32, C.POINTER(C.c_double), C.POINTER(C.c_double), u32p]),
        "fz_tokenizer_from_gguf": (I, [P, pp]),
        "fz_tokenizer_new": (I, [C.POINTER(C.c_char_p), C.POINTER(C.c_int64), S, C.POINTER(C.c_char_p), S, pp]),
        "fz_tokenizer_free": (None, [P]),
        "fz_tokenizer_vocab_size": (I, [P, C.POINTER(S)]),
        "fz_tokenizer_encode": (I, [P, C.c_char_p, S, u32p, S, C.POINTER(S)]),
        "fz_tokenizer_decode": (I, [P, u32p, S, C.c_char_p, S, C.POINTER(S)]),
        "fz_tokenizer_token_bytes": (I, [P, U32, C.c_char_p, S, C.POINTER(S)]),
        "fz_pretokenize": (I, [C.c_char_p, S, C.POINTER(S), S, C.POINTER(S)]),
        "fz_chat_template": (I, [C.c_char_p, S, C.c_char_p, S, C.POINTER(S)]),
        "fz_utf8_stream_new": (I, [pp]),
        "fz_utf8_stream_free": (None, [P]),
        "fz_utf8_stream_push": (I, [P, C.c_char_p, S, C.c_char_p, S, C.POINTER(S)]),
        "fz_utf8_stream_flush": (I, [P, C.c_char_p, S, C.POINTER(S)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _check(rc: int):
    if rc != FZ_OK:
        raise FurnaceError(rc, load_library().fz_last_error().decode(errors="replace"))


def _fp(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _u32p(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint32))


def version() -> str:
    return load_library().fz_version().decode()


# ---------------------------------------------------------------------------
# GGUF (src/gguf.rs)
# ---------------------------------------------------------------------------
@dataclass
class TensorInfo:
    """TensorInfo (src/gguf.rs:246-254): dims in ggml order."""
    name: str
    dims: list
    dtype: int
    offset: int
    nbytes: int

    def n_elements(self) -> int:
        return int(np.prod(self.dims)) if self.dims else 1


class GgufFile:
    def __init__(self, handle):
        self._h = handle
        L = load_library()
        v = C.c_uint32()
        nt, nm, ds = C.c_size_t(), C.c_size_t(), C.c_size_t()
        _check(L.fz_file_info(self._h, C.byref(v), C.byref(nt), C.byref(nm), C.byref(ds)))
        self.version, self.n_metadata, self.data_start = v.value, nm.value, ds.value
        self.tensors = []
        for i in range(nt.value):
            ti = _TensorInfo()
            _check(L.fz_tensor_at(self._h, i, C.byref(ti)))
            self.tensors.append(TensorInfo(ti.name.decode(), [ti.dims[k] for k in range(ti.n_dims)], ti.dtype,
                                           ti.offset, ti.nbytes))

    @classmethod
    def open(cls, path: str) -> "GgufFile":
        h = C.c_void_p()
        _check(load_library().fz_open(os.fsencode(path), C.byref(h)))
        return cls(h)

    @classmethod
    def from_bytes(cls, data: bytes) -> "GgufFile":
        h = C.c_void_p()
        buf = C.create_string_buffer(bytes(data), len(data)) if data else None
        _check(load_library().fz_open_bytes(buf, len(data), C.byref(h)))
        return cls(h)

    def close(self):
        if self._h:
            load_library().fz_file_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def tensor(self, name: str):
        """(TensorInfo, raw bytes) -- GgufFile::tensor (src/gguf.rs:412-434)."""
        ti = _TensorInfo()
        ptr = C.c_void_p()
        _check(load_library().fz_tensor(self._h, name.encode(), C.byref(ti), C.byref(ptr)))
        info = TensorInfo(ti.name.decode(), [ti.dims[k] for k in range(ti.n_dims)], ti.dtype, ti.offset, ti.nbytes)
        return info, C.string_at(ptr.value, ti.nbytes)

    def meta_u32(self, key: str) -> int:
        v = C.c_uint32()
        _check(load_library().fz_meta_u32(self._h, key.encode(), C.byref(v)))
        return v.value

    def meta_f32(self, key: str) -> float:
        v = C.c_float()
        _check(load_library().fz_meta_f32(self._h, key.encode(), C.byref(v)))
        return v.value

    def meta_str(self, key: str) -> str:
        v = C.c_char_p()
        _check(load_library().fz_meta_str(self._h, key.encode(), C.byref(v)))
        return v.value.decode()

    def meta_array_len(self, key: str) -> int:
        v = C.c_size_t()
        _check(load_library().fz_meta_array_len(self._h, key.encode(), C.byref(v)))
        return v.value


@dataclass
class Config:
    """Config (src/model.rs:27-38)."""
    n_layers: int
    n_heads: int
    n_kv_heads: int
    hidden: int
    ffn: int
    head_dim: int
    rope_theta: float
    rms_eps: float
    vocab: int
    context_length: int

    @classmethod
    def _from_c(cls, c: _Config) -> "Config":
        return cls(c.n_layers, c.n_heads, c.n_kv_heads, c.hidden, c.ffn, c.head_dim, c.rope_theta, c.rms_eps, c.vocab,
                   c.context_length)

    def _to_c(self) -> _Config:
        return _Config(self.n_layers, self.n_heads, self.n_kv_heads, self.hidden, self.ffn, self.head_dim,
                       self.rope_theta, self.rms_eps, self.vocab, self.context_length)

    @classmethod
    def from_gguf(cls, f: GgufFile) -> "Config":
        c = _Config()
        _check(load_library().fz_config_from_gguf(f._h, C.byref(c)))
        return cls._from_c(c)


# ---------------------------------------------------------------------------
# Model / KvCache (src/model.rs)
# ---------------------------------------------------------------------------
class Model:
    def __init__(self, handle):
        self._h = handle
        c = _Config()
        _check(load_library().fz_model_config(self._h, C.byref(c)))
        self.config = Config._from_c(c)
        self.rank, self.world = 0, 1  # tensor-parallel share (load_tp)

    @classmethod
    def load(cls, f: GgufFile, tp: int = 1, devices=None) -> "Model":
        """Model::load (src/model.rs:520-552): weights uploaded to HBM."""
        h = C.c_void_p()
        dev = (C.c_int * len(devices))(*devices) if devices else None
        _check(load_library().fz_model_load(f._h, tp, dev, C.byref(h)))
        return cls(h)

    @classmethod
    def load_tp(cls, f: GgufFile, rank: int, world: int, nccl_id: bytes, device: int) -> "Model":
        """Rank `rank`'s share of Model::load under tensor parallelism (one
        process per GPU); every rank calls it with the same nccl_id."""
        h = C.c_void_p()
        buf = C.create_string_buffer(bytes(nccl_id), max(len(nccl_id), 1)) if nccl_id else None
        _check(load_library().fz_model_load_tp(f._h, rank, world, buf, len(nccl_id or b""), device, C.byref(h)))
        m = cls(h)
        m.rank, m.world = rank, world
        return m

    def close(self):
        if self._h:
            load_library().fz_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def param_bytes(self):
        """(resident device bytes, GGUF bytes streamed per decode token)."""
        r, s = C.c_uint64(), C.c_uint64()
        _check(load_library().fz_model_bytes(self._h, C.byref(r), C.byref(s)))
        return r.value, s.value

    def forward_cached(self, tokens, cache: "KvCache", want_logits: bool = True):
        """Model::forward_cached (src/model.rs:579-592) -> logits [vocab]
        (or the argmax id when want_logits is False)."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32).reshape(-1)
        am = C.c_uint32()
        if want_logits:
            out = np.zeros(self.config.vocab, np.float32)
            _check(load_library().fz_forward(self._h, cache._h, _u32p(t), t.size, _fp(out), C.byref(am)))
            return out
        _check(load_library().fz_forward(self._h, cache._h, _u32p(t), t.size, None, C.byref(am)))
        return am.value

    def forward(self, tokens, cache: "KvCache", want_logits: bool = True):
        """forward_cached returning (logits or None, device argmax id)."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32).reshape(-1)
        am = C.c_uint32()
        out = np.zeros(self.config.vocab, np.float32) if want_logits else None
        _check(load_library().fz_forward(self._h, cache._h, _u32p(t), t.size, _fp(out) if want_logits else None,
                                         C.byref(am)))
        return out, am.value

    def forward_last(self, tokens, want_logits: bool = True):
        """Model::forward_last (src/model.rs:569-575), the uncached forward over
        positions 0..n-1: (logits or None, argmax id)."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32).reshape(-1)
        am = C.c_uint32()
        out = np.zeros(self.config.vocab, np.float32) if want_logits else None
        _check(load_library().fz_forward_last(self._h, _u32p(t), t.size, _fp(out) if want_logits else None,
                                              C.byref(am)))
        return out, am.value

    def stream(self):
        """(cudaStream_t as int, device ordinal) the model runs on."""
        st, dev = C.c_void_p(), C.c_int()
        _check(load_library().fz_model_stream(self._h, C.byref(st), C.byref(dev)))
        return st.value or 0, dev.value

    def step_profile(self, first: int, reps: int, cache: "KvCache"):
        """Per-op decode timings (src/perf.rs counterpart): {op: (ms, bytes, launches)}."""
        ms = (C.c_double * len(OPS))()
        by = (C.c_double * len(OPS))()
        ln = np.zeros(len(OPS), np.uint32)
        _check(load_library().fz_step_profile(self._h, cache._h, first, reps, ms, by, _u32p(ln)))
        return {op: (ms[i], by[i], int(ln[i])) for i, op in enumerate(OPS)}

    def decode_greedy(self, first: int, n_steps: int, cache: "KvCache", stop_ids=(), keep_logits=False):
        """The greedy loop of generate (src/generate.rs:122-141) on the device.
        Returns (ids, logits [n-1, vocab] or None)."""
        ids = np.zeros(max(1, n_steps), np.uint32)
        st = np.ascontiguousarray(list(stop_ids) or [0], dtype=np.uint32)
        lg = np.zeros((max(1, n_steps - 1), self.config.vocab), np.float32) if keep_logits else None
        n = C.c_uint32()
        _check(load_library().fz_decode_greedy(self._h, cache._h, first, n_steps, _u32p(st), len(stop_ids), _u32p(ids),
                                               _fp(lg) if keep_logits else None, C.byref(n)))
        k = n.value
        return ids[:k].copy(), (lg[: max(0, k - 1)] if keep_logits else None)


class KvCache:
    """KvCache (src/model.rs:321-363), resident in HBM."""

    def __init__(self, model: Model, max_ctx: int, kv_dtype: int = 0):
        """kv_dtype FZ_KV_F32 (the reference's f32 cache) or FZ_KV_F16
        (binary16 elements, rounded to nearest even when appended)."""
        self.model = model
        self.max_ctx = max_ctx
        self.kv_dtype = kv_dtype
        h = C.c_void_p()
        _check(load_library().fz_kv_new(model._h, max_ctx, kv_dtype, C.byref(h)))
        self._h = h

    def close(self):
        if self._h:
            load_library().fz_kv_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def len(self) -> int:
        v = C.c_uint32()
        _check(load_library().fz_kv_len(self._h, C.byref(v)))
        return v.value

    @len.setter
    def len(self, n: int):
        _check(load_library().fz_kv_set_len(self._h, n))

    def reset(self):
        """len = 0: the cache reused for a new sequence."""
        _check(load_library().fz_kv_reset(self._h))

    def bytes(self) -> int:
        """KvCache::bytes (src/model.rs:341-343): K and V bytes of this rank."""
        v = C.c_uint64()
        _check(load_library().fz_kv_bytes(self._h, C.byref(v)))
        return v.value

    def read(self, layer: int, which_v: bool, n: int) -> np.ndarray:
        """Cached K (or V) rows [0, n) as [n, kv_heads * head_dim]: every KV
        head, or this rank's under tensor parallelism."""
        c, m = self.model.config, self.model
        kvh = c.n_kv_heads // m.world
        out = np.zeros((n, kvh * c.head_dim), np.float32)
        _check(load_library().fz_kv_read(self._h, layer, int(which_v), n, _fp(out)))
        return out


# ---------------------------------------------------------------------------
# quant (src/quant.rs)
# ---------------------------------------------------------------------------
class quant:
    @staticmethod
    def dequantize(dtype: int, raw: bytes, n: int) -> np.ndarray:
        """quant::dequantize (src/quant.rs:261-281), on the device."""
        buf = np.frombuffer(bytes(raw), dtype=np.uint8) if len(raw) else np.zeros(1, np.uint8)
        out = np.zeros(max(n, 1), np.float32)
        _check(load_library().fz_dequant(dtype, buf.ctypes.data, len(raw), n, _fp(out)))
        return out[:n]

    @staticmethod
    def matmul_quant(a, raw: bytes, d_out: int, d_in: int, dtype: int) -> np.ndarray:
        """quant::matmul_quant (src/quant.rs:170-193), on the device."""
        a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1, d_in)
        buf = np.frombuffer(bytes(raw), dtype=np.uint8)
        out = np.zeros((a.shape[0], d_out), np.float32)
        _check(load_library().fz_matmul_quant(_fp(a), a.shape[0], buf.ctypes.data, buf.size, d_out, d_in, dtype,
                                              _fp(out)))
        return out

    @staticmethod
    def gemv(x, raw: bytes, d_out: int, d_in: int, dtype: int) -> np.ndarray:
        """One row of quant::matmul_quant (fz_gemv): y = W x."""
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(d_in)
        buf = np.frombuffer(bytes(raw), dtype=np.uint8)
        out = np.zeros(d_out, np.float32)
        _check(load_library().fz_gemv(dtype, buf.ctypes.data, d_out, d_in, _fp(x), _fp(out)))
        return out


class Sampler:
    """Sampler (src/sampler.rs:57-155): temperature (0 = greedy), top_k (0 =
    off), top_p (1 = off), repeat_penalty (1 = off), PCG32 seed."""

    def __init__(self, temperature: float, top_k: int, top_p: float, repeat_penalty: float, seed: int):
        h = C.c_void_p()
        _check(load_library().fz_sampler_new(temperature, top_k, top_p, repeat_penalty, seed, C.byref(h)))
        self._h = h

    def close(self):
        if self._h:
            load_library().fz_sampler_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def draws(self) -> int:
        d = C.c_uint64()
        _check(load_library().fz_sampler_draws(self._h, C.byref(d)))
        return d.value

    def sample(self, logits, recent=()) -> int:
        """Sampler::sample on host logits."""
        lg = np.ascontiguousarray(logits, dtype=np.float32)
        r = np.ascontiguousarray(recent, dtype=np.uint32) if len(recent) else np.zeros(1, np.uint32)
        out = C.c_uint32()
        _check(load_library().fz_sample_logits(self._h, _fp(lg), lg.size, _u32p(r), len(recent), C.byref(out)))
        return out.value

    def sample_model(self, model: "Model", recent=()) -> int:
        """Sampler::sample on the model's last logits, on the device."""
        r = np.ascontiguousarray(recent, dtype=np.uint32) if len(recent) else np.zeros(1, np.uint32)
        out = C.c_uint32()
        _check(load_library().fz_sample(model._h, self._h, _u32p(r), len(recent), C.byref(out)))
        return out.value


def generate_sampled(model: Model, prompt_ids, max_new: int, sampler: Sampler, stop_ids=(),
                     max_ctx: int | None = None) -> np.ndarray:
    """generate (src/generate.rs:83-157) with any sampler (fz_generate)."""
    p = np.ascontiguousarray(prompt_ids, dtype=np.uint32)
    max_ctx = max_ctx or min(model.config.context_length, 4096)
    cache = KvCache(model, max_ctx)
    st = np.ascontiguousarray(stop_ids, dtype=np.uint32) if len(stop_ids) else np.zeros(1, np.uint32)
    out = np.zeros(max(max_new, 1), np.uint32)
    n = C.c_uint32()
    _check(load_library().fz_generate(model._h, cache._h, sampler._h, _u32p(p), p.size, max_new, _u32p(st),
                                      len(stop_ids), _u32p(out), C.byref(n)))
    cache.close()
    return out[: n.value]


def generate(model: Model, prompt_ids, max_new: int, stop_ids=(), max_ctx: int | None = None, keep_logits=False,
             kv_dtype: int = 0):
    """generate (src/generate.rs:83-157) with the greedy sampler
    (temperature 0): prefill once, then decode on the device.  Returns
    (ids, per-step logits or None)."""
    p = np.ascontiguousarray(prompt_ids, dtype=np.uint32)
    max_ctx = max_ctx or min(model.config.context_length, 4096)
    if p.size + max_new > max_ctx:
        raise FurnaceError(FZ_EINVAL, f"prompt ({p.size}) + max tokens ({max_new}) exceeds context cap {max_ctx}")
    cache = KvCache(model, max_ctx, kv_dtype)
    logits, first = model.forward(p, cache, want_logits=keep_logits)
    ids, lg = model.decode_greedy(first, max_new, cache, stop_ids, keep_logits)
    if keep_logits:
        lg = np.concatenate([logits[None], lg], axis=0)[: len(ids)]
    return ids, lg


def tp_unique_id() -> bytes:
    """A fresh NCCL unique id (128 bytes) for fz_model_load_tp; made on one
    rank and handed to all (torch.distributed broadcast, a file, ...)."""
    buf = C.create_string_buffer(128)
    _check(load_library().fz_tp_unique_id(buf, 128))
    return buf.raw


def tp_slice(config: "Config", rank: int, world: int) -> dict:
    """This rank's share under tensor parallelism (fz_tp_slice_of)."""
    c, out = config._to_c(), _TpSlice()
    _check(load_library().fz_tp_slice_of(C.byref(c), rank, world, C.byref(out)))
    return {n: getattr(out, n) for n, _ in _TpSlice._fields_}



# ---------------------------------------------------------------------------
# tokenizer (src/tokenizer.rs) and text helpers (src/generate.rs), host side
# ---------------------------------------------------------------------------
def _grow(call, make, cap):
    """Run call(buffer, cap, count_ptr) and retry once with the reported size
    on FZ_ESPACE; returns (buffer, count)."""
    n = C.c_size_t()
    buf = make(cap)
    rc = call(buf, cap, C.byref(n))
    if rc == FZ_ESPACE:
        cap = n.value
        buf = make(cap)
        rc = call(buf, cap, C.byref(n))
    _check(rc)
    return buf, n.value


def _bytes_out(call, cap=256) -> bytes:
    buf, n = _grow(call, lambda k: C.create_string_buffer(max(k, 1)), cap)
    return buf.raw[:n]


class Tokenizer:
    """Byte-level BPE with the qwen2 pre-tokenizer (src/tokenizer.rs)."""

    def __init__(self, handle):
        self._h = handle

    @classmethod
    def from_gguf(cls, f: GgufFile) -> "Tokenizer":
        """Tokenizer::from_gguf (src/tokenizer.rs:67-90)."""
        h = C.c_void_p()
        _check(load_library().fz_tokenizer_from_gguf(f._h, C.byref(h)))
        return cls(h)

    @classmethod
    def new(cls, tokens, token_types, merges) -> "Tokenizer":
        """Tokenizer::new (src/tokenizer.rs:92-138): token strings, gguf
        token types, "left right" merges in rank order."""
        if len(token_types) != len(tokens):
            raise FurnaceError(FZ_EINVAL, f"{len(tokens)} tokens but {len(token_types)} token types")
        tb = [t.encode() for t in tokens]
        mb = [m.encode() for m in merges]
        ta = (C.c_char_p * max(len(tb), 1))(*tb)
        ty = (C.c_int64 * max(len(tb), 1))(*[int(x) for x in token_types])
        ma = (C.c_char_p * max(len(mb), 1))(*mb)
        h = C.c_void_p()
        _check(load_library().fz_tokenizer_new(ta, ty, len(tb), ma, len(mb), C.byref(h)))
        return cls(h)

    def close(self):
        if self._h:
            load_library().fz_tokenizer_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __len__(self) -> int:
        n = C.c_size_t()
        _check(load_library().fz_tokenizer_vocab_size(self._h, C.byref(n)))
        return n.value

    def encode(self, text: str) -> list[int]:
        """Tokenizer::encode (src/tokenizer.rs:140-149)."""
        b = text.encode()
        L = load_library()
        buf, n = _grow(lambda buf, cap, np_: L.fz_tokenizer_encode(self._h, b, len(b), buf, cap, np_),
                       lambda k: (C.c_uint32 * max(k, 1))(), len(b) + 8)
        return list(buf[:n])

    def decode(self, ids) -> str:
        """Tokenizer::decode (src/tokenizer.rs:151-157), lossy UTF-8."""
        a = np.ascontiguousarray(ids, dtype=np.uint32).reshape(-1)
        L = load_library()
        out = _bytes_out(lambda buf, cap, np_: L.fz_tokenizer_decode(self._h, _u32p(a), a.size, buf, cap, np_),
                         4 * a.size + 16)
        return out.decode()

    def token_bytes(self, token_id: int) -> bytes:
        """Tokenizer::token_bytes (src/tokenizer.rs:159-181)."""
        L = load_library()
        return _bytes_out(lambda buf, cap, np_: L.fz_tokenizer_token_bytes(self._h, token_id, buf, cap, np_), 64)


def pretokenize(text: str) -> list[str]:
    """The qwen2 pre-tokenizer split alone (src/tokenizer.rs:16, 215-232)."""
    b = text.encode()
    L = load_library()
    buf, n = _grow(lambda buf, cap, np_: L.fz_pretokenize(b, len(b), buf, cap, np_),
                   lambda k: (C.c_size_t * max(k, 1))(), len(b) + 1)
    out, start = [], 0
    for end in buf[:n]:
        out.append(b[start:end].decode())
        start = end
    return out


def chat_template(prompt: str) -> str:
    """chat_template (src/generate.rs:13-21)."""
    b = prompt.encode()
    L = load_library()
    return _bytes_out(lambda buf, cap, np_: L.fz_chat_template(b, len(b), buf, cap, np_), len(b) + 256).decode()


class Utf8Stream:
    """Utf8Stream (src/generate.rs:24-66): printable prefixes of a byte stream."""

    def __init__(self):
        h = C.c_void_p()
        _check(load_library().fz_utf8_stream_new(C.byref(h)))
        self._h = h

    def push(self, data: bytes) -> str:
        L = load_library()
        return _bytes_out(lambda buf, cap, np_: L.fz_utf8_stream_push(self._h, data, len(data), buf, cap, np_),
                          len(data) + 16).decode()

    def flush(self) -> str:
        L = load_library()
        return _bytes_out(lambda buf, cap, np_: L.fz_utf8_stream_flush(self._h, buf, cap, np_), 64).decode()

    def close(self):
        if self._h:
            load_library().fz_utf8_stream_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
