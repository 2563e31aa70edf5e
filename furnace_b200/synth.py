"""Seeded synthetic Qwen2 GGUF files for the benchmark configurations.

The reference is measured on real Qwen2.5 GGUF files; none are available
here, so every parity test and benchmark runs on files with the same shapes,
tensor names, metadata keys and quantization mixes, filled with seeded
N(0, 0.02) matmul weights, 1 + N(0, 0.05) norm weights and N(0, 0.02) biases.
The header layout follows what the reference parser reads
(src/gguf.rs:3-8, :315-363) and the metadata Config::from_gguf needs
(src/model.rs:41-60).  Tensor data is produced in parallel by synth.c.
"""

from __future__ import annotations

import ctypes as C
import hashlib
import mmap
import os
import struct
from dataclasses import dataclass, field

import numpy as np

from . import build as _build

F32, Q5_0, Q8_0, Q4_K, Q6_K = 0, 6, 8, 12, 14
BLOCK = {F32: (1, 4), Q8_0: (32, 34), Q5_0: (32, 22), Q4_K: (256, 144), Q6_K: (256, 210)}
ALIGN = 32


@dataclass
class Spec:
    name: str
    hidden: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    ffn: int
    vocab: int
    tied: bool
    context_length: int
    # dtype(tensor_name, layer_index) -> ggml type
    mix: str = "q8_0"
    rope_theta: float = 1e6
    rms_eps: float = 1e-6
    seed: int = 0
    extra: dict = field(default_factory=dict)

    @property
    def head_dim(self):
        return self.hidden // self.n_heads

    def dtype(self, kind: str, layer: int) -> int:
        """Quantization mix per configuration (the benchmark configurations C1-C5)."""
        if self.mix == "q8_0":
            return Q8_0
        if self.mix == "q4_k_m":
            even = layer % 2 == 0
            if kind == "ffn_down":
                if self.ffn % 256:
                    # K-quants need in % 256 == 0: Q5_0 (odd) / Q8_0 (even)
                    return Q8_0 if even else Q5_0
                return Q6_K if even else Q4_K
            if kind == "attn_v":
                return Q6_K if even else Q4_K
            if kind == "output":
                return Q6_K
            if kind == "token_embd":
                return Q6_K if self.tied else Q4_K
            return Q4_K
        if self.mix == "q5_0_q6_k":
            if kind in ("attn_q", "attn_k", "attn_v", "attn_output"):
                return Q5_0
            return Q6_K
        if self.mix == "mixed_small":
            # exercises every format and the Q5_0/Q8_0 fallbacks in 2-3 layers
            table = {"attn_q": Q4_K, "attn_k": Q5_0, "attn_v": Q6_K if layer % 2 == 0 else Q8_0,
                     "attn_output": Q8_0 if layer % 2 == 0 else Q4_K, "ffn_gate": Q6_K, "ffn_up": Q6_K,
                     "ffn_down": Q5_0 if layer % 2 else Q4_K, "output": Q6_K, "token_embd": Q4_K}
            return table[kind]
        raise ValueError(self.mix)


CONFIGS = {
    # the benchmark configurations C1-C5 (Qwen2.5 0.5B, 1.5B, 7B, 32B, 72B shapes)
    "c1": Spec("qwen2.5-0.5b-q8_0", 896, 24, 14, 2, 4864, 151936, True, 4096, "q8_0"),
    "c2": Spec("qwen2.5-1.5b-q4_k_m", 1536, 28, 12, 2, 8960, 151936, True, 4096, "q4_k_m"),
    "c3": Spec("qwen2.5-7b-q4_k_m", 3584, 28, 28, 4, 18944, 152064, False, 4096, "q4_k_m"),
    "c4": Spec("qwen2.5-32b-q5_0-q6_k", 5120, 64, 40, 8, 27648, 152064, False, 8704, "q5_0_q6_k"),
    "c5": Spec("qwen2.5-72b-q4_k_m", 8192, 80, 64, 8, 29568, 152064, False, 8704, "q4_k_m"),
    # small all-format case for fast tests
    "tiny": Spec("tiny-mixed", 512, 3, 8, 2, 768, 4096, False, 1024, "mixed_small"),
    "tiny_q8": Spec("tiny-q8_0", 256, 2, 4, 2, 512, 2048, True, 512, "q8_0"),
}


def spec(name: str, n_layers: int | None = None, **over) -> Spec:
    import dataclasses

    s = dataclasses.replace(CONFIGS[name], **over)
    if n_layers is not None:
        s = dataclasses.replace(s, n_layers=n_layers, name=f"{s.name}-L{n_layers}")
    return s


def tensor_list(s: Spec):
    """(name, dims in ggml order (in, out), dtype, mean, std) in file order."""
    H, F, V = s.hidden, s.ffn, s.vocab
    qd, kd = s.n_heads * s.head_dim, s.n_kv_heads * s.head_dim
    out = [("token_embd.weight", (H, V), s.dtype("token_embd", 0), 0.0, 0.02)]
    for i in range(s.n_layers):
        p = f"blk.{i}."
        out += [
            (p + "attn_norm.weight", (H,), F32, 1.0, 0.05),
            (p + "attn_q.weight", (H, qd), s.dtype("attn_q", i), 0.0, 0.02),
            (p + "attn_q.bias", (qd,), F32, 0.0, 0.02),
            (p + "attn_k.weight", (H, kd), s.dtype("attn_k", i), 0.0, 0.02),
            (p + "attn_k.bias", (kd,), F32, 0.0, 0.02),
            (p + "attn_v.weight", (H, kd), s.dtype("attn_v", i), 0.0, 0.02),
            (p + "attn_v.bias", (kd,), F32, 0.0, 0.02),
            (p + "attn_output.weight", (qd, H), s.dtype("attn_output", i), 0.0, 0.02),
            (p + "ffn_norm.weight", (H,), F32, 1.0, 0.05),
            (p + "ffn_gate.weight", (H, F), s.dtype("ffn_gate", i), 0.0, 0.02),
            (p + "ffn_up.weight", (H, F), s.dtype("ffn_up", i), 0.0, 0.02),
            (p + "ffn_down.weight", (F, H), s.dtype("ffn_down", i), 0.0, 0.02),
        ]
    out.append(("output_norm.weight", (H,), F32, 1.0, 0.05))
    if not s.tied:
        out.append(("output.weight", (H, V), s.dtype("output", 0), 0.0, 0.02))
    return out


def _nbytes(dims, dtype):
    n = int(np.prod(dims))
    be, bb = BLOCK[dtype]
    assert n % be == 0, (dims, dtype)
    return n // be * bb


def _s(x: str) -> bytes:
    b = x.encode()
    return struct.pack("<Q", len(b)) + b


def _kv_str(k, v):
    return _s(k) + struct.pack("<I", 8) + _s(v)


def _kv_u32(k, v):
    return _s(k) + struct.pack("<II", 4, v)


def _kv_f32(k, v):
    return _s(k) + struct.pack("<If", 6, v)


def header(s: Spec):
    meta = [
        _kv_str("general.architecture", "qwen2"),
        _kv_str("general.name", s.name),
        _kv_u32("general.alignment", ALIGN),
        _kv_u32("qwen2.block_count", s.n_layers),
        _kv_u32("qwen2.context_length", s.context_length),
        _kv_u32("qwen2.embedding_length", s.hidden),
        _kv_u32("qwen2.feed_forward_length", s.ffn),
        _kv_u32("qwen2.attention.head_count", s.n_heads),
        _kv_u32("qwen2.attention.head_count_kv", s.n_kv_heads),
        _kv_f32("qwen2.rope.freq_base", s.rope_theta),
        _kv_f32("qwen2.attention.layer_norm_rms_epsilon", s.rms_eps),
        _kv_str("tokenizer.ggml.model", "gpt2"),
        _kv_str("tokenizer.ggml.pre", "qwen2"),
        _s("tokenizer.ggml.tokens") + struct.pack("<IIQ", 9, 8, s.vocab) + b"".join(_s(f"<t{i}>") for i in range(s.vocab)),
        _s("tokenizer.ggml.token_type") + struct.pack("<IIQ", 9, 5, s.vocab) + np.ones(s.vocab, "<i4").tobytes(),
        _s("tokenizer.ggml.merges") + struct.pack("<IIQ", 9, 8, 0),
        _kv_u32("tokenizer.ggml.eos_token_id", s.vocab - 2),
        _kv_u32("tokenizer.ggml.bos_token_id", s.vocab - 1),
    ]
    tensors = tensor_list(s)
    infos, offsets, off = [], [], 0
    for name, dims, dt, _, _ in tensors:
        off = (off + ALIGN - 1) // ALIGN * ALIGN
        offsets.append(off)
        infos.append(_s(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
                     + struct.pack("<IQ", dt, off))
        off += _nbytes(dims, dt)
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(meta)) + b"".join(meta) + b"".join(infos)
    data_start = (len(head) + ALIGN - 1) // ALIGN * ALIGN
    return head, data_start, tensors, offsets, off


def _seed(global_seed: int, name: str) -> int:
    return int.from_bytes(hashlib.sha256(f"{global_seed}:{name}".encode()).digest()[:8], "little")


def _synth_lib():
    path = _build.build_synth()
    L = C.CDLL(path)
    L.fzs_fill.restype = C.c_int
    L.fzs_fill.argtypes = [C.c_void_p, C.c_uint32, C.c_uint64, C.c_uint64, C.c_float, C.c_float, C.c_uint64, C.c_int]
    L.fzs_quantize.restype = C.c_int
    L.fzs_quantize.argtypes = [C.c_void_p, C.c_uint64, C.c_uint64, C.c_uint32, C.c_void_p]
    return L


def quantize(x: np.ndarray, dtype: int) -> bytes:
    """Quantize a [rows, cols] f32 array to raw GGUF blocks."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    out = np.zeros(_nbytes((cols, rows), dtype), np.uint8)
    if _synth_lib().fzs_quantize(x.ctypes.data, rows, cols, dtype, out.ctypes.data) != 0:
        raise ValueError("bad shape or dtype for quantize")
    return out.tobytes()


def random_tensor(rows: int, cols: int, dtype: int, seed: int, mean=0.0, std=0.02, threads=None) -> bytes:
    """One seeded [rows, cols] tensor's raw bytes (same generator as files)."""
    out = np.zeros(_nbytes((cols, rows), dtype), np.uint8)
    rc = _synth_lib().fzs_fill(out.ctypes.data, dtype, rows, cols, mean, std, seed, threads or os.cpu_count() or 1)
    assert rc == 0
    return out.tobytes()


def write(s: Spec, path: str, threads: int | None = None) -> str:
    """Write the synthetic GGUF for spec `s` to `path` (skipped when a file
    with the same spec tag already exists next to it)."""
    tag = f"{path}.spec"
    desc = repr((s, 1))
    if os.path.exists(path) and os.path.exists(tag) and open(tag).read() == desc:
        return path
    head, data_start, tensors, offsets, total = header(s)
    size = data_start + total
    L = _synth_lib()
    threads = threads or os.cpu_count() or 1
    with open(path, "wb") as f:
        f.truncate(size)
        f.write(head)
    with open(path, "r+b") as f:
        mm = mmap.mmap(f.fileno(), size)
        base = C.addressof(C.c_char.from_buffer(mm))
        try:
            for (name, dims, dt, mean, std), off in zip(tensors, offsets):
                rows = int(np.prod(dims[1:])) if len(dims) > 1 else 1
                cols = dims[0]
                rc = L.fzs_fill(base + data_start + off, dt, rows, cols, mean, std, _seed(s.seed, name), threads)
                assert rc == 0, name
        finally:
            del base
            mm.flush()
            mm.close()
    with open(tag, "w") as f:
        f.write(desc)
    return path


def default_dir() -> str:
    for d in (os.environ.get("FURNACE_SYNTH_DIR"), "/dev/shm", "/tmp"):
        if d and os.path.isdir(d) and os.access(d, os.W_OK):
            return d
    return "."


def ensure(name: str, n_layers: int | None = None, directory: str | None = None, **over) -> str:
    s = spec(name, n_layers, **over)
    d = directory or default_dir()
    return write(s, os.path.join(d, f"furnace-synth-{s.name}-s{s.seed}.gguf"))


def prompt_ids(vocab: int, n: int, seed: int = 0) -> np.ndarray:
    """Uniform random prompt ids in [0, vocab) from a seeded stream."""
    return np.random.default_rng(seed).integers(0, vocab, size=n, dtype=np.int64).astype(np.uint32)
