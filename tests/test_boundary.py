"""The C-ABI library: loads without a GPU, exports every symbol
include/furnace.h declares, and its host logic (GGUF parsing, Config, error
reporting) follows the reference's (src/gguf.rs:506-610, src/model.rs:41-60).
CPU only: no call here launches a kernel."""

import os
import re
import struct

import pytest

import furnace_b200 as fz
from furnace_b200 import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "furnace.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fz_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = fz.load_library()
    decl = declared_symbols()
    assert len(decl) >= 25
    for name in decl:
        assert hasattr(L, name), name
    assert sorted(fz.EXPORTS) == decl
    assert "sm_100a" in fz.version()


def test_exported_symbols_are_exactly_the_header():
    """nm -D: no fz_ symbol beyond the header leaks out of the .so."""
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", fz.lib_path()], capture_output=True, text=True).stdout
    exported = sorted({l.split()[-1] for l in out.splitlines() if l.split() and l.split()[-1].startswith("fz_")})
    assert exported == declared_symbols()


def _synthetic_gguf():
    """src/gguf.rs:532-564: a v3 file with 1 tensor and 3 metadata keys."""
    b = bytearray(b"GGUF")
    b += struct.pack("<IQQ", 3, 1, 3)

    def s(x):
        return struct.pack("<Q", len(x)) + x.encode()

    b += s("general.architecture") + struct.pack("<I", 8) + s("qwen2")
    b += s("qwen2.rope.freq_base") + struct.pack("<If", 6, 1_000_000.0)
    b += s("tokenizer.ggml.tokens") + struct.pack("<IIQ", 9, 8, 2) + s("a") + s("b")
    b += s("blk.0.attn_q.weight") + struct.pack("<IQQIQ", 2, 896, 896, 8, 0)
    while len(b) % 32:
        b.append(0)
    return bytes(b + bytes([0xAB] * 64))


def test_parses_synthetic_file():
    f = fz.GgufFile.from_bytes(_synthetic_gguf())
    assert f.version == 3 and f.n_metadata == 3 and len(f.tensors) == 1
    assert f.meta_str("general.architecture") == "qwen2"
    assert f.meta_f32("qwen2.rope.freq_base") == 1_000_000.0
    assert f.meta_array_len("tokenizer.ggml.tokens") == 2
    t = f.tensors[0]
    assert (t.name, t.dims, t.dtype, t.offset) == ("blk.0.attn_q.weight", [896, 896], fz.Q8_0, 0)
    assert f.data_start % 32 == 0
    # the tensor's data runs past the 64-byte blob: lookup must fail
    with pytest.raises(fz.FurnaceError, match="runs past end of file"):
        f.tensor("blk.0.attn_q.weight")
    with pytest.raises(fz.FurnaceError, match="no tensor named"):
        f.tensor("nope")


def test_rejects_bad_magic_and_truncation():
    with pytest.raises(fz.FurnaceError, match="bad magic") as e:
        fz.GgufFile.from_bytes(b"GGML\x03\x00\x00\x00")
    assert e.value.code == fz.FZ_EFORMAT
    data = _synthetic_gguf()
    with pytest.raises(fz.FurnaceError, match="unexpected EOF"):
        fz.GgufFile.from_bytes(data[:40])
    bad_version = data[:4] + struct.pack("<I", 4) + data[8:]
    with pytest.raises(fz.FurnaceError, match="unsupported GGUF version"):
        fz.GgufFile.from_bytes(bad_version)
    with pytest.raises(fz.FurnaceError) as e:
        fz.GgufFile.open("/nonexistent/model.gguf")
    assert e.value.code == fz.FZ_EIO


def test_config_missing_keys_fail_cleanly():
    f = fz.GgufFile.from_bytes(_synthetic_gguf())
    with pytest.raises(fz.FurnaceError, match="qwen2.attention.head_count"):
        fz.Config.from_gguf(f)


@pytest.fixture(scope="module")
def tiny_path(tmp_path_factory):
    return synth.write(synth.spec("tiny"), str(tmp_path_factory.mktemp("g") / "tiny.gguf"))


def test_config_from_synthetic_file(tiny_path):
    f = fz.GgufFile.open(tiny_path)
    c = fz.Config.from_gguf(f)
    s = synth.spec("tiny")
    assert (c.n_layers, c.n_heads, c.n_kv_heads, c.hidden, c.ffn, c.head_dim, c.vocab) == (
        s.n_layers, s.n_heads, s.n_kv_heads, s.hidden, s.ffn, s.head_dim, s.vocab)
    assert c.rope_theta == 1e6 and abs(c.rms_eps - 1e-6) < 1e-12


def test_tensor_table_matches_gguf_py(tiny_path):
    """scripts/check_m1.py: name, dims, dtype and offset agree with gguf-py."""
    from gguf import GGUFReader

    ours = {t.name: t for t in fz.GgufFile.open(tiny_path).tensors}
    r = GGUFReader(tiny_path)
    assert len(ours) == len(r.tensors)
    for t in r.tensors:
        o = ours[t.name]
        assert o.dims == [int(x) for x in t.shape]
        assert o.dtype == int(t.tensor_type)
        assert r.data_offset + o.offset == t.data_offset
        assert o.nbytes == t.n_bytes


def test_tensor_bytes_zero_copy(tiny_path):
    f = fz.GgufFile.open(tiny_path)
    info, raw = f.tensor("blk.0.attn_q.weight")
    assert len(raw) == info.nbytes
    data = open(tiny_path, "rb").read()
    start = f.data_start + info.offset
    assert raw == data[start:start + info.nbytes]


def test_model_load_without_gpu_reports_cuda_error(tiny_path):
    """No CPU fallback: on a machine without a GPU the load fails loudly."""
    from tests.conftest import gpu_available

    if gpu_available():
        pytest.skip("GPU present")
    f = fz.GgufFile.open(tiny_path)
    with pytest.raises(fz.FurnaceError) as e:
        fz.Model.load(f)
    assert e.value.code in (fz.FZ_ECUDA, fz.FZ_ENOMEM)
