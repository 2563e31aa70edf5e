"""Synthetic GGUF files: valid for the reference's parser and decoders, the
requested quantization mix, and the requested value distributions.  CPU only."""

import numpy as np
import pytest

from furnace_b200 import synth


def test_quantizers_roundtrip_against_oracle(orc):
    rng = np.random.default_rng(1)
    x = rng.normal(0, 0.02, size=(4, 512)).astype(np.float32)
    for dt, tol in ((synth.Q8_0, 0.01), (synth.Q5_0, 0.1), (synth.Q4_K, 0.12), (synth.Q6_K, 0.04)):
        raw = synth.quantize(x, dt)
        y = orc.dequantize(dt, raw, x.size).reshape(x.shape)
        rel = np.linalg.norm(y - x) / np.linalg.norm(x)
        assert rel < tol, (dt, rel)


def test_dequant_of_synth_matches_gguf_py(orc):
    from gguf import GGMLQuantizationType as T
    from gguf import quants

    for dt, qt in ((synth.Q8_0, T.Q8_0), (synth.Q5_0, T.Q5_0), (synth.Q4_K, T.Q4_K), (synth.Q6_K, T.Q6_K)):
        raw = synth.random_tensor(8, 512, dt, seed=5)
        ref = quants.dequantize(np.frombuffer(raw, np.uint8).reshape(8, -1), qt).reshape(-1)
        ours = orc.dequantize(dt, raw, 8 * 512)
        assert np.array_equal(ours.view(np.uint32), ref.astype(np.float32).view(np.uint32))


def test_generator_is_seeded_and_thread_independent():
    a = synth.random_tensor(64, 256, synth.Q4_K, seed=9, threads=1)
    b = synth.random_tensor(64, 256, synth.Q4_K, seed=9, threads=7)
    c = synth.random_tensor(64, 256, synth.Q4_K, seed=10, threads=7)
    assert a == b and a != c


def test_distribution(orc):
    raw = synth.random_tensor(256, 256, synth.F32, seed=3, mean=1.0, std=0.05)
    v = np.frombuffer(raw, np.float32)
    assert abs(v.mean() - 1.0) < 1e-3 and abs(v.std() - 0.05) < 1e-3


@pytest.mark.parametrize("name", ["c1", "c2", "c3", "c4", "c5"])
def test_config_mixes(name):
    s = synth.spec(name)
    tl = synth.tensor_list(s)
    dts = {n: dt for n, _, dt, _, _ in tl}
    if name == "c1":
        assert set(dt for n, dt in dts.items() if n.endswith("weight") and "norm" not in n) == {synth.Q8_0}
        assert "output.weight" not in dts
    if name in ("c2", "c3", "c5"):
        assert dts["blk.0.attn_v.weight"] == synth.Q6_K and dts["blk.1.attn_v.weight"] == synth.Q4_K
        assert dts["blk.1.attn_q.weight"] == synth.Q4_K
    if name == "c5":
        assert dts["blk.0.ffn_down.weight"] == synth.Q8_0 and dts["blk.1.ffn_down.weight"] == synth.Q5_0
    if name == "c4":
        assert dts["blk.3.attn_q.weight"] == synth.Q5_0 and dts["blk.3.ffn_up.weight"] == synth.Q6_K
    head, ds, tensors, offs, total = synth.header(s) if name in ("c1", "c2") else (None, 0, tl, [], 0)
    if head is not None:
        assert ds % 32 == 0 and all(o % 32 == 0 for o in offs)


def test_tiny_file_loads_in_oracle(orc, tmp_path):
    p = synth.write(synth.spec("tiny"), str(tmp_path / "t.gguf"))
    m = orc.Model(p)
    assert (m.hidden, m.n_layers, m.vocab) == (512, 3, 4096)
    kv = m.kv_new(64)
    lg = m.forward_cached(synth.prompt_ids(m.vocab, 5), kv)
    assert lg.shape == (4096,) and np.isfinite(lg).all() and kv.len == 5


def test_oracle_cached_equals_uncached_bitwise(orc, tmp_path):
    """src/model.rs:697-729 at model level: prefill + decode steps give the
    exact logits of the uncached full recompute."""
    p = synth.write(synth.spec("tiny"), str(tmp_path / "t.gguf"))
    m = orc.Model(p)
    ids = synth.prompt_ids(m.vocab, 6, seed=2)
    kv = m.kv_new(16)
    m.forward_cached(ids[:4], kv)
    a = m.forward_cached(ids[4:5], kv)
    b = m.forward_cached(ids[5:6], kv)
    assert np.array_equal(a, m.forward_last(ids[:5]))
    assert np.array_equal(b, m.forward_last(ids[:6]))
