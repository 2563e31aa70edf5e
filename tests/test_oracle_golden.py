"""Pin the CPU oracle to the reference: its own known-answer tests and the
gguf-py dequantization golden vectors (tests/golden/).  CPU only."""

import json
import math
import os
import struct

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(__file__), "golden")
KAT = json.load(open(os.path.join(GOLD, "reference_kat.json")))
TYPES = {"Q8_0": (8, 32, 34), "Q5_0": (6, 32, 22), "Q4_K": (12, 256, 144), "Q6_K": (14, 256, 210)}


def _bytes(spec, size):
    b = bytearray(size)
    for k, v in spec.items():
        b[int(k)] = v
    return bytes(b)


def _f16(x):
    return struct.pack("<e", x)


@pytest.mark.parametrize("name", list(TYPES))
def test_dequant_matches_gguf_py_bitwise(orc, name):
    """scripts/check_m2.py:45 / check_m10.py:44 compare against gguf-py; we
    require bit equality."""
    g = np.load(os.path.join(GOLD, "dequant_gguf_py.npz"))
    dt, be, bb = TYPES[name]
    raw, want = g[f"{name}_raw"], g[f"{name}_f32"]
    got = orc.dequantize(dt, raw.tobytes(), want.size)
    assert got.view(np.uint32).tolist() == want.view(np.uint32).tolist()
    if f"{name}_quantized_raw" in g:
        raw, want = g[f"{name}_quantized_raw"], g[f"{name}_quantized_f32"]
        got = orc.dequantize(dt, raw.tobytes(), want.size)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_q8_0_known_answers(orc):
    k = KAT["q8_0_one_block"]
    raw = _f16(k["scale"]) + bytes((i - 16) & 0xFF for i in range(32))
    assert orc.dequantize(8, raw, 32).tolist() == k["expect"]
    # zero scale gives exact zeros (src/quant.rs:306-311)
    assert not orc.dequantize(8, _f16(0.0) + bytes([127] * 32), 32).any()
    k = KAT["q8_0_two_blocks"]
    raw = _f16(1.0) + bytes([3] * 32) + _f16(2.0) + bytes([3] * 32)
    out = orc.dequantize(8, raw, 64)
    assert out[0] == k["expect_0"] and out[32] == k["expect_32"]


def test_q8_0_rejects_wrong_length(orc):
    """src/quant.rs:322-328"""
    raw = _f16(1.0) + bytes(32)
    for data, n in ((raw[:33], 32), (raw, 64), (raw, 31)):
        with pytest.raises(orc.OracleError):
            orc.dequantize(8, data, n)


@pytest.mark.parametrize("case,dt,bb,n", [("q4_k_hand", 12, 144, 256), ("q6_k_hand", 14, 210, 256),
                                          ("q5_0_hand", 6, 22, 32)])
def test_k_and_q5_hand_computed(orc, case, dt, bb, n):
    k = KAT[case]
    out = orc.dequantize(dt, _bytes(k["bytes"], bb), n)
    for idx, v in k["expect"].items():
        assert out[int(idx)] == v, (case, idx)


def test_fused_q8_matmul_matches_dequant_reference(orc):
    """src/quant.rs:331-357"""
    raw = b""
    for o in range(3):
        for b in range(2):
            q = bytes(((j * 7 + o * 13 + b * 5) % 255 - 127) & 0xFF for j in range(32))
            raw += _f16(0.5 + o * 0.25) + q
    x = np.sin(np.arange(128, dtype=np.float32) * np.float32(0.31)).reshape(2, 64)
    w = orc.dequantize(8, raw, 3 * 64).reshape(3, 64)
    ref = orc.matmul(x, w)
    fused = orc.matmul_quant(x, raw, 3, 64, 8)
    assert fused.shape == ref.shape
    assert np.all(np.abs(fused - ref) < 1e-4)


def test_fused_k_matmul_matches_dequant_reference(orc):
    """src/quant.rs:433-454"""
    raw = bytes(((i * 37 + 11) % 251) for i in range(2 * 144))
    x = np.sin(np.arange(3 * 256, dtype=np.float32) * np.float32(0.17)).reshape(3, 256)
    w = orc.dequantize(12, raw, 2 * 256).reshape(2, 256)
    ref = orc.matmul(x, w)
    fused = orc.matmul_quant(x, raw, 2, 256, 12)
    assert np.all(np.abs(fused - ref) <= 1e-3 * np.maximum(np.abs(ref), 1.0))


def test_f32_passthrough(orc):
    """src/quant.rs:456-464"""
    raw = struct.pack("<3f", 1.5, -2.25, 0.0)
    assert orc.dequantize(0, raw, 3).tolist() == [1.5, -2.25, 0.0]


def test_matmul_hand_computed(orc):
    """src/tensor.rs:258-269"""
    a = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    w = np.array([[1, 0, 1], [0, 1, 0]], np.float32)
    assert orc.matmul(a, w).tolist() == [[4, 2], [10, 5]]


def test_rmsnorm_softmax_silu(orc):
    k = KAT["rmsnorm_hand"]
    assert np.allclose(orc.rmsnorm(k["x"], k["w"], k["eps"]), k["expect"], atol=k["tol"], rtol=0)
    # zero row stays finite with eps inside the sqrt (src/tensor.rs:289-297)
    assert orc.rmsnorm([0, 0, 0], [1, 1, 1], 1e-5).tolist() == [0, 0, 0]
    k = KAT["softmax_hand"]
    assert np.allclose(orc.softmax(np.array([k["x"]])), [k["expect"]], atol=k["tol"], rtol=0)
    s = orc.softmax(np.array([[1000.0, 1001.0]]))  # src/tensor.rs:307-316
    assert np.isfinite(s).all() and abs(s.sum() - 1) < 1e-6 and s[0, 1] > s[0, 0]
    k = KAT["silu_points"]
    assert np.allclose(orc.silu(k["x"]), k["expect"], atol=k["tol"], rtol=0)
    assert abs(orc.swiglu([1.0], [2.0])[0] - k["swiglu"]["expect"]) < k["tol"]


def test_rope_known_vector(orc):
    k = KAT["rope_pos1"]
    x = orc.rope(np.array(k["x"], np.float32), 1, k["head_dim"], k["theta"], 0)
    assert np.allclose(x[4:], k["expect_row1"], atol=k["tol"], rtol=0)
    # position 0 is identity (src/model.rs:614-620)
    assert orc.rope(np.array([1, 2, 3, 4], np.float32), 1, 4, 1e6, 0).tolist() == [1, 2, 3, 4]


def test_gqa_and_causal_mask(orc):
    k = KAT["gqa_map"]
    out = orc.attention(np.ones(8, np.float32), np.ones(4, np.float32), np.array(k["v"], np.float32), 4, 2, 2)
    assert out.reshape(-1).tolist() == k["expect"]
    # causal mask (src/model.rs:640-656): token 0 sees only itself
    q = np.array([1, 0, 0, 1, 1, 1], np.float32)
    kk = np.array([1, 1, 0, 1, 1, 0], np.float32)
    v = np.eye(3, 2, dtype=np.float32) * 0 + np.array([[1, 0], [0, 1], [5, 5]], np.float32)
    out = orc.attention(q, kk, v, 1, 1, 2)
    assert out[0].tolist() == [1.0, 0.0]  # only v[0]


def test_argmax_first_max_wins(orc):
    for xs, want in KAT["argmax_ties"]["cases"]:
        assert orc.argmax(xs) == want


def test_sampler_known_answers(orc):
    k = KAT["sampler_temperature"]
    c = orc.Sampler(1.0, 0, 1.0, 1.0, 7).filtered(k["logits"])
    assert c[0][0] == 1 and abs(c[0][1] - k["t1"][0]) < 1e-5 and abs(c[1][1] - k["t1"][1]) < 1e-5
    c = orc.Sampler(0.5, 0, 1.0, 1.0, 7).filtered(k["logits"])
    assert abs(c[0][1] - k["t05"][0]) < 1e-5 and abs(c[1][1] - k["t05"][1]) < 1e-5
    k = KAT["sampler_top_k"]
    c = orc.Sampler(1.0, k["k"], 1.0, 1.0, 7).filtered(k["logits"])
    assert [i for i, _ in c] == k["ids"] and abs(sum(p for _, p in c) - 1) < 1e-5
    k = KAT["sampler_top_p"]
    lg = np.log(np.array(k["probs"], np.float32))
    c = orc.Sampler(1.0, 0, k["p"], 1.0, 7).filtered(lg)
    assert [i for i, _ in c] == k["ids"]
    assert np.allclose([p for _, p in c], k["expect"], atol=1e-5)
    k = KAT["repeat_penalty"]
    assert orc.repeat_penalty(k["logits"], k["recent"], k["penalty"]).tolist() == k["expect"]


def test_sampler_draws_and_seeds(orc):
    """src/sampler.rs:454-480"""
    lg = [0.1, 3.0, 0.2]
    s = orc.Sampler(0.0, 40, 0.9, 1.0, 7)
    assert s.sample(lg) == 1 and s.draws() == 0
    s = orc.Sampler(0.7, 1, 0.9, 1.0, 7)
    assert s.sample(lg) == 1 and s.draws() == 0
    s = orc.Sampler(0.7, 40, 0.9, 1.0, 7)
    s.sample(lg)
    assert s.draws() == 1
    flat = [(i % 7) * 0.01 for i in range(100)]

    def run(seed):
        s = orc.Sampler(1.0, 0, 1.0, 1.0, seed)
        return [s.sample(flat) for _ in range(20)]

    assert run(42) == run(42) and run(42) != run(43)


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


def test_gguf_parse_synthetic(orc):
    data = _synthetic_gguf()
    v, nt, nm, ds = orc.parse_gguf_bytes(data)
    assert (v, nt, nm) == (3, 1, 3) and ds % 32 == 0 and data[ds] == 0xAB
    with pytest.raises(orc.OracleError, match="bad magic"):
        orc.parse_gguf_bytes(b"GGML\x03\x00\x00\x00")
    with pytest.raises(orc.OracleError):
        orc.parse_gguf_bytes(data[:40])


def test_half_rounding_matches_numpy(orc):
    """The f16 KV cache's rounding (binary32 -> binary16, nearest even, with
    gradual underflow and overflow to infinity) against numpy's cast."""
    rng = np.random.default_rng(5)
    x = np.concatenate([rng.normal(0, 3, 20000), rng.normal(0, 1e-5, 2000),
                        [0.0, -0.0, 65504, 65519.99, 65520, 1e30, -1e30, np.inf, -np.inf,
                         2.9802322e-8, 2.98e-8, 5.96e-8, 6.1035156e-05, 3.0517578e-05]]).astype(np.float32)
    mine = np.array([orc.float_to_half(float(v)) for v in x], np.uint16)
    with np.errstate(over="ignore"):
        ref = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(mine, ref)
