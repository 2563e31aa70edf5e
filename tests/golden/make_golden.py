"""Generate the golden fixtures under tests/golden/.

Run from the repository root:  python tests/golden/make_golden.py

dequant_gguf_py.npz
    Seeded raw GGUF blocks of Q8_0, Q5_0, Q4_K and Q6_K with their f32
    dequantization as computed by gguf-py 0.19.0 (`gguf.quants.dequantize`),
    the independent decoder the furnace reference checks itself against
    (scripts/check_m2.py:12-14,45 and scripts/check_m10.py:14-15,44).  The
    blocks cover ordinary scales plus f16 edge values (subnormal, signed
    zero, largest finite) and, for Q8_0/Q5_0, blocks produced by gguf-py's
    own quantizer from N(0, 0.02) data.

reference_kat.json
    The known-answer constants of the reference's unit tests, with the
    file:line each comes from.  These pin the oracle (and through it the CUDA
    path) to the reference's own expectations.
"""

import json
import os

import numpy as np
from gguf import GGMLQuantizationType as T
from gguf import quants

HERE = os.path.dirname(os.path.abspath(__file__))
BLOCK = {"Q8_0": (32, 34, T.Q8_0), "Q5_0": (32, 22, T.Q5_0), "Q4_K": (256, 144, T.Q4_K), "Q6_K": (256, 210, T.Q6_K)}
# f16 bit patterns: ordinary, subnormal, signed zero, largest finite, tiny normal
F16_EDGES = [0x3C00, 0x3800, 0x0001, 0x03FF, 0x8000, 0x0000, 0x7BFF, 0xFBFF, 0x0400, 0xB4CD]


def f16_bits(rng, n):
    """Random finite f16 bit patterns with magnitudes in [2^-14, 2^2)."""
    e = rng.integers(1, 17, size=n)
    m = rng.integers(0, 1024, size=n)
    s = rng.integers(0, 2, size=n)
    return ((s << 15) | (e << 10) | m).astype(np.uint16)


def random_blocks(name, rng, n):
    be, bb, _ = BLOCK[name]
    raw = rng.integers(0, 256, size=(n, bb), dtype=np.uint8)
    # scale fields: keep them finite so the expected values are comparable
    scale_offsets = {"Q8_0": [0], "Q5_0": [0], "Q4_K": [0, 2], "Q6_K": [208]}[name]
    bits = f16_bits(rng, n * len(scale_offsets)).reshape(n, -1)
    for k in range(min(n, len(F16_EDGES))):
        bits[k, 0] = F16_EDGES[k]
    for j, off in enumerate(scale_offsets):
        raw[:, off] = bits[:, j] & 0xFF
        raw[:, off + 1] = bits[:, j] >> 8
    return raw


def main():
    rng = np.random.default_rng(20260101)
    out = {}
    for name, (be, bb, qt) in BLOCK.items():
        raw = random_blocks(name, rng, 24)
        out[f"{name}_raw"] = raw.reshape(-1)
        out[f"{name}_f32"] = quants.dequantize(raw, qt).reshape(-1).astype(np.float32)
    for name in ("Q8_0", "Q5_0"):
        be, bb, qt = BLOCK[name]
        x = rng.normal(0.0, 0.02, size=(16, 4 * be)).astype(np.float32)
        raw = quants.quantize(x, qt)
        out[f"{name}_quantized_raw"] = raw.reshape(-1)
        out[f"{name}_quantized_f32"] = quants.dequantize(raw, qt).reshape(-1).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "dequant_gguf_py.npz"), **out)

    kat = {
        "_doc": "Known-answer constants of the furnace reference's unit tests (paths inside the furnace project).",
        "q8_0_one_block": {"src": "src/quant.rs:295-304", "scale": 0.5, "quants": "i-16 for i in 0..32",
                           "expect": [0.5 * (i - 16) for i in range(32)]},
        "q8_0_two_blocks": {"src": "src/quant.rs:313-320", "scales": [1.0, 2.0], "quant": 3, "expect_0": 3.0,
                            "expect_32": 6.0},
        "q4_k_hand": {"src": "src/quant.rs:360-387",
                      "bytes": {"0": 0x00, "1": 0x3C, "2": 0x00, "3": 0x38, "4": 3, "8": 2, "5": 5, "9": 1,
                                "12": 7, "16": 0x51, "80": 0x04},
                      "expect": {"0": 2.0, "32": 24.5, "128": 28.0, "1": -1.0}},
        "q6_k_hand": {"src": "src/quant.rs:390-413",
                      "bytes": {"208": 0x00, "209": 0x38, "192": 2, "194": 1, "196": 3, "198": 255, "0": 0x21,
                                "128": 0xC4},
                      "expect": {"0": -31.0, "32": -8.0, "64": -45.0, "96": -8.0}},
        "q5_0_hand": {"src": "src/quant.rs:416-431", "bytes": {"0": 0x00, "1": 0x38, "2": 1, "6": 0x51},
                      "expect": {"0": 0.5, "16": -5.5, "1": -8.0}},
        "rmsnorm_hand": {"src": "src/tensor.rs:280-287", "x": [3.0, 4.0], "w": [2.0, 0.5], "eps": 0.0,
                         "expect": [1.69706, 0.56569], "tol": 1e-5},
        "softmax_hand": {"src": "src/tensor.rs:300-305", "x": [0.0, float(np.log(np.float32(2.0)))],
                         "expect": [1.0 / 3.0, 2.0 / 3.0], "tol": 1e-6},
        "silu_points": {"src": "src/tensor.rs:319-329", "x": [0.0, 1.0, -1.0], "expect": [0.0, 0.731059, -0.268941],
                        "swiglu": {"gate": 1.0, "up": 2.0, "expect": 1.462117}, "tol": 1e-5},
        "rope_pos1": {"src": "src/model.rs:623-637", "x": [9, 9, 9, 9, 1, 2, 3, 4], "head_dim": 4, "theta": 4.0,
                      "expect_row1": [-1.9841108, -0.1625368, 2.4623778, 4.4691815], "tol": 1e-5},
        "gqa_map": {"src": "src/model.rs:732-743", "v": [10, 20, 30, 40],
                    "expect": [10, 20, 10, 20, 30, 40, 30, 40]},
        "argmax_ties": {"src": "src/generate.rs:226-229", "cases": [[[1.0, 5.0, 5.0, 2.0], 1], [[-3.0, -1.0, -2.0], 1]]},
        "sampler_temperature": {"src": "src/sampler.rs:400-412", "logits": [0.0, float(np.log(np.float32(3.0)))],
                                "t1": [0.75, 0.25], "t05": [0.9, 0.1]},
        "sampler_top_k": {"src": "src/sampler.rs:415-421", "logits": [5.0, 1.0, 4.0, 2.0, 3.0], "k": 2, "ids": [0, 2]},
        "sampler_top_p": {"src": "src/sampler.rs:424-433", "probs": [0.5, 0.3, 0.15, 0.05], "p": 0.8,
                          "ids": [0, 1], "expect": [0.625, 0.375]},
        "repeat_penalty": {"src": "src/sampler.rs:436-443", "logits": [2.0, -2.0, 1.0], "recent": [0, 1, 0],
                           "penalty": 2.0, "expect": [1.0, -4.0, 1.0]},
    }
    with open(os.path.join(HERE, "reference_kat.json"), "w") as f:
        json.dump(kat, f, indent=1)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
