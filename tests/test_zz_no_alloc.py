"""fz_dequant_dev_noalloc (device dequantize that allocates nothing), called
through the C ABI.

Each case is checked twice: against the existing entry point fz_dequant (the
same C ABI with host buffers) and against the CPU oracle's restatement of the
reference's block decoders (oracle.dequantize, src/quant.rs:17-133), so the
device repack + dequantization is not only compared with itself.

The file name sorts last, so in a full run the entry point is exercised after
every other test has used the device (and again when the file runs alone).
Dequantization is bit-exact, so the tolerance is equality of the f32 bits.
"""

import numpy as np
import pytest

import furnace_b200 as fz
from furnace_b200 import synth
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 8 << 20
Q5_0, Q8_0, Q4_K, Q6_K = 6, 8, 12, 14


@pytest.fixture(scope="module")
def torch_cuda():
    from tests.conftest import gpu_available

    if not gpu_available():
        pytest.fail("GPU tests need a CUDA device")
    import torch

    fz.load_library()
    return torch


def _to_dev(torch, raw: bytes):
    return torch.from_numpy(np.frombuffer(raw, dtype=np.uint8).copy()).cuda()


def _call(torch, dt, src, nbytes, n, out):
    stream = torch.cuda.current_stream().cuda_stream
    rc = fz.load_library().fz_dequant_dev_noalloc(dt, src.data_ptr(), nbytes, n, out.data_ptr(), stream)
    return rc


def _expect(dt, raw, n):
    """The oracle's dequantization, which fz_dequant must also equal bit for bit."""
    want = orc.dequantize(dt, raw, n)
    ours = fz.quant.dequantize(dt, raw, n)
    assert np.array_equal(ours.view(np.uint32), want.view(np.uint32))
    return want


def _same_bits(out, want):
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_two_consecutive_calls_match_oracle_and_fz_dequant(torch_cuda):
    torch = torch_cuda
    # different formats and sizes, queued back to back on one stream: the
    # second call reuses the scratch the first one filled
    cases = [(Q6_K, 48, 1024, 21), (Q4_K, 20, 2048, 22), (Q5_0, 33, 4096, 24)]
    srcs, outs, wants = [], [], []
    for dt, rows, cols, seed in cases:
        raw = synth.random_tensor(rows, cols, dt, seed=seed)
        wants.append(_expect(dt, raw, rows * cols))
        srcs.append((_to_dev(torch, raw), len(raw), rows * cols))
        outs.append(torch.full((rows * cols,), float("nan"), device="cuda"))
    for (dt, *_), (src, nbytes, n), out in zip(cases, srcs, outs):
        assert _call(torch, dt, src, nbytes, n, out) == fz.FZ_OK, fz.load_library().fz_last_error()
    torch.cuda.synchronize()
    for want, out in zip(wants, outs):
        _same_bits(out, want)


def test_repeat_call_and_ragged_block_count(torch_cuda):
    torch = torch_cuda
    # a prime block count gives one-block rows (the layout's largest blow-up);
    # the same call twice must give the same bits both times
    nblk = 4099
    raw = synth.random_tensor(1, 32 * nblk, Q8_0, seed=23)
    want = _expect(Q8_0, raw, 32 * nblk)
    src = _to_dev(torch, raw)
    for _ in range(2):
        out = torch.full((32 * nblk,), float("nan"), device="cuda")
        assert _call(torch, Q8_0, src, len(raw), 32 * nblk, out) == fz.FZ_OK
        torch.cuda.synchronize()
        _same_bits(out, want)


def test_q5_0_near_the_documented_limit(torch_cuda):
    torch = torch_cuda
    # Q5_0 has the largest layout blow-up (about 2.9x the GGUF bytes for a
    # prime block count); the largest prime count under 2 MiB of GGUF data
    # must still fit the scratch, twice in a row
    nblk = 95317
    assert nblk * 22 <= 2 << 20
    raw = synth.random_tensor(1, 32 * nblk, Q5_0, seed=25)
    want = _expect(Q5_0, raw, 32 * nblk)
    src = _to_dev(torch, raw)
    for _ in range(2):
        out = torch.full((32 * nblk,), float("nan"), device="cuda")
        assert _call(torch, Q5_0, src, len(raw), 32 * nblk, out) == fz.FZ_OK, fz.load_library().fz_last_error()
        torch.cuda.synchronize()
        _same_bits(out, want)


def test_rejects_tensor_beyond_scratch(torch_cuda):
    torch = torch_cuda
    # 300000 Q8_0 blocks repack to more than 8 MiB: refused on the host,
    # before anything is queued (the small buffers are never touched)
    src = torch.zeros(16, dtype=torch.uint8, device="cuda")
    out = torch.zeros(4, device="cuda")
    for nblk in (300000, 1 << 40):
        rc = _call(torch, Q8_0, src, 34 * nblk, 32 * nblk, out)
        assert rc == fz.FZ_EINVAL
        assert b"scratch" in fz.load_library().fz_last_error()
    torch.cuda.synchronize()
