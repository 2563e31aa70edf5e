"""Failure handling on one GPU, without a GPU fault.

A tensor-parallel rank whose peer never joins must get an error within the
configured limit instead of blocking forever (SURVEY-planned failure
detection; the reference itself only panics on misuse, src/model.rs:348-352).
The communicator is created non-blocking (ncclCommInitRankConfig with
blocking = 0); the library polls it, and past FURNACE_B200_NCCL_TIMEOUT_S it
aborts the communicator and returns FZ_ETIMEOUT.  Nothing runs on the device
while the rank waits, and the device stays usable afterwards.
"""

import time

import numpy as np
import pytest

import furnace_b200 as fz
from furnace_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    from tests.conftest import gpu_available

    if not gpu_available():
        pytest.fail("GPU tests need a CUDA device")
    fz.load_library()


def test_peer_that_never_joins_ends_in_a_timeout(tmp_path, monkeypatch, orc):
    path = synth.write(synth.spec("tiny"), str(tmp_path / "tiny.gguf"))
    f = fz.GgufFile.open(path)
    monkeypatch.setenv("FURNACE_B200_NCCL_TIMEOUT_S", "3")
    monkeypatch.setenv("NCCL_NVLS_ENABLE", "0")
    uid = fz.tp_unique_id()
    t0 = time.monotonic()
    with pytest.raises(fz.FurnaceError) as e:
        fz.Model.load_tp(f, 0, 2, uid, 0)  # rank 1 of 2 never joins
    waited = time.monotonic() - t0
    assert e.value.code == fz.FZ_ETIMEOUT, e.value
    assert 2.5 <= waited < 60, waited
    # the device still works: a one-GPU model gives the oracle's logits
    dev = fz.Model.load(f)
    ref = orc.Model(path)
    ids = synth.prompt_ids(ref.vocab, 6, seed=3)
    kd = fz.KvCache(dev, 16)
    got, _ = dev.forward(ids, kd)
    want = ref.forward_cached(ids, ref.kv_new(16))
    assert np.abs(got - want).max() <= 1e-3


def test_exchange_wait_runs_out_and_the_device_stays_usable(tmp_path, orc):
    """The residual exchange of tensor parallelism polls peer words with a
    bounded wait.  With a peer that never writes and a 20 ms limit, the GEMV
    records error 7 and returns, the call reports FZ_ETIMEOUT, and the next
    model on the device computes the oracle's logits."""
    L = fz.load_library()
    t0 = time.monotonic()
    rc = L.fz_selftest_exchange_timeout(0, 20000)
    assert rc == fz.FZ_ETIMEOUT, L.fz_last_error()
    assert time.monotonic() - t0 < 30
    path = synth.write(synth.spec("tiny"), str(tmp_path / "tiny.gguf"))
    dev = fz.Model.load(fz.GgufFile.open(path))
    ref = orc.Model(path)
    ids = synth.prompt_ids(ref.vocab, 5, seed=4)
    got, _ = dev.forward(ids, fz.KvCache(dev, 16))
    want = ref.forward_cached(ids, ref.kv_new(16))
    assert np.abs(got - want).max() <= 1e-3
