"""Tensor-parallel decode on 2 GPUs against the CPU oracle (one process per
GPU, NCCL inside the library, gloo only to hand out the NCCL id and to
collect results).  Needs two visible GPUs; skipped otherwise.

Bars as for one GPU: greedy ids identical to the oracle at every step,
logits within 1e-3 max-abs with identical argmax and top-5."""

import os
import socket

import numpy as np
import pytest

import furnace_b200 as fz
from furnace_b200 import synth
from tests.test_gpu_parity import _check_top5

pytestmark = pytest.mark.gpu
LOGIT_ABS = 1e-3


def _ngpus():
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0


def _rank(rank, world, port, path, n_prompt, n_new, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ids = [fz.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(ids, src=0)
        f = fz.GgufFile.open(path)
        m = fz.Model.load_tp(f, rank, world, ids[0], rank)
        prompt = synth.prompt_ids(m.config.vocab, n_prompt, seed=2)
        got_ids, got_lg = fz.generate(m, prompt, n_new, max_ctx=n_prompt + n_new, keep_logits=True)
        q.put((rank, (got_ids.tolist(), got_lg if rank == 0 else None), None))
        m.close()
        dist.barrier()
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e), None))
    finally:
        dist.destroy_process_group()


def _rank_prefill(rank, world, port, path, n_prompt, q):
    """One forward over the prompt (batched prefill for all but the last
    token), returning the logits and this rank's cached K/V rows."""
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ids = [fz.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(ids, src=0)
        f = fz.GgufFile.open(path)
        m = fz.Model.load_tp(f, rank, world, ids[0], rank)
        prompt = synth.prompt_ids(m.config.vocab, n_prompt, seed=5)
        kv = fz.KvCache(m, n_prompt + 4)
        lg, am = m.forward(prompt, kv)
        rows = {(li, w): kv.read(li, w, n_prompt) for li in range(m.config.n_layers) for w in (0, 1)}
        q.put((rank, (lg, am, rows), None))
        kv.close()
        m.close()
        dist.barrier()
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e), None))
    finally:
        dist.destroy_process_group()


def _spawn(target, world, *args):
    import torch.multiprocessing as mp

    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, world, port) + args + (q,)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, v, _ = q.get(timeout=600)
            res[r] = v
    finally:
        for p in procs:
            p.join(60)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert not isinstance(res[r], str), f"rank {r}: {res[r]}"
    return res


def _run_tp(path, n_prompt, n_new, world=2):
    from oracle import oracle

    res = _spawn(_rank, world, path, n_prompt, n_new)
    ref = oracle.Model(path)
    prompt = synth.prompt_ids(ref.vocab, n_prompt, seed=2)
    want_ids, want_lg, _, _ = ref.generate(prompt, n_new, keep_logits=True)
    for r in range(world):
        assert res[r][0] == want_ids.tolist(), f"rank {r} ids differ"
    got_lg = res[0][1]
    for s in range(len(want_ids)):
        err = np.abs(got_lg[s] - want_lg[s]).max()
        assert err <= LOGIT_ABS, f"step {s}: logits max-abs {err}"
        assert int(np.argmax(got_lg[s])) == int(np.argmax(want_lg[s])), f"step {s}: argmax"
        _check_top5(got_lg[s], want_lg[s], f"step {s}")


@pytest.fixture(scope="module", autouse=True)
def _two_gpus():
    if _ngpus() < 2:
        pytest.skip("tensor parallelism needs two GPUs")


def test_tp2_greedy_tiny(tmp_path):
    path = synth.write(synth.spec("tiny"), str(tmp_path / "tiny.gguf"))
    _run_tp(path, 9, 64)


@pytest.mark.slow
def test_tp2_greedy_c1():
    """C1 (Q8_0, 14 heads / 2 KV heads) split over 2 GPUs, 128 steps."""
    _run_tp(synth.ensure("c1"), 32, 128)


@pytest.mark.parametrize("over", [{}, {"hidden": 768, "n_heads": 12}], ids=["tiny", "tiny-768"])
def test_tp2_batched_prefill(tmp_path, over):
    """A 100-token prompt through the batched prefill on 2 ranks: each rank's
    cached K/V rows equal the oracle's rows of its KV heads (1e-4 of the
    largest element, as on one GPU), the prompt's logits meet the logits bar,
    and greedy decoding after it gives the oracle's ids.  With 12 heads of 64
    each rank's o_proj input (384 columns) widens to whole 256-element Q4_K
    blocks in odd layers, so ctx sits at an offset inside zero padding."""
    from oracle import oracle

    path = synth.write(synth.spec("tiny", **over), str(tmp_path / "tiny.gguf"))
    n, world = 100, 2
    res = _spawn(_rank_prefill, world, path, n)
    ref = oracle.Model(path)
    prompt = synth.prompt_ids(ref.vocab, n, seed=5)
    kr = ref.kv_new(n + 4)
    want = ref.forward_cached(prompt, kr)
    for r in range(world):
        lg, am, rows = res[r]
        _check_top5(lg, want, f"rank {r} prefill logits")
        assert np.abs(lg - want).max() <= LOGIT_ABS, f"rank {r}: logits max-abs {np.abs(lg - want).max()}"
        assert am == int(np.argmax(want)), f"rank {r}: argmax"
        kvh = ref.n_kv_heads // world
        cols = slice(r * kvh * ref.head_dim, (r + 1) * kvh * ref.head_dim)
        for (li, w), a in rows.items():
            b = kr.read(li, w, n)[:, cols]
            assert np.abs(a - b).max() <= 1e-4 * max(1.0, np.abs(b).max()), (r, li, w)
    _run_tp(path, n, 24)


def _need(n):
    if _ngpus() < n:
        pytest.skip(f"needs {n} GPUs")


@pytest.mark.slow
def test_tp4_greedy_c3_truncated():
    """C3 at TP4 (the benchmarked 7B shape, 2 of its 28 layers at full
    width): 7 query heads and 1 KV head per rank; each rank's o_proj input
    is 896 columns, 3.5 Q4_K super-blocks, so neighbours share a boundary
    block; the FFN's 74 super-blocks split 18/19/18/19 (fz_tp_slice_of cuts
    on 256-element boundaries).  A 40-token prompt (batched prefill), then 64
    greedy steps against the oracle."""
    _need(4)
    _run_tp(synth.ensure("c3", n_layers=2), 40, 64, world=4)


@pytest.mark.slow
@pytest.mark.parametrize("name", ["c4", "c5"])
def test_tp8_greedy_truncated_c4_c5(name):
    """TP8 on the 32B and 72B shapes (2 layers at full width): C4's FFN of
    108 super-blocks splits 13/14 alternately; C5's FFN of 29568 (not a
    multiple of 256, so ffn_down is Q8_0 / Q5_0 in 32-element blocks) splits
    into slices of 3584/3840 elements and a last one of 3712 (14.5 units of
    256).  40-token prompt, 64 greedy steps."""
    _need(8)
    _run_tp(synth.ensure(name, n_layers=2), 40, 64, world=8)
