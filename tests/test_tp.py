"""Tensor parallelism: host-side logic on the CPU.

* fz_tp_slice_of partitions heads, KV heads, the FFN (on 256-element
  boundaries) and the vocabulary, for every config and rank count the
  configs' head counts allow;
* the split's arithmetic, checked on the oracle's dequantized weights: the
  o_proj partial sums of the ranks' head slices (a slice that is not
  block-aligned shares its boundary block, the neighbour's columns
  multiplying zeros) add up to the full product;
* two gloo ranks exchange an NCCL id and load a model slice; without a GPU
  both fail cleanly with FZ_ECUDA (no hang, no partial state).
"""

import os

import numpy as np
import pytest

import furnace_b200 as fz
from furnace_b200 import synth


def _cfg(name):
    s = synth.spec(name)
    return fz.Config(s.n_layers, s.n_heads, s.n_kv_heads, s.hidden, s.ffn, s.hidden // s.n_heads, s.rope_theta,
                     s.rms_eps, s.vocab, s.context_length)


@pytest.mark.parametrize("name", ["tiny", "c1", "c2", "c3", "c4", "c5"])
def test_slices_partition_the_model(name):
    c = _cfg(name)
    for world in (1, 2, 4, 8):
        if c.n_heads % world or c.n_kv_heads % world:
            with pytest.raises(fz.FurnaceError) as e:
                fz.tp_slice(c, 0, world)
            assert e.value.code == fz.FZ_EINVAL
            continue
        sl = [fz.tp_slice(c, r, world) for r in range(world)]
        q = kv = f = v = 0
        for r, s in enumerate(sl):
            assert s["q_head0"] == q and s["q_heads"] == c.n_heads // world
            assert s["kv_head0"] == kv and s["kv_heads"] == c.n_kv_heads // world
            assert s["o_col0"] == s["q_head0"] * c.head_dim and s["o_cols"] == s["q_heads"] * c.head_dim
            # GQA groups stay whole: the rank's query heads use its KV heads
            g = c.n_heads // c.n_kv_heads
            assert s["q_head0"] // g == s["kv_head0"] and s["q_heads"] == g * s["kv_heads"]
            assert s["ffn0"] == f and s["ffn0"] % 256 == 0 and s["ffn_n"] > 0 and s["ffn_n"] % 16 == 0
            assert s["vocab0"] == v and s["vocab_pad"] % world == 0
            assert s["vocab0"] == r * (s["vocab_pad"] // world)
            q += s["q_heads"]
            kv += s["kv_heads"]
            f += s["ffn_n"]
            v += s["vocab_n"]
        assert (q, kv, f, v) == (c.n_heads, c.n_kv_heads, c.ffn, c.vocab)


def test_rank_out_of_range():
    c = _cfg("c3")
    for r, w in ((2, 2), (-1, 2), (0, 0)):
        with pytest.raises(fz.FurnaceError):
            fz.tp_slice(c, r, w)


def test_head_split_partials_sum_to_full_product(orc):
    """o_proj of the tiny model (Q4_K, 256-element blocks, 8 heads of 64):
    at 4 ranks each rank owns 128 columns, half a block."""
    raw = synth.random_tensor(512, 512, 12, seed=7)
    w = orc.dequantize(12, raw, 512 * 512).reshape(512, 512)
    ctx = np.random.default_rng(1).normal(0, 1, 512).astype(np.float32)
    full = w.astype(np.float64) @ ctx
    c = fz.Config(3, 8, 4, 512, 1024, 64, 1e6, 1e-6, 4096, 4096)
    total = np.zeros(512)
    for r in range(4):
        s = fz.tp_slice(c, r, 4)
        c0, c1 = s["o_col0"], s["o_col0"] + s["o_cols"]
        a0, a1 = c0 // 256 * 256, -(-c1 // 256) * 256  # the rank's block-aligned columns
        x = np.zeros(a1 - a0)
        x[c0 - a0:c1 - a0] = ctx[c0:c1]  # the neighbour's part of a shared block is zero
        total += w[:, a0:a1].astype(np.float64) @ x
    assert np.abs(total - full).max() <= 1e-9 * np.abs(full).max()


def _rank_main(rank, world, port, path, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ids = [None]
        if rank == 0:
            try:
                ids[0] = fz.tp_unique_id()
            except fz.FurnaceError:
                ids[0] = bytes(128)  # no NCCL bootstrap here: the load must still fail cleanly
        dist.broadcast_object_list(ids, src=0)
        f = fz.GgufFile.open(path)
        try:
            fz.Model.load_tp(f, rank, world, ids[0], 0)
            q.put((rank, "loaded"))
        except fz.FurnaceError as e:
            q.put((rank, e.code))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_share_an_id_and_fail_cleanly_without_gpu(tmp_path):
    from tests.conftest import gpu_available

    if gpu_available():
        pytest.skip("covered by the GPU tensor-parallel test")
    import socket

    import torch.multiprocessing as mp

    path = synth.write(synth.spec("tiny"), str(tmp_path / "tiny.gguf"))
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, path, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    got = dict(q.get(timeout=5) for _ in range(2))
    assert got == {0: fz.FZ_ECUDA, 1: fz.FZ_ECUDA}
