"""Benchmark: batch-1 greedy decode tokens/s (and achieved HBM GB/s) of the
furnace decode loop on B200.

Workload (N=1): configuration C3, the Qwen2.5-7B shape in the Q4_K_M mix
(synthetic seeded weights, same shapes/dtypes), 2048 random prompt ids
prefilled, then greedy decode at positions 2048.. .  A "step" is STEP_TOKENS
(16) decode tokens; --steps K times K steps (default 32 -> the config's 512
decode tokens).  Weights streamed per token (4.4 GB) exceed L2 (126 MB), so no
L2 flush is needed between steps.

value : decode tok/s with inputs resident in HBM, CUDA events on the
        library's stream around all K steps (max over ranks).
e2e   : the same metric through the public C-ABI call (fz_decode_greedy)
        with host buffers, one call per step, host->device token and
        device->host ids inside the timed region.
--impl reference : the reference path's CPU implementation (the C++
        restatement in oracle/, the reference itself cannot be built here)
        timed on the host cores, one decode token per step.

With --gpus N > 1 (torchrun, one process per GPU) the ranks form N / TP
groups of --tp TP consecutive ranks.  A group decodes one stream,
tensor-parallel over its TP GPUs (one NCCL communicator per group), and the
groups decode independent streams: value = total tokens/s of all groups;
scaling "strong" when one group spans all N GPUs, else "weak".  The default
TP is the largest degree <= N that divides N and both head counts: one
group over all N GPUs where the model allows it (C3 at N = 2 and 4), two
TP4 groups for C3 at N = 8 (28 query heads do not split 8 ways); --tp 1
gives N independent replicas.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
# rank 0 prints exactly one JSON line: keep NCCL's version banner off stdout
os.environ["NCCL_DEBUG"] = "WARN"
# Under tensor parallelism the decode step's NCCL traffic is setup and an
# 8-byte argmax all-reduce per token (the residual exchange runs over peer
# memory); only the batched prefill all-reduces [T, H] partials.  NVLink
# SHARP (NVLS) stays off unless the caller sets it, as in the measured runs.
os.environ.setdefault("NCCL_NVLS_ENABLE", "0")

STEP_TOKENS = 16
CONFIG = "c3"
PREFILL = 2048


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default=CONFIG)
    ap.add_argument("--prefill", type=int, default=PREFILL)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tp", type=int, default=None,
                    help="tensor-parallel group size (divides --gpus); default: the largest the model allows")
    ap.add_argument("--kv", default="f32", choices=["f32", "f16"],
                    help="KV cache elements (f32: the reference's; f16: the 32B config's 8K-context cache)")
    ap.add_argument("--layers", type=int, default=None,
                    help="layer-truncated variant of the config (same per-layer shapes; for large configs)")
    return ap.parse_args()


class Dist:
    """torch.distributed (gloo) only for the barrier and the max-over-ranks."""

    def __init__(self, n):
        self.rank = int(os.environ.get("RANK", 0))
        self.world = int(os.environ.get("WORLD_SIZE", 1))
        self.local = int(os.environ.get("LOCAL_RANK", 0))
        self.pg = None
        if self.world > 1:
            import datetime

            import torch.distributed as td

            td.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
            self.pg = td

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch

        t = torch.tensor([v], dtype=torch.float64)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def bcast(self, obj):
        """rank 0's obj on every rank."""
        if not self.pg:
            return obj
        box = [obj]
        self.pg.broadcast_object_list(box, src=0)
        return box[0]

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


class Cudart:
    """CUDA events on the library's stream (the same libcudart it links)."""

    def __init__(self):
        import ctypes as C

        for name in ("libcudart.so.12", "libcudart.so"):
            try:
                self.L = C.CDLL(name)
                break
            except OSError:
                continue
        else:
            self.L = C.CDLL("/usr/local/cuda/lib64/libcudart.so")
        self.C = C

    def event(self):
        e = self.C.c_void_p()
        assert self.L.cudaEventCreate(self.C.byref(e)) == 0
        return e

    def record(self, e, stream):
        assert self.L.cudaEventRecord(e, self.C.c_void_p(stream)) == 0

    def elapsed_ms(self, a, b):
        assert self.L.cudaEventSynchronize(b) == 0
        t = self.C.c_float()
        assert self.L.cudaEventElapsedTime(self.C.byref(t), a, b) == 0
        return t.value

    def set_device(self, d):
        self.L.cudaSetDevice(d)


class ClockSampler:
    """nvidia-smi clocks/throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.idx)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.t.join(timeout=2)
        mhz, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                mhz.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(mhz)}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


def ncu_traffic(config: str, layers, tp: int):
    """DRAM bytes of one decode token's k_gemv launches from the committed
    ncu summary, when that summary was taken on this workload (same config,
    full depth, one GPU); None otherwise."""
    p = os.path.join(ROOT, "profiles", "gemv_traffic.json")
    if not os.path.exists(p):
        return None
    try:
        d = json.load(open(p))
    except Exception:
        return None
    if d.get("config") != config or layers is not None or tp != 1:
        return None
    return d


def cpu_model() -> str:
    """The host CPU's model name (/proc/cpuinfo), or "unknown"."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_baseline(path, vocab, context, budget_s=15.0):
    """The reference path's CPU restatement (oracle/) on all host cores,
    decoding at the GPU arm's positions: the cache holds `context` positions
    (seeded synthetic rows; a decode step's cost does not depend on the
    cached values), then greedy decode tokens until ~budget_s of decode time."""
    from oracle import oracle

    cores = os.cpu_count() or 1
    oracle.set_threads(cores)
    m = oracle.Model(path)
    kv = m.kv_new(context + 64)
    kv.fill_synthetic(context, seed=1)
    n, dec, tok = 0, 0.0, 1
    while n < 32 and (dec < budget_s or n < 2):
        t0 = time.perf_counter()
        lg = m.forward_cached([tok], kv)
        dec += time.perf_counter() - t0
        tok = int(lg.argmax())
        n += 1
    m.close()
    return {"value": n / dec, "unit": "tok/s", "cores": cores, "kind": "port", "cpu": cpu_model(),
            "sample": f"{n} greedy decode tokens at positions {context}-{context + n - 1} (context filled with "
                      f"seeded synthetic K/V rows), same synthetic GGUF, oracle/ C++ restatement of the reference "
                      f"CPU path, {cores} threads"}


def run_reference(args, dist):
    """--impl reference: the reference's CPU path (restated) on host cores, at
    the GPU arm's context: positions prefill.. of the same model."""
    from furnace_b200 import synth
    from oracle import oracle

    if dist.rank != 0:
        return
    path = synth.ensure(args.config, args.layers)
    spec = synth.spec(args.config, args.layers)
    cores = os.cpu_count() or 1
    oracle.set_threads(cores)
    m = oracle.Model(path)
    kv = m.kv_new(args.prefill + args.warmup + args.steps + 16)
    kv.fill_synthetic(args.prefill, seed=1)
    tok = 1
    for _ in range(args.warmup):
        tok = int(m.forward_cached([tok], kv).argmax())
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tok = int(m.forward_cached([tok], kv).argmax())
    dt = time.perf_counter() - t0
    v = args.steps / dt
    p0 = args.prefill + args.warmup
    sample = (f"one greedy decode token per step (a sample of the {STEP_TOKENS}-token step) at positions "
              f"{p0}-{p0 + args.steps - 1}, the {args.prefill}-position context filled with seeded synthetic K/V "
              f"rows, oracle/ C++ restatement of the reference CPU path (Rust toolchain absent), {cores} threads")
    line = {"metric": "decode_tok_per_s", "value": v, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt * 1000 / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": workload_config(spec, args, args.steps * STEP_TOKENS, f"cpu{cores}", 1),
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": "port", "cpu": cpu_model(),
                             "sample": sample},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def workload_config(spec, args, total_tokens, parallelism, groups):
    """The workload both arms report (same keys and values but parallelism)."""
    return {"workload": f"{spec.name}: {args.prefill}-token context, then greedy decode (batch 1) at positions "
                        f"{args.prefill}..", "model": spec.name, "global_batch": groups,
            "seq_len": args.prefill + total_tokens, "parallelism": parallelism,
            "l2": "inputs larger than L2: the weights streamed per token exceed 126 MB", "kv": args.kv}


def default_tp(world: int, spec) -> int:
    """The largest tensor-parallel degree <= world that divides world and the
    query and KV head counts: one group over every GPU when the model allows
    it (strong scaling), else groups of that size side by side."""
    for t in range(world, 0, -1):
        if world % t == 0 and spec.n_heads % t == 0 and spec.n_kv_heads % t == 0:
            return t
    return 1


def run_ours(args, dist):
    import furnace_b200 as fz
    from furnace_b200 import synth

    spec = synth.spec(args.config, args.layers)
    if dist.rank == 0:
        path = synth.ensure(args.config, args.layers)
    dist.barrier()
    path = synth.ensure(args.config, args.layers)
    dev = dist.local
    cud = Cudart()
    cud.set_device(dev)
    f = fz.GgufFile.open(path)
    # tensor-parallel groups of `tp` consecutive ranks (see the module docstring)
    tp = default_tp(dist.world, spec) if args.tp is None else max(1, min(args.tp, dist.world))
    if dist.world % tp or spec.n_heads % tp or spec.n_kv_heads % tp:
        raise SystemExit(f"--tp {tp} must divide --gpus {dist.world} and the head counts")
    groups = dist.world // tp
    t_load = time.perf_counter()
    if tp > 1:
        ids = dist.bcast([fz.tp_unique_id() for _ in range(groups)] if dist.rank == 0 else None)
        model = fz.Model.load_tp(f, dist.rank % tp, tp, ids[dist.rank // tp], dev)
    else:
        model = fz.Model.load(f, devices=[dev])
    load_s = time.perf_counter() - t_load
    cfg = model.config
    resident, per_tok = model.param_bytes()
    stream, _ = model.stream()
    T = STEP_TOKENS
    total_tokens = args.steps * T
    max_ctx = args.prefill + max(args.warmup * T, 2 * T) + total_tokens + 8
    kv = fz.KvCache(model, max_ctx, fz.FZ_KV_F16 if args.kv == "f16" else fz.FZ_KV_F32)
    prompt = synth.prompt_ids(cfg.vocab, args.prefill, seed=dist.rank // tp)  # one prompt per TP group
    t0 = time.perf_counter()
    _, first = model.forward(prompt, kv, want_logits=False)
    prefill_s = time.perf_counter() - t0
    base = kv.len
    # warm-up steps (untimed), then rewind so the timed tokens sit at base..
    tok = first
    for _ in range(args.warmup):
        ids, _ = model.decode_greedy(tok, T + 1, kv)
        tok = int(ids[-1])
    kv.len = base
    # ---- device-timed region: K steps enqueued back to back -------------
    sampler = ClockSampler(dev)
    sampler.start()
    time.sleep(0.3)
    dist.barrier()
    e0, e1 = cud.event(), cud.event()
    cud.record(e0, stream)
    ids, _ = model.decode_greedy(first, total_tokens + 1, kv)
    cud.record(e1, stream)
    ms = cud.elapsed_ms(e0, e1)
    dist.barrier()
    clocks = sampler.stop()
    ms = dist.max(ms)
    tok_s = total_tokens * groups / (ms / 1000.0)
    ms_tok = ms / total_tokens
    # ---- e2e: public API, one call per step, host buffers ---------------
    kv.len = base
    dist.barrier()
    t0 = time.perf_counter()
    tok = first
    for _ in range(args.steps):
        ids2, _ = model.decode_greedy(tok, T + 1, kv)
        tok = int(ids2[-1])
    e2e_s = dist.max(time.perf_counter() - t0)
    e2e = {"value": total_tokens * groups / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 4 + 32,
           "d2h_bytes_per_step": 4 * (T + 1) + 32,
           "note": "fz_decode_greedy per step; h2d = seed token + step state, d2h = ids + status"}
    # ---- where a token's time goes, and its algorithmic bytes ------------
    # fz_step_profile: CUDA events around each launch outside the graph
    # (serialised, so only the shares are meaningful); the bytes are the
    # algorithmic bytes of every op at the timed region's mean position
    kv.len = base + total_tokens // 2
    prof = model.step_profile(first, T, kv)
    bytes_tok = sum(v[1] for v in prof.values()) / T  # weights, KV rows read, vectors
    peak, peak_src = measured_peaks()
    achieved = bytes_tok / (ms_tok / 1000.0) / 1e9
    prof_ms = sum(v[0] for v in prof.values())
    ops = {o: {"ms_per_token": prof[o][0] / T, "share": prof[o][0] / prof_ms if prof_ms else None,
               "gbs": (prof[o][1] / (prof[o][0] / 1000.0) / 1e9) if prof[o][0] else None} for o in prof}
    traffic = ncu_traffic(args.config, args.layers, tp)
    roofline = {"kernel": "decode step (k_gemv x4, k_attn, k_attn_combine per layer; lm_head k_gemv)", "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_source": f"{peak_src} hbm_gbs (burst copy)",
                "bytes_per_launch": bytes_tok, "launch_us": ms_tok * 1000.0,
                "how": "algorithmic bytes of one token (GGUF weight bytes of every matrix, the KV rows read at the "
                       "timed region's mean position, vectors) / the device-timed ms per token of the timed region",
                "traffic": traffic.get("dram_bytes_per_launch") if traffic else None,
                "traffic_source": traffic.get("source") if traffic else None}
    hbm = per_tok * tok_s / groups / 1e9  # this rank's weight bytes per token x the group's token rate
    out = {
        "metric": "decode_tok_per_s", "value": tok_s, "unit": "tok/s", "n_gpus": dist.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "strong" if groups == 1 else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(spec, args, total_tokens, f"tp{tp}" + (f"x{groups}" if groups > 1 else ""),
                                  groups),
        "hbm_gbs_per_gpu": hbm, "hbm_frac_of_8tbs": hbm / 8000.0, "hbm_frac_of_measured": hbm / peak,
        "bytes_per_token": per_tok, "ms_per_token": ms_tok, "prefill_s": prefill_s,
        "load": {"s": load_s, "gb": resident / 1e9,
                 "note": "host wall clock of fz_model_load(_tp): GGUF bytes of this rank's share from the "
                         "page cache to the device and the repack into the chunk layout"},
        "prefill": {"tokens": args.prefill, "s": prefill_s, "tok_s": args.prefill / prefill_s,
                    "path": ("tcgen05 GEMM (fp16 hi/lo split, f32 accumulation) for all but the last prompt token"
                             + (f", residual partials all-reduced over {tp} ranks (NCCL)" if tp > 1 else ""))
                    if args.prefill > 8 else "decode step per token",
                    "note": "host wall clock of fz_forward over the prompt, including the per-layer weight "
                            "dequantization into GEMM panels"},
        "gpu_launches": (6 * cfg.n_layers + 3) * total_tokens, "clocks": clocks, "e2e": e2e,
        "roofline": roofline,
        "ops": ops, "ops_timing": "CUDA events per launch outside the graph, serialised: shares only",
    }
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(path, cfg.vocab, base)
    if dist.rank == 0:
        print(json.dumps(out), flush=True)
    kv.close()
    model.close()


def main():
    args = parse()
    dist = Dist(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, dist)
        else:
            run_ours(args, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
