"""Build the native parts in-tree (the built files travel with the repo).

- furnace_b200/_build/libfurnace_cuda.so : the product (CUDA kernels for
  sm_100a + the C ABI of include/furnace.h), compiled with nvcc.
- furnace_b200/_build/libfzsynth.so      : seeded synthetic GGUF data.
"""

from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "_build")
LIB = os.path.join(OUT, "libfurnace_cuda.so")
SYNTH = os.path.join(OUT, "libfzsynth.so")

CUDA_SOURCES = ["kernels.cu", "runtime.cu", "noalloc.cu"]
CXX_SOURCES = ["gguf.cpp", "nccl_dyn.cpp", "tokenizer.cpp"]
HEADERS = sorted(f for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))) + [os.path.join("..", "..", "include", "furnace.h")]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r


def build_cuda(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OUT, exist_ok=True)
    srcs = [os.path.join(CSRC, s) for s in CUDA_SOURCES + CXX_SOURCES]
    deps = srcs + [os.path.join(CSRC, h) for h in HEADERS] + [__file__]
    if not force and not _stale(LIB, deps):
        return LIB
    objs = []
    # host code keeps the reference's f32 operation order (no FMA contraction):
    # the sampler's softmax / top-p arithmetic must match it exactly
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                    "-Xcompiler", "-ffp-contract=off", "--expt-relaxed-constexpr"]
    if verbose:
        flags += ["-Xptxas", "-v"]
    for s in srcs:
        o = os.path.join(OUT, os.path.basename(s) + ".o")
        if force or _stale(o, [s] + [os.path.join(CSRC, h) for h in HEADERS] + [__file__]):
            r = _run([NVCC] + flags + ["-c", s, "-o", o])
            if verbose:
                print(r.stderr)
        objs.append(o)
    tmp = LIB + ".tmp"
    _run([NVCC] + ARCH + ["-shared", "-o", tmp] + objs + ["-lcudart", "-ldl"])
    os.replace(tmp, LIB)
    return LIB


def build_synth(force: bool = False) -> str:
    os.makedirs(OUT, exist_ok=True)
    src = os.path.join(CSRC, "synth.c")
    if force or _stale(SYNTH, [src]):
        tmp = SYNTH + ".tmp"
        _run(["gcc", "-O2", "-shared", "-fPIC", "-pthread", "-o", tmp, src, "-lm"])
        os.replace(tmp, SYNTH)
    return SYNTH


def build_all(force: bool = False) -> None:
    build_synth(force)
    build_cuda(force)


if __name__ == "__main__":
    import sys

    build_synth("--force" in sys.argv)
    print(build_cuda("--force" in sys.argv, verbose="-v" in sys.argv))
