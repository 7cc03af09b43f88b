"""Builds the in-tree native libraries of the sampler.

    libzs_sampler.so   CUDA kernels (sm_100a) + C ABI + zen:: C++ API
    libzs_workload.so  synthetic logits generator (host C)
    bench_host_api     timing driver of the drop-in C++ API (zen::sample_token)

Both land next to this file, so they travel with the source tree.  Rebuilds
only when a source is newer than its library (or force=True).

    python -m zeninfer_b200.build [--force]
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")

SAMPLER_SO = os.path.join(HERE, "libzs_sampler.so")
WORKLOAD_SO = os.path.join(HERE, "libzs_workload.so")
HOST_API_BENCH = os.path.join(HERE, "bench_host_api")

SAMPLER_SOURCES = ["zs_sampler.cu", "zs_noalloc_scratch.cu", "sample_shim.cpp"]
SAMPLER_DEPS = SAMPLER_SOURCES + ["zs_kernels.cuh", "zs_device.cuh", "zs_stats.cuh", "zs_lmhead.cuh"]

NVCC_ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = NVCC_ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                          "-Xcompiler", "-fvisibility=default"]
HOST_ARCH = "-march=x86-64-v3"


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed: " + " ".join(cmd) + "\n" + r.stdout + r.stderr)


def build_sampler(force: bool = False, verbose_ptxas: bool = False) -> str:
    deps = [os.path.join(CSRC, f) for f in SAMPLER_DEPS]
    deps += [os.path.join(INCLUDE, "zs_sampler.h"), os.path.join(INCLUDE, "zen", "sample.h")]
    if not force and not _stale(SAMPLER_SO, deps):
        return SAMPLER_SO
    tmp = SAMPLER_SO + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, "-shared", f"-I{INCLUDE}", "-o", tmp]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    # -Bsymbolic: the library's zen:: functions call their own definitions even in
    # a process that also loads another sample.h implementation.
    cmd += [os.path.join(CSRC, f) for f in SAMPLER_SOURCES] + ["-ldl", "-Xlinker", "-Bsymbolic"]
    _run(cmd)
    os.replace(tmp, SAMPLER_SO)
    return SAMPLER_SO


def build_workload(force: bool = False) -> str:
    src = os.path.join(CSRC, "workload.c")
    if not force and not _stale(WORKLOAD_SO, [src]):
        return WORKLOAD_SO
    tmp = WORKLOAD_SO + ".tmp"
    _run(["gcc", "-std=c11", "-O2", HOST_ARCH, "-fPIC", "-ffp-contract=off", "-shared",
          "-o", tmp, src, "-lm", "-lpthread"])
    os.replace(tmp, WORKLOAD_SO)
    return WORKLOAD_SO


def build_host_api_bench(force: bool = False) -> str:
    """The C++ program bench.py runs to time zen::sample_token through the library."""
    src = os.path.join(CSRC, "bench_host_api.cpp")
    deps = [src, SAMPLER_SO, os.path.join(INCLUDE, "zen", "sample.h")]
    if not force and not _stale(HOST_API_BENCH, deps):
        return HOST_API_BENCH
    tmp = HOST_API_BENCH + ".tmp"
    _run(["g++", "-std=c++17", "-O2", HOST_ARCH, f"-I{INCLUDE}", "-o", tmp, src,
          f"-L{HERE}", "-l:libzs_sampler.so", "-Wl,-rpath,$ORIGIN"])
    os.replace(tmp, HOST_API_BENCH)
    return HOST_API_BENCH


def build_all(force: bool = False) -> None:
    build_workload(force)
    build_sampler(force)
    build_host_api_bench(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
    print(SAMPLER_SO)
    print(WORKLOAD_SO)
