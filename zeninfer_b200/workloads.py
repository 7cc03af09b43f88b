"""The five sampler workloads: synthetic Qwen2.5-0.5B lm_head logits rows
([rows][151936] f32) with their sampling parameters and per-row seeds.

There is no model or dataset here, so seeded laws stand in for real logits
(zeninfer_b200/csrc/workload.c documents them).  Rows are generated on the host
by libzs_workload.so; every consumer reads byte-identical data.

    1  batch 1      N(0, 2^2) + 16 peaks        temp 0.7, top-k 40, seed 42; and greedy
    2  batch 256    N(0, 2.5^2)+off + 8 peaks   temp 0.7, top-k 40, top-p 0.9, seeds 0..255
    3  batch 1024   -1.1 log(rank+1) + N(0,.3^2) temp 1.0, top-p 0.95, no top-k
    4  batch 512    round(8 N(0, 1.5^2)) / 8    top-k 1024, temp 0.8; and greedy
    5  batch 4096   as 2                        temp 0.7, top-k 50, top-p 0.9

The temp 0.7 / top-k 40 of workload 1 is the README's CLI example; the
generate defaults (src/main.cpp:570-576) are greedy.
"""

from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, field
from typing import List

import numpy as np

from .sampler import SamplingParams, rng_seed

HERE = os.path.dirname(os.path.abspath(__file__))
WORKLOAD_SO = os.path.join(HERE, "libzs_workload.so")
VOCAB = 151936  # Qwen2.5-0.5B

_lib = None


def _wl():
    global _lib
    if _lib is None:
        if not os.path.exists(WORKLOAD_SO):
            raise RuntimeError(f"{WORKLOAD_SO} is not built; run python -m zeninfer_b200.build")
        L = C.CDLL(WORKLOAD_SO)
        L.zw_generate.argtypes = [C.c_int, C.c_uint64, C.c_int64, C.c_int, C.c_int, C.c_void_p,
                                  C.c_int64, C.c_int]
        L.zw_generate.restype = C.c_int
        _lib = L
    return _lib


@dataclass
class Workload:
    cfg: int
    batch: int
    params: SamplingParams
    greedy_too: bool = False
    seeds: List[int] = field(default_factory=list)  # rng seed per row

    def row_seeds(self, row0: int = 0, rows: int | None = None) -> np.ndarray:
        rows = self.batch - row0 if rows is None else rows
        return np.asarray([self.seed_of(row0 + r) for r in range(rows)], dtype=np.uint64)

    def seed_of(self, row: int) -> int:
        return 42 if self.cfg == 1 else row

    def row_states(self, row0: int = 0, rows: int | None = None) -> np.ndarray:
        return np.asarray([rng_seed(int(s)) for s in self.row_seeds(row0, rows)], dtype=np.uint64)


WORKLOADS = {
    1: Workload(1, 1, SamplingParams(temp=0.7, top_k=40), greedy_too=True),
    2: Workload(2, 256, SamplingParams(temp=0.7, top_k=40, top_p=0.9)),
    3: Workload(3, 1024, SamplingParams(temp=1.0, top_p=0.95)),
    4: Workload(4, 512, SamplingParams(temp=0.8, top_k=1024), greedy_too=True),
    5: Workload(5, 4096, SamplingParams(temp=0.7, top_k=50, top_p=0.9)),
}

DATA_SEED = 0


def generate(cfg: int, rows: int, row0: int = 0, V: int = VOCAB, out: np.ndarray | None = None,
             nthreads: int | None = None, seed: int = DATA_SEED) -> np.ndarray:
    """Rows row0 .. row0+rows-1 of workload `cfg` as float32 [rows, V] (or into `out`,
    any C-contiguous float32 array whose last dimension is >= V)."""
    if out is None:
        out = np.empty((rows, V), dtype=np.float32)
    assert out.dtype == np.float32 and out.flags["C_CONTIGUOUS"]
    ld = out.shape[-1] if out.ndim > 1 else V
    if nthreads is None:
        nthreads = min(64, os.cpu_count() or 1)
    rc = _wl().zw_generate(cfg, seed, row0, rows, V, out.ctypes.data, ld, nthreads)
    if rc != 0:
        raise ValueError("zw_generate rejected its arguments")
    return out
