"""Generates tests/golden/sampler_golden.npz from the reference itself.

The reference has no known-answer tests for its sampler, so the golden vectors
are outputs of its own src/sample.cpp, compiled unchanged into
oracle/_ref/libzen_ref.so (oracle/Makefile, target `ref`), on seeded inputs:

  rng     zen::Rng(seed).next() x 8 and the first uniform(), for a few seeds
  cases   small rows (n <= 2048) covering the branches of sample_token
          (src/sample.cpp:32-102): greedy, top-k, default shortlist, nucleus,
          k > n, top_p <= 0, extreme temperatures, the repetition penalty
          (compounding duplicates, out-of-range ids, window edges), ties,
          +-inf, NaN (greedy only: with a NaN in the row the reference's
          nth_element/sort comparator is not a strict weak order, so its
          sampled pick is libstdc++'s business, not the algorithm's)
  rows    full-vocabulary rows of the five synthetic workloads (regenerated
          from zw_generate by (workload, row); only their ids are stored)

For every case the fixture stores the reference's id, its Rng's next() after
the call, and a `tie` flag: the drawn value occurs more than once in the row,
so another shortlist order may return another id with the same value.

    python tests/golden/make_golden.py        (needs the reference sources)
"""

from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from zeninfer_b200 import SamplingParams as P  # noqa: E402
from zeninfer_b200 import workloads as W  # noqa: E402

OUT = os.path.join(HERE, "sampler_golden.npz")
NMAX = 2048
HMAX = 96

RNG_SEEDS = np.array([0, 1, 42, 0x9E3779B97F4A7C15, (1 << 63) + 5, (1 << 64) - 1], dtype=np.uint64)

SAMPLING = [
    P(),                                           # greedy
    P(temp=0.7, top_k=40, top_p=0.9),
    P(temp=1.0, top_p=0.95),                       # default shortlist of 256
    P(temp=0.8, top_k=1024),
    P(temp=1.2, top_k=1),
    P(temp=0.9, top_k=5000),                       # k > n
    P(temp=1.0, top_k=50, top_p=0.0),              # top_p <= 0: m = 1
    P(temp=1e-3, top_k=64, top_p=0.99),
    P(temp=25.0, top_k=300, top_p=0.5),
    P(temp=0.6, top_k=0, top_p=1.0),
]

PENALTY = [
    P(temp=0.0, repeat_penalty=1.3, repeat_last_n=64),
    P(temp=0.7, top_k=40, top_p=0.9, repeat_penalty=1.3, repeat_last_n=64),
    P(temp=0.8, top_k=20, repeat_penalty=0.5, repeat_last_n=8),
    P(temp=1.0, top_p=0.9, repeat_penalty=2.0, repeat_last_n=0),     # empty window
    P(temp=1.0, top_k=10, repeat_penalty=1.7, repeat_last_n=-3),     # negative window
    P(temp=0.9, top_k=30, repeat_penalty=1.1, repeat_last_n=200),    # window > history
]


def _row(rng, n, kind):
    if kind == "normal":
        return rng.normal(0.0, 2.0, n).astype(np.float32)
    if kind == "peaked":
        x = rng.normal(0.0, 1.0, n).astype(np.float32)
        x[rng.choice(n, size=min(n, 8), replace=False)] += np.float32(7.0)
        return x
    if kind == "ties":
        return (np.round(rng.normal(0.0, 1.5, n) * 2.0) / 2.0).astype(np.float32)
    if kind == "equal":
        return np.full(n, 0.25, dtype=np.float32)
    raise ValueError(kind)


def _cases():
    rng = np.random.default_rng(20260101)
    cases = []  # (x, params, history list, seed)
    for n in (1, 2, 3, 17, 64, 256, 300, 1000, 2048):
        for kind in ("normal", "peaked"):
            for p in SAMPLING:
                cases.append((_row(rng, n, kind), p, [], int(rng.integers(1, 1 << 62))))
    for n in (40, 512, 2048):
        for kind in ("ties", "equal"):
            for p in SAMPLING[:4] + SAMPLING[6:7]:
                cases.append((_row(rng, n, kind), p, [], int(rng.integers(1, 1 << 62))))
    for n in (16, 300, 2048):
        for p in PENALTY:
            for trial in range(3):
                x = _row(rng, n, "peaked")
                x[: n // 2] = -np.abs(x[: n // 2])  # both signs among penalised ids
                hl = int(rng.integers(1, HMAX + 1))
                h = rng.integers(0, n, size=hl).astype(np.int32)
                if hl > 4:
                    h[rng.integers(0, hl, size=hl // 3)] = h[0]          # duplicates compound
                    h[1] = -1                                           # out of range: skipped
                    h[2] = n
                    h[3] = np.int32(2**31 - 1)
                cases.append((x, p, h.tolist(), int(rng.integers(1, 1 << 62))))
    # special values
    for p in (SAMPLING[0], SAMPLING[1], SAMPLING[2], SAMPLING[6]):
        for n in (8, 700):
            x = _row(rng, n, "normal")
            x[n // 3] = np.inf
            cases.append((x, p, [], 7))
            x = _row(rng, n, "normal")
            x[::3] = -np.inf
            cases.append((x, p, [], 8))
    for n in (5, 900):
        x = _row(rng, n, "normal")
        x[0] = np.nan
        cases.append((x, SAMPLING[0], [], 9))            # NaN at index 0: greedy returns 0
        x = _row(rng, n, "normal")
        x[n // 2] = np.nan
        cases.append((x, SAMPLING[0], [], 10))           # NaN elsewhere: never the max
    return cases


def _tie(x, n, rid):
    v = x[rid]
    return bool(np.count_nonzero(x[:n] == v) > 1)


def main():
    oracle.build(with_reference=True)
    cases = _cases()
    C = len(cases)
    logits = np.zeros((C, NMAX), dtype=np.float32)
    ns = np.zeros(C, dtype=np.int32)
    params = np.zeros(C, dtype=oracle.PARAMS_DTYPE)
    hist = np.zeros((C, HMAX), dtype=np.int32)
    hist_len = np.zeros(C, dtype=np.int32)
    seeds = np.zeros(C, dtype=np.uint64)
    for i, (x, p, h, s) in enumerate(cases):
        logits[i, : x.size] = x
        ns[i] = x.size
        params[i] = (p.temp, p.top_k, p.top_p, p.repeat_penalty, p.repeat_last_n)
        hist[i, : len(h)] = h
        hist_len[i] = len(h)
        seeds[i] = s
    ids = np.zeros(C, dtype=np.int32)
    nxt = np.zeros(C, dtype=np.uint64)
    tie = np.zeros(C, dtype=bool)
    for i in range(C):  # one call per case: n differs
        pi = [P(*[float(params[i][f]) if f in ("temp", "top_p", "repeat_penalty")
                  else int(params[i][f]) for f in oracle.PARAMS_DTYPE.names])]
        hi = hist[i: i + 1] if hist_len[i] else None
        hli = hist_len[i: i + 1] if hist_len[i] else None
        r_ids, r_next = oracle.reference_sample(logits[i: i + 1], pi, seeds[i: i + 1], hi, hli,
                                                nthreads=1, ld=NMAX, n=int(ns[i]))
        ids[i], nxt[i] = r_ids[0], r_next[0]
        tie[i] = _tie(logits[i], int(ns[i]), int(ids[i]))
    rng_next = np.zeros((len(RNG_SEEDS), 8), dtype=np.uint64)
    rng_uniform = np.zeros(len(RNG_SEEDS), dtype=np.float64)
    for j, s in enumerate(RNG_SEEDS):
        rng_next[j], rng_uniform[j] = oracle.reference_rng_stream(int(s), 8)
    # full-vocabulary workload rows
    wl_cfg, wl_row, wl_ids, wl_tie = [], [], [], []
    for cfg in (1, 2, 3, 4, 5):
        wl = W.WORKLOADS[cfg]
        rows = 1 if cfg == 1 else 4
        x = W.generate(cfg, rows)
        seeds_w = np.array(wl.row_seeds(0, rows), dtype=np.uint64)
        for p in [wl.params] + ([P()] if wl.greedy_too else []):
            r_ids, _ = oracle.reference_sample(x, p, seeds_w)
            for r in range(rows):
                wl_cfg.append(cfg if p is wl.params else -cfg)  # negative: greedy variant
                wl_row.append(r)
                wl_ids.append(int(r_ids[r]))
                wl_tie.append(_tie(x[r], x.shape[1], int(r_ids[r])))
    np.savez_compressed(
        OUT, logits=logits, n=ns, params=params, hist=hist, hist_len=hist_len, seeds=seeds,
        ids=ids, next_after=nxt, tie=tie, rng_seeds=RNG_SEEDS, rng_next=rng_next,
        rng_uniform=rng_uniform, wl_cfg=np.array(wl_cfg, dtype=np.int32),
        wl_row=np.array(wl_row, dtype=np.int32), wl_ids=np.array(wl_ids, dtype=np.int32),
        wl_tie=np.array(wl_tie, dtype=bool))
    print(f"{OUT}: {C} cases ({int(tie.sum())} with ties), {len(wl_ids)} workload rows, "
          f"{os.path.getsize(OUT)} bytes")


if __name__ == "__main__":
    main()
