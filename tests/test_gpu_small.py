"""The one-launch small-batch path (zs_small_kernel: a cluster of 16 CTAs per row,
merged through distributed shared memory) against the select + merge launches on
the same rows, and against the restatement: ids, Rng states, shortlists and
probabilities bit for bit, for batches of 1 to 8 rows, greedy and sampled rows,
per-row parameters, ties, a NaN at index 0, row lengths that leave a ragged tail,
repeat penalties (repeated ids, ids at slice edges and in the tail, out-of-range
ids, windows up to the kernel's 256), and the shapes the path declines (longer
windows, unaligned rows, log Z)."""

import numpy as np
import pytest

from tests.gpu_util import compare, run_gpu, run_oracle
from zeninfer_b200 import SamplingParams, rng_seed
from zeninfer_b200 import workloads as W

pytestmark = pytest.mark.gpu

V = W.VOCAB


def _states(n, base=5):
    return np.asarray([rng_seed(i + base) for i in range(n)], dtype=np.uint64)


def _both(sampler, x, params, cand_ld, **kw):
    out = {}
    try:
        for name, rows in (("small", 8), ("launches", 0)):
            sampler.set_small_batch(rows)
            out[name] = run_gpu(sampler, x, params, _states(x.shape[0]), cand_ld=cand_ld, **kw)
    finally:
        sampler.set_small_batch(8)
    return out


def _same(a, b):
    assert np.array_equal(a["ids"], b["ids"])
    assert np.array_equal(a["states"], b["states"])
    if "cand_ids" in a:
        assert np.array_equal(a["cand_ids"], b["cand_ids"])
        assert np.array_equal(a["cand_probs"].view(np.uint64), b["cand_probs"].view(np.uint64))
    for f in ("k", "m", "pos", "r", "sum", "boundary"):
        assert np.array_equal(a["info"][f], b["info"][f], equal_nan=True), f


@pytest.mark.parametrize("rows", [1, 2, 5, 8])
@pytest.mark.parametrize("params", [SamplingParams(temp=0.7, top_k=40),
                                    SamplingParams(),
                                    SamplingParams(temp=1.0, top_p=0.95),
                                    SamplingParams(temp=0.9, top_k=1),
                                    SamplingParams(temp=1.3, top_k=200, top_p=0.5)])
def test_small_batch_matches_launches(sampler, rows, params):
    x = W.generate(1 if rows == 1 else 2, rows, row0=70)
    k = params.top_k if params.top_k > 0 else 256
    cl = k if params.temp > 0 else 0
    got = _both(sampler, x, params, cl)
    _same(got["small"], got["launches"])
    compare(got["small"], run_oracle(x, params, _states(rows), cand_ld=cl))


def test_small_batch_per_row_params_and_ties(sampler):
    rows = 6
    x = W.generate(4, rows, row0=3)  # values on a 1/8 grid: ties everywhere
    plist = [SamplingParams(), SamplingParams(temp=0.8, top_k=256),
             SamplingParams(temp=0.5, top_k=3), SamplingParams(temp=1.0, top_p=0.9),
             SamplingParams(temp=2.0, top_k=64, top_p=0.99), SamplingParams(temp=1e-3)]
    got = _both(sampler, x, plist, 256)
    _same(got["small"], got["launches"])
    compare(got["small"], run_oracle(x, plist, _states(rows), cand_ld=256))


@pytest.mark.parametrize("n", [16384, 20001, 151933])
def test_small_batch_ragged_rows(sampler, n):
    """Row lengths that leave a scalar tail in the last CTA's slice."""
    import torch
    rows = 3
    rng = np.random.default_rng(n)
    xf = rng.normal(0, 2, size=(rows, n)).astype(np.float32)
    for p in (SamplingParams(temp=0.7, top_k=40, top_p=0.9), SamplingParams()):
        k = 40 if p.temp > 0 else 0
        got = _both(sampler, xf, p, k)
        _same(got["small"], got["launches"])
        compare(got["small"], run_oracle(xf, p, _states(rows), cand_ld=k))


def test_small_batch_special_values(sampler):
    rows, n = 4, 30000
    rng = np.random.default_rng(9)
    x = rng.normal(0, 1, size=(rows, n)).astype(np.float32)
    x[0, 0] = np.nan          # greedy returns 0
    x[1, 12345] = np.inf
    x[2, :] = 0.25            # all equal: the lowest ids win
    x[3, ::3] = -np.inf
    got = _both(sampler, x, SamplingParams(), 0)
    _same(got["small"], got["launches"])
    assert got["small"]["ids"][0] == 0
    assert got["small"]["ids"][2] == 0
    p = SamplingParams(temp=0.8, top_k=40)
    got = _both(sampler, x[1:], p, 40)
    _same(got["small"], got["launches"])
    compare(got["small"], run_oracle(x[1:], p, _states(rows - 1), cand_ld=40))


def _penalty_history(x, rows, hist_ld, seed):
    """Windows that hit the rows' top ids (so the penalty changes the shortlist),
    repeat ids (the penalty compounds), and reach the edges of the 16 slices, the
    scalar tail, id 0 and ids outside the vocabulary."""
    rng = np.random.default_rng(seed)
    n = x.shape[1]
    per = ((n + 15) // 16 + 3) & ~3
    hist = rng.integers(0, n, size=(rows, hist_ld)).astype(np.int32)
    for r in range(rows):
        top = np.argsort(-x[r], kind="stable")[:24]
        k = min(hist_ld, 48)
        hist[r, -k:] = rng.choice(np.concatenate([top, top[:6]]), size=k)
        edges = [0, n - 1, per - 1, per, 5 * per - 1, 5 * per, -3, n + 7]
        hist[r, -len(edges) - 1:-1] = np.asarray(edges, dtype=np.int64).astype(np.int32)
    return hist


@pytest.mark.parametrize("rows,win,n", [(1, 64, V), (4, 64, V), (8, 256, V), (3, 64, 20001)])
def test_small_batch_penalty(sampler, rows, win, n):
    """Penalised rows run in the small-batch kernel: the same ids, states,
    shortlists and probabilities as the launches and the restatement."""
    xf = W.generate(2, rows, row0=41)[:, :n].copy()
    xf[0, 0] = -np.inf if rows > 1 else xf[0, 0]  # id 0 penalised from -inf
    hist = _penalty_history(xf, rows, win + 8, 7 + rows)
    hl = np.full(rows, win + 8, dtype=np.int32)
    if rows > 1:
        hl[-1] = win // 2  # a history shorter than repeat_last_n
    for p in (SamplingParams(temp=0.7, top_k=40, top_p=0.9, repeat_penalty=1.3,
                             repeat_last_n=win),
              SamplingParams(temp=0.0, repeat_penalty=2.0, repeat_last_n=win),
              SamplingParams(temp=1.0, top_p=0.95, repeat_penalty=0.8, repeat_last_n=win)):
        k = p.top_k if p.top_k > 0 else 256
        cl = k if p.temp > 0 else 0
        got = _both(sampler, xf, p, cl, history=hist, history_len=hl)
        _same(got["small"], got["launches"])
        compare(got["small"], run_oracle(xf, p, _states(rows), history=hist, history_len=hl,
                                         cand_ld=cl))


def test_small_batch_penalty_nan_at_zero(sampler):
    """logits[0] NaN stays NaN under the penalty: greedy returns 0 either way."""
    rows = 2
    x = W.generate(1, rows, row0=5)
    x[:, 0] = np.nan
    hist = np.zeros((rows, 16), dtype=np.int32)  # id 0, sixteen times
    hl = np.full(rows, 16, dtype=np.int32)
    p = SamplingParams(temp=0.0, repeat_penalty=1.5, repeat_last_n=16)
    got = _both(sampler, x, p, 0, history=hist, history_len=hl)
    _same(got["small"], got["launches"])
    assert (got["small"]["ids"] == 0).all()


def test_small_batch_declined_shapes(sampler):
    """Windows longer than 256, log Z and unaligned rows take the launches; same
    results."""
    x = W.generate(2, 4, row0=11)
    rng = np.random.default_rng(1)
    hist = rng.integers(0, V, size=(4, 300)).astype(np.int32)
    hl = np.full(4, 300, dtype=np.int32)
    p = SamplingParams(temp=0.7, top_k=40, top_p=0.9, repeat_penalty=1.2, repeat_last_n=257)
    got = _both(sampler, x, p, 40, history=hist, history_len=hl)
    _same(got["small"], got["launches"])
    compare(got["small"], run_oracle(x, p, _states(4), history=hist, history_len=hl, cand_ld=40))
    got = _both(sampler, x, SamplingParams(temp=0.7, top_k=40), 40, want_log_z=True)
    _same(got["small"], got["launches"])
    import torch
    from zeninfer_b200 import states_to_tensor, tensor_to_states
    xo = np.zeros((4, V + 1), dtype=np.float32)  # ld = V + 1: rows not 16-byte aligned
    xo[:, :V] = x
    xd = torch.from_numpy(xo).to(sampler.device)[:, :V]
    res = {}
    try:
        for name, rows in (("small", 8), ("launches", 0)):
            sampler.set_small_batch(rows)
            st = states_to_tensor(_states(4), sampler.device)
            ids = sampler.sample(xd, SamplingParams(temp=0.7, top_k=40), st, sync_check=True).ids
            res[name] = (ids.cpu().numpy(), tensor_to_states(st))
    finally:
        sampler.set_small_batch(8)
    assert np.array_equal(res["small"][0], res["launches"][0])
    assert np.array_equal(res["small"][1], res["launches"][1])
