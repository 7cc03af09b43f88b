"""Speculative opening thresholds (zs_set_speculation): long row slices of long
shortlists start their filter from a threshold sampled from the slice; the merge
certifies each row against the thresholds its slices used and redoes the others
exactly.  Every mode must give the same ids, Rng states, shortlists and
probabilities: checked on the workloads that speculate (slices of at least 32,768
columns, shortlists of at least 128), on rows whose order defeats a sample
(sorted, front-loaded), and with every speculated row redone."""

import numpy as np
import pytest

from tests.gpu_util import compare, run_gpu, run_oracle
from zeninfer_b200 import SamplingParams, rng_seed
from zeninfer_b200 import workloads as W

pytestmark = pytest.mark.gpu

V = W.VOCAB


def _states(n):
    return np.asarray([rng_seed(i + 3) for i in range(n)], dtype=np.uint64)


def _modes(sampler, x, p, cand_ld):
    out = {}
    try:
        for mode in ("on", "off", "redo_all"):
            sampler.set_speculation(mode)
            out[mode] = run_gpu(sampler, x, p, _states(x.shape[0]), cand_ld=cand_ld)
    finally:
        sampler.set_speculation("on")
    return out


def _same(a, b):
    assert np.array_equal(a["ids"], b["ids"])
    assert np.array_equal(a["states"], b["states"])
    assert np.array_equal(a["cand_ids"], b["cand_ids"])
    assert np.array_equal(a["cand_probs"].view(np.uint64), b["cand_probs"].view(np.uint64))


@pytest.mark.parametrize("cfg,rows,params", [
    (3, 1024, SamplingParams(temp=1.0, top_p=0.95)),             # the 256 shortlist
    (4, 512, SamplingParams(temp=0.8, top_k=1024)),              # long config, ties
    (5, 512, SamplingParams(temp=0.9, top_k=200, top_p=0.95)),   # 43,800-column slices
    (2, 400, SamplingParams(temp=1.0, top_k=128)),               # the smallest speculated k
])
def test_speculation_modes_agree(sampler, cfg, rows, params):
    x = W.generate(cfg, rows, row0=31)
    k = params.top_k if params.top_k > 0 else 256
    got = _modes(sampler, x, params, k)
    _same(got["on"], got["off"])
    _same(got["on"], got["redo_all"])
    compare(got["on"], run_oracle(x, params, _states(rows), cand_ld=k))


@pytest.mark.parametrize("order", ["descending", "ascending", "front_loaded", "clustered"])
def test_speculation_adversarial_rows(sampler, order):
    """Orders a strided sample misreads: sorted rows, the best values moved to the
    front, and the best values clustered between the sample's chunks."""
    rows = 512
    rng = np.random.default_rng(11)
    x = rng.normal(0, 1, size=(rows, V)).astype(np.float32)
    if order == "descending":
        x = -np.sort(-x, axis=1)
    elif order == "ascending":
        x = np.sort(x, axis=1)
    elif order == "front_loaded":
        idx = np.argsort(-x, axis=1)[:, :4096]
        for r in range(rows):
            top = x[r, idx[r]].copy()
            x[r, idx[r]] = x[r, :4096]
            x[r, :4096] = top
    else:  # 400 large values in one run per 20,000 columns
        for r in range(rows):
            for c0 in range(1000 + 37 * r % 500, V - 400, 20000):
                x[r, c0:c0 + 400] = rng.normal(6, 0.5, size=400)
    x = np.ascontiguousarray(x)
    for p in (SamplingParams(temp=1.0, top_p=0.95), SamplingParams(temp=0.8, top_k=1024)):
        k = p.top_k if p.top_k > 0 else 256
        got = _modes(sampler, x, p, k)
        _same(got["on"], got["off"])
        _same(got["on"], got["redo_all"])
        compare(got["on"], run_oracle(x, p, _states(rows), cand_ld=k))


def test_speculation_mode_rejects_unknown(sampler):
    with pytest.raises(ValueError):
        sampler.set_speculation("maybe")
