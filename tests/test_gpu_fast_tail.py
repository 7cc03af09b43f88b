"""The certified parallel tail, taken by calls that want only the ids (no row
info, no candidate lists), against the sequential tail of the same kernels (a
call with row info) and against the restatement: ids and Rng states bit for bit.
Shortlists of at least 128 on every path that draws: the CTA merge (64 rows), the
warp merge (320 rows), the one-launch small batch (4 rows) and the large-shortlist
kernel (top-k 3000); with and without a nucleus, tie-heavy rows, a top_p the first
term already reaches, and rows the parallel tail hands back to the sequential
loops (NaN at index 0, top_p = 0)."""

import numpy as np
import pytest

from tests.gpu_util import compare, run_gpu, run_oracle
from zeninfer_b200 import SamplingParams, rng_seed, states_to_tensor, tensor_to_states
from zeninfer_b200 import workloads as W

pytestmark = pytest.mark.gpu

PARAMS = [SamplingParams(temp=1.0, top_p=0.95),                # the 256 shortlist
          SamplingParams(temp=0.8, top_k=1024),
          SamplingParams(temp=1.3, top_k=200, top_p=0.5),
          SamplingParams(temp=0.7, top_k=128),
          SamplingParams(temp=1.0, top_k=300, top_p=0.01)]     # m = 1


def _states(n, base=11):
    return np.asarray([rng_seed(i + base) for i in range(n)], dtype=np.uint64)


def _ids_only(sampler, x, params, states):
    import torch
    xd = torch.from_numpy(np.ascontiguousarray(x)).to(sampler.device)
    st = states_to_tensor(states, sampler.device)
    ids = sampler.sample(xd, params, st, sync_check=True).ids
    return ids.cpu().numpy(), tensor_to_states(st)


def _check(sampler, x, params):
    rows = x.shape[0]
    ids, st = _ids_only(sampler, x, params, _states(rows))
    exact = run_gpu(sampler, x, params, _states(rows))
    assert np.array_equal(ids, exact["ids"])
    assert np.array_equal(st, exact["states"])
    o = run_oracle(x, params, _states(rows))
    compare(exact, o, check_cands=False)
    assert np.array_equal(st, o["states"])


@pytest.mark.parametrize("rows,cfg", [(64, 3), (320, 2), (4, 1)])
@pytest.mark.parametrize("pi", range(len(PARAMS)))
def test_fast_tail_matches_sequential(sampler, rows, cfg, pi):
    p = PARAMS[pi]
    if rows == 4 and p.top_k == 1024:
        pytest.skip("shortlists above 256 do not take the small-batch path")
    x = W.generate(cfg, rows, row0=500 + 7 * pi)
    _check(sampler, x, p)


def test_fast_tail_ties_and_per_row(sampler):
    rows = 72
    x = W.generate(4, rows, row0=9)  # values on a grid: tie groups at the cut
    plist = [PARAMS[i % len(PARAMS)] for i in range(rows)]
    _check(sampler, x, plist)


def test_fast_tail_large_shortlist(sampler):
    x = W.generate(2, 6, row0=77)
    _check(sampler, x, SamplingParams(temp=0.9, top_k=3000, top_p=0.9))


def test_fast_tail_hands_back(sampler):
    """Rows the parallel tail cannot certify take the sequential loops."""
    rows = 40
    x = W.generate(2, rows, row0=123)
    x[0, 0] = np.nan
    plist = [SamplingParams(temp=1.0, top_k=256, top_p=0.0) if r % 2 else
             SamplingParams(temp=1.0, top_k=256, top_p=0.9) for r in range(rows)]
    _check(sampler, x, plist)
