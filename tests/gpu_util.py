"""Helpers shared by the GPU parity tests: run the CUDA sampler and the oracle
on the same rows and compare under the parity rules.

Parity rules (per row):
  * greedy ids, top-k candidate sets and order: bit-exact against the
    restatement (value descending, id ascending);
  * against the unchanged reference: ids bit-exact on rows whose shortlist has
    no tie crossing the k boundary or the drawn position; otherwise the drawn
    logit value is bit-exact (libstdc++ orders equal values its own way);
  * sampled ids may differ only where the draw lies within 1e-6 of a CDF
    boundary (counted);
  * shortlist probabilities within 1e-5 relative.
"""

from __future__ import annotations

import numpy as np

import oracle
from zeninfer_b200 import states_to_tensor, tensor_to_states

PROB_RTOL = 1e-5
BOUNDARY_EPS = 1e-6


def run_gpu(sampler, x, params, states, history=None, history_len=None, cand_ld=0,
            want_log_z=False, ld=None):
    """x: host float32 [B, V] (or [B, ld] with V columns used when ld given)."""
    import torch
    dev = sampler.device
    xd = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    st = states_to_tensor(states, dev)
    h = hl = None
    if history is not None:
        h = torch.from_numpy(np.ascontiguousarray(history, dtype=np.int32)).to(dev)
        hl = torch.from_numpy(np.ascontiguousarray(history_len, dtype=np.int32)).to(dev)
    res = sampler.sample(xd, params, st, h, hl, row_info=True, cand_ld=cand_ld,
                         want_log_z=want_log_z, sync_check=True)
    out = {"ids": res.ids.cpu().numpy(), "states": tensor_to_states(st), "info": res.row_info}
    if cand_ld:
        out["cand_ids"] = res.cand_ids.cpu().numpy()
        out["cand_probs"] = res.cand_probs.cpu().numpy()
    return out


def run_oracle(x, params, states, history=None, history_len=None, cand_ld=0, full_z=False):
    st = np.array(states, dtype=np.uint64, copy=True)
    ids, info, cid, cv, cp = oracle.oracle_sample(x, params, st, history, history_len,
                                                  cand_ld=cand_ld, full_z=full_z)
    return {"ids": ids, "states": st, "info": info, "cand_ids": cid, "cand_vals": cv,
            "cand_probs": cp}


def compare(g, o, check_cands=True):
    """Asserts GPU == restatement; returns the number of boundary rows."""
    ids_eq = g["ids"] == o["ids"]
    near = o["info"]["boundary"] < BOUNDARY_EPS
    bad = ~ids_eq & ~near
    assert not bad.any(), f"id mismatch on rows {np.nonzero(bad)[0][:10]}"
    assert np.array_equal(g["states"], o["states"]), "rng states differ"
    gi, oi = g["info"], o["info"]
    assert np.array_equal(gi["k"], oi["k"]), "shortlist sizes differ"
    far = ~near
    assert np.array_equal(gi["m"][far], oi["m"][far]), \
        f"nucleus sizes differ on rows {np.nonzero((gi['m'] != oi['m']) & far)[0][:10]}"
    assert np.array_equal(gi["r"], oi["r"]), "uniform draws differ"
    if check_cands and o.get("cand_ids") is not None and "cand_ids" in g:
        k = oi["k"]
        for r in range(len(k)):
            kr = min(int(k[r]), g["cand_ids"].shape[1])
            assert np.array_equal(g["cand_ids"][r, :kr], o["cand_ids"][r, :kr]), f"candidates row {r}"
            gp, op = g["cand_probs"][r, :kr], o["cand_probs"][r, :kr]
            np.testing.assert_allclose(gp, op, rtol=PROB_RTOL, atol=0)
    return int((~ids_eq & near).sum())


def compare_reference(x, g_ids, params, seeds, tie_ok=True, history=None, history_len=None):
    """Against the unchanged reference: ids equal, or (with ties) equal logit values."""
    ref_ids, _ = oracle.reference_sample(x, params, seeds, history, history_len)
    eq = ref_ids == g_ids
    if eq.all():
        return 0
    rows = np.nonzero(~eq)[0]
    if tie_ok:
        vals_ok = x[rows, ref_ids[rows]] == x[rows, g_ids[rows]]
        assert vals_ok.all(), f"reference mismatch beyond tie groups on rows {rows[~vals_ok][:10]}"
    else:
        raise AssertionError(f"reference id mismatch on rows {rows[:10]}")
    return len(rows)
