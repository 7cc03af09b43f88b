"""The lm_head epilogue's threshold rules, restated on the CPU (no device code runs).

zs_lmhead_kernel (zeninfer_b200/csrc/zs_lmhead.cuh) keeps, per row and vocabulary
slice, the keys above a threshold, and a row's slices share a lower bound: a slice
whose buffer held more than keff keys publishes the value order g of its keff-th best
key, and the others take it as "value >= value(g)" through lm_adopt's order c = g - 1
under the strict test v > value_of_ord(c).  These tests check that encoding for every
kind of float32 (signed zeros, denormals, infinities, NaN), and that slices run with
the shared bound, in any interleaving and with heavy value ties across slices, keep
every key of the row's keff best, so the merge of their blocks is the row's top keff.
The restatements follow zs_device.cuh (ord_of, value_of_ord) and zs_lmhead.cuh
(lm_adopt, lm_pass_mask, lm_compact_row) line by line."""

import numpy as np
import pytest

F32_MIN_NORMAL_NEG_MAX = 0x00800000  # ord_of(-FLT_MAX)


def ord_of(v):
    """zs_device.cuh ord_of: NaN -> 0, -0 -> +0, then the monotone bit map."""
    v = np.asarray(v, dtype=np.float32).copy()
    nan = np.isnan(v)
    v[v == 0] = np.float32(0.0)
    u = v.view(np.uint32)
    o = np.where(u & np.uint32(0x80000000), ~u, u | np.uint32(0x80000000)).astype(np.uint32)
    o[nan] = 0
    return o


def value_of_ord(o):
    o = np.asarray(o, dtype=np.uint32)
    u = np.where(o & np.uint32(0x80000000), o & np.uint32(0x7FFFFFFF), ~o).astype(np.uint32)
    v = u.view(np.float32).copy()
    v[o == 0] = np.float32(np.nan)
    return v


def adopt(g):
    """lm_adopt: the order c taken for a published g, or None (not taken)."""
    if g <= F32_MIN_NORMAL_NEG_MAX:
        return None
    c = g - 1
    if c == 0x7FFFFFFF:
        c = 0x7FFFFFFE
    return c


def passes(v, c):
    """lm_pass_mask for a closed buffer: v > value(c), or any non-NaN for order 0."""
    v = np.asarray(v, dtype=np.float32)
    if c == 0:
        return ~np.isnan(v)
    with np.errstate(invalid="ignore"):
        return v > value_of_ord(np.array([c], dtype=np.uint32))[0]


def _special_values():
    f = np.float32
    tiny = np.finfo(np.float32).tiny
    denorm = np.float32(1e-45)
    vals = [0.0, -0.0, denorm, -denorm, 2 * denorm, -2 * denorm, tiny, -tiny, 1.0, -1.0,
            np.finfo(np.float32).max, -np.finfo(np.float32).max, np.inf, -np.inf, np.nan,
            0.5, -0.5, 3.0, 1e30, -1e30]
    v = np.array(vals, dtype=np.float32)
    # every neighbour of each value, and a random sample of all bit patterns
    u = v.view(np.uint32).astype(np.int64)
    nb = np.concatenate([u - 1, u + 1]) % (1 << 32)
    rnd = np.random.default_rng(5).integers(0, 1 << 32, size=20000, dtype=np.int64)
    allu = np.concatenate([u, nb, rnd]).astype(np.uint32)
    return np.unique(allu).view(np.float32)


def test_order_round_trip():
    v = _special_values()
    o = ord_of(v)
    back = value_of_ord(o)
    ok = ~np.isnan(v)
    assert np.array_equal(ord_of(back[ok]), o[ok])
    # monotone: the order sorts like the value (NaN lowest, -0 == +0)
    a, b = v[ok], o[ok]
    idx = np.argsort(a, kind="stable")
    assert np.all(np.diff(b[idx].astype(np.int64)) >= 0)


def test_adopted_bound_is_value_at_least_g():
    """For every published g (an order of a non-NaN value) that lm_adopt takes, the
    strict test with c passes exactly the non-NaN values whose order is >= g."""
    v = _special_values()
    ov = ord_of(v)
    gs = np.unique(ord_of(v[~np.isnan(v)]))
    taken = 0
    for g in gs.tolist():
        c = adopt(g)
        if c is None:
            assert g <= F32_MIN_NORMAL_NEG_MAX
            continue
        taken += 1
        want = (~np.isnan(v)) & (ov >= g)
        assert np.array_equal(passes(v, c), want), (hex(g), hex(c))
    assert taken > 100
    # the two special cases: g at +-0 passes both zeros, g just above -FLT_MAX passes it not
    c0 = adopt(int(ord_of(np.array([0.0], dtype=np.float32))[0]))
    assert passes(np.array([0.0, -0.0, -1e-45], dtype=np.float32), c0).tolist() == [True, True, False]


def _keys(vals, ids):
    """(order << 32) | ~id, the sampler's key: value descending, id ascending."""
    return (ord_of(vals).astype(np.uint64) << np.uint64(32)) | (
        ~ids.astype(np.uint32)).astype(np.uint64)


def _slack(keff):
    """lm_slack: keys an intermediate compaction may keep beyond keff."""
    return min(keff // 4, max(0, 88 - keff))


def _run_slices(vals, S, keff, cap, order_rng, reverse=False, slack=False):
    """Slices of one row processed in an interleaving drawn from order_rng (or, with
    `reverse`, each slice whole from the last to the first), chunk by chunk (32
    columns), with the buffer, compaction and shared bound of the epilogue; returns
    the union of the slices' final blocks (keys).  With `slack` an intermediate
    compaction keeps, like the radix walk that stops early, every key at or above
    some key T whose rank lies anywhere in [keff, keff + lm_slack(keff)] (drawn from
    order_rng) and takes T as its threshold; the final block is exact."""
    n = len(vals)
    bounds = [(s * n) // S for s in range(S + 1)]
    state = []
    for s in range(S):
        state.append({"col": bounds[s], "end": bounds[s + 1], "buf": [], "open": True,
                      "tau": 0})
    shared = 0
    live = list(range(S))
    while live:
        s = live[-1] if reverse else int(order_rng.choice(live))
        st = state[s]
        c0 = st["col"]
        c1 = min(c0 + 32, st["end"])
        chunk = np.arange(c0, c1)
        v = vals[chunk]
        if st["open"]:
            pm = np.ones(len(chunk), dtype=bool)
        else:
            pm = passes(v, st["tau"])
        if len(st["buf"]) + int(pm.sum()) > cap:
            # lm_compact_row: keep the keff best (or the slack bucket), publish, take
            # the higher threshold
            r = int(order_rng.integers(0, _slack(keff) + 1)) if slack else 0
            buf = sorted(st["buf"], reverse=True)
            buf = buf[:min(len(buf), keff + r)]
            t = int(buf[-1] >> np.uint64(32))
            shared = max(shared, t)
            if not (not st["open"] and st["tau"] > t):
                st["tau"] = t
            st["open"] = False
            st["buf"] = buf
            pm = passes(v, st["tau"])
        st["buf"].extend(_keys(v[pm], chunk[pm]).tolist())
        st["col"] = c1
        # once per "tile" (here: every chunk) the slice takes the shared bound
        c = adopt(shared) if shared else None
        if c is not None and (st["open"] or c > st["tau"]):
            st["tau"], st["open"] = c, False
        if c1 >= st["end"]:
            live.remove(s)
    out = []
    for st in state:
        buf = sorted(st["buf"], reverse=True)
        out.extend(buf[:keff] if len(buf) > keff else buf)
    return np.array(out, dtype=np.uint64)


@pytest.mark.parametrize("slack", [False, True])
@pytest.mark.parametrize("case", range(12))
def test_shared_bound_keeps_the_top_keff(case, slack):
    """Rows with heavy ties (values from a few levels, so equal values sit in every
    slice), signed zeros, -inf and NaN; random interleavings of the slices."""
    rng = np.random.default_rng(100 + case)
    n = int(rng.integers(600, 5000))
    levels = np.array([0.0, -0.0, 1.0, 2.0, 2.5, -1.0, -np.inf, np.nan, 3.0, 1e-45],
                      dtype=np.float32)
    if case % 3 == 0:
        vals = levels[rng.integers(0, len(levels), size=n)]
    elif case % 3 == 1:
        vals = np.round(rng.normal(0, 2, size=n) * 2).astype(np.float32) / np.float32(2)
    else:
        vals = np.where(rng.random(n) < 0.5, np.float32(0.0), np.float32(-0.0))
        vals[rng.integers(0, n, size=5)] = np.nan
    keff = int(rng.integers(1, 89))
    S = int(rng.integers(2, 10))
    got = _run_slices(vals, S, keff, 120, rng, slack=slack)
    allk = np.sort(_keys(vals, np.arange(n)))[::-1]
    want = allk[:keff]
    top = np.sort(got)[::-1][:keff]
    assert np.array_equal(top, want)


@pytest.mark.parametrize("slack", [False, True])
@pytest.mark.parametrize("keff", [1, 7, 50, 88])
@pytest.mark.parametrize("top", [2.5, 0.0, -0.0, -np.inf])
def test_shared_bound_ties_across_slices(keff, top, slack):
    """More than keff copies of the row's best value in every slice, the slices run
    from the last to the first: each publishes the tied value, and the earlier slices,
    whose copies have the smaller ids and so are the row's keff best, must still keep
    values equal to the bound.  (A strict bound, value > value(g), loses them.)"""
    rng = np.random.default_rng(keff)
    S, per = 6, 640
    n = S * per
    below = np.float32(-1e30) if top != -np.inf else np.float32(np.nan)
    vals = np.full(n, below, dtype=np.float32)
    for s in range(S):
        idx = s * per + rng.choice(per, size=keff + 40, replace=False)
        vals[idx] = np.float32(top)
    got = _run_slices(vals, S, keff, 120, rng, reverse=True, slack=slack)
    want = np.sort(_keys(vals, np.arange(n)))[::-1][:keff]
    assert np.array_equal(np.sort(got)[::-1][:keff], want)
