"""The oracle (C restatement of src/sample.cpp) pinned against the reference.

Two pins, both on CPU:
  * tests/golden/sampler_golden.npz -- outputs of the reference's own
    sample.cpp on seeded cases (tests/golden/make_golden.py); needs nothing at
    run time but the restatement;
  * the reference compiled unchanged (oracle/_ref/libzen_ref.so) on fresh
    seeded rows, where it is built.

Rule: ids equal; where the drawn value occurs more than once in the row the
reference's shortlist order among equal values (libstdc++ introselect) may pick
another id, and then the drawn VALUES are equal.  The restatement uses the
reference's own f64 expressions and summation order, so no boundary tolerance.
"""

import ctypes as C
import os

import numpy as np
import pytest

import oracle
from zeninfer_b200 import Rng, SamplingParams, rng_seed
from zeninfer_b200 import workloads as W

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "sampler_golden.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def _params_of(rec):
    return SamplingParams(float(rec["temp"]), int(rec["top_k"]), float(rec["top_p"]),
                          float(rec["repeat_penalty"]), int(rec["repeat_last_n"]))


def test_rng_golden(golden):
    for seed, outs, u in zip(golden["rng_seeds"], golden["rng_next"], golden["rng_uniform"]):
        r = Rng(int(seed))
        assert [r.next() for _ in range(8)] == [int(v) for v in outs]
        assert Rng(int(seed)).uniform() == u
        st = np.array([rng_seed(int(seed))], dtype=np.uint64)
        assert oracle.olib().zo_rng_uniform(st.ctypes.data_as(C.POINTER(C.c_uint64))) == u


def test_golden_cases(golden):
    L = golden
    ties = 0
    for i in range(len(L["ids"])):
        n = int(L["n"][i])
        x = L["logits"][i: i + 1, :n]
        p = _params_of(L["params"][i])
        hl = int(L["hist_len"][i])
        h = L["hist"][i: i + 1] if hl else None
        hlen = L["hist_len"][i: i + 1] if hl else None
        st = np.array([rng_seed(int(L["seeds"][i]))], dtype=np.uint64)
        ids, info, *_ = oracle.oracle_sample(x, p, st, h, hlen, nthreads=1)
        ref = int(L["ids"][i])
        if int(ids[0]) != ref:
            assert L["tie"][i], f"case {i}: oracle {ids[0]} reference {ref} (no tie)"
            assert x[0, ids[0]] == x[0, ref], f"case {i}: drawn values differ"
            ties += 1
        # the rng advanced exactly as the reference's: same next() afterwards
        nxt = Rng(0)
        nxt.state = int(st[0])
        assert nxt.next() == int(L["next_after"][i]), f"case {i}: rng draws differ"
    assert ties <= int(L["tie"].sum())


def test_golden_workload_rows(golden):
    L = golden
    for cfg in (1, 2, 3, 4, 5):
        for sign in (1, -1):
            sel = np.nonzero(L["wl_cfg"] == sign * cfg)[0]
            if sel.size == 0:
                continue
            rows = int(L["wl_row"][sel].max()) + 1
            x = W.generate(cfg, rows)
            wl = W.WORKLOADS[cfg]
            p = wl.params if sign > 0 else SamplingParams()
            st = np.array([rng_seed(int(s)) for s in wl.row_seeds(0, rows)], dtype=np.uint64)
            ids, *_ = oracle.oracle_sample(x, p, st)
            for j in sel:
                r = int(L["wl_row"][j])
                ref = int(L["wl_ids"][j])
                if ids[r] != ref:
                    assert L["wl_tie"][j] and x[r, ids[r]] == x[r, ref], (cfg, sign, r)


def test_argmax_edges():
    rng = np.random.default_rng(1)
    rows = [np.array([np.nan, 1.0, 2.0], np.float32), np.array([1.0, np.nan, 3.0], np.float32),
            np.array([3.0, 3.0, 1.0], np.float32), np.array([-np.inf, -np.inf], np.float32),
            np.array([0.0, -0.0, 0.0], np.float32), np.array([np.inf, 1.0, np.inf], np.float32),
            np.array([5.0], np.float32)]
    rows += [(np.round(rng.normal(0, 1, 1000) * 4) / 4).astype(np.float32) for _ in range(20)]
    expect = [0, 2, 0, 0, 0, 0, 0]
    for i, r in enumerate(rows):
        o = oracle.oracle_argmax(r)
        if i < len(expect):
            assert o == expect[i], (i, o)
        if oracle.have_reference():
            assert o == oracle.reference_argmax(r)


needs_ref = pytest.mark.skipif(not oracle.have_reference(), reason="reference not built")


@needs_ref
@pytest.mark.parametrize("cfg", [1, 2, 3, 4, 5])
def test_workloads_against_reference(cfg):
    """Fresh rows of each workload (full vocabulary), restatement vs reference."""
    wl = W.WORKLOADS[cfg]
    rows = 1 if cfg == 1 else 24
    x = W.generate(cfg, rows, row0=100 if cfg != 1 else 0)
    seeds = np.arange(1, rows + 1, dtype=np.uint64) * np.uint64(7919)
    for p in [wl.params] + ([SamplingParams()] if wl.greedy_too else []):
        st = np.array([rng_seed(int(s)) for s in seeds], dtype=np.uint64)
        ids, info, *_ = oracle.oracle_sample(x, p, st)
        ref, nxt = oracle.reference_sample(x, p, seeds)
        for r in range(rows):
            if ids[r] != ref[r]:
                assert np.count_nonzero(x[r] == x[r, ref[r]]) > 1, (cfg, r)
                assert x[r, ids[r]] == x[r, ref[r]], (cfg, r)
            s = Rng(0)
            s.state = int(st[r])
            assert s.next() == int(nxt[r]), (cfg, r)
        if cfg != 4:  # continuous values: no ties at all
            assert np.array_equal(ids, ref)


@needs_ref
def test_penalty_against_reference():
    rng = np.random.default_rng(11)
    n, rows = 4096, 64
    x = rng.normal(0, 2, size=(rows, n)).astype(np.float32)
    hist = rng.integers(-5, n + 5, size=(rows, 128)).astype(np.int32)
    hist[:, 10:40] = hist[:, :1]  # one id repeated 31 times: the penalty compounds
    hlen = rng.integers(0, 129, size=rows).astype(np.int32)
    seeds = np.arange(rows, dtype=np.uint64) + np.uint64(3)
    for p in (SamplingParams(temp=0.8, top_k=40, top_p=0.9, repeat_penalty=1.3, repeat_last_n=64),
              SamplingParams(repeat_penalty=1.5, repeat_last_n=100),
              SamplingParams(temp=1.0, repeat_penalty=0.7, repeat_last_n=7)):
        st = np.array([rng_seed(int(s)) for s in seeds], dtype=np.uint64)
        ids, *_ = oracle.oracle_sample(x, p, st, hist, hlen)
        ref, _ = oracle.reference_sample(x, p, seeds, hist, hlen)
        assert np.array_equal(ids, ref)


@needs_ref
def test_per_row_params_against_reference():
    rng = np.random.default_rng(5)
    rows, n = 40, 3000
    x = rng.normal(0, 1.5, size=(rows, n)).astype(np.float32)
    plist = [SamplingParams(temp=float(rng.uniform(0.0, 2.0)) if r % 5 else 0.0,
                            top_k=int(rng.integers(0, 400)), top_p=float(rng.uniform(0.3, 1.0)))
             for r in range(rows)]
    seeds = np.arange(rows, dtype=np.uint64) + np.uint64(99)
    st = np.array([rng_seed(int(s)) for s in seeds], dtype=np.uint64)
    ids, *_ = oracle.oracle_sample(x, plist, st)
    ref, _ = oracle.reference_sample(x, plist, seeds)
    assert np.array_equal(ids, ref)


def test_restatement_internal_consistency():
    """Shortlist sorted (value desc, id asc), probabilities sum to 1, the drawn
    position is the first CDF entry above r, and the boundary is that distance."""
    rng = np.random.default_rng(3)
    x = rng.normal(0, 2, size=(16, 5000)).astype(np.float32)
    p = SamplingParams(temp=0.9, top_k=100, top_p=0.8)
    st = np.array([rng_seed(i + 1) for i in range(16)], dtype=np.uint64)
    ids, info, cid, cv, cp = oracle.oracle_sample(x, p, st, cand_ld=100)
    for r in range(16):
        order = sorted(range(5000), key=lambda i: (-x[r, i], i))[:100]
        assert list(cid[r]) == order
        assert abs(cp[r].sum() - 1.0) < 1e-12
        m, pos, u = int(info["m"][r]), int(info["pos"][r]), float(info["r"][r])
        rescale = 0.0
        for i in range(m):  # sequential, as the reference sums
            rescale += float(cp[r, i])
        acc, want = 0.0, m - 1
        for i in range(m):
            acc += float(cp[r, i]) / rescale
            if u < acc:
                want = i
                break
        assert pos == want
        assert ids[r] == cid[r, pos]


def _stats_numpy(x, topn):
    """src/main.cpp:473-503 in numpy (sequential f64 sum kept as a loop of adds)."""
    B, n = x.shape
    k = max(1, min(topn, n))
    out = {"min": [], "max": [], "z": [], "top_ids": [], "top_p": []}
    for r in range(B):
        row = x[r].astype(np.float64)
        mx, mn = -1e30, 1e30
        for v in row:
            mx = v if mx < v else mx
            mn = v if v < mn else mn
        z = 0.0
        for v in np.exp(row - mx):
            z += float(v)
        ids = sorted(range(n), key=lambda i: (-x[r, i] if x[r, i] == x[r, i] else np.inf, i))[:k]
        out["min"].append(mn)
        out["max"].append(mx)
        out["z"].append(z)
        out["top_ids"].append(ids)
        out["top_p"].append([np.exp(float(x[r, i]) - mx) / z if z else np.nan for i in ids])
    return {kk: np.array(v) for kk, v in out.items()}


@pytest.mark.parametrize("topn", [0, 1, 8, 50, 3000])
def test_logits_stats_restatement(topn):
    rng = np.random.default_rng(topn + 1)
    x = rng.normal(0, 2, size=(4, 2000)).astype(np.float32)
    x[1] = np.round(x[1] * 2) / 2     # ties
    x[2, 5] = np.nan                   # NaN: never counted, never in the top
    x[3, :] = -np.inf                  # nothing above the -1e30 start
    x[3, 7] = -np.inf
    o = oracle.oracle_logits_stats(x, topn)
    r = _stats_numpy(x, topn)
    np.testing.assert_array_equal(o["min"], r["min"])
    np.testing.assert_array_equal(o["max"], r["max"])
    np.testing.assert_allclose(o["z"], r["z"], rtol=1e-13, equal_nan=True)
    np.testing.assert_array_equal(o["top_ids"][:3], r["top_ids"][:3])
    np.testing.assert_allclose(o["top_p"], r["top_p"], rtol=1e-13, equal_nan=True)
    assert o["max"][3] == -1e30 and o["min"][3] == -np.inf


def _generate_case(rows=24, n=3000, T=20, eos=7):
    rng = np.random.default_rng(23)
    steps = []
    for t in range(T):
        x = rng.normal(0, 1.5, size=(rows, n)).astype(np.float32)
        x[:, 100:105] += 4.0  # a few ids dominate, so the penalty window matters
        steps.append(x)
    for r, t in ((1, 3), (5, 0), (9, 11), (13, 19), (20, 6)):
        steps[t][r, eos] = 60.0  # these rows draw eos at that step (p ~ 1)
    plist = []
    for r in range(rows):
        if r % 6 == 0:
            plist.append(SamplingParams(temp=0.0, repeat_penalty=1.5, repeat_last_n=4))
        elif r % 6 == 1:
            plist.append(SamplingParams(temp=0.9, top_k=0, top_p=1.0))
        else:
            plist.append(SamplingParams(temp=0.8, top_k=40, top_p=0.9, repeat_penalty=1.3,
                                        repeat_last_n=6))
    seeds = np.arange(rows, dtype=np.uint64) + np.uint64(1000)
    return steps, plist, seeds, eos


@needs_ref
def test_generate_loop_against_reference():
    """The generate-loop restatement (history = generated ids, eos stops the row
    without being appended, one draw per non-greedy step) against a loop over the
    unchanged reference's sample_token carrying each row's Rng state."""
    steps, plist, seeds, eos = _generate_case()
    rows, T = steps[0].shape[0], len(steps)
    st = np.array([rng_seed(int(s)) for s in seeds], dtype=np.uint64)
    o = oracle.oracle_generate(steps, plist, st, eos)
    for r in range(rows):
        state, gen, toks = rng_seed(int(seeds[r])), [], []
        for t in range(T):
            hist = np.array([gen if gen else [0]], dtype=np.int32)
            ids, _ = oracle.reference_sample(steps[t][r:r + 1], plist[r], np.array([state], np.uint64),
                                             hist, np.array([len(gen)], np.int32))
            if plist[r].temp > 0:
                g = Rng(state)
                g.next()
                state = g.state
            toks.append(int(ids[0]))
            if ids[0] == eos:
                break
            gen.append(int(ids[0]))
        assert o["tokens"][r, :len(toks)].tolist() == toks, r
        assert (o["tokens"][r, len(toks):] == -1).all()
        assert o["gen"][r] == gen
        assert int(st[r]) == state
    assert all(o["done"][r] for r in (1, 5, 9, 13, 20))  # the planted eos rows


def _lm_case(B=6, E=96, V=700, seed=3):
    rng = np.random.default_rng(seed)
    hidden = rng.normal(0, 3.0, size=(B, E)).astype(np.float32)
    hidden[0, :] *= 1e-3  # a small row: the eps term matters
    norm_w = rng.uniform(0.5, 1.5, size=E).astype(np.float32)
    w = oracle.f32_to_bf16_bits(rng.normal(0, 0.05, size=(V, E)).astype(np.float32))
    return hidden, norm_w, w


@needs_ref
def test_lmhead_restatement_against_reference():
    """rmsnorm + matvec (src/model.cpp:401-403): the restatement's xn before the
    bfloat16 rounding equals zen::rmsnorm's exactly (checked through the rounding
    of the reference's xn), and on bfloat16-valued inputs its logits equal
    zen::matvec_f32 with the scalar implementation exactly; the AVX2 one (float
    accumulators) within its own rounding."""
    hidden, norm_w, w = _lm_case()
    eps = 1e-6
    xn_b, lg = oracle.oracle_lmhead(hidden, norm_w, eps, w)
    wf = oracle.bf16_bits_to_f32(w)
    xn_ref, lg_ref_full = oracle.reference_lmhead(hidden, norm_w, eps, wf, impl=0)
    assert np.array_equal(oracle.f32_to_bf16_bits(xn_ref), xn_b)
    ref_on_bf16 = oracle.reference_matvec(oracle.bf16_bits_to_f32(xn_b), wf, impl=0)
    assert np.array_equal(ref_on_bf16, lg)
    avx = oracle.reference_matvec(oracle.bf16_bits_to_f32(xn_b), wf, impl=1)
    mag = np.abs(oracle.bf16_bits_to_f32(xn_b)).astype(np.float64) @ np.abs(wf).astype(np.float64).T
    assert np.all(np.abs(avx.astype(np.float64) - lg) <= 1e-6 * mag + 1e-30)
    # the full-precision reference differs only by the rounding of xn to bfloat16
    assert np.all(np.abs(lg_ref_full.astype(np.float64) - lg) <= 2.0 ** -8 * mag + 1e-30)


@needs_ref
@pytest.mark.parametrize("E", [896, 200, 20])
def test_lmhead_f32_restatement_against_reference(E):
    """The f32 lm_head in the reference's default (AVX2) summation order
    (src/kernels.cpp:52-78): xn and logits bit-exact against zen::rmsnorm and
    zen::matvec_f32_impl(Avx2) on bfloat16-valued weights, with a hidden size that
    is a multiple of 32, one with a tail of 8 summed in double, and one below 32."""
    rng = np.random.default_rng(E)
    B, V = 3, 257
    hidden = rng.normal(0, 3, size=(B, E)).astype(np.float32)
    hidden[1] *= np.float32(1e-3)
    norm_w = rng.uniform(0.5, 1.5, size=E).astype(np.float32)
    w = oracle.f32_to_bf16_bits(rng.normal(0, 0.05, size=(V, E)).astype(np.float32))
    xn, lg = oracle.oracle_lmhead_f32(hidden, norm_w, 1e-6, w)
    xn_ref, lg_ref = oracle.reference_lmhead(hidden, norm_w, 1e-6, oracle.bf16_bits_to_f32(w),
                                             impl=1)
    assert np.array_equal(xn.view(np.uint32), xn_ref.view(np.uint32))
    assert np.array_equal(lg.view(np.uint32), lg_ref.view(np.uint32))


def test_bf16_rounding_helpers():
    x = np.array([1.0, 1.00390625, 1.005859375, -2.5, 3.0e38, np.inf, -0.0], dtype=np.float32)
    b = oracle.f32_to_bf16_bits(x)
    back = oracle.bf16_bits_to_f32(b)
    assert back[0] == 1.0 and back[1] == 1.0  # halfway, ties to even
    assert back[2] == np.float32(1.0078125)
    assert back[3] == -2.5 and np.isinf(back[5]) and np.signbit(back[6])
    assert np.isnan(oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(np.array([np.nan], np.float32))))[0]


@needs_ref
def test_full_vocab_top_p_against_reference():
    """top_k >= n makes the shortlist the whole row (k = min(top_k, n) = n): the
    nucleus over the full vocabulary.  Restatement and reference agree exactly."""
    rng = np.random.default_rng(41)
    rows, n = 24, 3000
    ranks = np.argsort(rng.random((rows, n)), axis=1)
    x = (-1.1 * np.log(ranks + 1.0) + rng.normal(0, 0.3, size=(rows, n))).astype(np.float32)
    seeds = np.arange(rows, dtype=np.uint64) + np.uint64(7)
    for top_k in (n, 2 ** 31 - 1):
        p = SamplingParams(temp=1.0, top_k=top_k, top_p=0.95)
        st = np.array([rng_seed(int(s)) for s in seeds], dtype=np.uint64)
        ids, info, *_ = oracle.oracle_sample(x, p, st)
        ref, _ = oracle.reference_sample(x, p, seeds)
        assert np.array_equal(ids, ref)
        assert (info["k"] == n).all() and (info["m"] > 256).all()
