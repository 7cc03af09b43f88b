"""The lm_head fused with the sampler (zs_lmhead_sample) against the oracle.

Model::eval ends with rmsnorm + matvec over output.weight (src/model.cpp:401-403)
and cmd_generate samples the result (src/main.cpp:628).  The fused path computes
the logits on the tensor cores (bf16 xn and weights, f32 accumulation) and selects
the shortlist in the GEMM epilogue.  Parity, per case:
  * logits (written by the same kernel) against the restatement on the same bf16
    inputs within the recursive-summation bound  |d| <= (E + 2) 2^-24 sum|xn_i w_i|,
    and against the unchanged reference's f32 lm_head within the bf16 rounding of
    xn, |d| <= 2^-8 sum|xn_i w_i|;
  * ids and Rng states bit-exact against zs_sample run on those logits, which is
    itself checked against the restatement under the sampler's parity rules.
The cases below force the fused route (the default takes two passes up to 1024
rows), so the epilogue's selection is covered at every size, up to the 2048 and
4096 rows the default route sends to it; one test checks that the routes agree bit
for bit, and two build logits that tie exactly across vocabulary slices
(duplicated weight rows) and at zero (all-zero weight rows, +0 and -0), where the
slices' shared threshold bound decides which keys may enter a row's buffer."""

import numpy as np
import pytest

import oracle
from tests.gpu_util import compare, run_gpu, run_oracle
from zeninfer_b200 import SamplingParams, rng_seed, states_to_tensor, tensor_to_states

pytestmark = pytest.mark.gpu

EPS = 1e-6
_MODELS = {}


def _model(V, E, seed=7):
    """bf16 output.weight [V, E] (as torch CPU tensor) and output_norm [E]."""
    import torch
    key = (V, E, seed)
    if key not in _MODELS:
        g = torch.Generator().manual_seed(seed)
        w = (torch.randn(V, E, generator=g) * 0.05).to(torch.bfloat16)
        nw = torch.rand(E, generator=g) + 0.5
        _MODELS.clear()
        _MODELS[key] = (w, nw)
    return _MODELS[key]


def _hidden(B, E, seed):
    import torch
    g = torch.Generator().manual_seed(1000 + seed)
    h = torch.randn(B, E, generator=g) * 3.0
    if B > 1:
        h[1] *= 1e-3  # a small row: the eps term of rmsnorm matters
    return h


def _run(sampler, hidden, nw, w, params, seeds, with_logits=True, history=None, hlen=None,
         route="fused", tiles="auto"):
    import torch
    dev = sampler.device
    B, V = hidden.shape[0], w.shape[0]
    st = states_to_tensor([rng_seed(int(s)) for s in seeds], dev)
    lg = None
    if with_logits:
        lg = torch.full((B, (V + 3) // 4 * 4), float("nan"), dtype=torch.float32, device=dev)
    h = hl = None
    if history is not None:
        h = torch.from_numpy(history).to(dev)
        hl = torch.from_numpy(hlen).to(dev)
    sampler.set_lmhead_route(route)
    sampler.set_lmhead_tiles(tiles)
    try:
        ids = sampler.lmhead_sample(hidden.to(dev), nw.to(dev), w.to(dev), params, st, eps=EPS,
                                    history=h, history_len=hl, out_logits=lg)
    finally:
        sampler.set_lmhead_route("auto")
        sampler.set_lmhead_tiles("auto")
    sampler.check_device_status()
    out = {"ids": ids.cpu().numpy(), "states": tensor_to_states(st)}
    if lg is not None:
        out["logits"] = lg[:, :V].cpu().numpy()
    return out


def _w_bits(w):
    import torch
    return w.view(torch.int16).numpy().view(np.uint16)


_WF = {}


def _w_f32(w):
    """float32 copy of the bf16 weights and its absolute values (cached)."""
    if _WF.get("src") is not w:
        _WF.clear()
        wf = oracle.bf16_bits_to_f32(_w_bits(w))
        _WF.update(src=w, wf=wf, absw=np.abs(wf))
    return _WF["wf"], _WF["absw"]


def _check_logits(got, hidden, nw, w, rows, against_reference=False):
    h = hidden.numpy()[rows]
    wb = _w_bits(w)
    xn_b, lg = oracle.oracle_lmhead(h, nw.numpy(), EPS, wb)
    wf, absw = _w_f32(w)
    # sum |xn_i w_i| per logit; float32 is ample for a bound (scaled up by 1.01)
    mag = (np.abs(oracle.bf16_bits_to_f32(xn_b)) @ absw.T).astype(np.float64) * 1.01
    E = h.shape[1]
    d = np.abs(got[rows].astype(np.float64) - lg.astype(np.float64))
    assert np.all(d <= (E + 2) * 2.0 ** -24 * mag + 1e-30), float((d / (mag + 1e-30)).max())
    if against_reference and oracle.have_reference():
        _, ref = oracle.reference_lmhead(h, nw.numpy(), EPS, wf, impl=0)
        d2 = np.abs(got[rows].astype(np.float64) - ref.astype(np.float64))
        assert np.all(d2 <= 2.0 ** -8 * mag + 1e-30)


def _check_sampling(sampler, res, params, seeds, history=None, hlen=None):
    """ids/states bit-exact vs zs_sample on the kernel's own logits, and that
    against the restatement."""
    st0 = np.array([rng_seed(int(s)) for s in seeds], dtype=np.uint64)
    g = run_gpu(sampler, res["logits"], params, st0, history, hlen)
    assert np.array_equal(res["ids"], g["ids"])
    assert np.array_equal(res["states"], g["states"])
    o = run_oracle(res["logits"], params, st0, history, hlen)
    compare(g, o)


def _mixed_params(B):
    out = []
    for r in range(B):
        out.append([SamplingParams(temp=0.0),
                    SamplingParams(temp=0.7, top_k=40, top_p=0.9),
                    SamplingParams(temp=1.0, top_k=1),
                    SamplingParams(temp=0.8, top_k=64, top_p=0.95),
                    SamplingParams(temp=1.3, top_k=7),
                    SamplingParams(temp=0.9, top_k=88, top_p=0.97)][r % 6])
    return out


def test_lmhead_small_shapes(sampler):
    """A vocabulary that is not a multiple of the 128-column tile, a hidden size of
    two K stages, a batch smaller than one row tile, per-row params."""
    V, E, B = 1000, 128, 5
    w, nw = _model(V, E, seed=3)
    hidden = _hidden(B, E, 3)
    params = _mixed_params(B)
    seeds = np.arange(B, dtype=np.uint64) + np.uint64(11)
    res = _run(sampler, hidden, nw, w, params, seeds)
    _check_logits(res["logits"], hidden, nw, w, np.arange(B), against_reference=True)
    _check_sampling(sampler, res, params, seeds)


def test_lmhead_full_vocab_batch(sampler):
    """The Qwen2.5-0.5B lm_head shape (151,936 x 896) at 300 rows (warp merge),
    temp 0.7, top-k 50, top-p 0.9; then the same rows without the logits output."""
    V, E, B = 151936, 896, 300
    w, nw = _model(V, E)
    hidden = _hidden(B, E, 5)
    p = SamplingParams(temp=0.7, top_k=50, top_p=0.9)
    seeds = np.arange(B, dtype=np.uint64) * np.uint64(7) + np.uint64(1)
    res = _run(sampler, hidden, nw, w, p, seeds)
    _check_logits(res["logits"], hidden, nw, w, np.array([0, 1, 2, 150, 299]),
                  against_reference=True)
    _check_sampling(sampler, res, p, seeds)
    res2 = _run(sampler, hidden, nw, w, p, seeds, with_logits=False)
    assert np.array_equal(res2["ids"], res["ids"])
    assert np.array_equal(res2["states"], res["states"])


def test_lmhead_batch_one_and_mixed(sampler):
    """Decode-sized batches: one row, and 37 rows with per-row params."""
    V, E = 151936, 896
    w, nw = _model(V, E)
    for B, params in ((1, SamplingParams(temp=0.7, top_k=40)), (37, _mixed_params(37))):
        hidden = _hidden(B, E, 9 + B)
        seeds = np.arange(B, dtype=np.uint64) + np.uint64(5)
        res = _run(sampler, hidden, nw, w, params, seeds)
        _check_logits(res["logits"], hidden, nw, w, np.arange(min(B, 3)))
        _check_sampling(sampler, res, params, seeds)


def test_lmhead_two_pass_route(sampler):
    """Rows the epilogue does not hold (a repeat penalty, top-k above 88, the
    default 256-token shortlist) go through the written logits and zs_sample."""
    V, E, B = 151936, 896, 24
    w, nw = _model(V, E)
    hidden = _hidden(B, E, 21)
    params = []
    for r in range(B):
        params.append([SamplingParams(temp=0.7, top_k=40, top_p=0.9, repeat_penalty=1.3,
                                      repeat_last_n=16),
                       SamplingParams(temp=0.8, top_k=100),
                       SamplingParams(temp=0.9)][r % 3])
    rng = np.random.default_rng(4)
    hist = rng.integers(0, V, size=(B, 32)).astype(np.int32)
    hlen = rng.integers(0, 33, size=B).astype(np.int32)
    seeds = np.arange(B, dtype=np.uint64) + np.uint64(101)
    res = _run(sampler, hidden, nw, w, params, seeds, history=hist, hlen=hlen)
    _check_logits(res["logits"], hidden, nw, w, np.arange(2))
    _check_sampling(sampler, res, params, seeds, hist, hlen)
    # without out_logits the logits live in handle scratch; same draws
    res2 = _run(sampler, hidden, nw, w, params, seeds, with_logits=False, history=hist, hlen=hlen)
    assert np.array_equal(res2["ids"], res["ids"])


@pytest.mark.parametrize("B", [16, 300])
def test_lmhead_routes_agree(sampler, B):
    """Fused, two-pass and the default route give the same ids, Rng states and
    logits, bit for bit (16 rows: the default takes two passes; up to 8 rows it takes
    the exact route, tested below)."""
    V, E = 151936, 896
    w, nw = _model(V, E)
    hidden = _hidden(B, E, 41)
    params = _mixed_params(B)
    seeds = np.arange(B, dtype=np.uint64) + np.uint64(77)
    got = {r: _run(sampler, hidden, nw, w, params, seeds, route=r)
           for r in ("fused", "two_pass", "auto")}
    for r in ("two_pass", "auto"):
        assert np.array_equal(got[r]["ids"], got["fused"]["ids"]), r
        assert np.array_equal(got[r]["states"], got["fused"]["states"]), r
        assert np.array_equal(got[r]["logits"].view(np.uint32),
                              got["fused"]["logits"].view(np.uint32)), r
    _check_sampling(sampler, got["auto"], params, seeds)


@pytest.mark.parametrize("B,tiles", [(5, "pair"), (37, "pair"), (300, "single"),
                                     (300, "pair"), (2048, "single")])
def test_lmhead_tiles(sampler, B, tiles):
    """One-CTA tiles and CTA-pair tiles (tcgen05 cta_group::2, 256 x 256), each
    forced where the default would take the other: pairs at 5 and 37 rows (the
    second CTA's rows all lie outside the batch), single CTAs at 300 and 2048 rows.
    Logits within the bounds, ids and Rng states against zs_sample on those logits
    and the restatement, both routes, and the same logits and draws, bit for bit, as
    the other tiling."""
    V, E = 151936, 896
    w, nw = _model(V, E)
    hidden = _hidden(B, E, 90 + B)
    params = _mixed_params(B)
    seeds = np.arange(B, dtype=np.uint64) + np.uint64(13)
    other = "single" if tiles == "pair" else "pair"
    res = _run(sampler, hidden, nw, w, params, seeds, tiles=tiles)
    _check_logits(res["logits"], hidden, nw, w, np.array([0, 1, B // 2, B - 1]),
                  against_reference=True)
    _check_sampling(sampler, res, params, seeds)
    two = _run(sampler, hidden, nw, w, params, seeds, route="two_pass", tiles=tiles)
    _check_logits(two["logits"], hidden, nw, w, np.array([0, B - 1]))
    _check_sampling(sampler, two, params, seeds)
    alt = _run(sampler, hidden, nw, w, params, seeds, tiles=other)
    _check_sampling(sampler, alt, params, seeds)
    # the two MMA shapes add the same products in the same K order: bit-equal logits,
    # so bit-equal draws
    assert np.array_equal(alt["logits"].view(np.uint32), res["logits"].view(np.uint32))
    assert np.array_equal(alt["ids"], res["ids"])
    assert np.array_equal(alt["states"], res["states"])


@pytest.mark.parametrize("B,E,V", [(1, 896, 151936), (4, 896, 151936), (8, 896, 151936),
                                   (2, 200, 1000), (4, 2048, 3000), (8, 64, 777)])
def test_lmhead_exact_route(sampler, B, E, V):
    """The exact route: f32 xn and the reference's AVX2 summation order
    (src/kernels.cpp:52-78).  Logits bit-exact against the restatement (itself
    pinned to the reference) and, where the reference is built, against
    zen::rmsnorm + zen::matvec_f32_impl(Avx2) directly; a hidden size with a tail of
    8 past the last multiple of 32, the largest hidden size, and the smallest.  Ids
    and Rng states against zs_sample on those logits and the restatement; the default
    route takes it up to 8 rows."""
    w, nw = _model(V, E, seed=11)
    hidden = _hidden(B, E, 120 + B)
    params = _mixed_params(B)
    seeds = np.arange(B, dtype=np.uint64) + np.uint64(21)
    res = _run(sampler, hidden, nw, w, params, seeds, route="exact")
    _, lg = oracle.oracle_lmhead_f32(hidden.numpy(), nw.numpy(), EPS, _w_bits(w))
    assert np.array_equal(res["logits"].view(np.uint32), lg.view(np.uint32))
    if oracle.have_reference():
        _, ref = oracle.reference_lmhead(hidden.numpy(), nw.numpy(), EPS, _w_f32(w)[0], impl=1)
        assert np.array_equal(res["logits"].view(np.uint32), ref.view(np.uint32))
    _check_sampling(sampler, res, params, seeds)
    auto = _run(sampler, hidden, nw, w, params, seeds, route="auto")
    assert np.array_equal(auto["logits"].view(np.uint32), res["logits"].view(np.uint32))
    assert np.array_equal(auto["ids"], res["ids"])
    assert np.array_equal(auto["states"], res["states"])
    # without out_logits (handle scratch), and through zs_lmhead_logits
    res2 = _run(sampler, hidden, nw, w, params, seeds, with_logits=False, route="exact")
    assert np.array_equal(res2["ids"], res["ids"])
    dev = sampler.device
    lg2 = sampler.lmhead_logits(hidden.to(dev), nw.to(dev), w.to(dev), eps=EPS)
    sampler.check_device_status()
    assert np.array_equal(lg2.cpu().numpy().view(np.uint32), lg.view(np.uint32))


@pytest.mark.parametrize("B,E", [(9, 128), (5, 2048)])
def test_lmhead_exact_route_limits(sampler, B, E):
    """The exact route holds up to 8 rows and 8192 values of rows x hidden size: 9
    rows, or 5 rows of 2048, are refused, not run another way."""
    from zeninfer_b200._native import SamplerError
    V = 1000
    w, nw = _model(V, E, seed=3)
    hidden = _hidden(B, E, 3)
    with pytest.raises(SamplerError):
        _run(sampler, hidden, nw, w, SamplingParams(temp=0.7, top_k=40),
             np.arange(B, dtype=np.uint64), route="exact")


def test_lmhead_tiles_rejects_unknown(sampler):
    with pytest.raises(ValueError):
        sampler.set_lmhead_tiles("quad")


def test_lmhead_route_rejects_unknown(sampler):
    with pytest.raises(ValueError):
        sampler.set_lmhead_route("fastest")


def test_lmhead_rejects_bad_shapes(sampler):
    import torch
    from zeninfer_b200._native import SamplerError
    dev = sampler.device
    w = torch.zeros((256, 60), dtype=torch.bfloat16, device=dev)
    with pytest.raises(SamplerError):  # hidden size below one K stage
        sampler.lmhead_sample(torch.zeros((1, 60), device=dev), torch.ones(60, device=dev), w,
                              SamplingParams(), None)


@pytest.mark.parametrize("B", [40, 300])
def test_lmhead_logits_alone(sampler, B):
    """zs_lmhead_logits (the lm_head without sampling) writes the same logits as the
    fused entry's logits output, bit for bit, and they are within the bound of the
    restatement; 40 rows store directly, 300 rows through shared memory and TMA."""
    V, E = 151936, 896
    w, nw = _model(V, E)
    hidden = _hidden(B, E, 33)
    p = SamplingParams(temp=0.7, top_k=50, top_p=0.9)
    seeds = np.arange(B, dtype=np.uint64) + np.uint64(3)
    res = _run(sampler, hidden, nw, w, p, seeds)
    dev = sampler.device
    lg = sampler.lmhead_logits(hidden.to(dev), nw.to(dev), w.to(dev), eps=EPS)
    sampler.check_device_status()
    got = lg.cpu().numpy()
    assert np.array_equal(got, res["logits"])
    _check_logits(got, hidden, nw, w, np.array([0, 1, B - 1]))


@pytest.mark.parametrize("B", [2048, 4096])
def test_lmhead_fused_at_routed_batches(sampler, B):
    """The batch sizes the default route sends to the fused kernel, with the
    benchmark's parameters: ids and Rng states against zs_sample on the kernel's own
    logits and the restatement on every row; the same ids without the logits
    output; logits within the bounds on a few rows."""
    V, E = 151936, 896
    w, nw = _model(V, E)
    hidden = _hidden(B, E, 60 + B)
    p = SamplingParams(temp=0.7, top_k=50, top_p=0.9)
    seeds = np.arange(B, dtype=np.uint64) + np.uint64(9)
    res = _run(sampler, hidden, nw, w, p, seeds)
    _check_logits(res["logits"], hidden, nw, w, np.array([0, 1, B // 2, B - 1]),
                  against_reference=True)
    _check_sampling(sampler, res, p, seeds)
    res2 = _run(sampler, hidden, nw, w, p, seeds, with_logits=False)
    assert np.array_equal(res2["ids"], res["ids"])
    assert np.array_equal(res2["states"], res["states"])
    auto = _run(sampler, hidden, nw, w, p, seeds, with_logits=False, route="auto")
    assert np.array_equal(auto["ids"], res["ids"])


def _tied_model(V, E, seed, zero_rows):
    """Weights whose second half repeats the first (every logit occurs twice, the
    copies V/2 columns apart, so in different vocabulary slices) with all-zero rows
    (and their copies) at `zero_rows`."""
    import torch
    g = torch.Generator().manual_seed(seed)
    half = V // 2
    base = (torch.randn(half, E, generator=g) * 0.05).to(torch.bfloat16)
    base[zero_rows] = 0
    w = torch.cat([base, base], 0)
    nw = torch.rand(E, generator=g) + 0.5
    return w, nw


@pytest.mark.parametrize("B", [300, 2048])
def test_lmhead_ties_across_slices(sampler, B):
    """Random weights, every logit doubled across slices, zero rows: ids and Rng
    states of the fused route equal zs_sample's on the same logits, bit for bit."""
    V, E = 151936, 896
    zero = np.arange(0, V // 2, 1777)
    w, nw = _tied_model(V, E, 5, zero)
    hidden = _hidden(B, E, 70)
    params = _mixed_params(B)
    seeds = np.arange(B, dtype=np.uint64) + np.uint64(31)
    res = _run(sampler, hidden, nw, w, params, seeds)
    lg = res["logits"]
    assert np.array_equal(lg[:, :V // 2].view(np.uint32), lg[:, V // 2:].view(np.uint32))
    _check_sampling(sampler, res, params, seeds)
    two = _run(sampler, hidden, nw, w, params, seeds, route="two_pass")
    assert np.array_equal(two["ids"], res["ids"])
    assert np.array_equal(two["states"], res["states"])


@pytest.mark.parametrize("B", [300, 2048])
def test_lmhead_ties_at_zero(sampler, B):
    """Every row's best logits are exact zeros, tied across slices: all weight rows
    point against one hidden direction (their logits negative) except zero rows.
    Hidden rows along that direction (all entries negative) make every product at a
    zero row -0; rows with a few positive entries add +0 products (the sign the
    tensor cores give the sums is theirs to choose: either way the ids must match
    zs_sample's on the same logits).  Shortlists of 20 (inside the
    tie group of 2 x 19 zeros), 38 (exactly the group) and 50 and 88 (past it)."""
    import torch
    V, E = 151936, 896
    half = V // 2
    g = torch.Generator().manual_seed(12)
    d = -(0.5 + torch.rand(E, generator=g))          # all entries negative
    scale = 0.5 + torch.rand(half, 1, generator=g)
    base = (scale * (-d)[None, :] * 0.02).to(torch.bfloat16)  # logits < 0 along d
    zero = np.arange(7, half, 4001)[:19]
    base[zero] = 0
    w = torch.cat([base, base], 0)
    nw = torch.rand(E, generator=g) + 0.5
    c = 0.5 + torch.rand(B, 1, generator=g)
    hidden = c * d[None, :]
    noisy = torch.arange(B) % 2 == 1
    hidden[noisy] += torch.randn(int(noisy.sum()), E, generator=g) * 0.05
    hidden[noisy, :8] = hidden[noisy, :8].abs()  # a few positive entries: +0 at zero rows
    params = [[SamplingParams(temp=0.7, top_k=20), SamplingParams(temp=0.7, top_k=38, top_p=0.9),
               SamplingParams(temp=1.0, top_k=50), SamplingParams(temp=0.9, top_k=88),
               SamplingParams()][r % 5] for r in range(B)]
    seeds = np.arange(B, dtype=np.uint64) + np.uint64(57)
    res = _run(sampler, hidden, nw, w, params, seeds)
    lg = res["logits"]
    zs = np.concatenate([zero, zero + half])
    assert np.all(lg[:, zs] == 0)
    assert lg[:, np.setdiff1d(np.arange(V), zs)].max() < 0
    _check_sampling(sampler, res, params, seeds)
    two = _run(sampler, hidden, nw, w, params, seeds, route="two_pass")
    assert np.array_equal(two["ids"], res["ids"])
    assert np.array_equal(two["states"], res["states"])
