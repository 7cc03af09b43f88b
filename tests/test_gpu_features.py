"""CUDA sampler against the reference's golden vectors and the restatement on
the branches of sample_token that the workload tests do not reach: the
repetition penalty (fast window and the large-window path), large top-k, log Z,
odd shapes and strides, per-row parameters, the vocab-sharded layout (all
shards on one GPU), the zen:: C++ API and the argmax entry point."""

import os
import subprocess

import numpy as np
import pytest

import oracle
from tests.gpu_util import BOUNDARY_EPS, compare, run_gpu, run_oracle
from zeninfer_b200 import (Rng, SamplingParams, rng_seed, sample_token, states_to_tensor,
                           tensor_to_states)
from zeninfer_b200 import sharding
from zeninfer_b200 import workloads as W

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden", "sampler_golden.npz")
V = W.VOCAB


def _states(seeds):
    return np.asarray([rng_seed(int(s)) for s in seeds], dtype=np.uint64)


def _params_of(rec):
    return SamplingParams(float(rec["temp"]), int(rec["top_k"]), float(rec["top_p"]),
                          float(rec["repeat_penalty"]), int(rec["repeat_last_n"]))


def test_golden_vectors(sampler):
    """Every golden case of the reference, batched by row length (per-row params,
    rows at a stride of 2048 floats)."""
    import torch
    L = np.load(GOLDEN)
    dev = sampler.device
    xg = torch.from_numpy(L["logits"]).to(dev)
    for n in np.unique(L["n"]):
        sel = np.nonzero(L["n"] == n)[0]
        x = xg[torch.from_numpy(sel).to(dev)][:, :n]  # rows 2048 floats apart
        plist = [_params_of(L["params"][i]) for i in sel]
        seeds = L["seeds"][sel]
        hist = torch.from_numpy(L["hist"][sel]).to(dev)
        hl = torch.from_numpy(L["hist_len"][sel]).to(dev)
        st = states_to_tensor(_states(seeds), dev)
        ids = sampler.sample(x, plist, st, hist, hl, sync_check=True).ids.cpu().numpy()
        after = tensor_to_states(st)
        o_st = _states(seeds)
        _, info, *_ = oracle.oracle_sample(L["logits"][sel][:, :n], plist, o_st,
                                           L["hist"][sel], L["hist_len"][sel])
        for j, i in enumerate(sel):
            ref = int(L["ids"][i])
            if ids[j] != ref:
                xr = L["logits"][i, :n]
                ok = (L["tie"][i] and xr[ids[j]] == xr[ref]) or info["boundary"][j] < BOUNDARY_EPS
                assert ok, f"golden case {i} (n={n}): gpu {ids[j]} reference {ref}"
            r = Rng(0)
            r.state = int(after[j])
            assert r.next() == int(L["next_after"][i]), f"golden case {i}: rng"


def test_golden_workload_rows(sampler):
    L = np.load(GOLDEN)
    for cfg in (1, 2, 3, 4, 5):
        for sign in (1, -1):
            sel = np.nonzero(L["wl_cfg"] == sign * cfg)[0]
            if sel.size == 0:
                continue
            rows = int(L["wl_row"][sel].max()) + 1
            x = W.generate(cfg, rows)
            wl = W.WORKLOADS[cfg]
            p = wl.params if sign > 0 else SamplingParams()
            g = run_gpu(sampler, x, p, _states(wl.row_seeds(0, rows)))
            o = run_oracle(x, p, _states(wl.row_seeds(0, rows)))
            for j in sel:
                r, ref = int(L["wl_row"][j]), int(L["wl_ids"][j])
                if g["ids"][r] != ref:
                    assert ((L["wl_tie"][j] and x[r, g["ids"][r]] == x[r, ref])
                            or o["info"]["boundary"][r] < BOUNDARY_EPS), (cfg, sign, r)


def _history(rows, L, n, seed, dup=True):
    rng = np.random.default_rng(seed)
    h = rng.integers(-3, n + 3, size=(rows, L)).astype(np.int32)
    if dup:
        h[:, 5:25] = h[:, :1]
    hl = rng.integers(0, L + 1, size=rows).astype(np.int32)
    return h, hl


@pytest.mark.parametrize("params", [
    SamplingParams(temp=0.7, top_k=40, top_p=0.9, repeat_penalty=1.3, repeat_last_n=64),
    SamplingParams(repeat_penalty=1.5, repeat_last_n=64),                       # greedy
    SamplingParams(temp=1.0, top_p=0.95, repeat_penalty=0.8, repeat_last_n=300),
    SamplingParams(temp=0.9, top_k=100, repeat_penalty=1.2, repeat_last_n=700),  # large window
    SamplingParams(temp=0.8, top_k=2000, repeat_penalty=1.1, repeat_last_n=100),  # keff > 2048
    SamplingParams(temp=0.9, top_k=600, repeat_penalty=1.2, repeat_last_n=200),  # long warp config
    SamplingParams(temp=0.8, top_k=40, repeat_penalty=1.3, repeat_last_n=200),   # window > 64
])
def test_penalty(sampler, params):
    rows = 64
    x = W.generate(2, rows, row0=300)
    h, hl = _history(rows, 800, V, 4)
    k = params.top_k if params.top_k > 0 else 256
    cl = k if params.temp > 0 else 0
    st = _states(range(rows))
    compare(run_gpu(sampler, x, params, st, h, hl, cand_ld=cl),
            run_oracle(x, params, st, h, hl, cand_ld=cl))


@pytest.mark.parametrize("k", [2049, 5000, 40000, V])
def test_large_top_k(sampler, k):
    rows = 8
    x = W.generate(3, rows, row0=9)
    p = SamplingParams(temp=1.1, top_k=k, top_p=0.97)
    st = _states(range(rows))
    compare(run_gpu(sampler, x, p, st, cand_ld=min(k, 6000)),
            run_oracle(x, p, st, cand_ld=min(k, 6000)))


@pytest.mark.parametrize("params", [SamplingParams(temp=0.7, top_k=50, top_p=0.9),
                                    SamplingParams(), SamplingParams(temp=1.5, top_k=3000)])
def test_log_z(sampler, params):
    rows = 32
    x = W.generate(5, rows, row0=11)
    st = _states(range(rows))
    g = run_gpu(sampler, x, params, st, want_log_z=True)
    o = run_oracle(x, params, st, full_z=True)
    np.testing.assert_allclose(g["info"]["log_z"], o["info"]["log_z"], rtol=0, atol=2e-4)


@pytest.mark.parametrize("n", [1, 2, 3, 5, 17, 255, 1000, 4097, 8191, 8193, 65537])
@pytest.mark.parametrize("pad", [0, 1, 3])
def test_odd_shapes(sampler, n, pad):
    """Row lengths around the tile sizes, row strides that break 16-byte alignment."""
    import torch
    rows = 5
    rng = np.random.default_rng(n * 7 + pad)
    xf = rng.normal(0, 2, size=(rows, n + pad)).astype(np.float32)
    dev = sampler.device
    xd = torch.from_numpy(xf).to(dev)[:, :n]
    for p in (SamplingParams(), SamplingParams(temp=0.8, top_k=40, top_p=0.9),
              SamplingParams(temp=1.0, top_k=1), SamplingParams(temp=0.5, top_k=10 * n + 7),
              SamplingParams(temp=1e-3, top_p=0.0)):
        st = _states(range(1, rows + 1))
        std = states_to_tensor(st, dev)
        ids = sampler.sample(xd, p, std, sync_check=True).ids.cpu().numpy()
        ost = st.copy()
        oids, info, *_ = oracle.oracle_sample(np.ascontiguousarray(xf[:, :n]), p, ost)
        bad = (ids != oids) & (info["boundary"] >= BOUNDARY_EPS)
        assert not bad.any(), (n, pad, p, ids, oids)
        assert np.array_equal(tensor_to_states(std), ost)


def test_special_values(sampler):
    rows, n = 6, 3000
    rng = np.random.default_rng(2)
    x = rng.normal(0, 1, size=(rows, n)).astype(np.float32)
    x[0, 100] = np.inf
    x[1, ::2] = -np.inf
    x[2, :] = 0.5            # all equal
    x[3, 7] = np.nan         # NaN away from index 0: never the max
    x[4, 0] = np.nan         # NaN at index 0: greedy returns 0
    x[5, :1000] = -0.0
    for p in (SamplingParams(), SamplingParams(temp=0.8, top_k=40, top_p=0.9)):
        for r in range(rows):
            if p.temp > 0 and r in (3, 4):
                continue  # with a NaN in the row the reference's comparator is not an order
            st = _states([r + 1])
            compare(run_gpu(sampler, x[r: r + 1], p, st), run_oracle(x[r: r + 1], p, st),
                    check_cands=False)


def test_per_row_params(sampler):
    rows = 300
    rng = np.random.default_rng(8)
    x = W.generate(2, rows, row0=40)
    plist = []
    for r in range(rows):
        t = 0.0 if r % 7 == 0 else float(rng.uniform(0.2, 2.0))
        plist.append(SamplingParams(temp=t, top_k=int(rng.choice([0, 1, 5, 40, 256, 1024, 2048])),
                                    top_p=float(rng.choice([1.0, 0.9, 0.5, 0.0]))))
    st = _states(range(rows))
    compare(run_gpu(sampler, x, plist, st), run_oracle(x, plist, st))


@pytest.mark.parametrize("world", [2, 3, 8])
@pytest.mark.parametrize("params", [SamplingParams(temp=0.7, top_k=50, top_p=0.9),
                                    SamplingParams(),
                                    SamplingParams(temp=1.0, top_p=0.95, repeat_penalty=1.3,
                                                   repeat_last_n=64)])
def test_vocab_shards_on_one_gpu(sampler, world, params):
    """Every rank's partials computed on one GPU, gathered by a plain copy, then
    merged: ids and rng states equal the unsharded call."""
    import torch
    from zeninfer_b200 import Sampler
    rows = 96
    dev = sampler.device
    x = torch.from_numpy(W.generate(5, rows, row0=500)).to(dev)
    h, hl = _history(rows, 96, V, 6)
    hd, hld = torch.from_numpy(h).to(dev), torch.from_numpy(hl).to(dev)
    nbytes = Sampler.shard_partial_bytes(rows, V, world, params)
    recv = torch.empty(world * nbytes, dtype=torch.uint8, device=dev)
    for g in range(world):
        lo, n = sharding.vocab_range(V, world, g)
        sampler.shard_partials(x[:, lo:lo + n], lo, V, world, params,
                               recv[g * nbytes:(g + 1) * nbytes], hd, hld, want_log_z=True)
    st_sh = states_to_tensor(_states(range(rows)), dev)
    res = sampler.shard_merge(recv, world, rows, V, params, st_sh, row_info=True,
                              want_log_z=True)
    sampler.check_device_status()
    st_one = states_to_tensor(_states(range(rows)), dev)
    one = sampler.sample(x, params, st_one, hd, hld, row_info=True, want_log_z=True,
                         sync_check=True)
    assert np.array_equal(res.ids.cpu().numpy(), one.ids.cpu().numpy())
    assert np.array_equal(tensor_to_states(st_sh), tensor_to_states(st_one))
    np.testing.assert_allclose(res.row_info["log_z"], one.row_info["log_z"], rtol=0, atol=2e-4)


@pytest.mark.parametrize("world,rows", [(2, 96), (3, 97), (8, 97)])
@pytest.mark.parametrize("params", [SamplingParams(temp=0.7, top_k=50, top_p=0.9),
                                    SamplingParams(temp=0.8, top_k=1024),
                                    SamplingParams(temp=1.0, top_k=1500, top_p=0.9),
                                    SamplingParams(temp=1.0, top_p=0.95, repeat_penalty=1.3,
                                                   repeat_last_n=64)])
def test_vocab_shard_row_owner_merge_on_one_gpu(sampler, world, rows, params):
    """The row-owner exchange emulated on one GPU: every rank's partials computed
    here; each owner's buffer gets only the zs_shard_row_spans of its rows from every
    rank (everything else is filler bytes), and zs_shard_merge_rows merges only those
    rows.  Over all owners, ids and rng states equal the unsharded call."""
    import torch
    from zeninfer_b200 import Sampler
    dev = sampler.device
    x = torch.from_numpy(W.generate(5, rows, row0=700)).to(dev)
    h, hl = _history(rows, 96, V, 6)
    hd, hld = torch.from_numpy(h).to(dev), torch.from_numpy(hl).to(dev)
    nbytes = Sampler.shard_partial_bytes(rows, V, world, params)
    full = torch.empty(world * nbytes, dtype=torch.uint8, device=dev)
    for g in range(world):
        lo, n = sharding.vocab_range(V, world, g)
        sampler.shard_partials(x[:, lo:lo + n], lo, V, world, params,
                               full[g * nbytes:(g + 1) * nbytes], hd, hld)
    st_sh = states_to_tensor(_states(range(rows)), dev)
    ids_sh = torch.full((rows,), -7, dtype=torch.int32, device=dev)
    covered = np.zeros(rows, dtype=bool)
    for o in range(world):
        r0, n = Sampler.shard_owner_rows(rows, world, o)
        assert not covered[r0:r0 + n].any()
        covered[r0:r0 + n] = True
        owner_buf = torch.full((world * nbytes,), 0xA5, dtype=torch.uint8, device=dev)
        for off, ln in Sampler.shard_row_spans(rows, V, world, params, r0, n):
            assert 0 <= off and off + ln <= nbytes
            for g in range(world):
                owner_buf[g * nbytes + off:g * nbytes + off + ln] = \
                    full[g * nbytes + off:g * nbytes + off + ln]
        sampler.shard_merge(owner_buf, world, rows, V, params, st_sh, out=ids_sh, rows=(r0, n))
    assert covered.all()
    sampler.check_device_status()
    st_one = states_to_tensor(_states(range(rows)), dev)
    one = sampler.sample(x, params, st_one, hd, hld, sync_check=True)
    assert np.array_equal(ids_sh.cpu().numpy(), one.ids.cpu().numpy())
    assert np.array_equal(tensor_to_states(st_sh), tensor_to_states(st_one))


def test_argmax_entry(sampler):
    import torch
    rows, n = 16, 10007
    rng = np.random.default_rng(4)
    x = (np.round(rng.normal(0, 1, size=(rows, n)) * 2) / 2).astype(np.float32)
    x[0, 0] = np.nan
    x[1, 5] = np.nan
    x[2, 9] = np.inf
    x[3, :] = -np.inf
    got = sampler.argmax(torch.from_numpy(x).to(sampler.device)).cpu().numpy()
    want = [oracle.oracle_argmax(r) for r in x]
    assert list(got) == want
    if oracle.have_reference():
        assert want == [oracle.reference_argmax(r) for r in x]


def test_host_row_api(sampler):
    """argmax_token / sample_token of the reference's one-row host API."""
    x = W.generate(2, 3, row0=2000)
    for r in range(3):
        rng = Rng(100 + r)
        st = np.array([rng.state], dtype=np.uint64)
        p = SamplingParams(temp=0.7, top_k=40, top_p=0.9, repeat_penalty=1.2)
        hist = [5, 17, int(np.argmax(x[r])), 5]
        got = sample_token(x[r], None, p, hist, rng)
        oid, *_ = oracle.oracle_sample(x[r: r + 1], p, st, np.array([hist], np.int32),
                                       np.array([len(hist)], np.int32))
        assert got == int(oid[0]) and rng.state == int(st[0])


CPP_DRIVER = r"""
#include <cstdio>
#include <vector>
#include "zen/sample.h"
int main(int argc, char** argv) {
    int rows = 0, n = 0;
    FILE* f = std::fopen(argv[1], "rb");
    if (!f || std::fread(&rows, 4, 1, f) != 1 || std::fread(&n, 4, 1, f) != 1) return 2;
    std::vector<float> x((size_t)rows * n);
    if (std::fread(x.data(), 4, x.size(), f) != x.size()) return 2;
    std::fclose(f);
    zen::SamplingParams sp;
    sp.temp = 0.7f;
    sp.top_k = 40;
    sp.top_p = 0.9f;
    sp.repeat_penalty = 1.1f;
    std::vector<int32_t> history = {3, 9, 27};
    for (int r = 0; r < rows; ++r) {
        zen::Rng rng(1000 + r);
        int id = zen::sample_token(x.data() + (size_t)r * n, n, sp, history, rng);
        int g = zen::argmax_token(x.data() + (size_t)r * n, n);
        std::printf("%d %d %llu\n", id, g, (unsigned long long)rng.state());
    }
    return 0;
}
"""


def test_cpp_api_on_device(sampler, tmp_path):
    """The drop-in zen/sample.h API from C++ (one host row per call)."""
    from zeninfer_b200 import _native
    rows = 4
    x = W.generate(2, rows, row0=3000)
    data = tmp_path / "rows.bin"
    with open(data, "wb") as f:
        f.write(np.array([rows, V], np.int32).tobytes())
        f.write(x.tobytes())
    src = tmp_path / "drv.cpp"
    src.write_text(CPP_DRIVER)
    exe = tmp_path / "drv"
    libdir = os.path.dirname(_native.SAMPLER_SO)
    subprocess.run(["g++", "-std=c++17", "-O1", f"-I{ROOT}/include", str(src), "-o", str(exe),
                    f"-L{libdir}", "-lzs_sampler", f"-Wl,-rpath,{libdir}"], check=True)
    out = subprocess.run([str(exe), str(data)], capture_output=True, text=True, check=True).stdout
    p = SamplingParams(temp=0.7, top_k=40, top_p=0.9, repeat_penalty=1.1)
    hist = np.array([[3, 9, 27]] * rows, np.int32)
    st = _states(range(1000, 1000 + rows))
    oids, *_ = oracle.oracle_sample(x, p, st, hist, np.full(rows, 3, np.int32))
    for r, line in enumerate(out.strip().split("\n")):
        id_, g, s = line.split()
        assert int(id_) == oids[r] and int(s) == int(st[r])
        assert int(g) == oracle.oracle_argmax(x[r])


@pytest.mark.parametrize("topn", [1, 8, 50, 1024])
def test_logits_stats(sampler, topn):
    """The `logits` command's display numbers on the device against the restatement."""
    import torch
    rows = 6
    x = np.concatenate([W.generate(2, 3, row0=70), W.generate(4, 3, row0=70)])  # ties in 3..5
    x[1, 9] = np.nan
    x[2, :] = -np.inf
    g = sampler.logits_stats(torch.from_numpy(x).to(sampler.device), topn)
    o = oracle.oracle_logits_stats(x, topn)
    np.testing.assert_array_equal(g["min"].cpu().numpy(), o["min"])
    np.testing.assert_array_equal(g["max"].cpu().numpy(), o["max"])
    np.testing.assert_allclose(g["z"].cpu().numpy(), o["z"], rtol=1e-12, equal_nan=True)
    ids = g["top_ids"].cpu().numpy()
    live = [0, 1, 3, 4, 5]  # row 2 has no finite value: its top is any order of -inf ties
    np.testing.assert_array_equal(ids[live], o["top_ids"][live])
    np.testing.assert_allclose(g["top_p"].cpu().numpy()[live], o["top_p"][live], rtol=1e-12)


def test_logits_stats_short_rows(sampler):
    import torch
    rng = np.random.default_rng(12)
    for n, pad in ((1, 0), (5, 3), (17000, 1), (40000, 2)):
        xf = rng.normal(0, 1, size=(3, n + pad)).astype(np.float32)
        xd = torch.from_numpy(xf).to(sampler.device)[:, :n]
        g = sampler.logits_stats(xd, 10)
        o = oracle.oracle_logits_stats(np.ascontiguousarray(xf[:, :n]), 10)
        np.testing.assert_array_equal(g["top_ids"].cpu().numpy(), o["top_ids"])
        np.testing.assert_allclose(g["z"].cpu().numpy(), o["z"], rtol=1e-12)


def test_device_wait_timeout_is_reported(sampler):
    """A device wait that runs out (a barrier nothing completes) is reported as
    ZS_ERR_DEVICE_TIMEOUT by the next status check, the flag is then cleared, and
    the context keeps working."""
    import ctypes as C
    import torch
    from zeninfer_b200 import _native
    L = _native.lib()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert L.zs_selftest_wait_timeout(sampler._h, stream) == 0
    assert L.zs_check_device_status(sampler._h, stream) == 4  # ZS_ERR_DEVICE_TIMEOUT
    assert b"bounded wait" in L.zs_last_error()
    assert L.zs_check_device_status(sampler._h, stream) == 0  # cleared
    x = W.generate(2, 8, row0=123)
    p = SamplingParams(temp=0.7, top_k=40, top_p=0.9)
    st = _states(range(8))
    compare(run_gpu(sampler, x, p, st), run_oracle(x, p, st))


def test_full_vocab_top_p_against_reference(sampler):
    """The nucleus over the whole 151,936-token vocabulary (top_k = n): device ids
    against the unchanged reference on workload 3 rows (log-rank logits, nucleus of
    tens of thousands of tokens), and the nucleus sizes against the restatement."""
    rows = 6
    x = W.generate(3, rows, row0=500)
    p = SamplingParams(temp=1.0, top_k=2 ** 31 - 1, top_p=0.95)
    seeds = np.arange(rows, dtype=np.uint64) + np.uint64(900)
    g = run_gpu(sampler, x, p, _states(seeds))
    o = run_oracle(x, p, _states(seeds))
    compare(g, o, check_cands=False)
    assert (o["info"]["m"] > 10000).all()
    ref, _ = oracle.reference_sample(x, p, seeds)
    near = o["info"]["boundary"] < BOUNDARY_EPS
    assert np.array_equal(g["ids"][~near], ref[~near])


@pytest.mark.parametrize("k", [3000, V])
def test_large_top_k_ties(sampler, k):
    """The large-shortlist path on heavily tied rows (workload 4: values on a 0.125
    grid): the shortlist order among equal values (id ascending) is the sort's
    stability, checked entry by entry against the restatement."""
    rows = 6
    x = W.generate(4, rows, row0=31)
    p = SamplingParams(temp=0.8, top_k=k, top_p=0.9)
    st = _states(range(rows))
    compare(run_gpu(sampler, x, p, st, cand_ld=6000), run_oracle(x, p, st, cand_ld=6000))
