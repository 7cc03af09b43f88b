"""zs_sample_noalloc (fixed static scratch, no allocation) against zs_sample.

Collected last on purpose (file name): it must pass both alone in a fresh
process and after every other test has used the allocating entry point.
Both entry points are called through the C ABI, twice in a row from the same
rng states, so the second call also checks the advanced states.
"""

import ctypes as C

import numpy as np
import pytest

from zeninfer_b200 import SamplingParams, rng_seed, states_to_tensor, tensor_to_states
from zeninfer_b200 import _native
from zeninfer_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _noalloc(x, params, states, out, status, history=None, history_len=None):
    import torch
    L = _native.lib()
    prm = params.to_c()
    hist_ptr = history.data_ptr() if history is not None else None
    hist_ld = history.shape[1] if history is not None else 0
    hl_ptr = history_len.data_ptr() if history_len is not None else None
    s = L.zs_sample_noalloc(x.data_ptr(), x.stride(0), x.shape[0], x.shape[1], C.byref(prm),
                            hist_ptr, hist_ld, hl_ptr, states.data_ptr(), out.data_ptr(),
                            status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    return s


def _two_calls_each(sampler, x, params, seeds, history=None, history_len=None):
    import torch
    dev = sampler.device
    st_ref = states_to_tensor(np.array([rng_seed(int(s)) for s in seeds], dtype=np.uint64), dev)
    st_na = st_ref.clone()
    ref_ids, na_ids = [], []
    for _ in range(2):
        res = sampler.sample(x, params, st_ref, history, history_len, sync_check=True)
        ref_ids.append(res.ids.cpu().numpy())
    out = torch.empty(x.shape[0], dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    free0 = None
    for i in range(2):
        if i == 1:
            free0 = torch.cuda.mem_get_info(dev)[0]
        s = _noalloc(x, params, st_na, out, status, history, history_len)
        _native.check(s, "zs_sample_noalloc")
        torch.cuda.synchronize()
        na_ids.append(out.cpu().numpy().copy())
    free1 = torch.cuda.mem_get_info(dev)[0]
    assert free1 == free0, "device memory changed across a zs_sample_noalloc call"
    assert int(status.item()) == 0, "a kernel reported a device timeout"
    for i in range(2):
        assert np.array_equal(ref_ids[i], na_ids[i]), f"ids differ on call {i}"
    assert np.array_equal(tensor_to_states(st_ref), tensor_to_states(st_na)), "rng states differ"


@pytest.mark.parametrize("cfg,rows,params", [
    (5, 4096, W.WORKLOADS[5].params),                       # the benchmark batch, top-k 50
    (2, 256, SamplingParams(temp=1.0, top_p=0.95)),         # default shortlist, split rows
    (3, 1, SamplingParams(temp=0.8, top_k=1024)),           # one row, many slices
    (4, 700, SamplingParams(temp=0.9, top_k=1024, top_p=0.9)),  # fewer slices than zs_sample
    (1, 64, SamplingParams()),                              # greedy
])
def test_noalloc_matches_sample(sampler, cfg, rows, params):
    import torch
    x = torch.from_numpy(W.generate(cfg, rows)).to(sampler.device)
    _two_calls_each(sampler, x, params, range(rows))


def test_noalloc_penalty(sampler):
    import torch
    rows = 128
    dev = sampler.device
    x = torch.from_numpy(W.generate(2, rows, row0=5)).to(dev)
    rng = np.random.default_rng(3)
    hist = torch.from_numpy(rng.integers(0, W.VOCAB, size=(rows, 96), dtype=np.int32)).to(dev)
    hl = torch.from_numpy(rng.integers(0, 97, size=rows, dtype=np.int32)).to(dev)
    p = SamplingParams(temp=0.7, top_k=40, top_p=0.9, repeat_penalty=1.3, repeat_last_n=64)
    _two_calls_each(sampler, x, p, range(rows), hist, hl)


def test_noalloc_rejects_oversized_batch(sampler):
    import torch
    rows = 4096  # top_k 1024 at one slice per row needs about 50 MB of scratch
    dev = sampler.device
    x = torch.randn((rows, W.VOCAB), dtype=torch.float32, device=dev)
    st = torch.zeros(rows, dtype=torch.int64, device=dev)
    out = torch.empty(rows, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    L = _native.lib()
    prm = SamplingParams(temp=0.8, top_k=1024).to_c()
    s = L.zs_sample_noalloc(x.data_ptr(), x.stride(0), rows, W.VOCAB, C.byref(prm), None, 0, None,
                            st.data_ptr(), out.data_ptr(), status.data_ptr(),
                            torch.cuda.current_stream().cuda_stream)
    assert s == 1  # ZS_ERR_INVALID_ARGUMENT, before any launch
    assert b"fixed scratch" in L.zs_last_error()


@pytest.mark.parametrize("top_k,limit", [(1024, 2072), (256, 14208)])
def test_noalloc_stated_limits(sampler, top_k, limit):
    """The largest batches include/zs_sampler.h states for the fixed scratch (no
    penalty, 151,936 columns): `limit` rows run, `limit + 1` are rejected before any
    launch."""
    import torch
    dev = sampler.device
    x = torch.randn((limit + 1, W.VOCAB), dtype=torch.float32, device=dev)
    st = states_to_tensor(np.array([rng_seed(i) for i in range(limit + 1)], dtype=np.uint64), dev)
    out = torch.empty(limit + 1, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    L = _native.lib()
    prm = SamplingParams(temp=0.8, top_k=top_k).to_c()
    stream = torch.cuda.current_stream().cuda_stream
    s = L.zs_sample_noalloc(x.data_ptr(), x.stride(0), limit, W.VOCAB, C.byref(prm), None, 0,
                            None, st.data_ptr(), out.data_ptr(), status.data_ptr(), stream)
    assert s == 0, L.zs_last_error()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    s = L.zs_sample_noalloc(x.data_ptr(), x.stride(0), limit + 1, W.VOCAB, C.byref(prm), None,
                            0, None, st.data_ptr(), out.data_ptr(), status.data_ptr(), stream)
    assert s == 1 and b"fixed scratch" in L.zs_last_error()
    del x
