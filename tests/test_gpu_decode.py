"""The device-resident generate loop (zs_decode_step) against the restatement of
cmd_generate's loop (src/main.cpp:626-632): per step every running row samples
with its generated history, a row that draws eos stops without appending it, and
stopped rows draw nothing.  Full vocabulary; the history buffer is shorter than
the run, so the keep-the-penalty-window shift is exercised."""

import numpy as np
import pytest

import oracle
from tests.gpu_util import BOUNDARY_EPS
from zeninfer_b200 import SamplingParams, rng_seed, states_to_tensor, tensor_to_states
from zeninfer_b200._native import SamplerError
from zeninfer_b200 import workloads as W

pytestmark = pytest.mark.gpu

EOS = 151645  # tokenizer.ggml.eos_token_id default of cmd_generate


def _case(B, T, seed_row0=0):
    steps = []
    for t in range(T):
        x = W.generate(2, B, row0=seed_row0 + t * B)
        x[:, 1000:1004] += 7.0  # a few ids dominate, so repeats and the penalty matter
        steps.append(x)
    planted = {(3, 2), (7, 0), (12, 9), (20, T - 1)}
    planted = {(r, t) for r, t in planted if r < B and t < T}
    for r, t in planted:
        steps[t][r, EOS] = 80.0
    return steps, planted


def _params(B):
    out = []
    for r in range(B):
        if r % 5 == 0:
            out.append(SamplingParams(temp=0.0, repeat_penalty=1.5, repeat_last_n=4))
        elif r % 5 == 1:
            out.append(SamplingParams(temp=0.9))
        else:
            out.append(SamplingParams(temp=0.7, top_k=40, top_p=0.9, repeat_penalty=1.3,
                                      repeat_last_n=6))
    return out


def _run_device(sampler, steps, params, seeds, hist_ld):
    import torch
    dev = sampler.device
    B, T = steps[0].shape[0], len(steps)
    rng = states_to_tensor([rng_seed(int(s)) for s in seeds], dev)
    done = torch.zeros(B, dtype=torch.int32, device=dev)
    hist = torch.zeros((B, hist_ld), dtype=torch.int32, device=dev) if hist_ld else None
    hlen = torch.zeros(B, dtype=torch.int32, device=dev) if hist_ld else None
    tokens = torch.full((B, T), -2, dtype=torch.int32, device=dev)
    for t in range(T):
        x = torch.from_numpy(steps[t]).to(dev)
        sampler.decode_step(x, params, rng, done, EOS, hist, hlen, tokens=tokens, step=t)
    torch.cuda.synchronize()
    out = {"tokens": tokens.cpu().numpy(), "done": done.cpu().numpy().astype(bool),
           "rng": tensor_to_states(rng)}
    if hist_ld:
        out["hist"] = hist.cpu().numpy()
        out["hlen"] = hlen.cpu().numpy()
    return out


def _check(dev, o, states, hist_ld):
    B, T = o["tokens"].shape
    diverged = 0
    for r in range(B):
        # a draw within BOUNDARY_EPS of a CDF boundary may legitimately differ; the
        # row's later steps then follow another history, so compare up to there
        near = np.flatnonzero(o["boundary"][r] < BOUNDARY_EPS)
        upto = T if near.size == 0 else int(near[0])
        if upto < T:
            diverged += 1
        assert np.array_equal(dev["tokens"][r, :upto], o["tokens"][r, :upto]), r
        if upto < T:
            continue
        assert dev["done"][r] == o["done"][r], r
        assert int(dev["rng"][r]) == int(states[r]), r
        if hist_ld:
            n = int(dev["hlen"][r])
            gen = o["gen"][r]
            assert n <= hist_ld and n <= len(gen), r
            assert dev["hist"][r, :n].tolist() == gen[len(gen) - n:], r
            if len(gen) < hist_ld:
                assert n == len(gen), r
    assert diverged <= max(1, B // 16)


def test_decode_loop_matches_generate_loop(sampler):
    B, T, hist_ld = 32, 16, 8
    steps, planted = _case(B, T)
    params = _params(B)
    seeds = np.arange(B, dtype=np.uint64) + np.uint64(77)
    dev = _run_device(sampler, steps, params, seeds, hist_ld)
    st = np.array([rng_seed(int(s)) for s in seeds], dtype=np.uint64)
    o = oracle.oracle_generate(steps, params, st, EOS)
    _check(dev, o, st, hist_ld)
    for r, t in planted:
        if t == 0 or o["boundary"][r, :t].min() >= BOUNDARY_EPS:
            assert dev["done"][r] and dev["tokens"][r, t] == EOS
            assert (dev["tokens"][r, t + 1:] == -1).all()


@pytest.mark.parametrize("B", [1, 4, 8])
def test_decode_loop_small_batches(sampler, B):
    """Decode-sized batches (the one-launch cluster path, penalised rows included)
    against the generate loop's restatement."""
    T, hist_ld = 12, 8
    steps, planted = _case(B, T, seed_row0=900)
    params = _params(B)
    seeds = np.arange(B, dtype=np.uint64) + np.uint64(5)
    dev = _run_device(sampler, steps, params, seeds, hist_ld)
    st = np.array([rng_seed(int(s)) for s in seeds], dtype=np.uint64)
    o = oracle.oracle_generate(steps, params, st, EOS)
    _check(dev, o, st, hist_ld)


def test_decode_loop_shared_params_no_history(sampler):
    B, T = 48, 6
    steps, _ = _case(B, T, seed_row0=5000)
    p = SamplingParams(temp=0.8, top_k=50, top_p=0.95)
    seeds = np.arange(B, dtype=np.uint64) * np.uint64(3) + np.uint64(1)
    dev = _run_device(sampler, steps, p, seeds, 0)
    st = np.array([rng_seed(int(s)) for s in seeds], dtype=np.uint64)
    o = oracle.oracle_generate(steps, p, st, EOS)
    _check(dev, o, st, 0)


def test_decode_step_rejects_short_history(sampler):
    import torch
    dev = sampler.device
    x = torch.zeros((2, 1000), dtype=torch.float32, device=dev)
    rng = torch.ones(2, dtype=torch.int64, device=dev)
    done = torch.zeros(2, dtype=torch.int32, device=dev)
    hist = torch.zeros((2, 6), dtype=torch.int32, device=dev)
    hlen = torch.zeros(2, dtype=torch.int32, device=dev)
    with pytest.raises(SamplerError):
        sampler.decode_step(x, SamplingParams(temp=0.7, repeat_penalty=1.2, repeat_last_n=6),
                            rng, done, 999999, hist, hlen)
    # without a penalty the history length does not matter
    sampler.decode_step(x, SamplingParams(temp=0.7, repeat_last_n=6), rng, done, 999999, hist, hlen)
    torch.cuda.synchronize()
    assert hlen.cpu().tolist() == [1, 1]


def test_decode_steps_in_a_cuda_graph(sampler):
    """Six steps of zs_decode_step captured once in a CUDA graph (after one eager
    call has sized the handle's scratch) and replayed give the tokens, stop flags,
    Rng states and histories of the same steps run eagerly."""
    import torch
    dev = sampler.device
    B, T, hist_ld = 16, 6, 16
    steps, _ = _case(B, T, seed_row0=7000)
    p = SamplingParams(temp=0.7, top_k=40, top_p=0.9, repeat_penalty=1.2, repeat_last_n=8)
    seeds = np.arange(B, dtype=np.uint64) + np.uint64(55)
    xs = [torch.from_numpy(x).to(dev) for x in steps]

    def fresh():
        return {"rng": states_to_tensor([rng_seed(int(s)) for s in seeds], dev),
                "done": torch.zeros(B, dtype=torch.int32, device=dev),
                "hist": torch.zeros((B, hist_ld), dtype=torch.int32, device=dev),
                "hlen": torch.zeros(B, dtype=torch.int32, device=dev),
                "tok": torch.full((B, T), -2, dtype=torch.int32, device=dev)}

    def run(st):
        for t in range(T):
            sampler.decode_step(xs[t], p, st["rng"], st["done"], EOS, st["hist"], st["hlen"],
                                tokens=st["tok"], step=t)

    eager = fresh()
    run(eager)
    warm = fresh()
    sampler.decode_step(xs[0], p, warm["rng"], warm["done"], EOS, warm["hist"], warm["hlen"],
                        tokens=warm["tok"], step=0)
    torch.cuda.synchronize()
    cap = fresh()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run(cap)
    graph.replay()
    torch.cuda.synchronize()
    sampler.check_device_status()
    for k in ("tok", "done", "hist", "hlen"):
        assert torch.equal(cap[k], eager[k]), k
    assert np.array_equal(tensor_to_states(cap["rng"]), tensor_to_states(eager["rng"]))
