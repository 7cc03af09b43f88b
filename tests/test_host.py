"""Host-side logic on CPU: the Rng, parameter and state marshalling, the
synthetic workload generator, and the multi-GPU layouts."""

import ctypes as C

import numpy as np
import pytest

import oracle
from zeninfer_b200 import (Rng, SamplingParams, _native, rng_seed, states_to_tensor,
                           tensor_to_states)
from zeninfer_b200 import sharding
from zeninfer_b200 import workloads as W


def test_rng_matches_oracle():
    rng = np.random.default_rng(0)
    for seed in [0, 1, 42] + [int(v) for v in rng.integers(0, 2**63, size=20, dtype=np.int64)]:
        r = Rng(seed)
        st = np.array([rng_seed(seed)], dtype=np.uint64)
        for _ in range(5):
            u = oracle.olib().zo_rng_uniform(st.ctypes.data_as(C.POINTER(C.c_uint64)))
            assert r.uniform() == u
            assert r.state == int(st[0])


def test_params_layout():
    assert C.sizeof(_native.ZsParams) == 20 == oracle.PARAMS_DTYPE.itemsize
    p = SamplingParams(temp=0.5, top_k=7, top_p=0.25, repeat_penalty=1.5, repeat_last_n=9).to_c()
    assert (p.temp, p.top_k, p.top_p, p.repeat_penalty, p.repeat_last_n) == (0.5, 7, 0.25, 1.5, 9)
    d = SamplingParams()
    assert (d.temp, d.top_k, d.top_p, d.repeat_penalty, d.repeat_last_n) == (0.0, 0, 1.0, 1.0, 64)
    assert C.sizeof(_native.ZsRowInfo) == 48
    assert C.sizeof(_native.ZsExtras) == 32


def test_states_roundtrip():
    s = np.array([0, 1, 2**63, 2**64 - 1, 0x9E3779B97F4A7C15], dtype=np.uint64)
    t = states_to_tensor(s, "cpu")
    assert str(t.dtype) == "torch.int64"
    assert np.array_equal(tensor_to_states(t), s)


def test_workload_generator_is_deterministic_and_row_addressed():
    for cfg in (1, 2, 3, 4, 5):
        a = W.generate(cfg, 6, V=4096)
        b = W.generate(cfg, 4, row0=2, V=4096, nthreads=1)
        assert np.array_equal(a[2:], b)
        assert np.isfinite(a).all()
    c4 = W.generate(4, 2, V=4096)
    assert np.array_equal(np.round(c4 * 8) / 8, c4)  # quantised workload: heavy ties


def test_workload_seeds():
    assert list(W.WORKLOADS[1].row_seeds(0, 1)) == [42]
    assert list(W.WORKLOADS[5].row_seeds(10, 3)) == [10, 11, 12]


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_row_and_vocab_ranges(world):
    for batch in (0, 1, 7, 4096):
        got = [sharding.row_range(batch, world, g) for g in range(world)]
        assert sum(c for _, c in got) == batch
        assert all(got[g][0] + got[g][1] == got[g + 1][0] for g in range(world - 1))
        assert max(c for _, c in got) - min(c for _, c in got) <= 1
    for V in (151936, 1000, 9):
        if V < world:
            continue
        got = [sharding.vocab_range(V, world, g) for g in range(world)]
        assert got[0][0] == 0 and got[-1][0] + got[-1][1] == V
        assert all(got[g][0] + got[g][1] == got[g + 1][0] for g in range(world - 1))
    assert sharding.vocab_range(151936, 8, 7) == (7 * 18992, 18992)


def test_logits_file_roundtrip(tmp_path):
    from zeninfer_b200 import logits_io
    x = np.random.default_rng(1).normal(0, 1, size=(3, 1000)).astype(np.float32)
    p = str(tmp_path / "l.bin")
    logits_io.write_logits(p, x)
    assert (tmp_path / "l.bin").stat().st_size == x.size * 4  # raw <f4, no header
    y = logits_io.read_logits(p, n_vocab=1000)
    assert y.shape == (3, 1000) and np.array_equal(np.asarray(y), x)
    with pytest.raises(ValueError):
        logits_io.read_logits(p, n_vocab=999)
