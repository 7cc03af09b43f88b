"""The exact lm_head route's summation order, simulated on the CPU (no device code runs).

zs_lm_exact_kernel (zeninfer_b200/csrc/zs_lmhead.cuh) computes a logit on 8 lanes of a
warp: lane p holds the reference's accumulators 4p .. 4p + 3 (accumulator l takes
w[i] * xn[i] for i = l, l + 32, ... by fused multiply-add, in order), then adds lanes
2 apart, 4 apart and 1 apart with shuffles, then [0] + [2], [1] + [3] and those two,
then the columns past the last multiple of 32 in double.  This test replays exactly
those steps (float32 roundings, fused multiply-adds through the C library's fmaf) and
checks them bit for bit against the oracle's restatement of the reference's AVX2 dot
product (src/kernels.cpp:52-78, zo_dot_avx2_order), itself pinned to the reference in
tests/test_oracle.py."""

import ctypes as C
import ctypes.util

import numpy as np
import pytest

import oracle

_libm = C.CDLL(ctypes.util.find_library("m"))
_libm.fmaf.argtypes = [C.c_float, C.c_float, C.c_float]
_libm.fmaf.restype = C.c_float
f32 = np.float32


def _fmaf(a, b, c):
    return f32(_libm.fmaf(float(a), float(b), float(c)))


def _warp_dot(w, x):
    """The kernel's steps for one logit (w, x float32 of length E)."""
    E = len(w)
    n32 = E & ~31
    acc = [[f32(0.0)] * 4 for _ in range(8)]  # acc[p][c]: lane p, accumulator 4p + c
    for blk in range(0, n32, 32):
        for p in range(8):
            for c in range(4):
                i = blk + 4 * p + c
                acc[p][c] = _fmaf(w[i], x[i], acc[p][c])
    v = [[acc[p][c] for c in range(4)] for p in range(8)]
    for d in (2, 4, 1):  # __shfl_down_sync by 2, 4, 1 within the row's 8 lanes
        v = [[f32(v[p][c] + v[p + d][c]) if p + d < 8 else v[p][c] for c in range(4)]
             for p in range(8)]
    t20 = f32(v[0][0] + v[0][2])
    t21 = f32(v[0][1] + v[0][3])
    t3 = f32(t20 + t21)
    total = float(t3)
    for i in range(n32, E):  # the tail in double (products of floats are exact)
        total = total + float(w[i]) * float(x[i])
    return f32(total)


@pytest.mark.parametrize("E", [896, 200, 64, 40])
def test_exact_route_order_matches_avx2_restatement(E):
    lib = oracle.olib()
    lib.zo_dot_avx2_order.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
    lib.zo_dot_avx2_order.restype = C.c_float
    rng = np.random.default_rng(E)
    for trial in range(6):
        w = oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(
            rng.normal(0, 0.05, size=E).astype(np.float32)))
        x = (rng.normal(0, 1.0, size=E) * (10.0 ** rng.integers(-3, 3))).astype(np.float32)
        if trial == 5:  # cancellation-heavy: the order of additions shows
            x[::2] *= f32(1e4)
        want = f32(lib.zo_dot_avx2_order(w.ctypes.data, x.ctypes.data, E))
        got = _warp_dot(w, x)
        assert np.array_equal(np.array([got]).view(np.uint32), np.array([want]).view(np.uint32)), (E, trial)
