"""Checkers for the B200 sampler -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this package.  The product (zeninfer_b200/) never does.

    restatement   liboracle.so        C restatement of src/sample.cpp with a total
                                      shortlist order (value desc, id asc); exposes
                                      the shortlist, p_i, m, r, boundary distance
    reference     _ref/libzen_ref.so  the reference's src/sample.cpp compiled
                                      unchanged, with a row-loop harness

Both are built by oracle/Makefile (`make -C oracle`).
"""

from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libzen_ref.so")

ROW_INFO_DTYPE = np.dtype([("max_logit", "<f4"), ("k", "<i4"), ("m", "<i4"), ("pos", "<i4"),
                           ("r", "<f8"), ("sum", "<f8"), ("boundary", "<f8"), ("log_z", "<f8")])

PARAMS_DTYPE = np.dtype([("temp", "<f4"), ("top_k", "<i4"), ("top_p", "<f4"),
                         ("repeat_penalty", "<f4"), ("repeat_last_n", "<i4")])


def params_array(params, batch=None) -> np.ndarray:
    """SamplingParams-like object(s) (or a PARAMS_DTYPE array) -> PARAMS_DTYPE array."""
    if isinstance(params, np.ndarray) and params.dtype == PARAMS_DTYPE:
        return np.ascontiguousarray(params)
    if not isinstance(params, (list, tuple)):
        params = [params]
    arr = np.zeros(len(params), dtype=PARAMS_DTYPE)
    for i, p in enumerate(params):
        arr[i] = (p.temp, p.top_k, p.top_p, p.repeat_penalty, p.repeat_last_n)
    return arr


_olib = None
_rlib = None


def _ptr(a):
    return None if a is None else a.ctypes.data


def olib():
    global _olib
    if _olib is None:
        if not os.path.exists(ORACLE_SO):
            raise RuntimeError(f"{ORACLE_SO} missing; run make -C oracle")
        L = C.CDLL(ORACLE_SO)
        vp = C.c_void_p
        L.zo_sample_rows.argtypes = [vp, C.c_int64, C.c_int, C.c_int, vp, C.c_int, vp, C.c_int64,
                                     vp, vp, vp, vp, vp, vp, C.c_int, vp, C.c_int, C.c_int]
        L.zo_sample_rows.restype = C.c_int
        L.zo_argmax.argtypes = [vp, C.c_int]
        L.zo_argmax.restype = C.c_int32
        L.zo_rng_seed.argtypes = [C.c_uint64]
        L.zo_rng_seed.restype = C.c_uint64
        L.zo_rng_uniform.argtypes = [C.POINTER(C.c_uint64)]
        L.zo_rng_uniform.restype = C.c_double
        L.zo_logits_stats.argtypes = [vp, C.c_int64, C.c_int, C.c_int, C.c_int, vp, vp, vp, vp,
                                      vp, C.c_int64]
        L.zo_logits_stats.restype = C.c_int
        L.zo_lmhead_rows.argtypes = [vp, C.c_int64, C.c_int, C.c_int, vp, C.c_float, vp, C.c_int,
                                     vp, vp, C.c_int64, C.c_int]
        L.zo_lmhead_rows.restype = C.c_int
        L.zo_lmhead_f32_rows.argtypes = [vp, C.c_int64, C.c_int, C.c_int, vp, C.c_float, vp,
                                         C.c_int, vp, vp, C.c_int64]
        L.zo_lmhead_f32_rows.restype = C.c_int
        _olib = L
    return _olib


def rlib():
    global _rlib
    if _rlib is None:
        if not os.path.exists(REF_SO):
            raise RuntimeError(f"{REF_SO} missing; run make -C oracle ref (needs the reference)")
        L = C.CDLL(REF_SO)
        vp = C.c_void_p
        L.zref_sample_rows.argtypes = [vp, C.c_int64, C.c_int, C.c_int, vp, C.c_int, vp, C.c_int64,
                                       vp, vp, vp, vp, C.c_int]
        L.zref_sample_rows.restype = C.c_int
        L.zref_argmax.argtypes = [vp, C.c_int]
        L.zref_argmax.restype = C.c_int32
        L.zref_rng_stream.argtypes = [C.c_uint64, C.c_int, vp, vp]
        L.zref_rng_stream.restype = None
        L.zref_lmhead_rows.argtypes = [vp, C.c_int64, C.c_int, C.c_int, vp, C.c_float, vp, C.c_int,
                                       vp, vp, C.c_int64, C.c_int, C.c_int]
        L.zref_lmhead_rows.restype = C.c_int
        L.zref_matvec_rows.argtypes = [vp, C.c_int, C.c_int, vp, C.c_int, vp, C.c_int64, C.c_int,
                                       C.c_int]
        L.zref_matvec_rows.restype = C.c_int
        _rlib = L
    return _rlib


def have_reference() -> bool:
    return os.path.exists(REF_SO)


def oracle_sample(logits: np.ndarray, params, states: np.ndarray, history=None, history_len=None,
                  cand_ld: int = 0, full_z: bool = False, nthreads: int | None = None):
    """Restatement over rows of `logits` [B, ld] (first n = logits.shape[1] columns
    unless `n` differs).  states: uint64 [B] xorshift64* states, advanced in place.
    Returns (ids int32[B], infos ROW_INFO_DTYPE[B], cand_ids, cand_vals, cand_probs)."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    B, n = logits.shape
    par = params_array(params)
    per_row = 1 if len(par) > 1 else 0
    if per_row and len(par) != B:
        raise ValueError("need one params entry per row")
    ids = np.zeros(B, dtype=np.int32)
    infos = np.zeros(B, dtype=ROW_INFO_DTYPE)
    cid = cv = cp = None
    if cand_ld > 0:
        cid = np.full((B, cand_ld), -1, dtype=np.int32)
        cv = np.zeros((B, cand_ld), dtype=np.float32)
        cp = np.zeros((B, cand_ld), dtype=np.float64)
    h = hl = None
    hld = 0
    if history is not None:
        h = np.ascontiguousarray(history, dtype=np.int32)
        hl = np.ascontiguousarray(history_len, dtype=np.int32)
        hld = h.shape[1]
    assert states.dtype == np.uint64 and states.flags["C_CONTIGUOUS"]
    nthreads = nthreads or min(64, os.cpu_count() or 1)
    olib().zo_sample_rows(logits.ctypes.data, n, B, n, par.ctypes.data, per_row, _ptr(h), hld,
                          _ptr(hl), states.ctypes.data, ids.ctypes.data, _ptr(cid), _ptr(cv),
                          _ptr(cp), cand_ld, infos.ctypes.data, 1 if full_z else 0, nthreads)
    return ids, infos, cid, cv, cp


def oracle_generate(step_logits, params, states: np.ndarray, eos: int):
    """cmd_generate's loop (src/main.cpp:626-632) for B independent sequences over
    precomputed logits, one [B, n] array per step:
        next = sample_token(logits, n, sp, gen, rng); if next == eos: stop;
        gen.push_back(next)
    with gen the row's whole generated history (prompt excluded).  states (uint64
    [B]) are advanced in place.  Returns dict: tokens int32 [B, T] (-1 once stopped),
    gen (list of lists), done bool [B], boundary float64 [B, T] (distance of the
    draw to the nearest CDF boundary; inf for greedy and stopped rows)."""
    T = len(step_logits)
    B = step_logits[0].shape[0]
    par = params_array(params)
    per_row = len(par) > 1
    gen = [[] for _ in range(B)]
    done = np.zeros(B, dtype=bool)
    tokens = np.full((B, T), -1, dtype=np.int32)
    boundary = np.full((B, T), np.inf)
    for t in range(T):
        run = np.flatnonzero(~done)
        if run.size == 0:
            break
        L = max(1, max(len(gen[r]) for r in run))
        h = np.zeros((run.size, L), dtype=np.int32)
        hl = np.zeros(run.size, dtype=np.int32)
        for j, r in enumerate(run):
            h[j, :len(gen[r])] = gen[r]
            hl[j] = len(gen[r])
        st = np.ascontiguousarray(states[run])
        ids, info, _, _, _ = oracle_sample(step_logits[t][run], par[run] if per_row else par, st,
                                           h, hl)
        states[run] = st
        for j, r in enumerate(run):
            tokens[r, t] = ids[j]
            if info["k"][j] > 0:
                boundary[r, t] = info["boundary"][j]
            if ids[j] == eos:
                done[r] = True
            else:
                gen[r].append(int(ids[j]))
    return {"tokens": tokens, "gen": gen, "done": done, "boundary": boundary}


def oracle_lmhead(hidden: np.ndarray, norm_w: np.ndarray, eps: float, w_bf16: np.ndarray,
                  nthreads: int | None = None):
    """The lm_head (src/model.cpp:401-403) as the device computes it: rmsnorm, xn
    rounded to bfloat16, then the reference's in-order double dot products over
    the bfloat16 weights (w_bf16: uint16 [V, E] bit patterns), one float rounding.
    Returns (xn_bf16 uint16 [B, E], logits float32 [B, V])."""
    h = np.ascontiguousarray(hidden, dtype=np.float32)
    B, E = h.shape
    w = np.ascontiguousarray(w_bf16, dtype=np.uint16)
    V = w.shape[0]
    nw = np.ascontiguousarray(norm_w, dtype=np.float32)
    xn = np.zeros((B, E), dtype=np.uint16)
    logits = np.zeros((B, V), dtype=np.float32)
    nthreads = nthreads or min(64, os.cpu_count() or 1)
    olib().zo_lmhead_rows(h.ctypes.data, E, B, E, nw.ctypes.data, float(eps), w.ctypes.data, V,
                          xn.ctypes.data, logits.ctypes.data, V, nthreads)
    return xn, logits


def oracle_lmhead_f32(hidden: np.ndarray, norm_w: np.ndarray, eps: float, w_bf16: np.ndarray):
    """The lm_head as the reference computes it by default (src/model.cpp:401-403 with
    src/kernels.cpp:52-78): rmsnorm to f32, then the AVX2 dot product's summation
    order (32 fused multiply-add accumulators, its reduction tree, the tail in
    double) over the bfloat16 weights (w_bf16: uint16 [V, E] bit patterns).  Returns
    (xn float32 [B, E], logits float32 [B, V])."""
    h = np.ascontiguousarray(hidden, dtype=np.float32)
    B, E = h.shape
    w = np.ascontiguousarray(w_bf16, dtype=np.uint16)
    V = w.shape[0]
    nw = np.ascontiguousarray(norm_w, dtype=np.float32)
    xn = np.zeros((B, E), dtype=np.float32)
    logits = np.zeros((B, V), dtype=np.float32)
    olib().zo_lmhead_f32_rows(h.ctypes.data, E, B, E, nw.ctypes.data, float(eps), w.ctypes.data,
                              V, xn.ctypes.data, logits.ctypes.data, V)
    return xn, logits


def reference_lmhead(hidden: np.ndarray, norm_w: np.ndarray, eps: float, w_f32: np.ndarray,
                     impl: int = 0, nthreads: int | None = None):
    """The unchanged reference: zen::rmsnorm then zen::matvec_f32_impl (impl 0
    scalar, 1 AVX2) per row.  Returns (xn float32 [B, E], logits float32 [B, V])."""
    h = np.ascontiguousarray(hidden, dtype=np.float32)
    B, E = h.shape
    w = np.ascontiguousarray(w_f32, dtype=np.float32)
    V = w.shape[0]
    nw = np.ascontiguousarray(norm_w, dtype=np.float32)
    xn = np.zeros((B, E), dtype=np.float32)
    logits = np.zeros((B, V), dtype=np.float32)
    nthreads = nthreads or min(64, os.cpu_count() or 1)
    rlib().zref_lmhead_rows(h.ctypes.data, E, B, E, nw.ctypes.data, float(eps), w.ctypes.data, V,
                            xn.ctypes.data, logits.ctypes.data, V, impl, nthreads)
    return xn, logits


def reference_matvec(xn: np.ndarray, w_f32: np.ndarray, impl: int = 0,
                     nthreads: int | None = None) -> np.ndarray:
    """zen::matvec_f32_impl over caller-supplied rows xn [B, E]; float32 [B, V]."""
    x = np.ascontiguousarray(xn, dtype=np.float32)
    B, E = x.shape
    w = np.ascontiguousarray(w_f32, dtype=np.float32)
    V = w.shape[0]
    out = np.zeros((B, V), dtype=np.float32)
    nthreads = nthreads or min(64, os.cpu_count() or 1)
    rlib().zref_matvec_rows(x.ctypes.data, B, E, w.ctypes.data, V, out.ctypes.data, V, impl,
                            nthreads)
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round to nearest even (NaN kept quiet)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((u + np.uint32(0x7fff) + ((u >> 16) & np.uint32(1))) >> 16).astype(np.uint16)
    nan = (u & np.uint32(0x7fffffff)) > np.uint32(0x7f800000)
    r[nan] = ((u[nan] >> 16) | np.uint32(0x40)).astype(np.uint16)
    return r


def oracle_logits_stats(logits: np.ndarray, topn: int):
    """The `logits` command's display numbers (src/main.cpp:473-503) per row of
    `logits` [B, n]: dict of min, max, z (float64 [B]), top_ids (int32 [B, k]) and
    top_p (float64 [B, k]), k = clamp(topn, 1, n), top-N in value-desc, id-asc order."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    B, n = x.shape
    k = max(1, min(topn, n))
    out = {"min": np.zeros(B), "max": np.zeros(B), "z": np.zeros(B),
           "top_ids": np.full((B, k), -1, dtype=np.int32), "top_p": np.zeros((B, k))}
    rc = olib().zo_logits_stats(x.ctypes.data, n, B, n, topn, out["min"].ctypes.data,
                                out["max"].ctypes.data, out["z"].ctypes.data,
                                out["top_ids"].ctypes.data, out["top_p"].ctypes.data, k)
    if rc != 0:
        raise ValueError("zo_logits_stats failed")
    return out


def reference_sample(logits: np.ndarray, params, seeds: np.ndarray, history=None,
                     history_len=None, nthreads: int | None = None, ld: int | None = None,
                     n: int | None = None):
    """The unchanged reference, one zen::Rng(seeds[r]) per row.
    Returns (ids int32[B], next_after uint64[B]) -- the Rng's next() after the call."""
    B = logits.shape[0]
    ld = logits.shape[1] if ld is None else ld
    n = logits.shape[1] if n is None else n
    par = params_array(params)
    per_row = 1 if len(par) > 1 else 0
    ids = np.zeros(B, dtype=np.int32)
    nxt = np.zeros(B, dtype=np.uint64)
    seeds = np.ascontiguousarray(seeds, dtype=np.uint64)
    h = hl = None
    hld = 0
    if history is not None:
        h = np.ascontiguousarray(history, dtype=np.int32)
        hl = np.ascontiguousarray(history_len, dtype=np.int32)
        hld = h.shape[1]
    nthreads = nthreads or min(64, os.cpu_count() or 1)
    rlib().zref_sample_rows(logits.ctypes.data, ld, B, n, par.ctypes.data, per_row, _ptr(h), hld,
                            _ptr(hl), seeds.ctypes.data, ids.ctypes.data, nxt.ctypes.data,
                            nthreads)
    return ids, nxt


def reference_argmax(row: np.ndarray, n: int | None = None) -> int:
    row = np.ascontiguousarray(row, dtype=np.float32)
    return int(rlib().zref_argmax(row.ctypes.data, row.size if n is None else n))


def oracle_argmax(row: np.ndarray, n: int | None = None) -> int:
    row = np.ascontiguousarray(row, dtype=np.float32)
    return int(olib().zo_argmax(row.ctypes.data, row.size if n is None else n))


def reference_rng_stream(seed: int, count: int):
    out = np.zeros(count, dtype=np.uint64)
    u = C.c_double()
    rlib().zref_rng_stream(seed, count, out.ctypes.data, C.addressof(u))
    return out, u.value


def build(with_reference: bool | None = None) -> None:
    """make -C oracle: the restatement, and the reference part where its sources
    exist (oracle/Makefile's REF_SRC); with_reference=True requires them."""
    import subprocess
    targets = ["oracle", "ref" if with_reference else "ref-if-present"]
    if with_reference is False:
        targets = ["oracle"]
    r = subprocess.run(["make", "-s", "-C", HERE, *targets], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + r.stdout + r.stderr)
