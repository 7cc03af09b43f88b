"""Python face of the B200 sampler: zeninfer's sample.h API plus a batched
device API, both over the C ABI (include/zs_sampler.h).

Reference interface (namespace zen, src/sample.h):
    SamplingParams           src/sample.h:9-15
    Rng (xorshift64*)        src/sample.h:18-26, src/sample.cpp:15-22
    argmax_token             src/sample.h:28,    src/sample.cpp:24-30
    sample_token             src/sample.h:36-37, src/sample.cpp:32-102

argmax_token / sample_token take one host row, like the reference; Sampler
takes [B, V] CUDA tensors and per-row xorshift64* states, stream-ordered.
Torch provides device memory and streams; all compute is in libzs_sampler.so.
"""

from __future__ import annotations

import ctypes as C
import threading
from dataclasses import dataclass
from typing import Optional, Sequence, Union

import numpy as np

from . import _native

MASK64 = (1 << 64) - 1
RNG_DEFAULT_SEED = 0x9E3779B97F4A7C15

ROW_INFO_DTYPE = np.dtype([("max_logit", "<f4"), ("k", "<i4"), ("m", "<i4"), ("pos", "<i4"),
                           ("r", "<f8"), ("sum", "<f8"), ("boundary", "<f8"), ("log_z", "<f8")])
assert ROW_INFO_DTYPE.itemsize == 48


@dataclass
class SamplingParams:
    """zen::SamplingParams (src/sample.h:9-15), same defaults."""
    temp: float = 0.0            # <= 0 means greedy
    top_k: int = 0               # 0 = disabled (256-token shortlist)
    top_p: float = 1.0           # 1.0 = disabled
    repeat_penalty: float = 1.0  # 1.0 = disabled
    repeat_last_n: int = 64

    def to_c(self) -> _native.ZsParams:
        return _native.ZsParams(self.temp, int(self.top_k), self.top_p, self.repeat_penalty,
                                int(self.repeat_last_n))


class Rng:
    """zen::Rng: xorshift64*, seed 0 replaced by 0x9E3779B97F4A7C15."""

    def __init__(self, seed: int):
        seed &= MASK64
        self.state = seed if seed else RNG_DEFAULT_SEED

    def next(self) -> int:
        s = self.state
        s ^= s >> 12
        s ^= (s << 25) & MASK64
        s ^= s >> 27
        self.state = s
        return (s * 2685821657736338717) & MASK64

    def uniform(self) -> float:
        return float(self.next() >> 11) * (1.0 / 9007199254740992.0)


def rng_seed(seed: int) -> int:
    """State that zen::Rng(seed) starts from."""
    seed &= MASK64
    return seed if seed else RNG_DEFAULT_SEED


def states_to_tensor(states, device):
    """uint64 states -> int64 CUDA tensor holding the same bits."""
    import torch
    arr = np.asarray(states, dtype=np.uint64).view(np.int64)
    return torch.from_numpy(arr.copy()).to(device)


def tensor_to_states(t) -> np.ndarray:
    return t.detach().cpu().numpy().view(np.uint64)


@dataclass
class SampleResult:
    ids: "object"                          # torch int32 [B]
    row_info: Optional[np.ndarray] = None  # ROW_INFO_DTYPE [B] (host)
    cand_ids: Optional["object"] = None    # torch int32 [B, cand_ld]
    cand_probs: Optional["object"] = None  # torch float64 [B, cand_ld]


def _params_array(params, batch):
    if isinstance(params, SamplingParams):
        return (_native.ZsParams * 1)(params.to_c()), 0
    params = list(params)
    if len(params) != batch:
        raise ValueError("need one SamplingParams per row")
    return (_native.ZsParams * batch)(*[p.to_c() for p in params]), 1


def _stream_ptr(stream):
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    return C.c_void_p(stream.cuda_stream)


class Sampler:
    """Batched device sampler bound to one CUDA device (a zs_handle)."""

    def __init__(self, device: Union[int, str, None] = None):
        import torch
        if not torch.cuda.is_available():
            raise RuntimeError("the B200 sampler needs a CUDA device")
        dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                           torch.device(device).index if not isinstance(device, int) else device)
        self.device = dev
        self._lib = _native.lib()
        h = C.c_void_p()
        with torch.cuda.device(dev):
            _native.check(self._lib.zs_create(dev.index, C.byref(h)), "zs_create")
        self._h = h

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            self._lib.zs_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _extras(self, batch, row_info, cand_ld, want_log_z):
        import torch
        ex = _native.ZsExtras()
        info_buf = cand_ids = cand_probs = None
        if row_info or want_log_z:
            info_buf = torch.zeros((batch, 48), dtype=torch.uint8, device=self.device)
            ex.row_info = info_buf.data_ptr()
        if cand_ld > 0:
            cand_ids = torch.full((batch, cand_ld), -1, dtype=torch.int32, device=self.device)
            cand_probs = torch.zeros((batch, cand_ld), dtype=torch.float64, device=self.device)
            ex.cand_ids = cand_ids.data_ptr()
            ex.cand_probs = cand_probs.data_ptr()
            ex.cand_ld = cand_ld
        ex.want_log_z = 1 if want_log_z else 0
        return ex, info_buf, cand_ids, cand_probs

    def sample(self, logits, params, rng_state=None, history=None, history_len=None, out=None,
               row_info=False, cand_ld=0, want_log_z=False, stream=None,
               sync_check=False) -> SampleResult:
        """sample_token over every row of `logits` ([B, V] float32 CUDA, row stride
        may exceed V).  rng_state: int64 CUDA [B] xorshift64* states, advanced in
        place for non-greedy rows.  history: int32 CUDA [B, L] with lengths
        history_len int32 CUDA [B]."""
        import torch
        if logits.dim() == 1:
            logits = logits.unsqueeze(0)
        if logits.dtype != torch.float32 or logits.device != self.device or logits.stride(1) != 1:
            raise ValueError("logits must be float32, unit column stride, on the sampler's device")
        B, V = logits.shape
        par, per_row = _params_array(params, B)
        if out is None:
            out = torch.empty(B, dtype=torch.int32, device=self.device)
        ex, info_buf, cand_ids, cand_probs = self._extras(B, row_info, cand_ld, want_log_z)
        hist_ptr = hist_len_ptr = None
        hist_ld = 0
        if history is not None:
            if history_len is None:
                raise ValueError("history needs history_len")
            history = history.to(torch.int32).contiguous()
            history_len = history_len.to(torch.int32).contiguous()
            hist_ptr, hist_len_ptr = history.data_ptr(), history_len.data_ptr()
            hist_ld = history.shape[1] if history.dim() == 2 else 0
        rng_ptr = rng_state.data_ptr() if rng_state is not None else None
        st = _stream_ptr(stream)
        _native.check(self._lib.zs_sample(self._h, logits.data_ptr(), logits.stride(0), B, V, par,
                                          per_row, hist_ptr, hist_ld, hist_len_ptr, rng_ptr,
                                          out.data_ptr(), C.byref(ex), st), "zs_sample")
        if sync_check:
            _native.check(self._lib.zs_check_device_status(self._h, st), "zs_sample (device)")
        info = None
        if info_buf is not None:
            info = info_buf.cpu().numpy().view(ROW_INFO_DTYPE).reshape(B)
        return SampleResult(out, info, cand_ids, cand_probs)

    def decode_step(self, logits, params, rng_state, done, eos: int, history=None,
                    history_len=None, out=None, tokens=None, step: int = 0, stream=None):
        """One step of the generate loop (src/main.cpp:626-632) on the device: sample
        every running row, stop rows that drew `eos` (not appended), append the
        others' ids to `history` ([B, L] int32 CUDA, lengths `history_len`), keep
        stopped rows' Rng states.  `done` is int32 CUDA [B]; `tokens` ([B, T] int32
        CUDA, optional) receives the ids (-1 for stopped rows) at column `step`.
        Returns the ids ([B] int32 CUDA)."""
        import torch
        if logits.dim() == 1:
            logits = logits.unsqueeze(0)
        if logits.dtype != torch.float32 or logits.device != self.device or logits.stride(1) != 1:
            raise ValueError("logits must be float32, unit column stride, on the sampler's device")
        B, V = logits.shape
        par, per_row = _params_array(params, B)
        if out is None:
            out = torch.empty(B, dtype=torch.int32, device=self.device)
        for t, name, dt in ((rng_state, "rng_state", torch.int64), (done, "done", torch.int32)):
            if t.dtype != dt or not t.is_contiguous() or t.numel() != B:
                raise ValueError(f"{name} must be a contiguous {dt} tensor of {B} entries")
        hist_ptr = hist_len_ptr = None
        hist_ld = 0
        if history is not None:
            if (history_len is None or history.dtype != torch.int32 or history_len.dtype != torch.int32
                    or not history.is_contiguous() or history.dim() != 2):
                raise ValueError("history ([B, L] int32, contiguous) needs history_len (int32)")
            hist_ptr, hist_len_ptr, hist_ld = history.data_ptr(), history_len.data_ptr(), history.shape[1]
        tok_ptr, tok_ld = None, 0
        if tokens is not None:
            if tokens.dtype != torch.int32 or tokens.dim() != 2 or tokens.stride(1) != 1:
                raise ValueError("tokens must be [B, T] int32 with unit column stride")
            tok_ptr, tok_ld = tokens.data_ptr(), tokens.stride(0)
            if step >= tokens.shape[1]:
                raise ValueError("step outside tokens")
        _native.check(self._lib.zs_decode_step(self._h, logits.data_ptr(), logits.stride(0), B, V,
                                               par, per_row, hist_ptr, hist_ld, hist_len_ptr,
                                               rng_state.data_ptr(), done.data_ptr(), int(eos),
                                               out.data_ptr(), tok_ptr, tok_ld, int(step),
                                               _stream_ptr(stream)), "zs_decode_step")
        return out

    def lmhead_sample(self, hidden, norm_w, weight, params, rng_state=None, eps: float = 1e-6,
                      history=None, history_len=None, out=None, out_logits=None, stream=None):
        """The lm_head (rmsnorm with `norm_w`, then hidden . weight^T; src/model.cpp:
        401-403) fused with sample_token for every row of `hidden` ([B, E] float32
        CUDA).  weight: bfloat16 CUDA [V, E], contiguous.  out_logits (optional,
        float32 CUDA [B, >= V], row stride a multiple of 4) receives the logits the
        sampling used.  Returns the ids ([B] int32 CUDA)."""
        import torch
        if hidden.dim() == 1:
            hidden = hidden.unsqueeze(0)
        if hidden.dtype != torch.float32 or hidden.stride(1) != 1 or hidden.device != self.device:
            raise ValueError("hidden must be float32 with unit column stride on the sampler's device")
        if weight.dtype != torch.bfloat16 or not weight.is_contiguous() or weight.dim() != 2:
            raise ValueError("weight must be a contiguous bfloat16 [V, E] tensor")
        B, E = hidden.shape
        V = weight.shape[0]
        if weight.shape[1] != E or norm_w.numel() != E or norm_w.dtype != torch.float32:
            raise ValueError("weight [V, E] and norm_w [E] float32 must match hidden's E")
        par, per_row = _params_array(params, B)
        if out is None:
            out = torch.empty(B, dtype=torch.int32, device=self.device)
        hist_ptr = hist_len_ptr = None
        hist_ld = 0
        if history is not None:
            if history_len is None:
                raise ValueError("history needs history_len")
            history = history.to(torch.int32).contiguous()
            history_len = history_len.to(torch.int32).contiguous()
            hist_ptr, hist_len_ptr, hist_ld = history.data_ptr(), history_len.data_ptr(), history.shape[1]
        lptr, lld = None, 0
        if out_logits is not None:
            if out_logits.dtype != torch.float32 or out_logits.stride(1) != 1:
                raise ValueError("out_logits must be float32 with unit column stride")
            lptr, lld = out_logits.data_ptr(), out_logits.stride(0)
        rng_ptr = rng_state.data_ptr() if rng_state is not None else None
        _native.check(self._lib.zs_lmhead_sample(
            self._h, hidden.data_ptr(), hidden.stride(0), norm_w.contiguous().data_ptr(),
            float(eps), weight.data_ptr(), B, E, V, par, per_row, hist_ptr, hist_ld, hist_len_ptr,
            rng_ptr, out.data_ptr(), lptr, lld, _stream_ptr(stream)), "zs_lmhead_sample")
        return out

    def lmhead_logits(self, hidden, norm_w, weight, eps: float = 1e-6, out=None, stream=None):
        """The lm_head alone (rmsnorm with `norm_w`, then hidden . weight^T;
        src/model.cpp:401-403) for every row of `hidden` ([B, E] float32 CUDA); weight
        bfloat16 CUDA [V, E].  Up to 8 rows (or with the "exact" route) in f32 exactly
        as the reference computes it, else on the tensor cores with xn rounded to
        bf16.  Returns float32 logits [B, V] (or fills `out`, whose row stride must be
        a multiple of 4)."""
        import torch
        if hidden.dim() == 1:
            hidden = hidden.unsqueeze(0)
        if hidden.dtype != torch.float32 or hidden.stride(1) != 1 or hidden.device != self.device:
            raise ValueError("hidden must be float32 with unit column stride on the sampler's device")
        if weight.dtype != torch.bfloat16 or not weight.is_contiguous() or weight.dim() != 2:
            raise ValueError("weight must be a contiguous bfloat16 [V, E] tensor")
        B, E = hidden.shape
        V = weight.shape[0]
        if weight.shape[1] != E or norm_w.numel() != E or norm_w.dtype != torch.float32:
            raise ValueError("weight [V, E] and norm_w [E] float32 must match hidden's E")
        if out is None:
            out = torch.empty((B, (V + 3) // 4 * 4), dtype=torch.float32, device=self.device)[:, :V]
        if out.dtype != torch.float32 or out.stride(1) != 1:
            raise ValueError("out must be float32 with unit column stride")
        _native.check(self._lib.zs_lmhead_logits(
            self._h, hidden.data_ptr(), hidden.stride(0), norm_w.contiguous().data_ptr(),
            float(eps), weight.data_ptr(), B, E, V, out.data_ptr(), out.stride(0),
            _stream_ptr(stream)), "zs_lmhead_logits")
        return out

    def argmax(self, logits, out=None, stream=None):
        """argmax_token per row."""
        import torch
        if logits.dim() == 1:
            logits = logits.unsqueeze(0)
        B, V = logits.shape
        if out is None:
            out = torch.empty(B, dtype=torch.int32, device=self.device)
        _native.check(self._lib.zs_argmax(self._h, logits.data_ptr(), logits.stride(0), B, V,
                                          out.data_ptr(), _stream_ptr(stream)), "zs_argmax")
        return out

    def logits_stats(self, logits, topn: int = 8, stream=None) -> dict:
        """The `logits` command's display numbers (src/main.cpp:473-503) for every
        row of `logits` ([B, V] float32 CUDA): min, max and Z = sum exp(x - max)
        (float64 [B]), the top-N ids (value descending, then id ascending) and their
        p = exp(x - max) / Z ([B, k], k = clamp(topn, 1, V)), all on the device."""
        import torch
        if logits.dim() == 1:
            logits = logits.unsqueeze(0)
        if logits.dtype != torch.float32 or logits.device != self.device or logits.stride(1) != 1:
            raise ValueError("logits must be float32, unit column stride, on the sampler's device")
        B, V = logits.shape
        k = max(1, min(int(topn), V))
        f64 = dict(dtype=torch.float64, device=self.device)
        out = {"min": torch.empty(B, **f64), "max": torch.empty(B, **f64),
               "z": torch.empty(B, **f64),
               "top_ids": torch.full((B, k), -1, dtype=torch.int32, device=self.device),
               "top_p": torch.zeros((B, k), **f64)}
        _native.check(self._lib.zs_logits_stats(
            self._h, logits.data_ptr(), logits.stride(0), B, V, k, out["min"].data_ptr(),
            out["max"].data_ptr(), out["z"].data_ptr(), out["top_ids"].data_ptr(),
            out["top_p"].data_ptr(), _stream_ptr(stream)), "zs_logits_stats")
        return out

    LMHEAD_ROUTES = {"auto": 0, "fused": 1, "two_pass": 2, "exact": 3}

    def set_lmhead_route(self, route: str) -> None:
        """How lmhead_sample takes the shortlist: "auto" (exact up to 8 rows, two
        passes below 1024 rows, fused from 1024), "fused" (in the GEMM epilogue whenever
        the rows allow it; no logits buffer), "two_pass" (tensor-core logits, then
        sample; the same results as "fused") or "exact" (f32 logits bit-exact with
        the reference's lm_head, then sample; up to 8 rows, rows x hidden size
        up to 8192)."""
        if route not in self.LMHEAD_ROUTES:
            raise ValueError(f"route must be one of {sorted(self.LMHEAD_ROUTES)}")
        _native.check(self._lib.zs_set_lmhead_route(self._h, self.LMHEAD_ROUTES[route]),
                      "zs_set_lmhead_route")

    LMHEAD_TILES = {"auto": 0, "single": 1, "pair": 2}

    def set_lmhead_tiles(self, mode: str) -> None:
        """Tiles of the lm_head GEMM: "auto" (CTA pairs from 512 rows up), "single"
        (one CTA per 128 x 128 tile) or "pair" (two CTAs of a cluster per 256 x 256
        tile).  Same logits, ids and Rng states either way."""
        if mode not in self.LMHEAD_TILES:
            raise ValueError(f"mode must be one of {sorted(self.LMHEAD_TILES)}")
        _native.check(self._lib.zs_set_lmhead_tiles(self._h, self.LMHEAD_TILES[mode]),
                      "zs_set_lmhead_tiles")

    def set_timing(self, enable: bool) -> None:
        """Bracket every kernel of this sampler with CUDA events (measurement only)."""
        _native.check(self._lib.zs_set_timing(self._h, 1 if enable else 0), "zs_set_timing")

    def get_timing(self) -> dict:
        """Per-kernel device time and launch counts since the last call."""
        t = _native.ZsTiming()
        _native.check(self._lib.zs_get_timing(self._h, C.byref(t)), "zs_get_timing")
        return {f: getattr(t, f) for f, _ in t._fields_}

    def check_device_status(self, stream=None) -> None:
        _native.check(self._lib.zs_check_device_status(self._h, _stream_ptr(stream)),
                      "device status")

    # ---- vocab-sharded mode ----
    @staticmethod
    def shard_partial_bytes(batch, n_vocab_total, n_ranks, params) -> int:
        par, per_row = _params_array(params, batch)
        out = C.c_int64()
        _native.check(_native.lib().zs_shard_partial_bytes(batch, n_vocab_total, n_ranks, par,
                                                           per_row, C.byref(out)),
                      "zs_shard_partial_bytes")
        return out.value

    def shard_partials(self, logits_local, vocab_offset, n_vocab_total, n_ranks, params,
                       partial_out, history=None, history_len=None, want_log_z=False,
                       stream=None):
        B, n_local = logits_local.shape
        par, per_row = _params_array(params, B)
        hist_ptr = history.data_ptr() if history is not None else None
        hist_len_ptr = history_len.data_ptr() if history_len is not None else None
        hist_ld = history.shape[1] if history is not None else 0
        _native.check(self._lib.zs_shard_partials(
            self._h, logits_local.data_ptr(), logits_local.stride(0), B, n_local, vocab_offset,
            n_vocab_total, n_ranks, par, per_row, hist_ptr, hist_ld, hist_len_ptr,
            partial_out.data_ptr(), 1 if want_log_z else 0, _stream_ptr(stream)),
            "zs_shard_partials")

    def shard_merge(self, gathered, n_ranks, batch, n_vocab_total, params, rng_state, out=None,
                    row_info=False, cand_ld=0, want_log_z=False, stream=None,
                    rows=None) -> SampleResult:
        """Merges the gathered blocks of every row, or of rows = (row_begin, row_count)
        only (zs_shard_merge_rows: only those rows' entries of out and rng_state are
        written)."""
        import torch
        par, per_row = _params_array(params, batch)
        if out is None:
            out = torch.empty(batch, dtype=torch.int32, device=self.device)
        r0, n = (0, batch) if rows is None else rows
        ex, info_buf, cand_ids, cand_probs = self._extras(batch, row_info, cand_ld, want_log_z)
        _native.check(self._lib.zs_shard_merge_rows(
            self._h, gathered.data_ptr(), n_ranks, batch, r0, n, n_vocab_total, par, per_row,
            rng_state.data_ptr() if rng_state is not None else None, out.data_ptr(),
            C.byref(ex), _stream_ptr(stream)), "zs_shard_merge_rows")
        info = None
        if info_buf is not None:
            info = info_buf.cpu().numpy().view(ROW_INFO_DTYPE).reshape(batch)
        return SampleResult(out, info, cand_ids, cand_probs)

    @staticmethod
    def shard_owner_rows(batch, n_ranks, rank):
        """(row_begin, row_count) that `rank` merges in the row-owner exchange."""
        r0, n = C.c_int32(), C.c_int32()
        _native.check(_native.lib().zs_shard_owner_rows(batch, n_ranks, rank, C.byref(r0),
                                                        C.byref(n)), "zs_shard_owner_rows")
        return r0.value, n.value

    @staticmethod
    def shard_row_spans(batch, n_vocab_total, n_ranks, params, row_begin, row_count):
        """[(offset, length), ...]: the byte ranges of a rank's block area that the merge
        of rows [row_begin, row_begin + row_count) reads."""
        par, per_row = _params_array(params, batch)
        sp = (C.c_int64 * 6)()
        k = C.c_int32()
        _native.check(_native.lib().zs_shard_row_spans(batch, n_vocab_total, n_ranks, par,
                                                       per_row, row_begin, row_count, sp,
                                                       C.byref(k)), "zs_shard_row_spans")
        return [(sp[2 * i], sp[2 * i + 1]) for i in range(k.value)]

    _SPEC_MODES = {"off": 0, "on": 1, "redo_all": 2}

    def set_speculation(self, mode: str) -> None:
        """zs_set_speculation: "on" (default), "off", or "redo_all" (every speculated
        row redone exactly: a test of the redo path)."""
        if mode not in self._SPEC_MODES:
            raise ValueError(f"speculation mode must be one of {sorted(self._SPEC_MODES)}")
        _native.check(self._lib.zs_set_speculation(self._h, self._SPEC_MODES[mode]),
                      "zs_set_speculation")

    def set_small_batch(self, max_rows: int) -> None:
        """zs_set_small_batch: batches up to max_rows rows in one cluster launch (0: off)."""
        _native.check(self._lib.zs_set_small_batch(self._h, int(max_rows)), "zs_set_small_batch")

    def set_collective_timeout(self, timeout_ms: int) -> None:
        """zs_sample_sharded's bound on its collectives (0: asynchronous, no bound)."""
        _native.check(self._lib.zs_set_collective_timeout(self._h, int(timeout_ms)),
                      "zs_set_collective_timeout")


    def sample_sharded(self, logits_local, vocab_offset, n_vocab_total, n_ranks, params,
                       rng_state, nccl_comm, out=None, history=None, history_len=None,
                       row_info=False, stream=None):
        """zs_sample_sharded: the whole vocab-sharded step over `nccl_comm` (an
        ncclComm_t as an int) in one call: the row-owner exchange, or with
        row_info=True one all-gather and a merge of every row on every rank.
        Every rank passes the same batch, params and rng states and gets the same
        ids.  Returns the ids, or (ids, row info) with row_info=True."""
        import torch
        B, n_local = logits_local.shape
        par, per_row = _params_array(params, B)
        if out is None:
            out = torch.empty(B, dtype=torch.int32, device=self.device)
        hist_ptr = history.data_ptr() if history is not None else None
        hist_len_ptr = history_len.data_ptr() if history_len is not None else None
        hist_ld = history.shape[1] if history is not None else 0
        ex, info_buf, _, _ = self._extras(B, row_info, 0, False)
        _native.check(self._lib.zs_sample_sharded(
            self._h, logits_local.data_ptr(), logits_local.stride(0), B, n_local, vocab_offset,
            n_vocab_total, n_ranks, par, per_row, hist_ptr, hist_ld, hist_len_ptr,
            rng_state.data_ptr() if rng_state is not None else None, out.data_ptr(),
            C.byref(ex) if row_info else None, C.c_void_p(nccl_comm),
            _stream_ptr(stream)), "zs_sample_sharded")
        if row_info:
            return out, info_buf.cpu().numpy().view(ROW_INFO_DTYPE).reshape(B)
        return out


# ---- the reference's host-row API ----
_default = threading.local()


def _default_sampler() -> Sampler:
    s = getattr(_default, "sampler", None)
    if s is None:
        s = Sampler()
        _default.sampler = s
    return s


def argmax_token(logits: Sequence[float], n: Optional[int] = None) -> int:
    """argmax_token (src/sample.cpp:24-30) of one host row."""
    import torch
    x = np.ascontiguousarray(np.asarray(logits, dtype=np.float32).reshape(-1))
    n = x.size if n is None else n
    if n <= 0:
        return 0
    s = _default_sampler()
    d = torch.from_numpy(x[:n].copy()).to(s.device)
    return int(s.argmax(d.view(1, n)).item())


def sample_token(logits: Sequence[float], n: Optional[int], params: SamplingParams,
                 history: Sequence[int], rng: Rng) -> int:
    """sample_token (src/sample.cpp:32-102) of one host row; rng advances like zen::Rng&."""
    import torch
    x = np.ascontiguousarray(np.asarray(logits, dtype=np.float32).reshape(-1))
    n = x.size if n is None else n
    if n <= 0:
        return 0
    s = _default_sampler()
    d = torch.from_numpy(x[:n].copy()).to(s.device).view(1, n)
    st = states_to_tensor([rng.state], s.device)
    h = hl = None
    hist = list(history)
    if hist and params.repeat_penalty != 1.0:
        h = torch.tensor([hist], dtype=torch.int32, device=s.device)
        hl = torch.tensor([len(hist)], dtype=torch.int32, device=s.device)
    res = s.sample(d, params, st, h, hl, sync_check=True)
    rng.state = int(tensor_to_states(st)[0])
    return int(res.ids.item())
