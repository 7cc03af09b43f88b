"""ctypes binding of libzs_sampler.so (include/zs_sampler.h).

The library is the product: there is no fallback.  If it is missing or cannot
be loaded, every entry point raises.
"""

from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
SAMPLER_SO = os.path.join(HERE, "libzs_sampler.so")

# Every symbol include/zs_sampler.h declares.
EXPORTS = (
    "zs_create", "zs_destroy", "zs_last_error", "zs_status_string", "zs_abi_version",
    "zs_rng_seed", "zs_sample", "zs_argmax", "zs_check_device_status",
    "zs_shard_partial_bytes", "zs_shard_partials", "zs_shard_merge", "zs_sample_sharded",
    "zs_sample_noalloc", "zs_set_timing", "zs_get_timing", "zs_logits_stats",
    "zs_selftest_wait_timeout", "zs_decode_step", "zs_lmhead_sample", "zs_lmhead_logits",
    "zs_set_lmhead_route", "zs_shard_owner_rows", "zs_shard_row_spans", "zs_shard_merge_rows",
    "zs_set_collective_timeout", "zs_set_speculation", "zs_set_small_batch",
    "zs_set_lmhead_tiles",
)

ZS_OK = 0


class ZsParams(C.Structure):
    _fields_ = [("temp", C.c_float), ("top_k", C.c_int32), ("top_p", C.c_float),
                ("repeat_penalty", C.c_float), ("repeat_last_n", C.c_int32)]


class ZsRowInfo(C.Structure):
    _fields_ = [("max_logit", C.c_float), ("k", C.c_int32), ("m", C.c_int32), ("pos", C.c_int32),
                ("r", C.c_double), ("sum", C.c_double), ("boundary", C.c_double),
                ("log_z", C.c_double)]


class ZsExtras(C.Structure):
    _fields_ = [("row_info", C.c_void_p), ("cand_ids", C.c_void_p), ("cand_probs", C.c_void_p),
                ("cand_ld", C.c_int32), ("want_log_z", C.c_int32)]


class ZsTiming(C.Structure):
    _fields_ = [("select_ms", C.c_double), ("merge_ms", C.c_double), ("large_ms", C.c_double),
                ("select_launches", C.c_int64), ("merge_launches", C.c_int64),
                ("large_launches", C.c_int64), ("launches", C.c_int64),
                ("lmhead_ms", C.c_double), ("lmhead_launches", C.c_int64),
                ("lmnorm_ms", C.c_double), ("lmnorm_launches", C.c_int64)]


class SamplerError(RuntimeError):
    def __init__(self, status: int, what: str, detail: str):
        super().__init__(f"{what}: status {status} ({detail})")
        self.status = status


_lib = None


def lib() -> C.CDLL:
    """Loads libzs_sampler.so once; raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(SAMPLER_SO):
        raise RuntimeError(f"{SAMPLER_SO} is not built; run python -m zeninfer_b200.build")
    L = C.CDLL(SAMPLER_SO, mode=C.RTLD_LOCAL)
    vp, i32, i64, u64 = C.c_void_p, C.c_int32, C.c_int64, C.c_uint64
    L.zs_create.argtypes = [C.c_int, C.POINTER(vp)]
    L.zs_destroy.argtypes = [vp]
    L.zs_last_error.restype = C.c_char_p
    L.zs_status_string.restype = C.c_char_p
    L.zs_status_string.argtypes = [C.c_int]
    L.zs_rng_seed.restype = u64
    L.zs_rng_seed.argtypes = [u64]
    L.zs_sample.argtypes = [vp, vp, i64, i32, i32, C.POINTER(ZsParams), i32, vp, i64, vp, vp, vp,
                            C.POINTER(ZsExtras), vp]
    L.zs_argmax.argtypes = [vp, vp, i64, i32, i32, vp, vp]
    L.zs_check_device_status.argtypes = [vp, vp]
    L.zs_shard_partial_bytes.argtypes = [i32, i32, i32, C.POINTER(ZsParams), i32, C.POINTER(i64)]
    L.zs_shard_partials.argtypes = [vp, vp, i64, i32, i32, i32, i32, i32, C.POINTER(ZsParams), i32,
                                    vp, i64, vp, vp, i32, vp]
    L.zs_shard_merge.argtypes = [vp, vp, i32, i32, i32, C.POINTER(ZsParams), i32, vp, vp,
                                 C.POINTER(ZsExtras), vp]
    L.zs_sample_sharded.argtypes = [vp, vp, i64, i32, i32, i32, i32, i32, C.POINTER(ZsParams), i32,
                                    vp, i64, vp, vp, vp, C.POINTER(ZsExtras), vp, vp]
    L.zs_shard_owner_rows.argtypes = [i32, i32, i32, C.POINTER(i32), C.POINTER(i32)]
    L.zs_shard_row_spans.argtypes = [i32, i32, i32, C.POINTER(ZsParams), i32, i32, i32,
                                     C.POINTER(i64), C.POINTER(i32)]
    L.zs_shard_merge_rows.argtypes = [vp, vp, i32, i32, i32, i32, i32, C.POINTER(ZsParams), i32,
                                      vp, vp, C.POINTER(ZsExtras), vp]
    L.zs_set_collective_timeout.argtypes = [vp, i32]
    L.zs_set_speculation.argtypes = [vp, i32]
    L.zs_set_small_batch.argtypes = [vp, i32]
    L.zs_selftest_wait_timeout.argtypes = [vp, vp]
    L.zs_lmhead_logits.argtypes = [vp, vp, i64, vp, C.c_float, vp, i32, i32, i32, vp, i64, vp]
    L.zs_lmhead_sample.argtypes = [vp, vp, i64, vp, C.c_float, vp, i32, i32, i32,
                                   C.POINTER(ZsParams), i32, vp, i64, vp, vp, vp, vp, i64, vp]
    L.zs_decode_step.argtypes = [vp, vp, i64, i32, i32, C.POINTER(ZsParams), i32, vp, i64, vp, vp,
                                 vp, i32, vp, vp, i64, i64, vp]
    L.zs_logits_stats.argtypes = [vp, vp, i64, i32, i32, i32, vp, vp, vp, vp, vp, vp]
    L.zs_set_timing.argtypes = [vp, i32]
    L.zs_set_lmhead_route.argtypes = [vp, i32]
    L.zs_set_lmhead_tiles.argtypes = [vp, i32]
    L.zs_get_timing.argtypes = [vp, C.POINTER(ZsTiming)]
    L.zs_sample_noalloc.argtypes = [vp, i64, i32, i32, C.POINTER(ZsParams), vp, i64, vp, vp, vp,
                                    vp, vp]
    for name in EXPORTS:
        f = getattr(L, name)
        if f.restype is C.c_int or name in ("zs_create", "zs_destroy", "zs_sample", "zs_argmax",
                                            "zs_check_device_status", "zs_shard_partial_bytes",
                                            "zs_shard_partials", "zs_shard_merge",
                                            "zs_sample_sharded", "zs_sample_noalloc",
                                            "zs_set_timing", "zs_get_timing",
                                            "zs_logits_stats", "zs_selftest_wait_timeout",
                                            "zs_decode_step", "zs_lmhead_sample",
                                            "zs_lmhead_logits", "zs_set_lmhead_route",
                                            "zs_shard_owner_rows", "zs_shard_row_spans",
                                            "zs_shard_merge_rows", "zs_set_collective_timeout",
                                            "zs_set_speculation", "zs_set_small_batch",
                                            "zs_set_lmhead_tiles"):
            f.restype = C.c_int
    _lib = L
    return L


def check(status: int, what: str) -> None:
    if status != ZS_OK:
        detail = lib().zs_last_error().decode(errors="replace")
        raise SamplerError(status, what, detail)
