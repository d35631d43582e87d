"""ctypes binding of the C ABI declared in include/qwen600_sampler.h.

The library is the in-tree libqwen600_sampler.so built by
qwen600_engine_b200/build.py.  There is no fallback: if it is missing or
cannot be loaded, importing this module raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqwen600_sampler.so")

QS_OK = 0
QS_ERR_INVALID = -1
QS_ERR_CUDA = -2
QS_ERR_ALLOC = -3
QS_ERR_UNSUPPORTED = -4

QS_F32 = 0
QS_BF16 = 1

QS_FLAG_WRITE_PENALIZED = 1
QS_FLAG_INDEX_TIES = 2

# Every symbol the header declares (the CPU test checks the .so exports them).
EXPORTS = (
    "qs_build_sampler", "qs_free_sampler", "qs_set_params", "qs_get_params",
    "qs_set_rng_state", "qs_get_rng_state", "qs_reset_sampler_history", "qs_sample",
    "qs_sample_rows", "qs_sample_rows_debug", "qs_sample_host", "qs_sample_rows_host", "qs_last_error",
    "qs_max_vocab", "qs_profile_enable", "qs_profile_reset", "qs_profile_read",
    "qs_profile_phases", "qs_profile_phases_read",
    "qs_argmax_rows_static", "qs_lm_head", "qs_lm_head_sample", "qs_lm_head_logits",
    "qs_lm_head_status", "qs_lm_head_set_wait_limit", "qs_lm_head_shard", "qs_ipc_handle_bytes", "qs_ipc_alloc", "qs_ipc_open",
    "qs_ipc_close", "qs_ipc_free", "qs_shard_handshake", "qs_copy_async",
)


class Params(C.Structure):
    _fields_ = [("temperature", C.c_float), ("topp", C.c_float), ("minp", C.c_float),
                ("top_k", C.c_int), ("repetition_penalty", C.c_float),
                ("frequency_penalty", C.c_float), ("presence_penalty", C.c_float)]


class RowDebug(C.Structure):
    _fields_ = [("token", C.c_int), ("greedy", C.c_int), ("n_topk", C.c_int),
                ("n_minp", C.c_int), ("n_final", C.c_int), ("draw_pos", C.c_int),
                ("exact_ties", C.c_int), ("sum_fallback", C.c_int), ("max_logit", C.c_float),
                ("sum", C.c_float), ("r", C.c_float), ("renorm_sum", C.c_float)]


class Profile(C.Structure):
    _fields_ = [("stream_ms", C.c_double), ("finish_ms", C.c_double), ("ties_ms", C.c_double),
                ("emit_ms", C.c_double), ("calls", C.c_longlong), ("launches", C.c_longlong),
                ("row_launches", C.c_longlong), ("timed_calls", C.c_longlong),
                ("tie_clusters", C.c_longlong)]


ROW_DEBUG_FIELDS = [f for f, _ in RowDebug._fields_]


class SamplerError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"qwen600 sampler error {code}: {msg}")
        self.code = code


def _load() -> C.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing; build it with `python -m qwen600_engine_b200.build` "
            "(or __graft_entry__.build()).  There is no CPU fallback.")
    lib = C.CDLL(LIB_PATH)
    vp, i32, u32 = C.c_void_p, C.c_int, C.c_uint
    P = C.POINTER
    lib.qs_build_sampler.argtypes = [P(vp), P(Params), i32, i32, i32, C.c_ulonglong, i32]
    lib.qs_free_sampler.argtypes = [vp]
    lib.qs_set_params.argtypes = [vp, P(Params)]
    lib.qs_get_params.argtypes = [vp, P(Params)]
    lib.qs_set_rng_state.argtypes = [vp, P(C.c_ulonglong), i32]
    lib.qs_get_rng_state.argtypes = [vp, P(C.c_ulonglong), i32]
    lib.qs_reset_sampler_history.argtypes = [vp]
    lib.qs_sample.argtypes = [vp, vp, i32, i32, vp, vp, u32]
    lib.qs_sample_rows.argtypes = [vp, vp, i32, i32, i32, vp, vp, vp, i32, vp, vp, vp, u32]
    lib.qs_sample_rows_debug.argtypes = [vp, vp, i32, i32, i32, vp, vp, vp, i32, vp, vp, vp,
                                         vp, vp, vp, i32, vp, u32]
    lib.qs_sample_host.argtypes = [vp, vp, i32, vp, u32]
    lib.qs_sample_rows_host.argtypes = [vp, vp, i32, i32, i32, vp, vp, vp, i32, vp, vp, vp, u32]
    lib.qs_profile_enable.argtypes = [vp, i32]
    lib.qs_profile_reset.argtypes = [vp]
    lib.qs_profile_read.argtypes = [vp, P(Profile)]
    lib.qs_profile_phases.argtypes = [vp, i32]
    lib.qs_profile_phases_read.argtypes = [vp, i32, P(C.c_longlong), i32]
    lib.qs_argmax_rows_static.argtypes = [vp, i32, i32, i32, vp, vp, vp, i32, C.c_float, C.c_float,
                                          C.c_float, vp, vp]
    lib.qs_lm_head.argtypes = [vp, vp, vp, i32, i32, i32, vp, vp, vp, vp]
    lib.qs_lm_head_sample.argtypes = [vp, vp, vp, vp, i32, i32, vp, vp, u32]
    lib.qs_lm_head_logits.argtypes = [vp, P(vp)]
    lib.qs_lm_head_status.argtypes = [vp, vp]
    lib.qs_lm_head_set_wait_limit.argtypes = [C.c_ulonglong]
    lib.qs_lm_head_shard.argtypes = [vp, vp, vp, i32, i32, i32, i32, i32, vp, P(vp), i32, i32, vp, vp]
    lib.qs_ipc_handle_bytes.argtypes = []
    lib.qs_ipc_alloc.argtypes = [C.c_size_t, P(vp), vp]
    lib.qs_ipc_open.argtypes = [vp, P(vp)]
    lib.qs_ipc_close.argtypes = [vp]
    lib.qs_ipc_free.argtypes = [vp]
    lib.qs_shard_handshake.argtypes = [P(vp), i32, i32, C.c_size_t, u32, C.c_ulonglong, vp, vp]
    lib.qs_copy_async.argtypes = [vp, vp, C.c_size_t, vp]
    lib.qs_last_error.restype = C.c_char_p
    lib.qs_last_error.argtypes = []
    lib.qs_max_vocab.argtypes = []
    for name in EXPORTS:
        if name not in ("qs_last_error",):
            getattr(lib, name).restype = C.c_int
    return lib


lib = _load()


def check(rc: int) -> None:
    if rc != QS_OK:
        raise SamplerError(rc, lib.qs_last_error().decode(errors="replace"))
