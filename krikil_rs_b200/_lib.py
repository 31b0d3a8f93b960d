"""ctypes binding of lib/libkrikil_cuda.so (the C ABI of include/krikil_cuda.h).

The shared library is built in-tree (``make -C krikil_rs_b200``); importing this
module fails loudly if it is missing -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
# KRIKIL_CHECKED=1 loads the checked build (make CHECKED=1), whose kernels
# report violated preconditions on device data (krk_check_status).
CHECKED = os.environ.get("KRIKIL_CHECKED", "0") == "1"
LIB_PATH = os.path.join(_HERE, "lib", "libkrikil_cuda_checked.so" if CHECKED else "libkrikil_cuda.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is missing: build it with `make -C {_HERE}{' CHECKED=1' if CHECKED else ''}` "
                      "(or __graft_entry__.build())")

lib = C.CDLL(LIB_PATH)

_vp = C.c_void_p
_fp = C.c_void_p  # device or host float pointers are passed as raw addresses
_i32 = C.c_int
_i64 = C.c_int64
_f32 = C.c_float

# name: (restype, argtypes)
_SIGS = {
    "krk_last_error": (C.c_char_p, []),
    "krk_status_string": (C.c_char_p, [_i32]),
    "krk_abi_version": (_i32, []),
    "krk_model_load": (_i32, [C.c_char_p, _i32, C.POINTER(_vp)]),
    "krk_model_free": (_i32, [_vp]),
    "krk_model_device": (_i32, [_vp, C.POINTER(_i32)]),
    "krk_model_stream": (_i32, [_vp, C.POINTER(_vp)]),
    "krk_state_create": (_i32, [_vp, _i32, _i32, C.POINTER(_vp)]),
    "krk_state_free": (_i32, [_vp]),
    "krk_state_reset": (_i32, [_vp, _vp]),
    "krk_state_batch": (_i32, [_vp, C.POINTER(_i32)]),
    "krk_state_context_limit": (_i32, [_vp, C.POINTER(_i32)]),
    "krk_state_positions": (_i32, [_vp, _vp]),
    "krk_prefill": (_i32, [_vp, _vp, _vp, _vp, _vp]),
    "krk_step": (_i32, [_vp, _vp, _vp, _vp]),
    "krk_generate_greedy": (_i32, [_vp, _vp, _vp, _vp, _i32, _f32, _i32, _vp, _vp]),
    "krk_state_export": (_i32, [_vp, _i32, _i32, _i32, _vp, _i64]),
    "krk_launch_count": (_i32, [C.POINTER(C.c_uint64)]),
    "krk_checked_build": (_i32, []),
    "krk_check_status": (_i32, [C.POINTER(C.c_uint32), _i32]),
    "krk_state_profile": (_i32, [_vp, _i32]),
    "krk_state_profile_read": (_i32, [_vp, _i32, C.POINTER(C.c_double), C.POINTER(_i64)]),
    "krk_state_profile_units": (_i32, [_vp, _i32, C.POINTER(_i64)]),
    "krk_state_set_decode_streams": (_i32, [_vp, _i32]),
    "krk_state_set_step_graphs": (_i32, [_vp, _i32]),
    "krk_generate_sample": (_i32, [_vp, _vp, _vp, _vp, _i32, _f32, _f32, _i32, _f32, _vp, _i32, _vp, _vp]),
    "krk_k_sample": (_i32, [_fp, _i64, _i32, _i32, _vp, _f32, _f32, _i32, _f32, _vp, _vp, _vp]),
    "krk_rng_seed_state": (_i32, [C.c_uint64, _vp]),
    "krk_k_rmsnorm_rows": (_i32, [_fp, _fp, _f32, _i64, _i32, _fp, _vp]),
    "krk_k_rmsnorm_fm": (_i32, [_fp, _i32, _fp, _f32, _i32, _i32, _fp, _i32, _vp]),
    "krk_k_gated_rmsnorm_residual": (_i32, [_fp, _fp, _fp, _fp, _f32, _i64, _i32, _fp, _vp]),
    "krk_k_gemm": (_i32, [_fp, _i32, _fp, _i32, _fp, _i32, _i32, _i32, _i32, _i32, _i32, _vp]),
    "krk_k_gemm_tiled": (_i32, [_fp, _i32, _fp, _i32, _fp, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _vp]),
    "krk_k_gemm_tile_rows": (_i32, [_i32, _i32]),
    "krk_k_embed": (_i32, [_vp, _fp, _i32, _i32, _i32, _fp, _i32, _vp]),
    "krk_k_pointwise": (_i32, [_i32, _fp, _fp, _i64, _vp]),
    "krk_k_conv_ssd_step": (_i32, [_fp] * 12 + [_i32] * 4 + [_vp]),
    "krk_k_conv_ssd_scan": (_i32, [_fp] * 12 + [_i32] * 5 + [_vp]),
    "krk_attn_work_floats": (C.c_size_t, [_i32, _i32, _i32, _i32, _i32]),
    "krk_k_rope_kv_attn_decode": (_i32, [_fp] * 8 + [_i32] * 5 + [_f32, _vp]),
    "krk_k_greedy": (_i32, [_fp, _i64, _i32, _i32, _vp, _f32, _vp, _vp]),
    "krk_k_gemm_sgemm_order": (_i32, [_fp, _i32, _fp, _i32, _fp, _i32, _i32, _i32, _i32, _vp]),
    "krk_k_attn_prefill_rows": (_i32, [_i32, _i32]),
    "krk_k_rope_kv_attn_prefill": (_i32, [_fp, _i64, _fp, _fp, _i64, _i64, _i64, _vp, _vp] + [_i32] * 4
                                   + [_f32, _vp] + [_i32] * 3 + [_fp, _i64, _i64, _vp]),
    "krk_k_rope_kv_attn_decode_noalloc": (_i32, [_fp] * 7 + [_i32] * 5 + [_f32, _vp]),
    "krk_k_wait_probe": (_i32, [_fp, _i32, _i32, _vp, _vp]),
    # include/krikil_text.h
    "krk_tokenizer_load": (_i32, [C.c_char_p, C.POINTER(_vp)]),
    "krk_tokenizer_free": (_i32, [_vp]),
    "krk_tokenizer_encode": (_i32, [_vp, C.c_char_p, C.c_size_t, _vp, C.c_size_t, C.POINTER(C.c_size_t)]),
    "krk_tokenizer_decode": (_i32, [_vp, _vp, C.c_size_t, _i32, C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)]),
    "krk_tokenizer_token_to_id": (_i32, [_vp, C.c_char_p, C.POINTER(_i64)]),
    "krk_tokenizer_eos_token_id": (_i32, [_vp, C.POINTER(C.c_uint32)]),
    "krk_tokenizer_vocab_size": (_i32, [_vp, C.POINTER(C.c_size_t)]),
    "krk_tokenizer_resolve_path": (_i32, [C.c_char_p, C.c_char_p, C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)]),
    "krk_chat_template_render": (_i32, [C.c_char_p, C.POINTER(C.c_char_p), C.POINTER(C.c_char_p), C.c_size_t, _i32,
                                        C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)]),
    "krk_default_chat_template": (C.c_char_p, []),
}

for _name, (_res, _args) in _SIGS.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args

EXPORTED = tuple(_SIGS)

OK, BAD_TOKEN, CONTEXT_OVERFLOW, EMPTY, IO, NOT_FOUND, INVALID, CUDA, CHECK_FAILED = range(9)
CHECK_TOKEN, CHECK_POSITION, CHECK_TABLE, CHECK_COLUMN = 1, 2, 4, 8  # krk_check_status bits

# krk_state_profile_read classes
PROF_CLASSES = ("device_total", "gemm", "ssd_step", "attn_decode", "norm", "conv", "ssd_scan", "attn_prefill",
                "other")


class KrikilError(RuntimeError):
    """A non-zero krk_status, with the library's message."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{message} [{lib.krk_status_string(status).decode()}]")
        self.status = status
        self.message = message


def check(status: int) -> None:
    if status != OK:
        raise KrikilError(status, (lib.krk_last_error() or b"").decode(errors="replace"))


def launch_count() -> int:
    n = C.c_uint64(0)
    check(lib.krk_launch_count(C.byref(n)))
    return int(n.value)
