"""Loads libah_cuda.so (the sm_100a kernels behind include/ah_cuda.h).

There is no CPU fallback: if the library is missing or CUDA is unavailable the
calls fail loudly with AhError.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libah_cuda.so")

AH_OK, AH_EINVAL, AH_ENOMEM, AH_ECUDA, AH_ENCCL, AH_ETIMEOUT, AH_EUNSUPPORTED = 0, -1, -2, -3, -4, -5, -6
AH_INJECT_ALLOC, AH_INJECT_NCCL, AH_INJECT_LAUNCH = 1, 2, 3

vp = C.c_void_p
i64 = C.c_int64
i32 = C.c_int
u64 = C.c_uint64
u32 = C.c_uint32
f32 = C.c_float
sz = C.c_size_t

# name -> (restype, argtypes); mirrors include/ah_cuda.h
SIGNATURES = {
    "ah_strerror": (C.c_char_p, [i32]),
    "ah_last_error": (C.c_char_p, []),
    "ah_version": (i32, []),
    "ah_device_init": (i32, [i32]),
    "ah_check_device_error": (i32, [vp]),
    "ah_device_alloc_count": (i64, []),
    "ah_debug_inject_failure": (i32, [i32, i64]),
    "ah_debug_residual_add_peer": (i32, [vp, vp, i32, i32, i32, vp, vp, vp, vp]),
    "ah_debug_tc_mma_rate": (i32, [i32, i32, vp]),
    "ah_packed_bytes": (i64, [i64]),
    "ah_n_groups": (i64, [i64, i64]),
    "ah_quantized_bytes": (i64, [i64, i64]),
    "ah_f16_to_f32": (i32, [vp, vp, i64, vp]),
    "ah_bf16_to_f32": (i32, [vp, vp, i64, vp]),
    "ah_f32_to_f16": (i32, [vp, vp, i64, vp]),
    "ah_dequant_q8_0_f32": (i32, [vp, vp, i64, vp]),
    "ah_dequant_q4_0_f32": (i32, [vp, vp, i64, vp]),
    "ah_dequant_layer": (i32, [vp, vp, vp, i64, i64, vp]),
    "ah_dequantize_to_f32": (i32, [vp, i64, u32, i64, vp, C.POINTER(i64), vp]),
    "ah_quantize_q4": (i32, [vp, i64, i64, vp, vp, vp]),
    "ah_quantize_q8_0": (i32, [vp, i64, vp, vp]),
    "ah_quantize_q4_0": (i32, [vp, i64, vp, vp]),
    "ah_fill_normal": (i32, [vp, i64, f32, f32, u64, i64, vp]),
    "ah_synth_q4_0": (i32, [vp, i64, i64, i64, i64, i64, f32, u64, vp]),
    "ah_synth_f16": (i32, [vp, i64, f32, f32, u64, i64, vp]),
    "ah_q4w_from_q4_0": (i32, [vp, i64, i64, C.POINTER(vp), vp]),
    "ah_q4w_from_engine": (i32, [vp, vp, i64, i64, C.POINTER(vp), vp]),
    "ah_q4w_destroy": (i32, [vp]),
    "ah_q4w_shape": (i32, [vp, C.POINTER(i64), C.POINTER(i64)]),
    "ah_q4w_weight_bytes": (i64, [vp]),
    "ah_q4w_gemv_host": (i32, [vp, vp, vp, i32, vp]),
    "ah_arena_page_granularity": (i32, [C.POINTER(sz)]),
    "ah_arena_create": (i32, [sz, sz, i64, C.POINTER(vp)]),
    "ah_arena_destroy": (i32, [vp]),
    "ah_arena_commit_page": (i32, [vp, i64]),
    "ah_arena_evict_page": (i32, [vp, i64, i32, vp, vp]),
    "ah_arena_page_state": (i32, [vp, i64, C.POINTER(i32), C.POINTER(vp)]),
    "ah_arena_gemv_4bit": (i32, [vp, i64, vp, vp, vp, vp, i64, i64, i64, vp]),
    "ah_ssm_workspace_bytes": (i32, [vp, C.POINTER(sz)]),
    "ah_ssm_forward": (i32, [vp, vp, vp, vp, vp, vp, vp, sz, vp]),
    "ah_q4w_planes": (i32, [vp, C.POINTER(vp), C.POINTER(sz), C.POINTER(vp), C.POINTER(sz), C.POINTER(i32)]),
    "ah_dedup_table_local": (i32, [vp, i64, vp, i64, i32, i32, C.c_float, C.POINTER(vp)]),
    "ah_dedup_table_global": (i32, [vp, i64, vp, i64, i32, i32, C.c_float, i32, vp, i64, vp, vp, C.POINTER(vp)]),
    "ah_dedup_table_remap": (i32, [vp, i64, i32, i32, C.c_float, i32, vp, i64, vp, vp, vp, i64, C.POINTER(vp)]),
    "ah_dedup_table_destroy": (i32, [vp]),
    "ah_dedup_decompress_f32": (i32, [vp, vp, i64, vp, i64, vp, i64, i64, vp, vp]),
    "ah_dedup_to_q4w": (i32, [vp, vp, i64, vp, i64, vp, i64, i64, i64, C.POINTER(vp), vp]),
    "ah_dedup_into_q4w": (i32, [vp, vp, i64, vp, i64, vp, i64, vp, vp]),
    "ah_host_dedup_decompress_all": (i32, [vp, i64, vp, i64, i64, i32, i32, C.c_float, vp, i64, vp, i64, vp, i64,
                                           vp]),
    "ah_q4w_gemv": (i32, [vp, vp, vp, i32, vp]),
    "ah_q4w_gemm_workspace_bytes": (i32, [vp, i64, C.POINTER(C.c_size_t)]),
    "ah_q4w_gemm": (i32, [vp, vp, i64, i64, vp, i64, vp, C.c_size_t, vp]),
    "ah_q4w_gemm_noalloc": (i32, [vp, vp, i64, i64, vp, i64, vp]),
    "ah_q4w_gemv_tc_workspace_bytes": (i32, [vp, C.POINTER(C.c_size_t)]),
    "ah_q4w_gemv_tc": (i32, [vp, vp, i64, i32, vp, i64, i32, vp, C.c_size_t, vp]),
    "ah_gemv_4bit_into": (i32, [vp, vp, vp, vp, i64, i64, i64, vp]),
    "ah_matvec_4bit_into": (i32, [vp, vp, vp, vp, i64, i64, vp]),
    "ah_gemv_4bit_rows": (i32, [vp, vp, vp, vp, i64, i64, i64, i64, vp]),
    "ah_swiglu_4bit_into": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, vp, vp, vp, vp]),
    "ah_q4w_from_engine_gate_up": (i32, [vp, vp, vp, vp, i64, i64, C.POINTER(vp), vp]),
    "ah_q4w_from_q4_0_gate_up": (i32, [vp, vp, i64, i64, C.POINTER(vp), vp]),
    "ah_q4w_swiglu": (i32, [vp, vp, vp, vp, vp, i32, vp]),
    "ah_host_gemv_4bit_worker_scalar": (i32, [vp, vp, vp, vp, sz, sz, sz, sz]),
    "ah_host_swiglu_4bit_into": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, sz, sz, sz, vp, vp, vp]),
    "ah_model_create": (i32, [vp, C.POINTER(vp)]),
    "ah_nccl_unique_id": (i32, [vp, C.c_size_t]),
    "ah_model_create_tp": (i32, [vp, i32, i32, vp, C.POINTER(vp)]),
    "ah_model_load_tensor_engine": (i32, [vp, i32, i32, vp, vp, vp]),
    "ah_model_load_tensor_f32": (i32, [vp, i32, i32, vp, vp]),
    "ah_model_ipc_handle": (i32, [vp, vp, C.c_size_t]),
    "ah_model_ipc_open": (i32, [vp, vp, C.c_size_t]),
    "ah_model_shard": (i32, [vp, C.POINTER(i32), C.POINTER(i32), C.POINTER(i32), C.POINTER(i32), C.POINTER(i32),
                             C.POINTER(i32)]),
    "ah_model_destroy": (i32, [vp]),
    "ah_model_load_tensor": (i32, [vp, i32, i32, vp, vp]),
    "ah_model_init_random": (i32, [vp, u64, f32, f32, f32]),
    "ah_model_tensor_seed": (u64, [u64, i32, i32]),
    "ah_model_generate": (i32, [vp, vp, i32, i32, i32, vp, vp]),
    "ah_model_reset": (i32, [vp, i32, vp]),
    "ah_model_forward": (i32, [vp, vp, vp, vp]),
    "ah_model_decode": (i32, [vp, i32, vp, vp]),
    "ah_model_position": (i32, [vp, C.POINTER(i32)]),
    "ah_model_set_prefill": (i32, [vp, i32]),
    "ah_model_set_batched_gemv": (i32, [vp, i32]),
    "ah_q4w_gemm_ex": (i32, [vp, vp, i64, i64, vp, i64, i32, vp, f32, vp, sz, vp]),
    "ah_model_set_sampling": (i32, [vp, f32, i32, u64]),
    "ah_sample_workspace_bytes": (sz, [i32, i64]),
    "ah_sample_logits": (i32, [vp, i64, i32, i64, f32, i32, u64, i64, vp, vp, sz, vp]),
    "ah_sample_uniform": (f32, [u64, i64, i32]),
    "ah_host_gemv_4bit_into": (i32, [vp, vp, vp, vp, sz, sz, sz]),
    "ah_host_dequant_layer": (i32, [vp, vp, vp, sz, sz]),
    "ah_host_quantize": (i32, [vp, sz, sz, vp, vp]),
    "ah_host_f16_bytes_to_f32": (i32, [vp, sz, vp]),
    "ah_host_bf16_bytes_to_f32": (i32, [vp, sz, vp]),
    "ah_host_dequantize_to_f32": (i32, [vp, sz, u32, sz, vp, C.POINTER(sz)]),
}


class AhError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{message} (status {status})")
        self.status = status


_lib = None


def lib():
    """The loaded library; raises AhError if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise AhError(AH_EUNSUPPORTED, f"{LIB_PATH} is missing: run agent_harness_b200/build.py")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != AH_OK:
        msg = lib().ah_last_error().decode(errors="replace")
        raise AhError(rc, msg or lib().ah_strerror(rc).decode())


def call(name: str, *args) -> int:
    rc = getattr(lib(), name)(*args)
    check(rc)
    return rc
