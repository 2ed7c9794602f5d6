"""ctypes binding of libttk.so, the C ABI of include/ttk.h.

Loading fails loudly when the library is missing: there is no CPU path.
`call(name, *args)` checks the returned status and raises TtkError with
ttk_last_error(). Pointers are plain ints (e.g. torch.Tensor.data_ptr()).
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libttk.so")

P = C.c_void_p
I64 = C.c_int64
I32 = C.c_int
F32 = C.c_float
U64 = C.c_uint64
SZ = C.c_size_t

# name -> (restype, argtypes); status-returning functions use I32.
SIGS = {
    "ttk_last_error": (C.c_char_p, []),
    "ttk_version": (C.c_char_p, []),
    "ttk_init": (I32, [I32]),
    "ttk_device_count": (I32, [P]),
    "ttk_current_device": (I32, [P]),
    "ttk_device_status": (I32, [P]),
    "ttk_synchronize": (I32, []),
    "ttk_selftest_wait_timeout": (I32, [C.c_uint, C.c_uint64, P]),
    "ttk_event_query": (I32, [P, P]),
    "ttk_stream_begin_capture": (I32, [P]),
    "ttk_stream_end_capture": (I32, [P, P]),
    "ttk_graph_launch": (I32, [P, P]),
    "ttk_graph_destroy": (I32, [P]),
    "ttk_pool_trim": (I32, [P]),
    "ttk_set_block_cache": (I32, [I32]),
    "ttk_launch_count": (I64, []),
    "ttk_malloc": (I32, [P, SZ, P]),
    "ttk_free": (I32, [P, P]),
    "ttk_pool_stats": (I32, [P, P]),
    "ttk_pool_high_water": (I32, [P, P, I32]),
    "ttk_host_alloc": (I32, [P, SZ]),
    "ttk_host_free": (I32, [P]),
    "ttk_memcpy_h2d": (I32, [P, P, SZ, P]),
    "ttk_memcpy_d2h": (I32, [P, P, SZ, P]),
    "ttk_memcpy_d2h_async": (I32, [P, P, SZ, P]),
    "ttk_memcpy_d2d": (I32, [P, P, SZ, P]),
    "ttk_memset": (I32, [P, I32, SZ, P]),
    "ttk_stream_create": (I32, [P]),
    "ttk_stream_destroy": (I32, [P]),
    "ttk_stream_synchronize": (I32, [P]),
    "ttk_event_create": (I32, [P]),
    "ttk_event_destroy": (I32, [P]),
    "ttk_event_record": (I32, [P, P]),
    "ttk_stream_wait_event": (I32, [P, P]),
    "ttk_event_elapsed_ms": (I32, [P, P, P]),
    "ttk_event_synchronize": (I32, [P]),
    "ttk_gemm_set_precision": (I32, [I32]),
    "ttk_gemm_get_precision": (I32, []),
    "ttk_gemm_set_cta_pairs": (I32, [I32]),
    "ttk_gemm_set_split_k": (I32, [I32]),
    "ttk_gemm_get_split_k": (I32, []),
    "ttk_gemm_split_k_slices": (I32, [I32, I32, I64, I64, I64, I64]),
    "ttk_gemm_get_cta_pairs": (I32, []),
    "ttk_gemm_set_fp32_max_macs": (I32, [I64]),
    "ttk_gemm_get_fp32_max_macs": (I64, []),
    "ttk_gemm_uses_fp32": (I32, [I64, I64, I64, I64]),
    "ttk_gemm_workspace_size": (SZ, [I32, I32, I64, I64, I64, I64]),
    "ttk_gemm": (I32, [I32, I32, I64, I64, I64, I64, F32, P, I64, I64, P, I64, I64, F32, P, I64,
                       I64, P, SZ, P]),
    "ttk_gemm_noalloc_max_workspace": (SZ, []),
    "ttk_gemm_noalloc": (I32, [I32, I32, I64, I64, I64, I64, F32, P, I64, I64, P, I64, I64, F32, P,
                               I64, I64, P]),
    "ttk_split_tf32": (I32, [P, I64, I64, I64, I64, I64, P, I64, P]),
    "ttk_gemm_split_bytes": (C.c_size_t, [I64, I64, I64]),
    "ttk_gemm_split": (I32, [P, I64, I64, I64, I64, I64, P, P]),
    "ttk_gemm_splits": (I32, [I32, I32, I64, I64, I64, I64, F32, P, P, F32, P, I64, I64, P]),
    "ttk_gemm_presplit": (I32, [I32, I32, I64, I64, I64, I64, F32, P, I64, P, I64, F32, P, I64,
                                I64, P]),
    "ttk_profile_enable": (I32, [I32]),
    "ttk_profile_read": (I32, [P, P, P]),
    "ttk_rmsnorm_fwd": (I32, [P, P, P, P, I64, I64, F32, P]),
    "ttk_rmsnorm_fwd_split": (I32, [P, P, P, P, I64, I64, F32, P, P]),
    "ttk_rmsnorm_bwd_workspace_size": (SZ, [I64, I64]),
    "ttk_rmsnorm_bwd": (I32, [P, P, P, P, P, I32, P, I64, I64, P, SZ, P]),
    "ttk_swiglu_fwd": (I32, [P, P, P, I64, P]),
    "ttk_swiglu_bwd": (I32, [P, P, P, P, P, I32, I64, P]),
    "ttk_swiglu_fwd_split": (I32, [P, P, P, I64, I64, P]),
    "ttk_swiglu_bwd_split": (I32, [P, P, P, P, P, I64, I64, P]),
    "ttk_cross_entropy": (I32, [P, P, I64, I64, P, P, F32, P]),
    "ttk_loss_finalize": (I32, [P, F32, P, P]),
    "ttk_attention_fwd_workspace_size": (SZ, [I64, I64, I64, I64]),
    "ttk_attention_fwd": (I32, [P, P, P, P, P, P, P, I64, I64, I64, I64, F32, P, SZ, P]),
    "ttk_attention_fwd_split": (I32, [P, P, P, P, P, P, P, P, I64, I64, I64, I64, F32, P, SZ,
                                       P]),
    "ttk_attention_set_impl": (I32, [I32]),
    "ttk_attention_get_impl": (I32, []),
    "ttk_attention_bwd_workspace_size": (SZ, [I64, I64, I64, I64]),
    "ttk_attention_bwd": (I32, [P, P, P, P, P, P, P, P, P, P, P, I32, I64, I64, I64, I64, F32, P,
                                SZ, P]),
    "ttk_attention_bwd_ex_workspace_size": (SZ, [I64] * 4),
    "ttk_attention_bwd_ex": (I32, [P] * 11 + [I32] + [I64] * 4 + [F32, P, P, SZ, P]),
    "ttk_attention_bwd_split": (I32, [P] * 11 + [I32] + [I64] * 4 + [F32, P, P, SZ, P, P, P, P]),
    "ttk_embedding_fwd": (I32, [P, P, P, I64, I64, I64, P]),
    "ttk_embedding_bwd_workspace_size": (SZ, [I64]),
    "ttk_embedding_bwd": (I32, [P, P, P, I64, I64, I64, P, SZ, P]),
    "ttk_index_check": (I32, [P, I64, I64, P, P]),
    "ttk_rope_fwd": (I32, [P, P, P, P, I64, I64, I64, I64, P]),
    "ttk_dropout_mask": (I32, [P, I64, F32, U64, P]),
    "ttk_gather_windows": (I32, [P, P, I64, I64, P, P, P]),
    "ttk_rope_bwd": (I32, [P, P, P, P, I32, I64, I64, I64, I64, P]),
    "ttk_nll_fwd": (I32, [P, P, I64, I64, P, P]),
    "ttk_nll_bwd": (I32, [P, I64, I64, P, P, P]),
    "ttk_rope_table_grad": (I32, [P, P, I64, I64, I64, I64, P, P, P]),
    "ttk_axpy_dev": (I32, [P, P, P, I64, I32, P]),
    "ttk_softmax_fwd": (I32, [P, P, I64, I64, I32, P]),
    "ttk_softmax_bwd": (I32, [P, P, P, I32, I64, I64, I32, P]),
    "ttk_sumsq_multi": (I32, [P, P, I32, P, P]),
    "ttk_adamw_multi": (I32, [P, P, P, P, P, I32, F32, F32, F32, F32, F32, I64, P, F32, F32, P]),
    "ttk_adamw_multi_sched": (I32, [P, P, P, P, P, I32, F32, F32, F32, F32, P, P, F32, F32, P]),
    "ttk_adamw_sched_set": (I32, [P, F32, F32, F32, I64, P]),
    "ttk_sgd": (I32, [P, P, P, I64, F32, F32, F32, P]),
    "ttk_binary": (I32, [I32, P, P, P, P, P, P, I32, P]),
    "ttk_binary_bwd": (I32, [I32, I32, P, P, P, P, P, P, P, I32, P]),
    "ttk_unary": (I32, [I32, P, P, I64, F32, P]),
    "ttk_unary_bwd": (I32, [I32, P, P, P, I64, F32, P]),
    "ttk_reduce_mid": (I32, [P, P, I64, I64, I64, I32, P]),
    "ttk_sum_all": (I32, [P, I64, P, I32, P]),
    "ttk_strided_copy": (I32, [P, P, P, P, I32, I32, I32, P]),
    "ttk_fill": (I32, [P, F32, I64, P]),
    "ttk_axpy": (I32, [F32, P, P, I64, P]),
    "ttk_reduce_to": (I32, [P, P, I32, C.c_uint, P, I32, P]),
    "ttk_init_normal": (I32, [P, I64, F32, U64, P]),
    "ttk_dist_unique_id": (I32, [P]),
    "ttk_dist_init": (I32, [I32, I32, P, P]),
    "ttk_dist_destroy": (I32, [P]),
    "ttk_dist_allreduce_f32": (I32, [P, P, I64, P]),
    "ttk_dist_allreduce_f64": (I32, [P, P, I64, P]),
    "ttk_dist_async_error": (I32, [P, P]),
    "ttk_dist_abort": (I32, [P]),
}

# int-returning functions that return a value, not a status
VALUE_FNS = {"ttk_gemm_get_precision", "ttk_attention_get_impl", "ttk_gemm_uses_fp32",
             "ttk_gemm_get_cta_pairs", "ttk_gemm_get_split_k", "ttk_gemm_split_k_slices"}
STATUS_FNS = {k for k, (r, _) in SIGS.items() if r is I32 and k not in VALUE_FNS}


class TtkError(RuntimeError):
    pass


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m tinytrain_b200.build` "
                "(the CUDA kernels are the only implementation; there is no CPU path)")
        _lib = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)
        for name, (res, args) in SIGS.items():
            fn = getattr(_lib, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
    return _lib


def exported(name: str) -> bool:
    return getattr(lib(), name, None) is not None


def last_error() -> str:
    m = lib().ttk_last_error()
    return m.decode() if m else ""


def call(name: str, *args):
    fn = getattr(lib(), name)
    r = fn(*args)
    if name in STATUS_FNS and r != 0:
        raise TtkError(f"{name} failed ({r}): {last_error()}")
    return r


def ptr_array(ptrs):
    arr = (C.c_void_p * max(len(ptrs), 1))(*ptrs)
    return arr


def i64_array(vals):
    return (C.c_int64 * max(len(vals), 1))(*vals)


def device_status() -> int:
    v = C.c_uint(0)
    call("ttk_device_status", C.byref(v))
    return v.value
