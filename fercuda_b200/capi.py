"""ctypes binding of the fercuda C ABI (libfercuda_capi.so and the native
libptx_core.so / libptx_kernels.so), mirroring include/fercuda/** and
include/ptx/** struct for struct.

The libraries are the product; this module only loads them. It raises
FerNativeError when they are missing - there is no Python fallback path.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
LIBDIR = PKG / "lib"


class FerNativeError(RuntimeError):
    pass


# ------------------------------------------------------------------ constants

FER_STATUS_OK, FER_STATUS_INVALID_ARGUMENT, FER_STATUS_NOT_FOUND, FER_STATUS_INTERNAL_ERROR = 0, 1, 2, 3
FER_MEMORY_CUSTOM_POOL, FER_MEMORY_CUDA_MALLOC, FER_MEMORY_CUDA_MANAGED, FER_MEMORY_AUTO = 0, 1, 2, 0xFFFFFFFF
(FER_DTYPE_F32, FER_DTYPE_F16, FER_DTYPE_BF16, FER_DTYPE_I8, FER_DTYPE_U8, FER_DTYPE_I16, FER_DTYPE_U16,
 FER_DTYPE_I32, FER_DTYPE_U32, FER_DTYPE_I64, FER_DTYPE_U64, FER_DTYPE_F64) = range(12)

FER_JIT_BACKEND_NVRTC, FER_JIT_BACKEND_AUTO = 0, 0xFFFFFFFF
FER_JIT_MODE_PERMISSIVE, FER_JIT_MODE_STRICT = 0, 1
FER_JIT_SOURCE_CUDA, FER_JIT_SOURCE_PTX = 0, 1
(FER_JIT_ARG_BUFFER, FER_JIT_ARG_SCALAR_I32, FER_JIT_ARG_SCALAR_U32, FER_JIT_ARG_SCALAR_I64,
 FER_JIT_ARG_SCALAR_U64, FER_JIT_ARG_SCALAR_F32, FER_JIT_ARG_SCALAR_F64) = range(7)
FER_JIT_ACCESS_READ, FER_JIT_ACCESS_WRITE, FER_JIT_ACCESS_READ_WRITE = 0, 1, 2
FER_JIT_WILDCARD_U32 = 0xFFFFFFFF
FER_JIT_WILDCARD_U64 = 0xFFFFFFFFFFFFFFFF

FER_JIT_INTENT_ABI_VERSION = 1
(FER_JIT_INTENT_OP_AFFINE_F32, FER_JIT_INTENT_OP_SOFTMAX_F32, FER_JIT_INTENT_OP_REDUCE_SUM_F32,
 FER_JIT_INTENT_OP_REDUCE_MAX_F32, FER_JIT_INTENT_OP_CONV2D_F32) = range(5)
FER_JIT_INTENT_FUSION_NONE = 0
FER_JIT_INTENT_FUSION_RELU = 1
FER_JIT_INTENT_FUSION_MUL_SIGMOID_INPUT = 2

FER_ROWS_SOFTMAX, FER_ROWS_LAYER_NORM, FER_ROWS_FAST = 1, 2, 4
(FER_CHAIN_LOAD, FER_CHAIN_AFFINE, FER_CHAIN_ADD_SCALAR, FER_CHAIN_MUL_SCALAR, FER_CHAIN_RELU, FER_CHAIN_SIGMOID,
 FER_CHAIN_EXP, FER_CHAIN_TANH, FER_CHAIN_GELU_TANH, FER_CHAIN_SILU, FER_CHAIN_NEG, FER_CHAIN_ABS, FER_CHAIN_CLAMP,
 FER_CHAIN_ADD, FER_CHAIN_SUB, FER_CHAIN_MUL, FER_CHAIN_DIV, FER_CHAIN_MAX, FER_CHAIN_MIN, FER_CHAIN_RELU_LT,
 FER_CHAIN_FMA) = range(21)

DTYPE_SIZE = {FER_DTYPE_F32: 4, FER_DTYPE_F16: 2, FER_DTYPE_BF16: 2, FER_DTYPE_I8: 1, FER_DTYPE_U8: 1,
              FER_DTYPE_I16: 2, FER_DTYPE_U16: 2, FER_DTYPE_I32: 4, FER_DTYPE_U32: 4, FER_DTYPE_I64: 8,
              FER_DTYPE_U64: 8, FER_DTYPE_F64: 8}

# ------------------------------------------------------------------ structs


class fer_status_t(C.Structure):
    _fields_ = [("code", C.c_int32), ("message", C.c_char_p)]


class fer_pool_config_t(C.Structure):
    _fields_ = [("mutable_bytes", C.c_uint64), ("immutable_bytes", C.c_uint64), ("cuda_reserve", C.c_uint64),
                ("verbose", C.c_uint8), ("memory_regime", C.c_uint32)]


class fer_buffer_desc_t(C.Structure):
    _fields_ = [("dtype", C.c_uint32), ("rank", C.c_uint32), ("dims", C.c_uint32 * 4), ("immutable", C.c_uint8),
                ("tag", C.c_uint32)]


class fer_matmul_request_t(C.Structure):
    _fields_ = [("a", C.c_uint64), ("b", C.c_uint64), ("out", C.c_uint64), ("memory_regime", C.c_uint32)]


class fer_layer_norm_request_t(C.Structure):
    _fields_ = [("x", C.c_uint64), ("out", C.c_uint64), ("eps", C.c_float), ("memory_regime", C.c_uint32)]


class fer_tensor_spec_t(C.Structure):
    _fields_ = [("dtype", C.c_uint32), ("rank", C.c_uint32), ("dims", C.c_uint32 * 4), ("immutable", C.c_uint8),
                ("tag", C.c_uint32), ("memory_regime", C.c_uint32)]


class fer_tensor_handle_t(C.Structure):
    _fields_ = [("id", C.c_uint64)]


ALLOC_FN = C.CFUNCTYPE(C.c_void_p, C.c_uint64, C.c_uint32, C.c_uint32, C.c_void_p)
FREE_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_void_p)
HOT_ALLOC_FN = C.CFUNCTYPE(C.c_void_p, C.c_void_p, C.c_uint64)
HOT_FREE_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_void_p)
DELETER_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_void_p)


class fer_custom_allocator_t(C.Structure):
    _fields_ = [("alloc", ALLOC_FN), ("free", FREE_FN), ("user_ctx", C.c_void_p)]


class fer_gpu_hot_allocator_t(C.Structure):
    _fields_ = [("runtime", C.c_void_p), ("alloc", HOT_ALLOC_FN), ("free", HOT_FREE_FN)]


class fer_jit_source_t(C.Structure):
    _fields_ = [("kind", C.c_uint32), ("code", C.c_char_p), ("code_len", C.c_size_t)]


class fer_jit_options_t(C.Structure):
    _fields_ = [("backend", C.c_uint32), ("mode", C.c_uint32), ("arch", C.c_char_p),
                ("extra_nvrtc_opts", C.c_char_p), ("cache_dir", C.c_char_p), ("enable_disk_cache", C.c_uint8)]


class fer_jit_compile_result_t(C.Structure):
    _fields_ = [("cache_hit", C.c_uint8), ("backend_name", C.c_char_p), ("log", C.c_char_p)]


class fer_jit_arg_desc_t(C.Structure):
    _fields_ = [("kind", C.c_uint32), ("access", C.c_uint32), ("name", C.c_char_p), ("expected_dtype", C.c_uint32),
                ("expected_rank", C.c_uint32), ("expected_bytes", C.c_uint64), ("expected_dims", C.c_uint32 * 4)]


class fer_jit_kernel_sig_t(C.Structure):
    _fields_ = [("args", C.POINTER(fer_jit_arg_desc_t)), ("arg_count", C.c_size_t)]


class fer_jit_launch_cfg_t(C.Structure):
    _fields_ = [("grid_x", C.c_uint32), ("grid_y", C.c_uint32), ("grid_z", C.c_uint32), ("block_x", C.c_uint32),
                ("block_y", C.c_uint32), ("block_z", C.c_uint32), ("shared_mem_bytes", C.c_uint32),
                ("memory_regime", C.c_uint32)]


class _argval(C.Union):
    _fields_ = [("buffer_id", C.c_uint64), ("i32", C.c_int32), ("u32", C.c_uint32), ("i64", C.c_int64),
                ("u64", C.c_uint64), ("f32", C.c_float), ("f64", C.c_double)]


class fer_jit_arg_value_t(C.Structure):
    _fields_ = [("kind", C.c_uint32), ("as_", _argval)]


class fer_jit_arg_pack_t(C.Structure):
    _fields_ = [("args", C.POINTER(fer_jit_arg_value_t)), ("arg_count", C.c_size_t)]


class fer_jit_stats_t(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("compile_count", "cache_hit_count", "launch_count", "compile_time_us",
                                          "launch_time_us", "disk_cache_entries", "disk_cache_bytes",
                                          "memory_cache_entries")]


class fer_jit_intent_t(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("abi_version", "op", "fusion_mask", "caps_mask", "memory_regime", "n")] + \
               [("alpha", C.c_float), ("beta", C.c_float)] + \
               [(n, C.c_uint32) for n in ("height", "width", "channels", "kernel_h", "kernel_w", "pad_h", "pad_w",
                                          "stride_h", "stride_w", "num_filters")]


class fer_jit_intent_bindings_t(C.Structure):
    _fields_ = [("input", C.c_uint64), ("output", C.c_uint64), ("weights", C.c_uint64), ("bias", C.c_uint64)]


class fer_rows_request_t(C.Structure):
    _fields_ = [("x", C.c_uint64), ("out", C.c_uint64), ("gamma", C.c_uint64), ("beta", C.c_uint64),
                ("eps", C.c_float), ("ops", C.c_uint32), ("memory_regime", C.c_uint32)]


class fer_chain_op_t(C.Structure):
    _fields_ = [("opcode", C.c_uint32), ("arg", C.c_uint32), ("p0", C.c_float), ("p1", C.c_float)]


class fer_gemm_request_t(C.Structure):
    _fields_ = [("a", C.c_uint64), ("b", C.c_uint64), ("out", C.c_uint64), ("flags", C.c_uint32),
                ("memory_regime", C.c_uint32)]


class fer_transformer_config_t(C.Structure):
    _fields_ = [("layers", C.c_uint32), ("d_model", C.c_uint32), ("heads", C.c_uint32), ("ffn", C.c_uint32),
                ("vocab", C.c_uint32), ("max_tokens", C.c_uint32), ("eps", C.c_float), ("reserved", C.c_uint32)]


class fer_transformer_profile_t(C.Structure):
    _fields_ = [("gemm_ms", C.c_double), ("attn_ms", C.c_double), ("norm_ms", C.c_double), ("other_ms", C.c_double),
                ("gemm_flops", C.c_double), ("attn_flops", C.c_double), ("forwards", C.c_uint64),
                ("launches", C.c_uint64)]


class fer_pool_stats_t(C.Structure):
    _fields_ = [("pool_bytes", C.c_uint64), ("allocated_bytes", C.c_uint64), ("peak_allocated_bytes", C.c_uint64),
                ("largest_free_block", C.c_uint64), ("total_allocations", C.c_uint64), ("total_frees", C.c_uint64),
                ("allocated_blocks", C.c_uint32), ("free_blocks", C.c_uint32)]


class TLSFPoolStats(C.Structure):
    _fields_ = [("total_pool_size", C.c_size_t), ("allocated_bytes", C.c_size_t), ("free_bytes", C.c_size_t),
                ("peak_allocated", C.c_size_t), ("largest_free_block", C.c_size_t),
                ("smallest_free_block", C.c_size_t), ("total_blocks", C.c_uint32), ("free_blocks", C.c_uint32),
                ("allocated_blocks", C.c_uint32), ("fallback_count", C.c_uint32),
                ("utilization_percent", C.c_float), ("fragmentation_ratio", C.c_float),
                ("external_fragmentation", C.c_float), ("free_list_counts", C.c_uint32 * 34),
                ("hash_collisions", C.c_uint32), ("max_chain_length", C.c_uint32), ("avg_chain_length", C.c_float),
                ("total_allocations", C.c_uint64), ("total_frees", C.c_uint64), ("total_splits", C.c_uint32),
                ("total_merges", C.c_uint32), ("is_healthy", C.c_bool), ("needs_defrag", C.c_bool)]


class TLSFHealthReport(C.Structure):
    _fields_ = [("is_valid", C.c_bool), ("has_memory_leaks", C.c_bool), ("has_corrupted_blocks", C.c_bool),
                ("has_broken_chains", C.c_bool), ("has_hash_errors", C.c_bool), ("error_count", C.c_int),
                ("error_messages", (C.c_char * 256) * 16)]


class GPUHotConfig(C.Structure):
    _fields_ = [("pool_fraction", C.c_float), ("fixed_pool_size", C.c_size_t), ("min_pool_size", C.c_size_t),
                ("max_pool_size", C.c_size_t), ("reserve_vram", C.c_size_t), ("enable_leak_detection", C.c_bool),
                ("enable_pool_health", C.c_bool), ("warning_threshold", C.c_float),
                ("force_daemon_mode", C.c_bool), ("quiet_init", C.c_bool), ("max_streams", C.c_uint),
                ("single_pool_strict", C.c_bool)]


# ------------------------------------------------------------------ prototypes

S = fer_status_t
P = C.c_void_p
u8, u32, u64, f32, sz = C.c_uint8, C.c_uint32, C.c_uint64, C.c_float, C.c_size_t
pu8, pu32, pu64, psz = C.POINTER(u8), C.POINTER(u32), C.POINTER(u64), C.POINTER(sz)

CAPI_PROTOTYPES = {
    # include/fercuda/api/c_api.h
    "fer_session_create": (S, [C.c_int32, C.POINTER(fer_pool_config_t), C.POINTER(P)]),
    "fer_session_destroy": (S, [P]),
    "fer_register_custom_allocator": (S, [P, u32, C.POINTER(fer_custom_allocator_t)]),
    "fer_register_gpu_hot_allocator": (S, [P, u32, C.POINTER(fer_gpu_hot_allocator_t)]),
    "fer_unregister_custom_allocator": (S, [P, u32]),
    "fer_set_default_memory_regime": (S, [P, u32]),
    "fer_get_default_memory_regime": (S, [P, pu32]),
    "fer_list_registered_regimes": (S, [P, pu32, sz, psz]),
    "fer_alloc_buffer": (S, [P, C.POINTER(fer_buffer_desc_t), pu64]),
    "fer_alloc_buffer_in_regime": (S, [P, C.POINTER(fer_buffer_desc_t), u32, pu64]),
    "fer_import_external_buffer": (S, [P, C.POINTER(fer_buffer_desc_t), P, u32, pu64]),
    "fer_import_external_buffer_with_deleter": (S, [P, C.POINTER(fer_buffer_desc_t), P, u32, DELETER_FN, P, pu64]),
    "fer_export_buffer_device_ptr": (S, [P, u64, C.POINTER(P)]),
    "fer_free_buffer": (S, [P, u64]),
    "fer_upload_f32": (S, [P, u64, P, sz]),
    "fer_download_f32": (S, [P, u64, P, sz]),
    "fer_upload_bytes": (S, [P, u64, P, sz]),
    "fer_download_bytes": (S, [P, u64, P, sz]),
    "fer_submit_matmul": (S, [P, C.POINTER(fer_matmul_request_t), pu64]),
    "fer_submit_layer_norm": (S, [P, C.POINTER(fer_layer_norm_request_t), pu64]),
    "fer_set_session_stream": (S, [P, u64]),
    "fer_get_session_stream": (S, [P, pu64]),
    "fer_job_status": (S, [P, u64, pu8]),
    "fer_job_wait": (S, [P, u64]),
    "fer_stream_attach": (S, [P, u64]),
    "fer_stream_current": (S, [P, pu64]),
    "fer_tensor_create": (S, [P, C.POINTER(fer_tensor_spec_t), C.POINTER(fer_tensor_handle_t)]),
    "fer_tensor_attach_external": (S, [P, C.POINTER(fer_tensor_spec_t), P, DELETER_FN, P,
                                       C.POINTER(fer_tensor_handle_t)]),
    "fer_tensor_device_ptr": (S, [P, fer_tensor_handle_t, C.POINTER(P)]),
    "fer_tensor_release": (S, [P, fer_tensor_handle_t]),
    "fer_tensor_upload": (S, [P, fer_tensor_handle_t, P, sz]),
    "fer_tensor_download": (S, [P, fer_tensor_handle_t, P, sz]),
    "fer_tensor_run_affine_f32": (S, [P, fer_tensor_handle_t, fer_tensor_handle_t, u32, f32, f32, u32, u32, u32, pu64]),
    # include/fercuda/jit/api.h, intent/intent.h
    "fer_jit_compile": (S, [P, C.POINTER(fer_jit_source_t), C.POINTER(fer_jit_options_t), C.POINTER(P),
                            C.POINTER(fer_jit_compile_result_t)]),
    "fer_jit_release_program": (S, [P, P]),
    "fer_jit_get_kernel": (S, [P, P, C.c_char_p, C.POINTER(fer_jit_kernel_sig_t), C.POINTER(P)]),
    "fer_jit_release_kernel": (S, [P, P]),
    "fer_jit_launch": (S, [P, P, C.POINTER(fer_jit_launch_cfg_t), C.POINTER(fer_jit_arg_pack_t), pu64]),
    "fer_jit_cache_clear": (S, [P]),
    "fer_jit_get_stats": (S, [P, C.POINTER(fer_jit_stats_t)]),
    "fer_jit_run_intent": (S, [P, C.POINTER(fer_jit_intent_t), C.POINTER(fer_jit_intent_bindings_t), pu64]),
    # include/fercuda/b200/ext.h
    "fer_submit_rows": (S, [P, C.POINTER(fer_rows_request_t), pu64]),
    "fer_jit_run_chain_f32": (S, [P, C.POINTER(fer_chain_op_t), u32, pu64, u32, u64, pu64]),
    "fer_submit_gemm": (S, [P, C.POINTER(fer_gemm_request_t), pu64]),
    "fer_transformer_create": (S, [P, C.POINTER(fer_transformer_config_t), pu64]),
    "fer_transformer_init_weights": (S, [P, u64, u64, f32]),
    "fer_transformer_weight_buffer": (S, [P, u64, pu64]),
    "fer_transformer_forward": (S, [P, u64, u64, u64, pu64]),
    "fer_transformer_forward_host": (S, [P, u64, P, u32, u32, P, u32]),
    "fer_transformer_destroy": (S, [P, u64]),
    "fer_transformer_profile": (S, [P, u64, u32]),
    "fer_transformer_profile_read": (S, [P, u64, C.POINTER(fer_transformer_profile_t)]),
    "fer_transformer_kv_create": (S, [P, u64, u32, u32, pu64]),
    "fer_transformer_kv_destroy": (S, [P, u64, u64]),
    "fer_transformer_kv_length": (S, [P, u64, u64, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]),
    "fer_transformer_prefill": (S, [P, u64, u64, u64, u64, pu64]),
    "fer_transformer_decode": (S, [P, u64, u64, u64, u64, pu64]),
    "fer_session_device_errors": (S, [P, pu32, u8]),
    "fer_pool_get_stats": (S, [P, C.POINTER(fer_pool_stats_t)]),
    "fer_pool_alloc_raw": (S, [P, u64, C.POINTER(P)]),
    "fer_pool_free_raw": (S, [P, P]),
    "fer_comm_unique_id": (S, [pu8]),
    "fer_comm_init": (S, [P, pu8, C.c_int32, C.c_int32, u32]),
    "fer_comm_destroy": (S, [P]),
    "fer_transformer_broadcast_weights": (S, [P, u64, C.c_int32, pu64]),
    "fer_transformer_shard": (S, [u32, C.c_int32, C.c_int32, pu32, pu32]),
    "fer_buffer_row_digests": (S, [P, u64, u64, u32, pu64]),
}

CORE_PROTOTYPES = {
    # include/ptx/memory/ptx_tlsf_allocator.h
    "ptx_tlsf_create": (P, [sz, C.c_bool]),
    "ptx_tlsf_create_from_pool": (P, [P, sz, C.c_bool]),
    "ptx_tlsf_destroy": (None, [P]),
    "ptx_tlsf_alloc": (P, [P, sz]),
    "ptx_tlsf_alloc_debug": (P, [P, sz, C.c_char_p, C.c_int]),
    "ptx_tlsf_free": (None, [P, P]),
    "ptx_tlsf_realloc": (P, [P, P, sz]),
    "ptx_tlsf_alloc_owned": (P, [P, sz, u32]),
    "ptx_tlsf_free_owner": (None, [P, u32]),
    "ptx_tlsf_get_owner_stats": (None, [P, P]),
    "ptx_tlsf_get_events": (None, [P, P]),
    "ptx_tlsf_get_stats": (None, [P, C.POINTER(TLSFPoolStats)]),
    "ptx_tlsf_validate": (None, [P, C.POINTER(TLSFHealthReport)]),
    "ptx_tlsf_can_allocate": (C.c_bool, [P, sz]),
    "ptx_tlsf_get_max_allocatable": (sz, [P]),
    "ptx_tlsf_owns_ptr": (C.c_bool, [P, P]),
    "ptx_tlsf_get_block_info": (C.c_bool, [P, P, psz, C.POINTER(C.c_bool)]),
    "ptx_tlsf_pin_block": (None, [P, P]),
    "ptx_tlsf_unpin_block": (None, [P, P]),
    "ptx_tlsf_defragment": (None, [P]),
    "ptx_tlsf_compact": (None, [P]),
    "ptx_tlsf_reset_stats": (None, [P]),
    "ptx_tlsf_set_warning_threshold": (None, [P, f32]),
    "ptx_tlsf_set_warnings_enabled": (None, [P, C.c_bool]),
    # include/ptx/gpu/gpu_hot_runtime.h
    "gpu_hot_default_config": (GPUHotConfig, []),
    "gpu_hot_init": (P, [C.c_int, C.c_char_p]),
    "gpu_hot_init_with_config": (P, [C.c_int, C.c_char_p, C.POINTER(GPUHotConfig)]),
    "gpu_hot_shutdown": (None, [P]),
    "gpu_hot_alloc": (P, [P, sz]),
    "gpu_hot_free": (None, [P, P]),
    "gpu_hot_alloc_async": (P, [P, sz, P]),
    "gpu_hot_free_async": (None, [P, P, P]),
    "gpu_hot_poll_deferred": (None, [P, C.c_int]),
    "gpu_hot_can_allocate": (C.c_bool, [P, sz]),
    "gpu_hot_get_max_allocatable": (sz, [P]),
    "gpu_hot_owns_ptr": (C.c_bool, [P, P]),
    "gpu_hot_alloc_owned": (P, [P, sz, u32]),
    "gpu_hot_free_owner": (None, [P, u32]),
    "gpu_hot_get_owner_stats": (None, [P, P]),
    "gpu_hot_get_alloc_events": (None, [P, P]),
    "gpu_hot_get_stream": (P, [P, C.c_int]),
    "gpu_hot_get_tlsf_stats": (None, [P, C.POINTER(TLSFPoolStats)]),
    "gpu_hot_validate_tlsf_pool": (None, [P, C.POINTER(TLSFHealthReport)]),
}

KERNEL_PROTOTYPES = {
    # include/ptx/gpu/tensor_ops.h
    "ptx_tensor_add_f32": (None, [P, P, P, sz, P]),
    "ptx_tensor_mul_f32": (None, [P, P, P, sz, P]),
    "ptx_tensor_relu_f32": (None, [P, P, sz, P]),
    "ptx_tensor_sigmoid_f32": (None, [P, P, sz, P]),
    "ptx_tensor_affine_f32": (None, [P, P, sz, f32, f32, P]),
    "ptx_tensor_softmax_f32": (None, [P, P, sz, sz, P]),
    "ptx_tensor_softmax_layer_norm_f32": (None, [P, P, P, P, sz, sz, f32, P]),
    "ptx_tensor_layer_norm_rows_f32": (None, [P, P, P, P, sz, sz, f32, P]),
    "ptx_tensor_reduce_f32_noalloc": (C.c_int, [P, P, sz, C.c_int, P]),
    # include/fercuda/b200/ext.h (native launchers)
    "fer_fill_normal_bf16": (C.c_int, [P, sz, u64, f32, P]),
}

_LIBS: dict[str, C.CDLL] = {}


def _bind(lib: C.CDLL, protos: dict) -> None:
    for name, (res, args) in protos.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def _load(name: str, protos: dict) -> C.CDLL:
    if name in _LIBS:
        return _LIBS[name]
    path = LIBDIR / name
    if not path.exists():
        raise FerNativeError(f"{path} is not built; run `make -C fercuda_b200/csrc` (or __graft_entry__.build())")
    lib = C.CDLL(str(path))
    _bind(lib, protos)
    _LIBS[name] = lib
    return lib


def core() -> C.CDLL:
    return _load("libptx_core.so", CORE_PROTOTYPES)


def kernels() -> C.CDLL:
    return _load("libptx_kernels.so", KERNEL_PROTOTYPES)


def capi() -> C.CDLL:
    core()
    kernels()
    return _load("libfercuda_capi.so", CAPI_PROTOTYPES)


def lib_paths() -> list[str]:
    return [str(LIBDIR / n) for n in ("libfercuda_capi.so", "libptx_core.so", "libptx_kernels.so")]


# ------------------------------------------------------------------ helpers


class FerError(RuntimeError):
    def __init__(self, fn: str, st: fer_status_t):
        self.code = st.code
        self.msg = (st.message or b"").decode()
        super().__init__(f"{fn} -> code {st.code}: {self.msg}")


def check(fn: str, st: fer_status_t) -> None:
    if st.code != FER_STATUS_OK:
        raise FerError(fn, st)


def desc(dtype: int, shape, immutable: bool = False, tag: int = 0) -> fer_buffer_desc_t:
    d = fer_buffer_desc_t()
    d.dtype = dtype
    d.rank = len(shape)
    for i, s in enumerate(shape):
        d.dims[i] = int(s)
    d.immutable = 1 if immutable else 0
    d.tag = tag
    return d


COMM_UNIQUE_ID_BYTES = 128


def comm_unique_id() -> bytes:
    """fer_comm_unique_id: a fresh NCCL unique id (one rank makes it)."""
    buf = (C.c_uint8 * COMM_UNIQUE_ID_BYTES)()
    check("fer_comm_unique_id", capi().fer_comm_unique_id(buf))
    return bytes(buf)


def transformer_shard(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """fer_transformer_shard: (first sequence, count) of rank's shard."""
    first, count = C.c_uint32(), C.c_uint32()
    check("fer_transformer_shard", capi().fer_transformer_shard(global_batch, world, rank, C.byref(first),
                                                                C.byref(count)))
    return first.value, count.value


class Session:
    """Thin owner of a fer_session_t* with the calls the tests and the bench need."""

    def __init__(self, device: int = 0, pool_bytes: int = 256 << 20, regime: int = FER_MEMORY_CUSTOM_POOL):
        self.lib = capi()
        cfg = fer_pool_config_t()
        cfg.mutable_bytes = pool_bytes // 2
        cfg.immutable_bytes = pool_bytes - pool_bytes // 2
        cfg.memory_regime = regime
        self.ptr = C.c_void_p()
        check("fer_session_create", self.lib.fer_session_create(device, C.byref(cfg), C.byref(self.ptr)))

    def close(self) -> None:
        if self.ptr:
            check("fer_session_destroy", self.lib.fer_session_destroy(self.ptr))
            self.ptr = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def call(self, name: str, *args) -> fer_status_t:
        return getattr(self.lib, name)(self.ptr, *args)

    def alloc(self, dtype: int, shape, regime: int = FER_MEMORY_AUTO, immutable: bool = False) -> int:
        bid = C.c_uint64()
        d = desc(dtype, shape, immutable)
        check("fer_alloc_buffer_in_regime", self.call("fer_alloc_buffer_in_regime", C.byref(d), regime, C.byref(bid)))
        return bid.value

    def free(self, bid: int) -> None:
        check("fer_free_buffer", self.call("fer_free_buffer", bid))

    def ptr_of(self, bid: int) -> int:
        p = C.c_void_p()
        check("fer_export_buffer_device_ptr", self.call("fer_export_buffer_device_ptr", bid, C.byref(p)))
        return p.value or 0

    def upload(self, bid: int, arr) -> None:
        check("fer_upload_bytes", self.call("fer_upload_bytes", bid, arr.ctypes.data_as(C.c_void_p), arr.nbytes))

    def download(self, bid: int, arr) -> None:
        check("fer_download_bytes", self.call("fer_download_bytes", bid, arr.ctypes.data_as(C.c_void_p), arr.nbytes))

    def wait(self, job: int) -> None:
        check("fer_job_wait", self.call("fer_job_wait", job))

    def stream(self) -> int:
        s = C.c_uint64()
        check("fer_get_session_stream", self.call("fer_get_session_stream", C.byref(s)))
        return s.value

    def comm_init(self, uid: bytes, rank: int, world: int, timeout_ms: int = 0) -> None:
        buf = (C.c_uint8 * COMM_UNIQUE_ID_BYTES).from_buffer_copy(uid)
        check("fer_comm_init", self.call("fer_comm_init", buf, rank, world, timeout_ms))

    def comm_destroy(self) -> None:
        check("fer_comm_destroy", self.call("fer_comm_destroy"))

    def row_digests(self, bid: int, row_bytes: int, rows: int) -> list[int]:
        out = (C.c_uint64 * rows)()
        check("fer_buffer_row_digests", self.call("fer_buffer_row_digests", bid, row_bytes, rows, out))
        return list(out)

    def device_errors(self, clear: bool = True) -> int:
        v = C.c_uint32()
        check("fer_session_device_errors", self.call("fer_session_device_errors", C.byref(v), 1 if clear else 0))
        return v.value

    def rows(self, x: int, out: int, ops: int, eps: float = 1e-5, gamma: int = 0, beta: int = 0) -> int:
        r = fer_rows_request_t(x, out, gamma, beta, eps, ops, FER_MEMORY_AUTO)
        job = C.c_uint64()
        check("fer_submit_rows", self.call("fer_submit_rows", C.byref(r), C.byref(job)))
        return job.value

    def affine(self, x: int, out: int, n: int, alpha: float, beta: float, fusion: int) -> int:
        job = C.c_uint64()
        check("fer_tensor_run_affine_f32",
              self.call("fer_tensor_run_affine_f32", fer_tensor_handle_t(x), fer_tensor_handle_t(out), n, alpha, beta,
                        fusion, 0, FER_MEMORY_AUTO, C.byref(job)))
        return job.value

    def matmul(self, a: int, b: int, out: int) -> int:
        r = fer_matmul_request_t(a, b, out, FER_MEMORY_AUTO)
        job = C.c_uint64()
        check("fer_submit_matmul", self.call("fer_submit_matmul", C.byref(r), C.byref(job)))
        return job.value

    def gemm(self, a: int, b: int, out: int) -> int:
        r = fer_gemm_request_t(a, b, out, 0, FER_MEMORY_AUTO)
        job = C.c_uint64()
        check("fer_submit_gemm", self.call("fer_submit_gemm", C.byref(r), C.byref(job)))
        return job.value

    def import_ptr(self, dtype: int, shape, ptr: int) -> int:
        """Registers external device memory (e.g. a torch tensor) as a buffer."""
        bid = C.c_uint64()
        d = desc(dtype, shape)
        check("fer_import_external_buffer",
              self.call("fer_import_external_buffer", C.byref(d), C.c_void_p(ptr), FER_MEMORY_AUTO, C.byref(bid)))
        return bid.value

    def chain(self, ops, inputs, out: int) -> int:
        arr = (fer_chain_op_t * len(ops))(*[fer_chain_op_t(*o) for o in ops])
        ins = (C.c_uint64 * len(inputs))(*inputs)
        job = C.c_uint64()
        check("fer_jit_run_chain_f32",
              self.call("fer_jit_run_chain_f32", arr, len(ops), ins, len(inputs), out, C.byref(job)))
        return job.value


class Transformer:
    """A model of fer_transformer_* owned by a Session."""

    def __init__(self, session: "Session", layers, d_model, heads, ffn, vocab, max_tokens, eps=1e-5):
        self.s = session
        self.cfg = fer_transformer_config_t(layers, d_model, heads, ffn, vocab, max_tokens, eps, 0)
        mid = C.c_uint64()
        check("fer_transformer_create", session.call("fer_transformer_create", C.byref(self.cfg), C.byref(mid)))
        self.id = mid.value

    def init_weights(self, seed: int, stddev: float = 0.02) -> None:
        check("fer_transformer_init_weights", self.s.call("fer_transformer_init_weights", self.id, seed, stddev))

    def weight_elements(self) -> int:
        """bf16 elements of the weight buffer: embedding [V, d], then per layer
        Wqkv [d, 3d], Wo [d, d], W1 [d, F], W2 [F, d], then the LM head [d, V],
        each tensor starting on a 128-element boundary."""
        up = lambda n: (n + 127) & ~127
        c = self.cfg
        d, F, V = c.d_model, c.ffn, c.vocab
        off = up(V * d)
        for _ in range(c.layers):
            off = up(off + 3 * d * d)
            off = up(off + d * d)
            off = up(off + d * F)
            off = up(off + F * d)
        return up(off + d * V)

    def weight_buffer(self) -> int:
        b = C.c_uint64()
        check("fer_transformer_weight_buffer", self.s.call("fer_transformer_weight_buffer", self.id, C.byref(b)))
        return b.value

    def broadcast_weights(self, root: int = 0) -> int:
        """fer_transformer_broadcast_weights over the session's communicator;
        returns the bytes broadcast."""
        n = C.c_uint64()
        check("fer_transformer_broadcast_weights",
              self.s.call("fer_transformer_broadcast_weights", self.id, root, C.byref(n)))
        return n.value

    def forward(self, tokens: int, logits: int) -> int:
        job = C.c_uint64()
        check("fer_transformer_forward", self.s.call("fer_transformer_forward", self.id, tokens, logits, C.byref(job)))
        return job.value

    def forward_host(self, tokens: np.ndarray, logits: np.ndarray, chunk_seqs: int = 0) -> None:
        """fer_transformer_forward_host: host i32 tokens [batch, seq] in, host
        f32 logits [batch, seq, vocab] (any C-contiguous shape of that size)
        out, the D2H copy of each chunk of sequences overlapped with the
        next chunk's forward. Returns when the logits are in `logits`."""
        if tokens.dtype != np.int32 or tokens.ndim != 2 or not tokens.flags.c_contiguous:
            raise ValueError("tokens must be a C-contiguous int32 [batch, seq] array")
        if logits.dtype != np.float32 or not logits.flags.c_contiguous or not logits.flags.writeable:
            raise ValueError("logits must be a writeable C-contiguous float32 array")
        b, n = tokens.shape
        if logits.size != b * n * self.cfg.vocab:
            raise ValueError(f"logits must hold batch x seq x vocab = {b * n * self.cfg.vocab} floats")
        check("fer_transformer_forward_host",
              self.s.call("fer_transformer_forward_host", self.id, tokens.ctypes.data, b, n, logits.ctypes.data,
                          chunk_seqs))

    def kv_create(self, max_batch: int, max_seq: int) -> int:
        cid = C.c_uint64()
        check("fer_transformer_kv_create",
              self.s.call("fer_transformer_kv_create", self.id, max_batch, max_seq, C.byref(cid)))
        return cid.value

    def kv_destroy(self, cache: int) -> None:
        check("fer_transformer_kv_destroy", self.s.call("fer_transformer_kv_destroy", self.id, cache))

    def kv_length(self, cache: int) -> tuple[int, int]:
        b, n = C.c_uint32(), C.c_uint32()
        check("fer_transformer_kv_length", self.s.call("fer_transformer_kv_length", self.id, cache, C.byref(b),
                                                       C.byref(n)))
        return b.value, n.value

    def prefill(self, cache: int, tokens: int, logits: int) -> int:
        job = C.c_uint64()
        check("fer_transformer_prefill",
              self.s.call("fer_transformer_prefill", self.id, cache, tokens, logits, C.byref(job)))
        return job.value

    def decode(self, cache: int, tokens: int, logits: int) -> int:
        job = C.c_uint64()
        check("fer_transformer_decode", self.s.call("fer_transformer_decode", self.id, cache, tokens, logits,
                                                    C.byref(job)))
        return job.value

    def profile(self, enable: bool) -> None:
        check("fer_transformer_profile", self.s.call("fer_transformer_profile", self.id, 1 if enable else 0))

    def profile_read(self) -> fer_transformer_profile_t:
        p = fer_transformer_profile_t()
        check("fer_transformer_profile_read", self.s.call("fer_transformer_profile_read", self.id, C.byref(p)))
        return p

    def close(self) -> None:
        if self.id:
            check("fer_transformer_destroy", self.s.call("fer_transformer_destroy", self.id))
            self.id = 0


def config1_chain(a: float, b: float):
    """y = relu(a*x + b) * sigmoid(x) as a chain program."""
    return [(FER_CHAIN_LOAD, 0, 0.0, 0.0), (FER_CHAIN_AFFINE, 0, a, b), (FER_CHAIN_RELU, 0, 0.0, 0.0),
            (FER_CHAIN_LOAD, 0, 0.0, 0.0), (FER_CHAIN_SIGMOID, 0, 0.0, 0.0), (FER_CHAIN_MUL, 0, 0.0, 0.0)]


os.environ.setdefault("FERCUDA_LIBDIR", str(LIBDIR))
