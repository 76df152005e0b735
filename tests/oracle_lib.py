"""Loader for the oracle (test infrastructure): oracle/liboracle.so, the CPU
restatement of the reference algorithms, and oracle/_ref/*.so, the
reference's own sources compiled in place by oracle/Makefile."""
from __future__ import annotations

import ctypes as C
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
ORACLE = ROOT / "oracle"
REF = ORACLE / "_ref"

_cache: dict[str, C.CDLL] = {}

P = C.c_void_p


def load() -> C.CDLL:
    if "orc" in _cache:
        return _cache["orc"]
    lib = C.CDLL(str(ORACLE / "liboracle.so"))
    sz, f, i = C.c_size_t, C.c_float, C.c_int
    lib.orc_chain_f32.argtypes = [P, P, sz, f, f, i]
    lib.orc_affine_intent_f32.argtypes = [P, P, sz, f, f, i]
    lib.orc_softmax_rows_f32.argtypes = [P, P, sz, sz, i]
    lib.orc_layer_norm_f32.argtypes = [P, P, sz, f]
    lib.orc_softmax_layernorm_rows_f32.argtypes = [P, P, sz, sz, f, i]
    lib.orc_matmul_f32.argtypes = [P, P, P, i, i, i, i, i, i]
    lib.orc_matmul_bf16_tile.argtypes = [P, P, P, i, i, i, i, i, i, i]
    lib.orc_tlsf_create.restype = P
    lib.orc_tlsf_create.argtypes = [C.c_uint64]
    lib.orc_tlsf_destroy.argtypes = [P]
    lib.orc_tlsf_alloc.restype = C.c_uint64
    lib.orc_tlsf_alloc.argtypes = [P, C.c_uint64]
    lib.orc_tlsf_free.argtypes = [P, C.c_uint64]
    lib.orc_tlsf_allocated_bytes.restype = C.c_uint64
    lib.orc_tlsf_allocated_bytes.argtypes = [P]
    lib.orc_tlsf_block_count.restype = C.c_uint32
    lib.orc_tlsf_block_count.argtypes = [P]
    _cache["orc"] = lib
    return lib


def ref_tlsf() -> C.CDLL | None:
    path = REF / "libref_tlsf.so"
    if not path.exists():
        return None
    if "tlsf" not in _cache:
        lib = C.CDLL(str(path))
        lib.ptx_tlsf_create_from_pool.restype = P
        lib.ptx_tlsf_create_from_pool.argtypes = [P, C.c_size_t, C.c_bool]
        lib.ptx_tlsf_alloc.restype = P
        lib.ptx_tlsf_alloc.argtypes = [P, C.c_size_t]
        lib.ptx_tlsf_free.argtypes = [P, P]
        lib.ptx_tlsf_destroy.argtypes = [P]
        _cache["tlsf"] = lib
    return _cache["tlsf"]


def ref_kernels() -> C.CDLL | None:
    path = REF / "libref_kernels.so"
    if not path.exists():
        return None
    if "kern" not in _cache:
        lib = C.CDLL(str(path))
        sz, f, i = C.c_size_t, C.c_float, C.c_int
        lib.ptx_tensor_affine_f32.argtypes = [P, P, sz, f, f, P]
        lib.ptx_tensor_relu_f32.argtypes = [P, P, sz, P]
        lib.ptx_tensor_sigmoid_f32.argtypes = [P, P, sz, P]
        lib.ptx_tensor_mul_f32.argtypes = [P, P, P, sz, P]
        lib.ptx_tensor_add_f32.argtypes = [P, P, P, sz, P]
        lib.ptx_tensor_softmax_f32.argtypes = [P, P, sz, sz, P]
        lib.refshim_matmul_f32.argtypes = [P, P, P, i, i, i, P]
        lib.refshim_layer_norm_f32.argtypes = [P, P, i, f, P]
        _cache["kern"] = lib
    return _cache["kern"]


def ptr(a) -> C.c_void_p:
    return a.ctypes.data_as(C.c_void_p)
