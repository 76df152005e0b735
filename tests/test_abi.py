"""The drop-in boundary on CPU: the libraries load without a GPU, export every
entry point the public headers declare, keep the reference's struct layouts,
and fail loudly (no CPU fallback) when no GPU is present."""
import ctypes as C
import re
import subprocess
import tempfile
from pathlib import Path

import pytest

from fercuda_b200 import capi

ROOT = Path(__file__).resolve().parents[1]
HEADERS = {
    "libfercuda_capi.so": ["include/fercuda/api/c_api.h", "include/fercuda/jit/api.h",
                           "include/fercuda/jit/intent/intent.h", "include/fercuda/b200/ext.h"],
    "libptx_core.so": ["include/ptx/memory/ptx_tlsf_allocator.h", "include/ptx/gpu/gpu_hot_runtime.h"],
    "libptx_kernels.so": ["include/ptx/gpu/tensor_ops.h", "include/fercuda/b200/native.h"],
    "libptx_hook.so": ["include/ptx/ptx_hook.h"],
}


def _reference_dir() -> Path:
    """$FERCUDA_REFERENCE_DIR, else oracle/Makefile's default (absent on a GPU box)."""
    import os

    env = os.environ.get("FERCUDA_REFERENCE_DIR")
    if env:
        return Path(env)
    out = subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), "print-ref"], capture_output=True, text=True)
    return Path(out.stdout.strip() or "/nonexistent")


REFERENCE = _reference_dir()


def declared(header: Path) -> list[str]:
    text = header.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    text = re.sub(r"static inline[^{]*\{.*?\n\}", "", text, flags=re.S)
    text = re.sub(r"#define[^\n]*(\\\n[^\n]*)*", "", text)
    text = re.sub(r"typedef[^;{]*;", "", text)
    names = re.findall(r"\b([A-Za-z_][A-Za-z0-9_]*)\s*\([^;{]*\)\s*;", text)
    return [n for n in names if n not in ("sizeof",)]


@pytest.mark.parametrize("lib", sorted(HEADERS))
def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(capi.LIBDIR / lib)], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    names = [n for h in HEADERS[lib] for n in declared(ROOT / h)]
    assert len(names) >= 4
    missing = sorted(set(names) - exported)
    assert not missing, missing


def test_bindings_load_and_match_prototypes():
    lib = capi.capi()
    for name in capi.CAPI_PROTOTYPES:
        assert hasattr(lib, name)
    core = capi.core()
    for name in capi.CORE_PROTOTYPES:
        assert hasattr(core, name)
    k = capi.kernels()
    for name in capi.KERNEL_PROTOTYPES:
        assert hasattr(k, name)


LAYOUT_PROBE = r"""
#include <stdio.h>
#include <stddef.h>
#include "fercuda/api/c_api.h"
#include "fercuda/jit/api.h"
#define S(t) printf(#t " %zu\n", sizeof(t));
#define O(t, f) printf(#t "." #f " %zu\n", offsetof(t, f));
int main(void) {
  S(fer_status_t) S(fer_pool_config_t) S(fer_buffer_desc_t) S(fer_matmul_request_t)
  S(fer_layer_norm_request_t) S(fer_tensor_spec_t) S(fer_tensor_handle_t) S(fer_custom_allocator_t)
  S(fer_gpu_hot_allocator_t) S(fer_jit_source_t) S(fer_jit_options_t) S(fer_jit_compile_result_t)
  S(fer_jit_arg_desc_t) S(fer_jit_kernel_sig_t) S(fer_jit_launch_cfg_t) S(fer_jit_arg_value_t)
  S(fer_jit_arg_pack_t) S(fer_jit_stats_t) S(fer_jit_intent_t) S(fer_jit_intent_bindings_t)
  O(fer_buffer_desc_t, tag) O(fer_pool_config_t, memory_regime) O(fer_jit_arg_desc_t, expected_dims)
  O(fer_jit_intent_t, alpha) O(fer_jit_intent_t, num_filters) O(fer_tensor_spec_t, memory_regime)
  O(fer_jit_options_t, enable_disk_cache)
  printf("FER_JIT_INTENT_ABI_VERSION %u\n", (unsigned)FER_JIT_INTENT_ABI_VERSION);
  printf("FER_DTYPE_F64 %d\n", (int)FER_DTYPE_F64);
  printf("FER_MEMORY_AUTO %u\n", (unsigned)FER_MEMORY_AUTO);
  return 0;
}
"""


def probe_layout(include_dir: Path) -> str:
    with tempfile.TemporaryDirectory() as d:
        src = Path(d) / "probe.c"
        exe = Path(d) / "probe"
        src.write_text(LAYOUT_PROBE)
        subprocess.run(["gcc", "-std=c11", f"-I{include_dir}", str(src), "-o", str(exe)], check=True)
        return subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout


def test_struct_layouts_match_ctypes():
    lines = dict(line.rsplit(" ", 1) for line in probe_layout(ROOT / "include").splitlines())
    for name in ("fer_status_t", "fer_pool_config_t", "fer_buffer_desc_t", "fer_jit_arg_desc_t", "fer_jit_intent_t",
                 "fer_jit_launch_cfg_t", "fer_jit_arg_value_t", "fer_jit_options_t", "fer_tensor_spec_t"):
        assert int(lines[name]) == C.sizeof(getattr(capi, name)), name


@pytest.mark.skipif(not REFERENCE.is_dir(), reason="reference headers not present")
def test_struct_layouts_identical_to_reference_headers():
    """Same sizes, offsets and enum values as the reference's own headers."""
    assert probe_layout(ROOT / "include") == probe_layout(REFERENCE / "include")


def test_session_create_fails_loudly_without_gpu():
    try:
        import torch

        if torch.cuda.is_available():
            pytest.skip("GPU present")
    except Exception:
        pass
    lib = capi.capi()
    s = C.c_void_p()
    st = lib.fer_session_create(0, None, C.byref(s))
    assert st.code == capi.FER_STATUS_INTERNAL_ERROR and not s.value


def test_null_arguments():
    lib = capi.capi()
    assert lib.fer_session_create(0, None, None).code == capi.FER_STATUS_INVALID_ARGUMENT
    assert lib.fer_alloc_buffer(None, None, None).code == capi.FER_STATUS_INVALID_ARGUMENT
    assert lib.fer_jit_run_intent(None, None, None, None).code == capi.FER_STATUS_INVALID_ARGUMENT
    assert lib.fer_submit_rows(None, None, None).code == capi.FER_STATUS_INVALID_ARGUMENT
    assert lib.fer_session_destroy(None).code == capi.FER_STATUS_OK
