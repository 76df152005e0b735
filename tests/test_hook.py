"""libptx_hook.so, the LD_PRELOAD allocation interposer, on the CPU.

The hook is preloaded into a small C program (tests/hook/hook_driver.c) that
links a stand-in for the CUDA runtime and driver (tests/hook/fake_cuda.c,
host memory); a second preloaded library (tests/hook/fake_hot.c) serves the
hook's gpu_hot_* calls from a host range carved by libptx_core.so's own TLSF
allocator. The checks follow the reference interposer
(native/core/hooks/cuda_intercept.c): which calls the pool serves in each
PTX_HOOK_MODE, the fallbacks when the pool cannot be made, 256-byte pitches,
and refusal of foreign frees in tlsf mode. The same driver runs against the
real CUDA libraries in tests/test_gpu_hook.py.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import pytest

from fercuda_b200 import capi

HERE = Path(__file__).resolve().parent / "hook"
CUDA_INC = "/usr/local/cuda/include"
HOOK = capi.LIBDIR / "libptx_hook.so"

INTERPOSED = [
    "cudaMalloc", "cudaFree", "cudaMallocAsync", "cudaFreeAsync", "cudaMallocFromPoolAsync", "cudaMallocManaged",
    "cudaMallocPitch", "cudaMallocHost", "cudaHostAlloc", "cudaFreeHost", "cuMemAlloc", "cuMemAlloc_v2",
    "cuMemFree", "cuMemFree_v2", "cuMemAllocAsync", "cuMemFreeAsync", "cuMemAllocManaged", "cuMemAllocPitch",
    "cuMemAllocPitch_v2", "cuMemAllocFromPoolAsync",
]


def _cc(args: list[str]) -> None:
    subprocess.run(["gcc", "-O1", "-Wall", "-Werror", *args], check=True, capture_output=True, text=True)


@pytest.fixture(scope="module")
def fakes(tmp_path_factory) -> Path:
    d = tmp_path_factory.mktemp("hook")
    _cc(["-shared", "-fPIC", "-o", str(d / "libfake_cuda.so"), str(HERE / "fake_cuda.c")])
    _cc(["-shared", "-fPIC", "-o", str(d / "libfake_hot.so"), str(HERE / "fake_hot.c"), f"-L{capi.LIBDIR}",
         "-lptx_core", f"-Wl,-rpath,{capi.LIBDIR}"])
    _cc([f"-I{CUDA_INC}", "-o", str(d / "hook_driver"), str(HERE / "hook_driver.c"), f"-L{d}", "-lfake_cuda",
         f"-Wl,-rpath,{d}", "-ldl"])
    return d


def run(fakes: Path, scenario: str, preload: bool = True, **env) -> subprocess.CompletedProcess:
    e = {k: v for k, v in os.environ.items() if not k.startswith(("PTX_", "FAKE_"))}
    e.pop("LD_PRELOAD", None)
    if preload:
        e["LD_PRELOAD"] = f"{HOOK} {fakes / 'libfake_hot.so'}"
    e.update(env)
    r = subprocess.run([str(fakes / "hook_driver"), scenario], env=e, capture_output=True, text=True, timeout=60)
    assert "FAIL" not in r.stdout, r.stdout + r.stderr
    assert r.returncode == 0, r.stdout + r.stderr
    return r


def test_hook_exports_every_interposed_entry_point():
    lib = C.CDLL(str(HOOK))
    for name in INTERPOSED + ["ptx_hook_set_thread_mode", "ptx_hook_get_thread_mode", "ptx_hook_get_stats",
                              "ptx_hook_get_runtime"]:
        assert hasattr(lib, name), name


def test_thread_mode_round_trips():
    lib = C.CDLL(str(HOOK))
    assert lib.ptx_hook_get_thread_mode() == 0
    lib.ptx_hook_set_thread_mode(2)
    assert lib.ptx_hook_get_thread_mode() == 2
    lib.ptx_hook_set_thread_mode(0)


def test_native_program_without_hook(fakes):
    run(fakes, "native", preload=False)


def test_tlsf_mode_serves_everything_from_the_pool(fakes):
    r = run(fakes, "pool")
    assert r.stdout.count("ok ") >= 25
    assert "is not a pool pointer" in r.stderr            # the foreign frees were reported


def test_cuda_mode_passes_through(fakes):
    run(fakes, "cuda", PTX_HOOK_MODE="cuda")


def test_mode_names_are_case_insensitive(fakes):
    run(fakes, "cuda", PTX_HOOK_MODE="CUDA")


def test_hybrid_thread_mode(fakes):
    run(fakes, "hybrid", PTX_HOOK_MODE="hybrid")


def test_disabled_pool(fakes):
    run(fakes, "disabled", PTX_HOOK_DISABLE="1")


def test_pool_that_cannot_be_made_behaves_as_disabled(fakes):
    r = run(fakes, "disabled", FAKE_HOT_FAIL="1")
    assert "could not make" in r.stderr


def test_hybrid_fallback_when_the_pool_cannot_be_made(fakes):
    run(fakes, "fallback", PTX_HOOK_MODE="hybrid", PTX_HOOK_HYBRID_FALLBACK="1", FAKE_HOT_FAIL="1")


def test_adopts_a_runtime_from_the_environment(fakes):
    run(fakes, "adopt")


def test_verbose_logs_routed_calls(fakes):
    r = run(fakes, "hybrid", PTX_HOOK_MODE="hybrid", PTX_HOOK_VERBOSE="1")
    assert "[ptx_hook] loaded, mode hybrid" in r.stderr
    assert "cudaMalloc(65536) = " in r.stderr
    assert "pool allocations 1, frees 1" in r.stderr
