"""libptx_hook.so on a GPU: the CUDA allocation calls of an unmodified
program served from the TLSF pool under LD_PRELOAD.

- tests/hook/hook_driver.c, linked against the CUDA runtime and driver, runs
  each scenario (tlsf / cuda / hybrid modes, disabled pool, adopted runtime)
  with and without the hook;
- fer_alloc_bench, the allocator benchmark, runs the reference claim's
  workload (64 KiB cudaMalloc + cudaFree pairs) both ways: every pair under
  the hook is served by the pool, and the pool is faster than cudaMalloc;
- PyTorch runs under the hook: its caching allocator's cudaMalloc / cudaFree
  land in the pool and its kernels compute on pool memory.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

from fercuda_b200 import capi

pytestmark = pytest.mark.gpu

HERE = Path(__file__).resolve().parent / "hook"
CUDA = "/usr/local/cuda"
HOOK = capi.LIBDIR / "libptx_hook.so"
BENCH = capi.LIBDIR / "fer_alloc_bench"
POOL = str(512 << 20)


@pytest.fixture(scope="module")
def driver(tmp_path_factory) -> Path:
    d = tmp_path_factory.mktemp("hookgpu")
    exe = d / "hook_driver"
    subprocess.run(["gcc", "-O1", "-Wall", "-Werror", f"-I{CUDA}/include", "-o", str(exe), str(HERE / "hook_driver.c"),
                    f"-L{CUDA}/lib64", "-lcudart", f"-L{CUDA}/lib64/stubs", "-lcuda", f"-Wl,-rpath,{CUDA}/lib64",
                    "-ldl"], check=True, capture_output=True, text=True)
    return exe


def env(preload: bool, **extra) -> dict:
    e = {k: v for k, v in os.environ.items() if not k.startswith("PTX_")}
    e.pop("LD_PRELOAD", None)
    if preload:
        e["LD_PRELOAD"] = str(HOOK)
        e["PTX_POOL_SIZE"] = POOL
    e.update(extra)
    return e


def run(cmd: list[str], e: dict, timeout: int = 300) -> subprocess.CompletedProcess:
    r = subprocess.run(cmd, env=e, capture_output=True, text=True, timeout=timeout)
    assert "FAIL" not in r.stdout, r.stdout + r.stderr
    assert r.returncode == 0, r.stdout + r.stderr
    return r


@pytest.mark.parametrize("scenario,preload,extra", [
    ("native", False, {}),
    ("pool", True, {}),
    ("cuda", True, {"PTX_HOOK_MODE": "cuda"}),
    ("hybrid", True, {"PTX_HOOK_MODE": "hybrid"}),
    ("disabled", True, {"PTX_HOOK_DISABLE": "1"}),
    ("adopt", True, {}),
])
def test_driver_scenarios(driver, scenario, preload, extra):
    run([str(driver), scenario], env(preload, **extra))


def _kv(text: str) -> dict:
    return dict(line.split("=", 1) for line in text.splitlines() if "=" in line)


def test_alloc_bench_pool_beats_cudamalloc():
    args = [str(BENCH), "--iters", "20000", "--warmup", "500", "--bytes", "65536"]
    native = _kv(run(args, env(False)).stdout)
    hooked = _kv(run(args, env(True)).stdout)
    assert native["mode"] == "cudaMalloc" and hooked["mode"] == "tlsf"
    assert int(hooked["pool_allocs"]) == 500 + 2 * 20000 == int(hooked["pool_frees"])
    assert float(hooked["ns_per_alloc_free"]) * 5 < float(native["ns_per_alloc_free"]), (native, hooked)


TORCH_PROBE = r"""
import ctypes, torch
hook = ctypes.CDLL(None)
n = (ctypes.c_uint64 * 3)()
x = torch.arange(1 << 20, device="cuda", dtype=torch.float32)
y = (x * 2.0).sum().item()
assert y == float((1 << 20) * ((1 << 20) - 1)), y
hook.ptx_hook_get_runtime.restype = ctypes.c_void_p
hook.gpu_hot_owns_ptr.restype = ctypes.c_bool
hook.gpu_hot_owns_ptr.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
rt = hook.ptx_hook_get_runtime()
assert rt and hook.gpu_hot_owns_ptr(rt, x.data_ptr())
del x
torch.cuda.synchronize()
torch.cuda.empty_cache()
hook.ptx_hook_get_stats(ctypes.byref(n, 0), ctypes.byref(n, 8), ctypes.byref(n, 16))
assert n[0] >= 1 and n[1] >= 1, list(n)
print("torch-under-hook ok", list(n))
"""


def test_torch_allocations_land_in_the_pool():
    r = run([sys.executable, "-c", TORCH_PROBE], env(True, PTX_POOL_SIZE=str(2 << 30)), timeout=600)
    assert "torch-under-hook ok" in r.stdout
