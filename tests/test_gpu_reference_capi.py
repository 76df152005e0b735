"""The reference's own C-API tests (tests/c_api/*.cpp), compiled unchanged
against this repository's include/ and linked to its libfercuda_capi.so by
`make -C oracle capi-tests` (part of build(); the binaries sit in
oracle/_ref/capi/), run on the GPU: each must exit 0, as it does against the
reference library. They hold the reference's golden values (2x2 matmul
{19,22,43,50}, layer norm of {1,2,3,4}, affine+relu over 512 elements) and
its contracts (job ids, buffer ids, JIT cache hits, strict-mode signatures,
custom allocators, imported pointers, stream hand-off)."""
import os
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
BIN = ROOT / "oracle" / "_ref" / "capi"
TESTS = ["bridge", "custom_allocator", "jit_stub", "jit_exec", "jit_lowering", "jit_intent", "external_ptr_interop",
         "stream_handoff", "helper_api"]


def device_sm() -> int:
    import torch

    major, minor = torch.cuda.get_device_capability(0)
    return 10 * major + minor


@pytest.mark.parametrize("name", TESTS)
def test_reference_capi_test_passes(name, tmp_path):
    exe = BIN / f"test_c_api_{name}"
    assert exe.exists(), f"{exe} missing: build() compiles it when the reference tree is present"
    env = dict(os.environ)
    p = subprocess.run([str(exe)], cwd=tmp_path, env=env, capture_output=True, text=True, timeout=300)
    if name == "jit_lowering" and device_sm() >= 99:
        # The test's first contract compiles a source marked
        # `fercuda:require_sm>=99` and expects a rejection: true on the GPUs
        # it was written for, not on SM 10.0, where the reference's own gate
        # (capability_lowering_pass.cpp:17-18, sm = 10 * major + minor)
        # accepts the source exactly as this library does. The test stops at
        # that check; its other contracts (fusion notes in the compile log)
        # are restated in test_gpu_capi.py::test_jit_lowering_contracts.
        assert p.returncode == 1 and p.stderr.strip() == "FAIL: expected lowering capability rejection", p.stderr
        return
    assert p.returncode == 0, f"rc {p.returncode}\n{p.stdout[-2000:]}\n{p.stderr[-2000:]}"
