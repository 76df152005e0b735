"""Launch modes do not change results: the transformer forward gives the
same logits bits with programmatic dependent launch of the GEMM and
attention kernels on (default) and off (FERCUDA_GEMM_PDL=0, FERCUDA_PDL=0),
and with the CUDA graph of the forward off (FERCUDA_XFMR_GRAPH=0). Each mode
is read once per process, so each runs in a child process; the children
compare per-sequence digests of the logits (fer_buffer_row_digests)."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]

CHILD = r"""
import json, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
from fercuda_b200 import capi, synth
L, d, h, F, V, B, S = 2, 256, 4, 512, 1000, 4, 256
with capi.Session(0, pool_bytes=1 << 30) as s:
    m = capi.Transformer(s, L, d, h, F, V, B * S)
    m.init_weights(4, 0.02)
    u = synth.uniform01(5, B * S)
    toks = np.minimum((u * V).astype(np.int32), V - 1).reshape(B, S)
    bt = s.alloc(capi.FER_DTYPE_I32, [B, S])
    bl = s.alloc(capi.FER_DTYPE_F32, [B, S, V])
    s.upload(bt, toks)
    out = []
    for _ in range(3):                      # eager, captured, replayed
        s.wait(m.forward(bt, bl))
        out.append(s.row_digests(bl, 4 * S * V, B))
    assert s.device_errors() == 0
    m.close()
print(json.dumps(out))
"""


def run_mode(env_extra):
    env = dict(os.environ)
    env.update(env_extra)
    p = subprocess.run([sys.executable, "-c", CHILD, str(ROOT)], env=env, capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stderr[-2000:]
    return json.loads(p.stdout.strip().splitlines()[-1])


def test_programmatic_launch_and_graphs_keep_the_bits():
    base = run_mode({})
    assert base[0] == base[1] == base[2]
    for extra in ({"FERCUDA_GEMM_PDL": "0"}, {"FERCUDA_PDL": "0"}, {"FERCUDA_XFMR_GRAPH": "0"}):
        got = run_mode(extra)
        assert got[0] == base[0], extra
        assert got[0] == got[1] == got[2], extra


CHAIN_CHILD = r"""
import hashlib, json, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
from fercuda_b200 import capi, synth
n = (1 << 20) + 3                            # float4 body and scalar tail
x = (synth.uniform01(0, n).astype(np.float32) * 8.0 - 4.0).astype(np.float32)
with capi.Session(0, pool_bytes=256 << 20) as s:
    bx, by = s.alloc(capi.FER_DTYPE_F32, [n]), s.alloc(capi.FER_DTYPE_F32, [n])
    s.upload(bx, x)
    fusion = capi.FER_JIT_INTENT_FUSION_RELU | capi.FER_JIT_INTENT_FUSION_MUL_SIGMOID_INPUT
    out = []
    for _ in range(3):
        s.wait(s.affine(bx, by, n, 1.5, -0.25, fusion))
        y = np.empty(n, np.float32)
        s.download(by, y)
        out.append(hashlib.sha256(y.tobytes()).hexdigest())
    assert s.device_errors() == 0
print(json.dumps(out))
"""


def test_chain_launch_paths_keep_the_bits():
    """The fused elementwise chain launched through the driver by a function
    resolved once (default), through the runtime (FERCUDA_CHAIN_DRIVER_LAUNCH=0)
    and without programmatic launch (FERCUDA_CHAIN_PDL=0) gives the same
    output bits."""
    def run(extra):
        env = dict(os.environ)
        env.update(extra)
        p = subprocess.run([sys.executable, "-c", CHAIN_CHILD, str(ROOT)], env=env, capture_output=True, text=True,
                           timeout=300)
        assert p.returncode == 0, p.stderr[-2000:]
        return json.loads(p.stdout.strip().splitlines()[-1])

    base = run({})
    assert base[0] == base[1] == base[2]
    assert run({"FERCUDA_CHAIN_DRIVER_LAUNCH": "0"}) == base
    assert run({"FERCUDA_CHAIN_PDL": "0"}) == base
