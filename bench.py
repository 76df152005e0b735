"""Benchmark of the hot path; rank 0 prints one JSON line.

Default workload: the decoder-only transformer forward (8 layers, d 1024,
16 heads, ffn 4096, vocab 32000, seq 512, global batch 64; bf16 weights
N(0, 0.02) from seed 4, tokens uniform from seed 5), batch-sharded over the
N GPUs of the launch (one process per GPU), weights initialised on rank 0 and
broadcast once over NCCL, no collective inside a forward. One step is one
forward of the whole global batch; `value` is global tokens per second over
the slowest rank's device time (strong scaling: the batch is fixed).

Other workloads (--workload), each also reported under `subresults` of the
default run on one GPU:
  softmax_layernorm  row softmax -> layer norm over f32 [4096, 4096]      HBM GB/s
  fused_elementwise  relu(1.5x - 0.25) * sigmoid(x), f32 2^20             HBM GB/s
  gemm               bf16 8192^3 -> f32, deterministic tcgen05 GEMM       TFLOP/s
  tlsf               1M-op alloc/free trace (256 B - 16 MiB, 60/40, live <= 64 GiB),
                     each allocation filled by a kernel; alloc latency   ns (p50)
  decode             KV-cache decoding on the benchmark model, 64 sequences
                     after a 512-token prompt, one token each per step   tokens/s

Timing: CUDA events on the session stream over exactly K steps after W
warm-up steps, barrier + synchronize on both sides, max over ranks.
`e2e` repeats the step through the public C ABI with pinned host buffers
(inputs uploaded and results downloaded inside the timed region).
`--impl reference` times the reference's CPU implementation of the path: the
oracle port (oracle/), all host threads, rank 0 only.
"""
from __future__ import annotations

import argparse
import ctypes as C
import datetime
import json
import os
import re
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from fercuda_b200 import sharding  # noqa: E402  (numpy only; no native library)

FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
METRIC_HBM = "HBM GB/s (fused elementwise, softmax)"
METRIC_TOK = "transformer fwd tokens/s"


def peak(key: str):
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        if key in d:
            return float(d[key]), "measured"
    return FALLBACK[key], "fallback"


def profiled_traffic(name: str):
    """Per-launch DRAM bytes of a kernel from its committed ncu summary
    (a `traffic_bytes_per_launch: N` line in profiles/<name>.md), or None."""
    p = ROOT / "profiles" / f"{name}.md"
    if not p.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9]+)", p.read_text())
    return int(m.group(1)) if m else None


def host_threads() -> int:
    try:
        return len(_ORIG_AFFINITY) or len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 20 ms."""

    def __init__(self, index: int):
        self.index, self.samples, self.proc, self.t0, self.t1 = index, [], None, None, None

    def start(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "20"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        threading.Thread(target=self._read, daemon=True).start()

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), [x.strip() for x in line.split(",")]))

    def mark(self, start: bool):
        if start:
            self.t0 = time.time()
        else:
            self.t1 = time.time()

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.12)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=2)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        lo, hi = (self.t0 or 0) - 0.06, (self.t1 or time.time()) + 0.06
        sel = [s for t, s in self.samples if lo <= t <= hi] or [s for _, s in self.samples[-3:]]
        num = lambda v: v.replace(".", "", 1).isdigit()
        sm = [float(s[1]) for s in sel if len(s) > 8 and num(s[1])]
        smax = [float(s[2]) for s in sel if len(s) > 8 and num(s[2])]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in sel if len(s) > 8 for i in range(4) if s[5 + i] == "Active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(sel)}


# ================================================================ workloads


class Rows:
    """Row softmax -> layer norm, f32 [4096, 4096] (fer_submit_rows)."""
    metric, unit, kernel = METRIC_HBM, "GB/s", "rows_fast_softmax_layernorm_4096x4096"
    exact = False

    def __init__(self, s, capi, synth, rows=4096, cols=4096, exact=False):
        self.s, self.capi, self.rows, self.cols = s, capi, rows, cols
        self.exact = exact
        self.kernel = "rows_softmax_layernorm_4096x4096" if exact else "rows_fast_softmax_layernorm_4096x4096"
        self.eps = synth.SOFTMAX_LAYERNORM["eps"]
        self.x = synth.softmax_layernorm_input(rows, cols)
        self.pairs = []
        for _ in range(3):
            bx, by = s.alloc(capi.FER_DTYPE_F32, [rows, cols]), s.alloc(capi.FER_DTYPE_F32, [rows, cols])
            s.upload(bx, self.x)
            self.pairs.append((bx, by))
        ops = capi.FER_ROWS_SOFTMAX | capi.FER_ROWS_LAYER_NORM | (0 if exact else capi.FER_ROWS_FAST)
        self.req = [capi.fer_rows_request_t(bx, by, 0, 0, self.eps, ops, capi.FER_MEMORY_AUTO) for bx, by in self.pairs]
        self.job = C.c_uint64()
        self.units_per_step = 8 * rows * cols           # algorithmic bytes
        self.launches_per_step = 1
        self.h2d = self.d2h = 4 * rows * cols
        self.hx = self.hy = None

    def step(self, i):
        st = self.s.call("fer_submit_rows", C.byref(self.req[i % 3]), C.byref(self.job))
        if st.code:
            raise RuntimeError(st.message)

    def config(self, world):
        c = self.describe(world)
        if self.exact:
            c["path"] = "reference order (bit-identical to the reference kernels)"
            c["api"] = "fer_submit_rows (SOFTMAX|LAYER_NORM)"
        return c

    @staticmethod
    def describe(world, rows=4096, cols=4096):
        return {"workload": f"softmax_layernorm_{rows}x{cols}_f32", "rows": rows, "cols": cols,
                "path": "fast deterministic (<= 1e-5 of the reference order, bit-identical run to run)",
                "eps": 1e-5, "gamma": 1.0, "beta": 0.0, "input": "N(0,1) seed 1",
                "l2": "rotating 3 input/output pairs (384 MiB > 126 MB L2)", "api": "fer_submit_rows (SOFTMAX|LAYER_NORM|FAST)",
                "parallelism": f"replicas x{world}"}

    def e2e_prepare(self, torch):
        self.hx = torch.from_numpy(self.x.reshape(-1)).pin_memory().numpy()
        self.hy = torch.empty(self.hx.size, dtype=torch.float32).pin_memory().numpy()

    def e2e_step(self):
        bx, by = self.pairs[0]
        self.s.upload(bx, self.hx)
        self.step(0)
        self.s.download(by, self.hy)

    def roofline(self, kern_ms):
        pk, src = peak("hbm_gbs")
        ach = self.units_per_step / (kern_ms * 1e-3) / 1e9
        kernel = "rows_bulk_kernel" if getattr(self, "exact", True) else "rows_fast_kernel"
        return {"bound": "hbm", "achieved": round(ach, 1), "peak": pk, "unit": "GB/s", "frac": round(ach / pk, 4),
                "traffic": profiled_traffic(self.kernel), "algorithmic_bytes_per_launch": self.units_per_step,
                "peak_source": src, "kernel": kernel, "kernel_ms_per_launch": round(kern_ms, 5)}

    @staticmethod
    def cpu(threads, reps=3):
        from fercuda_b200 import synth
        from tests import oracle_lib

        x = synth.softmax_layernorm_input()
        y = np.empty_like(x)
        orc = oracle_lib.load()
        fn = lambda: orc.orc_softmax_layernorm_rows_f32(x.ctypes.data_as(C.c_void_p), y.ctypes.data_as(C.c_void_p),
                                                        x.shape[0], x.shape[1], C.c_float(1e-5), threads)
        fn()
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        dt = (time.perf_counter() - t0) / reps
        return 8 * x.size / dt / 1e9, f"full 4096x4096 batch, mean of {reps} passes", threads


class Chain(Rows):
    """y = relu(1.5x - 0.25) * sigmoid(x), f32 2^20 (fer_tensor_run_affine_f32)."""
    kernel = "fused_chain_2p20"

    def __init__(self, s, capi, synth, n=1 << 20):
        self.s, self.capi = s, capi
        c = synth.FUSED_ELEMENTWISE
        self.n, self.a, self.b = n, c["a"], c["b"]
        # sizes above 2^22 repeat the seeded 2^22 prefix (bandwidth sweeps)
        self.x = synth.fused_elementwise_input(n) if n <= (1 << 22) else np.resize(
            synth.fused_elementwise_input(1 << 22), n)
        self.nbuf = max(2, min(48, (384 << 20) // (8 * n)))
        self.pairs = []
        for _ in range(self.nbuf):
            bx, by = s.alloc(capi.FER_DTYPE_F32, [n]), s.alloc(capi.FER_DTYPE_F32, [n])
            s.upload(bx, self.x)
            self.pairs.append((bx, by))
        self.fusion = capi.FER_JIT_INTENT_FUSION_RELU | capi.FER_JIT_INTENT_FUSION_MUL_SIGMOID_INPUT
        self.job = C.c_uint64()
        self.units_per_step = 8 * n
        self.launches_per_step = 1
        self.h2d = self.d2h = 4 * n
        s.wait(s.affine(*self.pairs[0], n, self.a, self.b, self.fusion))   # NVRTC compile outside timing

    def steps_native(self, first, k):
        """k steps issued by a C loop over the same public call
        (fer_bench_affine_loop), so that Python's per-call cost does not
        starve a few-microsecond kernel."""
        if k == 0:
            return
        if not hasattr(self, "_loop"):
            lib = C.CDLL(str(self.capi.LIBDIR / "libfercuda_bench.so"))
            lib.fer_bench_affine_loop.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32,
                                                  C.c_float, C.c_float, C.c_uint32, C.c_uint32, C.c_uint32,
                                                  C.c_void_p]
            self._ins = (C.c_uint64 * self.nbuf)(*[p[0] for p in self.pairs])
            self._outs = (C.c_uint64 * self.nbuf)(*[p[1] for p in self.pairs])
            self._loop = lib.fer_bench_affine_loop
        rc = self._loop(self.s.ptr, self._ins, self._outs, self.nbuf, self.n, self.a, self.b, self.fusion, k,
                        first % self.nbuf, None)
        if rc:
            raise RuntimeError(f"fer_tensor_run_affine_f32 failed with status {rc}")

    def step(self, i):
        bx, by = self.pairs[i % self.nbuf]
        st = self.s.lib.fer_tensor_run_affine_f32(self.s.ptr, self.capi.fer_tensor_handle_t(bx),
                                                  self.capi.fer_tensor_handle_t(by), self.n, self.a, self.b,
                                                  self.fusion, 0, self.capi.FER_MEMORY_AUTO, C.byref(self.job))
        if st.code:
            raise RuntimeError(st.message)

    def config(self, world):
        return self.describe(world, self.n)

    @staticmethod
    def describe(world, n=1 << 20):
        nbuf = max(2, min(48, (384 << 20) // (8 * n)))
        return {"workload": f"fused_elementwise_relu_affine_mul_sigmoid_{n}_f32", "n": n, "a": 1.5,
                "b": -0.25, "input": "U(-4,4) seed 0",
                "l2": f"rotating {nbuf} input/output pairs ({nbuf * 8 * n >> 20} MiB > 126 MB L2)",
                "api": "fer_tensor_run_affine_f32 (fusion RELU|MUL_SIGMOID_INPUT), issued back to back from C",
                "parallelism": f"replicas x{world}"}

    def roofline(self, kern_ms):
        r = super().roofline(kern_ms)
        r["kernel"] = "fer_chain_v4 (JIT)"
        return r

    @staticmethod
    def cpu(threads, reps=20):
        from fercuda_b200 import synth
        from tests import oracle_lib

        x = synth.fused_elementwise_input()
        y = np.empty_like(x)
        orc = oracle_lib.load()
        fn = lambda: orc.orc_chain_f32(x.ctypes.data_as(C.c_void_p), y.ctypes.data_as(C.c_void_p), x.size,
                                       C.c_float(1.5), C.c_float(-0.25), threads)
        fn()
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        dt = (time.perf_counter() - t0) / reps
        return 8 * x.size / dt / 1e9, f"full 2^20 batch, mean of {reps} passes", threads


class Gemm:
    """bf16 8192^3 -> f32, deterministic tcgen05 GEMM (fer_submit_gemm)."""
    metric, unit, kernel = "deterministic GEMM TFLOP/s (bf16 in, f32 accumulate)", "TFLOP/s", "gemm_tc2_8192"

    def __init__(self, s, capi, synth, m=8192, n=8192, k=8192):
        self.s, self.capi, self.m, self.n, self.k = s, capi, m, n, k
        # A is the first m*k draws of the device generator's seed-3 stream, B the
        # next k*n (one fill over both, then two buffer views of it)
        self.bab = s.alloc(capi.FER_DTYPE_BF16, [m * k + k * n])
        base = s.ptr_of(self.bab)
        rc = capi.kernels().fer_fill_normal_bf16(C.c_void_p(base), m * k + k * n, synth.GEMM["seed"],
                                                 C.c_float(1.0 / np.sqrt(k)), C.c_void_p(s.stream()))
        if rc:
            raise RuntimeError(f"fer_fill_normal_bf16 failed: {rc}")
        self.ba = s.import_ptr(capi.FER_DTYPE_BF16, [m, k], base)
        self.bb = s.import_ptr(capi.FER_DTYPE_BF16, [k, n], base + 2 * m * k)
        self.bo = s.alloc(capi.FER_DTYPE_F32, [m, n])
        self.req = capi.fer_gemm_request_t(self.ba, self.bb, self.bo, 0, capi.FER_MEMORY_AUTO)
        self.job = C.c_uint64()
        self.units_per_step = 2.0 * m * n * k
        self.launches_per_step = 1
        self.h2d = 2 * (m * k + k * n)
        self.d2h = 4 * m * n

    def step(self, i):
        st = self.s.call("fer_submit_gemm", C.byref(self.req), C.byref(self.job))
        if st.code:
            raise RuntimeError(st.message)

    def config(self, world):
        return self.describe(world)

    @staticmethod
    def describe(world, m=8192, n=8192, k=8192):
        return {"workload": f"gemm_bf16_{m}x{n}x{k}_f32out", "m": m, "n": n, "k": k,
                "input": "N(0, 1/sqrt(K)) seed 3 (device generator: A the first M*K draws, B the next K*N)",
                "l2": "operands 256 MiB + output 256 MiB exceed L2",
                "api": "fer_submit_gemm", "parallelism": f"replicas x{world}"}

    def e2e_prepare(self, torch):
        self.ha = torch.empty(self.m * self.k, dtype=torch.int16).pin_memory().numpy()
        self.hb = torch.empty(self.k * self.n, dtype=torch.int16).pin_memory().numpy()
        self.s.download(self.ba, self.ha)
        self.s.download(self.bb, self.hb)
        self.hc = torch.empty(self.m * self.n, dtype=torch.float32).pin_memory().numpy()

    def e2e_step(self):
        self.s.upload(self.ba, self.ha)
        self.s.upload(self.bb, self.hb)
        self.step(0)
        self.s.download(self.bo, self.hc)

    def roofline(self, kern_ms):
        pk, src = peak("bf16_tflops")
        ach = self.units_per_step / (kern_ms * 1e-3) / 1e12
        return {"bound": "tensor", "achieved": round(ach, 1), "peak": pk, "unit": "TFLOP/s", "frac": round(ach / pk, 4),
                "traffic": profiled_traffic(self.kernel), "algorithmic_flops_per_launch": self.units_per_step,
                "peak_source": src + " (burst)", "kernel": "gemm_bf16_tc2_kernel (2-CTA clusters)",
                "kernel_ms_per_launch": round(kern_ms, 5)}

    @staticmethod
    def cpu(threads, tiles=4):
        """The reference's chain (sequential fmaf over K per output) on sampled
        64x64 output tiles; TFLOP/s extrapolates per-output time to the matrix."""
        from tests import oracle_lib

        # operand values do not change the chain's timing: numpy's generator
        # with the workload's distribution, bf16 by truncation
        m, n, k = 64 * tiles, 8192, 8192
        rng = np.random.default_rng(3)
        bits = lambda shape: (rng.standard_normal(shape, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)
        a, b = bits((m, k)), bits((k, n))
        orc = oracle_lib.load()
        out = np.empty((64, 64), np.float32)
        t0 = time.perf_counter()
        for t in range(tiles):
            r0, c0 = 64 * t, (t * 3001) % (n - 64)
            orc.orc_matmul_bf16_tile(oracle_lib.ptr(a), oracle_lib.ptr(b), oracle_lib.ptr(out), m, k, n, r0, r0 + 64,
                                     c0, c0 + 64)
        dt = time.perf_counter() - t0
        return 2.0 * tiles * 64 * 64 * k / dt / 1e12, f"{tiles} sampled 64x64 output tiles, K=8192", 1


class Transformer:
    """Decoder-only transformer forward, batch-sharded (fer_transformer_forward)."""
    metric, unit, kernel = METRIC_TOK, "tokens/s", "gemm_tc_transformer_b8"
    e2e_api = ("fer_transformer_forward_host (pinned host tokens in, pinned host logits out; the D2H copy of each "
               "chunk of sequences under the next chunk's forward)")

    def __init__(self, s, capi, synth, rank=0, world=1, dist=None, torch=None, batch=None):
        cfg = dict(synth.TRANSFORMER)
        if batch:
            cfg["batch"] = batch
        self.s, self.capi, self.cfg = s, capi, cfg
        self.world, self.rank = world, rank
        L, d, h, F, V, S, B = (cfg[k] for k in ("layers", "d_model", "heads", "ffn", "vocab", "seq", "batch"))
        if B % world:
            raise SystemExit(f"global batch {B} does not split over {world} GPUs")
        self.B_local, self.S, self.V = B // world, S, V
        self.global_tokens = B * S
        T = self.B_local * S
        self.model = capi.Transformer(s, L, d, h, F, V, T, cfg["eps"])
        if rank == 0:
            self.model.init_weights(cfg["weight_seed"], 0.02)
        else:
            # other weights until the broadcast arrives, so equal logits
            # digests across GPU counts show that it did
            self.model.init_weights(0x5EED0000 + rank, 0.02)
        self.broadcast_bytes = 0
        if world > 1:
            self._broadcast_weights(dist)
        u = synth.uniform01(cfg["token_seed"], B * S)
        toks = np.minimum((u * V).astype(np.int32), V - 1).reshape(B, S)
        first, count = capi.transformer_shard(B, world, rank)
        self.first_seq = first
        self.toks = np.ascontiguousarray(toks[first:first + count])
        self.bt = s.alloc(capi.FER_DTYPE_I32, [self.B_local, S])
        self.bl = s.alloc(capi.FER_DTYPE_F32, [self.B_local, S, V])
        s.upload(self.bt, self.toks)
        self.units_per_step = self.global_tokens
        self.launches_per_step = 2 + 7 * L     # embed+LN1, 7 per layer, final LN, LM head
        self.h2d = 4 * T
        self.d2h = 4 * T * V

    def _broadcast_weights(self, dist):
        """Rank 0's weights reach every rank once: fer_transformer_broadcast_weights,
        one NCCL broadcast over NVLink/NVSwitch on a communicator the session
        owns (fer_comm_init), released right after (no per-step collective)."""
        uid = sharding.share_unique_id(dist, self.capi.comm_unique_id() if self.rank == 0 else None)
        self.s.comm_init(uid, self.rank, self.world, 120_000)
        self.broadcast_bytes = self.model.broadcast_weights(0)
        self.s.comm_destroy()

    def digests(self):
        """Per-sequence digests of this rank's logits (fer_buffer_row_digests)."""
        return self.s.row_digests(self.bl, 4 * self.S * self.V, self.B_local)

    def step(self, i):
        self.model.forward(self.bt, self.bl)

    def config(self, world):
        return self.describe(world, self.cfg["batch"])

    @staticmethod
    def describe(world, batch=None):
        from fercuda_b200 import synth

        c = dict(synth.TRANSFORMER)
        c["batch"] = batch or c["batch"]
        return {"workload": f"decoder_transformer_fwd_L8_d1024_h16_F4096_V32000_S512_B{c['batch']}",
                "model": "decoder-only pre-LN",
                "layers": c["layers"], "d_model": c["d_model"], "heads": c["heads"], "ffn": c["ffn"],
                "vocab": c["vocab"], "seq_len": c["seq"], "global_batch": c["batch"], "local_batch": c["batch"] // world,
                "weights": "bf16 N(0,0.02) seed 4 (device-generated on rank 0, NCCL broadcast once)",
                "tokens": "uniform seed 5", "parallelism": f"dp{world} (batch-sharded, no per-step collective)",
                "l2": "weights 333 MB + activations > 1 GB per step exceed L2", "api": "fer_transformer_forward"}

    def e2e_prepare(self, torch):
        self.ht = torch.from_numpy(self.toks).pin_memory().numpy()
        self.hl = torch.empty(self.B_local * self.S * self.V, dtype=torch.float32).pin_memory().numpy()

    def e2e_step(self):
        # host tokens in, host logits out: the D2H copy of each chunk of
        # sequences runs under the next chunk's forward
        self.model.forward_host(self.ht, self.hl)

    def roofline_from_profile(self, prof, ms_per_step):
        """GEMM roofline of the timed steps: each kernel class's share of a
        forward comes from the event-instrumented pass (fer_transformer_profile),
        its time from the timed region (share x ms_per_step), so
        achieved = GEMM FLOPs per forward / (share x ms_per_step) follows
        from the line's own ms_per_step."""
        # the GEMMs run inside a long, power-capped step (20+ forwards back to
        # back), so the denominator is the sustained bf16 GEMM rate
        pk, src = peak("bf16_tflops_sustained")
        fw = max(1, prof.forwards)
        total = prof.gemm_ms + prof.attn_ms + prof.norm_ms + prof.other_ms
        share = {k: getattr(prof, k) / total for k in ("gemm_ms", "attn_ms", "norm_ms", "other_ms")}
        gemm_flops = prof.gemm_flops / fw
        attn_flops = prof.attn_flops / fw
        ach = gemm_flops / (share["gemm_ms"] * ms_per_step * 1e-3) / 1e12
        per_launch = gemm_flops / (4 * self.cfg["layers"] + 1)   # mean over the GEMMs of a forward
        return {"bound": "tensor", "achieved": round(ach, 1), "peak": pk, "unit": "TFLOP/s",
                "frac": round(ach / pk, 4), "traffic": profiled_traffic(self.kernel),
                "traffic_note": "ncu DRAM bytes per GEMM launch, mean over the 33 GEMMs of a B=8 forward",
                "algorithmic_flops_per_launch": round(per_launch), "gemm_flops_per_forward": round(gemm_flops),
                "peak_source": src + " (sustained)", "kernel": "gemm_bf16_tc2_kernel (all GEMMs of the forward)",
                "share_of_forward": round(share["gemm_ms"], 4),
                "attention_tflops": round(attn_flops / (share["attn_ms"] * ms_per_step * 1e-3) / 1e12, 1)
                if prof.attn_ms else None,
                "attention_share": round(share["attn_ms"], 4), "norm_share": round(share["norm_ms"], 4),
                "forward_tflops": round((gemm_flops + attn_flops) / (ms_per_step * 1e-3) / 1e12, 1),
                "how": "shares from the event pass x the timed ms_per_step",
                "event_pass_ms_per_forward": round(total / fw, 4)}

    @staticmethod
    def cpu(threads, seqs=1):
        """numpy restatement (oracle/transformer_ref.py) on `seqs` full
        sequences of 512 tokens; weights from numpy's generator with the same
        distribution (the oracle's timing does not depend on the values)."""
        from fercuda_b200 import synth
        from oracle import transformer_ref as ref

        c = synth.TRANSFORMER
        if not hasattr(Transformer, "_cpu_w"):
            o = ref.weight_offsets(c["layers"], c["d_model"], c["ffn"], c["vocab"])
            w = np.random.default_rng(c["weight_seed"]).standard_normal(o["total"], dtype=np.float32)
            w *= np.float32(0.02)
            Transformer._cpu_w = (w.view(np.uint32) >> 16).astype(np.uint16)
        wbits = Transformer._cpu_w
        toks = np.minimum((synth.uniform01(c["token_seed"], seqs * c["seq"]) * c["vocab"]).astype(np.int32),
                          c["vocab"] - 1).reshape(seqs, c["seq"])
        from threadpoolctl import threadpool_limits

        # torchrun sets OMP_NUM_THREADS=1 per rank; the CPU leg uses every host thread
        with threadpool_limits(limits=threads):
            t0 = time.perf_counter()
            ref.forward(toks, wbits, c["layers"], c["d_model"], c["heads"], c["ffn"], c["vocab"], c["eps"])
            dt = time.perf_counter() - t0
        return seqs * c["seq"] / dt, f"{seqs} sequence(s) x 512 tokens through the numpy restatement", threads


class Tlsf:
    """1M-op alloc/free trace through the TLSF pool, each block filled by a kernel."""
    metric, unit, kernel = "TLSF alloc latency p50 (ns)", "ns", None

    def __init__(self, s, capi, synth):
        self.s, self.capi, self.synth = s, capi, synth

    def run(self, ops=None, cmp_ops=50_000):
        import ctypes

        lib = ctypes.CDLL(str(self.capi.LIBDIR / "libfercuda_bench.so"))
        core = self.capi.core()
        lib.fer_bench_pool_replay.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_size_t, C.c_int, C.c_void_p,
                                              C.c_void_p, C.POINTER(C.c_size_t), C.c_void_p, C.POINTER(C.c_size_t),
                                              C.POINTER(C.c_uint64), C.POINTER(C.c_double)]
        trace = self.synth.tlsf_trace(ops=ops)
        cfg = core.gpu_hot_default_config()
        cfg.fixed_pool_size = 80 << 30
        cfg.min_pool_size = 0
        rt = core.gpu_hot_init_with_config(int(os.environ.get("LOCAL_RANK", "0")), b"bench", C.byref(cfg))
        if not rt:
            raise RuntimeError("could not create an 80 GiB pool")
        stream = core.gpu_hot_get_stream(rt, 0)
        res = {}
        for name, use_cm, tr in (("tlsf", 0, trace), ("cudaMalloc", 1, trace[:cmp_ops]),
                                 ("tlsf_same_sample", 0, trace[:cmp_ops])):
            tr = np.ascontiguousarray(tr)   # a prefix of the trace frees only its own allocations
            na_max = int((tr > 0).sum())
            an = np.zeros(max(1, na_max), np.uint32)
            fn = np.zeros(max(1, len(tr) - na_max), np.uint32)
            na, nf, fb, wall = C.c_size_t(), C.c_size_t(), C.c_uint64(), C.c_double()
            rc = lib.fer_bench_pool_replay(rt if not use_cm else None, use_cm, tr.ctypes.data_as(C.c_void_p), len(tr),
                                           1, stream, an.ctypes.data_as(C.c_void_p), C.byref(na),
                                           fn.ctypes.data_as(C.c_void_p), C.byref(nf), C.byref(fb), C.byref(wall))
            a, f = an[:na.value], fn[:nf.value]
            res[name] = {"rc": rc, "ops": len(tr), "allocs": int(na.value), "frees": int(nf.value),
                         "alloc_p50_ns": float(np.percentile(a, 50)) if a.size else None,
                         "alloc_p99_ns": float(np.percentile(a, 99)) if a.size else None,
                         "free_p50_ns": float(np.percentile(f, 50)) if f.size else None,
                         "free_p99_ns": float(np.percentile(f, 99)) if f.size else None,
                         "fill_bytes": int(fb.value), "wall_s": round(wall.value, 3)}
        core.gpu_hot_shutdown(rt)
        return res

    @staticmethod
    def host_replay(lib_alloc, lib_free, handle, trace):
        """Per-op latency (ns) of a TLSF's bookkeeping over `trace`, timed in C
        (fer_bench_fn_replay) with the allocator's own entry points."""
        from fercuda_b200 import capi

        bench = C.CDLL(str(capi.LIBDIR / "libfercuda_bench.so"))
        bench.fer_bench_fn_replay.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p,
                                              C.POINTER(C.c_size_t), C.c_void_p, C.POINTER(C.c_size_t),
                                              C.POINTER(C.c_double)]
        tr = np.ascontiguousarray(trace, np.int64)
        na_max = int((tr > 0).sum())
        an = np.zeros(max(1, na_max), np.uint32)
        fn = np.zeros(max(1, len(tr) - na_max), np.uint32)
        na, nf, wall = C.c_size_t(), C.c_size_t(), C.c_double()
        addr = lambda f: C.cast(f, C.c_void_p).value
        rc = bench.fer_bench_fn_replay(addr(lib_alloc), addr(lib_free), handle, tr.ctypes.data_as(C.c_void_p), len(tr),
                                       an.ctypes.data_as(C.c_void_p), C.byref(na), fn.ctypes.data_as(C.c_void_p),
                                       C.byref(nf), C.byref(wall))
        a, f = an[:na.value], fn[:nf.value]
        return {"rc": rc, "ops": len(tr), "alloc_p50_ns": float(np.percentile(a, 50)),
                "alloc_p99_ns": float(np.percentile(a, 99)), "free_p50_ns": float(np.percentile(f, 50)),
                "free_p99_ns": float(np.percentile(f, 99)), "wall_s": round(wall.value, 3)}

    @staticmethod
    def cpu_reference(ops=1_000_000):
        """The reference TLSF (oracle/_ref, compiled from its own sources) and
        this package's TLSF, both host-only over the same fake 80 GiB range,
        replaying the same trace: allocator bookkeeping latency per op."""
        from fercuda_b200 import capi, synth
        from tests import oracle_lib

        ref = oracle_lib.ref_tlsf()
        if ref is None:
            return None
        trace = synth.tlsf_trace(ops=ops)
        base = C.c_void_p(1 << 40)
        out = {}
        for name, lib in (("reference", ref), ("fercuda_b200", capi.core())):
            lib.ptx_tlsf_create_from_pool.restype = C.c_void_p
            lib.ptx_tlsf_create_from_pool.argtypes = [C.c_void_p, C.c_size_t, C.c_bool]
            lib.ptx_tlsf_set_warnings_enabled.argtypes = [C.c_void_p, C.c_bool]
            lib.ptx_tlsf_destroy.argtypes = [C.c_void_p]
            h = lib.ptx_tlsf_create_from_pool(base, 80 << 30, False)
            lib.ptx_tlsf_set_warnings_enabled(h, False)
            out[name] = Tlsf.host_replay(lib.ptx_tlsf_alloc, lib.ptx_tlsf_free, h, trace)
            lib.ptx_tlsf_destroy(h)
        out["note"] = "host-only bookkeeping over a fake range, timed in C around each call, 1 thread"
        return out


class Decode:
    """Incremental decoding (fer_transformer_decode), run by decode_steps."""
    metric = "decode tokens/s (one token per sequence per step)"
    unit = "tokens/s"


WORKLOADS = {"transformer": Transformer, "softmax_layernorm": Rows, "fused_elementwise": Chain, "gemm": Gemm,
             "tlsf": Tlsf, "decode": Decode}


# ================================================================ runners


def timed_steps(wl, torch, stream, steps, warmup, dist, world):
    """W warm-up steps, then exactly `steps` steps between one pair of CUDA
    events on the session stream (barrier + synchronize on both sides).
    Returns the elapsed milliseconds; elapsed / steps is the average launch
    duration of a one-kernel step (host-side events per launch would make
    short kernels host-bound and are not recorded)."""
    run = getattr(wl, "steps_native", None)
    if run is None:
        def run(first, k):
            for i in range(first, first + k):
                wl.step(i)
    run(0, warmup)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0.record(stream)
    h0 = time.perf_counter()
    run(warmup, steps)
    wl.host_issue_s = time.perf_counter() - h0   # host time to issue the K steps
    t1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    return t0.elapsed_time(t1)


_ORIG_AFFINITY = set(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else set()


def unbind() -> None:
    """Back to every host thread the process started with (CPU baselines)."""
    if _ORIG_AFFINITY:
        os.sched_setaffinity(0, _ORIG_AFFINITY)


def bind_to_gpu_numa_node(torch, local: int) -> dict:
    """Pins this process to the host CPUs of its GPU's NUMA node (from sysfs)
    before any pinned host buffer is made, so those buffers are first touched,
    and therefore placed, in memory local to the GPU's PCIe root: the e2e
    download of the logits then does not cross the socket interconnect."""
    try:
        p = torch.cuda.get_device_properties(local)
        bus = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        dev = Path("/sys/bus/pci/devices") / bus
        node = int((dev / "numa_node").read_text().strip())
        cpus = set()
        for part in (dev / "local_cpulist").read_text().strip().split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= _ORIG_AFFINITY
        if cpus:
            os.sched_setaffinity(0, cpus)
        return {"pci": bus, "numa_node": node, "cpus": len(cpus)}
    except (OSError, ValueError, AttributeError) as e:
        return {"error": str(e)[:80]}


def max_over_ranks(v, torch, dist, world):
    return sharding.max_over_ranks(torch, dist, v, "cuda")


def subresults(s, capi, synth, torch, stream):
    """Short measurements of the other workloads (one GPU)."""
    out = {}
    for name, cls, steps in (("softmax_layernorm", Rows, 50), ("softmax_layernorm_reference_order", Rows, 50),
                             ("fused_elementwise", Chain, 2000), ("gemm", Gemm, 10)):
        wl = cls(s, capi, synth, exact=True) if name == "softmax_layernorm_reference_order" else cls(s, capi, synth)
        el = timed_steps(wl, torch, stream, steps, 5, None, 1)
        med = el / steps
        unit_scale = 1e9 if cls is not Gemm else 1e12
        out[name] = {"metric": cls.metric, "value": round(wl.units_per_step * steps / (el * 1e-3) / unit_scale, 2),
                     "unit": cls.unit, "steps": steps, "config": wl.config(1), "roofline": wl.roofline(med),
                     "device_error_bits": s.device_errors(),
                     "host_us_per_call": round(wl.host_issue_s / steps * 1e6, 3),
                     "device_us_per_call": round(med * 1e3, 3)}
        cv, sample, cores = cls.cpu(host_threads())
        out[name]["cpu_baseline"] = {"value": round(cv, 6), "unit": cls.unit, "cores": cores, "kind": "port",
                                     "sample": sample + " (oracle/, restatement of the reference's path)"}
        if cls is Gemm:
            y0, y1 = np.empty((wl.m, wl.n), np.float32), np.empty((wl.m, wl.n), np.float32)
            s.download(wl.bo, y0)
            wl.step(0)
            s.download(wl.bo, y1)
            out[name]["bit_identical_rerun"] = bool(np.array_equal(y0.view(np.uint32), y1.view(np.uint32)))
            for b in (wl.ba, wl.bb, wl.bo, wl.bab):
                s.free(b)
        else:
            for bx, by in wl.pairs:
                s.free(bx)
                s.free(by)
    out["decode"] = decode_steps(s, capi, synth, torch)
    out["alloc_hook"] = hook_alloc_pairs(capi)
    tl = Tlsf(s, capi, synth).run()
    out["tlsf"] = {"metric": Tlsf.metric, "value": tl["tlsf"]["alloc_p50_ns"], "unit": "ns", "results": tl,
                   "sample": "the full 1M-op trace (cudaMalloc: its first 50k ops)",
                   "reference_tlsf_host": Tlsf.cpu_reference()}
    return out


def compact(sub: dict) -> dict:
    """The figures of each subresult that the one-line summary keeps (the
    full records go to stderr): value, unit, roofline achieved / peak / frac,
    the CPU baseline's value, and the TLSF and allocator latencies."""
    out = {}
    for name, r in sub.items():
        c = {"value": r.get("value"), "unit": r.get("unit")}
        roof = r.get("roofline")
        if roof:
            c.update(achieved=roof.get("achieved"), peak=roof.get("peak"), frac=roof.get("frac"))
        if r.get("cpu_baseline"):
            c["cpu"] = r["cpu_baseline"]["value"]
        if name == "tlsf":
            t, cm = r["results"]["tlsf"], r["results"]["cudaMalloc"]
            c.update(ops=t["ops"], alloc_p99_ns=t["alloc_p99_ns"], free_p50_ns=t["free_p50_ns"],
                     cudaMalloc_p50_ns=cm["alloc_p50_ns"])
        if name == "alloc_hook":
            c["speedup_vs_cudamalloc"] = r.get("speedup_vs_cudamalloc")
        if "bit_identical_rerun" in r:
            c["bit_identical_rerun"] = r["bit_identical_rerun"]
        if name == "fused_elementwise":
            c.update(host_us_per_call=r.get("host_us_per_call"), device_us_per_call=r.get("device_us_per_call"))
        out[name] = c
    return out


def decode_steps(s, capi, synth, torch, batch=64, prompt=512, steps=32):
    """Incremental decoding on the benchmark model: prefill `prompt` tokens of
    `batch` sequences into a KV cache (last-position logits), then `steps`
    decode calls (one token per sequence each) timed with CUDA events on the
    session stream. Roofline: the bytes a step must move (every weight once,
    the KV cache read up to the current position, the new K/V written)
    against the measured HBM copy rate."""
    c = synth.TRANSFORMER
    L, d, h, F, V = c["layers"], c["d_model"], c["heads"], c["ffn"], c["vocab"]
    m = capi.Transformer(s, L, d, h, F, V, batch * prompt, c["eps"])
    m.init_weights(c["weight_seed"], 0.02)
    u = synth.uniform01(c["token_seed"], batch * (prompt + steps + 5))
    toks = np.minimum((u * V).astype(np.int32), V - 1).reshape(batch, prompt + steps + 5)
    cache = m.kv_create(batch, prompt + steps + 5)
    bt = s.alloc(capi.FER_DTYPE_I32, [batch, prompt])
    s.upload(bt, np.ascontiguousarray(toks[:, :prompt]))
    bl = s.alloc(capi.FER_DTYPE_F32, [batch, V])
    dts = []
    for k in range(steps + 5):
        b = s.alloc(capi.FER_DTYPE_I32, [batch])
        s.upload(b, np.ascontiguousarray(toks[:, prompt + k]))
        dts.append(b)
    ext = torch.cuda.ExternalStream(s.stream())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.wait(m.prefill(cache, bt, bl))             # warm-up (kernels, JIT, pool)
    torch.cuda.synchronize()
    e0.record(ext)
    s.wait(m.prefill(cache, bt, bl))
    e1.record(ext)
    torch.cuda.synchronize()
    prefill_ms = e0.elapsed_time(e1)
    for k in range(4):
        m.decode(cache, dts[k], bl)
    torch.cuda.synchronize()
    e0.record(ext)
    for k in range(4, 4 + steps):
        m.decode(cache, dts[k], bl)
    e1.record(ext)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    # one more step inside a profiler range (a no-op unless a profiler with
    # --profile-from-start off is attached): the launch list of one step
    torch.cuda.profiler.start()
    m.decode(cache, dts[4 + steps], bl)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    errs = s.device_errors()
    ctx = prompt + 4 + steps / 2                 # mean keys per step
    kv_bytes = L * batch * d * 2 * 2 * (ctx + 1)   # K and V read (bf16) plus the new row
    w_bytes = 2 * m.weight_elements()
    pk, src = peak("hbm_gbs")
    achieved = (kv_bytes + w_bytes) / (ms * 1e-3) / 1e9
    for b in dts + [bt, bl]:
        s.free(b)
    m.kv_destroy(cache)
    m.close()
    return {"metric": "decode tokens/s (one token per sequence per step)", "value": round(batch / (ms * 1e-3), 1),
            "unit": "tokens/s", "ms_per_step": round(ms, 4), "batch": batch, "prompt": prompt, "steps": steps,
            "prefill_ms": round(prefill_ms, 3), "prefill_tokens_per_s": round(batch * prompt / (prefill_ms * 1e-3), 1),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk, "unit": "GB/s",
                         "frac": round(achieved / pk, 4), "peak_source": src,
                         "bytes_per_step": int(kv_bytes + w_bytes),
                         "note": "every weight once + KV cache read to the current position + new K/V"},
            "api": "fer_transformer_prefill / fer_transformer_decode", "device_error_bits": errs}


def hook_alloc_pairs(capi, iters=50_000, cuda_iters=5_000, warmup=1_000, nbytes=65536):
    """The reference's allocator claim ("TLSF ~100-200x faster than cudaMalloc
    for alloc+free"; workload tests/bench/bench_alloc_vs_cudamalloc.cu:21-25,
    89-114): fer_alloc_bench times 64 KiB cudaMalloc + cudaFree pairs natively
    and under LD_PRELOAD=libptx_hook.so (pairs served by the TLSF pool), each
    in its own process. A native pair costs hundreds of microseconds on a
    B200, so the native leg runs `cuda_iters` pairs (seconds) instead of the
    claim's 50,000 (minutes); the hooked leg runs all `iters`."""
    import subprocess

    res = {}
    for name, preload, n in (("cudaMalloc", False, cuda_iters), ("tlsf_hook", True, iters)):
        args = [str(capi.LIBDIR / "fer_alloc_bench"), "--iters", str(n), "--warmup", str(warmup if preload else 100),
                "--bytes", str(nbytes)]
        env = {k: v for k, v in os.environ.items() if not k.startswith("PTX_") and k != "LD_PRELOAD"}
        if preload:
            env.update(LD_PRELOAD=str(capi.LIBDIR / "libptx_hook.so"), PTX_POOL_SIZE=str(256 << 20))
        r = subprocess.run(args, env=env, capture_output=True, text=True, timeout=600)
        kv = dict(line.split("=", 1) for line in r.stdout.splitlines() if "=" in line)
        res[name] = {"rc": r.returncode, **{k: (v if k == "mode" else float(v)) for k, v in kv.items()}}
    ok = all(v["rc"] == 0 for v in res.values())
    speedup = (res["cudaMalloc"]["ns_per_alloc_free"] / res["tlsf_hook"]["ns_per_alloc_free"]) if ok else None
    return {"metric": "64 KiB cudaMalloc+cudaFree pair, ns", "value": res["tlsf_hook"].get("ns_per_alloc_free"),
            "unit": "ns", "speedup_vs_cudamalloc": round(speedup, 1) if speedup else None,
            "reference_published": "TLSF ~100-200x faster than cudaMalloc for alloc+free (README.md:311)",
            "sample": f"hook: {iters} pairs after {warmup} warm-up; cudaMalloc: {cuda_iters} pairs after 100; "
                      "host clock, each leg in its own process", "results": res}


def run_reference(args, rank):
    if rank != 0:
        return
    threads = host_threads()
    cls = WORKLOADS[args.workload]
    if cls is Tlsf:
        r = Tlsf.cpu_reference()
        v = r["reference"]["alloc_p50_ns"] if r else None
        line = {"metric": Tlsf.metric, "value": v, "unit": "ns", "impl": "reference",
                "n_gpus": args.gpus, "steps": 1, "warmup": 0, "higher_is_better": False, "results": r,
                "cpu_baseline": {"value": v, "unit": "ns", "cores": 1,
                                 "kind": "reference", "sample": "full 1M-op trace, reference TLSF built from source"},
                "e2e": {"value": v, "unit": "ns", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        emit(line)
        return
    if cls is Decode:
        emit({"impl": "reference", "unavailable": "the reference has no KV-cache decoding path to time "
                                                  "(its transformer is a full forward only)"})
        return
    vals = []
    for _ in range(args.warmup if cls is not Transformer else 1):
        cls.cpu(threads)
    for _ in range(args.steps):
        v, sample, cores = cls.cpu(threads)
        vals.append(v)
    v = float(np.mean(vals))
    # one full step of the workload at the sampled rate (the sample itself is
    # bounded: see cpu_baseline.sample)
    d = cls.describe(args.gpus)
    if cls is Transformer:
        units = d["global_batch"] * d["seq_len"]                 # tokens
    elif cls is Rows:
        units = 8.0 * d["rows"] * d["cols"] / 1e9               # GB
    elif cls is Chain:
        units = 8.0 * d["n"] / 1e9                              # GB
    else:
        units = 2.0 * d["m"] * d["n"] * d["k"] / 1e12           # TFLOP
    ms_step = units / v * 1e3 if v > 0 else None
    line = {"metric": cls.metric, "value": round(v, 4), "unit": cls.unit, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 3) if ms_step else None,
            "ms_per_step_note": "one full step at the sampled CPU rate",
            "higher_is_better": True, "scaling": "strong" if cls is Transformer else "weak",
            "vs_baseline": None, "dtype": "bf16" if cls in (Transformer, Gemm) else "f32", "data": "synthetic",
            "config": cls.describe(args.gpus), "impl": "reference",
            "cpu_baseline": {"value": round(v, 4), "unit": cls.unit, "cores": cores, "kind": "port",
                             "sample": sample + " (oracle/, restatement of the reference's path)"},
            "e2e": {"value": round(v, 4), "unit": cls.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)


def cls_name_binds(workload: str) -> bool:
    """Workloads whose e2e leg moves host buffers (every one but the
    host-latency ones) run bound to their GPU's NUMA node."""
    return workload not in ("tlsf", "decode")


def emit(line: dict) -> None:
    """The result line goes to the process's original stdout; everything the
    native libraries print goes to stderr (fd 1 is redirected in main)."""
    os.write(_OUT_FD, (json.dumps(line) + "\n").encode())


_OUT_FD = 1


def main():
    global _OUT_FD
    _OUT_FD = os.dup(1)
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="transformer", choices=sorted(WORKLOADS))
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--no-subresults", action="store_true")
    ap.add_argument("--elements", type=int, default=None,
                    help="fused_elementwise only: stream length (default 2^20, the configured workload)")
    ap.add_argument("--global-batch", type=int, default=None,
                    help="transformer only: a smaller global batch (profiling case); default 64")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    numa = bind_to_gpu_numa_node(torch, local) if cls_name_binds(args.workload) else None
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=torch.device("cuda", local))

    from fercuda_b200 import capi, synth

    cls = WORKLOADS[args.workload]
    pool = 12 << 30 if cls is Transformer else 4 << 30
    if cls is Chain and args.elements:
        # the session pool is split into mutable / immutable halves; the
        # rotating x / y buffers all come from the mutable half
        nbuf = max(2, min(48, (384 << 20) // (8 * args.elements)))
        pool = max(pool, 2 * (2 * nbuf * 4 * args.elements) + (1 << 30))
    s = capi.Session(local, pool_bytes=pool)
    stream = torch.cuda.ExternalStream(s.stream())

    if cls is Decode:
        if rank == 0:
            clocks = ClockSampler(local)
            clocks.start()
            time.sleep(0.25)
            clocks.mark(True)
            r = decode_steps(s, capi, synth, torch, steps=args.steps)
            clocks.mark(False)
            line = {"metric": r["metric"], "value": r["value"], "unit": r["unit"], "n_gpus": 1, "steps": args.steps,
                    "warmup": 4, "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "weak",
                    "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                    "config": {"workload": "decode_L8_d1024_h16_F4096_V32000_B64_prompt512",
                               "batch": r["batch"], "prompt": r["prompt"]},
                    "roofline": r["roofline"], "prefill_ms": r["prefill_ms"], "clocks": clocks.stop(),
                    "device_error_bits": r["device_error_bits"], "api": r["api"]}
            emit(line)
        s.close()
        if world > 1:
            dist.destroy_process_group()
        return

    if cls is Tlsf:
        if rank == 0:
            tl = Tlsf(s, capi, synth).run()
            line = {"metric": Tlsf.metric, "value": tl["tlsf"]["alloc_p50_ns"], "unit": "ns", "n_gpus": world,
                    "steps": 1, "warmup": 0, "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
                    "dtype": "int64", "data": "synthetic",
                    "config": {"workload": "tlsf_stress_1M_ops_seed2", "pool": "80 GiB", "fill": "fer_fill_u32 per alloc"},
                    "results": tl, "host_only": (host := Tlsf.cpu_reference()),
                    "cpu_baseline": {"value": ((host or {}).get("reference") or {}).get("alloc_p50_ns"),
                                                    "unit": "ns", "cores": 1, "kind": "reference",
                                                    "sample": "full trace, reference TLSF host-only"}}
            emit(line)
        s.close()
        if world > 1:
            dist.destroy_process_group()
        return

    wl = cls(s, capi, synth, rank=rank, world=world, dist=dist, torch=torch, batch=args.global_batch) \
        if cls is Transformer \
        else (cls(s, capi, synth, n=args.elements) if cls is Chain and args.elements else cls(s, capi, synth))

    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.25)
    clocks.mark(True)
    elapsed = timed_steps(wl, torch, stream, args.steps, args.warmup, dist, world)
    clocks.mark(False)
    clk = clocks.stop()
    elapsed = max_over_ranks(elapsed, torch, dist, world)
    errs = s.device_errors()
    prof = None
    if cls is Transformer:
        # per-class device time from event pairs around every launch, on a
        # separate pass so that the timed steps above carry no extra events
        wl.model.profile(True)
        for i in range(3):
            wl.step(i)
        prof = wl.model.profile_read()
        wl.model.profile(False)

    # end to end through the C ABI with pinned host buffers
    e2e_steps = args.e2e_steps or (5 if cls is Transformer else max(3, min(args.steps, 20)))
    wl.e2e_prepare(torch)
    wl.e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = time.perf_counter()
    for _ in range(e2e_steps):
        wl.e2e_step()
    e2e_rank_s = time.perf_counter() - e0
    e2e_s = max_over_ranks(e2e_rank_s, torch, dist, world)
    # this rank's host<->device rate over the e2e steps (compute included)
    d2h_gbs = wl.d2h * e2e_steps / e2e_rank_s / 1e9
    d2h_all = [d2h_gbs]
    if world > 1:
        d2h_all = [None] * world
        dist.all_gather_object(d2h_all, round(d2h_gbs, 2))

    digest = None
    if cls is Transformer:
        # per-sequence digests of the logits of the last timed forward,
        # gathered in sequence order: equal across GPU counts bit for bit
        mine = wl.digests()
        if world > 1:
            parts = [None] * world
            dist.all_gather_object(parts, (wl.first_seq, mine))
        else:
            parts = [(wl.first_seq, mine)]
        seqs = [d for _, ds in sorted(parts) for d in ds]
        print(json.dumps({"rank": rank, "first_sequence": wl.first_seq,
                          "logits_digests": [f"{d:016x}" for d in mine]}), file=sys.stderr)
        import hashlib

        digest = {"sequences": len(seqs),
                  "all": hashlib.sha256(np.array(seqs, np.uint64).tobytes()).hexdigest()[:16],
                  "seq0": f"{seqs[0]:016x}", "seq63": f"{seqs[-1]:016x}"}

    # steady state: a longer untimed run (>= 200 steps, >= 1 s) with its own
    # clock samples, beside the K timed steps of the contract
    steady = None
    if cls is Transformer:
        n_steady = max(200, int(1000.0 / max(1e-3, elapsed / args.steps)))
        clocks2 = ClockSampler(local)
        clocks2.start()
        time.sleep(0.25)
        clocks2.mark(True)
        el2 = timed_steps(wl, torch, stream, n_steady, 0, dist, world)
        clocks2.mark(False)
        el2 = max_over_ranks(el2, torch, dist, world)
        steady = {"steps": n_steady, "ms_per_step": round(el2 / n_steady, 5),
                  "tokens_per_s": round(wl.global_tokens * n_steady / (el2 * 1e-3), 1), "clocks": clocks2.stop()}

    if rank == 0:
        if cls is Transformer:
            value = wl.global_tokens * args.steps / (elapsed * 1e-3)
            e2e_v = wl.global_tokens * e2e_steps / e2e_s
            roof = wl.roofline_from_profile(prof, elapsed / args.steps)
            launches = int(round(prof.launches / max(1, prof.forwards))) * args.steps
            unit_scale = 1.0
        else:
            unit_scale = 1e12 if cls is Gemm else 1e9
            value = wl.units_per_step * args.steps * world / (elapsed * 1e-3) / unit_scale
            e2e_v = wl.units_per_step * e2e_steps * world / e2e_s / unit_scale
            roof = wl.roofline(elapsed / args.steps)
            launches = wl.launches_per_step * args.steps
        cpu_base = None
        if world == 1:
            unbind()
            cv, sample, cores = cls.cpu(host_threads())
            cpu_base = {"value": round(cv, 4), "unit": cls.unit, "cores": cores, "kind": "port",
                        "sample": sample + " (oracle/, restatement of the reference's path)"}
        line = {"metric": cls.metric, "value": round(value, 3), "unit": cls.unit, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(elapsed / args.steps, 5),
                "higher_is_better": True, "scaling": "strong" if cls is Transformer else "weak",
                "vs_baseline": None, "dtype": "bf16" if cls in (Transformer, Gemm) else "f32", "data": "synthetic",
                "config": wl.config(world),
                "e2e": {"value": round(e2e_v, 3), "unit": cls.unit, "h2d_bytes_per_step": wl.h2d * world,
                        "d2h_bytes_per_step": wl.d2h * world, "steps": e2e_steps,
                        "api": getattr(wl, "e2e_api",
                                       "fer_upload_bytes + submit + fer_download_bytes (pinned host buffers)"),
                        "d2h_gbs_per_rank": [round(x, 2) for x in d2h_all], "numa": numa},
                "roofline": roof, "cpu_baseline": cpu_base, "clocks": clk, "gpu_launches": launches,
                "device_error_bits": errs}
        if cls is Transformer:
            line["weight_broadcast_bytes"] = wl.broadcast_bytes
            line["weight_broadcast"] = "fer_transformer_broadcast_weights (NCCL, C++)" if world > 1 else "none (1 GPU)"
            line["logits_digest"] = digest
            line["steady"] = steady
            line["profile_ms_per_forward"] = {k: round(getattr(prof, k) / max(1, prof.forwards), 4)
                                              for k in ("gemm_ms", "attn_ms", "norm_ms", "other_ms")}
        if world == 1 and cls is Transformer and not args.no_subresults:
            wl.model.close()
            s.free(wl.bl)
            full = subresults(s, capi, synth, torch, stream)
            print(json.dumps({"subresults": full}), file=sys.stderr)
            line["subresults"] = compact(full)
        emit(line)
    if world > 1:
        dist.barrier()
    s.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
