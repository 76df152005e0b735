"""Benchmark of the hot path, one JSON line on rank 0.

Default workload (N = 1): row softmax followed by layer norm (gamma 1, beta 0,
eps 1e-5) over f32 [4096, 4096], entries N(0,1) from seed 1 - one step is one
fused pass over the whole batch through fer_submit_rows. For N > 1 every rank
runs the same workload on its own GPU (replicas, weak scaling); `value` sums
all ranks' bytes over the slowest rank's time.

  value    algorithmic HBM bytes (read x + write y = 8 B/element) per second,
           device-timed with CUDA events over exactly K steps, inputs resident;
           L2 is defeated by rotating over 3 input/output pairs (384 MiB > L2)
  e2e      the same bytes per second through the C ABI with host buffers:
           fer_upload_bytes (pinned) + fer_submit_rows + fer_download_bytes
  roofline achieved GB/s of the fused row kernel (per-launch CUDA events)
           against the measured HBM copy bandwidth of MEASURED_PEAKS.json
  cpu_baseline the oracle (CPU restatement, C, all host threads) on the same
           workload

--impl reference runs the reference's CPU implementation of the path (the
oracle port) with all host threads on the same config instead.
--workload fused_elementwise measures y = relu(1.5x - 0.25) * sigmoid(x) over
2^20 f32 through fer_tensor_run_affine_f32 the same way.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import math
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

HBM_FALLBACK_GBS = 6650.0


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d.get("hbm_gbs", HBM_FALLBACK_GBS)), "measured"
    return HBM_FALLBACK_GBS, "fallback"


def profiled_traffic(name: str):
    """Per-launch DRAM bytes of a kernel from its committed ncu summary
    (a `traffic_bytes_per_launch: N` line in profiles/<name>.md), or None."""
    p = ROOT / "profiles" / f"{name}.md"
    if not p.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9]+)", p.read_text())
    return int(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 50 ms."""

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.proc = None
        self.t0 = self.t1 = None

    def start(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

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
        lo, hi = (self.t0 or 0) - 0.1, (self.t1 or time.time()) + 0.1
        sel = [s for t, s in self.samples if lo <= t <= hi] or [s for _, s in self.samples[-3:]]
        sm = [float(s[1]) for s in sel if len(s) > 8 and s[1].replace(".", "").isdigit()]
        smax = [float(s[2]) for s in sel if len(s) > 8 and s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in sel if len(s) > 8 for i in range(4) if s[5 + i] == "Active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(sel)}


# ------------------------------------------------------------------ workloads

class RowsWorkload:
    name = "softmax_layernorm"
    kernel = "rows_softmax_layernorm_4096x4096"

    def __init__(self, s, capi, synth, rows=4096, cols=4096):
        self.s, self.capi = s, capi
        self.rows, self.cols = rows, cols
        self.eps = synth.SOFTMAX_LAYERNORM["eps"]
        self.x = synth.softmax_layernorm_input(rows, cols)
        self.pairs = []
        for _ in range(3):
            bx, by = s.alloc(capi.FER_DTYPE_F32, [rows, cols]), s.alloc(capi.FER_DTYPE_F32, [rows, cols])
            s.upload(bx, self.x)
            self.pairs.append((bx, by))
        self.req = [capi.fer_rows_request_t(bx, by, 0, 0, self.eps, capi.FER_ROWS_SOFTMAX | capi.FER_ROWS_LAYER_NORM,
                                            capi.FER_MEMORY_AUTO) for bx, by in self.pairs]
        self.job = C.c_uint64()
        self.bytes_per_step = 8 * rows * cols
        self.h2d = self.d2h = 4 * rows * cols

    def step(self, i):
        st = self.s.call("fer_submit_rows", C.byref(self.req[i % 3]), C.byref(self.job))
        if st.code:
            raise RuntimeError(st.message)

    def config(self):
        return {"workload": f"softmax_layernorm_{self.rows}x{self.cols}_f32", "rows": self.rows, "cols": self.cols,
                "eps": self.eps, "gamma": 1.0, "beta": 0.0, "input": "N(0,1) seed 1",
                "l2": "rotating 3 input/output pairs (384 MiB > 126 MB L2)", "api": "fer_submit_rows"}

    def e2e_step(self, hx, hy):
        bx, by = self.pairs[0]
        self.s.upload(bx, hx)
        self.step(0)
        self.s.download(by, hy)

    def cpu(self, orc, threads, reps=3):
        y = np.empty_like(self.x)
        t0 = time.perf_counter()
        for _ in range(reps):
            orc.orc_softmax_layernorm_rows_f32(self.x.ctypes.data_as(C.c_void_p), y.ctypes.data_as(C.c_void_p),
                                               self.rows, self.cols, C.c_float(self.eps), threads)
        dt = (time.perf_counter() - t0) / reps
        return self.bytes_per_step / dt / 1e9, f"full {self.rows}x{self.cols} batch x{reps}"


class ChainWorkload:
    name = "fused_elementwise"
    kernel = "fused_chain_2p20"

    def __init__(self, s, capi, synth, n=1 << 20):
        self.s, self.capi = s, capi
        c = synth.FUSED_ELEMENTWISE
        self.n, self.a, self.b = n, c["a"], c["b"]
        self.x = synth.fused_elementwise_input(n)
        self.nbuf = max(3, (384 << 20) // (8 * n))
        self.pairs = []
        for _ in range(self.nbuf):
            bx, by = s.alloc(capi.FER_DTYPE_F32, [n]), s.alloc(capi.FER_DTYPE_F32, [n])
            s.upload(bx, self.x)
            self.pairs.append((bx, by))
        self.fusion = capi.FER_JIT_INTENT_FUSION_RELU | capi.FER_JIT_INTENT_FUSION_MUL_SIGMOID_INPUT
        self.job = C.c_uint64()
        self.lib = s.lib
        self.bytes_per_step = 8 * n
        self.h2d = self.d2h = 4 * n
        s.wait(s.affine(*self.pairs[0], n, self.a, self.b, self.fusion))   # compile once

    def step(self, i):
        bx, by = self.pairs[i % self.nbuf]
        st = self.lib.fer_tensor_run_affine_f32(self.s.ptr, self.capi.fer_tensor_handle_t(bx),
                                                self.capi.fer_tensor_handle_t(by), self.n, self.a, self.b,
                                                self.fusion, 0, self.capi.FER_MEMORY_AUTO, C.byref(self.job))
        if st.code:
            raise RuntimeError(st.message)

    def config(self):
        return {"workload": f"fused_elementwise_relu_affine_mul_sigmoid_{self.n}_f32", "n": self.n, "a": self.a,
                "b": self.b, "input": "U(-4,4) seed 0",
                "l2": f"rotating {self.nbuf} input/output pairs ({self.nbuf * 8 * self.n >> 20} MiB > 126 MB L2)",
                "api": "fer_tensor_run_affine_f32 (fusion RELU|MUL_SIGMOID_INPUT)"}

    def e2e_step(self, hx, hy):
        bx, by = self.pairs[0]
        self.s.upload(bx, hx)
        self.step(0)
        self.s.download(by, hy)

    def cpu(self, orc, threads, reps=20):
        y = np.empty_like(self.x)
        t0 = time.perf_counter()
        for _ in range(reps):
            orc.orc_chain_f32(self.x.ctypes.data_as(C.c_void_p), y.ctypes.data_as(C.c_void_p), self.n,
                              C.c_float(self.a), C.c_float(self.b), threads)
        dt = (time.perf_counter() - t0) / reps
        return self.bytes_per_step / dt / 1e9, f"full 2^20 batch x{reps}"


WORKLOADS = {"softmax_layernorm": RowsWorkload, "fused_elementwise": ChainWorkload}


# ------------------------------------------------------------------ main

def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(args, rank, world):
    """The reference's CPU implementation of the path (oracle port), rank 0."""
    if rank != 0:
        return
    from fercuda_b200 import synth
    from tests import oracle_lib

    orc = oracle_lib.load()
    threads = host_threads()
    if args.workload == "softmax_layernorm":
        x = synth.softmax_layernorm_input()
        rows, cols = x.shape
        y = np.empty_like(x)
        fn = lambda: orc.orc_softmax_layernorm_rows_f32(x.ctypes.data_as(C.c_void_p), y.ctypes.data_as(C.c_void_p),
                                                        rows, cols, C.c_float(1e-5), threads)
        nbytes = 8 * rows * cols
        cfg = RowsWorkload.config(type("W", (), {"rows": rows, "cols": cols, "eps": 1e-5})())
    else:
        x = synth.fused_elementwise_input()
        y = np.empty_like(x)
        fn = lambda: orc.orc_chain_f32(x.ctypes.data_as(C.c_void_p), y.ctypes.data_as(C.c_void_p), x.size,
                                       C.c_float(1.5), C.c_float(-0.25), threads)
        nbytes = 8 * x.size
        cfg = {"workload": f"fused_elementwise_relu_affine_mul_sigmoid_{x.size}_f32"}
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn()
    dt = time.perf_counter() - t0
    v = nbytes * args.steps / dt / 1e9
    line = {"metric": "HBM GB/s (fused elementwise, softmax)", "value": round(v, 3), "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt / args.steps * 1e3, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg, "impl": "reference",
            "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": "full batch per step (oracle/oracle.c restatement of the reference kernels)"},
            "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="softmax_layernorm", choices=sorted(WORKLOADS))
    ap.add_argument("--e2e-steps", type=int, default=None)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))

    from fercuda_b200 import capi, synth

    s = capi.Session(local, pool_bytes=2 << 30)
    wl = WORKLOADS[args.workload](s, capi, synth)
    stream = torch.cuda.ExternalStream(s.stream())

    for i in range(args.warmup):
        wl.step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    t_all0, t_all1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks.mark(True)
    t_all0.record(stream)
    for i in range(args.steps):
        starts[i].record(stream)
        wl.step(args.warmup + i)
        ends[i].record(stream)
    t_all1.record(stream)
    torch.cuda.synchronize()
    clocks.mark(False)
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    elapsed_ms = t_all0.elapsed_time(t_all1)
    kern_ms = [a.elapsed_time(b) for a, b in zip(starts, ends)]
    t = torch.tensor([elapsed_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms = float(t.item())
    errs = s.device_errors()

    # end to end through the C ABI with pinned host buffers
    e2e_steps = args.e2e_steps or max(3, min(args.steps, 20))
    hx = torch.from_numpy(wl.x.reshape(-1)).pin_memory().numpy()
    hy = torch.empty(hx.size, dtype=torch.float32).pin_memory().numpy()
    wl.e2e_step(hx, hy)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = time.perf_counter()
    for _ in range(e2e_steps):
        wl.e2e_step(hx, hy)
    e2e_s = time.perf_counter() - e0
    te = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_s = float(te.item())

    if rank == 0:
        peak, peak_src = peaks()
        med = float(np.median(kern_ms))
        achieved = wl.bytes_per_step / (med * 1e-3) / 1e9
        value = wl.bytes_per_step * args.steps * world / (elapsed_ms * 1e-3) / 1e9
        cpu_base = None
        if world == 1:
            from tests import oracle_lib

            cv, sample = wl.cpu(oracle_lib.load(), host_threads())
            cpu_base = {"value": round(cv, 3), "unit": "GB/s", "cores": host_threads(), "kind": "port",
                        "sample": sample + ", oracle/oracle.c (C restatement of the reference kernels), all host threads"}
        traffic = profiled_traffic(wl.kernel)
        line = {
            "metric": "HBM GB/s (fused elementwise, softmax)", "value": round(value, 2), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(elapsed_ms / args.steps, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": wl.config(),
            "e2e": {"value": round(wl.bytes_per_step * e2e_steps * world / e2e_s / 1e9, 3), "unit": "GB/s",
                    "h2d_bytes_per_step": wl.h2d, "d2h_bytes_per_step": wl.d2h, "steps": e2e_steps,
                    "api": "fer_upload_bytes + submit + fer_download_bytes, pinned host buffers"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "algorithmic_bytes_per_launch": wl.bytes_per_step, "peak_source": peak_src,
                         "kernel_ms_median": round(med, 5)},
            "cpu_baseline": cpu_base,
            "clocks": clk,
            "gpu_launches": args.steps,
            "device_error_bits": errs,
        }
        print(json.dumps(line), flush=True)
    s.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
