#!/usr/bin/env python
"""Benchmark of the B200 conv/GEMM backend (one JSON line on rank 0).

Workload (N=1 and per rank for N>1, weak scaling by batch): BASELINE config 2,
one int8 QLinearConv layer x u8 [32,256,14,14] * w s8 [256,256,3,3], pads 1,
NCHW in/out, requant R1 (what nnr dispatches for this layer), seeded
synthetic data (numpy PCG64, seed 1).

  value  device-resident throughput (TOPS) of the whole operator (NCHW->NHWC
         reorder + implicit-GEMM conv), inputs already in HBM, L2 flushed
         between timed steps (a 256 MB write), CUDA events on the launching
         stream, max over ranks.
  e2e    the same operator through the C ABI with host buffers: pinned H2D of
         x, the operator, D2H of y, all inside the timed region.
  roofline  the conv kernel alone (NHWC input, same kernel the operator
         launches) against the int8 tensor peak.

--impl reference times nnr's own CPU implementation of the layer (its
AVX-512 VNNI direct conv compiled from the nnr sources into oracle/_ref,
plus the R1 requant of exec_direct_int8) on the host cores, or the C
restatement when that harness is unavailable.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "QLinearConv TOPS vs int8 tensor peak"
UNIT = "TOPS"
WORKLOAD = "config2_qlinearconv_u8_32x256x14x14_k3x3"
L2_FLUSH_BYTES = 256 << 20


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples the SM clock and the clock-event (throttle) reasons through NVML
    (read-only queries) every 50 ms while the GPU is under load. The device is
    looked up by its UUID, so CUDA_VISIBLE_DEVICES remapping does not matter."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}

    def __init__(self, torch_index: int):
        self.torch_index = torch_index
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self.error = None

    def __enter__(self):
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(self.torch_index).uuid)
            h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)

            def run():
                while not self._stop.is_set():
                    try:
                        mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                        rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.samples.append((mhz, rs))
                    except Exception as e:  # noqa: BLE001
                        self.error = str(e)
                    self._stop.wait(0.05)

            self.t = threading.Thread(target=run, daemon=True)
            self.t.start()
        except Exception as e:  # noqa: BLE001
            self.error = str(e)
        return self

    def __exit__(self, *a):
        self._stop.set()
        if hasattr(self, "t"):
            self.t.join(timeout=2)

    def summary(self):
        sm = [m for m, _ in self.samples]
        reasons = sorted({k for _, rs in self.samples for k, bit in self.REASONS.items() if rs & bit})
        out = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz, "reasons": reasons,
               "samples": len(sm), "source": "NVML during spin-up + timed region"}
        if self.error and not sm:
            out["error"] = self.error
        return out


# ------------------------------------------------------------------ reference arm
def reference_arm(args, rank, world):
    if rank != 0:
        return 0
    from nnr_b200 import workloads as W
    from oracle import oracle as O
    case = W.config2_qlinearconv()
    kind = "reference"
    fn = lambda: O.ref_qlinearconv_direct(case.x, case.w, case.w_scale, case.bias, case.x_scale, case.x_zp,
                                          case.y_scale, case.y_zp, pads=case.pads)
    cores = None
    if fn() is None:
        kind = "port"
        fn = lambda: O.qlinearconv(case.x, case.w, case.w_scale, case.bias, case.x_scale, case.x_zp, case.y_scale,
                                   case.y_zp, pads=case.pads, formula=O.R1)
        cores = O.num_threads()
    else:
        cores = O.ref_lib().ref_get_threads()
    for _ in range(args.warmup):
        fn()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    ms = 1000 * sum(times) / len(times)
    tops = case.ops / (ms / 1000) / 1e12
    line = {"metric": METRIC, "value": round(tops, 4), "unit": UNIT, "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic (seeded numpy PCG64)",
            "config": {"workload": WORKLOAD, "batch_per_gpu": 32},
            "cpu_baseline": {"value": round(tops, 4), "unit": UNIT, "cores": cores, "kind": kind,
                             "sample": "the full config-2 layer (32 images) per step on the host cores"},
            "e2e": {"value": round(tops, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def cpu_baseline(case):
    """nnr's own kernel (or the C restatement) on a bounded sample: repeat the
    full layer for ~10 s."""
    from oracle import oracle as O
    kind = "reference"
    fn = lambda: O.ref_qlinearconv_direct(case.x, case.w, case.w_scale, case.bias, case.x_scale, case.x_zp,
                                          case.y_scale, case.y_zp, pads=case.pads)
    if fn() is None:
        kind = "port"
        fn = lambda: O.qlinearconv(case.x, case.w, case.w_scale, case.bias, case.x_scale, case.x_zp, case.y_scale,
                                   case.y_zp, pads=case.pads, formula=O.R1)
        cores = O.num_threads()
    else:
        cores = O.ref_lib().ref_get_threads()
    fn()
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < 10.0:
        fn()
        n += 1
    dt = (time.perf_counter() - t0) / n
    return {"value": round(case.ops / dt / 1e12, 4), "unit": UNIT, "cores": cores, "kind": kind,
            "sample": f"full config-2 layer (32 images) x {n} repetitions, {dt * 1000:.2f} ms each"}


# ------------------------------------------------------------------ B200 arm
def main():
    args = parse()
    rank, world, local = dist_env()
    if args.impl == "reference":
        return reference_arm(args, rank, world)
    assert args.warmup >= 3, "at least 3 warm-up steps"

    import torch
    import torch.distributed as dist
    from nnr_b200 import ops, workloads as W
    from nnr_b200._lib import RQ_AUTO

    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    ops.init(local)
    dev = torch.device("cuda", local)

    case = W.config2_qlinearconv()
    op = ops.QLinearConv(case.x.shape, case.w, case.w_scale, case.w_zp, case.bias, case.x_scale, case.x_zp,
                         case.y_scale, case.y_zp, pads=case.pads, requant=RQ_AUTO)
    # The conv kernel the operator launches, alone (roofline): the operator
    # reorders the NCHW input into an x_zp-bordered NHWC copy and runs the
    # im2col kernel on it with zero pads; op_k does exactly that on a copy
    # prepared once.
    n_, c_, h_, w_ = case.x.shape
    x_pad = np.full((n_, h_ + 2, w_ + 2, c_), case.x_zp, np.uint8)
    x_pad[:, 1:-1, 1:-1, :] = case.x.transpose(0, 2, 3, 1)
    op_k = ops.QLinearConv((n_, c_, h_ + 2, w_ + 2), case.w, case.w_scale, case.w_zp, case.bias, case.x_scale,
                           case.x_zp, case.y_scale, case.y_zp, pads=(0, 0, 0, 0), requant=1, in_layout="NHWC")
    stream = torch.cuda.Stream(device=dev)
    x = torch.from_numpy(case.x).to(dev)
    x_nhwc = torch.from_numpy(x_pad).to(dev)
    y = torch.empty(op.y_shape, dtype=torch.uint8, device=dev)
    ws = torch.empty(max(op.workspace_size(), 1), dtype=torch.uint8, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    x_host = torch.from_numpy(case.x).pin_memory()
    y_host = torch.empty(op.y_shape, dtype=torch.uint8).pin_memory()

    def step():
        op.exec(x, y, ws, stream=stream)

    def step_kernel():
        op_k.exec(x_nhwc, y, None, stream=stream)

    def step_e2e():
        with torch.cuda.stream(stream):
            x.copy_(x_host, non_blocking=True)
            op.exec(x, y, ws, stream=stream)
            y_host.copy_(y, non_blocking=True)

    def timed(fn, steps):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for i in range(steps):
            with torch.cuda.stream(stream):
                flush.zero_()
            ev[i][0].record(stream)
            fn()
            ev[i][1].record(stream)
        stream.synchronize()
        return sum(a.elapsed_time(b) for a, b in ev)  # ms

    for _ in range(args.warmup):
        step(); step_kernel(); step_e2e()
    stream.synchronize()
    assert ops.device_status() == 0

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    with ClockSampler(local) as clk:
        # Spin the GPU up to its load clocks (it idles near 120 MHz) before
        # timing: ~1 s of back-to-back steps, sampled as well.
        t_end = time.perf_counter() + 1.0
        while time.perf_counter() < t_end:
            for _ in range(50):
                step()
            stream.synchronize()
        barrier()
        total_ms = timed(step, args.steps)
        barrier()
        k_ms = timed(step_kernel, args.steps)
        e2e_ms = timed(step_e2e, args.steps)
        barrier()
    assert ops.device_status() == 0

    t = torch.tensor([total_ms, k_ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, k_ms, e2e_ms = t.tolist()

    ms = total_ms / args.steps
    value = world * case.ops / (ms / 1e3) / 1e12
    e2e_val = world * case.ops / (e2e_ms / args.steps / 1e3) / 1e12
    k_avg = k_ms / args.steps
    achieved = case.ops / (k_avg / 1e3) / 1e12

    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    bf16 = peaks.get("bf16_tflops")
    if bf16:
        peak, peak_note = 2.0 * bf16, "2x measured bf16 burst (MEASURED_PEAKS.json): dense int8 runs at twice the bf16 rate"
    else:
        peak, peak_note = 2.0 * 1590.0, "2x fallback bf16 1.59 PFLOP/s"

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u8", "data": "synthetic (seeded numpy PCG64, BASELINE config 2)",
            "config": {"workload": WORKLOAD, "batch_per_gpu": 32, "layout": "NCHW in/out (nnr default)",
                       "requant": "R1 (nnr exec_direct_int8)", "l2": "flushed between timed steps (256 MB write)",
                       "parallelism": f"dp{world} (independent replicas, batch-sharded)"},
            "e2e": {"value": round(e2e_val, 3), "unit": UNIT, "h2d_bytes_per_step": int(case.x.nbytes),
                    "d2h_bytes_per_step": int(np.prod(op.y_shape))},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(peak, 1), "unit": "TOPS",
                         "frac": round(achieved / peak, 4), "traffic": None, "kernel_ms": round(k_avg, 5),
                         "peak_source": peak_note},
            "gpu_launches": 2 * args.steps,
            "clocks": clk.summary(),
        }
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline(case)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
