#!/usr/bin/env python
"""Benchmark of the B200 conv/GEMM backend (one JSON line on rank 0).

Metric (BASELINE): int8 ResNet-50 images/s at 1/2/4/8 B200; QLinearConv TOPS
vs int8 tensor peak.

Workload: BASELINE config 4, the ResNet-50 v1 QDQ int8 network built from
seed 3 (nnr_b200/resnet50.py), 32 images per GPU (weak scaling: rank r runs
images [32r, 32r + 32) of the seeded 256-image N(0,1) batch). One step is one
forward pass of the batch: QuantizeLinear of the fp32 input, 53 QLinearConv,
MaxPool, 16 QLinearAdd, DQ-GAP-Q, QLinearMatMul and DQ + bias, replayed from
one captured CUDA graph.

  value     images/s of the device-resident forward (input already in HBM),
            L2 flushed (192 MB write, 1.5x the 126 MB L2) before every timed step, CUDA events on
            the launching stream, max over ranks.
  e2e       the same forward through the public API with host buffers:
            every step a pinned H2D of its fp32 input batch, the forward and
            a D2H of the fp32 logits, pipelined (DeviceNetwork.forward_many:
            a step's H2D runs on a copy stream into one of two staging
            buffers while the previous step computes; each forward is the
            graph captured on its staging buffer), L2 flushed before each
            forward, one CUDA-event window over all steps; the serial form
            (copy, forward, copy per step) is reported beside it as
            serial_value, and the measured H2D GB/s of the link beside both.
  roofline  the tcgen05 conv/matmul kernels of the forward: every step is
            timed alone (10 launches replayed from a CUDA graph, CUDA events
            on the launching stream); the engine steps' share of those times
            scaled to the timed forward gives their time inside it;
            algorithmic int8 ops / that time vs the int8 tensor peak (the
            larger of a live library int8 GEMM probe and 2x the measured
            bf16 burst), plus the per-layer attainable roofline
            (max of tensor and HBM floors per layer).
  qlinearconv_config2  BASELINE config 2 (one QLinearConv layer, NCHW in/out,
            requant R1): operator and kernel TOPS.

--impl reference runs nnr's own CPU runtime (compiled from its sources into
oracle/_ref) on the same QDQ graph at batch 32 on all host threads. nnr's int8
QLinearConv/QLinearMatMul need the absent Xbyak JIT, so nnr runs the QDQ convs
on its fake-quant float path; without the runtime it falls back to the C
restatement of nnr's int8 operators.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import pickle
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "int8 ResNet-50 images/s at 1/2/4/8 B200; QLinearConv TOPS vs int8 tensor peak"
UNIT = "images/s"
WORKLOAD = "config4_resnet50_v1_qdq_int8_b32_per_gpu"
BATCH = 32
L2_FLUSH_BYTES = 192 << 20  # 1.5x the 126 MB L2


# DRAM bytes (read + write) of all tc_gemm_kernel launches of one batch-32
# forward, summed over one ncu capture of the forward's launch list
# (ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum).
TC_TRAFFIC_BYTES = 473_100_000


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def load_model(batch, rank, world, barrier):
    """Rank 0 builds the seeded model once and shares it with the other ranks
    (the build includes a float calibration pass on the CPU)."""
    from nnr_b200 import replicas, resnet50
    port = os.environ.get("MASTER_PORT", "0")
    return replicas.build_once(lambda: resnet50.build(batch=batch), f"resnet50_s3_b{batch}_{port}", rank, world,
                               barrier)


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
                        self.samples.append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
                                             pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)))
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


# ------------------------------------------------------------------ CPU side
def host_cpu_info():
    """The host CPU as the reference arm sees it: model, logical and physical
    cores, the AVX-512 / VNNI / AMX flags nnr's x64 dispatch keys on, and the
    flags the C restatement was compiled with."""
    model, flags, phys = None, set(), set()
    cur = {}
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if ":" not in line:
                if cur:
                    phys.add((cur.get("physical id"), cur.get("core id")))
                cur = {}
                continue
            k, v = (x.strip() for x in line.split(":", 1))
            cur[k] = v
            if k == "model name" and model is None:
                model = v
            if k == "flags" and not flags:
                flags = set(v.split())
        if cur:
            phys.add((cur.get("physical id"), cur.get("core id")))
    except OSError:
        pass
    want = ["avx2", "fma", "avx512f", "avx512bw", "avx512vl", "avx512_vnni", "avx512_bf16", "avx512_fp16",
            "amx_int8", "amx_bf16"]
    return {"model": model, "logical_cores": os.cpu_count(), "usable_cores": len(os.sched_getaffinity(0)),
            "physical_cores": len(phys) or None, "isa_flags": [f for f in want if f in flags],
            "compiler": "gcc -O3 -march=x86-64-v3 -ffp-contract=off -fopenmp (oracle/Makefile)"}


def cpu_threads() -> int:
    """All host threads this process may use, set explicitly: torchrun exports
    OMP_NUM_THREADS=1 to its workers, which must not decide the baseline."""
    return len(os.sched_getaffinity(0))


def cpu_forward_fn(model, images):
    """One oracle forward of `images` images on the host cores (OpenMP)."""
    from nnr_b200 import resnet50
    from oracle import oracle as O
    O.set_threads(cpu_threads())
    x = resnet50.input_batch(0, images)
    return (lambda: O.run_qmodel(model, x)), O.num_threads()


NNR_SAMPLE_NOTE = ("nnr's own loader, graph passes and run loop (oracle/_ref/libnnr_cpu.so, compiled from the nnr "
                   "sources) on the config-4 QDQ ONNX graph. nnr's int8 QLinearConv/QLinearMatMul need the absent "
                   "Xbyak JIT, so its QDQ convs run as DequantizeLinear -> fp32 Conv -> QuantizeLinear (nnr's "
                   "fake-quant float path) and the residual adds as QLinearAdd. Memory planner and nChw16c layout "
                   "off: with them on nnr is slower and its logits are wrong on this graph.")


def nnr_cpu_forward_fn(model, batch):
    """One forward of nnr's own CPU runtime on the config-4 QDQ graph, or None
    when the runtime was not built."""
    from nnr_b200 import onnx_models, resnet50
    from oracle import nnr_ref as R
    if not R.available():
        return None
    R.set_threads(cpu_threads())
    net = R.NnrModel(onnx_models.resnet50_qdq(model), memory_planning=False, no_blocked=True)
    net.set("input", resnet50.input_batch(0, batch))

    def fn():
        net.run()
    return fn


def cpu_baseline(model, seconds=10.0):
    """The reference CPU timing beside the GPU line: nnr's own runtime on a
    bounded sample (4 images per forward, about `seconds` of CPU work), and
    the C restatement of nnr's int8 operators as a second figure."""
    from nnr_b200 import resnet50
    out = {}
    fn = nnr_cpu_forward_fn(resnet50.build(batch=4), 4)
    if fn is not None:
        fn()
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            fn()
            n += 1
        dt = (time.perf_counter() - t0) / n
        out = {"value": round(4.0 / dt, 3), "unit": UNIT, "cores": cpu_threads(), "kind": "reference",
               "sample": f"4 images per forward x {n} forwards ({dt * 1000:.0f} ms each). " + NNR_SAMPLE_NOTE}
    pfn, cores = cpu_forward_fn(model, 1)
    pfn()
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds / 2:
        pfn()
        n += 1
    dt = (time.perf_counter() - t0) / n
    port = {"value": round(1.0 / dt, 3), "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"1 image per forward x {n} forwards ({dt * 1000:.0f} ms each): the C restatement of nnr's "
                      "int8 operators (the oracle), exact int8 arithmetic"}
    if not out:
        out = port
    else:
        out["port"] = port
    out["cpu"] = host_cpu_info()
    return out


def nnr_cpu_other_configs(seconds=3.0):
    """nnr's own CPU runtime on BASELINE configs 1, 3 (fp32 Gemm) and 5
    (MobileNetV2, an 8-image sample; memory planner and nChw16c layout off,
    as nnr's logits are wrong with them on), all host threads: the CPU
    figures beside the GPU operator timings."""
    from nnr_b200 import mobilenetv2, onnx_models as M, workloads as W
    from oracle import nnr_ref as R
    if not R.available():
        return None
    R.set_threads(cpu_threads())

    def timed(net):
        net.run()
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            net.run()
            n += 1
        return (time.perf_counter() - t0) / n * 1e3
    c1 = W.config1_conv_relu()
    n1 = R.NnrModel(M.conv(c1.x.shape, c1.w, c1.bias, pads=c1.pads, post="Relu"))
    n1.set("x", c1.x)
    c3 = W.config3_matmul()
    n3 = R.NnrModel(M.gemm(4096, 768, 3072, c3.b_f32, c3.c_f32))
    n3.set("a", c3.a_f32)
    mb = mobilenetv2.build(batch=8)
    n5 = R.NnrModel(M.mobilenetv2(mb), memory_planning=False, no_blocked=True)
    n5.set("input", mobilenetv2.input_batch(0, 8))
    ms1, ms3, ms5 = timed(n1), timed(n3), timed(n5)
    return {"cores": cpu_threads(), "kind": "reference",
            "config1_conv_relu_ms": round(ms1, 4), "config3_gemm_fp32_ms": round(ms3, 3),
            "config5_mobilenetv2_images_per_s": round(8 / ms5 * 1e3, 2),
            "note": "nnr's CPU runtime compiled from its sources (oracle/_ref/libnnr_cpu.so)"}


def reference_arm(args, rank, world):
    """nnr's own CPU runtime on the GPU arm's config (batch 32 per step), all
    host threads; the C restatement when the runtime was not built."""
    if rank != 0:
        return 0
    from nnr_b200 import resnet50
    model = resnet50.build(batch=BATCH)
    fn = nnr_cpu_forward_fn(model, BATCH)
    if fn is not None:
        kind, cores, per_step = "reference", cpu_threads(), BATCH
        sample = f"the whole batch of {BATCH} per step. " + NNR_SAMPLE_NOTE
    else:
        fn, cores = cpu_forward_fn(model, 1)
        kind, per_step = "port", 1
        sample = "1 image of the batch per step, C restatement of nnr's int8 operators on the host cores"
    for _ in range(args.warmup):
        fn()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    ms = 1000 * sum(times) / len(times)
    val = per_step * 1000.0 / ms
    line = {"metric": METRIC, "value": round(val, 3), "unit": UNIT, "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 (fake-quant)" if kind == "reference" else "u8",
            "data": "synthetic (seeded numpy PCG64)",
            "config": {"workload": WORKLOAD, "sample": sample},
            "cpu_baseline": {"value": round(val, 3), "unit": UNIT, "cores": cores, "kind": kind, "sample": sample,
                             "cpu": host_cpu_info()},
            "e2e": {"value": round(val, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ B200 arm
def node_ops(model, i):
    """Algorithmic int8 ops (2 x MACs) of tensor-core node i."""
    nd = model.nodes[i]
    if nd.op == "QLinearConv":
        n, oh, ow, oc = model.shapes[nd.output]
        w = nd.attrs["w"]
        return 2 * n * oh * ow * oc * w.shape[1] * w.shape[2] * w.shape[3]
    b = nd.attrs["b"]
    return 2 * model.shapes[nd.output][0] * b.shape[0] * b.shape[1]


def node_bytes(model, net, t):
    """Compulsory HBM bytes of engine step t: u8 input (or the fp32 image the
    stem quantises), s8 weights, u8 output, plus the u8 residual of a fused
    QLinearAdd."""
    kind, j, ins, out, i = net.steps[t]
    nd = model.nodes[i]
    elem_in = 4 if ins[0] == "input" else 1
    b = int(np.prod(model.shapes[ins[0]])) * elem_in + int(np.prod(model.shapes[out]))
    b += nd.attrs["w"].size if nd.op == "QLinearConv" else nd.attrs["b"].size
    if kind == "QConvAdd":
        b += int(np.prod(model.shapes[ins[1]]))
    return b


def nnr_plugin_e2e(model, x_np, steps, device, flush, torch):
    """The same forward through nnr's own application path with the CUDA
    backend (libnnr_cuda.so: nnr's loader, fusion passes and run loop,
    preferred_backend = CUDA): the batch sits in nnr's own input tensor
    (host memory, filled in place), and every step is run() (upload, the
    replayed device graph, download) plus reading the logits; host wall
    clock around each step, L2 flushed before it."""
    from nnr_b200 import nnr_cuda as NC, onnx_models as M
    if not NC.available():
        return {"unavailable": "libnnr_cuda.so not built"}
    net = NC.NnrCudaModel(M.resnet50_qdq(model), device=device)
    try:
        net.input_array("input")[...] = x_np
        for _ in range(3):
            net.run()
            net.get("logits")
        ts = []
        for _ in range(steps):
            flush.zero_()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            net.run()
            net.get("logits")
            ts.append(time.perf_counter() - t0)
        st = net.stats()
    finally:
        net.close()
    ms = statistics.median(ts) * 1e3
    return {"value": round(x_np.shape[0] / ms * 1e3, 1), "unit": UNIT, "ms_per_step": round(ms, 4),
            "h2d_bytes_per_step": int(x_np.nbytes), "d2h_bytes_per_step": int(x_np.shape[0] * 1000 * 4),
            "n_gpus": 1, "graph_replays": st.get("graph_replays"), "device_ops": st.get("device_ops"),
            "host_ops": st.get("host_ops"),
            "mode": "nnr context_t::run() with the CUDA backend (nnr's memory planner off: its run() clears every "
                    "planned host slot each call), graph inputs/outputs page-locked, median of per-step wall clock"}


def int8_peak_probe(torch, dev, n=8192, reps=10):
    """Dense int8 tensor throughput of a large library GEMM (torch._int_mm,
    cuBLASLt; a probe only, not on the hot path): best of `reps` 8192^3
    multiplies, CUDA events."""
    try:
        a = torch.randint(-128, 127, (n, n), dtype=torch.int8, device=dev)
        b = torch.randint(-128, 127, (n, n), dtype=torch.int8, device=dev).t()
        for _ in range(3):
            torch._int_mm(a, b)
        best = float("inf")
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._int_mm(a, b)
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1))
        del a, b
        return {"tops": round(2 * n ** 3 / (best / 1e3) / 1e12, 1), "shape": f"{n}^3 s8 x s8 -> s32",
                "how": "torch._int_mm best of 10, CUDA events"}
    except Exception as e:  # noqa: BLE001
        return {"tops": None, "error": str(e)[:200]}


def config2_qlinearconv(ops, W, torch, dev, stream, flush, steps=50):
    """the QLinearConv operator (NCHW in/out, R1) and its
    conv kernel alone (on the x_zp-bordered NHWC copy the operator makes)."""
    case = W.config2_qlinearconv()
    op = ops.QLinearConv(case.x.shape, case.w, case.w_scale, case.w_zp, case.bias, case.x_scale, case.x_zp,
                         case.y_scale, case.y_zp, pads=case.pads)
    n_, c_, h_, w_ = case.x.shape
    x_pad = np.full((n_, h_ + 2, w_ + 2, c_), case.x_zp, np.uint8)
    x_pad[:, 1:-1, 1:-1, :] = case.x.transpose(0, 2, 3, 1)
    op_k = ops.QLinearConv((n_, c_, h_ + 2, w_ + 2), case.w, case.w_scale, case.w_zp, case.bias, case.x_scale,
                           case.x_zp, case.y_scale, case.y_zp, pads=(0, 0, 0, 0), requant=1, in_layout="NHWC")
    x = torch.from_numpy(case.x).to(dev)
    xk = torch.from_numpy(x_pad).to(dev)
    y = torch.empty(op.y_shape, dtype=torch.uint8, device=dev)
    ws = torch.empty(max(op.workspace_size(), 1), dtype=torch.uint8, device=dev)

    def timed(fn):
        for _ in range(5):
            fn()
        tot = 0.0
        for _ in range(steps):
            with torch.cuda.stream(stream):
                flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            e1.synchronize()
            tot += e0.elapsed_time(e1)
        return tot / steps

    op_ms = timed(lambda: op.exec(x, y, ws, stream=stream))
    k_ms = timed(lambda: op_k.exec(xk, y, None, stream=stream))
    return {"op_tops": round(case.ops / op_ms / 1e9, 1), "op_ms": round(op_ms, 5),
            "kernel_tops": round(case.ops / k_ms / 1e9, 1), "kernel_ms": round(k_ms, 5), "ops": case.ops}


def other_rows(ops, W, torch, dev, stream, flush, steps=30):
    """The other BASELINE configs as operator timings (device-resident inputs,
    L2 flushed before each step): config 1 fp32 Conv+Relu (NCHW in/out),
    config 3 fp32 Gemm and int8 QLinearMatMul. fp32 runs as split-bf16 (three
    bf16 products per multiply-add), so its peak is a third of the measured
    bf16 one."""
    def timed(fn):
        for _ in range(5):
            fn()
        tot = 0.0
        for _ in range(steps):
            with torch.cuda.stream(stream):
                flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            e1.synchronize()
            tot += e0.elapsed_time(e1)
        return tot / steps

    c1 = W.config1_conv_relu()
    conv = ops.Conv(c1.x.shape, c1.w, c1.bias, pads=c1.pads, post="Relu")
    x1 = torch.from_numpy(c1.x).to(dev)
    y1 = torch.empty(conv.y_shape, dtype=torch.float32, device=dev)
    ws1 = torch.empty(max(conv.workspace_size(), 1), dtype=torch.uint8, device=dev)
    ms1 = timed(lambda: conv.exec(x1, y1, None, ws1, stream=stream))
    f1 = 2 * 64 * 56 * 56 * 64 * 9
    c3 = W.config3_matmul()
    gemm = ops.Gemm(4096, c3.b_f32, c3.c_f32)
    a3 = torch.from_numpy(c3.a_f32).to(dev)
    y3 = torch.empty((4096, 3072), dtype=torch.float32, device=dev)
    ws3 = torch.empty(max(gemm.workspace_size(), 1), dtype=torch.uint8, device=dev)
    ms3 = timed(lambda: gemm.exec(a3, y3, ws3, stream=stream))
    qmm = ops.QLinearMatMul(4096, c3.b_s8, c3.a_scale, c3.a_zp, c3.b_scale, c3.b_zp, c3.y_scale, c3.y_zp)
    aq = torch.from_numpy(c3.a_u8).to(dev)
    yq = torch.empty((4096, 3072), dtype=torch.uint8, device=dev)
    wsq = torch.empty(max(qmm.workspace_size(), 1), dtype=torch.uint8, device=dev)
    msq = timed(lambda: qmm.exec(aq, yq, wsq, stream=stream))
    f3 = 2 * 4096 * 768 * 3072
    # config 5: MobileNetV2 fp32, batch 128 per GPU, one captured graph per forward
    from nnr_b200 import fgraph, mobilenetv2
    mb = mobilenetv2.build(batch=128)
    mnet = fgraph.FloatNetwork(mb, dev.index or 0)
    mnet.stream = stream  # launched (and timed) on the bench's stream
    mnet.view("input").copy_(torch.from_numpy(mobilenetv2.input_batch(0, 128)))
    mnet.capture()
    ms5 = timed(lambda: mnet.launch())
    # its depthwise 3x3 convs (CUDA cores, HBM bound): each step alone, inputs
    # far above L2 at batch 128; algorithmic bytes = input + output + weights
    dw_ms, dw_bytes, dw_best = 0.0, 0, None
    for t, (kind, j, ins, out, i) in enumerate(mnet.steps):
        nd = mb.nodes[i]
        if nd.op != "Conv" or nd.attrs.get("group", 1) == 1:
            continue
        ms = timed(lambda: mnet.run_step(t, stream.cuda_stream))
        # (an output linked to its projection is written as two bf16 planes
        # with the projection's padded channel stride: counted as written)
        n_out = int(np.prod(mb.shapes[out]))
        if out in mnet.plane_links:
            n_out = n_out // mb.shapes[out][3] * mnet.plane_links[out]
        nbytes = 4 * (int(np.prod(mb.shapes[ins[0]])) + n_out + nd.attrs["w"].size)
        dw_ms += ms
        dw_bytes += nbytes
        gbs = nbytes / ms / 1e6
        if dw_best is None or gbs > dw_best[1]:
            dw_best = (out, gbs)
    mnet.close()
    del mnet
    return {"config5_mobilenetv2_fp32": {"images_per_s": round(128 / ms5 * 1e3, 1), "ms_per_128": round(ms5, 4),
                                         "tflops": round(2 * mb.macs_per_image() * 128 / ms5 / 1e9, 1)},
            "config5_depthwise_f32": {"ms_per_128": round(dw_ms, 4), "gb_per_s": round(dw_bytes / dw_ms / 1e6, 1),
                                      "best_layer": dw_best[0], "best_gb_per_s": round(dw_best[1], 1),
                                      "bytes": dw_bytes, "how": "every depthwise step of the forward alone, "
                                      "CUDA events; bytes = fp32 input + output (fp32, or the two bf16 planes "
                                      "a linked projection reads) + weights"},
            "config1_conv_relu_fp32": {"ms": round(ms1, 5), "tflops": round(f1 / ms1 / 1e9, 1)},
            "config3_gemm_fp32": {"ms": round(ms3, 5), "tflops": round(f3 / ms3 / 1e9, 1)},
            "config3_qlinearmatmul": {"ms": round(msq, 5), "tops": round(f3 / msq / 1e9, 1)},
            "fp32_peak_note": "split-bf16: 3 bf16 products per fp32 multiply-add; peak = measured bf16 / 3"}


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.impl == "reference":
        return reference_arm(args, rank, world)
    assert args.warmup >= 3, "at least 3 warm-up steps"

    import torch
    import torch.distributed as dist
    from nnr_b200 import graph, ops, resnet50, workloads as W

    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    ops.init(local)
    dev = torch.device("cuda", local)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    model = load_model(BATCH, rank, world, barrier)
    net = graph.DeviceNetwork(model, local)
    from nnr_b200 import replicas
    x_np = resnet50.input_batch(replicas.shard_offset(rank, BATCH), BATCH)
    x_host = torch.from_numpy(x_np).pin_memory()
    out_host = torch.empty(model.shapes["logits"], dtype=torch.float32).pin_memory()
    x_host2 = torch.from_numpy(resnet50.input_batch(BATCH * (rank + world), BATCH)).pin_memory()
    out_host2 = torch.empty(model.shapes["logits"], dtype=torch.float32).pin_memory()
    net.view("input").copy_(x_host)
    stream = net.stream
    # (8-byte elements: torch's fill writes them at ~6.6 TB/s, 30 us for the
    # 192 MB, where a byte-element fill takes 54 us)
    flush = torch.empty(L2_FLUSH_BYTES // 8, dtype=torch.int64, device=dev)
    # steps that launch the tcgen05 engine (conv, conv + fused add, matmul): (step, node)
    tc_steps = [(t, st_[4]) for t, st_ in enumerate(net.steps) if st_[0] in ("QLinearConv", "QLinearMatMul", "QConvAdd", "QQConv")]
    tc_nodes = [i for _, i in tc_steps]
    n_pad_copies = sum(1 for st_ in net.steps if st_[0] == "QLinearConv" and net.ops[st_[4]] is not None
                       and any(net.ops[st_[4]].input_padding()) and st_[2][0] not in net.padded)

    net.capture()
    for _ in range(args.warmup):
        net.launch()
        net.forward(x_host, out_host)
    stream.synchronize()
    assert ops.device_status() == 0

    def timed(fn, steps):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for i in range(steps):
            with torch.cuda.stream(stream):
                flush.zero_()
            ev[i][0].record(stream)
            fn()
            ev[i][1].record(stream)
        stream.synchronize()
        return sum(a.elapsed_time(b) for a, b in ev)

    def step_times(reps=5):
        """Device time of every step of the forward: 10 launches of the step
        captured in a CUDA graph, replayed `reps` times, CUDA events on the
        network's stream (no host gaps between launches; L2 warm). Only the
        shares are used: scaled to the timed forward they give each step's
        time inside it (the whole-forward graph overlaps each kernel's
        prologue with its predecessor, so the isolated times add up to a
        little more than the forward)."""
        times = []
        for t_ in range(len(net.steps)):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for _ in range(10):
                    net.run_step(t_)
            g.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                with torch.cuda.stream(stream):
                    g.replay()
            e1.record(stream)
            stream.synchronize()
            times.append(e0.elapsed_time(e1) / (10 * reps))
        return times

    def h2d_gbs(reps=10):
        """Host-to-device bandwidth of this rank's pinned input batch (CUDA
        events on the copy stream; the e2e line is bounded by this link)."""
        buf = torch.empty_like(net.view("input"))
        cs = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(cs):
            buf.copy_(x_host, non_blocking=True)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(cs)
            for _ in range(reps):
                buf.copy_(x_host, non_blocking=True)
            e1.record(cs)
        e1.synchronize()
        return x_np.nbytes * reps / (e0.elapsed_time(e1) / 1e3) / 1e9

    with ClockSampler(local) as clk:
        t_end = time.perf_counter() + 1.5  # reach load clocks (the GPU idles near 120 MHz)
        while time.perf_counter() < t_end:
            for _ in range(10):
                net.launch()
            stream.synchronize()
        barrier()
        dev_ms = timed(net.launch, args.steps)
        barrier()
        e2e_serial_ms = timed(lambda: net.forward(x_host, out_host), args.steps)
        barrier()
        # pipelined serving loop (DeviceNetwork.forward_many): step i's H2D on a
        # copy stream overlaps step i-1's forward; every step still copies its
        # input from pinned host memory, flushes L2 and reads its logits back,
        # all inside the one timed window
        xs = [x_host, x_host2] * ((args.steps + 1) // 2)
        outs = [out_host, out_host2] * ((args.steps + 1) // 2)
        net.forward_many(xs[:2], outs[:2], between=flush.zero_)
        stream.synchronize()
        pe0, pe1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        pe0.record(stream)
        net.forward_many(xs[:args.steps], outs[:args.steps], between=flush.zero_)
        pe1.record(stream)
        stream.synchronize()
        e2e_ms = pe0.elapsed_time(pe1)
        barrier()
        stimes = step_times()
        link_gbs = h2d_gbs()
        int8_probe = int8_peak_probe(torch, dev) if rank == 0 else None
        c2 = config2_qlinearconv(ops, W, torch, dev, stream, flush) if rank == 0 else None
        rows = other_rows(ops, W, torch, dev, stream, flush) if rank == 0 else None
        plugin = nnr_plugin_e2e(model, x_np, args.steps, local, flush, torch) if rank == 0 else None
    assert ops.device_status() == 0

    dev_ms, e2e_ms, e2e_serial_ms = replicas.max_over_ranks([dev_ms, e2e_ms, e2e_serial_ms], world,
                                                            dist if world > 1 else None, dev)
    ms = dev_ms / args.steps
    value = replicas.job_rate(BATCH, world, ms)
    e2e_val = replicas.job_rate(BATCH, world, e2e_ms / args.steps)

    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    bf16 = peaks.get("bf16_tflops")
    hbm = peaks.get("hbm_gbs") or 6650.0
    if rows and "config5_depthwise_f32" in rows:
        rows["config5_depthwise_f32"]["frac_of_hbm"] = round(rows["config5_depthwise_f32"]["gb_per_s"] / hbm, 4)
    two_bf16 = 2.0 * (bf16 or 1590.0)
    # int8 peak: the larger of the live library int8 GEMM probe and twice the
    # measured bf16 burst (dense int8 runs at twice the bf16 rate on B200);
    # taking the larger keeps every fraction conservative
    probe_tops = int8_probe["tops"] if int8_probe else None
    if probe_tops and probe_tops > two_bf16:
        peak, peak_note = probe_tops, "measured int8 GEMM probe (torch._int_mm, cuBLASLt), above 2x measured bf16"
    else:
        peak = two_bf16
        peak_note = ("2x measured bf16 burst (MEASURED_PEAKS.json), above the measured int8 GEMM probe"
                     if bf16 else "2x fallback bf16 1.59 PFLOP/s")

    # per-step times inside the timed forward: isolated shares x the forward
    share_scale = ms / sum(stimes)
    in_fwd = [t_ * share_scale for t_ in stimes]
    tc_time = {i: in_fwd[t_] for t_, i in tc_steps}
    k_ms = sum(tc_time.values())
    k_ops = sum(node_ops(model, i) for i in tc_nodes)
    achieved = k_ops / (k_ms / 1e3) / 1e12
    three = [i for i in tc_nodes if model.nodes[i].op == "QLinearConv" and model.nodes[i].attrs["w"].shape[2] == 3]
    three_ms = sum(tc_time[i] for i in three)
    three_tops = sum(node_ops(model, i) for i in three) / (three_ms / 1e3) / 1e12
    # per-layer attainable time: the slower of the tensor floor and the HBM
    # floor (u8 input + s8 weights + u8 output (+ u8 residual), each once)
    att_ms = 0.0
    for t_, i in tc_steps:
        att_ms += max(node_ops(model, i) / (peak * 1e12), node_bytes(model, net, t_) / (hbm * 1e9)) * 1e3
    if c2:
        c2["kernel_frac_of_int8_peak"] = round(c2["kernel_tops"] / peak, 4)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u8",
            "data": "synthetic: seeded ResNet-50 QDQ weights (He-normal, per-channel int8) and N(0,1) images",
            "config": {"workload": WORKLOAD, "batch_per_gpu": BATCH, "global_batch": BATCH * world,
                       "image": "3x224x224 fp32 NCHW input", "graph": "one captured CUDA graph per forward",
                       "l2": "flushed between timed steps (192 MB write, 1.5x L2)",
                       "parallelism": f"dp{world} (batch-sharded replicas, no data-path collective)"},
            "e2e": {"value": round(e2e_val, 1), "unit": UNIT, "h2d_bytes_per_step": int(x_np.nbytes),
                    "d2h_bytes_per_step": int(np.prod(model.shapes["logits"]) * 4),
                    "mode": "pipelined (DeviceNetwork.forward_many): H2D of step i into staging buffer i%2 overlaps "
                            "step i-1's forward, which is the CUDA graph captured on its own staging buffer (no "
                            "device-to-device input copy); the logits go to the host from a device copy on a "
                            "third stream; one timed window over all steps, L2 flushed before each forward",
                    "serial_value": round(world * BATCH / (e2e_serial_ms / args.steps / 1e3), 1),
                    "h2d_gbs_per_rank": round(link_gbs, 1),
                    "link_bound_images_per_s": round(world * BATCH / (x_np.nbytes / (link_gbs * 1e9)), 1),
                    "serial_mode": "DeviceNetwork.forward: H2D, forward, D2H in sequence, per-step events",
                    "nnr_plugin": plugin},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TOPS",
                         "frac": round(achieved / peak, 4), "traffic": TC_TRAFFIC_BYTES,
                         "traffic_unit": "bytes per forward (DRAM read + write of all tc_gemm launches, one ncu capture)",
                         "kernel": "tc_gemm_kernel: all 53 QLinearConv (16 with the residual QLinearAdd fused) + the QLinearMatMul of one forward",
                         "kernel_ms_per_forward": round(k_ms, 4), "ops_per_forward": int(k_ops),
                         "kernel_ms_source": "timed forward x the tc steps' share of the isolated per-step times",
                         "conv3x3_tops": round(three_tops, 1), "conv3x3_frac": round(three_tops / peak, 4),
                         "conv3x3_ms_per_forward": round(three_ms, 4),
                         "attainable_ms_per_forward": round(att_ms, 4),
                         "attainable_frac": round(att_ms / k_ms, 4),
                         "attainable_note": "sum over tc layers of max(ops / int8 peak, compulsory u8 bytes / HBM)",
                         "peak_source": peak_note, "int8_probe": int8_probe, "hbm_gbs": hbm},
            "qlinearconv_config2": c2,
            "other_configs": rows,
            # steps + the stem's space-to-depth reorder + the input copies of
            # shifted-patch convs whose producer does not write them padded
            "gpu_launches": (len(net.steps) + 1 + n_pad_copies) * args.steps,
            "clocks": clk.summary(),
        }
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline(model)
            if rows is not None:
                rows["cpu_nnr"] = nnr_cpu_other_configs()
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
