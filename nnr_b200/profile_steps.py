"""Per-step timing of the ResNet-50 QDQ forward on one GPU.

    python -m nnr_b200.profile_steps [--batch 32] [--json out.json]
        times every step of the forward: each step is captured 10x into its
        own CUDA graph and replayed (back to back, L2 warm), CUDA events on the
        network's stream; prints per-kind totals and the slowest steps.

    python -m nnr_b200.profile_steps --only b0.out --repeat 3
        launches only the step producing tensor b0.out, 3 times (a target
        for an ncu capture: -k regex:tc_gemm -s 1 -c 1).

    python -m nnr_b200.profile_steps --forward 3
        replays the captured whole-network graph 3 times and nothing else
        (a target for an ncu launch list of one forward: skip the first 58
        launches, capture the next 58).

    python -m nnr_b200.profile_steps --op gemm_f32 --repeat 3
        launches one BASELINE operator alone (after one untimed launch):
        gemm_f32 / qmatmul (config 3), conv_f32 (config 1), gemm_bf16 (the
        config-3 shape on bf16 tensors), qdw (an int8 depthwise QLinearConv
        over 32 x 56 x 56 x 144); prints its CUDA-event time per launch.
"""
from __future__ import annotations

import argparse
import json
import sys


def step_ops(model, node_index: int) -> int:
    nd = model.nodes[node_index]
    if nd.op == "Conv":
        w = nd.attrs["w"]
        n, oh, ow, oc = model.shapes[nd.output]
        return 2 * n * oh * ow * oc * w.shape[1] * w.shape[2] * w.shape[3]
    if nd.op == "Gemm":
        b = nd.attrs["b"]
        return 2 * model.shapes[nd.output][0] * b.shape[0] * b.shape[1]
    if nd.op == "QLinearConv":
        n, oh, ow, oc = model.shapes[nd.output]
        w = nd.attrs["w"]
        return 2 * n * oh * ow * oc * w.shape[1] * w.shape[2] * w.shape[3]
    if nd.op == "QLinearMatMul":
        b = nd.attrs["b"]
        return 2 * model.shapes[nd.output][0] * b.shape[0] * b.shape[1]
    return 0


def op_target(name: str, repeat: int) -> int:
    """Launches one operator `repeat` times (plus one untimed launch first)
    with inputs resident on cuda:0 and reports its time per launch."""
    import numpy as np
    import torch
    from . import ops, workloads as W
    ops.init(0)
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(0)
    if name in ("gemm_f32", "qmatmul", "gemm_bf16"):
        c3 = W.config3_matmul()
        if name == "gemm_f32":
            op, x = ops.Gemm(4096, c3.b_f32, c3.c_f32), torch.from_numpy(c3.a_f32).to(dev)
        elif name == "qmatmul":
            op = ops.QLinearMatMul(4096, c3.b_s8, c3.a_scale, c3.a_zp, c3.b_scale, c3.b_zp, c3.y_scale, c3.y_zp)
            x = torch.from_numpy(c3.a_u8).to(dev)
        else:
            op = ops.GemmHalf(4096, torch.from_numpy(c3.b_f32).to(torch.bfloat16), torch.from_numpy(c3.c_f32).to(
                torch.bfloat16), dtype=ops.DT_BF16)
            x = torch.from_numpy(c3.a_f32).to(dev).to(torch.bfloat16)
        flops = 2 * 4096 * 768 * 3072
    elif name == "conv_f32":
        c1 = W.config1_conv_relu()
        op = ops.Conv(c1.x.shape, c1.w, c1.bias, pads=c1.pads, post="Relu")
        x = torch.from_numpy(c1.x).to(dev)
        flops = 2 * 64 * 56 * 56 * 64 * 9
    else:
        n, h, w, c = 32, 56, 56, 144
        wt = rng.integers(-127, 128, (c, 1, 3, 3)).astype(np.int8)
        op = ops.QLinearConv((n, c, h, w), wt, np.full(c, 0.005, np.float32), None, None, 0.02, 128, 0.4, 128,
                             pads=(1, 1, 1, 1), group=c, in_layout="NHWC", out_layout="NHWC")
        x = torch.from_numpy(rng.integers(0, 256, (n, h, w, c)).astype(np.uint8)).to(dev)
        flops = 2 * n * h * w * c * 9
    op.exec(x)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(repeat):
        op.exec(x)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / repeat
    print(json.dumps({"op": name, "us_per_launch": round(us, 2), "tops": round(flops / us / 1e6, 1),
                      "status": ops.device_status()}))
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="resnet50", choices=["resnet50", "mobilenetv2"])
    ap.add_argument("--batch", type=int, default=None, help="default: 32 (resnet50), 128 (mobilenetv2)")
    ap.add_argument("--only", default=None, help="output tensor of the one step to launch")
    ap.add_argument("--repeat", type=int, default=3)
    ap.add_argument("--json", default=None)
    ap.add_argument("--forward", type=int, default=0, help="replay the whole forward graph this many times")
    ap.add_argument("--op", default=None, choices=["gemm_f32", "qmatmul", "conv_f32", "gemm_bf16", "qdw"])
    a = ap.parse_args(argv)

    import torch
    from . import graph, resnet50
    if a.op:
        return op_target(a.op, a.repeat)

    if a.model == "resnet50":
        a.batch = a.batch or 32
        m = resnet50.build(batch=a.batch)
        net = graph.DeviceNetwork(m, 0)
        net.view("input").copy_(torch.from_numpy(resnet50.input_batch(0, a.batch)))
    else:
        from . import fgraph, mobilenetv2
        a.batch = a.batch or 128
        m = mobilenetv2.build(batch=a.batch)
        net = fgraph.FloatNetwork(m, 0)
        net.view("input").copy_(torch.from_numpy(mobilenetv2.input_batch(0, a.batch)))
    st = net.stream
    if a.forward:
        net.capture()
        for _ in range(a.forward):
            net.launch()
        torch.cuda.synchronize()
        print(f"replayed the forward graph x{a.forward} ({len(net.steps)} steps)")
        return 0
    if a.only:
        t = [k for k, s in enumerate(net.steps) if s[3] == a.only][0]
        for _ in range(a.repeat):
            net.run_step(t)
        torch.cuda.synchronize()
        print(f"launched step {t} ({net.steps[t][0]} -> {a.only}) x{a.repeat}")
        return 0

    net.run()
    torch.cuda.synchronize()
    rows = []
    for t, (kind, _, _, out, i) in enumerate(net.steps):
        g = torch.cuda.CUDAGraph()
        for _ in range(2):
            net.run_step(t)
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=st):
            for _ in range(10):
                net.run_step(t)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(5):
            with torch.cuda.stream(st):
                g.replay()
        e1.record(st)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / 50
        nd = m.nodes[i]
        ops = step_ops(m, i)
        k = nd.attrs["w"].shape[2] if nd.op in ("QLinearConv", "Conv") else None
        dw = nd.op == "Conv" and nd.attrs["group"] > 1
        label = kind + (f" {k}x{k}" if k else "") + (" dw" if dw else "")
        rows.append(dict(step=t, kind=label, output=out, us=round(us, 2),
                         tops=round(ops / us / 1e6, 1) if ops else None))
    total = sum(r["us"] for r in rows)
    by = {}
    for r in rows:
        c = by.setdefault(r["kind"], [0, 0.0])
        c[0] += 1
        c[1] += r["us"]
    summary = {k: {"steps": v[0], "us": round(v[1], 1), "share": round(v[1] / total, 3)} for k, v in by.items()}
    print(json.dumps({"batch": a.batch, "total_us": round(total, 1), "steps": len(rows)}))
    print(json.dumps(summary, indent=1))
    for r in sorted(rows, key=lambda r: -r["us"])[:15]:
        print(json.dumps(r))
    if a.json:
        with open(a.json, "w") as f:
            json.dump({"total_us": total, "by_kind": summary, "steps": rows}, f, indent=1)
    return 0


if __name__ == "__main__":
    sys.exit(main())
