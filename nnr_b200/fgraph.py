"""Device execution of an fp32 network (nnr_b200.mobilenetv2.FModel).

The fp32 counterpart of graph.DeviceNetwork: every Conv (dense convs on the
tensor cores as split-bf16, depthwise on CUDA cores, Clip fused as the
post-op), the residual Add fused into the producing 1x1 projection's
epilogue (nnrcu_conv_f32_run's residual, added after the post-op exactly as
the unfused Conv -> Add computes it), GlobalAveragePool and the FC Gemm run
through the C ABI on one stream, in node order, with all tensors and
workspaces in one planned arena; capture() records the forward into one CUDA
graph.

With split_links (the default), a depthwise Conv whose output feeds only a
1x1 projection writes that output directly as the projection's split-bf16
operand planes (nnrcu_conv_f32_run_to_planes / _run_planes), so the fp32
tensor between them is never stored and re-split; the projection's result
is bit-identical. Such a tensor has no fp32 view (plane_links lists them).
"""
from __future__ import annotations

import ctypes as C
from typing import Dict

import numpy as np

from .graph import ALIGN, Interval, check_plan, plan_arena


class FloatNetwork:
    def __init__(self, model, device: int = 0, reuse: bool = True, fuse_add: bool = True, split_links: bool = True):
        import torch
        from . import ops

        self.torch = torch
        self.model = model
        ops.init(device)
        self.dev = torch.device("cuda", device)
        self.ops, self.ws = [], []
        for nd in model.nodes:
            a = nd.attrs
            if nd.op == "Conv":
                x = nd.inputs[0]
                shp = model.shapes[x]
                lay = "NCHW" if x == "input" else "NHWC"
                logical = shp if lay == "NCHW" else (shp[0], shp[3], shp[1], shp[2])
                op = ops.Conv(logical, a["w"], a["b"], strides=(a["stride"],) * 2, pads=(a["pad"],) * 4,
                              group=a["group"], in_layout=lay, out_layout="NHWC", post=a["post"],
                              post_a=0.0, post_b=6.0)
            elif nd.op == "Gemm":
                op = ops.Gemm(model.shapes[nd.inputs[0]][0], a["b"], a["c"])
            else:
                op = None
            self.ops.append(op)
            self.ws.append(op.workspace_size() if op is not None else 0)
        self._schedule(fuse_add)
        self._link_planes(split_links)
        self._plan(reuse)
        self.stream = torch.cuda.Stream(device=self.dev)
        self.graph_exec = None

    def _schedule(self, fuse_add: bool):
        """One step per node, except that an Add whose first operand is a Conv
        output with no other consumer is done in that Conv's epilogue."""
        nodes = self.model.nodes
        consumers: Dict[str, int] = {}
        for nd in nodes:
            for x in nd.inputs:
                consumers[x] = consumers.get(x, 0) + 1
        producer = {nd.output: i for i, nd in enumerate(nodes)}
        fused = {}
        if fuse_add:
            for j, nd in enumerate(nodes):
                if nd.op == "Add":
                    i = producer.get(nd.inputs[0])
                    if i is not None and nodes[i].op == "Conv" and consumers[nd.inputs[0]] == 1:
                        fused[i] = j
        add_of = {j: i for i, j in fused.items()}
        self.steps = []  # (kind, node index, inputs, output, op node index)
        for j, nd in enumerate(nodes):
            if j in fused:
                continue
            if j in add_of:
                i = add_of[j]
                self.steps.append(("ConvAdd", j, [nodes[i].inputs[0], nd.inputs[1]], nd.output, i))
            else:
                self.steps.append((nd.op, j, list(nd.inputs), nd.output, j))
        self.fused_away = {nodes[i].output for i in fused}

    def _link_planes(self, enabled: bool):
        """plane_links[t] = cs for each depthwise output t consumed only by a
        1x1 Conv that reads pre-split planes with channel stride cs."""
        from ._lib import lib
        self.plane_links: Dict[str, int] = {}
        if not enabled:
            return
        uses: Dict[str, list] = {}
        for t, (_, _, ins, _, _) in enumerate(self.steps):
            for k, x in enumerate(ins):
                uses.setdefault(x, []).append((t, k))
        nodes = self.model.nodes
        for kind, _, _, out, i in self.steps:
            if kind != "Conv" or nodes[i].attrs["group"] == 1 or len(uses.get(out, [])) != 1:
                continue
            t, k = uses[out][0]
            ckind, _, _, _, ci = self.steps[t]
            if ckind not in ("Conv", "ConvAdd") or k != 0:
                continue
            cs = C.c_int()
            if lib.nnrcu_conv_f32_plane_stride(self.ops[ci]._op, C.byref(cs)) == 0:
                self.plane_links[out] = cs.value
                self.ws[ci] = 0  # reads the planes: no split workspace

    def _plane_bytes(self, name: str) -> int:
        n, h, w, _ = self.model.shapes[name]
        return (n * h * w * self.plane_links[name] * 2 + ALIGN - 1) // ALIGN * ALIGN

    def _nbytes(self, name: str) -> int:
        if name in self.plane_links:
            return 2 * self._plane_bytes(name)  # hi plane, then lo plane
        return int(np.prod(self.model.shapes[name])) * 4

    def _plan(self, reuse: bool):
        first: Dict[str, int] = {"input": -1}
        last: Dict[str, int] = {}
        for t, (_, _, ins, out, _) in enumerate(self.steps):
            first.setdefault(out, t)
            for x in ins:
                last[x] = t
        last["logits"] = len(self.steps)
        items = [Interval(n, self._nbytes(n), first[n], last.get(n, first[n])) for n in first]
        for t, (_, _, _, _, i) in enumerate(self.steps):
            if self.ws[i]:
                items.append(Interval(f"ws{i}", self.ws[i], t, t))
        if not reuse:
            items = [Interval(it.name, it.nbytes, -1, len(self.steps)) for it in items]
        self.offsets, self.arena_bytes = plan_arena(items)
        check_plan(items, self.offsets)
        self.arena = self.torch.empty(max(self.arena_bytes, ALIGN), dtype=self.torch.uint8, device=self.dev)
        base = self.arena.data_ptr()
        self.ptr = {k: base + v for k, v in self.offsets.items()}

    def view(self, name: str):
        if name in self.plane_links:
            raise KeyError(f"{name} is stored as split-bf16 planes (split_links=False keeps it fp32)")
        off = self.offsets[name]
        return self.arena[off:off + self._nbytes(name)].view(self.torch.float32).view(self.model.shapes[name])

    def run(self, stream=None) -> None:
        for t in range(len(self.steps)):
            self.run_step(t, stream)

    def run_step(self, t: int, stream=None) -> None:
        from ._lib import call
        st = C.c_void_p(self.stream.cuda_stream if stream is None else stream)
        P, m = self.ptr, self.model
        kind, j, ins, out, i = self.steps[t]
        ws = C.c_void_p(P[f"ws{i}"]) if self.ws[i] else None
        if kind in ("Conv", "ConvAdd"):
            res = C.c_void_p(P[ins[1]]) if kind == "ConvAdd" else None
            if out in self.plane_links:
                pb = self._plane_bytes(out)
                call("nnrcu_conv_f32_run_to_planes", self.ops[i]._op, C.c_void_p(P[ins[0]]), C.c_void_p(P[out]),
                     C.c_void_p(P[out] + pb), self.plane_links[out], st)
            elif ins[0] in self.plane_links:
                pb = self._plane_bytes(ins[0])
                call("nnrcu_conv_f32_run_planes", self.ops[i]._op, C.c_void_p(P[ins[0]]), C.c_void_p(P[ins[0]] + pb),
                     C.c_void_p(P[out]), res, st)
            else:
                call("nnrcu_conv_f32_run", self.ops[i]._op, C.c_void_p(P[ins[0]]), C.c_void_p(P[out]), res, ws, st)
        elif kind == "GlobalAveragePool":
            n, h, w, c = m.shapes[ins[0]]
            call("nnrcu_gap_f32_nhwc", C.c_void_p(P[ins[0]]), n, h * w, c, C.c_void_p(P[out]), st)
        elif kind == "Gemm":
            call("nnrcu_gemm_f32_run", self.ops[i]._op, C.c_void_p(P[ins[0]]), C.c_void_p(P[out]), ws, st)
        elif kind == "Add":
            raise ValueError("unfused Add: run with fuse_add=True")
        else:
            raise ValueError(f"unknown node {kind}")

    def capture(self) -> None:
        from ._lib import call
        self.run()
        self.stream.synchronize()
        st = C.c_void_p(self.stream.cuda_stream)
        call("nnrcu_graph_begin", st)
        try:
            self.run()
        finally:
            g = C.c_void_p()
            call("nnrcu_graph_end", st, C.byref(g))
        self.graph_exec = g

    def launch(self) -> None:
        from ._lib import call
        if self.graph_exec is not None:
            call("nnrcu_graph_launch", self.graph_exec, C.c_void_p(self.stream.cuda_stream))
        else:
            self.run()

    def forward(self, x_host, out_host=None):
        t = self.torch
        with t.cuda.stream(self.stream):
            self.view("input").copy_(x_host, non_blocking=True)
            self.launch()
            if out_host is None:
                out_host = t.empty(self.model.shapes["logits"], dtype=t.float32, pin_memory=True)
            out_host.copy_(self.view("logits"), non_blocking=True)
        return out_host

    def close(self):
        from ._lib import lib
        if self.graph_exec is not None:
            lib.nnrcu_graph_destroy(self.graph_exec)
            self.graph_exec = None
        for op in self.ops:
            if op is not None:
                op.close()
