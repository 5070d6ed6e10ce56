"""Device execution of a quantised network through libnnrcu.so.

This is the device side of nnr's context run loop for a graph whose nodes
all live on the device:
  * plan_arena() is the device arena of nnr's memory planner
    (memory_planner.cpp:33-337): tensor lifetimes (producer step .. last
    consumer step) packed into one device allocation, best fit by size,
    operator workspaces included as one-step lifetimes;
  * DeviceNetwork.run() enqueues every node on one stream, in order
    (nnr.cpp:908-1051's exec_steps loop);
  * DeviceNetwork.capture() records that sequence once into a CUDA graph
    (nnrcu_graph_begin/_end) that later runs replay with one launch.
All compute goes through the C ABI; torch only provides the arena buffer,
streams and host staging.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

ALIGN = 256


@dataclass
class Interval:
    name: str
    nbytes: int
    first: int      # first step that writes or reads it
    last: int       # last step that reads it


def plan_arena(items: Sequence[Interval]) -> Tuple[Dict[str, int], int]:
    """Assigns byte offsets so that tensors whose lifetimes overlap never
    share bytes. Largest first, each at the lowest offset that fits between
    the already-placed intervals it overlaps in time. Returns (offsets, size)."""
    placed: List[Tuple[int, int, Interval]] = []  # (offset, end, item)
    offsets: Dict[str, int] = {}
    for it in sorted(items, key=lambda i: (-i.nbytes, i.first, i.name)):
        size = (it.nbytes + ALIGN - 1) // ALIGN * ALIGN
        busy = sorted((o, e) for o, e, other in placed if not (other.last < it.first or it.last < other.first))
        off = 0
        for o, e in busy:
            if off + size <= o:
                break
            off = max(off, e)
        placed.append((off, off + size, it))
        offsets[it.name] = off
    total = max((e for _, e, _ in placed), default=0)
    return offsets, total


def check_plan(items: Sequence[Interval], offsets: Dict[str, int]) -> None:
    """Raises if two time-overlapping intervals share bytes (planner self-check)."""
    lst = list(items)
    for i, a in enumerate(lst):
        for b in lst[i + 1:]:
            if a.last < b.first or b.last < a.first:
                continue
            a0, a1 = offsets[a.name], offsets[a.name] + a.nbytes
            b0, b1 = offsets[b.name], offsets[b.name] + b.nbytes
            if a0 < b1 and b0 < a1:
                raise AssertionError(f"arena overlap: {a.name} and {b.name}")


class DeviceNetwork:
    """A nnr_b200.resnet50.QModel prepared on one device."""

    def __init__(self, model, device: int = 0, reuse: bool = True, fuse_add: bool = True):
        import torch
        from . import ops
        from ._lib import ConvDesc, call  # noqa: F401

        self.torch = torch
        self.model = model
        self.device = device
        ops.init(device)
        self.dev = torch.device("cuda", device)
        self.ops = []      # per node: prepared operator or None
        self.ws = []       # per node: workspace bytes
        qp = model.qparams
        for nd in model.nodes:
            a = nd.attrs
            if nd.op == "QLinearConv":
                x = nd.inputs[0]
                shp = model.shapes[x]
                lay = a["in_layout"]
                logical = shp if lay == "NCHW" else (shp[0], shp[3], shp[1], shp[2])
                xq, yq = qp[x], qp[nd.output]
                op = ops.QLinearConv(logical, a["w"], a["w_scale"], None, a["bias"], xq.scale, xq.zp, yq.scale, yq.zp,
                                     strides=(a["stride"],) * 2, pads=(a["pad"],) * 4, in_layout=lay,
                                     out_layout="NHWC", requant=a["requant"])
                self.ops.append(op)
                self.ws.append(op.workspace_size())
            elif nd.op == "QLinearMatMul":
                xq, yq = qp[nd.inputs[0]], qp[nd.output]
                op = ops.QLinearMatMul(model.shapes[nd.inputs[0]][0], a["b"], xq.scale, xq.zp, a["b_scale"],
                                       a["b_zp"], yq.scale, yq.zp)
                self.ops.append(op)
                self.ws.append(op.workspace_size())
            else:
                self.ops.append(None)
                self.ws.append(0)
        self.bias = {}
        for i, nd in enumerate(model.nodes):
            if nd.op == "DequantizeLinear" and nd.attrs.get("bias") is not None:
                self.bias[i] = torch.from_numpy(np.ascontiguousarray(nd.attrs["bias"], np.float32)).to(self.dev)
        self._schedule(fuse_add)
        self._link_padded()
        self._plan(reuse)
        self.stream = torch.cuda.Stream(device=self.dev)
        self.graph_exec = None

    # ------------------------------------------------------------------ schedule
    def _schedule(self, fuse_add: bool):
        """Steps to run: one per node, except that a QLinearAdd whose first
        operand is produced by a QLinearConv with no other consumer becomes one
        fused step (nnrcu_qlinearconv_run_add) at the add's position (its
        residual may come from a later node, e.g. the downsample conv)."""
        nodes = self.model.nodes
        consumers: Dict[str, int] = {}
        for nd in nodes:
            for x in nd.inputs:
                consumers[x] = consumers.get(x, 0) + 1
        producer = {nd.output: i for i, nd in enumerate(nodes)}
        fused_conv = {}
        if fuse_add:
            for j, nd in enumerate(nodes):
                if nd.op != "QLinearAdd":
                    continue
                a = nd.inputs[0]
                i = producer.get(a)
                if i is not None and nodes[i].op == "QLinearConv" and consumers.get(a, 0) == 1:
                    fused_conv[i] = j
        # QuantizeLinear whose only consumer is a space-to-depth QLinearConv
        # (the stem): quantised inside the conv's input reorder
        # (nnrcu_qlinearconv_run_quantize); the u8 image is never materialised
        fused_q = {}
        if fuse_add:
            for j, nd in enumerate(nodes):
                if nd.op != "QuantizeLinear" or consumers.get(nd.output, 0) != 1:
                    continue
                for i, c in enumerate(nodes):
                    if c.op == "QLinearConv" and c.inputs[0] == nd.output and self.ops[i] is not None \
                            and self.ops[i].space_to_depth:
                        fused_q[i] = j
        self.steps = []  # (kind, node index, inputs, output, conv node index)
        folded = set(fused_conv) | set(fused_q.values())
        add_of = {j: i for i, j in fused_conv.items()}
        for j, nd in enumerate(nodes):
            if j in folded:
                continue
            if j in add_of:
                i = add_of[j]
                self.steps.append(("QConvAdd", j, [nodes[i].inputs[0], nd.inputs[1]], nd.output, i))
            elif j in fused_q:
                q = nodes[fused_q[j]]
                self.steps.append(("QQConv", fused_q[j], [q.inputs[0]], nd.output, j))
            else:
                self.steps.append((nd.op, j, list(nd.inputs), nd.output, j))
        self.fused_away = {nodes[i].output for i in fused_conv} | {nodes[j].output for j in fused_q.values()}

    def _link_padded(self):
        """A conv that reads an x_zp-bordered copy of its input (reported by
        input_padding) gets that layout straight from its producer conv when
        it is the tensor's only consumer: the producer writes the interior of
        a dedicated padded buffer whose border is filled once here with the
        tensor's zero point, and the consumer skips its copy."""
        t = self.torch
        nodes, qp = self.model.nodes, self.model.qparams
        consumers: Dict[str, int] = {}
        for nd in nodes:
            for x in nd.inputs:
                consumers[x] = consumers.get(x, 0) + 1
        plain_conv = {out: i for kind, _, _, out, i in self.steps if kind == "QLinearConv"}
        self.padded = {}  # tensor name -> (pads, padded device buffer)
        for kind, _, ins, _, j in self.steps:
            if kind != "QLinearConv" or self.ops[j] is None:
                continue
            x = ins[0]
            pads = self.ops[j].input_padding()
            i = plain_conv.get(x)
            if not any(pads) or i is None or consumers.get(x, 0) != 1:
                continue
            n, h, w, c = self.model.shapes[x]
            buf = t.full((n, h + pads[0] + pads[2], w + pads[1] + pads[3], c), qp[x].zp, dtype=t.uint8,
                         device=self.dev)
            self.ops[i].set_padded_io(out_pads=pads)
            self.ops[j].set_padded_io(in_padded=True)
            self.ws[j] = 0
            self.padded[x] = (pads, buf)

    # ------------------------------------------------------------------ memory
    def _nbytes(self, name: str) -> int:
        elem = 4 if name in ("input", "logits") else 1
        return int(np.prod(self.model.shapes[name])) * elem

    def _plan(self, reuse: bool = True):
        steps = self.steps
        first: Dict[str, int] = {"input": -1}
        last: Dict[str, int] = {}
        for t, (_, _, ins, out, _) in enumerate(steps):
            first.setdefault(out, t)
            for x in ins:
                last[x] = t
        last["logits"] = len(steps)  # graph output lives to the end
        items = [Interval(name, self._nbytes(name), first[name], last.get(name, first[name])) for name in first
                 if name not in self.padded]
        for t, (_, _, _, _, ci) in enumerate(steps):
            if self.ws[ci]:
                items.append(Interval(f"ws{ci}", self.ws[ci], t, t))
        if not reuse:  # every tensor keeps its own slot (for inspecting intermediates)
            items = [Interval(it.name, it.nbytes, -1, len(steps)) for it in items]
        self.offsets, self.arena_bytes = plan_arena(items)
        check_plan(items, self.offsets)
        self.intervals = items
        self.arena = self.torch.empty(max(self.arena_bytes, ALIGN), dtype=self.torch.uint8, device=self.dev)
        base = self.arena.data_ptr()
        self.ptr = {k: base + v for k, v in self.offsets.items()}
        for name, (_, buf) in self.padded.items():
            self.ptr[name] = buf.data_ptr()

    def view(self, name: str):
        """A torch view of a tensor's arena slot (for inputs and inspection)."""
        t = self.torch
        shape = self.model.shapes[name]
        dtype = t.float32 if name in ("input", "logits") else t.uint8
        if name in self.padded:
            (pt, pl, _, _), buf = self.padded[name]
            return buf[:, pt:pt + shape[1], pl:pl + shape[2], :]
        off = self.offsets[name]
        return self.arena[off:off + self._nbytes(name)].view(dtype).view(shape)

    # ------------------------------------------------------------------ execution
    def run(self, stream=None) -> None:
        """Enqueues every step on the stream (no synchronisation)."""
        for t in range(len(self.steps)):
            self.run_step(t, stream)

    def run_step(self, t: int, stream=None) -> None:
        """Enqueues step t alone (same operators, same arena slots)."""
        from ._lib import LAYOUT_NCHW, call
        st = C.c_void_p(self.stream.cuda_stream if stream is None else stream)
        qp, m, P = self.model.qparams, self.model, self.ptr
        kind, j, ins, output, i = self.steps[t]
        nd = m.nodes[i]
        a = nd.attrs
        out = C.c_void_p(P[output])
        if kind == "QConvAdd":
            add = m.nodes[j]
            qb, qy = qp[add.inputs[1]], qp[add.output]
            ws = C.c_void_p(P[f"ws{i}"]) if self.ws[i] else None
            call("nnrcu_qlinearconv_run_add", self.ops[i]._op, C.c_void_p(P[ins[0]]), C.c_void_p(P[ins[1]]),
                 qb.scale, qb.zp, qy.scale, qy.zp, out, ws, st)
        elif kind == "QQConv":
            qn = m.nodes[j]
            q = qp[qn.output]
            ws = C.c_void_p(P[f"ws{i}"]) if self.ws[i] else None
            call("nnrcu_qlinearconv_run_quantize", self.ops[i]._op, C.c_void_p(P[ins[0]]), q.scale, q.zp, out, ws, st)
        elif nd.op == "QuantizeLinear":
            n, c, h, w = m.shapes[nd.inputs[0]]
            q = qp[nd.output]
            call("nnrcu_quantize_linear_u8", C.c_void_p(P[nd.inputs[0]]), out, n, c, h, w, q.scale, q.zp,
                 LAYOUT_NCHW, 0, st)
        elif nd.op in ("QLinearConv", "QLinearMatMul"):
            ws = C.c_void_p(P[f"ws{i}"]) if self.ws[i] else None
            fn = "nnrcu_qlinearconv_run" if nd.op == "QLinearConv" else "nnrcu_qlinearmatmul_run"
            call(fn, self.ops[i]._op, C.c_void_p(P[nd.inputs[0]]), out, ws, st)
        elif nd.op == "MaxPool":
            n, h, w, c = m.shapes[nd.inputs[0]]
            k, s_, p = a["k"], a["s"], a["pad"]
            call("nnrcu_maxpool_u8_nhwc", C.c_void_p(P[nd.inputs[0]]), out, n, h, w, c, k, k, s_, s_, p, p, p, p, st)
        elif nd.op == "QLinearAdd":
            qa, qb, qy = qp[nd.inputs[0]], qp[nd.inputs[1]], qp[nd.output]
            call("nnrcu_qlinearadd_u8", C.c_void_p(P[nd.inputs[0]]), qa.scale, qa.zp, C.c_void_p(P[nd.inputs[1]]),
                 qb.scale, qb.zp, qy.scale, qy.zp, out, int(np.prod(m.shapes[nd.output])), st)
        elif nd.op == "DqGapQ":
            n, h, w, c = m.shapes[nd.inputs[0]]
            qx, qy = qp[nd.inputs[0]], qp[nd.output]
            call("nnrcu_dq_gap_q_u8_nhwc", C.c_void_p(P[nd.inputs[0]]), n, h * w, c, qx.scale, qx.zp, qy.scale,
                 qy.zp, out, st)
        elif nd.op == "DequantizeLinear":
            rows, cols = m.shapes[nd.inputs[0]]
            qx = qp[nd.inputs[0]]
            b = C.c_void_p(self.bias[i].data_ptr()) if i in self.bias else None
            call("nnrcu_dequantize_linear_u8", C.c_void_p(P[nd.inputs[0]]), qx.scale, qx.zp, b, rows, cols, out, st)
        else:
            raise ValueError(f"unknown node {nd.op}")

    def capture(self) -> None:
        """Records run() once into a CUDA graph (nnrcu_graph_begin/_end)."""
        from ._lib import call
        self.run()           # first launches outside capture (module load, attribute set-up)
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
        """One forward pass: the captured graph if any, else the node loop."""
        from ._lib import call
        if self.graph_exec is not None:
            call("nnrcu_graph_launch", self.graph_exec, C.c_void_p(self.stream.cuda_stream))
        else:
            self.run()

    def forward(self, x_host, out_host=None):
        """Host fp32 NCHW input -> host fp32 logits: H2D, one forward, D2H."""
        t = self.torch
        xin = self.view("input")
        with t.cuda.stream(self.stream):
            xin.copy_(x_host, non_blocking=True)
            self.launch()
            if out_host is None:
                out_host = t.empty(self.model.shapes["logits"], dtype=t.float32, pin_memory=True)
            out_host.copy_(self.view("logits"), non_blocking=True)
        return out_host

    def _capture_staged(self):
        """Two extra CUDA graphs of the forward, each reading its fp32 input
        from its own staging buffer outside the arena (the arena's input slot
        may be reused by later steps while the next batch is being copied in).
        forward_many alternates between them, so no device-to-device copy of
        the input is needed."""
        from ._lib import call
        t = self.torch
        xin = self.view("input")
        self._stage = [t.empty_like(xin), t.empty_like(xin)]
        self._stage_graphs = []
        own = self.ptr["input"]
        st = C.c_void_p(self.stream.cuda_stream)
        try:
            for buf in self._stage:
                self.ptr["input"] = buf.data_ptr()
                call("nnrcu_graph_begin", st)
                try:
                    self.run()
                finally:
                    g = C.c_void_p()
                    call("nnrcu_graph_end", st, C.byref(g))
                self._stage_graphs.append(g)
        finally:
            self.ptr["input"] = own
        self._copy_stream = t.cuda.Stream(device=self.dev)
        self._staged = [t.cuda.Event(), t.cuda.Event()]
        self._consumed = [t.cuda.Event(), t.cuda.Event()]
        self._d2h_stream = t.cuda.Stream(device=self.dev)
        logits = self.view("logits")
        self._logits = [t.empty_like(logits), t.empty_like(logits)]
        self._kept = [t.cuda.Event(), t.cuda.Event()]
        self._read = [t.cuda.Event(), t.cuda.Event()]

    def forward_many(self, x_hosts, out_hosts, between=None):
        """Pipelined forwards over a sequence of host batches: batch i's
        host-to-device copy runs on a second stream into staging buffer i % 2
        while batch i-1 is computed; forward i is the CUDA graph captured on
        that staging buffer; its logits are copied to one of two device
        buffers and from there to out_hosts[i] on a third stream.
        `between` (optional) is enqueued on the network's stream before each
        forward. Returns after enqueueing, with self.stream ordered after the
        last host copy; the caller synchronises self.stream."""
        from ._lib import call
        t = self.torch
        if not hasattr(self, "_stage_graphs"):
            self.run()  # module load and attribute set-up happen outside capture
            self.stream.synchronize()
            self._capture_staged()
        logits = self.view("logits")
        cs, ds = self._copy_stream, self._d2h_stream
        cs.wait_stream(self.stream)  # (work already enqueued on the network's stream comes first)
        for i, (xh, oh) in enumerate(zip(x_hosts, out_hosts)):
            k = i & 1
            with t.cuda.stream(cs):
                if i >= 2:
                    cs.wait_event(self._consumed[k])   # forward i - 2 has finished with this buffer
                self._stage[k].copy_(xh, non_blocking=True)
                self._staged[k].record(cs)
            with t.cuda.stream(self.stream):
                self.stream.wait_event(self._staged[k])
                if between is not None:
                    between()
                call("nnrcu_graph_launch", self._stage_graphs[k], C.c_void_p(self.stream.cuda_stream))
                self._consumed[k].record(self.stream)
                # the logits leave through a device copy of their own, so that
                # the next forward does not queue behind the device-to-host copy
                if i >= 2:
                    self.stream.wait_event(self._read[k])  # logits i - 2 have reached the host
                self._logits[k].copy_(logits, non_blocking=True)
                self._kept[k].record(self.stream)
            with t.cuda.stream(ds):
                ds.wait_event(self._kept[k])
                oh.copy_(self._logits[k], non_blocking=True)
                self._read[k].record(ds)
        self.stream.wait_stream(ds)
        return out_hosts

    def close(self):
        from ._lib import lib
        if self.graph_exec is not None:
            lib.nnrcu_graph_destroy(self.graph_exec)
            self.graph_exec = None
        for g in getattr(self, "_stage_graphs", []):
            lib.nnrcu_graph_destroy(g)
        self._stage_graphs = []
        for op in self.ops:
            if op is not None:
                op.close()
