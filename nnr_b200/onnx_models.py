"""The BASELINE models and single-operator graphs as ONNX byte streams for
nnr's own loader (context_t::load, nnr.cpp:771).

resnet50_qdq(QModel) writes config 4 the way a QDQ export does, so that
nnr's passes rebuild the operator list nnr_b200.resnet50 holds:
  * each QLinearConv as DQ(x) -> Conv(DQ(w, per-channel, axis 0),
    DQ(bias int32)) -> Q(y): fuse_qdq_compute.cpp:101-205 turns it into a
    QLinearConv (the Relu of the float network is folded into Q's zp 0);
  * MaxPool as DQ -> MaxPool -> Q with the same scale/zp: fuse_qdq.cpp
    rewires MaxPool onto the u8 tensor;
  * each residual as DQ(a), DQ(b) -> Add -> Relu -> Q: fuse_qdq_compute.cpp
    :257-343 turns it into a QLinearAdd;
  * DQ -> GlobalAveragePool -> Q, Flatten of the u8 result, then the FC as
    DQ -> MatMul(DQ(b)) -> Q (a QLinearMatMul) and DQ -> Add(bias).
mobilenetv2(FModel) writes config 5 as Conv (+ Clip(0, 6)), Add,
GlobalAveragePool, Flatten and Gemm nodes (BatchNorm already folded).
All activations are NCHW at the graph boundary, as ONNX defines them.
"""
from __future__ import annotations

import numpy as np

from . import onnx_pb as P

f32 = np.float32


def _q(g: P.Graph, x: str, y: str, scale: float, zp: int) -> str:
    return g.node("QuantizeLinear", [x, g.scalar(f32(scale)), g.scalar(np.uint8(zp))], [y])


def _dq(g: P.Graph, x: str, y: str, scale: float, zp: int) -> str:
    return g.node("DequantizeLinear", [x, g.scalar(f32(scale)), g.scalar(np.uint8(zp))], [y])


def resnet50_qdq(model) -> bytes:
    """Config 4 (nnr_b200.resnet50.QModel) as a QDQ ONNX graph: input
    "input" f32 [N,3,224,224], output "logits" f32 [N,1000]."""
    g = P.Graph("resnet50_v1_qdq")
    qp = model.qparams
    n = model.batch
    g.input("input", P.FLOAT, model.shapes["input"])
    for k, nd in enumerate(model.nodes):
        a = nd.attrs
        if nd.op == "QuantizeLinear":
            q = qp[nd.output]
            _q(g, nd.inputs[0], nd.output, q.scale, q.zp)
        elif nd.op == "QLinearConv":
            x = nd.inputs[0]
            xq, yq = qp[x], qp[nd.output]
            w, ws, bias = a["w"], a["w_scale"].astype(f32), a["bias"].astype(np.int32)
            oc = w.shape[0]
            xd = _dq(g, x, f"{nd.output}.x", xq.scale, xq.zp)
            wq = g.init(f"{nd.output}.wq", w.astype(np.int8))
            g.init(f"{nd.output}.ws", ws)
            g.init(f"{nd.output}.wzp", np.zeros(oc, np.int8))
            wd = g.node("DequantizeLinear", [wq, f"{nd.output}.ws", f"{nd.output}.wzp"], [f"{nd.output}.w"], axis=0)
            bq = g.init(f"{nd.output}.bq", bias)
            g.init(f"{nd.output}.bs", (f32(xq.scale) * ws).astype(f32))
            g.init(f"{nd.output}.bzp", np.zeros(oc, np.int32))
            bd = g.node("DequantizeLinear", [bq, f"{nd.output}.bs", f"{nd.output}.bzp"], [f"{nd.output}.b"], axis=0)
            kk, s, p = w.shape[2], a["stride"], a["pad"]
            y = g.node("Conv", [xd, wd, bd], [f"{nd.output}.f"], kernel_shape=[kk, kk], strides=[s, s],
                       pads=[p, p, p, p], dilations=[1, 1], group=1)
            _q(g, y, nd.output, yq.scale, yq.zp)
        elif nd.op == "MaxPool":
            q = qp[nd.output]
            xd = _dq(g, nd.inputs[0], f"{nd.output}.x", q.scale, q.zp)
            y = g.node("MaxPool", [xd], [f"{nd.output}.f"], kernel_shape=[a["k"]] * 2, strides=[a["s"]] * 2,
                       pads=[a["pad"]] * 4)
            _q(g, y, nd.output, q.scale, q.zp)
        elif nd.op == "QLinearAdd":
            ad, bd = (_dq(g, t, f"{nd.output}.{i}", qp[t].scale, qp[t].zp) for i, t in enumerate(nd.inputs))
            s = g.node("Add", [ad, bd], [f"{nd.output}.sum"])
            r = g.node("Relu", [s], [f"{nd.output}.relu"])
            _q(g, r, nd.output, qp[nd.output].scale, qp[nd.output].zp)
        elif nd.op == "DqGapQ":
            x = nd.inputs[0]
            xd = _dq(g, x, f"{nd.output}.x", qp[x].scale, qp[x].zp)
            m = g.node("GlobalAveragePool", [xd], [f"{nd.output}.f"])
            q4 = _q(g, m, f"{nd.output}.q4", qp[nd.output].scale, qp[nd.output].zp)
            g.node("Flatten", [q4], [nd.output], axis=1)
        elif nd.op == "QLinearMatMul":
            x = nd.inputs[0]
            xd = _dq(g, x, f"{nd.output}.x", qp[x].scale, qp[x].zp)
            bq = g.init(f"{nd.output}.bq", a["b"].astype(np.int8))
            bd = g.node("DequantizeLinear", [bq, g.scalar(f32(a["b_scale"])), g.scalar(np.int8(a["b_zp"]))],
                        [f"{nd.output}.b"])
            y = g.node("MatMul", [xd, bd], [f"{nd.output}.f"])
            _q(g, y, nd.output, qp[nd.output].scale, qp[nd.output].zp)
        elif nd.op == "DequantizeLinear":
            x = nd.inputs[0]
            xd = _dq(g, x, f"{nd.output}.x", qp[x].scale, qp[x].zp)
            b = g.init(f"{nd.output}.bias", a["bias"].astype(f32))
            g.node("Add", [xd, b], [nd.output])
        else:
            raise ValueError(nd.op)
    g.output("logits", P.FLOAT, (n, 1000))
    return g.model()


def mobilenetv2(model) -> bytes:
    """Config 5 (nnr_b200.mobilenetv2.FModel): input "input" f32
    [N,3,224,224], output "logits" f32 [N,1000]."""
    g = P.Graph("mobilenetv2")
    g.input("input", P.FLOAT, model.shapes["input"])
    lo, hi = g.scalar(f32(0.0)), g.scalar(f32(6.0))
    for nd in model.nodes:
        a = nd.attrs
        if nd.op == "Conv":
            w = g.init(f"{nd.output}.w", a["w"])
            b = g.init(f"{nd.output}.b", a["b"])
            k, s, p = a["w"].shape[2], a["stride"], a["pad"]
            out = f"{nd.output}.f" if a["post"] == "Clip" else nd.output
            g.node("Conv", [nd.inputs[0], w, b], [out], kernel_shape=[k, k], strides=[s, s], pads=[p] * 4,
                   group=a["group"])
            if a["post"] == "Clip":
                g.node("Clip", [out, lo, hi], [nd.output])
        elif nd.op == "Add":
            g.node("Add", list(nd.inputs), [nd.output])
        elif nd.op == "GlobalAveragePool":
            m = g.node("GlobalAveragePool", list(nd.inputs), [f"{nd.output}.4d"])
            g.node("Flatten", [m], [nd.output], axis=1)
        elif nd.op == "Gemm":
            b = g.init(f"{nd.output}.B", a["b"])
            c = g.init(f"{nd.output}.C", a["c"])
            g.node("Gemm", [nd.inputs[0], b, c], [nd.output], transB=0)
        else:
            raise ValueError(nd.op)
    g.output("logits", P.FLOAT, model.shapes["logits"])
    return g.model()


# ------------------------------------------------------------------ single operators
def conv(x_shape, w, b=None, strides=(1, 1), pads=(0, 0, 0, 0), dilations=(1, 1), group=1, post=None,
         post_a=0.0, post_b=0.0, residual=False) -> bytes:
    """x -> Conv [-> post-op] [-> Add(r)] -> y. post: None, "Relu", "Clip"
    (post_a, post_b), "HardSwish", "Sigmoid", "LeakyRelu" (alpha post_a),
    "Tanh"."""
    g = P.Graph("conv")
    g.input("x", P.FLOAT, x_shape)
    ins = ["x", g.init("w", np.asarray(w, f32))]
    if b is not None:
        ins.append(g.init("b", np.asarray(b, f32)))
    kh, kw = w.shape[2], w.shape[3]
    n = x_shape[0]
    oc = w.shape[0]
    oh = (x_shape[2] + pads[0] + pads[2] - dilations[0] * (kh - 1) - 1) // strides[0] + 1
    ow = (x_shape[3] + pads[1] + pads[3] - dilations[1] * (kw - 1) - 1) // strides[1] + 1
    chain = ["Conv"] + ([post] if post else []) + (["Add"] if residual else [])
    names = [f"t{i}" for i in range(len(chain) - 1)] + ["y"]  # the last node writes the graph output
    y = g.node("Conv", ins, [names[0]], kernel_shape=[kh, kw], strides=list(strides), pads=list(pads),
               dilations=list(dilations), group=group)
    i = 1
    if post == "Clip":
        y = g.node("Clip", [y, g.scalar(f32(post_a)), g.scalar(f32(post_b))], [names[i]])
    elif post == "LeakyRelu":
        y = g.node("LeakyRelu", [y], [names[i]], alpha=float(post_a))
    elif post is not None:
        y = g.node(post, [y], [names[i]])
    if residual:
        g.input("r", P.FLOAT, (n, oc, oh, ow))
        g.node("Add", [y, "r"], ["y"])
    g.output("y", P.FLOAT, (n, oc, oh, ow))
    return g.model()


def gemm(m, k, n, b, c=None, alpha=1.0, beta=1.0, trans_a=0, trans_b=0) -> bytes:
    """a -> Gemm(a, B, C) -> y, B (and C) initializers."""
    g = P.Graph("gemm")
    g.input("a", P.FLOAT, (k, m) if trans_a else (m, k))
    ins = ["a", g.init("B", np.asarray(b, f32))]
    if c is not None:
        ins.append(g.init("C", np.asarray(c, f32)))
    g.node("Gemm", ins, ["y"], alpha=float(alpha), beta=float(beta), transA=int(trans_a), transB=int(trans_b))
    g.output("y", P.FLOAT, (m, n))
    return g.model()


def matmul(a_shape, b) -> bytes:
    """a -> MatMul(a, B) -> y, B an initializer."""
    g = P.Graph("matmul")
    g.input("a", P.FLOAT, a_shape)
    g.node("MatMul", ["a", g.init("B", np.asarray(b, f32))], ["y"])
    g.output("y", P.FLOAT, tuple(a_shape[:-1]) + (b.shape[1],))
    return g.model()


def matmul_dynamic(a_shape, b_shape, y_shape, post=None, elem=None) -> bytes:
    """a, b -> MatMul(a, b) [-> Relu] -> y, both operands graph inputs (nnr's
    MatMul with a run-time B); elem: the tensor type (FLOAT by default)."""
    elem = P.FLOAT if elem is None else elem
    g = P.Graph("matmul_dyn")
    g.input("a", elem, a_shape)
    g.input("b", elem, b_shape)
    if post:
        g.node("MatMul", ["a", "b"], ["m"])
        g.node(post, ["m"], ["y"])
    else:
        g.node("MatMul", ["a", "b"], ["y"])
    g.output("y", elem, y_shape)
    return g.model()


def quantize(shape, scale, zp) -> bytes:
    g = P.Graph("q")
    g.input("x", P.FLOAT, shape)
    _q(g, "x", "y", scale, zp)
    g.output("y", P.UINT8, shape)
    return g.model()


def dequantize_add(shape, scale, zp, bias) -> bytes:
    g = P.Graph("dq")
    g.input("x", P.UINT8, shape)
    _dq(g, "x", "d", scale, zp)
    g.node("Add", ["d", g.init("bias", np.asarray(bias, f32))], ["y"])
    g.output("y", P.FLOAT, shape)
    return g.model()


def qlinearadd(shape, a_scale, a_zp, b_scale, b_zp, y_scale, y_zp, relu=True) -> bytes:
    """DQ(a), DQ(b) -> Add [-> Relu] -> Q: nnr fuses it into QLinearAdd."""
    g = P.Graph("qadd")
    g.input("a", P.UINT8, shape)
    g.input("b", P.UINT8, shape)
    _dq(g, "a", "ad", a_scale, a_zp)
    _dq(g, "b", "bd", b_scale, b_zp)
    s = g.node("Add", ["ad", "bd"], ["s"])
    if relu:
        s = g.node("Relu", [s], ["r"])
    _q(g, s, "y", y_scale, y_zp)
    g.output("y", P.UINT8, shape)
    return g.model()


def maxpool_u8(shape, scale, zp, k=3, s=2, pad=1) -> bytes:
    """DQ -> MaxPool -> Q (same scale/zp): nnr runs MaxPool on the u8 tensor."""
    g = P.Graph("maxpool")
    g.input("x", P.UINT8, shape)
    _dq(g, "x", "d", scale, zp)
    g.node("MaxPool", ["d"], ["m"], kernel_shape=[k, k], strides=[s, s], pads=[pad] * 4)
    _q(g, "m", "y", scale, zp)
    n, c, h, w = shape
    g.output("y", P.UINT8, (n, c, (h + 2 * pad - k) // s + 1, (w + 2 * pad - k) // s + 1))
    return g.model()


def dq_gap_q(shape, x_scale, x_zp, y_scale, y_zp) -> bytes:
    g = P.Graph("gap")
    g.input("x", P.UINT8, shape)
    _dq(g, "x", "d", x_scale, x_zp)
    g.node("GlobalAveragePool", ["d"], ["m"])
    _q(g, "m", "y", y_scale, y_zp)
    g.output("y", P.UINT8, (shape[0], shape[1], 1, 1))
    return g.model()


def gap_f32(shape) -> bytes:
    g = P.Graph("gapf")
    g.input("x", P.FLOAT, shape)
    g.node("GlobalAveragePool", ["x"], ["y"])
    g.output("y", P.FLOAT, (shape[0], shape[1], 1, 1))
    return g.model()


def conv_half(x_shape, w_bits, b_bits, elem_type, strides=(1, 1), pads=(0, 0, 0, 0), post=None) -> bytes:
    """x -> Conv [-> Relu] -> y on 16-bit tensors (elem_type FLOAT16 or
    BFLOAT16; weights and bias given as uint16 bit patterns)."""
    g = P.Graph("conv16")
    g.input("x", elem_type, x_shape)
    ins = ["x", g.init("w", np.asarray(w_bits, np.uint16), elem_type)]
    if b_bits is not None:
        ins.append(g.init("b", np.asarray(b_bits, np.uint16), elem_type))
    kh, kw = w_bits.shape[2], w_bits.shape[3]
    n, oc = x_shape[0], w_bits.shape[0]
    oh = (x_shape[2] + pads[0] + pads[2] - kh) // strides[0] + 1
    ow = (x_shape[3] + pads[1] + pads[3] - kw) // strides[1] + 1
    y = g.node("Conv", ins, ["t" if post else "y"], kernel_shape=[kh, kw], strides=list(strides), pads=list(pads))
    if post:
        g.node(post, [y], ["y"])
    g.output("y", elem_type, (n, oc, oh, ow))
    return g.model()


def gemm_half(m, k, n, b_bits, c_bits, elem_type, beta=1.0, trans_b=0) -> bytes:
    g = P.Graph("gemm16")
    g.input("a", elem_type, (m, k))
    ins = ["a", g.init("B", np.asarray(b_bits, np.uint16), elem_type)]
    if c_bits is not None:
        ins.append(g.init("C", np.asarray(c_bits, np.uint16), elem_type))
    g.node("Gemm", ins, ["y"], beta=float(beta), transB=int(trans_b))
    g.output("y", elem_type, (m, n))
    return g.model()
