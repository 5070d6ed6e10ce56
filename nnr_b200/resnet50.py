"""ResNet-50 v1 QDQ int8 model, built from a seed.

The reference measures an int8 ResNet-50 QDQ graph that nnr's ONNX loader
turns into QLinear operators (graph_optimizer/fuse_qdq_compute.cpp). No model
file ships with it, so this module builds the same network synthetically and
returns it as the operator list nnr's fusion produces:

  QuantizeLinear(input, NCHW)
  QLinearConv 7x7/2 stem (3 -> 64, R3: nnr's first-layer path), out NHWC
  MaxPool 3x3/2 on u8 (quant-capable, fuse_qdq.cpp:96-100)
  16 bottlenecks [3,4,6,3] x (64,128,256,512), expansion 4, v1 (stride on the
    first 1x1): QLinearConv 1x1 / 3x3 / 1x1 (R2, nnr's NHWC packed path),
    a 1x1 downsample conv on the first block of each stage, and QLinearAdd
    for the residual (its Relu folded into the output quantiser, zp 0)
  DequantizeLinear -> GlobalAveragePool -> QuantizeLinear
  QLinearMatMul FC 2048 -> 1000 (R4), then DequantizeLinear + Add(bias)

Weights: He-normal N(0, sqrt(2/fan_in)), biases N(0, 0.01) (BN folded),
quantised per output channel, symmetric int8 (scale = max|w|/127, w_zp 0),
bias int32 = rint(b / (x_scale * w_scale)). Activations: u8, scales
calibrated as min/max over a seeded N(0,1) calibration batch run through the
float network (fp64 on the CPU); Relu outputs get zp 0. Scales are rounded to
float16-representable values so the model does not depend on the last bits
of the calibration arithmetic of the machine that builds it.

Generator: numpy.random.default_rng(seed): weights and biases in network
order, then the calibration batch; the benchmark input comes from
default_rng([seed, 1]) so that any slice of the 256-image batch can be drawn.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

STAGES = [(3, 64, 1), (4, 128, 2), (6, 256, 2), (3, 512, 2)]


@dataclass
class QParam:
    scale: float
    zp: int


@dataclass
class Node:
    op: str
    inputs: list
    output: str
    attrs: dict = field(default_factory=dict)


@dataclass
class QModel:
    nodes: list
    shapes: dict          # tensor name -> shape as laid out (NCHW for the input, NHWC after the stem)
    qparams: dict         # tensor name -> QParam
    batch: int

    def num_ops(self) -> int:
        total = 0
        for nd in self.nodes:
            if nd.op == "QLinearConv":
                n, oh, ow, oc = self.shapes[nd.output]
                w = nd.attrs["w"]
                total += 2 * n * oh * ow * oc * w.shape[1] * w.shape[2] * w.shape[3]
            elif nd.op == "QLinearMatMul":
                b = nd.attrs["b"]
                total += 2 * self.shapes[nd.output][0] * b.shape[0] * b.shape[1]
        return total


def _snap(scale: float) -> float:
    return float(np.float32(np.float16(scale))) if scale > 6e-5 else float(np.float32(scale))


def _asym(lo: float, hi: float) -> QParam:
    lo, hi = min(lo, 0.0), max(hi, 0.0)
    scale = _snap((hi - lo) / 255.0 if hi > lo else 1.0)
    zp = int(np.clip(np.rint(-lo / scale), 0, 255))
    return QParam(scale, zp)


def _relu_q(hi: float) -> QParam:
    return QParam(_snap(hi / 255.0 if hi > 0 else 1.0), 0)


def _quant_w(w: np.ndarray):
    oc = w.shape[0]
    amax = np.abs(w.reshape(oc, -1)).max(axis=1)
    scale = np.where(amax > 0, amax / 127.0, 1.0).astype(np.float32)
    q = np.clip(np.rint(w / scale.reshape((oc,) + (1,) * (w.ndim - 1))), -127, 127).astype(np.int8)
    return q, scale


def _float_params(rng: np.random.Generator):
    """He-normal conv/FC weights and small biases, in network order."""
    convs = []

    def conv(cin, cout, k):
        w = rng.normal(0.0, math.sqrt(2.0 / (cin * k * k)), size=(cout, cin, k, k))
        b = rng.normal(0.0, 0.01, size=cout)
        convs.append((w, b))
        return len(convs) - 1

    stem = conv(3, 64, 7)
    blocks = []
    cin = 64
    for nblk, width, stride in STAGES:
        for i in range(nblk):
            s = stride if i == 0 else 1
            c1 = conv(cin, width, 1)
            c2 = conv(width, width, 3)
            c3 = conv(width, width * 4, 1)
            ds = conv(cin, width * 4, 1) if i == 0 else None
            blocks.append((c1, c2, c3, ds, s))
            cin = width * 4
    fc_w = rng.normal(0.0, math.sqrt(2.0 / 2048), size=(2048, 1000))
    fc_b = rng.normal(0.0, 0.01, size=1000)
    return convs, stem, blocks, fc_w, fc_b


def _calibrate(convs, stem, blocks, fc_w, fc_b, xcal: np.ndarray):
    """Float fp64 forward; returns (min, max) of every quantised activation."""
    import torch
    import torch.nn.functional as F

    def t(a):
        return torch.from_numpy(np.asarray(a, np.float64))

    rng_ = {}
    x = t(xcal)
    rng_["input"] = (float(x.min()), float(x.max()))

    def cv(x, idx, s, p):
        w, b = convs[idx]
        return F.conv2d(x, t(w), t(b), stride=s, padding=p)

    y = F.relu(cv(x, stem, 2, 3))
    rng_["stem"] = (0.0, float(y.max()))
    y = F.max_pool2d(y, 3, 2, 1)
    for bi, (c1, c2, c3, ds, s) in enumerate(blocks):
        a = F.relu(cv(y, c1, s, 0))
        rng_[f"b{bi}.c1"] = (0.0, float(a.max()))
        a = F.relu(cv(a, c2, 1, 1))
        rng_[f"b{bi}.c2"] = (0.0, float(a.max()))
        a = cv(a, c3, 1, 0)
        rng_[f"b{bi}.c3"] = (float(a.min()), float(a.max()))
        if ds is not None:
            idn = cv(y, ds, s, 0)
            rng_[f"b{bi}.ds"] = (float(idn.min()), float(idn.max()))
        else:
            idn = y
        y = F.relu(a + idn)
        rng_[f"b{bi}.out"] = (0.0, float(y.max()))
    g = y.mean(dim=(2, 3))
    rng_["gap"] = (0.0, float(g.max()))
    logits = g @ t(fc_w) + t(fc_b)
    rng_["fc"] = (float(logits.min()), float(logits.max()))
    return rng_


def build(batch: int = 32, seed: int = 3, calib_images: int = 4) -> QModel:
    """The quantised ResNet-50 for a given per-device batch size."""
    rng = np.random.default_rng(seed)
    convs, stem, blocks, fc_w, fc_b = _float_params(rng)
    xcal = rng.normal(0.0, 1.0, size=(calib_images, 3, 224, 224))
    r = _calibrate(convs, stem, blocks, fc_w, fc_b, xcal)

    q = {"input": _asym(*r["input"]), "stem": _relu_q(r["stem"][1])}
    nodes, shapes = [], {}
    shapes["input"] = (batch, 3, 224, 224)
    nodes.append(Node("QuantizeLinear", ["input"], "q_input", {}))
    q["q_input"] = q["input"]
    shapes["q_input"] = (batch, 3, 224, 224)

    def qconv(name, x, idx, stride, pad, yq, requant, in_layout="NHWC", post=False):
        w, b = convs[idx]
        wq, ws = _quant_w(w.astype(np.float32))
        xq = q[x]
        bias = np.rint(b / (np.float64(xq.scale) * ws.astype(np.float64))).astype(np.int64)
        bias = np.clip(bias, -2**31, 2**31 - 1).astype(np.int32)
        if in_layout == "NCHW":
            n, c, h, wd = shapes[x]
        else:
            n, h, wd, c = shapes[x]
        k = w.shape[2]
        oh = (h + 2 * pad - k) // stride + 1
        ow = (wd + 2 * pad - k) // stride + 1
        q[name] = yq
        shapes[name] = (n, oh, ow, w.shape[0])
        nodes.append(Node("QLinearConv", [x], name, dict(w=wq, w_scale=ws, bias=bias, stride=stride, pad=pad,
                                                           requant=requant, in_layout=in_layout)))
        return name

    R2, R3 = 2, 3
    cur = qconv("stem", "q_input", stem, 2, 3, q["stem"], R3, in_layout="NCHW")
    n, h, w, c = shapes[cur]
    shapes["pool"] = (n, (h + 2 - 3) // 2 + 1, (w + 2 - 3) // 2 + 1, c)
    q["pool"] = q[cur]
    nodes.append(Node("MaxPool", [cur], "pool", dict(k=3, s=2, pad=1)))
    cur = "pool"
    for bi, (c1, c2, c3, ds, s) in enumerate(blocks):
        a = qconv(f"b{bi}.c1", cur, c1, s, 0, _relu_q(r[f"b{bi}.c1"][1]), R2)
        a = qconv(f"b{bi}.c2", a, c2, 1, 1, _relu_q(r[f"b{bi}.c2"][1]), R2)
        a = qconv(f"b{bi}.c3", a, c3, 1, 0, _asym(*r[f"b{bi}.c3"]), R2)
        idn = qconv(f"b{bi}.ds", cur, ds, s, 0, _asym(*r[f"b{bi}.ds"]), R2) if ds is not None else cur
        out = f"b{bi}.out"
        q[out] = _relu_q(r[out][1])
        shapes[out] = shapes[a]
        nodes.append(Node("QLinearAdd", [a, idn], out, {}))
        cur = out
    q["gap"] = _relu_q(r["gap"][1])
    shapes["gap"] = (shapes[cur][0], shapes[cur][3])
    nodes.append(Node("DqGapQ", [cur], "gap", {}))
    # QLinearMatMul takes a per-tensor B scale (QLinearMatMul.cpp:118-134)
    b_scale = float(np.float32(np.abs(fc_w).max() / 127.0))
    bq = np.clip(np.rint(fc_w / b_scale), -127, 127).astype(np.int8)
    q["fc"] = _asym(*r["fc"])
    shapes["fc"] = (shapes["gap"][0], 1000)
    nodes.append(Node("QLinearMatMul", ["gap"], "fc", dict(b=bq, b_scale=b_scale, b_zp=0)))
    shapes["logits"] = (shapes["gap"][0], 1000)
    nodes.append(Node("DequantizeLinear", ["fc"], "logits", dict(bias=fc_b.astype(np.float32))))
    return QModel(nodes, shapes, q, batch)


def input_batch(start: int, count: int, seed: int = 3) -> np.ndarray:
    """Images [start, start + count) of the 256-image N(0,1) benchmark batch."""
    rng = np.random.default_rng([seed, 1])
    per = 3 * 224 * 224
    if start:
        rng.standard_normal(size=start * per, dtype=np.float32)  # skip earlier images
    return rng.standard_normal(size=(count, 3, 224, 224), dtype=np.float32)
