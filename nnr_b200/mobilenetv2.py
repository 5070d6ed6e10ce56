"""MobileNetV2 fp32, built from a seed.

No model file ships with the reference, so this module builds the network
synthetically as the operator list nnr runs after its graph optimizer has
folded BatchNorm into the convs (graph_optimizer/fuse_conv_bn.cpp) and fused
the Clip(0, 6) activations into them as post-ops (fuse_post_ops.cpp):

  Conv 3x3/2 3 -> 32 + Clip(0, 6)            (NCHW input, NHWC from here on)
  17 inverted residual blocks, (t, c, n, s) = (1,16,1,1) (6,24,2,2) (6,32,3,2)
    (6,64,4,2) (6,96,3,1) (6,160,3,2) (6,320,1,1):
      Conv 1x1 expand (t != 1) + Clip, depthwise Conv 3x3/s + Clip,
      Conv 1x1 project (linear), Add of the block input when s == 1 and the
      channel count is unchanged (nnr keeps the Add unfused,
      fuse_post_ops.cpp:67)
  Conv 1x1 320 -> 1280 + Clip
  GlobalAveragePool, Gemm 1280 -> 1000 (+ bias)

Weights: He-normal N(0, sqrt(2 / fan_in)) with fan_in = (C / group) * KH * KW,
biases N(0, 0.01), fp32. Generator: numpy.random.default_rng(seed), weights and
biases in network order; the input comes from default_rng([seed, 1]), N(0, 1),
drawn per 128-image shard so that any slice of the 1024-image batch can be
produced independently.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

CFG = [(1, 16, 1, 1), (6, 24, 2, 2), (6, 32, 3, 2), (6, 64, 4, 2), (6, 96, 3, 1), (6, 160, 3, 2), (6, 320, 1, 1)]
IMAGE = 224


@dataclass
class Node:
    op: str
    inputs: list
    output: str
    attrs: dict = field(default_factory=dict)


@dataclass
class FModel:
    nodes: list
    shapes: dict      # tensor name -> shape as laid out (NCHW input, NHWC activations, [n, c] after the pool)
    batch: int

    def macs_per_image(self) -> int:
        total = 0
        for nd in self.nodes:
            if nd.op == "Conv":
                w = nd.attrs["w"]
                _, oh, ow, oc = self.shapes[nd.output]
                total += oh * ow * oc * w.shape[1] * w.shape[2] * w.shape[3]
            elif nd.op == "Gemm":
                total += nd.attrs["b"].shape[0] * nd.attrs["b"].shape[1]
        return total


def _out(h: int, k: int, s: int, p: int) -> int:
    return (h + 2 * p - k) // s + 1


def build(batch: int = 128, seed: int = 4) -> FModel:
    rng = np.random.default_rng(seed)
    nodes, shapes = [], {"input": (batch, 3, IMAGE, IMAGE)}

    def conv(name, x, cin, cout, k, s, group, clip):
        fan_in = (cin // group) * k * k
        w = rng.normal(0.0, math.sqrt(2.0 / fan_in), size=(cout, cin // group, k, k)).astype(np.float32)
        b = rng.normal(0.0, 0.01, size=cout).astype(np.float32)
        if x == "input":
            _, _, h, wd = shapes[x]
        else:
            _, h, wd, _ = shapes[x]
        p = k // 2
        oh, ow = _out(h, k, s, p), _out(wd, k, s, p)
        nodes.append(Node("Conv", [x], name, {"w": w, "b": b, "stride": s, "pad": p, "group": group,
                                               "post": "Clip" if clip else None}))
        shapes[name] = (batch, oh, ow, cout)
        return name

    x = conv("stem", "input", 3, 32, 3, 2, 1, True)
    cin = 32
    bi = 0
    for t, c, n, s in CFG:
        for i in range(n):
            stride = s if i == 0 else 1
            hidden = cin * t
            y = x
            if t != 1:
                y = conv(f"m{bi}.expand", y, cin, hidden, 1, 1, 1, True)
            y = conv(f"m{bi}.dw", y, hidden, hidden, 3, stride, hidden, True)
            y = conv(f"m{bi}.project", y, hidden, c, 1, 1, 1, False)
            if stride == 1 and cin == c:
                nodes.append(Node("Add", [y, x], f"m{bi}.out"))
                shapes[f"m{bi}.out"] = shapes[y]
                y = f"m{bi}.out"
            x, cin = y, c
            bi += 1
    x = conv("head", x, cin, 1280, 1, 1, 1, True)
    nodes.append(Node("GlobalAveragePool", [x], "gap"))
    shapes["gap"] = (batch, 1280)
    fc_w = rng.normal(0.0, math.sqrt(2.0 / 1280), size=(1280, 1000)).astype(np.float32)
    fc_b = rng.normal(0.0, 0.01, size=1000).astype(np.float32)
    nodes.append(Node("Gemm", ["gap"], "logits", {"b": fc_w, "c": fc_b}))
    shapes["logits"] = (batch, 1000)
    return FModel(nodes, shapes, batch)


def input_batch(start: int, count: int, seed: int = 4, shard: int = 128) -> np.ndarray:
    """Images [start, start + count) of the seeded N(0, 1) input batch."""
    out = np.empty((count, 3, IMAGE, IMAGE), np.float32)
    i = 0
    while i < count:
        img = start + i
        s, off = divmod(img, shard)
        take = min(count - i, shard - off)
        g = np.random.default_rng([seed, 1, s])
        block = g.standard_normal((shard, 3, IMAGE, IMAGE), dtype=np.float32)
        out[i:i + take] = block[off:off + take]
        i += take
    return out
