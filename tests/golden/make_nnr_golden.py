"""Generates the golden fixtures nnr_<name>.npz in this directory from nnr's
own CPU runtime (oracle/_ref/libnnr_cpu.so, compiled from the nnr sources by
`make -C oracle nnr NNR_SRC=<nnr>/src`): each case is a one-operator (or
small QDQ) ONNX graph written by nnr_b200.onnx_models, loaded, optimised and
run by nnr's context_t. Every fixture holds the inputs, the attributes (as
JSON) and nnr's output. Run from the repository root:

    make -C oracle nnr NNR_SRC=... && python tests/golden/make_nnr_golden.py

The same case list (CASES) drives the live comparisons in
tests/test_nnr_pin.py when the library is present.
"""
from __future__ import annotations

import json
import sys
import zlib
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

# name -> (kind, params)
CASES = {
    # QDQ glue: bit-exact
    "quantize_ragged": ("quantize", dict(shape=[2, 3, 17, 19], scale=0.037, zp=117, sigma=2.0)),
    "quantize_sat": ("quantize", dict(shape=[1, 4, 5, 7], scale=0.004, zp=3, sigma=3.0)),
    "qlinearadd_relu": ("qlinearadd", dict(shape=[2, 8, 13, 11], a=[0.05, 120], b=[0.031, 77], y=[0.06, 0])),
    "qlinearadd_asym": ("qlinearadd", dict(shape=[1, 24, 7, 9], a=[0.11, 3], b=[0.02, 250], y=[0.09, 131],
                                           relu=False)),
    "maxpool_3x3s2": ("maxpool", dict(shape=[2, 16, 21, 23], scale=0.05, zp=3)),
    "dq_gap_q": ("dq_gap_q", dict(shape=[2, 64, 7, 7], x=[0.05, 3], y=[0.02, 0])),
    "dequantize_bias": ("dequantize_add", dict(shape=[4, 1000], scale=0.1, zp=128)),
    # fp32: within 1e-5 of the fp64 restatement
    "conv_c64_3x3_relu": ("conv", dict(x=[1, 64, 20, 20], oc=64, k=3, s=1, p=1, g=1, post="Relu")),
    "conv_c3_3x3s2_clip": ("conv", dict(x=[2, 3, 33, 31], oc=16, k=3, s=2, p=1, g=1, post="Clip", a=0.0, b=6.0)),
    "conv_1x1_hardswish": ("conv", dict(x=[1, 16, 9, 9], oc=24, k=1, s=1, p=0, g=1, post="HardSwish")),
    "conv_5x5_sigmoid": ("conv", dict(x=[1, 8, 12, 12], oc=16, k=5, s=1, p=2, g=1, post="Sigmoid")),
    "conv_leakyrelu": ("conv", dict(x=[1, 12, 10, 10], oc=20, k=3, s=1, p=1, g=1, post="LeakyRelu", a=0.1)),
    # residual Add of a graph input: run with nnr's nChw16c layout off, since
    # nnr adds a channel-blocked conv output to an NCHW input element by
    # element without reordering it (a reference defect, not reproduced)
    "conv_tanh_add": ("conv", dict(x=[1, 16, 8, 8], oc=16, k=3, s=1, p=1, g=1, post="Tanh", residual=True,
                                   no_blocked=True)),
    "conv_dw_s1_clip": ("conv", dict(x=[2, 32, 14, 14], oc=32, k=3, s=1, p=1, g=32, post="Clip", a=0.0, b=6.0)),
    "conv_dw_s2": ("conv", dict(x=[2, 32, 15, 15], oc=32, k=3, s=2, p=1, g=32, post=None)),
    "gemm_bias": ("gemm", dict(m=64, k=96, n=80, c="row")),
    "gemm_trans_alpha_beta": ("gemm", dict(m=33, k=40, n=50, ta=1, tb=1, alpha=0.5, beta=2.0, c="full")),
    "matmul_batched": ("matmul", dict(a=[3, 17, 24], n=40)),
    # 16-bit I/O (nnr converts to fp32, computes, rounds back): within one
    # unit in the last place of the 16-bit result
    "conv_bf16_relu": ("conv16", dict(x=[2, 16, 9, 9], oc=24, k=3, p=1, et=16, post="Relu")),
    "conv_f16": ("conv16", dict(x=[1, 32, 8, 8], oc=16, k=1, p=0, et=10, post=None)),
    "gemm_bf16": ("gemm16", dict(m=33, k=40, n=50, et=16)),
    "gemm_f16": ("gemm16", dict(m=20, k=72, n=30, et=10)),
}


def to_bits16(x, et):
    """fp32 -> bf16 (et 16, nearest even) or fp16 (et 10) bit patterns."""
    x = np.ascontiguousarray(x, np.float32)
    if et == 10:
        return x.astype(np.float16).view(np.uint16)
    u = x.view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bits16_to_f32(b, et):
    b = np.ascontiguousarray(b, np.uint16)
    if et == 10:
        return b.view(np.float16).astype(np.float32)
    return (b.astype(np.uint32) << 16).view(np.float32)


def inputs_for(name, kind, p):
    """Seeded inputs of a case (numpy default_rng, seed = crc32 of the name)."""
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    f32 = np.float32
    if kind == "quantize":
        return {"x": rng.normal(0, p["sigma"], size=p["shape"]).astype(f32)}
    if kind == "qlinearadd":
        return {"a": rng.integers(0, 256, p["shape"]).astype(np.uint8),
                "b": rng.integers(0, 256, p["shape"]).astype(np.uint8)}
    if kind in ("maxpool", "dq_gap_q"):
        return {"x": rng.integers(0, 256, p["shape"]).astype(np.uint8)}
    if kind == "dequantize_add":
        return {"x": rng.integers(0, 256, p["shape"]).astype(np.uint8),
                "bias": rng.normal(0, 1, p["shape"][1]).astype(f32)}
    if kind == "conv":
        c = p["x"][1]
        d = {"x": rng.uniform(-1, 1, p["x"]).astype(f32),
             "w": rng.normal(0, 0.2, (p["oc"], c // p["g"], p["k"], p["k"])).astype(f32),
             "b": rng.normal(0, 0.1, p["oc"]).astype(f32)}
        if p.get("residual"):
            n, _, h, w = p["x"]
            oh = (h + 2 * p["p"] - p["k"]) // p["s"] + 1
            ow = (w + 2 * p["p"] - p["k"]) // p["s"] + 1
            d["r"] = rng.normal(0, 1, (n, p["oc"], oh, ow)).astype(f32)
        return d
    if kind == "gemm":
        m, k, n = p["m"], p["k"], p["n"]
        d = {"a": rng.normal(0, 1, (k, m) if p.get("ta") else (m, k)).astype(f32),
             "B": rng.normal(0, 0.1, (n, k) if p.get("tb") else (k, n)).astype(f32)}
        d["C"] = rng.normal(0, 0.1, (n,) if p["c"] == "row" else (m, n)).astype(f32)
        return d
    if kind == "matmul":
        return {"a": rng.normal(0, 1, p["a"]).astype(f32),
                "B": rng.normal(0, 0.1, (p["a"][-1], p["n"])).astype(f32)}
    if kind == "conv16":
        c = p["x"][1]
        return {"x": to_bits16(rng.uniform(-1, 1, p["x"]), p["et"]),
                "w": to_bits16(rng.normal(0, 0.2, (p["oc"], c, p["k"], p["k"])), p["et"]),
                "b": to_bits16(rng.normal(0, 0.1, p["oc"]), p["et"])}
    if kind == "gemm16":
        return {"a": to_bits16(rng.normal(0, 1, (p["m"], p["k"])), p["et"]),
                "B": to_bits16(rng.normal(0, 0.1, (p["k"], p["n"])), p["et"]),
                "C": to_bits16(rng.normal(0, 0.1, p["n"]), p["et"])}
    raise ValueError(kind)


def model_for(kind, p, d) -> bytes:
    from nnr_b200 import onnx_models as M
    if kind == "quantize":
        return M.quantize(p["shape"], p["scale"], p["zp"])
    if kind == "qlinearadd":
        return M.qlinearadd(p["shape"], *p["a"], *p["b"], *p["y"], relu=p.get("relu", True))
    if kind == "maxpool":
        return M.maxpool_u8(p["shape"], p["scale"], p["zp"])
    if kind == "dq_gap_q":
        return M.dq_gap_q(p["shape"], *p["x"], *p["y"])
    if kind == "dequantize_add":
        return M.dequantize_add(p["shape"], p["scale"], p["zp"], d["bias"])
    if kind == "conv":
        s = p["s"]
        return M.conv(p["x"], d["w"], d["b"], strides=(s, s), pads=(p["p"],) * 4, group=p["g"], post=p["post"],
                      post_a=p.get("a", 0.0), post_b=p.get("b", 0.0), residual=p.get("residual", False))
    if kind == "gemm":
        return M.gemm(p["m"], p["k"], p["n"], d["B"], d["C"], alpha=p.get("alpha", 1.0), beta=p.get("beta", 1.0),
                      trans_a=p.get("ta", 0), trans_b=p.get("tb", 0))
    if kind == "matmul":
        return M.matmul(p["a"], d["B"])
    if kind == "conv16":
        return M.conv_half(p["x"], d["w"], d["b"], p["et"], pads=(p["p"],) * 4, post=p["post"])
    if kind == "gemm16":
        return M.gemm_half(p["m"], p["k"], p["n"], d["B"], d["C"], p["et"])
    raise ValueError(kind)


GRAPH_INPUTS = {"quantize": ["x"], "qlinearadd": ["a", "b"], "maxpool": ["x"], "dq_gap_q": ["x"],
                "dequantize_add": ["x"], "conv": ["x", "r"], "gemm": ["a"], "matmul": ["a"], "conv16": ["x"],
                "gemm16": ["a"]}


def run_nnr(name):
    """nnr's output for case `name` (needs oracle/_ref/libnnr_cpu.so)."""
    from oracle import nnr_ref as R
    kind, p = CASES[name]
    d = inputs_for(name, kind, p)
    m = R.NnrModel(model_for(kind, p, d), no_blocked=p.get("no_blocked", False))
    for k in GRAPH_INPUTS[kind]:
        if k in d:
            m.set(k, d[k])
    m.run()
    y = m.get("y")
    m.close()
    return d, y


def main() -> int:
    from oracle import nnr_ref as R
    if not R.available():
        print("oracle/_ref/libnnr_cpu.so not built: run `make -C oracle nnr NNR_SRC=...`", file=sys.stderr)
        return 1
    for name, (kind, p) in CASES.items():
        d, y = run_nnr(name)
        np.savez_compressed(HERE / f"nnr_{name}.npz", y=y, params=json.dumps({"kind": kind, **p}), **d)
        print(name, kind, y.shape, y.dtype)
    return 0


if __name__ == "__main__":
    sys.exit(main())
