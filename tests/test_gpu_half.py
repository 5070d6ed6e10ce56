"""16-bit (bf16 / fp16) Conv and Gemm on one kind::f16 plane, and the fp32
MatMul of nnr's AVX-512 BF16 hosts, through the C ABI.

nnr's 16-bit paths convert to fp32, compute in fp32, apply the post-op and
round the result to the 16-bit type (Conv_exec_entry.h:188-381, Gemm.cpp:
297-513); the oracle does the same from the same 16-bit values (fp64 sums,
pinned to nnr in test_nnr_pin.py). The device's fp32 sums differ only in
order, so every 16-bit result must be within one unit in the last place of
the oracle's, plus the fp32 summation error (1e-5 of the sum of |terms|,
which matters only where terms cancel to a small result).
nnr's fp32 MatMul with a constant B on an AVX-512 BF16 host rounds both
operands to bf16 (MatMul.cpp:382-428); NNRCU_PREC_BF16 does the same and must
agree within 1e-5 relative L2.
"""
import importlib.util
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

_spec = importlib.util.spec_from_file_location("make_nnr_golden",
                                               Path(__file__).parent / "golden" / "make_nnr_golden.py")
G = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(G)
ET = {"bf16": 16, "f16": 10}
POST = {None: 0, "Relu": 1, "Clip": 2, "HardSwish": 3}


def ulp_ok(got_bits, want_bits, et, abs_sum):
    """Number of results off by more than one 16-bit ulp plus 1e-5 x the sum
    of |terms| (abs_sum, same layout)."""
    g = G.bits16_to_f32(got_bits, et).astype(np.float64)
    w = G.bits16_to_f32(want_bits, et).astype(np.float64)
    mant = 10 if et == 10 else 7
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(w), 1e-30))) - mant)
    bad = np.abs(g - w) > ulp * 1.0001 + 1e-5 * np.asarray(abs_sum, np.float64)
    return int(bad.sum())


def dev16(bits, dev):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(dev)


def host_bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


CONV_SHAPES = [
    # x shape, oc, k, stride, pad, in/out layout
    ((2, 16, 9, 9), 24, 3, 1, 1, "NCHW"),
    ((1, 64, 14, 14), 128, 1, 1, 0, "NHWC"),   # 1x1 over 64 channels: 2-D TMA A
    ((2, 32, 15, 15), 48, 3, 2, 1, "NHWC"),
    ((1, 3, 32, 32), 16, 3, 1, 1, "NCHW"),     # few channels: gathered A
    ((4, 256, 7, 7), 512, 3, 1, 1, "NHWC"),
]


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("shape", CONV_SHAPES)
@pytest.mark.parametrize("post", [None, "Relu", "Clip", "HardSwish"])
def test_conv_half(cuda_dev, dtype, shape, post):
    from nnr_b200 import ops
    xs, oc, k, s, p, lay = shape
    et = ET[dtype]
    rng = np.random.default_rng(oc * 7 + k)
    xb = G.to_bits16(rng.uniform(-1, 1, xs), et)
    wb = G.to_bits16(rng.normal(0, 0.2, (oc, xs[1], k, k)), et)
    bb = G.to_bits16(rng.normal(0, 0.1, oc), et)
    pa, pb = (0.0, 6.0) if post == "Clip" else (0.0, 0.0)
    ref = O.conv_f32(G.bits16_to_f32(xb, et), G.bits16_to_f32(wb, et), G.bits16_to_f32(bb, et), strides=(s, s),
                     pads=(p,) * 4, post=POST[post], post_a=pa, post_b=pb, in_layout="NCHW", out_layout=lay)
    want = G.to_bits16(ref, et)
    f = {k: np.abs(G.bits16_to_f32(v, et)) for k, v in (("x", xb), ("w", wb), ("b", bb))}
    abs_sum = O.conv_f32(f["x"], f["w"], f["b"], strides=(s, s), pads=(p,) * 4, in_layout="NCHW", out_layout=lay)
    op = ops.ConvHalf(xs, wb, bb, dtype=ops.DT_BF16 if dtype == "bf16" else ops.DT_F16, strides=(s, s),
                      pads=(p,) * 4, in_layout=lay, out_layout=lay, post=post, post_a=pa, post_b=pb)
    xin = xb if lay == "NCHW" else np.ascontiguousarray(xb.transpose(0, 2, 3, 1))
    y = op.exec(dev16(xin, cuda_dev))
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    got = host_bits(y)
    assert got.shape == want.shape
    assert ulp_ok(got, want, et, abs_sum) == 0


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("shape", [((2, 64, 14, 14), 128, 3, 1, 1, 4, "NHWC"), ((1, 128, 9, 11), 64, 3, 2, 1, 32, "NCHW")])
def test_grouped_conv_half(cuda_dev, dtype, shape):
    """Grouped (not depthwise) 16-bit Conv + Relu: the fp32 sums of each
    group, rounded once to the 16-bit type."""
    from nnr_b200 import ops
    xs, oc, k, s, p, g, lay = shape
    et = ET[dtype]
    rng = np.random.default_rng(oc + g)
    xb = G.to_bits16(rng.uniform(-1, 1, xs), et)
    wb = G.to_bits16(rng.normal(0, 0.2, (oc, xs[1] // g, k, k)), et)
    bb = G.to_bits16(rng.normal(0, 0.1, oc), et)
    kw = dict(strides=(s, s), pads=(p,) * 4, group=g, in_layout="NCHW", out_layout=lay)
    ref = O.conv_f32(G.bits16_to_f32(xb, et), G.bits16_to_f32(wb, et), G.bits16_to_f32(bb, et), post=1, **kw)
    want = G.to_bits16(ref, et)
    f = {k: np.abs(G.bits16_to_f32(v, et)) for k, v in (("x", xb), ("w", wb), ("b", bb))}
    abs_sum = O.conv_f32(f["x"], f["w"], f["b"], **kw)
    op = ops.ConvHalf(xs, wb, bb, dtype=ops.DT_BF16 if dtype == "bf16" else ops.DT_F16, strides=(s, s),
                      pads=(p,) * 4, in_layout=lay, out_layout=lay, post="Relu", group=g)
    xin = xb if lay == "NCHW" else np.ascontiguousarray(xb.transpose(0, 2, 3, 1))
    y = op.exec(dev16(xin, cuda_dev))
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert ulp_ok(host_bits(y), want, et, abs_sum) == 0


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("shape", [((2, 32, 17, 15), 3, 1, 1, 1, "NHWC", "NHWC"), ((2, 48, 16, 16), 3, 2, 1, 1, "NCHW", "NHWC"),
                                   ((1, 20, 11, 9), 5, 1, 2, 1, "NHWC", "NCHW"), ((1, 16, 12, 12), 3, 1, 2, 2, "NCHW", "NCHW"),
                                   ((1, 6, 8, 8), 3, 1, 1, 1, "NHWC", "NHWC")])
@pytest.mark.parametrize("post", [None, "Clip"])
def test_depthwise_conv_half(cuda_dev, dtype, shape, post):
    """16-bit depthwise Conv (group = C): fp32 sums of the widened values,
    rounded once (C % 4 != 0 takes the block-diagonal dense path)."""
    from nnr_b200 import ops
    xs, k, s, p, dil, lin, lout = shape
    c = xs[1]
    et = ET[dtype]
    rng = np.random.default_rng(c * 3 + k)
    xb = G.to_bits16(rng.uniform(-1, 1, xs), et)
    wb = G.to_bits16(rng.normal(0, 0.3, (c, 1, k, k)), et)
    bb = G.to_bits16(rng.normal(0, 0.1, c), et)
    pa, pb = (0.0, 0.5) if post == "Clip" else (0.0, 0.0)
    kw = dict(strides=(s, s), pads=(p,) * 4, dilations=(dil, dil), group=c, in_layout="NCHW", out_layout=lout)
    ref = O.conv_f32(G.bits16_to_f32(xb, et), G.bits16_to_f32(wb, et), G.bits16_to_f32(bb, et), post=POST[post],
                     post_a=pa, post_b=pb, **kw)
    want = G.to_bits16(ref, et)
    f = {k: np.abs(G.bits16_to_f32(v, et)) for k, v in (("x", xb), ("w", wb), ("b", bb))}
    abs_sum = O.conv_f32(f["x"], f["w"], f["b"], **kw)
    op = ops.ConvHalf(xs, wb, bb, dtype=ops.DT_BF16 if dtype == "bf16" else ops.DT_F16, strides=(s, s),
                      pads=(p,) * 4, dilations=(dil, dil), in_layout=lin, out_layout=lout, post=post, post_a=pa,
                      post_b=pb, group=c)
    xin = xb if lin == "NCHW" else np.ascontiguousarray(xb.transpose(0, 2, 3, 1))
    y = op.exec(dev16(xin, cuda_dev))
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    got = host_bits(y)
    assert got.shape == want.shape
    assert ulp_ok(got, want, et, abs_sum) == 0


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("m,k,n,c,trans_b", [(200, 192, 300, "row", 0), (64, 768, 256, "full", 1),
                                             (33, 40, 50, None, 0), (4096, 768, 3072, "row", 0)])
def test_gemm_half(cuda_dev, dtype, m, k, n, c, trans_b):
    from nnr_b200 import ops
    et = ET[dtype]
    rng = np.random.default_rng(m + n)
    ab = G.to_bits16(rng.normal(0, 1, (m, k)), et)
    bmat = rng.normal(0, 0.05, (n, k) if trans_b else (k, n))
    bb = G.to_bits16(bmat, et)
    cb = None if c is None else G.to_bits16(rng.normal(0, 0.1, n if c == "row" else (m, n)), et)
    ref = O.gemm_f32(G.bits16_to_f32(ab, et), G.bits16_to_f32(bb, et), None if cb is None else G.bits16_to_f32(cb, et),
                     beta=0.5 if cb is not None else 1.0, trans_b=trans_b)
    want = G.to_bits16(ref, et)
    abs_sum = O.gemm_f32(np.abs(G.bits16_to_f32(ab, et)), np.abs(G.bits16_to_f32(bb, et)),
                         None if cb is None else np.abs(G.bits16_to_f32(cb, et)),
                         beta=0.5 if cb is not None else 1.0, trans_b=trans_b)
    op = ops.GemmHalf(m, bb, cb, dtype=ops.DT_BF16 if dtype == "bf16" else ops.DT_F16,
                      beta=0.5 if cb is not None else 1.0, trans_b=trans_b)
    y = op.exec(dev16(ab, cuda_dev))
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert ulp_ok(host_bits(y), want, et, abs_sum) == 0


@pytest.mark.parametrize("shape", [(17, 24, 40), (4096, 768, 3072), (51, 2048, 1000)])
def test_matmul_bf16_host_precision(cuda_dev, shape):
    from nnr_b200 import ops
    from oracle import nnr_ref as R
    m, k, n = shape
    rng = np.random.default_rng(k)
    a = rng.normal(0, 1, (m, k)).astype(np.float32)
    b = rng.normal(0, 0.1, (k, n)).astype(np.float32)
    op = ops.MatMul(m, b, precision=ops.PREC_BF16)
    y = op.exec(torch.from_numpy(a).to(cuda_dev)).cpu().numpy()
    want = O.matmul_f32_bf16_host(a, b)
    e = np.linalg.norm(y.astype(np.float64) - want) / np.linalg.norm(want)
    assert e <= 1e-5
    if R.available() and m <= 64:
        from nnr_b200 import onnx_models as M
        net = R.NnrModel(M.matmul((m, k), b))
        net.set("a", a)
        net.run()
        nn = net.get("y")
        assert np.linalg.norm(y.astype(np.float64) - nn) / np.linalg.norm(nn) <= 1e-5
