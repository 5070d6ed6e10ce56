"""Parity of the device QLinearConv / QLinearMatMul with the CPU oracle.

Integer outputs must be bit-exact (nnr's tensor_equal compares integer
tensors exactly, src/nnr.cpp:503-606). Every call goes through the C ABI
(libnnrcu.so) via nnr_b200.ops.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle as O
from nnr_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _to_nhwc(x):
    return np.ascontiguousarray(x.transpose(0, 2, 3, 1))


def run_qconv(dev, case, formula=O.R1, in_layout="NCHW", out_layout="NCHW", fused_relu=False, requant=None):
    from nnr_b200 import ops
    from nnr_b200._lib import RQ_AUTO
    x_dev_np = case.x if in_layout == "NCHW" else _to_nhwc(case.x)
    op = ops.QLinearConv(case.x.shape, case.w, case.w_scale, case.w_zp, case.bias, case.x_scale, case.x_zp,
                         case.y_scale, case.y_zp, strides=case.strides, pads=case.pads, dilations=case.dilations,
                         in_layout=in_layout, out_layout=out_layout, fused_relu=fused_relu,
                         requant=formula if requant is None else requant)
    x = torch.from_numpy(x_dev_np).to(dev)
    y = op.exec(x)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    return y.cpu().numpy(), op


def oracle_qconv(case, formula, out_layout="NCHW", fused_relu=False):
    return O.qlinearconv(case.x, case.w, case.w_scale, case.bias, case.x_scale, case.x_zp, case.y_scale, case.y_zp,
                         strides=case.strides, pads=case.pads, dilations=case.dilations, formula=formula,
                         has_post=fused_relu, out_layout=out_layout)


def test_config2_bit_exact(cuda_dev):
    """BASELINE config 2 at full size; nnr dispatches exec_direct_int8 (R1)."""
    case = W.config2_qlinearconv()
    y, op = run_qconv(cuda_dev, case, requant=0)
    ref = oracle_qconv(case, O.R1)
    assert np.array_equal(y, ref), f"{(y != ref).sum()} mismatches"
    assert op.num_ops() == 7_398_752_256


def test_config2_nhwc_r2(cuda_dev):
    """Same layer inside an NHWC chain: nnr's packed NR48 path (R2)."""
    case = W.config2_qlinearconv(n=4)
    y, _ = run_qconv(cuda_dev, case, in_layout="NHWC", out_layout="NHWC", requant=0)
    ref = oracle_qconv(case, O.R2, out_layout="NHWC")
    assert np.array_equal(y, ref)


SHAPES = [
    # n, c, h, w, oc, kh, kw, strides, pads, dilations
    (2, 64, 13, 11, 96, 3, 3, (1, 1), (1, 1, 1, 1), (1, 1)),
    (3, 128, 28, 28, 128, 3, 3, (2, 2), (1, 1, 1, 1), (1, 1)),
    (2, 256, 14, 14, 64, 1, 1, (1, 1), (0, 0, 0, 0), (1, 1)),   # 1x1 -> TMA A path when NHWC
    (2, 64, 28, 28, 256, 1, 1, (2, 2), (0, 0, 0, 0), (1, 1)),   # 1x1 stride 2 (downsample)
    (1, 5, 9, 7, 17, 3, 3, (1, 1), (2, 0, 1, 1), (1, 1)),       # ragged channels, asymmetric pads
    (2, 32, 16, 16, 48, 3, 3, (1, 1), (2, 2, 2, 2), (2, 2)),    # dilation 2
    (1, 512, 7, 7, 512, 3, 3, (1, 1), (1, 1, 1, 1), (1, 1)),    # ResNet stage 4 3x3
    (1, 16, 5, 5, 256, 5, 5, (1, 1), (0, 0, 0, 0), (1, 1)),     # single output pixel
]


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("formula", [O.R1, O.R2, O.R3])
@pytest.mark.parametrize("layouts", [("NCHW", "NCHW"), ("NHWC", "NHWC")])
def test_random_shapes(cuda_dev, shape, formula, layouts):
    n, c, h, w, oc, kh, kw, s, p, d = shape
    rng = np.random.default_rng(hash((shape, formula)) & 0xffff)
    case = W.random_qconv(rng, n, c, h, w, oc, kh, kw, s, p, d)
    y, _ = run_qconv(cuda_dev, case, formula, layouts[0], layouts[1])
    ref = oracle_qconv(case, formula, layouts[1])
    assert np.array_equal(y, ref), f"{(y != ref).sum()} / {y.size} mismatches"


@pytest.mark.parametrize("formula", [O.R1, O.R2, O.R3])
def test_fused_relu_and_zero_points(cuda_dev, formula):
    """A fused Relu raises the lower clamp to y_zp for R1/R3; R2 ignores it
    (QLinearConv_reshape.h:326). x_zp = 0 (post-Relu activations) and odd zps."""
    rng = np.random.default_rng(7)
    for xz, yz in [(0, 0), (0, 37), (200, 3)]:
        case = W.random_qconv(rng, 2, 64, 12, 12, 64, 3, 3, (1, 1), (1, 1, 1, 1), x_zp=xz, y_zp=yz)
        y, _ = run_qconv(cuda_dev, case, formula, fused_relu=True)
        ref = oracle_qconv(case, formula, fused_relu=True)
        assert np.array_equal(y, ref)


def test_stem_auto_r3(cuda_dev):
    """ResNet stem 7x7/2 on a 3-channel NCHW input: nnr's first-layer path (R3)."""
    rng = np.random.default_rng(3)
    case = W.random_qconv(rng, 2, 3, 64, 64, 64, 7, 7, (2, 2), (3, 3, 3, 3), x_zp=128, y_zp=0)
    y, _ = run_qconv(cuda_dev, case, in_layout="NCHW", out_layout="NHWC", requant=0)
    ref = oracle_qconv(case, O.R3, out_layout="NHWC")
    assert np.array_equal(y, ref)


FIRST_GOLDEN = sorted((Path(__file__).parent / "golden").glob("qfirst_*.npz"))


@pytest.mark.parametrize("path", FIRST_GOLDEN, ids=lambda p: p.stem)
def test_first_layer_matches_nnr_golden(cuda_dev, path):
    """The stem formula picked automatically (R3) against nnr's own
    first-layer kernel output, NCHW outputs including the scalar tail of each
    row's last OW % 16 pixels."""
    from nnr_b200 import ops
    g = np.load(path)
    s, p, xz, yz, post, nhwc = (int(v) for v in g["attrs"])
    xs, ys = (float(v) for v in g["scales"])
    op = ops.QLinearConv(g["x"].shape, g["w"], g["w_scale"], None, g["bias"], xs, xz, ys, yz, strides=(s, s),
                         pads=(p,) * 4, in_layout="NCHW", out_layout="NHWC" if nhwc else "NCHW",
                         fused_relu=bool(post), requant=0)
    y = op.exec(torch.from_numpy(g["x"]).to(cuda_dev))
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    got = y.cpu().numpy()
    assert np.array_equal(got, g["y"]), f"{(got != g['y']).sum()} bytes differ from nnr's first-layer kernel"


S2D_SHAPES = [
    # stride-2 convs over <= 4 channels run as space-to-depth convs (16-byte taps)
    (2, 3, 64, 64, 64, 7, 7, (2, 2), (3, 3, 3, 3), (1, 1)),      # the ResNet stem
    (1, 3, 37, 29, 128, 7, 7, (2, 2), (3, 2, 3, 4), (1, 1)),     # odd sizes, asymmetric pads, N tile 128
    (2, 1, 20, 21, 48, 3, 3, (2, 2), (1, 1, 1, 1), (1, 1)),      # one channel, ragged N
    (1, 4, 16, 18, 32, 5, 5, (2, 2), (0, 2, 1, 0), (1, 1)),      # four channels, no top pad
    (3, 2, 15, 15, 64, 2, 2, (2, 2), (0, 0, 0, 0), (1, 1)),      # even kernel, one tap per s2d pixel
    (1, 3, 9, 9, 16, 3, 4, (2, 2), (2, 1, 0, 2), (1, 1)),        # taps not a multiple of 8
]


@pytest.mark.parametrize("shape", S2D_SHAPES)
@pytest.mark.parametrize("formula", [O.R1, O.R2, O.R3])
@pytest.mark.parametrize("layouts", [("NCHW", "NHWC"), ("NHWC", "NCHW")])
def test_space_to_depth_stride2(cuda_dev, shape, formula, layouts):
    n, c, h, w, oc, kh, kw, s, p, d = shape
    rng = np.random.default_rng(hash((shape, formula, "s2d")) & 0xffff)
    for xz in (0, 131):
        case = W.random_qconv(rng, n, c, h, w, oc, kh, kw, s, p, d, x_zp=xz)
        y, _ = run_qconv(cuda_dev, case, formula, layouts[0], layouts[1])
        ref = oracle_qconv(case, formula, layouts[1])
        assert np.array_equal(y, ref), f"x_zp {xz}: {(y != ref).sum()} / {y.size} mismatches"


def test_no_bias_per_tensor_scale(cuda_dev):
    rng = np.random.default_rng(11)
    case = W.random_qconv(rng, 1, 32, 10, 10, 32, 3, 3, (1, 1), (1, 1, 1, 1), per_channel=False, bias=False)
    for f in (O.R1, O.R2, O.R3):
        y, _ = run_qconv(cuda_dev, case, f)
        assert np.array_equal(y, oracle_qconv(case, f))


def test_repeat_and_graph_capture(cuda_dev):
    """Same op launched repeatedly and replayed from a captured CUDA graph."""
    from nnr_b200 import ops
    rng = np.random.default_rng(5)
    case = W.random_qconv(rng, 4, 64, 14, 14, 128, 3, 3, (1, 1), (1, 1, 1, 1))
    op = ops.QLinearConv(case.x.shape, case.w, case.w_scale, case.w_zp, case.bias, case.x_scale, case.x_zp,
                         case.y_scale, case.y_zp, pads=case.pads, requant=O.R1)
    x = torch.from_numpy(case.x).to(cuda_dev)
    y = torch.empty(op.y_shape, dtype=torch.uint8, device=cuda_dev)
    ws = torch.empty(max(op.workspace_size(), 1), dtype=torch.uint8, device=cuda_dev)
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        op.exec(x, y, ws, stream=s)
    for _ in range(3):
        y.zero_()
        g.replay()
    torch.cuda.synchronize()
    assert np.array_equal(y.cpu().numpy(), oracle_qconv(case, O.R1))


# ------------------------------------------------------------------ QLinearMatMul

def run_qmm(dev, a, b, a_scale, a_zp, b_scale, b_zp, y_scale, y_zp):
    from nnr_b200 import ops
    op = ops.QLinearMatMul(a.shape[0], b, a_scale, a_zp, b_scale, b_zp, y_scale, y_zp)
    y = op.exec(torch.from_numpy(a).to(dev))
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    return y.cpu().numpy()


def test_config3_qlinearmatmul_bit_exact(cuda_dev):
    c = W.config3_matmul()
    y = run_qmm(cuda_dev, c.a_u8, c.b_s8, c.a_scale, c.a_zp, c.b_scale, c.b_zp, c.y_scale, c.y_zp)
    ref = O.qlinearmatmul(c.a_u8, c.b_s8, c.a_scale, c.a_zp, c.b_scale, c.b_zp, c.y_scale, c.y_zp)
    assert np.array_equal(y, ref), f"{(y != ref).sum()} mismatches"


@pytest.mark.parametrize("m,k,n,b_zp", [(32, 2048, 1000, 0), (200, 100, 70, 0), (129, 256, 300, -3),
                                        (1, 768, 64, 5), (257, 48, 33, 0),
                                        # M <= 64: the CUDA-core dp4a path
                                        (64, 100, 70, -3), (7, 4096, 129, 2), (33, 16, 1000, 0)])
def test_qlinearmatmul_shapes(cuda_dev, m, k, n, b_zp):
    rng = np.random.default_rng(m * 7 + k)
    a = rng.integers(0, 256, size=(m, k)).astype(np.uint8)
    b = rng.integers(-127, 128, size=(k, n)).astype(np.int8)
    ys = 0.03 * 0.004 * 30.0 * np.sqrt(k)
    y = run_qmm(cuda_dev, a, b, 0.03, 117, 0.004, b_zp, ys, 100)
    ref = O.qlinearmatmul(a, b, 0.03, 117, 0.004, b_zp, ys, 100)
    assert np.array_equal(y, ref)


# Hardware-im2col path: NHWC inputs with a 128-byte multiple channel stride
# and >= 128 KB; x_zp = 0 so the TMA zero fill equals the padding value.
IM2COL_SHAPES = [
    (2, 128, 28, 28, 128, 3, 3, (1, 1), (1, 1, 1, 1), (1, 1)),
    (2, 256, 20, 18, 96, 3, 3, (2, 2), (1, 0, 1, 1), (1, 1)),
    (1, 128, 40, 40, 64, 3, 3, (1, 1), (2, 2, 2, 2), (2, 2)),
    (4, 128, 13, 15, 160, 5, 5, (2, 1), (2, 2, 2, 2), (1, 1)),
    (2, 64, 32, 32, 64, 3, 3, (1, 1), (1, 1, 1, 1), (1, 1)),     # 64-byte K slabs (SWIZZLE_64B)
    (3, 64, 30, 30, 128, 3, 3, (2, 2), (1, 1, 1, 1), (1, 1)),
    (2, 64, 24, 24, 256, 1, 1, (1, 1), (0, 0, 0, 0), (1, 1)),     # 1x1, 64-byte slabs, plain TMA
]


@pytest.mark.parametrize("shape", IM2COL_SHAPES)
@pytest.mark.parametrize("formula", [O.R1, O.R2])
def test_im2col_zero_zp(cuda_dev, shape, formula):
    n, c, h, w, oc, kh, kw, s, p, d = shape
    rng = np.random.default_rng(sum(shape[:7]) + formula)
    case = W.random_qconv(rng, n, c, h, w, oc, kh, kw, s, p, d, x_zp=0)
    for lay in (("NHWC", "NHWC"), ("NCHW", "NCHW")):
        y, _ = run_qconv(cuda_dev, case, formula, lay[0], lay[1])
        ref = oracle_qconv(case, formula, lay[1])
        assert np.array_equal(y, ref), f"{lay}: {(y != ref).sum()} / {y.size} mismatches"


@pytest.mark.parametrize("shape", IM2COL_SHAPES[:2])
def test_im2col_padded_copy_nonzero_zp(cuda_dev, shape):
    """NCHW input with x_zp != 0: reordered into an x_zp-bordered NHWC copy."""
    n, c, h, w, oc, kh, kw, s, p, d = shape
    rng = np.random.default_rng(77)
    case = W.random_qconv(rng, n, c, h, w, oc, kh, kw, s, p, d, x_zp=201)
    for f in (O.R1, O.R2):
        y, _ = run_qconv(cuda_dev, case, f, "NCHW", "NCHW")
        assert np.array_equal(y, oracle_qconv(case, f))


@pytest.mark.parametrize("shape", [(2, 64, 14, 14, 256, 1, 0), (1, 32, 7, 9, 17, 3, 1), (3, 128, 10, 10, 48, 3, 1)])
def test_conv_with_fused_residual_add(cuda_dev, shape):
    """nnrcu_qlinearconv_run_add == QLinearConv then QLinearAdd(conv, residual);
    odd element counts exercise QLinearAdd's scalar tail."""
    import ctypes as C
    from nnr_b200 import ops
    from nnr_b200._lib import check, lib
    n, c, h, w, oc, k, p = shape
    rng = np.random.default_rng(oc + k)
    case = W.random_qconv(rng, n, c, h, w, oc, k, k, (1, 1), (p,) * 4, x_zp=0)
    op = ops.QLinearConv(case.x.shape, case.w, case.w_scale, case.w_zp, case.bias, case.x_scale, case.x_zp,
                         case.y_scale, case.y_zp, pads=case.pads, in_layout="NHWC", out_layout="NHWC", requant=O.R2)
    conv = oracle_qconv(case, O.R2, out_layout="NHWC")
    res = rng.integers(0, 256, size=conv.shape).astype(np.uint8)
    rs, rz, ys, yz = 0.037, 101, 0.05, 7
    ref = O.qlinearadd_u8(conv, case.y_scale, case.y_zp, res, rs, rz, ys, yz)
    x = torch.from_numpy(_to_nhwc(case.x)).to(cuda_dev)
    r = torch.from_numpy(res).to(cuda_dev)
    y = torch.empty(conv.shape, dtype=torch.uint8, device=cuda_dev)
    ws = torch.empty(max(op.workspace_size(), 1), dtype=torch.uint8, device=cuda_dev)
    check(lib.nnrcu_qlinearconv_run_add(op._op, C.c_void_p(x.data_ptr()), C.c_void_p(r.data_ptr()), rs, rz, ys, yz,
                                        C.c_void_p(y.data_ptr()), C.c_void_p(ws.data_ptr()),
                                        C.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert np.array_equal(y.cpu().numpy(), ref)


@pytest.mark.parametrize("kind", ["1x1", "3x3", "shift"])
@pytest.mark.parametrize("y_scale", [1e-7, 0.05, 3.0])
def test_r2_zero_point_zero(cuda_dev, kind, y_scale):
    """R2 with y_zp = 0 (every Relu output) runs as one saturating conversion
    per value: rounding ties, both saturation ends and huge values agree with
    the clamp-then-round reference, fused Relu or not."""
    rng = np.random.default_rng(int(y_scale * 1e3) + len(kind))
    k, p = (1, 0) if kind == "1x1" else (3, 1)
    h = 56 if kind == "shift" else 13
    case = W.random_qconv(rng, 2, 64, h, h, 128, k, k, (1, 1), (p,) * 4, x_zp=17, y_zp=0)
    case.y_scale = y_scale
    for relu in (False, True):
        y, _ = run_qconv(cuda_dev, case, O.R2, "NHWC", "NHWC", fused_relu=relu)
        ref = oracle_qconv(case, O.R2, "NHWC", fused_relu=relu)
        assert np.array_equal(y, ref), f"relu {relu}: {(y != ref).sum()} / {y.size} mismatches"


@pytest.mark.parametrize("kind", ["1x1", "3x3"])
def test_saturating_scales(cuda_dev, kind):
    """Tiny output scales: R2 values far outside [0, 255] (the clamp before the
    float-adder rounding), and a fused QLinearAdd whose value passes 2^31,
    where the reference's x86 conversion yields INT_MIN (so 0, not 255).
    Outputs saturate heavily; both must still match bit for bit."""
    import ctypes as C
    from nnr_b200 import ops
    from nnr_b200._lib import check, lib
    rng = np.random.default_rng(11 if kind == "1x1" else 12)
    k, p = (1, 0) if kind == "1x1" else (3, 1)
    case = W.random_qconv(rng, 2, 64, 16, 16, 128, k, k, (1, 1), (p,) * 4, x_zp=0)
    case.y_scale = 1e-7
    y, _ = run_qconv(cuda_dev, case, O.R2, "NHWC", "NHWC")
    ref = oracle_qconv(case, O.R2, "NHWC")
    assert np.array_equal(y, ref)
    op = ops.QLinearConv(case.x.shape, case.w, case.w_scale, case.w_zp, case.bias, case.x_scale, case.x_zp,
                         case.y_scale, case.y_zp, pads=case.pads, in_layout="NHWC", out_layout="NHWC", requant=O.R2)
    res = rng.integers(0, 256, size=ref.shape).astype(np.uint8)
    rs, rz, ys, yz = 0.037, 101, 1e-9, 7
    want = O.qlinearadd_u8(ref, case.y_scale, case.y_zp, res, rs, rz, ys, yz)
    x = torch.from_numpy(_to_nhwc(case.x)).to(cuda_dev)
    r = torch.from_numpy(res).to(cuda_dev)
    out = torch.empty(ref.shape, dtype=torch.uint8, device=cuda_dev)
    ws = torch.empty(max(op.workspace_size(), 1), dtype=torch.uint8, device=cuda_dev)
    check(lib.nnrcu_qlinearconv_run_add(op._op, C.c_void_p(x.data_ptr()), C.c_void_p(r.data_ptr()), rs, rz, ys, yz,
                                        C.c_void_p(out.data_ptr()), C.c_void_p(ws.data_ptr()),
                                        C.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert np.array_equal(out.cpu().numpy(), want)


@pytest.mark.parametrize("shape", S2D_SHAPES[:4])
@pytest.mark.parametrize("in_layout", ["NCHW", "NHWC"])
def test_quantize_fused_into_space_to_depth(cuda_dev, shape, in_layout):
    """nnrcu_qlinearconv_run_quantize == QuantizeLinear then QLinearConv; an
    element count that is not a multiple of 16 exercises QuantizeLinear's
    scalar tail, and large inputs its saturation."""
    from nnr_b200 import ops
    n, c, h, w, oc, kh, kw, s, p, d = shape
    rng = np.random.default_rng(hash((shape, in_layout)) & 0xffff)
    case = W.random_qconv(rng, n, c, h, w, oc, kh, kw, s, p, d, x_zp=117)
    xf = (rng.standard_normal((n, c, h, w)) * 3.0).astype(np.float32)
    xf.flat[::97] *= 1e4
    qs = 0.021
    # QuantizeLinear's body/tail split follows the flat index of the tensor as laid out
    if in_layout == "NCHW":
        xq = O.quantize_u8(xf.ravel(), qs, 117).reshape(xf.shape)
    else:
        xq = O.quantize_u8(_to_nhwc(xf).ravel(), qs, 117).reshape(n, h, w, c).transpose(0, 3, 1, 2).copy()
    ref = O.qlinearconv(xq, case.w, case.w_scale, case.bias, case.x_scale, 117, case.y_scale, case.y_zp,
                        strides=case.strides, pads=case.pads, dilations=case.dilations, formula=O.R3,
                        out_layout="NHWC")
    op = ops.QLinearConv(xf.shape, case.w, case.w_scale, case.w_zp, case.bias, case.x_scale, 117, case.y_scale,
                         case.y_zp, strides=case.strides, pads=case.pads, dilations=case.dilations,
                         in_layout=in_layout, out_layout="NHWC", requant=O.R3)
    assert op.space_to_depth
    x = torch.from_numpy(xf if in_layout == "NCHW" else _to_nhwc(xf)).to(cuda_dev)
    y = op.exec_quantize(x, qs, 117)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert np.array_equal(y.cpu().numpy(), ref)



# Shifted-patch path (A_SHIFT): stride-1 spatial convs over whole 64/128-byte
# channel slabs, computed on the x_zp-bordered padded grid; a CTA keeps one
# N tile's weights resident (1, 2 or 4 N tiles of 64, or of 128 columns).
# n, c, h, w, oc, kh, kw, pads, dilations
SHIFT_SHAPES = [
    (4, 64, 56, 56, 64, 3, 3, (1, 1, 1, 1), (1, 1)),     # ResNet-50 stage 1 (largest patch: 256 rows)
    (2, 128, 28, 28, 128, 3, 3, (1, 1, 1, 1), (1, 1)),   # stage 2: one 128-wide N tile
    (2, 128, 10, 10, 256, 3, 3, (1, 1, 1, 1), (1, 1)),   # two 128-wide N tiles
    (3, 64, 17, 23, 100, 3, 3, (1, 1, 1, 1), (1, 1)),    # ragged N (2 tiles of 64), odd extents
    (2, 64, 9, 11, 256, 3, 3, (0, 2, 1, 0), (1, 1)),     # asymmetric pads, 4 N tiles
    (2, 128, 12, 12, 64, 3, 3, (2, 2, 2, 2), (2, 2)),    # dilation 2
    (1, 64, 8, 8, 64, 5, 5, (2, 2, 2, 2), (1, 1)),       # 25 K slabs: not resident, falls back
    (2, 64, 3, 5, 64, 3, 3, (1, 1, 1, 1), (1, 1)),       # whole images smaller than a tile
    (1, 64, 6, 120, 64, 3, 3, (1, 1, 1, 1), (1, 1)),     # patch over 256 rows: falls back
]


def _shift_case(shape, x_zp, seed):
    n, c, h, w, oc, kh, kw, p, d = shape
    rng = np.random.default_rng(seed)
    return W.random_qconv(rng, n, c, h, w, oc, kh, kw, (1, 1), p, d, x_zp=x_zp)


@pytest.mark.parametrize("shape", SHIFT_SHAPES)
@pytest.mark.parametrize("formula", [O.R1, O.R2])
@pytest.mark.parametrize("x_zp", [0, 93])
def test_shifted_patch_convs(cuda_dev, shape, formula, x_zp):
    case = _shift_case(shape, x_zp, sum(shape[:7]) + formula + x_zp)
    for lay in (("NHWC", "NHWC"), ("NCHW", "NHWC"), ("NHWC", "NCHW")):
        y, _ = run_qconv(cuda_dev, case, formula, lay[0], lay[1])
        ref = oracle_qconv(case, formula, lay[1])
        assert np.array_equal(y, ref), f"{lay}: {(y != ref).sum()} / {y.size} mismatches"


def test_shifted_patch_is_selected(cuda_dev):
    """NHWC input with x_zp = 0 needs no workspace on the im2col path; the
    shifted-patch path copies it into a padded buffer ([n][h+2][w+2][c])."""
    case = _shift_case(SHIFT_SHAPES[0], 0, 5)
    _, op = run_qconv(cuda_dev, case, O.R2, "NHWC", "NHWC")
    n, c, h, w = case.x.shape
    assert op.workspace_size() == n * (h + 2) * (w + 2) * c


@pytest.mark.parametrize("relu", [False, True])
def test_shifted_patch_fused_relu_and_add(cuda_dev, relu):
    import ctypes as C
    from nnr_b200 import ops
    from nnr_b200._lib import check, lib
    case = _shift_case(SHIFT_SHAPES[3], 0, 11)
    case.y_zp = 40
    op = ops.QLinearConv(case.x.shape, case.w, case.w_scale, case.w_zp, case.bias, case.x_scale, case.x_zp,
                         case.y_scale, case.y_zp, pads=case.pads, in_layout="NHWC", out_layout="NHWC", requant=O.R2,
                         fused_relu=relu)
    conv = oracle_qconv(case, O.R2, out_layout="NHWC", fused_relu=relu)
    rng = np.random.default_rng(3)
    res = rng.integers(0, 256, size=conv.shape).astype(np.uint8)
    rs, rz, ys, yz = 0.037, 101, 0.05, 7
    ref = O.qlinearadd_u8(conv, case.y_scale, case.y_zp, res, rs, rz, ys, yz)
    x = torch.from_numpy(_to_nhwc(case.x)).to(cuda_dev)
    r = torch.from_numpy(res).to(cuda_dev)
    y = torch.empty(conv.shape, dtype=torch.uint8, device=cuda_dev)
    ws = torch.empty(max(op.workspace_size(), 1), dtype=torch.uint8, device=cuda_dev)
    check(lib.nnrcu_qlinearconv_run_add(op._op, C.c_void_p(x.data_ptr()), C.c_void_p(r.data_ptr()), rs, rz, ys, yz,
                                        C.c_void_p(y.data_ptr()), C.c_void_p(ws.data_ptr()),
                                        C.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert np.array_equal(y.cpu().numpy(), ref)


def test_padded_output_feeds_padded_input(cuda_dev):
    """1x1 conv writing into the interior of an x_zp-bordered buffer, read as is
    by a shifted-patch 3x3 conv (nnrcu_qlinearconv_set_padded_io): both outputs
    equal the unpadded chain's, and the border keeps its fill."""
    from nnr_b200 import ops
    rng = np.random.default_rng(21)
    n, c, h, w = 2, 64, 20, 17
    c1 = W.random_qconv(rng, n, c, h, w, 64, 1, 1, (1, 1), (0, 0, 0, 0), x_zp=0)
    c1.y_zp = 57
    y1 = oracle_qconv(c1, O.R2, out_layout="NHWC")
    c2 = W.random_qconv(rng, n, 64, h, w, 128, 3, 3, (1, 1), (1, 1, 1, 1))
    c2.x = np.ascontiguousarray(y1.transpose(0, 3, 1, 2))
    c2.x_scale, c2.x_zp = c1.y_scale, c1.y_zp
    y2 = oracle_qconv(c2, O.R2, out_layout="NHWC")

    def mk(cs):
        return ops.QLinearConv(cs.x.shape, cs.w, cs.w_scale, cs.w_zp, cs.bias, cs.x_scale, cs.x_zp, cs.y_scale,
                               cs.y_zp, pads=cs.pads, in_layout="NHWC", out_layout="NHWC", requant=O.R2)
    op1, op2 = mk(c1), mk(c2)
    pads = op2.input_padding()
    assert pads == (1, 1, 1, 1)
    assert mk(c1).input_padding() == (0, 0, 0, 0)
    op1.set_padded_io(out_pads=pads)
    op2.set_padded_io(in_padded=True)
    buf = torch.full((n, h + 2, w + 2, 64), c1.y_zp, dtype=torch.uint8, device=cuda_dev)
    op1.exec(torch.from_numpy(_to_nhwc(c1.x)).to(cuda_dev), y=buf)
    out = op2.exec(buf)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    b = buf.cpu().numpy()
    assert np.array_equal(b[:, 1:h + 1, 1:w + 1, :], y1)
    border = np.ones(b.shape[:3], bool)
    border[:, 1:h + 1, 1:w + 1] = False
    assert (b[border] == c1.y_zp).all()
    assert np.array_equal(out.cpu().numpy(), y2)


# ------------------------------------------------------------------ depthwise (exec_dw_int8_nhwc)
DW_SHAPES = [
    # n, c, h, w, k, stride, pads, dilation, x_zp, w_zp, y_zp
    (2, 32, 14, 14, 3, 1, (1, 1, 1, 1), 1, 37, 0, 5),
    (4, 144, 28, 28, 3, 2, (1, 1, 1, 1), 1, 128, 0, 128),
    (1, 96, 13, 11, 3, 2, (1, 0, 1, 0), 1, 131, -2, 200),
    (2, 48, 9, 9, 5, 1, (2, 2, 2, 2), 2, 200, 0, 9),
    (1, 20, 6, 7, 3, 1, (1, 1, 1, 1), 1, 10, 3, 5),   # C % 16 != 0: the per-element kernel
    (3, 64, 10, 12, 3, 1, (0, 1, 1, 0), 1, 255, 0, 0),  # asymmetric pads, x_zp 255 (dp4a kernel)
    (1, 16, 5, 5, 7, 1, (3, 3, 3, 3), 1, 0, 0, 128),    # 49 taps: 13 groups of four, x_zp 0
]


@pytest.mark.parametrize("shape", DW_SHAPES)
@pytest.mark.parametrize("in_layout", ["NHWC", "NCHW"])
@pytest.mark.parametrize("fused_relu", [False, True])
def test_depthwise_bit_exact(cuda_dev, shape, in_layout, fused_relu):
    """Depthwise QLinearConv (group = C) against the restatement of nnr's
    exec_dw_int8_nhwc (pinned to nnr's kernels in test_oracle.py); a fused
    Relu leaves the result unchanged, as in nnr's depthwise path."""
    from nnr_b200 import ops
    n, c, h, w, k, s, pads, d, xz, wz, yz = shape
    rng = np.random.default_rng(c + 7 * h)
    x = rng.integers(0, 256, size=(n, h, w, c)).astype(np.uint8)
    wt = rng.integers(-127, 128, size=(c, 1, k, k)).astype(np.int8)
    ws = rng.uniform(0.002, 0.01, size=c).astype(np.float32)
    b = rng.integers(-2000, 2001, size=c).astype(np.int32)
    want = O.qdwconv_u8_nhwc(x, wt, ws, b, 0.02, xz, 0.4, yz, w_zp=wz, strides=(s, s), pads=pads, dilations=(d, d))
    op = ops.QLinearConv((n, c, h, w), wt, ws, np.int8(wz), b, 0.02, xz, 0.4, yz, strides=(s, s), pads=pads,
                         dilations=(d, d), group=c, in_layout=in_layout, out_layout="NHWC", fused_relu=fused_relu)
    xin = x if in_layout == "NHWC" else np.ascontiguousarray(x.transpose(0, 3, 1, 2))
    y = op.exec(torch.from_numpy(xin).to(cuda_dev))
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    got = y.cpu().numpy()
    assert np.array_equal(got, want), f"{(got != want).sum()} of {want.size} differ"


def test_depthwise_nchw_output_declined(cuda_dev):
    """nnr takes its int8 depthwise kernel for NHWC outputs only; an NCHW
    output is declined (NNRCU_ERR_UNSUPPORTED)."""
    from nnr_b200 import ops
    from nnr_b200._lib import NnrcuError
    wt = np.ones((16, 1, 3, 3), np.int8)
    with pytest.raises(NnrcuError, match="NHWC"):
        ops.QLinearConv((1, 16, 8, 8), wt, np.float32(0.01), None, None, 0.1, 0, 0.1, 0, pads=(1, 1, 1, 1), group=16,
                        in_layout="NHWC", out_layout="NCHW")


@pytest.mark.parametrize("shape", [
    # n, c, h, w, oc, k, stride, group
    (2, 64, 14, 14, 128, 3, 1, 4),      # 4 groups of 16 -> 32
    (1, 128, 9, 11, 64, 3, 2, 32),      # 32 groups (ResNeXt-like), stride 2
    (2, 24, 8, 8, 48, 1, 1, 3),         # 1x1, 3 groups
    (1, 32, 7, 7, 64, 3, 1, 32),        # group = C with a channel multiplier of 2 (not depthwise)
])
@pytest.mark.parametrize("layouts", [("NCHW", "NCHW"), ("NHWC", "NHWC")])
@pytest.mark.parametrize("x_zp", [0, 111])
def test_grouped_qlinearconv(cuda_dev, shape, layouts, x_zp):
    """Grouped (not depthwise) QLinearConv: nnr's VNNI im2col path, R1, per
    group. Reference: the oracle per group on the group's input and output
    channels, concatenated."""
    n, c, h, w, oc, k, s, g = shape
    rng = np.random.default_rng(c + oc + g)
    x = rng.integers(0, 256, size=(n, c, h, w)).astype(np.uint8)
    wt = rng.integers(-127, 128, size=(oc, c // g, k, k)).astype(np.int8)
    ws = rng.uniform(0.002, 0.01, size=oc).astype(np.float32)
    b = rng.integers(-2000, 2001, size=oc).astype(np.int32)
    p = k // 2
    cg, og = c // g, oc // g
    parts = [O.qlinearconv(x[:, i * cg:(i + 1) * cg], wt[i * og:(i + 1) * og], ws[i * og:(i + 1) * og],
                           b[i * og:(i + 1) * og], 0.02, x_zp, 0.3, 9, strides=(s, s), pads=(p,) * 4, formula=O.R1)
             for i in range(g)]
    ref = np.concatenate(parts, axis=1)
    from nnr_b200 import ops
    op = ops.QLinearConv((n, c, h, w), wt, ws, None, b, 0.02, x_zp, 0.3, 9, strides=(s, s), pads=(p,) * 4, group=g,
                         in_layout=layouts[0], out_layout=layouts[1])
    xin = x if layouts[0] == "NCHW" else _to_nhwc(x)
    y = op.exec(torch.from_numpy(np.ascontiguousarray(xin)).to(cuda_dev))
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    got = y.cpu().numpy()
    if layouts[1] == "NHWC":
        got = got.transpose(0, 3, 1, 2)
    assert np.array_equal(got, ref), f"{(got != ref).sum()} of {ref.size} differ"
