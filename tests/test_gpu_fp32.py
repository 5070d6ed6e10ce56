"""fp32 Conv / Gemm / MatMul on the device vs the oracle.

Tolerance: max |y - ref| / rms(ref) <= 1e-4, i.e. the
max error normalised by the output's L2 norm per element. The dense paths run
as split-bf16 (3 products, fp32 accumulation) on the tensor cores.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from nnr_b200 import workloads as W

pytestmark = pytest.mark.gpu

TOL = 1e-4


def rel_err(y, ref):
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    return float(np.max(np.abs(y.astype(np.float64) - ref))) / max(rms, 1e-30)


def run_conv(dev, x, w, bias, in_layout="NCHW", out_layout="NCHW", residual=None, **kw):
    from nnr_b200 import ops
    shape = x.shape if in_layout == "NCHW" else (x.shape[0], x.shape[3], x.shape[1], x.shape[2])
    op = ops.Conv(shape, w, bias, in_layout=in_layout, out_layout=out_layout, **kw)
    r = None if residual is None else torch.from_numpy(residual).to(dev)
    y = op.exec(torch.from_numpy(x).to(dev), residual=r)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    return y.cpu().numpy()


def test_config1_conv_relu(cuda_dev):
    c = W.config1_conv_relu()
    y = run_conv(cuda_dev, c.x, c.w, c.bias, pads=c.pads, post="Relu")
    ref = O.conv_f32(c.x, c.w, c.bias, pads=c.pads, post=1)
    assert rel_err(y, ref) <= TOL


@pytest.mark.parametrize("case", [
    dict(n=2, c=64, h=28, w=28, oc=128, k=3, s=2, p=1, post="Clip"),
    dict(n=2, c=128, h=20, w=18, oc=64, k=3, s=1, p=1, post="Relu"),   # hardware im2col, 2 slabs per tap
    dict(n=2, c=16, h=20, w=20, oc=96, k=1, s=1, p=0, post="Clip"),    # 1x1, 64-byte K slabs (MobileNet expand)
    dict(n=1, c=40, h=14, w=14, oc=24, k=1, s=1, p=0, post=None),      # 1x1, channels padded to 64
    dict(n=2, c=3, h=33, w=31, oc=32, k=3, s=2, p=1, post="Clip"),     # explicit im2col, K 27 -> 32
    dict(n=1, c=96, h=14, w=14, oc=160, k=1, s=1, p=0, post=None),      # 1x1 -> TMA A path (NHWC)
    dict(n=2, c=3, h=32, w=32, oc=32, k=3, s=2, p=1, post="HardSwish"),  # stem
    dict(n=1, c=24, h=9, w=9, oc=40, k=5, s=1, p=2, post="Sigmoid"),
    dict(n=1, c=8, h=7, w=7, oc=8, k=3, s=1, p=1, post="LeakyRelu"),
    dict(n=1, c=16, h=6, w=6, oc=16, k=3, s=1, p=0, post="Tanh"),
])
@pytest.mark.parametrize("layout", ["NCHW", "NHWC"])
def test_conv_shapes(cuda_dev, case, layout):
    rng = np.random.default_rng(case["c"] * 31 + case["oc"])
    x = rng.uniform(-1, 1, size=(case["n"], case["c"], case["h"], case["w"])).astype(np.float32)
    w = rng.normal(0, np.sqrt(2.0 / (case["c"] * case["k"] ** 2)),
                   size=(case["oc"], case["c"], case["k"], case["k"])).astype(np.float32)
    b = rng.normal(0, 0.1, size=case["oc"]).astype(np.float32)
    p = case["p"]
    post_id = {None: 0, "Relu": 1, "Clip": 2, "HardSwish": 3, "Sigmoid": 4, "LeakyRelu": 5, "Tanh": 6}[case["post"]]
    pa, pb = (0.0, 6.0) if case["post"] == "Clip" else ((0.1, 0.0) if case["post"] == "LeakyRelu" else (0.0, 0.0))
    xin = x if layout == "NCHW" else np.ascontiguousarray(x.transpose(0, 2, 3, 1))
    y = run_conv(cuda_dev, xin, w, b, layout, layout, strides=(case["s"],) * 2, pads=(p,) * 4, post=case["post"],
                 post_a=pa, post_b=pb)
    ref = O.conv_f32(x, w, b, strides=(case["s"],) * 2, pads=(p,) * 4, post=post_id, post_a=pa, post_b=pb,
                     out_layout=layout)
    assert rel_err(y, ref) <= TOL


@pytest.mark.parametrize("s", [1, 2])
@pytest.mark.parametrize("layout", ["NCHW", "NHWC"])
@pytest.mark.parametrize("hw", [(28, 28), (13, 15)])
def test_depthwise_clip(cuda_dev, s, layout, hw):
    """MobileNetV2 depthwise 3x3 + ReLU6 (Clip(0,6)); 13x15 leaves partial
    four-output strips at the row ends."""
    rng = np.random.default_rng(s)
    c = 96
    x = rng.normal(0, 1, size=(2, c) + hw).astype(np.float32)
    w = rng.normal(0, 0.3, size=(c, 1, 3, 3)).astype(np.float32)
    b = rng.normal(0, 0.1, size=c).astype(np.float32)
    xin = x if layout == "NCHW" else np.ascontiguousarray(x.transpose(0, 2, 3, 1))
    y = run_conv(cuda_dev, xin, w, b, layout, layout, strides=(s, s), pads=(1, 1, 1, 1), group=c, post="Clip",
                 post_a=0.0, post_b=6.0)
    ref = O.conv_f32(x, w, b, strides=(s, s), pads=(1, 1, 1, 1), group=c, post=2, post_a=0.0, post_b=6.0,
                     out_layout=layout)
    assert rel_err(y, ref) <= TOL


@pytest.mark.parametrize("shape", [(2, 64, 14, 14, 128, 3, 1, 4), (1, 128, 9, 11, 64, 3, 2, 32),
                                   (1, 32, 7, 7, 64, 3, 1, 32)])
@pytest.mark.parametrize("layout", ["NCHW", "NHWC"])
def test_grouped_conv(cuda_dev, shape, layout):
    """Grouped (not depthwise) fp32 Conv + Relu against the fp64 grouped
    restatement (nnr's grouped im2col path computes each group on its own)."""
    n, c, h, w_, oc, k, s, g = shape
    rng = np.random.default_rng(oc + g)
    x = rng.normal(0, 1, size=(n, c, h, w_)).astype(np.float32)
    w = rng.normal(0, 0.2, size=(oc, c // g, k, k)).astype(np.float32)
    b = rng.normal(0, 0.1, size=oc).astype(np.float32)
    p = k // 2
    xin = x if layout == "NCHW" else np.ascontiguousarray(x.transpose(0, 2, 3, 1))
    y = run_conv(cuda_dev, xin, w, b, layout, layout, strides=(s, s), pads=(p,) * 4, group=g, post="Relu")
    ref = O.conv_f32(x, w, b, strides=(s, s), pads=(p,) * 4, group=g, post=1, out_layout=layout)
    assert rel_err(y, ref) <= TOL


@pytest.mark.parametrize("c,oc,hw,s,k", [(40, 24, 15, 1, 3), (96, 24, 28, 2, 3), (64, 32, 9, 1, 5), (144, 144, 14, 1, 3)])
def test_depthwise_to_planes_chain(cuda_dev, c, oc, hw, s, k):
    """Depthwise -> 1x1 through pre-split planes (nnrcu_conv_f32_run_to_planes
    then nnrcu_conv_f32_run_planes) is bit-identical to the two convs through
    nnrcu_conv_f32_run, including channel counts that need padded planes, and
    twice in a row over the same planes buffer (poisoned first)."""
    import ctypes as C
    from nnr_b200 import ops
    from nnr_b200._lib import call
    rng = np.random.default_rng(c + oc + hw)
    n = 3
    x = rng.uniform(-1, 1, size=(n, hw, hw, c)).astype(np.float32)
    wd = rng.normal(0, 0.3, size=(c, 1, k, k)).astype(np.float32)
    bd = rng.normal(0, 0.1, size=c).astype(np.float32)
    wp = rng.normal(0, 0.2, size=(oc, c, 1, 1)).astype(np.float32)
    bp = rng.normal(0, 0.1, size=oc).astype(np.float32)
    p = k // 2
    dw = ops.Conv((n, c, hw, hw), wd, bd, strides=(s, s), pads=(p,) * 4, group=c, in_layout="NHWC",
                  out_layout="NHWC", post="Clip", post_a=0.0, post_b=6.0)
    oh = (hw + 2 * p - k) // s + 1
    pj = ops.Conv((n, c, oh, oh), wp, bp, in_layout="NHWC", out_layout="NHWC")
    xd = torch.from_numpy(x).to(cuda_dev)
    mid = dw.exec(xd)
    want = pj.exec(mid).cpu().numpy()
    cs = C.c_int()
    call("nnrcu_conv_f32_plane_stride", pj._op, C.byref(cs))
    assert cs.value >= c and cs.value % 8 == 0
    pix = n * oh * oh
    planes = torch.empty(2 * pix * cs.value, dtype=torch.int16, device=cuda_dev)
    y = torch.empty_like(torch.from_numpy(want)).to(cuda_dev)
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(2):
        planes.fill_(-1)  # NaN bit patterns in every padding channel unless they are rewritten
        y.fill_(float("nan"))
        hi, lo = planes.data_ptr(), planes.data_ptr() + pix * cs.value * 2
        call("nnrcu_conv_f32_run_to_planes", dw._op, C.c_void_p(xd.data_ptr()), C.c_void_p(hi), C.c_void_p(lo),
             cs.value, st)
        call("nnrcu_conv_f32_run_planes", pj._op, C.c_void_p(hi), C.c_void_p(lo), C.c_void_p(y.data_ptr()), None, st)
        torch.cuda.synchronize()
        assert ops.device_status() == 0
        got = y.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_planes_declined_for_non_1x1(cuda_dev):
    import ctypes as C
    from nnr_b200 import ops
    from nnr_b200._lib import lib
    w = np.zeros((16, 16, 3, 3), np.float32)
    op = ops.Conv((1, 16, 8, 8), w, None, pads=(1, 1, 1, 1), in_layout="NHWC", out_layout="NHWC")
    cs = C.c_int()
    assert lib.nnrcu_conv_f32_plane_stride(op._op, C.byref(cs)) == -2


def test_conv_residual_add(cuda_dev):
    """Projection conv followed by the residual Add (MobileNetV2 block output)."""
    rng = np.random.default_rng(9)
    x = rng.normal(0, 1, size=(2, 14, 14, 64)).astype(np.float32)
    w = rng.normal(0, 0.1, size=(32, 64, 1, 1)).astype(np.float32)
    r = rng.normal(0, 1, size=(2, 14, 14, 32)).astype(np.float32)
    y = run_conv(cuda_dev, x, w, None, "NHWC", "NHWC", residual=r)
    ref = O.conv_f32(x, w, None, in_layout="NHWC", out_layout="NHWC", residual=r)
    assert rel_err(y, ref) <= TOL


def test_config3_gemm_f32(cuda_dev):
    from nnr_b200 import ops
    c = W.config3_matmul()
    op = ops.Gemm(4096, c.b_f32, c.c_f32)
    y = op.exec(torch.from_numpy(c.a_f32).to(cuda_dev))
    torch.cuda.synchronize()
    y = y.cpu().numpy()
    for r0 in (0, 2048, 4000):
        ref = O.gemm_f32(c.a_f32, c.b_f32, c.c_f32, rows=(r0, r0 + 96))
        assert rel_err(y[r0:r0 + 96], ref) <= TOL


@pytest.mark.parametrize("ta,tb,alpha,beta,cshape,post", [
    (0, 0, 1.0, 1.0, "row", "Relu"),
    (1, 0, 0.5, 2.0, "full", None),
    (0, 1, 1.0, 0.0, None, "Sigmoid"),
    (1, 1, -1.5, 1.0, "row", "Tanh"),
])
def test_gemm_variants(cuda_dev, ta, tb, alpha, beta, cshape, post):
    from nnr_b200 import ops
    rng = np.random.default_rng(ta * 2 + tb)
    m, k, n = 200, 72, 130
    a = rng.normal(0, 1, size=(k, m) if ta else (m, k)).astype(np.float32)
    b = rng.normal(0, 0.1, size=(n, k) if tb else (k, n)).astype(np.float32)
    cm = None if cshape is None else rng.normal(0, 1, size=(n,) if cshape == "row" else (m, n)).astype(np.float32)
    op = ops.Gemm(m, b, cm, alpha, beta, ta, tb, post=post)
    y = op.exec(torch.from_numpy(a).to(cuda_dev))
    torch.cuda.synchronize()
    post_id = {None: 0, "Relu": 1, "Sigmoid": 4, "Tanh": 6}[post]
    ref = O.gemm_f32(a, b, cm, alpha, beta, ta, tb, post=post_id)
    assert rel_err(y.cpu().numpy(), ref) <= TOL


def test_matmul_small_k(cuda_dev):
    from nnr_b200 import ops
    rng = np.random.default_rng(1)
    a = rng.normal(0, 1, size=(300, 24)).astype(np.float32)
    b = rng.normal(0, 1, size=(24, 50)).astype(np.float32)
    op = ops.MatMul(300, b)
    y = op.exec(torch.from_numpy(a).to(cuda_dev))
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), O.gemm_f32(a, b, beta=0.0)) <= TOL
