"""Seeded synthetic inputs for the benchmark configurations.

Generator: numpy.random.default_rng(seed) (PCG64), tensors drawn in the
order the configuration lists them. "U{a..b}" is inclusive integers
(rng.integers(a, b + 1)); "U(a,b)" is rng.uniform; "N(mu, sigma)" is
rng.normal cast to float32. The reference publishes no dataset for these
configs; these arrays stand in for them with the stated shapes and
distributions.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np


@dataclass
class QConvCase:
    x: np.ndarray            # u8 NCHW
    w: np.ndarray            # s8 OIHW
    w_scale: np.ndarray      # f32 [oc]
    w_zp: np.ndarray         # s8 [oc]
    bias: np.ndarray         # s32 [oc]
    x_scale: float
    x_zp: int
    y_scale: float
    y_zp: int
    strides: tuple = (1, 1)
    pads: tuple = (1, 1, 1, 1)
    dilations: tuple = (1, 1)

    @property
    def ops(self) -> int:
        n, c, h, w = self.x.shape
        oc, _, kh, kw = self.w.shape
        oh = (h + self.pads[0] + self.pads[2] - kh) // self.strides[0] + 1
        ow = (w + self.pads[1] + self.pads[3] - kw) // self.strides[1] + 1
        return 2 * n * oc * oh * ow * c * kh * kw


def config2_qlinearconv(n: int = 32, seed: int = 1) -> QConvCase:
    """QLinearConv x u8 [32,256,14,14], w s8 [256,256,3,3]."""
    rng = np.random.default_rng(seed)
    x = rng.integers(0, 256, size=(32, 256, 14, 14)).astype(np.uint8)
    w = rng.integers(-127, 128, size=(256, 256, 3, 3)).astype(np.int8)
    w_scale = rng.uniform(0.002, 0.01, size=256).astype(np.float32)
    w_zp = np.zeros(256, np.int8)
    bias = rng.integers(-2000, 2001, size=256).astype(np.int32)
    if n != 32:
        x = x[:n].copy()
    return QConvCase(x, w, w_scale, w_zp, bias, 0.02, 128, 0.05, 128)


@dataclass
class MatMulCase:
    a_u8: np.ndarray
    b_s8: np.ndarray
    a_scale: float = 0.03
    a_zp: int = 128
    b_scale: float = 0.004
    b_zp: int = 0
    y_scale: float = 0.1
    y_zp: int = 128
    a_f32: np.ndarray = field(default=None)
    b_f32: np.ndarray = field(default=None)
    c_f32: np.ndarray = field(default=None)


def config3_matmul(seed: int = 2) -> MatMulCase:
    """QLinearMatMul [4096,768]x[768,3072] and fp32 Gemm of the same shape."""
    rng = np.random.default_rng(seed)
    a = rng.integers(0, 256, size=(4096, 768)).astype(np.uint8)
    b = rng.integers(-127, 128, size=(768, 3072)).astype(np.int8)
    af = rng.normal(0.0, 1.0, size=(4096, 768)).astype(np.float32)
    bf = rng.normal(0.0, 0.02, size=(768, 3072)).astype(np.float32)
    cf = rng.normal(0.0, 0.01, size=3072).astype(np.float32)
    return MatMulCase(a, b, a_f32=af, b_f32=bf, c_f32=cf)


@dataclass
class ConvF32Case:
    x: np.ndarray
    w: np.ndarray
    bias: np.ndarray
    pads: tuple = (1, 1, 1, 1)
    strides: tuple = (1, 1)


def config1_conv_relu(seed: int = 0) -> ConvF32Case:
    """fp32 Conv+Relu X[1,64,56,56], W[64,64,3,3], pads 1."""
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1.0, 1.0, size=(1, 64, 56, 56)).astype(np.float32)
    w = rng.normal(0.0, math.sqrt(2.0 / 576.0), size=(64, 64, 3, 3)).astype(np.float32)
    b = rng.normal(0.0, 0.01, size=64).astype(np.float32)
    return ConvF32Case(x, w, b)


def random_qconv(rng: np.random.Generator, n, c, h, w, oc, kh, kw, strides=(1, 1), pads=(0, 0, 0, 0),
                 dilations=(1, 1), x_zp=None, y_zp=None, per_channel=True, bias=True) -> QConvCase:
    """A random QLinearConv problem for parity sweeps."""
    x = rng.integers(0, 256, size=(n, c, h, w)).astype(np.uint8)
    wt = rng.integers(-127, 128, size=(oc, c, kh, kw)).astype(np.int8)
    ws = rng.uniform(0.002, 0.01, size=oc if per_channel else 1).astype(np.float32)
    b = rng.integers(-2000, 2001, size=oc).astype(np.int32) if bias else None
    xz = int(rng.integers(0, 256)) if x_zp is None else x_zp
    yz = int(rng.integers(0, 256)) if y_zp is None else y_zp
    # y_scale chosen so that outputs span the u8 range instead of saturating
    y_scale = float(0.02 * 0.006 * 40.0 * math.sqrt(c * kh * kw))
    return QConvCase(x, wt, ws, np.zeros(oc, np.int8), b, 0.02, xz, y_scale, yz, tuple(strides), tuple(pads),
                     tuple(dilations))
