"""Generates the golden QLinearConv fixtures in this directory from nnr's own
int8 direct-convolution kernel (oracle/_ref/libnnr_ref_int8.so, compiled from
the nnr sources by `make -C oracle ref`) on an AVX-512 VNNI host.

Each fixture qconv_<name>.npz holds the inputs, the attributes, nnr's raw
int32 dot products (before zero-point compensation) and nnr's u8 output of
exec_direct_int8 (R1). The depthwise fixtures qdw_<name>.npz hold nnr's
exec_dw_int8_nhwc kernels' u8 output (depthwise_int8_avx512.h); the
first-layer fixtures qfirst_<name>.npz nnr's exec_first_layer_int8 output (R3,
conv_first_layer_int8_avx512.h). Run from the
repository root:

    make -C oracle ref && python tests/golden/make_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import zlib

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle import oracle as O  # noqa: E402

CASES = {
    # name: (n, c, h, w, oc, k, stride, pad, x_zp, y_zp, y_scale, fused_relu)
    "c64_14x14_k3": (1, 64, 14, 14, 64, 3, 1, 1, 128, 128, 1.3, False),
    "c32_9x11_k3_s2": (2, 32, 9, 11, 48, 3, 2, 1, 77, 10, 0.9, True),
    "c16_7x7_k1": (1, 16, 7, 7, 32, 1, 1, 0, 0, 200, 0.2, False),
    "c8_12x12_k5_p2": (1, 8, 12, 12, 16, 5, 1, 2, 255, 0, 0.6, True),
}


# depthwise (qdw_<name>.npz): nnr's exec_dw_int8_nhwc kernels on NHWC u8
DW_CASES = {
    # name: (n, c, h, w, k, stride, pad, dilation, x_zp, w_zp, y_zp)
    "c32_14x14_k3": (2, 32, 14, 14, 3, 1, 1, 1, 37, 0, 5),
    "c64_15x17_k3_s2": (1, 64, 15, 17, 3, 2, 1, 1, 128, 3, 0),
    "c48_9x9_k5_d2": (2, 48, 9, 9, 5, 1, 2, 2, 200, 0, 9),
}


# first-layer (qfirst_<name>.npz): nnr's exec_first_layer_int8 kernel (R3;
# conv_first_layer_int8_avx512.h), NCHW u8 input with at most 4 channels;
# output widths that are not multiples of 16 exercise the NCHW scalar tail
FIRST_CASES = {
    # name: (n, c, h, w, oc, k, stride, pad, x_zp, y_zp, y_scale, fused_relu, out_layout, w_scale)
    # (w_scale None: random per channel; 50 with x_scale 0.02 and y_scale 2
    # makes acc * cs * inv_y a multiple of 1/2, where the body's
    # fma(f, inv_y, y_zp) and the tail's rne(f * inv_y) + y_zp round ties
    # differently for an odd y_zp)
    "c3_38x38_k7_s2_nchw": (1, 3, 38, 38, 24, 7, 2, 3, 128, 3, 0.5, False, "NCHW", None),
    "c3_30x46_k7_s2_nhwc_relu": (2, 3, 30, 46, 32, 7, 2, 3, 114, 9, 0.4, True, "NHWC", None),
    "c4_21x21_k3_nchw_relu": (1, 4, 21, 21, 20, 3, 1, 1, 0, 17, 0.3, True, "NCHW", None),
    "c3_16x16_k3_s2_nchw": (2, 3, 16, 16, 16, 3, 2, 1, 255, 128, 0.25, False, "NCHW", None),
    "c3_20x21_k3_nchw_ties": (1, 3, 20, 21, 16, 3, 1, 1, 0, 7, 2.0, False, "NCHW", 50.0),
}


def main_first() -> int:
    for name, (n, c, h, w, oc, k, s, p, xz, yz, ys, post, lay, wsc) in FIRST_CASES.items():
        rng = np.random.default_rng(zlib.crc32(("first" + name).encode()))
        x = rng.integers(0, 256, size=(n, c, h, w)).astype(np.uint8)
        if wsc is None:
            wt = rng.integers(-127, 128, size=(oc, c, k, k)).astype(np.int8)
            ws = rng.uniform(0.002, 0.01, size=oc).astype(np.float32)
            b = rng.integers(-2000, 2001, size=oc).astype(np.int32)
        else:
            x = rng.integers(0, 24, size=(n, c, h, w)).astype(np.uint8)
            wt = rng.integers(-3, 4, size=(oc, c, k, k)).astype(np.int8)
            ws = np.full(oc, wsc, np.float32)
            b = rng.integers(-40, 41, size=oc).astype(np.int32)
        y = O.ref_qconv_first_layer(x, wt, ws, b, 0.02, xz, ys, yz, strides=(s, s), pads=(p, p), has_post=post,
                                    out_layout=lay)
        if y is None:
            print("nnr's kernel declined (no AVX-512 VNNI on this host)", file=sys.stderr)
            return 1
        np.savez_compressed(HERE / f"qfirst_{name}.npz", x=x, w=wt, w_scale=ws, bias=b,
                            attrs=np.array([s, p, xz, yz, int(post), int(lay == "NHWC")], np.int64),
                            scales=np.array([0.02, ys], np.float32), y=y)
        print(name, y.shape, "saturated", float(np.mean((y == 0) | (y == 255))))
    return 0


def main_dw() -> int:
    for name, (n, c, h, w, k, s, p, d, xz, wz, yz) in DW_CASES.items():
        rng = np.random.default_rng(zlib.crc32(("dw" + name).encode()))
        x = rng.integers(0, 256, size=(n, h, w, c)).astype(np.uint8)
        wt = rng.integers(-127, 128, size=(c, 1, k, k)).astype(np.int8)
        ws = rng.uniform(0.002, 0.01, size=c).astype(np.float32)
        b = rng.integers(-2000, 2001, size=c).astype(np.int32)
        y = O.ref_qdwconv_nhwc(x, wt, ws, b, 0.02, xz, 0.4, yz, w_zp=wz, strides=(s, s), pads=(p,) * 4,
                               dilations=(d, d))
        if y is None:
            print("nnr's kernel declined (no AVX-512 VNNI on this host)", file=sys.stderr)
            return 1
        np.savez_compressed(HERE / f"qdw_{name}.npz", x=x, w=wt, w_scale=ws, bias=b,
                            attrs=np.array([s, p, d, xz, wz, yz], np.int64), scales=np.array([0.02, 0.4], np.float32),
                            y=y)
        print(name, y.shape, "saturated", float(np.mean((y == 0) | (y == 255))))
    return 0


def main() -> int:
    if O.ref_lib() is None:
        print("oracle/_ref/libnnr_ref_int8.so not built: run `make -C oracle ref`", file=sys.stderr)
        return 1
    for name, (n, c, h, w, oc, k, s, p, xz, yz, ys, post) in CASES.items():
        rng = np.random.default_rng(zlib.crc32(name.encode()))
        x = rng.integers(0, 256, size=(n, c, h, w)).astype(np.uint8)
        wt = rng.integers(-127, 128, size=(oc, c, k, k)).astype(np.int8)
        ws = rng.uniform(0.002, 0.01, size=oc).astype(np.float32)
        b = rng.integers(-2000, 2001, size=oc).astype(np.int32)
        r = O.ref_qlinearconv_direct(x, wt, ws, b, 0.02, xz, ys, yz, strides=(s, s), pads=(p,) * 4, has_post=post,
                                     want_raw=True)
        if r is None:
            print("nnr's kernel declined (no AVX-512 VNNI on this host)", file=sys.stderr)
            return 1
        y, raw = r
        np.savez_compressed(HERE / f"qconv_{name}.npz", x=x, w=wt, w_scale=ws, bias=b,
                            attrs=np.array([s, p, xz, yz, int(post)], np.int64),
                            scales=np.array([0.02, ys], np.float32), raw=raw, y=y)
        print(name, y.shape, "saturated", float(np.mean((y == 0) | (y == 255))))
    return 0


if __name__ == "__main__":
    sys.exit(main() or main_dw() or main_first())
