"""Generates the golden QLinearConv fixtures in this directory from nnr's own
int8 direct-convolution kernel (oracle/_ref/libnnr_ref_int8.so, compiled from
the nnr sources by `make -C oracle ref`) on an AVX-512 VNNI host.

Each fixture qconv_<name>.npz holds the inputs, the attributes, nnr's raw
int32 dot products (before zero-point compensation) and nnr's u8 output of
exec_direct_int8 (R1). The depthwise fixtures qdw_<name>.npz hold nnr's
exec_dw_int8_nhwc kernels' u8 output (depthwise_int8_avx512.h). Run from the
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
    sys.exit(main() or main_dw())
