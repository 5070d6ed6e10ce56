"""Parity of the device glue operators around the int8 convs (MaxPool,
QLinearAdd, DequantizeLinear -> GlobalAveragePool -> QuantizeLinear) with
the CPU oracle, each called alone through the C ABI on shapes beyond the
ones ResNet-50 gives them: other windows and pads, channel counts that are
not a multiple of 16 (the scalar kernels), rows too wide for the
shared-memory column max, ragged element counts.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


# n, h, w, c, (kh, kw), (sh, sw), (pt, pl, pb, pr)
MAXPOOL_SHAPES = [
    (4, 112, 112, 64, (3, 3), (2, 2), (1, 1, 1, 1)),     # ResNet-50
    (2, 17, 23, 32, (3, 3), (2, 2), (1, 1, 1, 1)),       # odd extents
    (3, 20, 20, 48, (2, 3), (1, 2), (0, 1, 1, 0)),       # rectangular window, asymmetric pads
    (2, 9, 9, 16, (5, 5), (1, 1), (2, 2, 2, 2)),         # window wider than a padded border
    (2, 13, 11, 24, (3, 3), (2, 2), (1, 1, 1, 1)),       # c % 16 != 0: scalar kernel
    (1, 6, 400, 128, (3, 3), (2, 2), (1, 1, 1, 1)),      # 51200-byte rows: no shared-memory column max
]


@pytest.mark.parametrize("shape", MAXPOOL_SHAPES)
def test_maxpool(cuda_dev, shape):
    from nnr_b200 import ops
    from nnr_b200._lib import call
    n, h, w, c, (kh, kw), (sh, sw), pads = shape
    rng = np.random.default_rng(n * h + w * c)
    x = rng.integers(0, 256, size=(n, h, w, c)).astype(np.uint8)
    oh = (h + pads[0] + pads[2] - kh) // sh + 1
    ow = (w + pads[1] + pads[3] - kw) // sw + 1
    ref = np.empty((n, oh, ow, c), np.uint8)
    rc = O.lib().oracle_maxpool_u8_nhwc(x.ctypes.data_as(C.c_void_p), ref.ctypes.data_as(C.c_void_p), n, h, w, c,
                                        kh, kw, sh, sw, *pads)
    assert rc == 0
    xd = torch.from_numpy(x).to(cuda_dev)
    yd = torch.empty((n, oh, ow, c), dtype=torch.uint8, device=cuda_dev)
    call("nnrcu_maxpool_u8_nhwc", _ptr(xd), _ptr(yd), n, h, w, c, kh, kw, sh, sw, *pads, _stream())
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert np.array_equal(yd.cpu().numpy(), ref)


@pytest.mark.parametrize("n", [1, 15, 16, 17, 4099, 802816])
def test_qlinearadd(cuda_dev, n):
    from nnr_b200 import ops
    from nnr_b200._lib import call
    rng = np.random.default_rng(n)
    a = rng.integers(0, 256, size=n).astype(np.uint8)
    b = rng.integers(0, 256, size=n).astype(np.uint8)
    args = (0.031, 120, 0.017, 131, 0.04, 90)
    ref = O.qlinearadd_u8(a, args[0], args[1], b, args[2], args[3], args[4], args[5])
    ad, bd = torch.from_numpy(a).to(cuda_dev), torch.from_numpy(b).to(cuda_dev)
    yd = torch.empty(n, dtype=torch.uint8, device=cuda_dev)
    call("nnrcu_qlinearadd_u8", _ptr(ad), args[0], args[1], _ptr(bd), args[2], args[3], args[4], args[5], _ptr(yd),
         n, _stream())
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert np.array_equal(yd.cpu().numpy(), ref)


@pytest.mark.parametrize("n,h,w,c", [(32, 7, 7, 2048), (3, 5, 4, 40), (1, 1, 1, 16), (2, 9, 9, 7)])
def test_dq_gap_q(cuda_dev, n, h, w, c):
    from nnr_b200 import ops
    from nnr_b200._lib import call
    rng = np.random.default_rng(n * c + h)
    x = rng.integers(0, 256, size=(n, h, w, c)).astype(np.uint8)
    ref = O.dq_gap_q_u8_nhwc(x, 0.05, 7, 0.03, 3)
    xd = torch.from_numpy(x).to(cuda_dev)
    yd = torch.empty((n, c), dtype=torch.uint8, device=cuda_dev)
    call("nnrcu_dq_gap_q_u8_nhwc", _ptr(xd), n, h * w, c, 0.05, 7, 0.03, 3, _ptr(yd), _stream())
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert np.array_equal(yd.cpu().numpy(), ref)
