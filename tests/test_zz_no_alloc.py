"""nnrcu_qlinearmatmul_noalloc: the QLinearMatMul entry point for callers that
cannot allocate device memory when they run an operator (their device memory
is reserved up front by another allocator, or allocation after start-up is
forbidden). It keeps its derived data in a fixed static device array instead
of allocating.

Checked through the C ABI against the regular entry point
(nnrcu_qlinearmatmul_create/_run) on two calls in a row, bit-exact like every
integer result here. The second call has a smaller, different problem, so
leftovers of the first call in the shared array would show up. This file
is named to be collected last.
"""
import ctypes as C

import numpy as np
import pytest


def _noalloc(a_dev, b_dev, y_dev, m, k, n, a_scale, a_zp, b_scale, b_zp, y_scale, y_zp, stream):
    from nnr_b200 import _lib
    return _lib.lib.nnrcu_qlinearmatmul_noalloc(C.c_void_p(a_dev.data_ptr()), C.c_void_p(b_dev.data_ptr()),
                                                C.c_void_p(y_dev.data_ptr()), m, k, n, a_scale, a_zp, b_scale, b_zp,
                                                y_scale, y_zp, C.c_void_p(stream))


@pytest.mark.gpu
def test_noalloc_matches_regular_entry_point_twice(cuda_dev):
    import torch
    from nnr_b200 import ops
    from nnr_b200._lib import check

    cases = [
        # m, k, n, a_zp, b_zp, y_zp
        (512, 768, 3072, 128, 0, 128),
        (300, 256, 200, 117, -3, 90),
    ]
    stream = torch.cuda.current_stream().cuda_stream
    for i, (m, k, n, a_zp, b_zp, y_zp) in enumerate(cases):
        rng = np.random.default_rng(40 + i)
        a = rng.integers(0, 256, size=(m, k)).astype(np.uint8)
        b = rng.integers(-127, 128, size=(k, n)).astype(np.int8)
        a_scale, b_scale = 0.03, 0.004
        y_scale = a_scale * b_scale * 30.0 * float(np.sqrt(k))

        regular = ops.QLinearMatMul(m, b, a_scale, a_zp, b_scale, b_zp, y_scale, y_zp)
        a_dev = torch.from_numpy(a).to(cuda_dev)
        y_ref = regular.exec(a_dev)

        b_dev = torch.from_numpy(b).to(cuda_dev)
        y_dev = torch.full((m, n), 0xAB, dtype=torch.uint8, device=cuda_dev)
        check(_noalloc(a_dev, b_dev, y_dev, m, k, n, a_scale, a_zp, b_scale, b_zp, y_scale, y_zp, stream))
        torch.cuda.synchronize()
        assert ops.device_status() == 0
        got, want = y_dev.cpu().numpy(), y_ref.cpu().numpy()
        assert np.array_equal(got, want), f"call {i}: {(got != want).sum()} bytes differ"


@pytest.mark.gpu
def test_noalloc_rejects_oversize(cuda_dev):
    import torch
    from nnr_b200 import _lib
    m, k, n = 64, 4096, 4096  # 16 MiB of transposed B > the static limit
    a = torch.zeros((m, k), dtype=torch.uint8, device=cuda_dev)
    b = torch.zeros((k, n), dtype=torch.int8, device=cuda_dev)
    y = torch.zeros((m, n), dtype=torch.uint8, device=cuda_dev)
    rc = _noalloc(a, b, y, m, k, n, 0.1, 0, 0.1, 0, 0.1, 0, torch.cuda.current_stream().cuda_stream)
    assert rc == -1
    assert "static limit" in _lib.last_error()
