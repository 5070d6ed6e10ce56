"""nnrcu_qlinearmatmul_noalloc: the QLinearMatMul entry point for callers that
cannot allocate device memory when they run an operator (their device memory
is reserved up front by another allocator, or allocation after start-up is
forbidden). It keeps its derived data in a fixed static device array instead
of allocating.

Checked through the C ABI, bit-exact like every integer result here, on
several calls in a row:
- against the regular entry point (nnrcu_qlinearmatmul_create/_run);
- against the CPU oracle (the restatement of QLinearMatMul's R4 requant);
- the cases cover the TMA path (k a multiple of 128), the gather path
  (k < 128) and a partial last 128-byte K slab, with b_zp zero and non-zero;
  each later call is a smaller, different problem, so leftovers of an earlier
  call in the shared array would show up;
- the device's free memory (cudaMemGetInfo) is the same before and after the
  calls that follow the first one (the first call may load the module).
This file is named to be collected last.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O


def _noalloc(a_dev, b_dev, y_dev, m, k, n, a_scale, a_zp, b_scale, b_zp, y_scale, y_zp, stream):
    from nnr_b200 import _lib
    return _lib.lib.nnrcu_qlinearmatmul_noalloc(C.c_void_p(a_dev.data_ptr()), C.c_void_p(b_dev.data_ptr()),
                                                C.c_void_p(y_dev.data_ptr()), m, k, n, a_scale, a_zp, b_scale, b_zp,
                                                y_scale, y_zp, C.c_void_p(stream))


CASES = [
    # m, k, n, a_zp, b_zp, y_zp
    (512, 768, 3072, 128, 0, 128),   # TMA path, whole K slabs
    (300, 256, 200, 117, -3, 90),    # row sums (b_zp != 0), ragged n
    (70, 48, 96, 5, 7, 200),         # gather path (k < 128)
    (130, 144, 300, 250, 0, 11),     # partial last K slab
]


@pytest.mark.gpu
def test_noalloc_matches_regular_entry_point_and_oracle(cuda_dev):
    import torch
    from nnr_b200 import ops
    from nnr_b200._lib import check

    stream = torch.cuda.current_stream().cuda_stream
    prepared = []
    for i, (m, k, n, a_zp, b_zp, y_zp) in enumerate(CASES):
        rng = np.random.default_rng(40 + i)
        a = rng.integers(0, 256, size=(m, k)).astype(np.uint8)
        b = rng.integers(-127, 128, size=(k, n)).astype(np.int8)
        a_scale, b_scale = 0.03, 0.004
        y_scale = a_scale * b_scale * 30.0 * float(np.sqrt(k))
        regular = ops.QLinearMatMul(m, b, a_scale, a_zp, b_scale, b_zp, y_scale, y_zp)
        a_dev = torch.from_numpy(a).to(cuda_dev)
        y_ref = regular.exec(a_dev).cpu().numpy()
        want = O.qlinearmatmul(a, b, a_scale, a_zp, b_scale, b_zp, y_scale, y_zp)
        assert np.array_equal(y_ref, want), f"case {i}: regular entry point differs from the oracle"
        b_dev = torch.from_numpy(b).to(cuda_dev)
        y_dev = torch.full((m, n), 0xAB, dtype=torch.uint8, device=cuda_dev)
        prepared.append((m, k, n, a_zp, b_zp, y_zp, a_scale, b_scale, y_scale, a_dev, b_dev, y_dev, want))
    torch.cuda.synchronize()

    free_after_first = None
    for i, (m, k, n, a_zp, b_zp, y_zp, a_scale, b_scale, y_scale, a_dev, b_dev, y_dev, want) in enumerate(prepared):
        check(_noalloc(a_dev, b_dev, y_dev, m, k, n, a_scale, a_zp, b_scale, b_zp, y_scale, y_zp, stream))
        torch.cuda.synchronize()
        if i == 0:
            free_after_first = torch.cuda.mem_get_info(cuda_dev)[0]
        assert ops.device_status() == 0
        got = y_dev.cpu().numpy()
        assert np.array_equal(got, want), f"call {i}: {(got != want).sum()} bytes differ"
    # a second pass over the same cases: the array keeps the previous call's bytes
    for i, (m, k, n, a_zp, b_zp, y_zp, a_scale, b_scale, y_scale, a_dev, b_dev, y_dev, want) in enumerate(prepared):
        y_dev.fill_(0x5C)
        torch.cuda.synchronize()
        check(_noalloc(a_dev, b_dev, y_dev, m, k, n, a_scale, a_zp, b_scale, b_zp, y_scale, y_zp, stream))
        torch.cuda.synchronize()
        assert np.array_equal(y_dev.cpu().numpy(), want), f"second pass, call {i}"
    assert torch.cuda.mem_get_info(cuda_dev)[0] == free_after_first, "device memory was allocated"


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
