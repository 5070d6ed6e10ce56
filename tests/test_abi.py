"""The C-ABI library loads on a machine without a GPU, exports every entry
point include/nnrcu.h declares, and rejects bad descriptors before touching
the device (no compute calls here)."""
import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "nnrcu.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*int\s+(nnrcu_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for must in ["nnrcu_init", "nnrcu_qlinearconv_create", "nnrcu_qlinearconv_run", "nnrcu_qlinearmatmul_create",
                 "nnrcu_qlinearmatmul_run", "nnrcu_conv_f32_create", "nnrcu_conv_f32_run", "nnrcu_gemm_f32_create",
                 "nnrcu_gemm_f32_run", "nnrcu_graph_begin", "nnrcu_graph_end", "nnrcu_graph_launch"]:
        assert must in syms


def test_library_exports_every_declared_symbol():
    from nnr_b200 import _lib
    lib = C.CDLL(str(_lib.LIB_PATH))
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, f"not exported: {missing}"
    # and the ctypes binding covers exactly the header
    assert set(_lib.SIGNATURES) == set(declared_symbols())


def test_library_is_sm100a_only():
    """The fatbin carries sm_100a code (checked through the file name of the
    build flags, not by disassembly)."""
    from nnr_b200 import build
    assert "arch=compute_100a,code=sm_100a" in " ".join(build.ARCH)


def _desc(**kw):
    from nnr_b200._lib import ConvDesc
    base = dict(n=1, c=8, h=8, w=8, oc=8, kh=3, kw=3, group=1, stride_h=1, stride_w=1, pad_top=1, pad_left=1,
                pad_bottom=1, pad_right=1, dil_h=1, dil_w=1, in_layout=0, out_layout=0, post_op=0, post_a=0.0,
                post_b=0.0, requant=0)
    base.update(kw)
    return ConvDesc(**base)


@pytest.mark.parametrize("bad", [dict(n=0), dict(c=-1), dict(stride_h=0), dict(pad_top=-1), dict(kh=20),
                                 dict(in_layout=7), dict(group=0)])
def test_qlinearconv_rejects_bad_descriptors(bad):
    import numpy as np
    from nnr_b200 import _lib
    d = _desc(**bad)
    w = np.zeros(8 * 8 * 3 * 3, np.int8)
    s = np.ones(1, np.float32)
    op = C.c_void_p()
    rc = _lib.lib.nnrcu_qlinearconv_create(C.byref(d), w.ctypes.data_as(C.c_void_p), s.ctypes.data_as(C.c_void_p),
                                           1, None, 0, None, 0.02, 128, 0.05, 128, C.byref(op))
    assert rc == -1
    assert _lib.last_error()
    assert not op


def test_qlinearconv_unsupported_cases_are_reported():
    """Non-zero weight zero points (grouped or not) are declined with
    NNRCU_ERR_UNSUPPORTED (nnr's registry then keeps the CPU operator); a
    group count that does not divide the channels is NNRCU_ERR_INVALID."""
    import numpy as np
    from nnr_b200 import _lib
    w = np.zeros(8 * 8 * 3 * 3, np.int8)
    s = np.ones(1, np.float32)
    op = C.c_void_p()
    d = _desc(group=3)
    rc = _lib.lib.nnrcu_qlinearconv_create(C.byref(d), w.ctypes.data_as(C.c_void_p), s.ctypes.data_as(C.c_void_p),
                                           1, None, 0, None, 0.02, 128, 0.05, 128, C.byref(op))
    assert rc == -1
    assert "group" in _lib.last_error()
    zp = np.ones(8, np.int8)
    for g in (1, 2):
        d = _desc(group=g)
        rc = _lib.lib.nnrcu_qlinearconv_create(C.byref(d), w.ctypes.data_as(C.c_void_p),
                                               s.ctypes.data_as(C.c_void_p), 1, zp.ctypes.data_as(C.c_void_p), 8,
                                               None, 0.02, 128, 0.05, 128, C.byref(op))
        assert rc == -2
        assert "zero point" in _lib.last_error()


def test_null_arguments():
    from nnr_b200 import _lib
    assert _lib.lib.nnrcu_qlinearconv_run(None, None, None, None, None) == -1
    assert _lib.lib.nnrcu_op_workspace_size(None, None) == -1
    assert _lib.lib.nnrcu_op_destroy(None) == 0
    assert _lib.lib.nnrcu_qlinearmatmul_create(0, 1, 1, 1.0, 0, None, 1.0, 0, 1.0, 0, None) == -1
