"""Python access to the CPU oracle (test infrastructure only).

liboracle.so is the C restatement in nnr_oracle.c; _ref/libnnr_ref_int8.so
(optional) is nnr's own int8 direct-conv kernel compiled from the nnr
sources by `make -C oracle ref`. Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference arm use this module, as the checker.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
REF = HERE / "_ref" / "libnnr_ref_int8.so"

R1, R2, R3 = 1, 2, 3


def build(ref: bool = False) -> None:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    if ref:
        subprocess.run(["make", "-s", "-C", str(HERE), "ref"], check=True)


def _load() -> C.CDLL:
    if not LIB.exists():
        build()
    lib = C.CDLL(str(LIB))
    lib.oracle_qlinearconv.restype = C.c_int
    lib.oracle_qlinearmatmul.restype = C.c_int
    lib.oracle_conv_f32.restype = C.c_int
    lib.oracle_gemm_f32.restype = C.c_int
    lib.oracle_num_threads.restype = C.c_int
    return lib


_lib = None
_ref = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        _lib = _load()
    return _lib


def ref_lib():
    """nnr's own kernel harness, or None when it was not built here."""
    global _ref
    if _ref is None and REF.exists():
        _ref = C.CDLL(str(REF))
        _ref.ref_qlinearconv_direct.restype = C.c_int
        _ref.ref_has_vnni.restype = C.c_int
        _ref.ref_get_threads.restype = C.c_int
    return _ref


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _f(v):
    return C.c_float(float(v))


def out_hw(h, w, kh, kw, strides, pads, dil):
    oh = (h + pads[0] + pads[2] - (dil[0] * (kh - 1) + 1)) // strides[0] + 1
    ow = (w + pads[1] + pads[3] - (dil[1] * (kw - 1) + 1)) // strides[1] + 1
    return oh, ow


def qlinearconv(x, w, w_scale, bias, x_scale, x_zp, y_scale, y_zp, strides=(1, 1), pads=(0, 0, 0, 0),
                dilations=(1, 1), formula=R1, has_post=False, in_layout="NCHW", out_layout="NCHW",
                want_acc=False):
    """x: u8 (NCHW [n,c,h,w] or NHWC [n,h,w,c]); w: s8 OIHW. Returns y (and the
    int32 accumulators, NCHW, when want_acc)."""
    x = np.ascontiguousarray(x, np.uint8)
    w = np.ascontiguousarray(w, np.int8)
    if in_layout == "NCHW":
        n, c, h, wd = x.shape
    else:
        n, h, wd, c = x.shape
    oc, _, kh, kw = w.shape
    oh, ow = out_hw(h, wd, kh, kw, strides, pads, dilations)
    ws = np.ascontiguousarray(np.atleast_1d(w_scale), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.int32)
    y = np.empty((n, oc, oh, ow) if out_layout == "NCHW" else (n, oh, ow, oc), np.uint8)
    acc = np.empty((n, oc, oh, ow), np.int32) if want_acc else None
    rc = lib().oracle_qlinearconv(
        _p(x), int(in_layout == "NHWC"), n, c, h, wd, _p(w), oc, kh, kw, strides[0], strides[1], pads[0], pads[1],
        pads[2], pads[3], dilations[0], dilations[1], _p(ws), ws.size, _p(b), _f(x_scale), C.c_uint8(x_zp),
        _f(y_scale), C.c_uint8(y_zp), int(formula), int(bool(has_post)), int(out_layout == "NHWC"), _p(y), _p(acc))
    if rc != 0:
        raise RuntimeError("oracle_qlinearconv failed")
    return (y, acc) if want_acc else y


def qlinearmatmul(a, b, a_scale, a_zp, b_scale, b_zp, y_scale, y_zp):
    a = np.ascontiguousarray(a, np.uint8)
    b = np.ascontiguousarray(b, np.int8)
    m, k = a.shape
    n = b.shape[1]
    y = np.empty((m, n), np.uint8)
    rc = lib().oracle_qlinearmatmul(_p(a), _p(b), m, k, n, _f(a_scale), C.c_uint8(a_zp), _f(b_scale),
                                    C.c_int8(b_zp), _f(y_scale), C.c_uint8(y_zp), _p(y))
    if rc != 0:
        raise RuntimeError("oracle_qlinearmatmul failed")
    return y


def conv_f32(x, w, bias=None, strides=(1, 1), pads=(0, 0, 0, 0), dilations=(1, 1), group=1, post=0, post_a=0.0,
             post_b=0.0, residual=None, in_layout="NCHW", out_layout="NCHW"):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    if in_layout == "NCHW":
        n, c, h, wd = x.shape
    else:
        n, h, wd, c = x.shape
    oc, _, kh, kw = w.shape
    oh, ow = out_hw(h, wd, kh, kw, strides, pads, dilations)
    y = np.empty((n, oc, oh, ow) if out_layout == "NCHW" else (n, oh, ow, oc), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    r = None if residual is None else np.ascontiguousarray(residual, np.float32)
    rc = lib().oracle_conv_f32(_p(x), int(in_layout == "NHWC"), n, c, h, wd, _p(w), oc, kh, kw, group, strides[0],
                               strides[1], pads[0], pads[1], pads[2], pads[3], dilations[0], dilations[1], _p(b),
                               int(post), _f(post_a), _f(post_b), _p(r), int(out_layout == "NHWC"), _p(y))
    if rc != 0:
        raise RuntimeError("oracle_conv_f32 failed")
    return y


def gemm_f32(a, b, c=None, alpha=1.0, beta=1.0, trans_a=0, trans_b=0, post=0, post_a=0.0, post_b=0.0, rows=None):
    """Y = post(alpha*op(A)op(B) + beta*C); rows=(r0, r1) computes only those rows."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    m, k = (a.shape[1], a.shape[0]) if trans_a else a.shape
    n = b.shape[0] if trans_b else b.shape[1]
    r0, r1 = rows if rows is not None else (0, m)
    cm = None if c is None else np.ascontiguousarray(c, np.float32)
    c_rows = 0 if cm is None else (1 if cm.size == n else m)
    y = np.empty((r1 - r0, n), np.float32)
    rc = lib().oracle_gemm_f32(_p(a), _p(b), _p(cm), m, n, k, int(trans_a), int(trans_b), _f(alpha), _f(beta),
                               c_rows, int(post), _f(post_a), _f(post_b), r0, r1 - r0, _p(y))
    if rc != 0:
        raise RuntimeError("oracle_gemm_f32 failed")
    return y


def ref_qlinearconv_direct(x, w, w_scale, bias, x_scale, x_zp, y_scale, y_zp, strides=(1, 1), pads=(0, 0, 0, 0),
                           has_post=False, want_raw=False):
    """nnr's exec_direct_int8 (its own AVX-512 VNNI kernel) on NCHW u8 input.
    Returns None when the harness is absent or the host lacks VNNI."""
    r = ref_lib()
    if r is None or not r.ref_has_vnni():
        return None
    x = np.ascontiguousarray(x, np.uint8)
    w = np.ascontiguousarray(w, np.int8)
    n, c, h, wd = x.shape
    oc, _, kh, kw = w.shape
    oh, ow = out_hw(h, wd, kh, kw, strides, pads, (1, 1))
    ws = np.ascontiguousarray(np.atleast_1d(w_scale), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.int32)
    y = np.empty((n, oc, oh, ow), np.uint8)
    raw = np.empty((n, oc, oh, ow), np.int32) if want_raw else None
    rc = r.ref_qlinearconv_direct(_p(x), n, c, h, wd, _p(w), oc, kh, kw, strides[0], strides[1], pads[0], pads[1],
                                  pads[2], pads[3], _p(ws), ws.size, _p(b), _f(x_scale), C.c_uint8(x_zp),
                                  _f(y_scale), C.c_uint8(y_zp), int(bool(has_post)), _p(y), _p(raw))
    if rc != 0:
        return None
    return (y, raw) if want_raw else y


def num_threads() -> int:
    return lib().oracle_num_threads()
