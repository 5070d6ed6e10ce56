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
        _ref.ref_qconv_first_layer.restype = C.c_int
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


def ref_qconv_first_layer(x, w, w_scale, bias, x_scale, x_zp, y_scale, y_zp, strides=(1, 1), pads=(0, 0),
                          has_post=False, out_layout="NCHW"):
    """nnr's first-layer int8 conv (the R3 stem kernel, its own AVX-512 VNNI
    code) on NCHW u8 input with at most 4 channels and symmetric pads
    (pad_h, pad_w). Returns None when the harness is absent or the host lacks
    VNNI."""
    r = ref_lib()
    if r is None or not r.ref_has_vnni():
        return None
    x = np.ascontiguousarray(x, np.uint8)
    w = np.ascontiguousarray(w, np.int8)
    n, c, h, wd = x.shape
    oc, _, kh, kw = w.shape
    oh, ow = out_hw(h, wd, kh, kw, strides, (pads[0], pads[1], pads[0], pads[1]), (1, 1))
    ws = np.ascontiguousarray(np.atleast_1d(w_scale), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.int32)
    y = np.empty((n, oc, oh, ow) if out_layout == "NCHW" else (n, oh, ow, oc), np.uint8)
    rc = r.ref_qconv_first_layer(_p(x), n, c, h, wd, _p(w), oc, kh, kw, strides[0], strides[1], pads[0], pads[1],
                                 _p(ws), ws.size, _p(b), _f(x_scale), C.c_uint8(x_zp), _f(y_scale), C.c_uint8(y_zp),
                                 int(bool(has_post)), int(out_layout == "NHWC"), _p(y))
    return None if rc != 0 else y


def _dw_args(x, w, w_scale, bias, strides, pads, dilations):
    x = np.ascontiguousarray(x, np.uint8)
    w = np.ascontiguousarray(w, np.int8)
    ws = np.ascontiguousarray(np.atleast_1d(w_scale), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.int32)
    n, h, wd, c = x.shape
    kh, kw = w.shape[2], w.shape[3]
    oh, ow = out_hw(h, wd, kh, kw, strides, pads, dilations)
    return x, w, ws, b, (n, c, h, wd, kh, kw, oh, ow)


def qdwconv_u8_nhwc(x, w, w_scale, bias, x_scale, x_zp, y_scale, y_zp, w_zp=0, strides=(1, 1), pads=(0, 0, 0, 0),
                    dilations=(1, 1)):
    """Depthwise QLinearConv on u8 NHWC x [n,h,w,c], w [c,1,kh,kw] s8, the
    restatement of nnr's exec_dw_int8_nhwc (nnr_oracle.c)."""
    x, w, ws, b, (n, c, h, wd, kh, kw, oh, ow) = _dw_args(x, w, w_scale, bias, strides, pads, dilations)
    y = np.empty((n, oh, ow, c), np.uint8)
    rc = lib().oracle_qdwconv_u8_nhwc(_p(x), n, c, h, wd, _p(w), kh, kw, strides[0], strides[1], *pads,
                                      dilations[0], dilations[1], _p(ws), ws.size, C.c_int8(w_zp), _p(b),
                                      _f(x_scale), C.c_uint8(x_zp), _f(y_scale), C.c_uint8(y_zp), _p(y))
    if rc != 0:
        raise RuntimeError("oracle_qdwconv_u8_nhwc failed")
    return y


def ref_qdwconv_nhwc(x, w, w_scale, bias, x_scale, x_zp, y_scale, y_zp, w_zp=0, strides=(1, 1), pads=(0, 0, 0, 0),
                     dilations=(1, 1), fill=0xAB):
    """nnr's own AVX-512 depthwise int8 kernel (oracle/_ref), or None when
    the harness is not built or the host lacks VNNI. Output bytes nnr does
    not write (channels past the last group of 16) keep `fill`."""
    r = ref_lib()
    if r is None or not r.ref_has_vnni():
        return None
    x, w, ws, b, (n, c, h, wd, kh, kw, oh, ow) = _dw_args(x, w, w_scale, bias, strides, pads, dilations)
    y = np.full((n, oh, ow, c), fill, np.uint8)
    rc = r.ref_qdwconv_nhwc(_p(x), n, c, h, wd, _p(w), kh, kw, strides[0], strides[1], *pads, dilations[0],
                            dilations[1], _p(ws), ws.size, C.c_int8(w_zp), _p(b), _f(x_scale), C.c_uint8(x_zp),
                            _f(y_scale), C.c_uint8(y_zp), _p(y))
    if rc != 0:
        raise RuntimeError("ref_qdwconv_nhwc failed")
    return y


def num_threads() -> int:
    return lib().oracle_num_threads()


def set_threads(n: int) -> None:
    """Sets the oracle's OpenMP thread count (overrides OMP_NUM_THREADS)."""
    lib().oracle_set_threads(int(n))


def round_bf16(x):
    """fp32 -> bf16 -> fp32, round to nearest even (nnr's float32_to_bfloat16,
    nnrconf.h:201-206, and the AVX-512 conversion it vectorises)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = ((u + (((u >> 16) & 1) + 0x7FFF)) >> 16) << 16
    return u.astype(np.uint32).view(np.float32)


def matmul_f32_bf16_host(a, b):
    """nnr's fp32 MatMul with a constant B on an AVX-512 BF16 host
    (MatMul.cpp:128-152 packs B to bf16, :382-428 exec_f32_via_bf16 converts
    A to bf16 and runs VDPBF16PS with fp32 accumulation): bf16(A) x bf16(B),
    accumulated here in fp64. a [..., k], b [k, n]."""
    a64 = round_bf16(a).astype(np.float64)
    b64 = round_bf16(b).astype(np.float64)
    return (a64 @ b64).astype(np.float32)


# ------------------------------------------------------------------ QDQ glue
def quantize_u8(x, scale, zp):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(x.shape, np.uint8)
    lib().oracle_quantize_u8(_p(x), _p(y), C.c_longlong(x.size), _f(scale), C.c_uint8(zp))
    return y


def maxpool_u8_nhwc(x, k=3, s=2, pads=(1, 1, 1, 1)):
    x = np.ascontiguousarray(x, np.uint8)
    n, h, w, c = x.shape
    oh = (h + pads[0] + pads[2] - k) // s + 1
    ow = (w + pads[1] + pads[3] - k) // s + 1
    y = np.empty((n, oh, ow, c), np.uint8)
    rc = lib().oracle_maxpool_u8_nhwc(_p(x), _p(y), n, h, w, c, k, k, s, s, *pads)
    if rc != 0:
        raise RuntimeError("oracle_maxpool_u8_nhwc failed")
    return y


def qlinearadd_u8(a, a_scale, a_zp, b, b_scale, b_zp, y_scale, y_zp):
    a = np.ascontiguousarray(a, np.uint8)
    b = np.ascontiguousarray(b, np.uint8)
    y = np.empty(a.shape, np.uint8)
    lib().oracle_qlinearadd_u8(_p(a), _f(a_scale), C.c_uint8(a_zp), _p(b), _f(b_scale), C.c_uint8(b_zp),
                               _f(y_scale), C.c_uint8(y_zp), _p(y), C.c_longlong(a.size))
    return y


def dq_gap_q_u8_nhwc(x, x_scale, x_zp, y_scale, y_zp):
    x = np.ascontiguousarray(x, np.uint8)
    n, h, w, c = x.shape
    y = np.empty((n, c), np.uint8)
    rc = lib().oracle_dq_gap_q_u8_nhwc(_p(x), n, h * w, c, _f(x_scale), C.c_uint8(x_zp), _f(y_scale),
                                       C.c_uint8(y_zp), _p(y))
    if rc != 0:
        raise RuntimeError("oracle_dq_gap_q_u8_nhwc failed")
    return y


def gap_f32_nhwc(x):
    """GlobalAveragePool of fp32 NHWC [n, h, w, c] -> [n, c]."""
    x = np.ascontiguousarray(x, np.float32)
    n, h, w, c = x.shape
    y = np.empty((n, c), np.float32)
    lib().oracle_gap_f32_nhwc(_p(x), n, h * w, c, _p(y))
    return y


def dequantize_u8(x, scale, zp, bias=None):
    x = np.ascontiguousarray(x, np.uint8)
    rows, cols = x.shape
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    y = np.empty(x.shape, np.float32)
    lib().oracle_dequantize_u8(_p(x), _f(scale), C.c_uint8(zp), _p(b), rows, cols, _p(y))
    return y


# ------------------------------------------------------------------ whole int8 network
def run_qmodel(model, x, keep=False):
    """Runs a quantised network (nnr_b200.resnet50.QModel) node by node on the
    CPU with the restated operators. x: fp32 NCHW input. Returns the fp32
    logits, plus every intermediate tensor when keep is set."""
    t = {"input": np.ascontiguousarray(x, np.float32)}
    qp = model.qparams
    for nd in model.nodes:
        a = nd.attrs
        if nd.op == "QuantizeLinear":
            t[nd.output] = quantize_u8(t[nd.inputs[0]], qp[nd.output].scale, qp[nd.output].zp)
        elif nd.op == "QLinearConv":
            xin = t[nd.inputs[0]]
            xq, yq = qp[nd.inputs[0]], qp[nd.output]
            t[nd.output] = qlinearconv(xin, a["w"], a["w_scale"], a["bias"], xq.scale, xq.zp, yq.scale, yq.zp,
                                       strides=(a["stride"],) * 2, pads=(a["pad"],) * 4, formula=a["requant"],
                                       in_layout=a["in_layout"], out_layout="NHWC")
        elif nd.op == "MaxPool":
            t[nd.output] = maxpool_u8_nhwc(t[nd.inputs[0]], a["k"], a["s"], (a["pad"],) * 4)
        elif nd.op == "QLinearAdd":
            qa, qb, qy = qp[nd.inputs[0]], qp[nd.inputs[1]], qp[nd.output]
            t[nd.output] = qlinearadd_u8(t[nd.inputs[0]], qa.scale, qa.zp, t[nd.inputs[1]], qb.scale, qb.zp,
                                         qy.scale, qy.zp)
        elif nd.op == "DqGapQ":
            qx, qy = qp[nd.inputs[0]], qp[nd.output]
            t[nd.output] = dq_gap_q_u8_nhwc(t[nd.inputs[0]], qx.scale, qx.zp, qy.scale, qy.zp)
        elif nd.op == "QLinearMatMul":
            qa, qy = qp[nd.inputs[0]], qp[nd.output]
            t[nd.output] = qlinearmatmul(t[nd.inputs[0]], a["b"], qa.scale, qa.zp, a["b_scale"], a["b_zp"],
                                         qy.scale, qy.zp)
        elif nd.op == "DequantizeLinear":
            qx = qp[nd.inputs[0]]
            t[nd.output] = dequantize_u8(t[nd.inputs[0]], qx.scale, qx.zp, a.get("bias"))
        else:
            raise ValueError(f"unknown node {nd.op}")
        if not keep:
            for name in nd.inputs:
                if name != "input" and all(name not in n2.inputs for n2 in model.nodes[model.nodes.index(nd) + 1:]):
                    t.pop(name, None)
    return (t["logits"], t) if keep else t["logits"]


# ------------------------------------------------------------------ whole fp32 network
def run_fmodel(model, x, keep=False):
    """Runs an fp32 network (nnr_b200.mobilenetv2.FModel) node by node on the
    CPU with the restated operators (fp64 accumulation). x: fp32 NCHW input.
    Returns the logits, plus every intermediate tensor when keep is set."""
    t = {"input": np.ascontiguousarray(x, np.float32)}
    for nd in model.nodes:
        a = nd.attrs
        if nd.op == "Conv":
            lay = "NCHW" if nd.inputs[0] == "input" else "NHWC"
            post = 2 if a["post"] == "Clip" else 0
            t[nd.output] = conv_f32(t[nd.inputs[0]], a["w"], a["b"], strides=(a["stride"],) * 2, pads=(a["pad"],) * 4,
                                    group=a["group"], post=post, post_a=0.0, post_b=6.0, in_layout=lay,
                                    out_layout="NHWC")
        elif nd.op == "Add":
            t[nd.output] = t[nd.inputs[0]] + t[nd.inputs[1]]
        elif nd.op == "GlobalAveragePool":
            t[nd.output] = gap_f32_nhwc(t[nd.inputs[0]])
        elif nd.op == "Gemm":
            t[nd.output] = gemm_f32(t[nd.inputs[0]], a["b"], a["c"])
        else:
            raise ValueError(nd.op)
    return (t["logits"], t) if keep else t["logits"]

