"""ctypes binding of libnnrcu.so (include/nnrcu.h).

The library is the product: there is no Python or CPU fallback. Importing
this module fails loudly when the shared object is missing, and every call
that returns a negative status raises NnrcuError with the library's message.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("NNRCU_LIB", _PKG / "libnnrcu.so"))

NNRCU_OK = 0
ERR_NAMES = {-1: "INVALID", -2: "UNSUPPORTED", -3: "CUDA", -4: "DEVICE", -5: "NOMEM"}

LAYOUT_NCHW, LAYOUT_NHWC = 0, 1
RQ_AUTO, RQ_R1, RQ_R2, RQ_R3 = 0, 1, 2, 3
POST_NONE, POST_RELU, POST_CLIP, POST_HARDSWISH, POST_SIGMOID, POST_LEAKYRELU, POST_TANH = range(7)


class NnrcuError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"nnrcu error {code} ({ERR_NAMES.get(code, '?')}): {msg}")
        self.code = code


class ConvDesc(C.Structure):
    _fields_ = [
        ("n", C.c_int), ("c", C.c_int), ("h", C.c_int), ("w", C.c_int),
        ("oc", C.c_int), ("kh", C.c_int), ("kw", C.c_int), ("group", C.c_int),
        ("stride_h", C.c_int), ("stride_w", C.c_int),
        ("pad_top", C.c_int), ("pad_left", C.c_int), ("pad_bottom", C.c_int), ("pad_right", C.c_int),
        ("dil_h", C.c_int), ("dil_w", C.c_int),
        ("in_layout", C.c_int), ("out_layout", C.c_int),
        ("post_op", C.c_int), ("post_a", C.c_float), ("post_b", C.c_float),
        ("requant", C.c_int),
    ]


P, I, F, SZ, U8, I8 = C.c_void_p, C.c_int, C.c_float, C.c_size_t, C.c_uint8, C.c_int8
PP = C.POINTER(C.c_void_p)

# name -> argtypes (all return int)
SIGNATURES = {
    "nnrcu_init": [I],
    "nnrcu_last_error": [C.c_char_p, SZ],
    "nnrcu_device_status": [C.POINTER(C.c_int)],
    "nnrcu_stream_create": [PP],
    "nnrcu_stream_destroy": [P],
    "nnrcu_stream_sync": [P],
    "nnrcu_malloc": [PP, SZ],
    "nnrcu_free": [P],
    "nnrcu_memcpy_h2d": [P, P, SZ, P],
    "nnrcu_memcpy_d2h": [P, P, SZ, P],
    "nnrcu_memset": [P, I, SZ, P],
    "nnrcu_host_register": [P, SZ],
    "nnrcu_host_unregister": [P],
    "nnrcu_graph_begin": [P],
    "nnrcu_graph_end": [P, PP],
    "nnrcu_graph_launch": [P, P],
    "nnrcu_graph_destroy": [P],
    "nnrcu_op_workspace_size": [P, C.POINTER(C.c_size_t)],
    "nnrcu_op_num_ops": [P, C.POINTER(C.c_int64)],
    "nnrcu_op_destroy": [P],
    "nnrcu_qlinearconv_create": [C.POINTER(ConvDesc), P, P, I, P, I, P, F, U8, F, U8, PP],
    "nnrcu_qlinearconv_run": [P, P, P, P, P],
    "nnrcu_qlinearconv_run_add": [P, P, P, F, U8, F, U8, P, P, P],
    "nnrcu_qlinearconv_input_padding": [P, P],
    "nnrcu_qlinearconv_set_padded_io": [P, I, I, I, I, I],
    "nnrcu_qlinearconv_run_quantize": [P, P, F, U8, P, P, P],
    "nnrcu_gap_f32_nhwc": [P, I, I, I, P, P],
    "nnrcu_add_f32": [P, P, P, SZ, SZ, P],
    "nnrcu_gemm_f32_create_ex": [I, I, I, I, I, F, F, P, P, I, I, F, F, I, PP],
    "nnrcu_matmul_f32_workspace": [I, I, I, C.POINTER(C.c_size_t)],
    "nnrcu_matmul_f32_run": [P, P, P, I, I, I, I, C.c_longlong, C.c_longlong, I, F, F, P, SZ, P],
    "nnrcu_matmul_half_workspace": [I, I, I, C.POINTER(C.c_size_t)],
    "nnrcu_matmul_half_run": [P, P, P, I, I, I, I, C.c_longlong, C.c_longlong, I, I, F, F, P, SZ, P],
    "nnrcu_conv_half_create": [P, I, P, P, PP],
    "nnrcu_conv_half_run": [P, P, P, P, P],
    "nnrcu_gemm_half_create": [I, I, I, I, I, F, F, I, P, P, I, I, F, F, PP],
    "nnrcu_gemm_half_run": [P, P, P, P, P],
    "nnrcu_qlinearmatmul_create": [I, I, I, F, U8, P, F, I8, F, U8, PP],
    "nnrcu_qlinearmatmul_run": [P, P, P, P, P],
    "nnrcu_qlinearmatmul_noalloc": [P, P, P, I, I, I, F, U8, F, I8, F, U8, P],
    "nnrcu_conv_f32_create": [C.POINTER(ConvDesc), P, P, PP],
    "nnrcu_conv_f32_run": [P, P, P, P, P, P],
    "nnrcu_conv_f32_plane_stride": [P, C.POINTER(C.c_int)],
    "nnrcu_conv_f32_run_to_planes": [P, P, P, P, C.c_int, P],
    "nnrcu_conv_f32_run_planes": [P, P, P, P, P, P],
    "nnrcu_gemm_f32_create": [I, I, I, I, I, F, F, P, P, I, I, F, F, PP],
    "nnrcu_gemm_f32_run": [P, P, P, P, P],
    "nnrcu_quantize_linear_u8": [P, P, I, I, I, I, F, U8, I, I, P],
    "nnrcu_maxpool_u8_nhwc": [P, P, I, I, I, I, I, I, I, I, I, I, I, I, P],
    "nnrcu_qlinearadd_u8": [P, F, U8, P, F, U8, F, U8, P, SZ, P],
    "nnrcu_dq_gap_q_u8_nhwc": [P, I, I, I, F, U8, F, U8, P, P],
    "nnrcu_dequantize_linear_u8": [P, F, U8, P, I, I, P, P],
    "nnrcu_nchw_to_nhwc": [P, P, I, I, I, I, I, P],
    "nnrcu_nhwc_to_nchw": [P, P, I, I, I, I, I, P],
}


def _load() -> C.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m nnr_b200.build` "
            "(there is no CPU fallback for the device operators)")
    lib = C.CDLL(str(LIB_PATH))
    for name, argt in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argt
        fn.restype = C.c_int
    return lib


lib = _load()


def last_error() -> str:
    buf = C.create_string_buffer(512)
    lib.nnrcu_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != NNRCU_OK:
        raise NnrcuError(rc, last_error())


def call(name: str, *args) -> None:
    check(getattr(lib, name)(*args))
