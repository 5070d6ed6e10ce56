"""Host-side operators over libnnrcu.so, mirroring nnr's operator_t interface.

Each class corresponds to the nnr operator of the same op_type. Constructing
one is nnr's init()+reshape(): attributes are validated, weights packed and
uploaded, requant constants computed (once). exec() is nnr's exec(): it
enqueues the device work on a stream and returns. Tensors are torch CUDA
tensors used purely as device buffers; no torch op touches the data.

Reference interface: src/nnr.h:331-461 (operator_t), backend/cpu/Conv.cpp,
QLinearConv.cpp, QLinearMatMul.cpp, Gemm.cpp, MatMul.cpp.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

import numpy as np
import torch

from . import _lib
from ._lib import (ConvDesc, LAYOUT_NCHW, LAYOUT_NHWC, POST_NONE, RQ_AUTO, call, lib)

_LAYOUTS = {"NCHW": LAYOUT_NCHW, "NHWC": LAYOUT_NHWC}
_POSTS = {None: 0, "Relu": 1, "Clip": 2, "HardSwish": 3, "Sigmoid": 4, "LeakyRelu": 5, "Tanh": 6}


def init(device: int = 0) -> None:
    """Selects the device on this thread and initialises the library there."""
    torch.cuda.set_device(device)
    call("nnrcu_init", device)


def device_status() -> int:
    st = C.c_int(0)
    call("nnrcu_device_status", C.byref(st))
    return st.value


def _stream(stream) -> int:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


def _ptr(t: Optional[torch.Tensor]):
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("device operators take CUDA tensors")
    if not t.is_contiguous():
        raise ValueError("tensors must be contiguous")
    return C.c_void_p(t.data_ptr())


def _host(a: Optional[np.ndarray], dtype):
    if a is None:
        return None, None
    arr = np.ascontiguousarray(np.asarray(a, dtype=dtype))
    return arr, arr.ctypes.data_as(C.c_void_p)


class DeviceArena:
    """Bump allocator over one device buffer: the device arena that nnr's
    memory planner slots map onto (memory_planner.h:13-51). Reset per run."""

    def __init__(self, nbytes: int, device: Optional[int] = None):
        dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        self.buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
        self.off = 0

    def alloc(self, nbytes: int) -> Optional[torch.Tensor]:
        if nbytes == 0:
            return None
        start = (self.off + 255) // 256 * 256
        if start + nbytes > self.buf.numel():
            raise MemoryError(f"arena of {self.buf.numel()} bytes exhausted")
        self.off = start + nbytes
        return self.buf[start:start + nbytes]

    def reset(self) -> None:
        self.off = 0


class Operator:
    op_type = ""

    def __init__(self):
        self._op = C.c_void_p()

    def _created(self):
        if not self._op:
            raise RuntimeError("operator not created")

    def workspace_size(self) -> int:
        self._created()
        n = C.c_size_t(0)
        call("nnrcu_op_workspace_size", self._op, C.byref(n))
        return n.value

    def num_ops(self) -> int:
        self._created()
        n = C.c_int64(0)
        call("nnrcu_op_num_ops", self._op, C.byref(n))
        return n.value

    def _workspace(self, workspace, device):
        need = self.workspace_size()
        if need == 0:
            return None, None
        if workspace is None:
            workspace = torch.empty(need, dtype=torch.uint8, device=device)
        if workspace.numel() * workspace.element_size() < need:
            raise ValueError(f"workspace too small ({need} bytes needed)")
        return workspace, _ptr(workspace)

    def close(self):
        if getattr(self, "_op", None):
            lib.nnrcu_op_destroy(self._op)
            self._op = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def conv_desc(x_shape, w_shape, strides, pads, dilations, group, in_layout, out_layout, post, post_a, post_b,
              requant) -> ConvDesc:
    n, c, h, w = x_shape
    oc, _, kh, kw = w_shape
    pads = list(pads) if pads is not None else [0, 0, 0, 0]
    return ConvDesc(n=n, c=c, h=h, w=w, oc=oc, kh=kh, kw=kw, group=group,
                    stride_h=strides[0], stride_w=strides[1],
                    pad_top=pads[0], pad_left=pads[1], pad_bottom=pads[2], pad_right=pads[3],
                    dil_h=dilations[0], dil_w=dilations[1],
                    in_layout=_LAYOUTS[in_layout], out_layout=_LAYOUTS[out_layout],
                    post_op=_POSTS[post] if not isinstance(post, int) else post,
                    post_a=post_a, post_b=post_b, requant=requant)


def conv_out_hw(h, w, kh, kw, strides, pads, dilations):
    oh = (h + pads[0] + pads[2] - (dilations[0] * (kh - 1) + 1)) // strides[0] + 1
    ow = (w + pads[1] + pads[3] - (dilations[1] * (kw - 1) + 1)) // strides[1] + 1
    return oh, ow


class QLinearConv(Operator):
    """ONNX QLinearConv (u8 activations, s8 weights, u8 output).

    x_shape is the logical NCHW shape [n, c, h, w]; in_layout / out_layout
    give the physical layout (nnr's memory_layout_t NCHW or NHWC).
    fused_relu mirrors nnr's post_fn being set by fuse_post_ops, which
    raises the lower clamp to y_zp (QLinearConv.cpp:419).
    """
    op_type = "QLinearConv"

    def __init__(self, x_shape: Sequence[int], w: np.ndarray, w_scale, w_zp, bias, x_scale: float, x_zp: int,
                 y_scale: float, y_zp: int, strides=(1, 1), pads=(0, 0, 0, 0), dilations=(1, 1), group: int = 1,
                 in_layout="NCHW", out_layout="NCHW", fused_relu: bool = False, requant: int = RQ_AUTO):
        super().__init__()
        w = np.ascontiguousarray(w, dtype=np.int8)
        self.x_shape = tuple(int(v) for v in x_shape)
        self.w_shape = w.shape
        self.strides, self.pads, self.dilations = tuple(strides), tuple(pads), tuple(dilations)
        self.in_layout, self.out_layout = in_layout, out_layout
        self.desc = conv_desc(self.x_shape, w.shape, strides, pads, dilations, group, in_layout, out_layout,
                              1 if fused_relu else 0, 0.0, 0.0, requant)
        ws_arr, ws_p = _host(np.atleast_1d(w_scale), np.float32)
        zp_arr, zp_p = _host(None if w_zp is None else np.atleast_1d(w_zp), np.int8)
        b_arr, b_p = _host(bias, np.int32)
        call("nnrcu_qlinearconv_create", C.byref(self.desc), w.ctypes.data_as(C.c_void_p), ws_p, ws_arr.size,
             zp_p, 0 if zp_arr is None else zp_arr.size, b_p, float(x_scale), int(x_zp), float(y_scale), int(y_zp),
             C.byref(self._op))
        n, c, h, wd = self.x_shape
        oh, ow = conv_out_hw(h, wd, w.shape[2], w.shape[3], self.strides, self.pads, self.dilations)
        self.y_shape = (n, w.shape[0], oh, ow) if out_layout == "NCHW" else (n, oh, ow, w.shape[0])
        # the library's space-to-depth form (stride 2 over <= 4 channels), which
        # accepts a fused QuantizeLinear (exec_quantize)
        self.space_to_depth = (c * 4 <= 16 and self.strides == (2, 2) and self.dilations == (1, 1)
                               and w.shape[2] * w.shape[3] > 1 and group == 1)

    def exec(self, x: torch.Tensor, y: Optional[torch.Tensor] = None, workspace=None, stream=None) -> torch.Tensor:
        if y is None:
            y = torch.empty(self.y_shape, dtype=torch.uint8, device=x.device)
        ws, ws_p = self._workspace(workspace, x.device)
        call("nnrcu_qlinearconv_run", self._op, _ptr(x), _ptr(y), ws_p, C.c_void_p(_stream(stream)))
        return y

    def input_padding(self):
        """(top, left, bottom, right) border of the x_zp-padded input copy this
        op makes in its workspace, or zeros (nnrcu_qlinearconv_input_padding)."""
        pads = (C.c_int * 4)()
        call("nnrcu_qlinearconv_input_padding", self._op, pads)
        return tuple(int(v) for v in pads)

    def set_padded_io(self, in_padded: bool = False, out_pads=(0, 0, 0, 0)) -> None:
        """Read an already padded input / write into a padded output buffer
        (nnrcu_qlinearconv_set_padded_io)."""
        call("nnrcu_qlinearconv_set_padded_io", self._op, 1 if in_padded else 0, *[int(v) for v in out_pads])

    def exec_quantize(self, x: torch.Tensor, x_scale: float, x_zp: int, y: Optional[torch.Tensor] = None,
                      workspace=None, stream=None) -> torch.Tensor:
        """QuantizeLinear(x fp32, x_scale, x_zp) followed by this QLinearConv in
        one call (nnrcu_qlinearconv_run_quantize)."""
        if y is None:
            y = torch.empty(self.y_shape, dtype=torch.uint8, device=x.device)
        ws, ws_p = self._workspace(workspace, x.device)
        call("nnrcu_qlinearconv_run_quantize", self._op, _ptr(x), float(x_scale), int(x_zp), _ptr(y), ws_p,
             C.c_void_p(_stream(stream)))
        return y


class QLinearMatMul(Operator):
    """ONNX QLinearMatMul with a constant 2-D B [k, n] (u8 A, s8 B, u8 Y).
    A's leading dims are folded into m (rows)."""
    op_type = "QLinearMatMul"

    def __init__(self, m: int, b: np.ndarray, a_scale, a_zp, b_scale, b_zp, y_scale, y_zp):
        super().__init__()
        b = np.ascontiguousarray(b, dtype=np.int8)
        k, n = b.shape
        self.m, self.k, self.n = int(m), int(k), int(n)
        call("nnrcu_qlinearmatmul_create", self.m, self.k, self.n, float(a_scale), int(a_zp),
             b.ctypes.data_as(C.c_void_p), float(b_scale), int(b_zp), float(y_scale), int(y_zp), C.byref(self._op))

    def exec(self, a: torch.Tensor, y: Optional[torch.Tensor] = None, workspace=None, stream=None) -> torch.Tensor:
        if y is None:
            y = torch.empty((self.m, self.n), dtype=torch.uint8, device=a.device)
        ws, ws_p = self._workspace(workspace, a.device)
        call("nnrcu_qlinearmatmul_run", self._op, _ptr(a), _ptr(y), ws_p, C.c_void_p(_stream(stream)))
        return y


class Conv(Operator):
    """ONNX Conv, fp32 (Conv+BN already folded by nnr's fuse_conv_bn), with
    the fused post-op (post in Relu/Clip/HardSwish/Sigmoid/LeakyRelu/Tanh)."""
    op_type = "Conv"

    def __init__(self, x_shape, w: np.ndarray, bias=None, strides=(1, 1), pads=(0, 0, 0, 0), dilations=(1, 1),
                 group: int = 1, in_layout="NCHW", out_layout="NCHW", post=None, post_a=0.0, post_b=0.0):
        super().__init__()
        w = np.ascontiguousarray(w, dtype=np.float32)
        self.x_shape = tuple(int(v) for v in x_shape)
        self.desc = conv_desc(self.x_shape, w.shape, strides, pads, dilations, group, in_layout, out_layout, post,
                              post_a, post_b, 0)
        b_arr, b_p = _host(bias, np.float32)
        call("nnrcu_conv_f32_create", C.byref(self.desc), w.ctypes.data_as(C.c_void_p), b_p, C.byref(self._op))
        n, c, h, wd = self.x_shape
        oh, ow = conv_out_hw(h, wd, w.shape[2], w.shape[3], tuple(strides), tuple(pads), tuple(dilations))
        self.y_shape = (n, w.shape[0], oh, ow) if out_layout == "NCHW" else (n, oh, ow, w.shape[0])

    def exec(self, x, y=None, residual=None, workspace=None, stream=None):
        if y is None:
            y = torch.empty(self.y_shape, dtype=torch.float32, device=x.device)
        ws, ws_p = self._workspace(workspace, x.device)
        call("nnrcu_conv_f32_run", self._op, _ptr(x), _ptr(y), _ptr(residual), ws_p, C.c_void_p(_stream(stream)))
        return y


class Gemm(Operator):
    """ONNX Gemm with a constant B: Y = post(alpha*op(A)op(B) + beta*C)."""
    op_type = "Gemm"

    def __init__(self, m, b: np.ndarray, c=None, alpha=1.0, beta=1.0, trans_a=0, trans_b=0, post=None, post_a=0.0,
                 post_b=0.0, precision: int = 0):
        """precision: PREC_SPLIT_BF16 (fp32 emulation) or PREC_BF16 (nnr's
        fp32 MatMul on AVX-512 BF16 hosts: bf16-rounded operands)."""
        super().__init__()
        b = np.ascontiguousarray(b, dtype=np.float32)
        n, k = (b.shape[0], b.shape[1]) if trans_b else (b.shape[1], b.shape[0])
        self.m, self.n, self.k = int(m), int(n), int(k)
        c_arr, c_p = _host(c, np.float32)
        c_rows = 0
        if c_arr is not None:
            c_rows = 1 if c_arr.size == n else (self.m if c_arr.size == self.m * n else -1)
            if c_rows < 0:
                raise ValueError("Gemm C must be [n] or [m, n]")
        call("nnrcu_gemm_f32_create_ex", self.m, self.n, self.k, int(trans_a), int(trans_b), float(alpha), float(beta),
             b.ctypes.data_as(C.c_void_p), c_p, c_rows, _POSTS[post] if not isinstance(post, int) else post,
             float(post_a), float(post_b), int(precision), C.byref(self._op))

    def exec(self, a, y=None, workspace=None, stream=None):
        if y is None:
            y = torch.empty((self.m, self.n), dtype=torch.float32, device=a.device)
        ws, ws_p = self._workspace(workspace, a.device)
        call("nnrcu_gemm_f32_run", self._op, _ptr(a), _ptr(y), ws_p, C.c_void_p(_stream(stream)))
        return y


class MatMul(Gemm):
    """ONNX MatMul with a constant 2-D B [k, n]: leading dims of A fold into m
    (MatMul.cpp:156-172)."""
    op_type = "MatMul"

    def __init__(self, m, b: np.ndarray, post=None, post_a=0.0, post_b=0.0, precision: int = 0):
        super().__init__(m, b, None, 1.0, 0.0, 0, 0, post, post_a, post_b, precision)


def matmul_broadcast(a_shape, b_shape):
    """nnr's MatMul shapes (MatMul.cpp:32-94): a 1-D A is [1, k], a 1-D B
    [k, 1] (the unit dims are kept in the output), batch dims broadcast
    numpy-style. Returns (out_shape, m, n, k, [(a_off, b_off)] per output
    batch in row-major order, offsets in elements)."""
    ad = [1, a_shape[0]] if len(a_shape) == 1 else list(a_shape)
    bd = [b_shape[0], 1] if len(b_shape) == 1 else list(b_shape)
    if ad[-1] != bd[-2]:
        raise ValueError(f"MatMul: inner dims {ad[-1]} and {bd[-2]} differ")
    nd = max(len(ad), len(bd))
    m, k, n = ad[-2], ad[-1], bd[-1]
    dims = [0] * nd
    dims[-2], dims[-1] = m, n
    for i in range(3, nd + 1):
        al = ad[-i] if i <= len(ad) else 1
        bl = bd[-i] if i <= len(bd) else 1
        if al != bl and al > 1 and bl > 1:
            raise ValueError("MatMul: batch dims do not broadcast")
        dims[-i] = max(al, bl)
    nb = nd - 2
    a_str, b_str = [0] * nb, [0] * nb
    sa, sb = m * k, k * n
    for i in range(nb - 1, -1, -1):
        ai, bi = i - (nb - (len(ad) - 2)), i - (nb - (len(bd) - 2))
        if ai >= 0 and ad[ai] > 1:
            a_str[i], sa = sa, sa * ad[ai]
        if bi >= 0 and bd[bi] > 1:
            b_str[i], sb = sb, sb * bd[bi]
    offs = []
    for idx in np.ndindex(*dims[:nb]) if nb else [()]:
        offs.append((sum(i * s for i, s in zip(idx, a_str)), sum(i * s for i, s in zip(idx, b_str))))
    return tuple(dims), m, n, k, offs


def matmul_f32(a: torch.Tensor, b: torch.Tensor, post=None, post_a=0.0, post_b=0.0, stream=None) -> torch.Tensor:
    """ONNX MatMul of two fp32 device tensors computed at run time (nnr's
    MatMul_operator with a non-initializer B), through nnrcu_matmul_f32_run.
    Runs of output batches whose A and B offsets advance by fixed strides go
    to one call."""
    a, b = a.contiguous(), b.contiguous()
    shape, m, n, k, offs = matmul_broadcast(tuple(a.shape), tuple(b.shape))
    y = torch.empty(shape, dtype=torch.float32, device=a.device)
    ws_bytes = C.c_size_t()
    call("nnrcu_matmul_f32_workspace", m, n, k, C.byref(ws_bytes))
    ws = torch.empty(max(ws_bytes.value, 1), dtype=torch.uint8, device=a.device)
    code = _POSTS[post] if not isinstance(post, int) else post
    i = 0
    while i < len(offs):
        j = i + 1
        sa = offs[j][0] - offs[i][0] if j < len(offs) else 0
        sb = offs[j][1] - offs[i][1] if j < len(offs) else 0
        while j < len(offs) and offs[j][0] - offs[j - 1][0] == sa and offs[j][1] - offs[j - 1][1] == sb \
                and sa >= 0 and sb >= 0:
            j += 1
        call("nnrcu_matmul_f32_run", C.c_void_p(a.data_ptr() + 4 * offs[i][0]), C.c_void_p(b.data_ptr() + 4 * offs[i][1]),
             C.c_void_p(y.data_ptr() + 4 * i * m * n), j - i, m, n, k, sa, sb, code, float(post_a), float(post_b),
             C.c_void_p(ws.data_ptr()), ws_bytes.value, C.c_void_p(_stream(stream)))
        i = j
    return y


def matmul_half(a: torch.Tensor, b: torch.Tensor, post=None, post_a=0.0, post_b=0.0, stream=None) -> torch.Tensor:
    """matmul_f32 for two bf16 (or two fp16) device tensors (nnr's 16-bit
    MatMul: fp32 products and sums, the result rounded to the type), through
    nnrcu_matmul_half_run."""
    if a.dtype != b.dtype or a.dtype not in (torch.bfloat16, torch.float16):
        raise TypeError("matmul_half: two bf16 or two fp16 tensors")
    dtype = DT_BF16 if a.dtype == torch.bfloat16 else DT_F16
    a, b = a.contiguous(), b.contiguous()
    shape, m, n, k, offs = matmul_broadcast(tuple(a.shape), tuple(b.shape))
    y = torch.empty(shape, dtype=a.dtype, device=a.device)
    ws_bytes = C.c_size_t()
    call("nnrcu_matmul_half_workspace", m, n, k, C.byref(ws_bytes))
    ws = torch.empty(max(ws_bytes.value, 1), dtype=torch.uint8, device=a.device)
    code = _POSTS[post] if not isinstance(post, int) else post
    for i, (ao, bo) in enumerate(offs):
        call("nnrcu_matmul_half_run", C.c_void_p(a.data_ptr() + 2 * ao), C.c_void_p(b.data_ptr() + 2 * bo),
             C.c_void_p(y.data_ptr() + 2 * i * m * n), 1, m, n, k, 0, 0, dtype, code, float(post_a), float(post_b),
             C.c_void_p(ws.data_ptr()), ws_bytes.value, C.c_void_p(_stream(stream)))
    return y


PREC_SPLIT_BF16, PREC_BF16 = 0, 1
DT_BF16, DT_F16 = 1, 2
_HALF_TORCH = {DT_BF16: "bfloat16", DT_F16: "float16"}


def _bits16(arr, dtype):
    """Raw 16-bit values of a torch bf16/fp16 tensor or a numpy array
    (float16, or uint16 bit patterns)."""
    if arr is None:
        return None
    if isinstance(arr, torch.Tensor):
        return arr.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    a = np.asarray(arr)
    return np.ascontiguousarray(a.view(np.uint16) if a.dtype == np.float16 else a.astype(np.uint16))


class ConvHalf(Operator):
    """ONNX Conv on bf16 or fp16 tensors (nnr's 16-bit I/O path,
    Conv_exec_entry.h:188-381): w and bias of the same type."""
    op_type = "Conv"

    def __init__(self, x_shape, w, bias=None, dtype=DT_BF16, strides=(1, 1), pads=(0, 0, 0, 0), dilations=(1, 1),
                 in_layout="NCHW", out_layout="NCHW", post=None, post_a=0.0, post_b=0.0, group=1):
        super().__init__()
        wb = _bits16(w, dtype)
        self.dtype = dtype
        self.x_shape = tuple(int(v) for v in x_shape)
        self.desc = conv_desc(self.x_shape, wb.shape, strides, pads, dilations, group, in_layout, out_layout,
                              post, post_a, post_b, 0)
        bb = _bits16(bias, dtype)
        call("nnrcu_conv_half_create", C.byref(self.desc), int(dtype), wb.ctypes.data_as(C.c_void_p),
             None if bb is None else bb.ctypes.data_as(C.c_void_p), C.byref(self._op))
        self._keep = (wb, bb)
        n, c, h, wd = self.x_shape
        oh, ow = conv_out_hw(h, wd, wb.shape[2], wb.shape[3], tuple(strides), tuple(pads), tuple(dilations))
        oc = wb.shape[0]
        self.y_shape = (n, oc, oh, ow) if out_layout == "NCHW" else (n, oh, ow, oc)

    def exec(self, x, y=None, workspace=None, stream=None):
        if y is None:
            y = torch.empty(self.y_shape, dtype=getattr(torch, _HALF_TORCH[self.dtype]), device=x.device)
        ws, ws_p = self._workspace(workspace, x.device)
        call("nnrcu_conv_half_run", self._op, _ptr(x), _ptr(y), ws_p, C.c_void_p(_stream(stream)))
        return y


class GemmHalf(Operator):
    """ONNX Gemm on bf16 or fp16 tensors with a constant B (Gemm.cpp:297-513)."""
    op_type = "Gemm"

    def __init__(self, m, b, c=None, dtype=DT_BF16, beta=1.0, trans_a=0, trans_b=0, post=None, post_a=0.0,
                 post_b=0.0):
        super().__init__()
        bb = _bits16(b, dtype)
        n, k = (bb.shape[0], bb.shape[1]) if trans_b else (bb.shape[1], bb.shape[0])
        self.m, self.n, self.k, self.dtype = int(m), int(n), int(k), dtype
        cb = _bits16(c, dtype)
        c_rows = 0 if cb is None else (1 if cb.size == n else self.m)
        call("nnrcu_gemm_half_create", self.m, self.n, self.k, int(trans_a), int(trans_b), 1.0, float(beta), int(dtype),
             bb.ctypes.data_as(C.c_void_p), None if cb is None else cb.ctypes.data_as(C.c_void_p), c_rows,
             _POSTS[post] if not isinstance(post, int) else post, float(post_a), float(post_b), C.byref(self._op))
        self._keep = (bb, cb)

    def exec(self, a, y=None, workspace=None, stream=None):
        if y is None:
            y = torch.empty((self.m, self.n), dtype=getattr(torch, _HALF_TORCH[self.dtype]), device=a.device)
        ws, ws_p = self._workspace(workspace, a.device)
        call("nnrcu_gemm_half_run", self._op, _ptr(a), _ptr(y), ws_p, C.c_void_p(_stream(stream)))
        return y
