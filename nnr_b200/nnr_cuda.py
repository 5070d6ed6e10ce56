"""nnr with its CUDA backend, from Python (nnr_b200/nnr_backend/libnnr_cuda.so).

An application of nnr loads an ONNX model into a context_t, prepares it and
runs it (nnr.h:482-590). With context_t::preferred_backend = CUDA, nnr's
registry resolves Conv, QLinearConv, QLinearMatMul, Gemm, MatMul and the QDQ
glue operators to the B200 operators of nnr_b200/nnr_backend, and nnr's own
loader, fusion passes (fuse_qdq_compute, fuse_post_ops), layout assignment
and memory planner shape the device run. This module is that application
path through the library's C entry points.

    m = NnrCudaModel(onnx_bytes, device=0)
    m.set("input", x); m.run(); y = m.get("logits")
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

LIB = Path(__file__).resolve().parent / "nnr_backend" / "libnnr_cuda.so"
_DT = {1: np.float32, 2: np.float64, 3: np.uint16, 4: np.uint16, 5: np.int8, 7: np.int32, 8: np.int64, 9: np.uint8}
# (FLOAT16 and BFLOAT16 tensors are returned as their uint16 bit patterns)
NCHW, NHWC = 0, 1
STATS = ("runs", "graph_replays", "h2d_bytes", "d2h_bytes", "device_ops", "host_ops", "host_glue",
         "arena_bytes", "const_bytes", "slots")

_lib = None


def available() -> bool:
    return LIB.exists()


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            raise FileNotFoundError(f"{LIB} is not built: make -C nnr_b200/nnr_backend NNR_SRC=<nnr>/src")
        _lib = C.CDLL(str(LIB))
        _lib.nnrcuda_load.restype = C.c_void_p
        _lib.nnrcuda_load.argtypes = [C.c_char_p, C.c_size_t, C.c_int, C.c_int, C.c_int]
        _lib.nnrcuda_free.argtypes = [C.c_void_p]
        _lib.nnrcuda_run.argtypes = [C.c_void_p]
        _lib.nnrcuda_num_nodes.argtypes = [C.c_void_p]
        _lib.nnrcuda_set_input.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_size_t]
        _lib.nnrcuda_input_buffer.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(C.c_void_p), C.POINTER(C.c_size_t)]
        _lib.nnrcuda_get.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_size_t]
        _lib.nnrcuda_tensor_info.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(C.c_int), C.POINTER(C.c_int),
                                             C.POINTER(C.c_int), C.POINTER(C.c_int)]
        _lib.nnrcuda_node.argtypes = [C.c_void_p, C.c_int, C.c_char_p, C.c_size_t, C.POINTER(C.c_int),
                                      C.POINTER(C.c_int)]
        _lib.nnrcuda_stats.argtypes = [C.c_void_p, C.POINTER(C.c_int64)]
        _lib.nnrcuda_last_error.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t]
    return _lib


class NnrCudaModel:
    """One nnr context on one GPU with preferred_backend = CUDA."""

    def __init__(self, model: bytes, device: int = 0, memory_planning: bool = False, graphs: bool = True):
        """memory_planning: nnr's host memory planner. With the graph on the
        device, the plan only decides which tensors share a device slot,
        while nnr's run() still clears every planned host slot on each call
        (memory_planner.cpp zero_pool: ~15 ms per ResNet-50 batch of 32), so
        it is off by default here."""
        self._buf = model  # nnr's tensors may alias the proto buffer: keep it alive
        self.h = lib().nnrcuda_load(model, len(model), device, int(memory_planning), int(graphs))
        if not self.h:
            raise RuntimeError("nnr could not load or prepare the model")

    def error(self) -> str:
        buf = C.create_string_buffer(1024)
        lib().nnrcuda_last_error(self.h, buf, 1024)
        return buf.value.decode()

    def set(self, name: str, arr: np.ndarray) -> None:
        arr = np.ascontiguousarray(arr)
        if lib().nnrcuda_set_input(self.h, name.encode(), arr.ctypes.data, arr.nbytes) != 0:
            raise RuntimeError(f"nnr: cannot set input {name}")

    def input_array(self, name: str) -> np.ndarray:
        """A writable numpy view of a graph input's own host buffer (filled in
        place, no copy through set()); valid until the model is closed."""
        shape, ty, _ = self.info(name)
        ptr, nbytes = C.c_void_p(), C.c_size_t()
        if lib().nnrcuda_input_buffer(self.h, name.encode(), C.byref(ptr), C.byref(nbytes)) != 0:
            raise KeyError(name)
        buf = (C.c_uint8 * nbytes.value).from_address(ptr.value)
        return np.frombuffer(buf, dtype=_DT[ty]).reshape(shape)

    def run(self) -> None:
        if lib().nnrcuda_run(self.h) != 0:
            raise RuntimeError(f"nnr run() failed: {self.error()}")

    def info(self, name: str):
        dims = (C.c_int * 8)()
        nd, ty, fmt = C.c_int(), C.c_int(), C.c_int()
        if lib().nnrcuda_tensor_info(self.h, name.encode(), dims, C.byref(nd), C.byref(ty), C.byref(fmt)) != 0:
            raise KeyError(name)
        return tuple(dims[:nd.value]), ty.value, fmt.value

    def get(self, name: str) -> np.ndarray:
        """A tensor's host copy (graph outputs, host-read tensors), in NCHW."""
        shape, ty, fmt = self.info(name)
        out = np.empty(shape, _DT[ty])
        if lib().nnrcuda_get(self.h, name.encode(), out.ctypes.data, out.nbytes) != 0:
            raise RuntimeError(f"nnr: cannot read {name}")
        if fmt == NHWC and len(shape) == 4:
            n, c, h, w = shape
            out = np.ascontiguousarray(out.reshape(n, h, w, c).transpose(0, 3, 1, 2))
        return out

    def nodes(self):
        """(op_type, skip, folded, on_device, output layout) per node after nnr's passes."""
        out = []
        buf = C.create_string_buffer(64)
        fl, fmt = C.c_int(), C.c_int()
        for i in range(lib().nnrcuda_num_nodes(self.h)):
            lib().nnrcuda_node(self.h, i, buf, 64, C.byref(fl), C.byref(fmt))
            out.append((buf.value.decode(), bool(fl.value & 1), bool(fl.value & 2), bool(fl.value & 4), fmt.value))
        return out

    def active(self):
        return [n for n in self.nodes() if not n[1] and not n[2]]

    def stats(self) -> dict:
        v = (C.c_int64 * 10)()
        if lib().nnrcuda_stats(self.h, v) != 0:
            return {}
        return dict(zip(STATS, list(v)))

    def close(self) -> None:
        if self.h:
            lib().nnrcuda_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass
