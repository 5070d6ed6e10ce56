"""nnr's own CPU runtime, loaded from oracle/_ref/libnnr_cpu.so (test
infrastructure only: the checker the restatement is pinned to, and the CPU
reference timing). Built by `make -C oracle nnr NNR_SRC=<nnr>/src` from the
nnr sources where they lie; absent when they were not available.

Usage:
    net = NnrModel(onnx_bytes)          # context_t::load + prepare
    net.set("x", x); net.run(); y = net.get("y")
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

LIB = Path(__file__).resolve().parent / "_ref" / "libnnr_cpu.so"

# nnr data_type_t (nnr.h:21-58) -> numpy
_DT = {1: np.float32, 2: np.float64, 3: np.uint16, 4: np.uint16, 5: np.int8, 7: np.int32, 8: np.int64, 9: np.uint8}
# (FLOAT16 and BFLOAT16 tensors are returned as their uint16 bit patterns)
NHWC, BLOCKED_16 = 1, 3  # memory_layout_t

_lib = None


def available() -> bool:
    return LIB.exists()


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            raise FileNotFoundError(f"{LIB} not built (make -C oracle nnr NNR_SRC=...)")
        _lib = C.CDLL(str(LIB))
        _lib.nnrh_load.restype = C.c_void_p
        _lib.nnrh_load.argtypes = [C.c_char_p, C.c_size_t, C.c_int, C.c_int, C.c_int]
        for f in ("nnrh_prepare", "nnrh_run", "nnrh_num_nodes"):
            getattr(_lib, f).argtypes = [C.c_void_p]
        _lib.nnrh_free.argtypes = [C.c_void_p]
        _lib.nnrh_set_input.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_size_t]
        _lib.nnrh_get.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_size_t]
        _lib.nnrh_get_raw.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_size_t]
        _lib.nnrh_tensor_info.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(C.c_int), C.POINTER(C.c_int),
                                          C.POINTER(C.c_int), C.POINTER(C.c_int)]
        _lib.nnrh_node.argtypes = [C.c_void_p, C.c_int, C.c_char_p, C.c_size_t, C.POINTER(C.c_int)]
    return _lib


def set_threads(n: int) -> None:
    """nnr's worker count (context_t::set_num_threads, before prepare/run)."""
    lib().nnrh_set_threads(int(n))


class NnrModel:
    def __init__(self, model: bytes, backend: int = 0, memory_planning: bool = True, no_blocked: bool = False):
        """no_blocked turns nnr's nChw16c layout off (context_t::set_no_blocked)."""
        self._buf = model  # nnr's tensors may alias the proto buffer: keep it alive
        self.h = lib().nnrh_load(model, len(model), backend, int(memory_planning), int(no_blocked))
        if not self.h:
            raise RuntimeError("nnr failed to load the model")
        if lib().nnrh_prepare(self.h) != 0:
            raise RuntimeError("nnr prepare() failed")

    def set(self, name: str, arr: np.ndarray) -> None:
        arr = np.ascontiguousarray(arr)
        if lib().nnrh_set_input(self.h, name.encode(), arr.ctypes.data, arr.nbytes) != 0:
            raise RuntimeError(f"nnr: cannot set input {name}")

    def run(self) -> None:
        if lib().nnrh_run(self.h) != 0:
            raise RuntimeError("nnr run() failed")

    def info(self, name: str):
        dims = (C.c_int * 8)()
        nd, ty, fmt = C.c_int(), C.c_int(), C.c_int()
        if lib().nnrh_tensor_info(self.h, name.encode(), dims, C.byref(nd), C.byref(ty), C.byref(fmt)) != 0:
            raise KeyError(name)
        return tuple(dims[:nd.value]), ty.value, fmt.value

    def get(self, name: str) -> np.ndarray:
        """The tensor as nnr holds it; a 4-D NHWC or nChw16c tensor is
        returned in NCHW."""
        shape, ty, fmt = self.info(name)
        if fmt == BLOCKED_16 and len(shape) == 4:
            n, c, h, w = shape
            cp = (c + 15) // 16 * 16
            blk = np.empty((n, cp // 16, h, w, 16), _DT[ty])
            if lib().nnrh_get_raw(self.h, name.encode(), blk.ctypes.data, blk.nbytes) != 0:
                raise RuntimeError(f"nnr: cannot read {name}")
            return np.ascontiguousarray(blk.transpose(0, 1, 4, 2, 3).reshape(n, cp, h, w)[:, :c])
        out = np.empty(shape, _DT[ty])
        if lib().nnrh_get(self.h, name.encode(), out.ctypes.data, out.nbytes) != 0:
            raise RuntimeError(f"nnr: cannot read {name}")
        if fmt == NHWC and len(shape) == 4:
            n, c, h, w = shape
            out = np.ascontiguousarray(out.reshape(n, h, w, c).transpose(0, 3, 1, 2))
        return out

    def nodes(self):
        """(op_type, skip, folded) for every graph node after nnr's passes."""
        out = []
        buf = C.create_string_buffer(64)
        fl = C.c_int()
        for i in range(lib().nnrh_num_nodes(self.h)):
            lib().nnrh_node(self.h, i, buf, 64, C.byref(fl))
            out.append((buf.value.decode(), bool(fl.value & 1), bool(fl.value & 2)))
        return out

    def close(self) -> None:
        if self.h:
            lib().nnrh_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass
