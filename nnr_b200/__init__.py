"""nnr_b200: B200-native (sm_100a) backend for nnr's conv/GEMM hot path.

The product is libnnrcu.so (C ABI in include/nnrcu.h). This package holds
its build script (build.py), the ctypes binding (_lib.py) and host-side
operator classes mirroring nnr's operator_t (ops.py). Importing the operator
layer requires the built library; there is no CPU fallback.
"""
__all__ = ["build", "ops"]
