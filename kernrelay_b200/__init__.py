"""KernRelay TP-MLP prefill hot path for B200 (sm_100a).

The product is libkernrelay.so (CUDA kernels + C++ runtime + C ABI in
include/kernrelay.h and include/kernrelay_b200.h).  Python modules here are thin
ctypes shims (libapi mirrors the reference's python/kernrelay/libapi.py) and
tooling (build, model directory generator).
"""
__all__ = ["libapi", "build", "model_gen"]
