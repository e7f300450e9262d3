"""tensor-compiler-webgpu_b200: a B200-native backend for the compiler's fused-kernel hot path.

The host side restates the compiler's kept layers (IR, autodiff, fusion pass,
step builders); the backend replaces the reference's ``src/gpu`` lowering,
code generator and runtime with hand-written sm_100a CUDA templates,
instantiated per fused node through NVRTC by the C-ABI library
``libtcb200.so`` and driven here through ctypes.

Import with ``importlib.import_module("tensor-compiler-webgpu_b200")``.
"""
from . import ir, autodiff, rng, fuse, steps  # noqa: F401

__all__ = ["ir", "autodiff", "rng", "fuse", "steps"]
