"""naivediffusion_b200 — NaiveDiffusion's denoiser forward step on B200.

The product is the C-ABI library libnd_denoise.so (include/nd_denoise.h):
hand-written sm_100a kernels (tcgen05/TMA GEMM with fused epilogues, tcgen05
flash attention, adaLN modulation, RMSNorm, GEMV) and the denoiser plug-in
that replaces the reference's DirectML graphs behind IDenoiser. This package
is the Python host side: ctypes bindings (_lib), op wrappers over torch
tensors (ops) and the IDenoiser mirror (denoiser).
"""
from . import _lib  # noqa: F401

__all__ = ["_lib"]
