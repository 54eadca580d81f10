"""Op-level host API over torch device tensors (torch is only the allocator
and stream here; every op runs the library's sm_100a kernels through the C
ABI in include/nd_denoise.h).

These mirror the operator checks of the reference's smoke command
(src/NaiveDiffusion.Cli/SmokeTest.cs) and the layer helpers they exercise
(src/NaiveDiffusion/Graph/Layers.cs, Graph/Transformer.cs).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._lib import LinearArgs, check, lib

_DT = {torch.bfloat16: _lib.ND_BF16, torch.float16: _lib.ND_F16, torch.float32: _lib.ND_F32}


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def sync() -> None:
    """Synchronize the current stream and raise on a kernel's timed-out wait."""
    check(lib().nd_op_sync(C.c_void_p(_stream())))


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None, *,
           epilogue: int = _lib.ND_EPI_STORE, out: torch.Tensor | None = None,
           residual: torch.Tensor | None = None, gate: torch.Tensor | None = None,
           group_split: int | None = None, qk_norm: torch.Tensor | None = None,
           rope_cos: torch.Tensor | None = None, rope_sin: torch.Tensor | None = None,
           qk_cols: int = 0, eps: float = 1e-6) -> torch.Tensor:
    """y = x . W^T + bias with a fused epilogue (Layers.Linear, Graph/Layers.cs:131-160).

    weight is [groups * out, in]; rows >= group_split use the second group.
    Residual epilogues update `residual` (fp32) in place and return it.
    """
    rows, k = x.shape
    groups = 1 if group_split is None or group_split >= rows else 2
    n = weight.shape[0] // groups
    resid_epi = epilogue in (_lib.ND_EPI_RESIDUAL_GATE, _lib.ND_EPI_RESIDUAL_ADD, _lib.ND_EPI_STORE_F32)
    if resid_epi:
        if residual is None:
            residual = torch.empty(rows, n, device=x.device, dtype=torch.float32)
    elif out is None:
        out = torch.empty(rows, n, device=x.device, dtype=x.dtype)
    a = LinearArgs()
    a.dtype = _DT[x.dtype]
    a.epilogue = epilogue
    a.rows, a.in_features, a.out_features = rows, k, n
    a.x, a.ldx = x.data_ptr(), x.stride(0)
    a.weight = weight.data_ptr()
    a.bias = _ptr(bias)
    a.group_split = group_split if group_split is not None else rows
    a.y = _ptr(out)
    a.ldy = out.stride(0) if out is not None else 0
    a.residual = _ptr(residual)
    a.ldr = residual.stride(0) if residual is not None else 0
    a.gate = _ptr(gate)
    a.qk_norm = _ptr(qk_norm)
    a.rope_cos = _ptr(rope_cos)
    a.rope_sin = _ptr(rope_sin)
    a.qk_cols = qk_cols
    a.eps = eps
    check(lib().nd_op_linear(C.byref(a), C.c_void_p(_stream())))
    return residual if resid_epi else out
