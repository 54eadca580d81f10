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
from ._lib import AttentionArgs, GemvArgs, LinearArgs, ModulateArgs, RmsNormArgs, check, lib

_DT = {torch.bfloat16: _lib.ND_BF16, torch.float16: _lib.ND_F16, torch.float32: _lib.ND_F32}


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _check_out(what: str, t: torch.Tensor, rows: int, cols: int, dtypes, device) -> None:
    """A caller's output tensor must hold what the op writes: the C ABI sees
    only its pointer and row stride."""
    if (t.dim() != 2 or t.shape[0] < rows or t.shape[1] < cols or t.stride(1) != 1 or t.dtype not in dtypes
            or t.device != device):
        raise ValueError(f"{what} must be a 2-D {'/'.join(str(d) for d in dtypes)} tensor of at least "
                         f"[{rows}, {cols}] with unit column stride on {device}, got {tuple(t.shape)} {t.dtype}")


def _check_vec(what: str, t: torch.Tensor | None, n: int, device) -> None:
    if t is not None and (t.dtype != torch.float32 or not t.is_contiguous() or t.numel() < n or t.device != device):
        raise ValueError(f"{what} must be a contiguous float32 tensor of at least {n} values on {device}")


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def sync() -> None:
    """Synchronize the current stream and raise on a kernel's timed-out wait."""
    check(lib().nd_op_sync(C.c_void_p(_stream())))


def wait_probe(limit_ns: int, ctas: int = 1, armed: bool = False) -> None:
    """Launch the bounded-wait probe (nd_op_wait_probe) on the current stream.
    Unarmed, its wait runs out after limit_ns and the next sync() raises
    NdError with ND_ERR_TIMEOUT; armed, it completes at once."""
    check(lib().nd_op_wait_probe(C.c_uint64(limit_ns), ctas, int(armed), C.c_void_p(_stream())))


def to_pairs(t: torch.Tensor) -> torch.Tensor:
    """fp32 [rows, cols] -> the ND_BF16X2 pair [rows, 2 * cols] (hi = bf16(t),
    lo = bf16(t - hi)), the operand format of fp32-compute GEMMs."""
    hi = t.float().bfloat16()
    lo = (t.float() - hi.float()).bfloat16()
    return torch.cat([hi, lo], dim=1).contiguous()


def from_pairs(p: torch.Tensor) -> torch.Tensor:
    """The fp32 value hi + lo of an ND_BF16X2 pair [rows, 2 * cols]."""
    c = p.shape[1] // 2
    return p[:, :c].float() + p[:, c:].float()


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None, *,
           epilogue: int = _lib.ND_EPI_STORE, out: torch.Tensor | None = None,
           residual: torch.Tensor | None = None, gate: torch.Tensor | None = None,
           group_split: int | None = None, qk_norm: torch.Tensor | None = None,
           rope_cos: torch.Tensor | None = None, rope_sin: torch.Tensor | None = None,
           qk_cols: int = 0, eps: float = 1e-6, scales: torch.Tensor | None = None,
           quant_group: int = 32, norm_span: int = 0, rope_period: int = 0,
           gate_stride: int = 0, pairs: bool = False, shared_weights: bool = False) -> torch.Tensor:
    """y = x . W^T + bias with a fused epilogue (Layers.Linear, Graph/Layers.cs:131-160).

    weight is [groups * out, in]; rows >= group_split use the second group.
    Residual epilogues update `residual` (fp32) in place and return it.
    An int8 weight (with `scales`, fp16 or fp32, `quant_group` 32 or 0 = per
    output channel) is widened inside the GEMM (BlockQuantizer's scheme).
    pairs=True: fp32 compute on ND_BF16X2 operands (x [rows, 2 * in], weight
    [groups * out, 2 * in]); the output is a pair [rows, 2 * out], or fp32
    [rows, out] for QK_NORM_ROPE.
    ND_EPI_SWIGLU: weight is the fused [gate; up] matrix [2F, in]; the output
    is [rows, F]. shared_weights=True: one weight matrix for every row, the
    bias / gate vectors chosen per row by group_split (any row).
    """
    rows, k = x.shape
    if pairs:
        k //= 2
    groups = 1 if shared_weights or group_split is None or group_split >= rows else 2
    n = weight.shape[0] // groups
    if epilogue in (_lib.ND_EPI_SWIGLU, _lib.ND_EPI_GEGLU):
        n //= 2
    resid_epi = epilogue in (_lib.ND_EPI_RESIDUAL_GATE, _lib.ND_EPI_RESIDUAL_ADD, _lib.ND_EPI_STORE_F32)
    if resid_epi:
        if residual is None:
            residual = torch.empty(rows, n, device=x.device, dtype=torch.float32)
        else:
            _check_out("linear: residual", residual, rows, n, (torch.float32,), x.device)
    elif out is not None:
        if pairs and epilogue == _lib.ND_EPI_QK_NORM_ROPE:
            _check_out("linear: out", out, rows, n, (torch.float32,), x.device)
        elif pairs:
            _check_out("linear: out", out, rows, 2 * n, (torch.bfloat16,), x.device)
        else:
            _check_out("linear: out", out, rows, n, (torch.float16, torch.bfloat16), x.device)
    if out is None and not resid_epi:
        if pairs and epilogue == _lib.ND_EPI_QK_NORM_ROPE:
            out = torch.empty(rows, n, device=x.device, dtype=torch.float32)
        elif pairs:
            out = torch.empty(rows, 2 * n, device=x.device, dtype=torch.bfloat16)
        else:
            out = torch.empty(rows, n, device=x.device, dtype=x.dtype)
    a = LinearArgs()
    a.dtype = _lib.ND_BF16X2 if pairs else _DT[x.dtype]
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
    a.norm_span = norm_span
    a.rope_period = rope_period
    a.gate_stride = gate_stride
    a.shared_weights = 1 if shared_weights else 0
    if weight.dtype == torch.int8:
        a.weight_dtype = _lib.ND_I8
        a.scales = scales.data_ptr()
        a.scale_dtype = _DT[scales.dtype]
        a.quant_group = quant_group
    check(lib().nd_op_linear(C.byref(a), C.c_void_p(_stream())))
    return residual if resid_epi else out


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int, *,
              out: torch.Tensor | None = None, batch: int = 1, key_limit: int = 0,
              causal: bool = False, scale: float = 0.0, head_dim: int = 128,
              out_pairs: bool = False, kv_heads: int = 0,
              workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Flash attention over packed heads (Layers.Attend, Graph/Layers.cs:260-279).

    q: [batch * q_rows, >= heads*128] (row stride q.stride(0)); k, v likewise
    with kv_rows per item. Returns out [batch * q_rows, heads * 128].
    fp32 q/k/v run the fp32 attention; out_pairs then writes an ND_BF16X2 pair.
    kv_heads < heads: grouped-query attention (k, v [rows, kv_heads * head_dim]).
    workspace: a zeroed uint8 tensor from attention_workspace(); with it the
    last partial wave of query tiles is split along the keys.
    """
    q_rows = q.shape[0] // batch
    kv_rows = k.shape[0] // batch
    if out is not None:
        _check_out("attention: out", out, q.shape[0], (2 if out_pairs else 1) * heads * head_dim,
                   (torch.bfloat16,) if out_pairs else (q.dtype,), q.device)
    if out is None:
        if out_pairs:
            out = torch.empty(q.shape[0], 2 * heads * head_dim, device=q.device, dtype=torch.bfloat16)
        else:
            out = torch.empty(q.shape[0], heads * head_dim, device=q.device, dtype=q.dtype)
    a = AttentionArgs()
    a.dtype = _DT[q.dtype]
    a.out_dtype = _lib.ND_BF16X2 if out_pairs else 0
    a.heads, a.head_dim, a.batch = heads, head_dim, batch
    a.q_rows, a.kv_rows, a.key_limit, a.causal = q_rows, kv_rows, key_limit, int(causal)
    a.q, a.ldq = q.data_ptr(), q.stride(0)
    a.k, a.ldk = k.data_ptr(), k.stride(0)
    a.v, a.ldv = v.data_ptr(), v.stride(0)
    a.out, a.ldo = out.data_ptr(), out.stride(0)
    a.scale = scale
    a.kv_heads = kv_heads
    if workspace is not None:
        if workspace.device != q.device or workspace.dtype != torch.uint8 or not workspace.is_contiguous():
            raise ValueError("attention: workspace must be a contiguous uint8 tensor on q's device")
        a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel()
    check(lib().nd_op_attention(C.byref(a), C.c_void_p(_stream())))
    return out


def attention_workspace(head_dim: int = 128, device="cuda") -> torch.Tensor:
    """A zeroed workspace for attention(..., workspace=) on `device` (one per
    stream; the kernel leaves it zeroed)."""
    n = int(lib().nd_attention_workspace_bytes(head_dim))
    if n <= 0:
        raise ValueError(f"attention_workspace: no workspace for head_dim {head_dim}")
    return torch.zeros(n, dtype=torch.uint8, device=device)


def modulate(x: torch.Tensor, shift: torch.Tensor | None, scale: torch.Tensor, *,
             out_dtype=torch.bfloat16, group_split: int | None = None, eps: float = 1e-6,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """LayerNorm(x) * (1 + scale) + shift (Transformer.Modulate, Graph/Transformer.cs:72-80).
    scale/shift: [width] or [2, width] (second row for rows >= group_split)."""
    rows, width = x.shape
    pairs = out_dtype == "pairs"
    groups = 2 if group_split is not None and group_split < rows else 1
    _check_vec("modulate: scale", scale, groups * width, x.device)
    _check_vec("modulate: shift", shift, groups * width, x.device)
    if out is None:
        out = torch.empty(rows, 2 * width if pairs else width, device=x.device,
                          dtype=torch.bfloat16 if pairs else out_dtype)
    else:
        _check_out("modulate: out", out, rows, 2 * width if pairs else width,
                   (torch.bfloat16,) if pairs else (torch.float32, torch.float16, torch.bfloat16), x.device)
    a = ModulateArgs()
    a.x, a.ldx = x.data_ptr(), x.stride(0)
    a.y, a.ldy, a.out_dtype = out.data_ptr(), out.stride(0), (_lib.ND_BF16X2 if pairs else _DT[out.dtype])
    a.rows, a.width = rows, width
    a.shift = _ptr(shift)
    a.scale = scale.data_ptr()
    a.vec_stride = width
    a.group_split = group_split if group_split is not None else rows
    a.eps = eps
    check(lib().nd_op_modulate(C.byref(a), C.c_void_p(_stream())))
    return out


def rmsnorm(x: torch.Tensor, weight: torch.Tensor | None, *, out_dtype=None, plus_one=False,
            eps: float = 1e-6, silu: bool = False) -> torch.Tensor:
    """x * rsqrt(mean(x^2) + eps) * (weight [+ 1]) over rows (CpuMath.RmsNorm),
    then SiLU when silu=True."""
    rows, width = x.shape
    out = torch.empty(rows, width, device=x.device, dtype=out_dtype or x.dtype)
    a = RmsNormArgs()
    a.x, a.ldx, a.in_dtype = x.data_ptr(), x.stride(0), _DT[x.dtype]
    a.y, a.ldy, a.out_dtype = out.data_ptr(), out.stride(0), _DT[out.dtype]
    a.rows, a.width = rows, width
    a.weight = _ptr(weight)
    a.plus_one = int(plus_one)
    a.eps = eps
    a.silu = int(silu)
    check(lib().nd_op_rmsnorm(C.byref(a), C.c_void_p(_stream())))
    return out


def head_norm_rope(x: torch.Tensor, heads: int, head_dim: int, weight: torch.Tensor,
                   cos: torch.Tensor | None = None, sin: torch.Tensor | None = None, eps: float = 1e-6) -> torch.Tensor:
    """In place: per-head RMSNorm * weight then rotate-half RoPE with row r's
    angles (Transformer.HeadNorm + Transformer.Rotate) over x [rows, >= heads * head_dim]."""
    check(lib().nd_op_head_norm_rope(C.c_void_p(x.data_ptr()), _DT[x.dtype], x.stride(0), x.shape[0], heads, head_dim,
                                     C.c_void_p(weight.data_ptr()), _ptr(cos), _ptr(sin), C.c_float(eps),
                                     C.c_void_p(_stream())))
    return x


def gemv(w: torch.Tensor, x: torch.Tensor, bias: torch.Tensor | None = None, *,
         pre_silu: bool = False, act: int = 0, w_pairs: bool = False, x_rows_per_vec: int = 0,
         bias_period: int = 0) -> torch.Tensor:
    """y[b] = act(W . pre(x[b]) + bias) for 1-4 fp32 rows x; W bf16/f16 [n, k]
    (w_pairs: an ND_BF16X2 pair [n, 2k]). x_rows_per_vec > 0: output row j
    reads input vector j // x_rows_per_vec (x holds ceil(n / x_rows_per_vec)
    vectors; y is [1, n]); bias_period > 0: bias index j % bias_period."""
    n, k = w.shape
    if w_pairs:
        k //= 2
    x = x.reshape(-1, k).contiguous()
    y = torch.empty(1 if x_rows_per_vec else x.shape[0], n, device=w.device, dtype=torch.float32)
    a = GemvArgs()
    a.w, a.w_dtype, a.n, a.k = w.data_ptr(), (_lib.ND_BF16X2 if w_pairs else _DT[w.dtype]), n, k
    a.x, a.batch, a.pre_silu = x.data_ptr(), 1 if x_rows_per_vec else x.shape[0], int(pre_silu)
    a.bias, a.act, a.y = _ptr(bias), act, y.data_ptr()
    a.x_rows_per_vec, a.bias_period = x_rows_per_vec, bias_period
    check(lib().nd_op_gemv(C.byref(a), C.c_void_p(_stream())))
    return y


def patchify(latent: torch.Tensor, patch: int, out_dtype=torch.bfloat16) -> torch.Tensor:
    """[B, C, H, W] fp32 -> [B*(H/p)*(W/p), C*p*p] (AnimaDit.Patchify order)."""
    b, c, h, w = latent.shape
    tok = torch.empty(b * (h // patch) * (w // patch), c * patch * patch, device=latent.device,
                      dtype=out_dtype)
    check(lib().nd_op_patchify(latent.data_ptr(), tok.data_ptr(), _DT[out_dtype], b, c, h, w, patch,
                               tok.stride(0), C.c_void_p(_stream())))
    return tok


def unpatchify(tokens: torch.Tensor, shape, patch: int) -> torch.Tensor:
    b, c, h, w = shape
    lat = torch.empty(b, c, h, w, device=tokens.device, dtype=torch.float32)
    check(lib().nd_op_unpatchify(tokens.data_ptr(), tokens.stride(0), lat.data_ptr(), b, c, h, w,
                                 patch, C.c_void_p(_stream())))
    return lat


def tile_gather(latent: torch.Tensor, rows, cols, tile: int) -> torch.Tensor:
    """latent [C, H, W] fp32 -> tiles [len(rows) * len(cols), C, tile, tile],
    tile (i, j) starting at (rows[i], cols[j]) (TiledVae.CopyTile)."""
    if latent.dim() != 3 or latent.dtype != torch.float32:
        raise ValueError("tile_gather: latent must be a float32 [C, H, W] tensor")
    latent = latent.contiguous()
    c, h, w = latent.shape
    r = (C.c_int32 * len(rows))(*rows)
    q = (C.c_int32 * len(cols))(*cols)
    tiles = torch.empty(len(rows) * len(cols), c, tile, tile, device=latent.device, dtype=torch.float32)
    check(lib().nd_op_tile_gather(latent.data_ptr(), c, h, w, r, len(rows), q, len(cols), tile, tiles.data_ptr(),
                                  C.c_void_p(_stream())))
    return tiles


def tile_blend(tiles: torch.Tensor, rows, cols, vertical: torch.Tensor, horizontal: torch.Tensor, height: int,
               width: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Decoded tiles [len(rows) * len(cols), C, side, side] crossfaded into
    out [C, height, width] (TiledVae.BlendTile + DivideByWeights); rows / cols
    in the tiles' own units, vertical / horizontal the two axes' ramps."""
    if tiles.dim() != 4 or tiles.dtype != torch.float32 or not tiles.is_contiguous():
        raise ValueError("tile_blend: tiles must be a contiguous float32 [tiles, C, side, side] tensor")
    t, c, side, _ = tiles.shape
    if t != len(rows) * len(cols) or tiles.shape[3] != side:
        raise ValueError(f"tile_blend: {len(rows)} x {len(cols)} square tiles expected, got {tuple(tiles.shape)}")
    for ramp in (vertical, horizontal):
        if ramp.dtype != torch.float32 or ramp.numel() != side or ramp.device != tiles.device:
            raise ValueError(f"tile_blend: the ramps must be float32 vectors of {side} on the tiles' device")
    if out is None:
        out = torch.empty(c, height, width, device=tiles.device, dtype=torch.float32)
    elif (tuple(out.shape) != (c, height, width) or out.dtype != torch.float32 or not out.is_contiguous()
          or out.device != tiles.device):
        raise ValueError(f"tile_blend: out must be a contiguous float32 [{c}, {height}, {width}] tensor")
    r = (C.c_int32 * len(rows))(*rows)
    q = (C.c_int32 * len(cols))(*cols)
    check(lib().nd_op_tile_blend(tiles.data_ptr(), c, side, r, len(rows), q, len(cols), vertical.data_ptr(),
                                 horizontal.data_ptr(), out.data_ptr(), height, width, C.c_void_p(_stream())))
    return out


def dequantize(q: torch.Tensor, scales: torch.Tensor, quant_group: int = 32,
               out_dtype=torch.bfloat16) -> torch.Tensor:
    """w = round(q * scale) in out_dtype (DmlOps.Dequantize, Dml/DmlOps.cs:208-228)."""
    rows, cols = q.shape
    out = torch.empty(rows, cols, device=q.device, dtype=out_dtype)
    check(lib().nd_op_dequantize(q.data_ptr(), scales.data_ptr(), _DT[scales.dtype], quant_group, rows,
                                 cols, out.data_ptr(), _DT[out_dtype], C.c_void_p(_stream())))
    return out


def quantize(w: torch.Tensor, quant_group: int = 32, scale_dtype=torch.float16):
    """BlockQuantizer on the device: (q int8 [rows, cols], scales [rows, cols / group] or [rows])."""
    rows, cols = w.shape
    g = quant_group or cols
    q = torch.empty(rows, cols, device=w.device, dtype=torch.int8)
    s = torch.empty(rows, cols // g, device=w.device, dtype=scale_dtype)
    check(lib().nd_op_quantize(w.data_ptr(), _DT[w.dtype], rows, cols, quant_group, _DT[scale_dtype],
                               q.data_ptr(), s.data_ptr(), C.c_void_p(_stream())))
    return q, s


_EPI_CONV = {"store": 0, "silu": 3, "store_f32": 5, "add_store": 8}


def conv2d(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None, *, stride: int = 1,
           epilogue: str = "store", addend: torch.Tensor | None = None,
           per_batch_bias: bool = False) -> torch.Tensor:
    """3x3 convolution, padding 1, over NHWC activations x [B, H, W, Cin] with
    weight [Cout, 3, 3, Cin rounded up to 64, the pad zero] (Layers.Conv2d,
    Graph/Layers.cs:115-128).
    bias: [Cout] fp32, or [B, Cout] with per_batch_bias."""
    b, h, w, cin = x.shape
    cout = weight.shape[0]
    ho, wo = (h + 2 - 3) // stride + 1, (w + 2 - 3) // stride + 1
    a = _lib.ConvArgs()
    a.dtype = _DT[x.dtype]
    a.epilogue = _EPI_CONV[epilogue]
    a.batch, a.height, a.width, a.in_channels, a.out_channels, a.stride = b, h, w, cin, cout, stride
    a.x, a.weight, a.bias = x.data_ptr(), weight.data_ptr(), _ptr(bias)
    a.per_batch_bias = 1 if per_batch_bias else 0
    a.bias_stride = bias.stride(0) if per_batch_bias else 0
    if epilogue == "store_f32":
        y = torch.empty(b, ho, wo, cout, device=x.device, dtype=torch.float32)
        a.y_f32 = y.data_ptr()
    else:
        y = torch.empty(b, ho, wo, cout, device=x.device, dtype=x.dtype)
        a.y = y.data_ptr()
    a.addend = _ptr(addend)
    check(lib().nd_op_conv2d(C.byref(a), C.c_void_p(_stream())))
    return y


def group_norm(x: torch.Tensor, groups: int, weight: torch.Tensor, bias: torch.Tensor | None = None, *,
               eps: float = 1e-5, silu: bool = False) -> torch.Tensor:
    """GroupNorm over NHWC x [B, pixels, C] (Layers.GroupNorm, Graph/Layers.cs:166-185),
    optionally followed by SiLU."""
    b, p, c = x.shape
    y = torch.empty_like(x)
    check(lib().nd_op_group_norm(x.data_ptr(), y.data_ptr(), _DT[x.dtype], b, p, c, groups, weight.data_ptr(),
                                 _ptr(bias), eps, 1 if silu else 0, C.c_void_p(_stream())))
    return y


def geglu(x: torch.Tensor) -> torch.Tensor:
    """[rows, 2F] -> [rows, F] = x[:, :F] * gelu(x[:, F:]) (UNetLayers.Geglu, Models/Sdxl/UNetLayers.cs:30-46)."""
    rows, two_f = x.shape
    y = torch.empty(rows, two_f // 2, device=x.device, dtype=x.dtype)
    check(lib().nd_op_geglu(x.data_ptr(), y.data_ptr(), _DT[x.dtype], rows, two_f // 2, C.c_void_p(_stream())))
    return y


def sampler_step(sampler: int, prediction: int, out: torch.Tensor, sample: torch.Tensor, *,
                 guidance: float = 1.0, last: torch.Tensor | None = None, noise: torch.Tensor | None = None,
                 denoised_out: torch.Tensor | None = None, next_input: torch.Tensor | None = None,
                 next_input_scale: float = 1.0, sigma: float, sigma_next: float, up: float = 0.0,
                 down: float = 0.0, rescale: float = 1.0, noise_scale: float = 0.0, shrink: float = 0.0,
                 weight: float = 0.0, second_order: bool = False) -> torch.Tensor:
    """Guidance combine + one solver step in place on `sample` (fp32, device),
    bit-identical to the reference's CPU step (Sampling/Schedulers.cs).
    out: [n] or [2, n] (uncond then cond)."""
    n = sample.numel()
    branches = out.numel() // n
    if branches not in (1, 2) or out.numel() != branches * n:
        raise ValueError(f"sampler_step: out must hold 1 or 2 branches of {n} values")
    for what, t in (("out", out), ("sample", sample), ("last", last), ("noise", noise),
                    ("denoised_out", denoised_out), ("next_input", next_input)):
        _check_vec(f"sampler_step: {what}", t, branches * n if what == "out" else n, sample.device)
    a = _lib.SamplerArgs()
    a.sampler, a.prediction, a.n, a.branches = sampler, prediction, n, branches
    a.out, a.guidance, a.sample = out.data_ptr(), guidance, sample.data_ptr()
    a.last_denoised, a.noise, a.denoised_out, a.next_input = _ptr(last), _ptr(noise), _ptr(denoised_out), _ptr(next_input)
    a.next_input_scale, a.sigma, a.sigma_next = next_input_scale, sigma, sigma_next
    a.up, a.down, a.rescale, a.noise_scale, a.shrink, a.weight = up, down, rescale, noise_scale, shrink, weight
    a.second_order = int(bool(second_order))
    check(lib().nd_op_sampler_step(C.byref(a), C.c_void_p(_stream())))
    return sample
