"""Host-side mirror of the reference's denoiser plug-in interface.

`CudaDenoiser` is what the C# `IDenoiser` (src/NaiveDiffusion/Pipeline/
IDenoiser.cs:10-32) becomes over libnd_denoise: `predict(latent, timestep,
sigma, conditioning)` plus the memory figures, disposable. `build_denoiser`
plays `IModelFamily.BuildDenoiser` (Pipeline/IModelFamily.cs:142-143): it
creates the native model, copies every (LoRA-folded) weight into HBM once and
finalizes. A C# host would bind the same C entry points (include/nd_denoise.h)
through P/Invoke; this module calls them through ctypes.
"""
from __future__ import annotations

import ctypes as C
import zlib
from dataclasses import dataclass, field

import numpy as np

from . import _lib
from ._lib import check, lib

FAMILY_MMDIT, FAMILY_ANIMA, FAMILY_SDXL, FAMILY_VAE_KL, FAMILY_QWEN_IMAGE = 0, 1, 2, 3, 4
FAMILY_VAE_WAN21, FAMILY_VAE_WAN22 = 5, 6
FAMILY_QWEN3_TEXT, FAMILY_LLM_ADAPTER = 7, 8


class ModelDesc(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "family", "width", "heads", "head_dim", "blocks", "mlp_width",
        "context_rows", "context_width", "latent_channels", "latent_height", "latent_width",
        "patch", "time_width", "batch", "compute", "weight_dtype", "quant_group",
        "quant_scale_dtype", "adaln_rank")] + [("eps", C.c_float), ("unet_levels", C.c_int),
        ("unet_mult", C.c_int * 4), ("unet_depth", C.c_int * 4), ("unet_resnets", C.c_int),
        ("add_width", C.c_int), ("kv_heads", C.c_int), ("vocab", C.c_int), ("source_rows", C.c_int),
        ("rope_theta", C.c_double)]


class NamedTensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("dtype", C.c_int), ("rank", C.c_int),
                ("shape", C.POINTER(C.c_int64)), ("data", C.c_void_p)]


class KernelTime(C.Structure):
    _fields_ = [("name", C.c_char_p), ("launches", C.c_int), ("total_ms", C.c_double),
                ("flops", C.c_double), ("bytes", C.c_double)]


class Memory(C.Structure):
    _fields_ = [("persistent_bytes", C.c_uint64), ("streamed_bytes", C.c_uint64),
                ("resident_bytes", C.c_uint64), ("temporary_bytes", C.c_uint64),
                ("graph_count", C.c_int)]


def _bind() -> C.CDLL:
    L = lib()
    if getattr(L, "_nd_denoiser_bound", False):
        return L
    P = C.c_void_p
    L.nd_device_open.argtypes = [C.c_int, C.POINTER(P)]
    L.nd_device_close.argtypes = [P]
    L.nd_denoiser_create.argtypes = [P, C.POINTER(ModelDesc), C.POINTER(P)]
    L.nd_denoiser_weight_info.argtypes = [P, C.c_int, C.POINTER(C.c_char_p), C.POINTER(C.c_int64),
                                          C.POINTER(C.c_int64), C.POINTER(C.c_int)]
    L.nd_denoiser_set_weight.argtypes = [P, C.c_char_p, C.c_int, C.POINTER(C.c_int64), C.c_int, P]
    L.nd_denoiser_set_weight_device.argtypes = [P, C.c_char_p, C.c_int, C.POINTER(C.c_int64), C.c_int, P]
    L.nd_denoiser_finalize.argtypes = [P]
    L.nd_denoiser_predict.argtypes = [P, P, C.c_double, C.c_double, C.c_int, C.POINTER(NamedTensor), P]
    L.nd_denoiser_predict_device.argtypes = [P, P, C.c_double, C.c_double, C.c_int,
                                             C.POINTER(NamedTensor), P, P]
    L.nd_denoiser_memory.argtypes = [P, C.POINTER(Memory)]
    L.nd_denoiser_profile.argtypes = [P, C.c_int, C.POINTER(KernelTime), C.c_int, C.POINTER(C.c_int)]
    L.nd_denoiser_destroy.argtypes = [P]
    L.nd_text_encode.argtypes = [P, P, C.c_int, P, C.c_int, C.c_int, P]
    L._nd_denoiser_bound = True
    return L


@dataclass
class MMDiTConfig:
    """A Qwen-Image-style dual-stream DiT. Defaults: benchmark configuration 3
    (60 blocks x 3072, 24 x 128 heads, MLP 12288, 16 x 128 x 168 latent in 2x2
    patches = 5376 image tokens, 256 text rows of 3584, bf16)."""
    width: int = 3072
    heads: int = 24
    blocks: int = 60
    mlp_width: int = 12288
    context_rows: int = 256
    context_width: int = 3584
    latent_channels: int = 16
    latent_height: int = 128
    latent_width: int = 168
    patch: int = 2
    time_width: int = 256
    compute: int = _lib.ND_BF16
    eps: float = 1e-6
    weight_dtype: int = 0           # 0: the compute dtype; _lib.ND_I8: int8 weight-only
    quant_group: int = 32           # int8: columns per scale (0 = per output channel)
    quant_scale_dtype: int = _lib.ND_F16

    @property
    def image_tokens(self) -> int:
        return (self.latent_height // self.patch) * (self.latent_width // self.patch)

    @property
    def tokens(self) -> int:
        return self.image_tokens + self.context_rows

    def desc(self) -> ModelDesc:
        d = ModelDesc()
        d.family = FAMILY_MMDIT
        d.width, d.heads, d.head_dim = self.width, self.heads, 128
        d.blocks, d.mlp_width = self.blocks, self.mlp_width
        d.context_rows, d.context_width = self.context_rows, self.context_width
        d.latent_channels, d.latent_height, d.latent_width = (
            self.latent_channels, self.latent_height, self.latent_width)
        d.patch, d.time_width, d.batch = self.patch, self.time_width, 1
        d.compute = self.compute
        d.weight_dtype = self.weight_dtype or self.compute
        d.quant_group = self.quant_group
        d.quant_scale_dtype = self.quant_scale_dtype
        d.eps = self.eps
        return d

    def quantized(self, rows: int, cols: int) -> bool:
        """Whether a [rows, cols] matrix is stored as int8 (ModelBuilder.Weight's
        rule: at least 65,536 elements, whole groups per row)."""
        g = self.quant_group or cols
        return self.weight_dtype == _lib.ND_I8 and rows * cols >= 65536 and cols % g == 0 and cols % 16 == 0

    def flops_per_step(self) -> float:
        """Algorithmic FLOPs of one step (1 MAC = 2 FLOP): block GEMMs, joint
        attention (QK^T and PV), modulation GEMV, embeddings and final layer."""
        D, F, N, ni = self.width, self.mlp_width, self.tokens, self.image_tokens
        gemm = N * (4 * D * D + 2 * D * F)
        attn = 2 * N * N * D
        mod = 2 * 6 * D * D
        per_block = gemm + attn + mod
        cin = self.latent_channels * self.patch ** 2
        emb = ni * cin * D + self.context_rows * self.context_width * D + ni * D * cin
        return 2.0 * (self.blocks * per_block + emb)


@dataclass
class QwenImageConfig:
    """Qwen-Image 2.1's single-stream DiT (Models/QwenImage/QwenImageDit.cs).
    Defaults: the released model's shape (32 blocks x 4096, 32 x 128 heads,
    SwiGLU 12288, 64-channel latent at patch 1, 4096-wide text rows; shapes
    from the reference's fixture FakeSafetensors.QwenImageDit) at 1024 x 1024
    (64 x 64 latent cells = 4096 image tokens) with 256 text rows, computing
    at fp16 (the reference's half-precision option)."""
    width: int = 4096
    heads: int = 32
    blocks: int = 32
    mlp_width: int = 12288
    context_rows: int = 256
    context_width: int = 4096
    latent_channels: int = 64
    latent_height: int = 64
    latent_width: int = 64
    time_width: int = 256
    compute: int = _lib.ND_F16
    eps: float = 1e-6
    weight_dtype: int = 0
    quant_group: int = 32
    quant_scale_dtype: int = _lib.ND_F16
    fused_gate_up: bool = True      # img_mlp.gate_up (Comfy-Org's layout) or gate_layer + proj

    @property
    def image_tokens(self) -> int:
        return self.latent_height * self.latent_width

    @property
    def tokens(self) -> int:
        return self.image_tokens + self.context_rows

    def desc(self) -> ModelDesc:
        d = ModelDesc()
        d.family = FAMILY_QWEN_IMAGE
        d.width, d.heads, d.head_dim = self.width, self.heads, 128
        d.blocks, d.mlp_width = self.blocks, self.mlp_width
        d.context_rows, d.context_width = self.context_rows, self.context_width
        d.latent_channels, d.latent_height, d.latent_width = (
            self.latent_channels, self.latent_height, self.latent_width)
        d.patch, d.time_width, d.batch = 1, self.time_width, 1
        d.compute = self.compute
        d.weight_dtype = self.weight_dtype or self.compute
        d.quant_group = self.quant_group
        d.quant_scale_dtype = self.quant_scale_dtype
        d.eps = self.eps
        return d

    def quantized(self, rows: int, cols: int) -> bool:
        g = self.quant_group or cols
        return self.weight_dtype == _lib.ND_I8 and rows * cols >= 65536 and cols % g == 0 and cols % 16 == 0

    def weight_shapes(self):
        """(name, shape, required) of every tensor the family reads. No biases."""
        D, F, cw, tw, C_ = self.width, self.mlp_width, self.context_width, self.time_width, self.latent_channels
        t = [("img_in.weight", (D, C_), True), ("txt_in.text_norm.weight", (cw,), True),
             ("txt_in.in_layer.weight", (D, cw), True), ("txt_in.out_layer.weight", (D, D), True),
             ("time_text_embed.timestep_embedder.linear_1.weight", (D, tw), True),
             ("time_text_embed.timestep_embedder.linear_2.weight", (D, D), True),
             ("modulation.1.weight", (4 * D, D), True), ("norm_out.linear.weight", (D, D), True),
             ("proj_out.weight", (C_, D), True)]
        for b in range(self.blocks):
            p = f"transformer_blocks.{b}."
            t += [(p + "attn.to_q.weight", (D, D), True), (p + "attn.to_k.weight", (D, D), True),
                  (p + "attn.to_v.weight", (D, D), True), (p + "attn.norm_q.weight", (128,), True),
                  (p + "attn.norm_k.weight", (128,), True), (p + "attn.to_out.0.weight", (D, D), True)]
            if self.fused_gate_up:
                t += [(p + "img_mlp.gate_up.weight", (2 * F, D), True)]
            else:
                t += [(p + "img_mlp.gate_layer.weight", (F, D), True), (p + "img_mlp.proj.weight", (F, D), True)]
            t += [(p + "img_mlp.out.weight", (D, F), True)]
        return t

    def flops_per_step(self, real_rows: int | None = None) -> float:
        """Algorithmic FLOPs of one step (1 MAC = 2 FLOP): block GEMMs (QKV,
        out, gate+up, down), the image rows' attention over every visible key
        and the text rows' causal attention, embeddings and the final layer."""
        D, F, ni, R = self.width, self.mlp_width, self.image_tokens, self.context_rows
        real = R if real_rows is None else real_rows
        M = ni + R
        gemm = M * (4 * D * D + 3 * D * F)
        attn = 2 * ni * (ni + real) * D + R * real * D
        emb = ni * self.latent_channels * D * 2 + R * self.context_width * D + R * D * D
        return 2.0 * (self.blocks * (gemm + attn) + emb)


@dataclass
class Qwen3TextConfig:
    """A Qwen3 decoder read as a text encoder (Text/Qwen/Qwen3TextModel.cs).
    Defaults: Qwen3-0.6B (Anima's: 1024 wide, 28 layers, 16 x 128 query heads,
    8 key/value heads, SwiGLU 3072, rotary base 1e6); Qwen3-VL-8B's language
    model is qwen3_vl_8b(). context_rows = most tokens per call."""
    width: int = 1024
    blocks: int = 28
    heads: int = 16
    kv_heads: int = 8
    mlp_width: int = 3072
    vocab: int = 151936
    rope_theta: float = 1e6
    context_rows: int = 512
    compute: int = _lib.ND_BF16
    eps: float = 1e-6

    @staticmethod
    def qwen3_vl_8b(**kw):
        return Qwen3TextConfig(width=4096, blocks=36, heads=32, kv_heads=8, mlp_width=12288, rope_theta=5e6, **kw)

    def desc(self) -> ModelDesc:
        d = ModelDesc()
        d.family = FAMILY_QWEN3_TEXT
        d.width, d.heads, d.head_dim, d.kv_heads = self.width, self.heads, 128, self.kv_heads
        d.blocks, d.mlp_width, d.vocab, d.rope_theta = self.blocks, self.mlp_width, self.vocab, self.rope_theta
        d.context_rows, d.batch = self.context_rows, 1
        d.compute = d.weight_dtype = self.compute
        d.eps = self.eps
        return d

    def weight_shapes(self):
        W, F, QW, KW = self.width, self.mlp_width, self.heads * 128, self.kv_heads * 128
        t = [("model.embed_tokens.weight", (self.vocab, W), True), ("model.norm.weight", (W,), True)]
        for l in range(self.blocks):
            p = f"model.layers.{l}."
            t += [(p + "input_layernorm.weight", (W,), True), (p + "self_attn.q_proj.weight", (QW, W), True),
                  (p + "self_attn.k_proj.weight", (KW, W), True), (p + "self_attn.v_proj.weight", (KW, W), True),
                  (p + "self_attn.q_norm.weight", (128,), True), (p + "self_attn.k_norm.weight", (128,), True),
                  (p + "self_attn.o_proj.weight", (W, QW), True), (p + "post_attention_layernorm.weight", (W,), True),
                  (p + "mlp.gate_proj.weight", (F, W), True), (p + "mlp.up_proj.weight", (F, W), True),
                  (p + "mlp.down_proj.weight", (W, F), True)]
        return t

    def flops(self, rows: int) -> float:
        W, F, QW, KW = self.width, self.mlp_width, self.heads * 128, self.kv_heads * 128
        per = rows * (W * (QW + 2 * KW) + QW * W + 3 * W * F) + rows * rows * QW
        return 2.0 * self.blocks * per


@dataclass
class LlmAdapterConfig:
    """Anima's LLM adapter (Models/Anima/LlmAdapter.cs): 6 blocks 1024 wide,
    16 x 64 heads, GELU MLP 4096, rotary base 1e4, T5's 32128-id table.
    context_rows = most T5 ids per call, source_rows = most Qwen3 rows."""
    width: int = 1024
    blocks: int = 6
    heads: int = 16
    head_dim: int = 64
    mlp_width: int = 4096
    vocab: int = 32128
    rope_theta: float = 1e4
    context_rows: int = 512
    source_rows: int = 512
    compute: int = _lib.ND_BF16
    eps: float = 1e-6

    def desc(self) -> ModelDesc:
        d = ModelDesc()
        d.family = FAMILY_LLM_ADAPTER
        d.width, d.heads, d.head_dim = self.width, self.heads, self.head_dim
        d.blocks, d.mlp_width, d.vocab, d.rope_theta = self.blocks, self.mlp_width, self.vocab, self.rope_theta
        d.context_rows, d.source_rows, d.batch = self.context_rows, self.source_rows, 1
        d.compute = d.weight_dtype = self.compute
        d.eps = self.eps
        return d

    def weight_shapes(self):
        W, F, hd = self.width, self.mlp_width, self.head_dim
        t = [("embed.weight", (self.vocab, W), True), ("out_proj.weight", (W, W), True), ("out_proj.bias", (W,), False),
             ("norm.weight", (W,), True)]
        for b in range(self.blocks):
            p = f"blocks.{b}."
            t += [(p + "norm_self_attn.weight", (W,), True), (p + "norm_cross_attn.weight", (W,), True),
                  (p + "norm_mlp.weight", (W,), True)]
            for a in ("self_attn", "cross_attn"):
                t += [(p + f"{a}.{n}_proj.weight", (W, W), True) for n in ("q", "k", "v", "o")]
                t += [(p + f"{a}.q_norm.weight", (hd,), True), (p + f"{a}.k_norm.weight", (hd,), True)]
            t += [(p + "mlp.0.weight", (F, W), True), (p + "mlp.0.bias", (F,), False),
                  (p + "mlp.2.weight", (W, F), True), (p + "mlp.2.bias", (W,), False)]
        return t


@dataclass
class AnimaConfig:
    """The Anima (Cosmos-Predict2 2B) DiT. Defaults: benchmark configuration 2
    (28 blocks x 2048, 16 x 128 heads, exact-GELU MLP 8192, low-rank adaLN
    256, 16 x 128 x 128 latent in 2x2 patches = 4096 tokens, cross-attention
    to 256 x 1024 text rows, batch 2 = the CFG branches, bf16)."""
    width: int = 2048
    heads: int = 16
    blocks: int = 28
    mlp_width: int = 8192
    adaln_rank: int = 256
    context_rows: int = 256
    context_width: int = 1024
    latent_channels: int = 16
    latent_height: int = 128
    latent_width: int = 128
    patch: int = 2
    batch: int = 2
    compute: int = _lib.ND_BF16
    eps: float = 1e-6
    weight_dtype: int = 0
    quant_group: int = 32
    quant_scale_dtype: int = _lib.ND_F16

    @property
    def tokens(self) -> int:
        return (self.latent_height // self.patch) * (self.latent_width // self.patch)

    def desc(self) -> ModelDesc:
        d = ModelDesc()
        d.family = FAMILY_ANIMA
        d.width, d.heads, d.head_dim = self.width, self.heads, 128
        d.blocks, d.mlp_width, d.adaln_rank = self.blocks, self.mlp_width, self.adaln_rank
        d.context_rows, d.context_width = self.context_rows, self.context_width
        d.latent_channels, d.latent_height, d.latent_width = (
            self.latent_channels, self.latent_height, self.latent_width)
        d.patch, d.time_width, d.batch = self.patch, self.width, self.batch
        d.compute = self.compute
        d.weight_dtype = self.weight_dtype or self.compute
        d.quant_group, d.quant_scale_dtype = self.quant_group, self.quant_scale_dtype
        d.eps = self.eps
        return d

    def quantized(self, rows: int, cols: int) -> bool:
        g = self.quant_group or cols
        return self.weight_dtype == _lib.ND_I8 and rows * cols >= 65536 and cols % g == 0 and cols % 16 == 0

    def weight_table(self):
        D, F, R, cw = self.width, self.mlp_width, self.adaln_rank, self.context_width
        t = [("x_embedder.proj.1.weight", D, 68, True), ("t_embedder.1.linear_1.weight", D, D, True),
             ("t_embedder.1.linear_2.weight", 3 * D, D, True), ("t_embedding_norm.weight", D, 1, True)]
        for b in range(self.blocks):
            p = f"blocks.{b}."
            for sub in ("adaln_modulation_self_attn", "adaln_modulation_cross_attn", "adaln_modulation_mlp"):
                t += [(p + sub + ".1.weight", R, D, True), (p + sub + ".2.weight", 3 * D, R, True)]
            t += [(p + "self_attn.q_proj.weight", D, D, True), (p + "self_attn.k_proj.weight", D, D, True),
                  (p + "self_attn.v_proj.weight", D, D, True), (p + "self_attn.output_proj.weight", D, D, True),
                  (p + "self_attn.q_norm.weight", 128, 1, True), (p + "self_attn.k_norm.weight", 128, 1, True),
                  (p + "cross_attn.q_proj.weight", D, D, True), (p + "cross_attn.k_proj.weight", D, cw, True),
                  (p + "cross_attn.v_proj.weight", D, cw, True), (p + "cross_attn.output_proj.weight", D, D, True),
                  (p + "cross_attn.q_norm.weight", 128, 1, True), (p + "cross_attn.k_norm.weight", 128, 1, True),
                  (p + "mlp.layer1.weight", F, D, True), (p + "mlp.layer2.weight", D, F, True)]
        t += [("final_layer.adaln_modulation.1.weight", R, D, True),
              ("final_layer.adaln_modulation.2.weight", 2 * D, R, True),
              ("final_layer.linear.weight", 64, D, True)]
        return t

    def flops_per_step(self) -> float:
        D, F, T, c, R = self.width, self.mlp_width, self.tokens, self.context_rows, self.adaln_rank
        per_image = (T * (4 * D * D + D * D + D * D + 2 * D * F) + c * self.context_width * 2 * D
                     + 2 * T * T * D + 2 * T * c * D)
        return 2.0 * self.batch * self.blocks * per_image


@dataclass
class UNetConfig:
    """The SDXL UNet. Defaults: benchmark configuration 5 (levels 320 / 640 /
    1280 with transformer depths 0 / 2 / 10, 64-wide heads, 2 resnets per
    level, cross-attention to 77 x 2048 text rows, add embedding 2816, 4 x 128
    x 128 latent, batch 2 = the CFG branches, fp16)."""
    width: int = 320
    mult: tuple = (1, 2, 4)
    depth: tuple = (0, 2, 10)
    resnets: int = 2
    context_rows: int = 77
    context_width: int = 2048
    add_width: int = 2816
    time_width: int = 320
    latent_height: int = 128
    latent_width: int = 128
    batch: int = 2
    compute: int = _lib.ND_F16
    latent_channels: int = 4

    def desc(self) -> ModelDesc:
        d = ModelDesc()
        d.family = FAMILY_SDXL
        d.width, d.head_dim = self.width, 64
        d.context_rows, d.context_width = self.context_rows, self.context_width
        d.latent_channels, d.latent_height, d.latent_width = 4, self.latent_height, self.latent_width
        d.time_width, d.batch, d.compute, d.weight_dtype = self.time_width, self.batch, self.compute, self.compute
        d.unet_levels = len(self.mult)
        for i, (m, dep) in enumerate(zip(self.mult, self.depth)):
            d.unet_mult[i], d.unet_depth[i] = m, dep
        d.unet_resnets, d.add_width = self.resnets, self.add_width
        return d

    def weight_shapes(self):
        """(name, checkpoint shape, required) in the library's registry order."""
        C0, cw, tw, aw = self.width, self.context_width, self.time_width, self.add_width
        out = []

        def conv(name, co, ci):
            out.append((name + ".weight", (co, ci, 3, 3), True))
            out.append((name + ".bias", (co,), False))

        def res(p, ci, co):
            out.extend([(p + ".norm1.weight", (ci,), True), (p + ".norm1.bias", (ci,), False)])
            conv(p + ".conv1", co, ci)
            out.extend([(p + ".norm2.weight", (co,), True), (p + ".norm2.bias", (co,), False)])
            conv(p + ".conv2", co, co)
            if ci != co:
                out.extend([(p + ".conv_shortcut.weight", (co, ci), True), (p + ".conv_shortcut.bias", (co,), False)])

        def t2d(p, c, dep):
            out.extend([(p + ".norm.weight", (c,), True), (p + ".norm.bias", (c,), False),
                        (p + ".proj_in.weight", (c, c), True), (p + ".proj_in.bias", (c,), False)])
            for j in range(dep):
                q = f"{p}.transformer_blocks.{j}"
                for n in ("norm1", "norm2", "norm3"):
                    out.extend([(f"{q}.{n}.weight", (c,), True), (f"{q}.{n}.bias", (c,), False)])
                out.extend([(q + ".attn1.to_q.weight", (c, c), True), (q + ".attn1.to_k.weight", (c, c), True),
                            (q + ".attn1.to_v.weight", (c, c), True),
                            (q + ".attn1.to_out.0.weight", (c, c), True), (q + ".attn1.to_out.0.bias", (c,), False),
                            (q + ".attn2.to_q.weight", (c, c), True), (q + ".attn2.to_k.weight", (c, cw), True),
                            (q + ".attn2.to_v.weight", (c, cw), True),
                            (q + ".attn2.to_out.0.weight", (c, c), True), (q + ".attn2.to_out.0.bias", (c,), False),
                            (q + ".ff.net.0.proj.weight", (8 * c, c), True), (q + ".ff.net.0.proj.bias", (8 * c,), False),
                            (q + ".ff.net.2.weight", (c, 4 * c), True), (q + ".ff.net.2.bias", (c,), False)])
            out.extend([(p + ".proj_out.weight", (c, c), True), (p + ".proj_out.bias", (c,), False)])

        conv("conv_in", C0, self.latent_channels)
        out.extend([("time_embedding.linear_1.weight", (1280, tw), True), ("time_embedding.linear_1.bias", (1280,), False),
                    ("time_embedding.linear_2.weight", (1280, 1280), True), ("time_embedding.linear_2.bias", (1280,), False),
                    ("add_embedding.linear_1.weight", (1280, aw), True), ("add_embedding.linear_1.bias", (1280,), False),
                    ("add_embedding.linear_2.weight", (1280, 1280), True), ("add_embedding.linear_2.bias", (1280,), False)])
        L = len(self.mult)
        chans = [C0]
        c = C0
        res_units = []
        for lvl in range(L):
            p = f"down_blocks.{lvl}"
            co = C0 * self.mult[lvl]
            for i in range(self.resnets):
                res(f"{p}.resnets.{i}", c, co)
                res_units.append((f"{p}.resnets.{i}", co))
                c = co
                if self.depth[lvl] > 0:
                    t2d(f"{p}.attentions.{i}", co, self.depth[lvl])
                chans.append(co)
            if lvl != L - 1:
                conv(f"{p}.downsamplers.0.conv", co, co)
                chans.append(co)
        res("mid_block.resnets.0", c, c)
        t2d("mid_block.attentions.0", c, self.depth[L - 1] or 1)
        res("mid_block.resnets.1", c, c)
        mid = [("mid_block.resnets.0", c), ("mid_block.resnets.1", c)]
        ups = []
        for i in range(L):
            lvl = L - 1 - i
            p = f"up_blocks.{i}"
            co = C0 * self.mult[lvl]
            for j in range(self.resnets + 1):
                skip = chans.pop()
                res(f"{p}.resnets.{j}", c + skip, co)
                ups.append((f"{p}.resnets.{j}", co))
                c = co
                if self.depth[lvl] > 0:
                    t2d(f"{p}.attentions.{j}", co, self.depth[lvl])
            if i != L - 1:
                conv(f"{p}.upsamplers.0.conv", co, co)
        out.extend([("conv_norm_out.weight", (c,), True), ("conv_norm_out.bias", (c,), False)])
        conv("conv_out", self.latent_channels, c)
        for name, co in res_units + mid + ups:
            out.extend([(name + ".time_emb_proj.weight", (co, 1280), True), (name + ".time_emb_proj.bias", (co,), False)])
        return out

    # Algorithmic FLOPs per image (1 MAC = 2 FLOP), walking UNetModel.Build's
    # layout (Models/Sdxl/UNetModel.cs:333-437): convolutions 2 Ho Wo Cout
    # Cin k^2, linear layers 2 rows in out, attention 4 Nq Nk C (QK^T and PV).
    def resblock_flops(self, ci: int, co: int, pixels: int) -> float:
        f = 2.0 * pixels * co * ci * 9 + 2.0 * pixels * co * co * 9 + 2.0 * 1280 * co
        return f + (2.0 * pixels * co * ci if ci != co else 0.0)

    def transformer2d_flops(self, c: int, pixels: int, depth: int) -> float:
        ctx, cw = self.context_rows, self.context_width
        per_block = (2.0 * pixels * c * c * 4 + 4.0 * pixels * pixels * c      # self-attention
                     + 2.0 * pixels * c * c * 2 + 2.0 * ctx * cw * c * 2       # cross q, out; k, v
                     + 4.0 * pixels * ctx * c                                   # cross attention
                     + 2.0 * pixels * c * 8 * c + 2.0 * pixels * 4 * c * c)     # GEGLU feed-forward
        return 2.0 * 2.0 * pixels * c * c + depth * per_block                  # proj_in / proj_out

    def flops_per_step(self) -> float:
        C0, L = self.width, len(self.mult)
        px = self.latent_height * self.latent_width
        f = 2.0 * px * C0 * self.latent_channels * 9 * 2                       # conv_in, conv_out
        f += 2.0 * (self.time_width * 1280 + 1280 * 1280 + self.add_width * 1280 + 1280 * 1280)
        chans, c = [C0], C0
        for lvl in range(L):
            co = C0 * self.mult[lvl]
            for _ in range(self.resnets):
                f += self.resblock_flops(c, co, px)
                c = co
                if self.depth[lvl]:
                    f += self.transformer2d_flops(co, px, self.depth[lvl])
                chans.append(co)
            if lvl != L - 1:
                px //= 4
                f += 2.0 * px * co * co * 9                                     # stride-2 conv
                chans.append(co)
        f += 2 * self.resblock_flops(c, c, px) + self.transformer2d_flops(c, px, self.depth[L - 1] or 1)
        for i in range(L):
            lvl = L - 1 - i
            co = C0 * self.mult[lvl]
            for _ in range(self.resnets + 1):
                f += self.resblock_flops(c + chans.pop(), co, px)
                c = co
                if self.depth[lvl]:
                    f += self.transformer2d_flops(co, px, self.depth[lvl])
            if i != L - 1:
                px *= 4
                f += 2.0 * px * co * co * 9                                     # conv after the upsample
        return self.batch * f


@dataclass
class VaeDecoderConfig:
    """The AutoencoderKL decoder (Vae/AutoencoderKl.cs). Defaults: the SDXL
    VAE (SdxlVae.Config: block_out_channels 128 / 256 / 512 / 512, 2 layers
    per block, 32 groups, eps 1e-6) decoding a 4 x 128 x 128 latent into a
    1024 x 1024 image."""
    width: int = 128
    mult: tuple = (1, 2, 4, 4)
    layers_per_block: int = 2
    latent_height: int = 128
    latent_width: int = 128
    batch: int = 1
    compute: int = _lib.ND_F16
    latent_channels: int = 4
    eps: float = 1e-6

    def desc(self) -> ModelDesc:
        d = ModelDesc()
        d.family = FAMILY_VAE_KL
        d.width = self.width
        d.latent_channels, d.latent_height, d.latent_width = 4, self.latent_height, self.latent_width
        d.batch, d.compute, d.weight_dtype, d.eps = self.batch, self.compute, self.compute, self.eps
        d.unet_levels = len(self.mult)
        for i, m in enumerate(self.mult):
            d.unet_mult[i] = m
        d.unet_resnets = self.layers_per_block
        return d

    @property
    def image_height(self) -> int:
        return self.latent_height << (len(self.mult) - 1)

    @property
    def image_width(self) -> int:
        return self.latent_width << (len(self.mult) - 1)

    def weight_shapes(self):
        L = len(self.mult)
        rev = [self.width * self.mult[L - 1 - i] for i in range(L)]
        out = [("post_quant_conv.weight", (4, 4, 1, 1), True), ("post_quant_conv.bias", (4,), False)]

        def conv(name, co, ci):
            out.append((name + ".weight", (co, ci, 3, 3), True))
            out.append((name + ".bias", (co,), False))

        def res(p, ci, co):
            out.extend([(p + ".norm1.weight", (ci,), True), (p + ".norm1.bias", (ci,), False)])
            conv(p + ".conv1", co, ci)
            out.extend([(p + ".norm2.weight", (co,), True), (p + ".norm2.bias", (co,), False)])
            conv(p + ".conv2", co, co)
            if ci != co:
                out.extend([(p + ".conv_shortcut.weight", (co, ci, 1, 1), True), (p + ".conv_shortcut.bias", (co,), False)])

        top = rev[0]
        conv("decoder.conv_in", top, 4)
        res("decoder.mid_block.resnets.0", top, top)
        a = "decoder.mid_block.attentions.0"
        out.extend([(a + ".group_norm.weight", (top,), True), (a + ".group_norm.bias", (top,), False)])
        for n in ("to_q", "to_k", "to_v", "to_out.0"):
            out.extend([(f"{a}.{n}.weight", (top, top), True), (f"{a}.{n}.bias", (top,), False)])
        res("decoder.mid_block.resnets.1", top, top)
        c = top
        for i in range(L):
            for j in range(self.layers_per_block + 1):
                res(f"decoder.up_blocks.{i}.resnets.{j}", c, rev[i])
                c = rev[i]
            if i != L - 1:
                conv(f"decoder.up_blocks.{i}.upsamplers.0.conv", c, c)
        out.extend([("decoder.conv_norm_out.weight", (c,), True), ("decoder.conv_norm_out.bias", (c,), False)])
        conv("decoder.conv_out", 3, c)
        return out

    def flops_per_step(self) -> float:
        """Convolutions, 1x1 shortcuts and the mid-block attention (1 MAC = 2 FLOP)."""
        L = len(self.mult)
        rev = [self.width * self.mult[L - 1 - i] for i in range(L)]
        h, w = self.latent_height, self.latent_width
        total = 0.0

        def conv(px, ci, co, k=9):
            return 2.0 * px * ci * co * k

        def res(px, ci, co):
            return conv(px, ci, co) + conv(px, co, co) + (conv(px, ci, co, 1) if ci != co else 0.0)

        px = h * w
        top = rev[0]
        total += conv(px, 4, top) + 2 * res(px, top, top) + 4 * 2.0 * px * top * top + 4.0 * px * px * top
        c = top
        for i in range(L):
            px = (h << i) * (w << i)
            for _ in range(self.layers_per_block + 1):
                total += res(px, c, rev[i])
                c = rev[i]
            if i != L - 1:
                total += conv(4 * px, c, c)
        total += conv((h << (L - 1)) * (w << (L - 1)), c, 3)
        return self.batch * total


@dataclass
class WanVaeConfig:
    """The Wan VAE decoders on one frame: version 21 (Vae/WanVae.cs, Anima's:
    base width 96, 16 latent channels, 8x) or 22 (Vae/Wan22Vae.cs, Qwen-Image
    2.1's: base width 144, 64 latent channels, five levels, 16x, the up
    shortcuts). Defaults: Wan 2.1 decoding a 16 x 128 x 128 latent into a
    1024 x 1024 image at fp16."""
    version: int = 21
    width: int = 96
    latent_channels: int = 16
    latent_height: int = 128
    latent_width: int = 128
    batch: int = 1
    resnets: int = 2                  # resblocks per level - 1 (the reference's ResnetsPerLevel)
    compute: int = _lib.ND_F16

    @property
    def scale(self) -> int:
        return 16 if self.version == 22 else 8

    @property
    def image_height(self) -> int:
        return self.latent_height * self.scale

    @property
    def image_width(self) -> int:
        return self.latent_width * self.scale

    def desc(self) -> ModelDesc:
        d = ModelDesc()
        d.family = FAMILY_VAE_WAN22 if self.version == 22 else FAMILY_VAE_WAN21
        d.width = self.width
        d.latent_channels, d.latent_height, d.latent_width = self.latent_channels, self.latent_height, self.latent_width
        d.batch, d.compute, d.weight_dtype = self.batch, self.compute, self.compute
        d.unet_resnets = self.resnets
        return d

    def levels(self):
        """(in, out, upsample-conv out or 0, shortcut mode or -1) per level:
        dims = width x [m_last, m reversed]; Wan 2.1's upsample convolution
        halves the width, Wan 2.2's keeps it and adds the up shortcut."""
        v22 = self.version == 22
        m = (1, 2, 4, 8, 8) if v22 else (1, 2, 4, 4)
        L = len(m)
        dims = [self.width * m[-1]] + [self.width * u for u in reversed(m)]
        temporal = (False, True, True, True)
        out = []
        for i in range(L):
            cin = dims[i] // 2 if (not v22 and i > 0) else dims[i]
            cout = dims[i + 1]
            up = 0 if i == L - 1 else (cout if v22 else cout // 2)
            mode = -1
            if v22 and up:
                mode = 0 if cin == up else (1 if temporal[L - 2 - i] else 2)
            out.append((cin, cout, up, mode))
        return out

    def weight_shapes(self):
        C, R = self.latent_channels, self.resnets
        lv = self.levels()
        top = lv[0][0]
        t = [("conv2.weight", (C, C, 1, 1), True), ("conv2.bias", (C,), False),
             ("decoder.conv1.weight", (top, C, 3, 3), True), ("decoder.conv1.bias", (top,), False)]

        def res(p, ci, co):
            r = [(p + ".residual.0.gamma", (ci,), True), (p + ".residual.2.weight", (co, ci, 3, 3), True),
                 (p + ".residual.2.bias", (co,), False), (p + ".residual.3.gamma", (co,), True),
                 (p + ".residual.6.weight", (co, co, 3, 3), True), (p + ".residual.6.bias", (co,), False)]
            if ci != co:
                r += [(p + ".shortcut.weight", (co, ci, 1, 1), True), (p + ".shortcut.bias", (co,), False)]
            return r
        t += res("decoder.middle.0", top, top)
        t += [("decoder.middle.1.norm.gamma", (top,), True), ("decoder.middle.1.to_qkv.weight", (3 * top, top, 1, 1), True),
              ("decoder.middle.1.to_qkv.bias", (3 * top,), False), ("decoder.middle.1.proj.weight", (top, top, 1, 1), True),
              ("decoder.middle.1.proj.bias", (top,), False)]
        t += res("decoder.middle.2", top, top)
        idx = 0
        for i, (ci, co, up, _mode) in enumerate(lv):
            pre = f"decoder.upsamples.{i}.upsamples." if self.version == 22 else "decoder.upsamples."
            if self.version == 22:
                idx = 0
            c = ci
            for _ in range(R + 1):
                t += res(f"{pre}{idx}", c, co)
                idx += 1
                c = co
            if up:
                t += [(f"{pre}{idx}.resample.1.weight", (up, co, 3, 3), True), (f"{pre}{idx}.resample.1.bias", (up,), False)]
                idx += 1
        last = lv[-1][1]
        img = 4 if self.version == 22 else 3
        t += [("decoder.head.0.gamma", (last,), True), ("decoder.head.2.weight", (img, last, 3, 3), True),
              ("decoder.head.2.bias", (img,), False)]
        return t

    def flops_per_step(self) -> float:
        """Convolutions, 1x1 shortcuts and the mid-block attention (1 MAC = 2 FLOP)."""
        h, w = self.latent_height, self.latent_width
        lv = self.levels()
        top = lv[0][0]

        def conv(px, ci, co, k=9):
            return 2.0 * px * ci * co * k

        def res(px, ci, co):
            return conv(px, ci, co) + conv(px, co, co) + (conv(px, ci, co, 1) if ci != co else 0.0)
        px = h * w
        total = conv(px, self.latent_channels, top) + 2 * res(px, top, top) + 4 * 2.0 * px * top * top + 4.0 * px * px * top
        for i, (ci, co, up, _m) in enumerate(lv):
            px = (h << i) * (w << i)
            c = ci
            for _ in range(self.resnets + 1):
                total += res(px, c, co)
                c = co
            if up:
                total += conv(4 * px, co, up)
        px = (h << (len(lv) - 1)) * (w << (len(lv) - 1))
        total += conv(px, lv[-1][1], 4 if self.version == 22 else 3)
        return self.batch * total


def _name_seed(name: str, seed: int) -> int:
    return (zlib.crc32(name.encode()) ^ (seed * 0x9E3779B1)) & 0xFFFFFFFF


def _table(cfg):
    return cfg.weight_table() if hasattr(cfg, "weight_table") else weight_table(cfg)


def synthetic_weights(cfg, seed: int = 0, only: tuple | None = None):
    """Seeded synthetic weights in the storage precision, one generator per
    tensor name: matrices and biases N(0, 0.02), norm weights 1 + N(0, 0.02).
    Yields (name, float32 array already rounded to bf16/fp16). `only`: name
    prefixes to generate (the others are skipped; each tensor's values do
    not depend on which others are drawn)."""
    if hasattr(cfg, "weight_shapes"):
        for name, shape, _req in cfg.weight_shapes():
            if only is not None and not name.startswith(only):
                continue
            rng = np.random.default_rng(_name_seed(name, seed))
            a = rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)
            if len(shape) == 1 and (("norm" in name and name.endswith(".weight")) or name.endswith(".gamma")):
                a += np.float32(1.0)
            if len(shape) > 1:
                a = _round(a, cfg.compute)
            yield name, a
        return
    for name, rows, cols, _req in _table(cfg):
        if only is not None and not name.startswith(only):
            continue
        rng = np.random.default_rng(_name_seed(name, seed))
        a = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02)
        if "norm" in name and name.endswith(".weight") and cols == 1:
            a += np.float32(1.0)
        if cols == 1:
            a = a.reshape(rows)
        else:
            a = _round(a, cfg.compute)
        yield name, a


def synthetic_weights_device(cfg, seed: int = 0, device="cuda"):
    """The same distributions as synthetic_weights, drawn on the GPU (a full
    benchmark-size model is 20 G parameters): one torch generator per tensor
    name. Yields (name, CUDA tensor): matrices in the compute dtype, vectors fp32."""
    import torch
    dt = {_lib.ND_BF16: torch.bfloat16, _lib.ND_F16: torch.float16}.get(cfg.compute, torch.float32)
    g = torch.Generator(device=device)
    if hasattr(cfg, "weight_shapes"):
        for name, shape, _req in cfg.weight_shapes():
            g.manual_seed(_name_seed(name, seed))
            t = torch.randn(*shape, device=device, generator=g) * 0.02
            if len(shape) == 1 and (("norm" in name and name.endswith(".weight")) or name.endswith(".gamma")):
                t += 1.0
            yield name, (t.to(dt) if len(shape) > 1 else t)
        return
    for name, rows, cols, _req in _table(cfg):
        g.manual_seed(_name_seed(name, seed))
        if cols == 1:
            t = torch.randn(rows, device=device, generator=g) * 0.02
            if "norm" in name and name.endswith(".weight"):
                t += 1.0
        else:
            t = (torch.randn(rows, cols, device=device, generator=g) * 0.02).to(dt)
        yield name, t


def _round(a: np.ndarray, dtype: int) -> np.ndarray:
    if dtype == _lib.ND_F32:
        return a
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a))
    t = t.to(torch.bfloat16 if dtype == _lib.ND_BF16 else torch.float16).float()
    return t.numpy()


def weight_table(cfg: MMDiTConfig):
    """(name, rows, cols, required) of every tensor the MMDiT family expects,
    in the order the native registry lists them (vectors have cols == 1)."""
    D, F, cw, tw = cfg.width, cfg.mlp_width, cfg.context_width, cfg.time_width
    cin = cfg.latent_channels * cfg.patch ** 2
    t = [("img_in.weight", D, cin, True), ("img_in.bias", D, 1, False),
         ("txt_norm.weight", cw, 1, True), ("txt_in.weight", D, cw, True), ("txt_in.bias", D, 1, False),
         ("time_text_embed.timestep_embedder.linear_1.weight", D, tw, True),
         ("time_text_embed.timestep_embedder.linear_1.bias", D, 1, False),
         ("time_text_embed.timestep_embedder.linear_2.weight", D, D, True),
         ("time_text_embed.timestep_embedder.linear_2.bias", D, 1, False),
         ("norm_out.linear.weight", 2 * D, D, True), ("norm_out.linear.bias", 2 * D, 1, False),
         ("proj_out.weight", cin, D, True), ("proj_out.bias", cin, 1, False)]
    mods = ["img_mod.1", "txt_mod.1"]
    projs = [["attn.to_q", "attn.to_k", "attn.to_v"], ["attn.add_q_proj", "attn.add_k_proj", "attn.add_v_proj"]]
    norms = [["attn.norm_q", "attn.norm_k"], ["attn.norm_added_q", "attn.norm_added_k"]]
    outs = ["attn.to_out.0", "attn.to_add_out"]
    ups = ["img_mlp.net.0.proj", "txt_mlp.net.0.proj"]
    downs = ["img_mlp.net.2", "txt_mlp.net.2"]
    for b in range(cfg.blocks):
        p = f"transformer_blocks.{b}."
        for s in range(2):
            t += [(p + mods[s] + ".weight", 6 * D, D, True), (p + mods[s] + ".bias", 6 * D, 1, False)]
            for j in range(3):
                t += [(p + projs[s][j] + ".weight", D, D, True), (p + projs[s][j] + ".bias", D, 1, False)]
            for j in range(2):
                t += [(p + norms[s][j] + ".weight", 128, 1, True)]
            t += [(p + outs[s] + ".weight", D, D, True), (p + outs[s] + ".bias", D, 1, False)]
            t += [(p + ups[s] + ".weight", F, D, True), (p + ups[s] + ".bias", F, 1, False)]
            t += [(p + downs[s] + ".weight", D, F, True), (p + downs[s] + ".bias", D, 1, False)]
    return t


class Device:
    """One GPU (nd_device_open)."""

    def __init__(self, ordinal: int = 0):
        L = _bind()
        h = C.c_void_p()
        check(L.nd_device_open(ordinal, C.byref(h)))
        self.handle = h
        self.ordinal = ordinal

    def close(self) -> None:
        if self.handle:
            _bind().nd_device_close(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class CudaDenoiser:
    """IDenoiser over libnd_denoise: Predict + the memory figures, disposable."""

    def __init__(self, device: Device, desc: ModelDesc):
        L = _bind()
        h = C.c_void_p()
        check(L.nd_denoiser_create(device.handle, C.byref(desc), C.byref(h)))
        self.handle = h
        self.device = device
        self.desc = desc
        self._side = None  # predict_device's stream when the caller names none

    # --- construction (IModelFamily.BuildDenoiser) ---------------------------
    def weight_info(self):
        L = _bind()
        out = []
        i = 0
        while True:
            name = C.c_char_p()
            rows, cols, req = C.c_int64(), C.c_int64(), C.c_int()
            if L.nd_denoiser_weight_info(self.handle, i, C.byref(name), C.byref(rows), C.byref(cols), C.byref(req)):
                break
            out.append((name.value.decode(), rows.value, cols.value, bool(req.value)))
            i += 1
        return out

    def set_weight(self, name: str, array) -> None:
        """Copy one tensor into HBM: a numpy array (host) or a torch CUDA tensor."""
        L = _bind()
        if hasattr(array, "data_ptr") and getattr(array, "is_cuda", False):
            import torch
            dt = {torch.float32: _lib.ND_F32, torch.float16: _lib.ND_F16, torch.bfloat16: _lib.ND_BF16}[array.dtype]
            t = array.contiguous()
            # The library copies on its own stream: make torch's producer finish first.
            torch.cuda.current_stream(t.device).synchronize()
            shape = (C.c_int64 * t.dim())(*t.shape)
            check(L.nd_denoiser_set_weight_device(self.handle, name.encode(), dt, shape, t.dim(),
                                                  C.c_void_p(t.data_ptr())))
            return
        a = np.ascontiguousarray(array)
        dt = {np.dtype(np.float32): _lib.ND_F32, np.dtype(np.float16): _lib.ND_F16}.get(a.dtype)
        if dt is None:
            raise TypeError(f"{name}: unsupported dtype {a.dtype}")
        shape = (C.c_int64 * a.ndim)(*a.shape)
        check(L.nd_denoiser_set_weight(self.handle, name.encode(), dt, shape, a.ndim,
                                       a.ctypes.data_as(C.c_void_p)))

    def set_weight_q8(self, name: str, q: np.ndarray, scales: np.ndarray, quant_group: int) -> None:
        """A matrix BlockQuantizer already quantized on the host: q int8
        [rows, cols], scales fp16 (given as uint16 bits or float16) or fp32."""
        L = _bind()
        q = np.ascontiguousarray(q, np.int8)
        s = np.ascontiguousarray(scales)
        sd = _lib.ND_F32 if s.dtype == np.float32 else _lib.ND_F16
        shape = (C.c_int64 * 2)(*q.shape)
        L.nd_denoiser_set_weight_q8.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(C.c_int64), C.c_int,
                                                C.c_void_p, C.c_int, C.c_void_p, C.c_int64]
        check(L.nd_denoiser_set_weight_q8(self.handle, name.encode(), shape, 2, q.ctypes.data, sd,
                                          s.ctypes.data, quant_group))

    def finalize(self) -> None:
        check(_bind().nd_denoiser_finalize(self.handle))

    # --- IDenoiser -------------------------------------------------------------
    @staticmethod
    def _cond(conditioning: dict, device: bool):
        keep = []
        arr = (NamedTensor * max(1, len(conditioning)))()
        for i, (name, value) in enumerate(conditioning.items()):
            if device:
                import torch
                dt = {torch.float32: _lib.ND_F32, torch.int32: _lib.ND_I32}[value.dtype]
                shape = (C.c_int64 * value.dim())(*value.shape)
                ptr, rank = value.data_ptr(), value.dim()
            else:
                a = np.ascontiguousarray(value)
                dt = {np.dtype(np.float32): _lib.ND_F32, np.dtype(np.int32): _lib.ND_I32}[a.dtype]
                shape = (C.c_int64 * a.ndim)(*a.shape)
                ptr, rank = a.ctypes.data, a.ndim
                keep.append(a)
            keep.append(shape)
            nm = name.encode()
            keep.append(nm)
            arr[i] = NamedTensor(nm, dt, rank, shape, ptr)
        return arr, keep

    def output_shape(self, latent_shape) -> tuple:
        """What predict returns for a latent of this shape: the latent's shape,
        or for a VAE decoder the [batch, 3, s h, s w] image."""
        d = self.desc
        b, _, h, w = latent_shape
        if d.family == FAMILY_VAE_KL:
            up = (d.unet_levels or 4) - 1
            return (b, 3, h << up, w << up)
        if d.family in (FAMILY_VAE_WAN21, FAMILY_VAE_WAN22):
            s = 16 if d.family == FAMILY_VAE_WAN22 else 8
            return (b, 3, h * s, w * s)
        return tuple(latent_shape)

    def predict(self, latent: np.ndarray, timestep: float, sigma: float, conditioning: dict,
                out: np.ndarray | None = None) -> np.ndarray:
        """One forward step from host memory (IDenoiser.Predict); `out` may be
        a caller-owned (e.g. pinned) float32 array of the output's shape."""
        lat = np.ascontiguousarray(latent, np.float32)
        shape = self.output_shape(lat.shape)
        if out is None:
            out = np.empty(shape, np.float32)
        elif out.shape != shape or out.dtype != np.float32 or not out.flags.c_contiguous:
            raise ValueError(f"out must be a contiguous float32 array of shape {shape}")
        arr, keep = self._cond(conditioning, device=False)
        check(_bind().nd_denoiser_predict(self.handle, lat.ctypes.data_as(C.c_void_p), timestep, sigma,
                                          len(conditioning), arr, out.ctypes.data_as(C.c_void_p)))
        del keep
        return out

    def text_encode(self, ids, source: np.ndarray | None = None, final_norm: bool = True) -> np.ndarray:
        """A text tower over token ids (nd_text_encode): Qwen3TextModel.Forward
        or LlmAdapter.Forward (source = the Qwen3 hidden states). Returns
        [len(ids), width] float32."""
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.empty((ids.size, self.desc.width), np.float32)
        src = None if source is None else np.ascontiguousarray(source, np.float32)
        check(_bind().nd_text_encode(self.handle, ids.ctypes.data_as(C.c_void_p), ids.size,
                                     None if src is None else src.ctypes.data_as(C.c_void_p),
                                     0 if src is None else src.shape[0], 1 if final_norm else 0,
                                     out.ctypes.data_as(C.c_void_p)))
        return out

    def predict_device(self, latent, timestep: float, sigma: float, conditioning: dict, out, stream=None):
        """The same over torch CUDA tensors, enqueued on `stream` (a cudaStream_t
        handle). stream=None: ordered with torch's current stream, as a torch op
        is -- the step runs on a stream of this object's own, after the current
        stream's work so far and before its work from here on. (The C ABI's
        null stream means the library's device stream, which is not ordered
        with torch's default stream.)"""
        import torch
        arr, keep = self._cond(conditioning, device=True)
        cur = None
        if stream is None:
            cur = torch.cuda.current_stream(latent.device)
            if self._side is None:
                self._side = torch.cuda.Stream(device=latent.device)
            self._side.wait_stream(cur)
            stream = self._side.cuda_stream
        check(_bind().nd_denoiser_predict_device(
            self.handle, C.c_void_p(latent.data_ptr()), timestep, sigma, len(conditioning), arr,
            C.c_void_p(out.data_ptr()), C.c_void_p(stream)))
        if cur is not None:
            cur.wait_stream(self._side)
        del keep
        return out

    def profile(self, steps: int = 1) -> list[dict]:
        """Per-kernel-class device time of one step (CUDA events around every
        launch of `steps` eager runs on the last staged inputs)."""
        arr = (KernelTime * 64)()
        n = C.c_int()
        check(_bind().nd_denoiser_profile(self.handle, steps, arr, 64, C.byref(n)))
        return [dict(name=arr[i].name.decode(), launches=arr[i].launches, ms=arr[i].total_ms,
                     flops=arr[i].flops, bytes=arr[i].bytes) for i in range(n.value)]

    def memory(self) -> Memory:
        m = Memory()
        check(_bind().nd_denoiser_memory(self.handle, C.byref(m)))
        return m

    @property
    def persistent_bytes(self) -> int:
        return self.memory().persistent_bytes

    @property
    def streamed_bytes(self) -> int:
        return self.memory().streamed_bytes

    @property
    def resident_bytes(self) -> int:
        return self.memory().resident_bytes

    @property
    def temporary_bytes(self) -> int:
        return self.memory().temporary_bytes

    @property
    def graph_count(self) -> int:
        return self.memory().graph_count

    def close(self) -> None:
        if self.handle:
            _bind().nd_denoiser_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def build_denoiser(device: Device, cfg, weights) -> CudaDenoiser:
    """IModelFamily.BuildDenoiser: create, copy every weight in, finalize.
    `weights` is an iterable of (name, array) or a dict."""
    d = CudaDenoiser(device, cfg.desc())
    try:
        items = weights.items() if isinstance(weights, dict) else weights
        for name, a in items:
            d.set_weight(name, a)
        d.finalize()
    except Exception:
        d.close()
        raise
    return d
