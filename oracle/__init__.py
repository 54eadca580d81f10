"""nd_oracle — TEST INFRASTRUCTURE, NOT PRODUCT CODE.

numpy front end of the C++ restatement of NaiveDiffusion's CPU layer
arithmetic (oracle/nd_oracle.cpp). Only tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / --impl reference legs may import this package, and
only as the checker or the timed CPU baseline. The product library
(naivediffusion_b200/libnd_denoise.so) never loads it.

Parity pinning: the reference is C# (.NET) and cannot be built here, so this
restatement is pinned by the known-answer checks of the reference's own unit
tests and smoke command, restated in tests/test_oracle.py.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"

_f = np.float32
_lib = None


def build(force: bool = False) -> Path:
    """Compile liboracle.so with the Makefile beside this file (g++ + OpenMP)."""
    src = HERE / "nd_oracle.cpp"
    if force or not LIB.exists() or LIB.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-B" if force else "-s", "-C", str(HERE)], check=True,
                       capture_output=True)
    return LIB


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(str(LIB))
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    return a.ctypes.data_as(C.c_void_p)


def _c(a, dtype=_f):
    return np.ascontiguousarray(a, dtype=dtype)


def threads() -> int:
    return int(lib().nd_oracle_threads())


# ------------------------------------------------------------------ dtypes

def to_f16_bits(x) -> np.ndarray:
    x = _c(x)
    y = np.empty(x.shape, np.uint16)
    lib().nd_oracle_f32_to_f16(_p(x), _p(y), C.c_int64(x.size))
    return y


def from_f16_bits(h) -> np.ndarray:
    h = _c(h, np.uint16)
    y = np.empty(h.shape, _f)
    lib().nd_oracle_f16_to_f32(_p(h), _p(y), C.c_int64(h.size))
    return y


def to_bf16_bits(x) -> np.ndarray:
    x = _c(x)
    y = np.empty(x.shape, np.uint16)
    lib().nd_oracle_f32_to_bf16(_p(x), _p(y), C.c_int64(x.size))
    return y


def from_bf16_bits(h) -> np.ndarray:
    h = _c(h, np.uint16)
    y = np.empty(h.shape, _f)
    lib().nd_oracle_bf16_to_f32(_p(h), _p(y), C.c_int64(h.size))
    return y


def round_bf16(x) -> np.ndarray:
    return from_bf16_bits(to_bf16_bits(x))


def round_f16(x) -> np.ndarray:
    return from_f16_bits(to_f16_bits(x))


# ------------------------------------------------------------------ layers

def linear(x, w, b=None) -> np.ndarray:
    """CpuMath.Linear (Tensors/CpuMath.cs:34-64)."""
    x = _c(x)
    w = _c(w)
    rows, inner = x.shape
    outer = w.shape[0]
    y = np.empty((rows, outer), _f)
    bb = None if b is None else _c(b)
    lib().nd_oracle_linear(_p(x), rows, inner, _p(w), _p(bb), _p(y), outer)
    return y


def layernorm(x, eps, weight=None, bias=None) -> np.ndarray:
    """CpuMath.LayerNorm (Tensors/CpuMath.cs:92-122); no affine when weight is None."""
    x = _c(x)
    rows, width = x.shape
    y = np.empty_like(x)
    w = None if weight is None else _c(weight)
    b = None if bias is None else _c(bias)
    lib().nd_oracle_layernorm(_p(x), rows, width, _p(w), _p(b), _p(y), C.c_float(eps))
    return y


def modulate(x, shift, scale, eps) -> np.ndarray:
    """Transformer.Modulate (Graph/Transformer.cs:72-80)."""
    x = _c(x)
    rows, width = x.shape
    y = np.empty_like(x)
    sh = None if shift is None else _c(shift)
    lib().nd_oracle_modulate(_p(x), rows, width, _p(sh), _p(_c(scale)), _p(y), C.c_float(eps))
    return y


def rmsnorm(x, weight, eps) -> np.ndarray:
    """CpuMath.RmsNorm (Tensors/CpuMath.cs:128-146) over the last axis."""
    x = _c(x)
    width = x.shape[-1]
    rows = x.size // width
    y = np.empty_like(x)
    w = None if weight is None else _c(weight)
    lib().nd_oracle_rmsnorm(_p(x), rows, width, _p(w), _p(y), C.c_float(eps))
    return y


def rope(x, heads, cos, sin) -> np.ndarray:
    """CpuMath.Rope (Tensors/CpuMath.cs:154-173), rotate-half; returns a copy."""
    y = _c(x).copy()
    rows = y.shape[0]
    dim = y.size // rows // heads
    lib().nd_oracle_rope(_p(y), rows, heads, dim, _p(_c(cos)), _p(_c(sin)))
    return y


def attention(q, k, v, heads, kv_heads=None, causal=False, key_len=0) -> np.ndarray:
    """CpuMath.Attention (Tensors/CpuMath.cs:203-248) plus the key-count mask."""
    q, k, v = _c(q), _c(k), _c(v)
    kv_heads = kv_heads or heads
    rows, key_rows = q.shape[0], k.shape[0]
    dim = q.shape[1] // heads
    y = np.empty_like(q)
    lib().nd_oracle_attention(_p(q), _p(k), _p(v), rows, key_rows, heads, kv_heads, dim,
                              int(causal), int(key_len), _p(y), C.c_int64(0), C.c_int64(0),
                              C.c_int64(0), C.c_int64(0))
    return y


def gelu(x) -> np.ndarray:
    y = _c(x).copy()
    lib().nd_oracle_gelu(_p(y), C.c_int64(y.size))
    return y


def gelu_tanh(x) -> np.ndarray:
    y = _c(x).copy()
    lib().nd_oracle_gelu_tanh(_p(y), C.c_int64(y.size))
    return y


def silu(x) -> np.ndarray:
    y = _c(x).copy()
    lib().nd_oracle_silu(_p(y), C.c_int64(y.size))
    return y


def sinusoid(time: float, width: int) -> np.ndarray:
    y = np.empty(width, _f)
    lib().nd_oracle_sinusoid(C.c_float(time), width, _p(y))
    return y


def qwen_rope_tables(rows, columns, text_len, context_rows):
    n = rows * columns + context_rows
    cos = np.empty((n, 64), _f)
    sin = np.empty((n, 64), _f)
    lib().nd_oracle_qwen_rope_tables(rows, columns, text_len, context_rows, _p(cos), _p(sin))
    return cos, sin


def anima_rope_tables(rows, columns, head_dim=128):
    n = rows * columns
    cos = np.empty((n, head_dim // 2), _f)
    sin = np.empty((n, head_dim // 2), _f)
    lib().nd_oracle_anima_rope_tables(rows, columns, head_dim, _p(cos), _p(sin))
    return cos, sin


# ------------------------------------------------------------------ int8

def quantize(w, group=32, scale_f16=True):
    """BlockQuantizer.Quantize (Tensors/BlockQuantizer.cs:34-105), group-generalised.
    Returns (q int8 [rows, cols], scales [rows, cols/group] as fp16 bits or fp32)."""
    w = _c(w)
    rows, cols = w.shape
    if group <= 0 or cols % group:
        raise ValueError(f"{cols} columns do not split into groups of {group}")
    q = np.empty((rows, cols), np.int8)
    s = np.empty((rows, cols // group), np.uint16 if scale_f16 else _f)
    rc = lib().nd_oracle_quantize(_p(w), rows, cols, group, int(scale_f16), _p(q), _p(s))
    if rc:
        raise ValueError("quantize: bad shape")
    return q, s


def dequantize(q, scales, group=32) -> np.ndarray:
    q = _c(q, np.int8)
    rows, cols = q.shape
    f16 = scales.dtype == np.uint16
    s = np.ascontiguousarray(scales)
    w = np.empty((rows, cols), _f)
    lib().nd_oracle_dequantize(_p(q), _p(s), int(f16), rows, cols, group, _p(w))
    return w


# ------------------------------------------------------------------ blocks

class _MMDiTStream(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "mod_w", "mod_b", "q_w", "q_b", "k_w", "k_b", "v_w", "v_b", "norm_q", "norm_k",
        "out_w", "out_b", "up_w", "up_b", "down_w", "down_b")]


class _AnimaBlock(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "self_mod1", "self_mod2", "cross_mod1", "cross_mod2", "mlp_mod1", "mlp_mod2",
        "sq", "sk", "sv", "so", "sq_norm", "sk_norm",
        "cq", "ck", "cv", "co", "cq_norm", "ck_norm", "fc1", "fc2")]


def mmdit_block(img: dict, txt: dict, x, n_img, temb, cos, sin, heads, key_len=0, eps=1e-6):
    """One dual-stream block (nd_oracle_mmdit_block). img/txt map the
    _MMDiTStream field names to float32 arrays. Returns the updated x."""
    keep = []

    def stream(d):
        s = _MMDiTStream()
        for name, _ in _MMDiTStream._fields_:
            a = _c(d[name])
            keep.append(a)
            setattr(s, name, a.ctypes.data)
        return s

    si, st = stream(img), stream(txt)
    x = _c(x).copy()
    width = x.shape[1]
    mlp = img["up_w"].shape[0]
    head_dim = width // heads
    lib().nd_oracle_mmdit_block(C.byref(si), C.byref(st), width, heads, head_dim, mlp, _p(x),
                                n_img, x.shape[0] - n_img, _p(_c(temb)), _p(_c(cos)),
                                _p(_c(sin)), int(key_len), C.c_float(eps))
    return x


def anima_block(w: dict, x, context, temb, lora, cos, sin, heads, eps=1e-6):
    keep = []
    s = _AnimaBlock()
    for name, _ in _AnimaBlock._fields_:
        a = _c(w[name])
        keep.append(a)
        setattr(s, name, a.ctypes.data)
    x = _c(x).copy()
    context = _c(context)
    width = x.shape[1]
    rank = w["self_mod1"].shape[0]
    mlp = w["fc1"].shape[0]
    lib().nd_oracle_anima_block(C.byref(s), width, heads, width // heads, mlp, rank, _p(x),
                                x.shape[0], _p(context), context.shape[0], context.shape[1],
                                _p(_c(temb)), _p(_c(lora)), _p(_c(cos)), _p(_c(sin)),
                                C.c_float(eps))
    return x


# ------------------------------------------------------------------ models

def patchify(latent, p):
    """[C, H, W] -> [(H/p)(W/p), C p p]; feature c*p*p + m*p + n of patch (i, j)
    is channel c at (p*i + m, p*j + n) (AnimaDit.Patchify, Models/Anima/AnimaDit.cs:193-247)."""
    c, h, w = latent.shape
    r, q = h // p, w // p
    return np.ascontiguousarray(latent.reshape(c, r, p, q, p).transpose(1, 3, 0, 2, 4).reshape(r * q, c * p * p))


def unpatchify(tokens, c, h, w, p):
    r, q = h // p, w // p
    return np.ascontiguousarray(tokens.reshape(r, q, c, p, p).transpose(2, 0, 3, 1, 4).reshape(c, h, w))


def mmdit_forward(w: dict, cfg, latent, context, sigma, cos=None, sin=None, key_len=0):
    """The dual-stream (Qwen-Image-style) denoiser step in fp32, composed from
    the restated primitives in the order of QwenImageDit.Build / .Block
    (Models/QwenImage/QwenImageDit.cs:309-505) with the dual-stream wiring of
    nd_oracle_mmdit_block. latent [1, C, H, W]; context [rows, width]."""
    D, p, eps = cfg.width, cfg.patch, cfg.eps
    C_, Hl, Wl = cfg.latent_channels, cfg.latent_height, cfg.latent_width
    n_img = (Hl // p) * (Wl // p)
    if cos is None:
        cos, sin = qwen_rope_tables(Hl // p, Wl // p, cfg.context_rows, cfg.context_rows)
    tok = patchify(np.asarray(latent, np.float32)[0], p)
    x_img = linear(tok, w["img_in.weight"], w.get("img_in.bias"))
    ctxn = rmsnorm(np.asarray(context, np.float32).reshape(cfg.context_rows, cfg.context_width),
                   w["txt_norm.weight"], eps)
    x_txt = linear(ctxn, w["txt_in.weight"], w.get("txt_in.bias"))
    x = np.concatenate([x_img, x_txt])
    tsin = sinusoid(np.float32(sigma * 1000.0), cfg.time_width)
    pre = "time_text_embed.timestep_embedder."
    h = silu(linear(tsin[None], w[pre + "linear_1.weight"], w.get(pre + "linear_1.bias")))
    temb = linear(h, w[pre + "linear_2.weight"], w.get(pre + "linear_2.bias"))[0]
    z = lambda n: np.zeros(n, np.float32)  # noqa: E731
    names = {
        0: dict(mod="img_mod.1", q="attn.to_q", k="attn.to_k", v="attn.to_v", nq="attn.norm_q",
                nk="attn.norm_k", out="attn.to_out.0", up="img_mlp.net.0.proj", down="img_mlp.net.2"),
        1: dict(mod="txt_mod.1", q="attn.add_q_proj", k="attn.add_k_proj", v="attn.add_v_proj",
                nq="attn.norm_added_q", nk="attn.norm_added_k", out="attn.to_add_out",
                up="txt_mlp.net.0.proj", down="txt_mlp.net.2"),
    }
    for b in range(cfg.blocks):
        pb = f"transformer_blocks.{b}."
        streams = []
        for s in range(2):
            n = names[s]
            g = lambda key, size: w.get(pb + n[key] + ".bias", z(size))  # noqa: E731
            streams.append(dict(
                mod_w=w[pb + n["mod"] + ".weight"], mod_b=g("mod", 6 * D),
                q_w=w[pb + n["q"] + ".weight"], q_b=g("q", D),
                k_w=w[pb + n["k"] + ".weight"], k_b=g("k", D),
                v_w=w[pb + n["v"] + ".weight"], v_b=g("v", D),
                norm_q=w[pb + n["nq"] + ".weight"], norm_k=w[pb + n["nk"] + ".weight"],
                out_w=w[pb + n["out"] + ".weight"], out_b=g("out", D),
                up_w=w[pb + n["up"] + ".weight"], up_b=g("up", cfg.mlp_width),
                down_w=w[pb + n["down"] + ".weight"], down_b=g("down", D)))
        x = mmdit_block(streams[0], streams[1], x, n_img, temb, cos, sin, cfg.heads, key_len, eps)
    emb = linear(silu(temb)[None], w["norm_out.linear.weight"], w.get("norm_out.linear.bias"))[0]
    y = modulate(x[:n_img], emb[D:], emb[:D], eps)
    out = linear(y, w["proj_out.weight"], w.get("proj_out.bias"))
    return unpatchify(out, C_, Hl, Wl, p)[None]


def anima_forward(w: dict, cfg, latent, context, sigma, cos=None, sin=None):
    """The Anima denoiser step in fp32 (AnimaDit.Build / .Predict,
    Models/Anima/AnimaDit.cs:124-134, 360-404), one batch item at a time.
    latent [B, 16, H, W]; context [B, rows, width]."""
    D, p, eps = cfg.width, cfg.patch, cfg.eps
    Hl, Wl = cfg.latent_height, cfg.latent_width
    if cos is None:
        cos, sin = anima_rope_tables(Hl // p, Wl // p, 128)
    tsin = sinusoid(np.float32(sigma), D)
    temb = rmsnorm(tsin[None], w["t_embedding_norm.weight"], eps)[0]
    lora = linear(silu(linear(tsin[None], w["t_embedder.1.linear_1.weight"])),
                  w["t_embedder.1.linear_2.weight"])[0]
    x_emb = np.ascontiguousarray(np.asarray(w["x_embedder.proj.1.weight"])[:, :64])
    outs = []
    for b in range(latent.shape[0]):
        x = linear(patchify(np.asarray(latent[b], np.float32), p), x_emb)
        for i in range(cfg.blocks):
            q = f"blocks.{i}."
            blk = dict(
                self_mod1=w[q + "adaln_modulation_self_attn.1.weight"], self_mod2=w[q + "adaln_modulation_self_attn.2.weight"],
                cross_mod1=w[q + "adaln_modulation_cross_attn.1.weight"], cross_mod2=w[q + "adaln_modulation_cross_attn.2.weight"],
                mlp_mod1=w[q + "adaln_modulation_mlp.1.weight"], mlp_mod2=w[q + "adaln_modulation_mlp.2.weight"],
                sq=w[q + "self_attn.q_proj.weight"], sk=w[q + "self_attn.k_proj.weight"],
                sv=w[q + "self_attn.v_proj.weight"], so=w[q + "self_attn.output_proj.weight"],
                sq_norm=w[q + "self_attn.q_norm.weight"], sk_norm=w[q + "self_attn.k_norm.weight"],
                cq=w[q + "cross_attn.q_proj.weight"], ck=w[q + "cross_attn.k_proj.weight"],
                cv=w[q + "cross_attn.v_proj.weight"], co=w[q + "cross_attn.output_proj.weight"],
                cq_norm=w[q + "cross_attn.q_norm.weight"], ck_norm=w[q + "cross_attn.k_norm.weight"],
                fc1=w[q + "mlp.layer1.weight"], fc2=w[q + "mlp.layer2.weight"])
            x = anima_block(blk, x, context[b], temb, lora, cos, sin, cfg.heads, eps)
        h = linear(silu(temb)[None], w["final_layer.adaln_modulation.1.weight"])
        f = linear(h, w["final_layer.adaln_modulation.2.weight"])[0] + lora[:2 * D]
        y = modulate(x, f[:D], f[D:], eps)
        out = linear(y, w["final_layer.linear.weight"])
        outs.append(unpatchify(out, cfg.latent_channels, Hl, Wl, p))
    return np.stack(outs)


def rope_pairs(x, heads, cos, sin) -> np.ndarray:
    """The rotation Qwen-Image's own model applies: adjacent feature pairs
    (2i, 2i+1) of every head turned by angle i. The reference's graph runs
    rotate-half on weights permuted pairs -> halves (QwenImageDit.PairsToHalves,
    Models/QwenImage/QwenImageDit.cs:261-279), which is this rotation with the
    features reordered; the oracle turns the pairs directly on the file's own
    weight order, so the device's permutation is checked, not repeated."""
    x = _c(x)
    rows = x.shape[0]
    h = x.reshape(rows, heads, -1)
    c = _c(cos)[:, None, :]
    s = _c(sin)[:, None, :]
    a, b = h[:, :, 0::2], h[:, :, 1::2]
    y = np.empty_like(h)
    y[:, :, 0::2] = a * c - b * s
    y[:, :, 1::2] = b * c + a * s
    return y.reshape(x.shape)


def qwen_image_forward(w: dict, cfg, latent, context, sigma, cos=None, sin=None, key_len=0):
    """Qwen-Image 2.1's single-stream step in fp32, composed in the order of
    QwenImageDit.Build / .Block / .Attention / .FeedForward
    (Models/QwenImage/QwenImageDit.cs:306-505): image rows then text rows,
    one modulation [2, 4D] (time sigma and time zero) shared by every block
    with tanh'd gates, image queries over the visible keys, text queries
    under QwenImageConditioning.CausalTable (causal, closed over the padding,
    Models/QwenImage/QwenImageConditioner.cs:66-78). latent [1, 64, H, W];
    context [rows, width]; key_len = image tokens + real text rows (0: all)."""
    D, H, F, eps = cfg.width, cfg.heads, cfg.mlp_width, cfg.eps
    C_, Hl, Wl, R = cfg.latent_channels, cfg.latent_height, cfg.latent_width, cfg.context_rows
    n_img = Hl * Wl
    real = key_len - n_img if key_len else R
    if cos is None:
        cos, sin = qwen_rope_tables(Hl, Wl, real, R)
    x_img = linear(patchify(np.asarray(latent, np.float32)[0], 1), w["img_in.weight"])
    ctx = np.asarray(context, np.float32).reshape(R, cfg.context_width)
    t = rmsnorm(ctx, np.asarray(w["txt_in.text_norm.weight"], np.float32) + np.float32(1), eps)
    t = linear(gelu_tanh(linear(t, w["txt_in.in_layer.weight"])), w["txt_in.out_layer.weight"])
    x = np.concatenate([x_img, t])
    tsin = np.stack([sinusoid(np.float32(sigma * 1000.0), cfg.time_width), sinusoid(np.float32(0), cfg.time_width)])
    pre = "time_text_embed.timestep_embedder."
    temb = linear(silu(linear(tsin, w[pre + "linear_1.weight"])), w[pre + "linear_2.weight"])
    mod = linear(silu(temb), w["modulation.1.weight"])
    scale_a, gate_a = mod[:, :D], np.tanh(mod[:, D:2 * D])
    scale_m, gate_m = mod[:, 2 * D:3 * D], np.tanh(mod[:, 3 * D:])

    def rows(v):  # the noise level's row over the image rows, time zero's over the text
        return np.concatenate([np.broadcast_to(v[0], (n_img, D)), np.broadcast_to(v[1], (R, D))])

    def mod_rows(x, scale):
        return np.concatenate([modulate(x[:n_img], None, scale[0], eps), modulate(x[n_img:], None, scale[1], eps)])

    img_keys = n_img + real if real < R else 0
    txt_keys = real if real < R else 0
    for b in range(cfg.blocks):
        p = f"transformer_blocks.{b}."
        n = mod_rows(x, scale_a)
        M = n.shape[0]

        def qk(name, norm):
            y = linear(n, w[p + name])
            y = rmsnorm(y.reshape(M * H, 128), w[p + norm], eps).reshape(M, D)
            return rope_pairs(y, H, cos, sin)
        q, k = qk("attn.to_q.weight", "attn.norm_q.weight"), qk("attn.to_k.weight", "attn.norm_k.weight")
        v = linear(n, w[p + "attn.to_v.weight"])
        a_img = attention(q[:n_img], k, v, H, key_len=img_keys)
        a_txt = attention(q[n_img:], k[n_img:], v[n_img:], H, causal=True, key_len=txt_keys)
        o = linear(np.concatenate([a_img, a_txt]), w[p + "attn.to_out.0.weight"])
        x = x + rows(gate_a) * o
        n = mod_rows(x, scale_m)
        if p + "img_mlp.gate_up.weight" in w:
            gu = linear(n, w[p + "img_mlp.gate_up.weight"])
        else:
            gu = np.concatenate([linear(n, w[p + "img_mlp.gate_layer.weight"]),
                                 linear(n, w[p + "img_mlp.proj.weight"])], axis=1)
        h = silu(np.ascontiguousarray(gu[:, :F])) * gu[:, F:]
        x = x + rows(gate_m) * linear(h, w[p + "img_mlp.out.weight"])
    scale = linear(silu(temb[:1]), w["norm_out.linear.weight"])[0]
    y = modulate(x[:n_img], None, scale, eps)
    out = linear(y, w["proj_out.weight"])
    return unpatchify(out, C_, Hl, Wl, 1)[None]


def causal_table(real: int, rows: int) -> np.ndarray:
    """QwenImageConditioning.CausalTable (Models/QwenImage/QwenImageConditioner.cs:66-78):
    row i may read key j when j <= i and j < real."""
    i = np.arange(rows)[:, None]
    j = np.arange(rows)[None, :]
    return ((j <= i) & (j < real)).astype(np.int32)


def group_norm(x, groups, weight=None, bias=None, eps=1e-5, silu=False):
    """GroupNorm over one image x [C, H, W] (or [C, HW])."""
    x = _c(x)
    ch = x.shape[0]
    HW = x.size // ch
    y = np.empty_like(x)
    w = None if weight is None else _c(weight)
    b = None if bias is None else _c(bias)
    lib().nd_oracle_group_norm(_p(x), ch, HW, groups, _p(w), _p(b), C_float(eps),
                               int(silu), _p(y))
    return y


def C_float(v):
    return C.c_float(v)


def conv2d(x, w, b=None, stride=1, pad=1):
    """x [Cin, H, W], w [Cout, Cin, k, k] -> [Cout, Ho, Wo]."""
    x = _c(x)
    w = _c(w)
    Cin, H, W = x.shape
    Cout, _, k, _ = w.shape
    Ho, Wo = (H + 2 * pad - k) // stride + 1, (W + 2 * pad - k) // stride + 1
    y = np.empty((Cout, Ho, Wo), _f)
    bb = None if b is None else _c(b)
    lib().nd_oracle_conv2d(_p(x), Cin, H, W, _p(w), _p(bb), Cout, k, stride, pad, _p(y))
    return y


def unet_resblock(w: dict, p: str, x, temb):
    """UNetModel.ResnetBlock (Models/Sdxl/UNetModel.cs:230-254) on one image
    x [C, H, W]: GN+SiLU, conv3x3, + the time projection, GN+SiLU, conv3x3,
    plus the (1x1-projected when the width changes) input."""
    h = group_norm(x, 32, w[p + ".norm1.weight"], w.get(p + ".norm1.bias"), 1e-5, True)
    h = conv2d(h, w[p + ".conv1.weight"], w.get(p + ".conv1.bias"))
    proj = linear(silu(temb)[None], w[p + ".time_emb_proj.weight"], w.get(p + ".time_emb_proj.bias"))[0]
    h = h + proj[:, None, None]
    h = group_norm(h, 32, w[p + ".norm2.weight"], w.get(p + ".norm2.bias"), 1e-5, True)
    h = conv2d(h, w[p + ".conv2.weight"], w.get(p + ".conv2.bias"))
    if p + ".conv_shortcut.weight" in w:
        sc = w[p + ".conv_shortcut.weight"]
        x = conv2d(x, sc.reshape(sc.shape[0], sc.shape[1], 1, 1), w.get(p + ".conv_shortcut.bias"), 1, 0)
    return x + h


def _unet_attn(w: dict, x, src, p, heads):
    q = linear(x, w[p + ".to_q.weight"])
    k = linear(src, w[p + ".to_k.weight"])
    v = linear(src, w[p + ".to_v.weight"])
    return linear(attention(q, k, v, heads), w[p + ".to_out.0.weight"], w.get(p + ".to_out.0.bias"))


def unet_transformer2d(w: dict, p: str, x, ctx):
    """UNetModel.Transformer2d (Models/Sdxl/UNetModel.cs:279-301) on one image
    x [C, H, W] with its context rows: GN (eps 1e-6), proj_in, the blocks
    (self-attention, cross-attention, GEGLU feed-forward, each after an
    LN with eps 1e-5), proj_out, plus the input."""
    c, h_, w_ = x.shape
    t = group_norm(x, 32, w[p + ".norm.weight"], w.get(p + ".norm.bias"), 1e-6).reshape(c, -1).T
    t = linear(np.ascontiguousarray(t), w[p + ".proj_in.weight"], w.get(p + ".proj_in.bias"))
    j = 0
    while f"{p}.transformer_blocks.{j}.norm1.weight" in w:
        q = f"{p}.transformer_blocks.{j}"
        heads = c // 64
        n = layernorm(t, 1e-5, w[q + ".norm1.weight"], w.get(q + ".norm1.bias"))
        t = t + _unet_attn(w, n, n, q + ".attn1", heads)
        n = layernorm(t, 1e-5, w[q + ".norm2.weight"], w.get(q + ".norm2.bias"))
        t = t + _unet_attn(w, n, ctx, q + ".attn2", heads)
        n = layernorm(t, 1e-5, w[q + ".norm3.weight"], w.get(q + ".norm3.bias"))
        hh = linear(n, w[q + ".ff.net.0.proj.weight"], w.get(q + ".ff.net.0.proj.bias"))
        inner = hh.shape[1] // 2
        t = t + linear(hh[:, :inner] * gelu(hh[:, inner:]), w[q + ".ff.net.2.weight"], w.get(q + ".ff.net.2.bias"))
        j += 1
    t = linear(t, w[p + ".proj_out.weight"], w.get(p + ".proj_out.bias"))
    return np.ascontiguousarray(t.T.reshape(c, h_, w_)) + x


def unet_forward(w: dict, cfg, latent, timestep, add, context):
    """The SDXL UNet step in fp32, one image at a time (UNetModel.Build,
    Models/Sdxl/UNetModel.cs:333-437). latent [B, 4, H, W]; add [B, aw];
    context [B, rows, width]."""
    from math import cos, exp, log, sin

    def tstep(t, dim):
        half = dim // 2
        f = [exp(-log(10000.0) * i / half) for i in range(half)]
        return np.array([cos(t * x) for x in f] + [sin(t * x) for x in f], np.float32)

    def mlp(x, p):
        return linear(silu(linear(x, w[p + ".linear_1.weight"], w.get(p + ".linear_1.bias"))),
                      w[p + ".linear_2.weight"], w.get(p + ".linear_2.bias"))

    def res(x, p, temb):
        return unet_resblock(w, p, x, temb)

    def t2d(x, p, ctx):
        return unet_transformer2d(w, p, x, ctx)

    L = len(cfg.mult)
    outs = []
    for b in range(latent.shape[0]):
        temb = mlp(tstep(timestep, cfg.time_width)[None], "time_embedding")[0] + \
            mlp(np.asarray(add[b], np.float32)[None], "add_embedding")[0]
        ctx = np.asarray(context[b], np.float32)
        x = conv2d(np.asarray(latent[b], np.float32), w["conv_in.weight"], w.get("conv_in.bias"))
        skips = [x]
        for lvl in range(L):
            for i in range(cfg.resnets):
                x = res(x, f"down_blocks.{lvl}.resnets.{i}", temb)
                if cfg.depth[lvl] > 0:
                    x = t2d(x, f"down_blocks.{lvl}.attentions.{i}", ctx)
                skips.append(x)
            if lvl != L - 1:
                x = conv2d(x, w[f"down_blocks.{lvl}.downsamplers.0.conv.weight"],
                           w.get(f"down_blocks.{lvl}.downsamplers.0.conv.bias"), stride=2)
                skips.append(x)
        x = res(x, "mid_block.resnets.0", temb)
        x = t2d(x, "mid_block.attentions.0", ctx)
        x = res(x, "mid_block.resnets.1", temb)
        for i in range(L):
            lvl = L - 1 - i
            for j in range(cfg.resnets + 1):
                x = np.concatenate([x, skips.pop()], 0)
                x = res(x, f"up_blocks.{i}.resnets.{j}", temb)
                if cfg.depth[lvl] > 0:
                    x = t2d(x, f"up_blocks.{i}.attentions.{j}", ctx)
            if i != L - 1:
                x = x.repeat(2, axis=1).repeat(2, axis=2)
                x = conv2d(x, w[f"up_blocks.{i}.upsamplers.0.conv.weight"], w.get(f"up_blocks.{i}.upsamplers.0.conv.bias"))
        x = group_norm(x, 32, w["conv_norm_out.weight"], w.get("conv_norm_out.bias"), 1e-5, True)
        outs.append(conv2d(x, w["conv_out.weight"], w.get("conv_out.bias")))
    return np.stack(outs)


def sampler_step(sampler, prediction, out, sample, guidance=1.0, last=None, noise=None, sigma=1.0,
                 sigma_next=0.0, up=0.0, down=0.0, rescale=1.0, noise_scale=0.0, shrink=0.0, weight=0.0,
                 second_order=False, want_denoised=False):
    """One guidance combine + solver step in the reference's arithmetic
    (Sampling/Schedulers.cs Step, Pipeline/GuidanceStrategy.cs Combine).
    out [branches, n]; sample [n] is returned updated (copies), with last."""
    out = _c(np.atleast_2d(out))
    branches, n = out.shape
    s = _c(sample).copy()
    lst = _c(last).copy() if last is not None else np.zeros(n, _f)
    nz = _c(noise) if noise is not None else None
    den = np.empty(n, _f) if want_denoised else None
    lib().nd_oracle_sampler_step(int(sampler), int(prediction), C.c_int64(n), int(branches), _p(out),
                                 C.c_float(guidance), _p(s), _p(lst), _p(nz), _p(den), C.c_float(sigma),
                                 C.c_float(sigma_next), C.c_double(up), C.c_double(down), C.c_double(rescale),
                                 C.c_double(noise_scale), C.c_double(shrink), C.c_double(weight),
                                 int(bool(second_order)))
    return (s, lst, den) if want_denoised else (s, lst)


def vae_decode(w: dict, cfg, latent):
    """AutoencoderKl.Decoder (Vae/AutoencoderKl.cs:78-116) in fp32, one image
    at a time: latent [B, 4, h, w] -> image [B, 3, 8h, 8w]."""
    eps = cfg.eps

    def res(x, p):
        h = group_norm(x, 32, w[p + ".norm1.weight"], w.get(p + ".norm1.bias"), eps, True)
        h = conv2d(h, w[p + ".conv1.weight"], w.get(p + ".conv1.bias"))
        h = group_norm(h, 32, w[p + ".norm2.weight"], w.get(p + ".norm2.bias"), eps, True)
        h = conv2d(h, w[p + ".conv2.weight"], w.get(p + ".conv2.bias"))
        if p + ".conv_shortcut.weight" in w:
            x = conv2d(x, w[p + ".conv_shortcut.weight"], w.get(p + ".conv_shortcut.bias"), 1, 0)
        return x + h

    def attn(x, p):
        c, hh, ww = x.shape
        t = np.ascontiguousarray(group_norm(x, 32, w[p + ".group_norm.weight"], w.get(p + ".group_norm.bias"),
                                            eps).reshape(c, -1).T)
        q = linear(t, w[p + ".to_q.weight"], w.get(p + ".to_q.bias"))
        k = linear(t, w[p + ".to_k.weight"], w.get(p + ".to_k.bias"))
        v = linear(t, w[p + ".to_v.weight"], w.get(p + ".to_v.bias"))
        o = linear(attention(q, k, v, 1), w[p + ".to_out.0.weight"], w.get(p + ".to_out.0.bias"))
        return np.ascontiguousarray(o.T.reshape(c, hh, ww)) + x

    L = len(cfg.mult)
    outs = []
    for b in range(latent.shape[0]):
        x = conv2d(np.asarray(latent[b], np.float32), w["post_quant_conv.weight"], w.get("post_quant_conv.bias"), 1, 0)
        x = conv2d(x, w["decoder.conv_in.weight"], w.get("decoder.conv_in.bias"))
        x = res(x, "decoder.mid_block.resnets.0")
        x = attn(x, "decoder.mid_block.attentions.0")
        x = res(x, "decoder.mid_block.resnets.1")
        for i in range(L):
            for j in range(cfg.layers_per_block + 1):
                x = res(x, f"decoder.up_blocks.{i}.resnets.{j}")
            if i != L - 1:
                x = x.repeat(2, axis=1).repeat(2, axis=2)
                x = conv2d(x, w[f"decoder.up_blocks.{i}.upsamplers.0.conv.weight"],
                           w.get(f"decoder.up_blocks.{i}.upsamplers.0.conv.bias"))
        x = group_norm(x, 32, w["decoder.conv_norm_out.weight"], w.get("decoder.conv_norm_out.bias"), eps, True)
        outs.append(conv2d(x, w["decoder.conv_out.weight"], w.get("decoder.conv_out.bias")))
    return np.stack(outs)


def vae_tile_starts(extent: int, tile: int, overlap: int) -> list:
    """VaeTiling.TileStarts (Vae/VaeTiling.cs:12-25): equal tiles, enough of
    them to keep every overlap at least `overlap` wide, origins spread evenly
    (Math.Round: half to even)."""
    if extent <= tile:
        return [0]
    count = ((extent - overlap) + (tile - overlap) - 1) // (tile - overlap)
    span = extent - tile
    return [int(round(float(i) * span / (count - 1))) for i in range(count)]


def vae_crossfade(starts, tile: int) -> np.ndarray:
    """VaeTiling.Crossfade (Vae/VaeTiling.cs:29-49), float32 as there."""
    weight = np.ones(tile, np.float32)
    if len(starts) > 1:
        step = min(starts[i] - starts[i - 1] for i in range(1, len(starts)))
        overlap = tile - step
        for i in range(overlap):
            ramp = _f(i + 1) / _f(overlap + 1)
            weight[i] = ramp
            weight[tile - 1 - i] = ramp
    return weight


def vae_window(rows, cols, side: int) -> np.ndarray:
    """VaeTiling.Window (Vae/VaeTiling.cs:55-68): window[y, x] = vertical[y] * horizontal[x]."""
    v, h = vae_crossfade(rows, side), vae_crossfade(cols, side)
    out = np.empty((side, side), np.float32)
    for y in range(side):
        out[y] = v[y] * h
    return out


def vae_tile_blend(tiles, rows, cols, height: int, width: int) -> np.ndarray:
    """BlendTile over the tiles in row-then-column order, then DivideByWeights
    (Vae/TiledVae.cs:84-121), in float32 one operation at a time: tiles
    [len(rows) * len(cols), C, side, side] -> [C, height, width]."""
    tiles = np.asarray(tiles, np.float32)
    side = tiles.shape[-1]
    win = vae_window(rows, cols, side)
    target = np.zeros((tiles.shape[1], height, width), np.float32)
    weight = np.zeros((height, width), np.float32)
    t = 0
    for top in rows:
        for left in cols:
            target[:, top:top + side, left:left + side] += tiles[t] * win
            weight[top:top + side, left:left + side] += win
            t += 1
    target *= _f(1.0) / weight
    return target


def vae_tiled_decode(decode, latent, scale: int, tile: int = 64, overlap: int = 8) -> np.ndarray:
    """TiledVaeDecoder.Run (Vae/TiledVae.cs:136-159) with the tile geometry of
    the TiledVae constructor (:43-55): `decode` maps one latent tile
    [C, t, t] to its image [3, t * scale, t * scale]; latent [1, C, h, w] ->
    image [1, 3, h * scale, w * scale]."""
    lat = np.asarray(latent, np.float32)[0]
    h, w = lat.shape[1] * scale, lat.shape[2] * scale
    t = min(tile, min(h, w) // scale)
    overlap = min(overlap, t // 2)
    rows = vae_tile_starts(h // scale, t, overlap)
    cols = vae_tile_starts(w // scale, t, overlap)
    tiles = np.stack([decode(np.ascontiguousarray(lat[:, r:r + t, c:c + t])) for r in rows for c in cols])
    return vae_tile_blend(tiles, [r * scale for r in rows], [c * scale for c in cols], h, w)[None]


def wan_channel_rms(x, gamma, silu_after=False):
    """WanVae.ChannelRmsNorm (Vae/WanVae.cs:111-121) over one image x [C, H, W]:
    each pixel's channels over sqrt(mean(x^2) + 1e-24 / C), times gamma."""
    c = x.shape[0]
    t = np.ascontiguousarray(np.asarray(x, np.float32).reshape(c, -1).T)
    y = rmsnorm(t, gamma, 1e-24 / c)
    if silu_after:
        y = silu(y)
    return np.ascontiguousarray(y.T.reshape(x.shape))


def wan22_up_shortcut(x, out_c, temporal):
    """Wan22Vae.UpShortcut (Vae/Wan22Vae.cs:121-155) for one image x [C, H, W]."""
    c = x.shape[0]
    if c == out_c:
        return x.repeat(2, axis=1).repeat(2, axis=2)
    if c != 2 * out_c:
        raise ValueError("an up level halves its channels at most")
    if temporal:
        return x[1::2].repeat(2, axis=1).repeat(2, axis=2)
    _, h, w = x.shape
    y = np.empty((out_c, 2 * h, 2 * w), np.float32)
    y[:, 0::2, :] = x[0::2].repeat(2, axis=2)
    y[:, 1::2, :] = x[1::2].repeat(2, axis=2)
    return y


def wan_vae_decode(w: dict, cfg, latent):
    """WanVae.Decoder / Wan22Vae.Decoder (Vae/WanVae.cs:170-207,
    Vae/Wan22Vae.cs:161-206) in fp32 on one frame, one image at a time:
    latent [B, C, h, w] -> image [B, 3, s h, s w] (Wan 2.2's RGB of RGBA)."""
    v22 = cfg.version == 22

    def res(x, p):
        h = conv2d(wan_channel_rms(x, w[p + ".residual.0.gamma"], True), w[p + ".residual.2.weight"],
                   w.get(p + ".residual.2.bias"))
        h = conv2d(wan_channel_rms(h, w[p + ".residual.3.gamma"], True), w[p + ".residual.6.weight"],
                   w.get(p + ".residual.6.bias"))
        if p + ".shortcut.weight" in w:
            x = conv2d(x, w[p + ".shortcut.weight"], w.get(p + ".shortcut.bias"), 1, 0)
        return x + h

    def attn(x, p):
        c, hh, ww = x.shape
        qkv = conv2d(wan_channel_rms(x, w[p + ".norm.gamma"]), w[p + ".to_qkv.weight"], w.get(p + ".to_qkv.bias"), 1, 0)
        part = lambda i: np.ascontiguousarray(qkv[i * c:(i + 1) * c].reshape(c, -1).T)  # noqa: E731
        o = np.ascontiguousarray(attention(part(0), part(1), part(2), 1).T.reshape(c, hh, ww))
        return conv2d(o, w[p + ".proj.weight"], w.get(p + ".proj.bias"), 1, 0) + x

    L = 5 if v22 else 4
    temporal = (False, True, True, True)
    outs = []
    for b in range(latent.shape[0]):
        x = conv2d(np.asarray(latent[b], np.float32), w["conv2.weight"], w.get("conv2.bias"), 1, 0)
        x = conv2d(x, w["decoder.conv1.weight"], w.get("decoder.conv1.bias"))
        x = res(x, "decoder.middle.0")
        x = attn(x, "decoder.middle.1")
        x = res(x, "decoder.middle.2")
        idx = 0
        for level in range(L):
            pre = f"decoder.upsamples.{level}.upsamples." if v22 else "decoder.upsamples."
            if v22:
                idx = 0
            inp = x
            for _ in range(cfg.resnets + 1):
                x = res(x, f"{pre}{idx}")
                idx += 1
            if level != L - 1:
                x = x.repeat(2, axis=1).repeat(2, axis=2)
                x = conv2d(x, w[f"{pre}{idx}.resample.1.weight"], w.get(f"{pre}{idx}.resample.1.bias"))
                idx += 1
                if v22:
                    x = x + wan22_up_shortcut(inp, x.shape[0], temporal[L - 2 - level])
        x = wan_channel_rms(x, w["decoder.head.0.gamma"], True)
        outs.append(conv2d(x, w["decoder.head.2.weight"], w.get("decoder.head.2.bias"))[:3])
    return np.stack(outs)


# ------------------------------------------------------------------ text towers

def rope_tables_1d(rows, dim, theta):
    """CpuMath.RopeTables (Tensors/CpuMath.cs:177-194): inverse frequencies in
    float32, angle = position * frequency, [rows, dim / 2] cos and sin."""
    half = dim // 2
    i = np.arange(half, dtype=np.float32)
    freq = np.float32(1) / np.power(np.float32(theta), np.float32(2) * i / np.float32(dim))
    ang = np.arange(rows, dtype=np.float32)[:, None] * freq[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def qwen3_text_forward(w: dict, cfg, ids, final_norm=True):
    """Qwen3TextModel.Forward (Text/Qwen/Qwen3TextModel.cs:47-104) in fp32:
    ids [rows] -> hidden states [rows, width]."""
    ids = np.asarray(ids, np.int64)
    n, W, H, KV, eps = ids.size, cfg.width, cfg.heads, cfg.kv_heads, cfg.eps
    x = np.ascontiguousarray(np.asarray(w["model.embed_tokens.weight"], np.float32)[ids])
    cos, sin = rope_tables_1d(n, 128, cfg.rope_theta)
    for l in range(cfg.blocks):
        p = f"model.layers.{l}."
        t = rmsnorm(x, w[p + "input_layernorm.weight"], eps)
        q = linear(t, w[p + "self_attn.q_proj.weight"])
        k = linear(t, w[p + "self_attn.k_proj.weight"])
        v = linear(t, w[p + "self_attn.v_proj.weight"])
        q = rmsnorm(q.reshape(n * H, 128), w[p + "self_attn.q_norm.weight"], eps).reshape(n, H * 128)
        k = rmsnorm(k.reshape(n * KV, 128), w[p + "self_attn.k_norm.weight"], eps).reshape(n, KV * 128)
        q = rope(q, H, cos, sin)
        k = rope(k, KV, cos, sin)
        a = attention(q, k, v, H, kv_heads=KV, causal=True)
        x = x + linear(a, w[p + "self_attn.o_proj.weight"])
        t = rmsnorm(x, w[p + "post_attention_layernorm.weight"], eps)
        g = silu(linear(t, w[p + "mlp.gate_proj.weight"]))
        x = x + linear(g * linear(t, w[p + "mlp.up_proj.weight"]), w[p + "mlp.down_proj.weight"])
    return rmsnorm(x, w["model.norm.weight"], eps) if final_norm else x


def llm_adapter_forward(w: dict, cfg, ids, context):
    """LlmAdapter.Forward (Models/Anima/LlmAdapter.cs:29-102) in fp32: T5 ids
    [rows] and Qwen3 hidden states [context_rows, width] -> [rows, width]."""
    ids = np.asarray(ids, np.int64)
    ctx = np.ascontiguousarray(context, np.float32)
    n, S, W, H, hd, eps = ids.size, ctx.shape[0], cfg.width, cfg.heads, cfg.head_dim, cfg.eps
    x = np.ascontiguousarray(np.asarray(w["embed.weight"], np.float32)[ids])
    cos, sin = rope_tables_1d(n, hd, cfg.rope_theta)
    ccos, csin = rope_tables_1d(S, hd, cfg.rope_theta)

    def attend(p, queries, source, qc, qs, kc, ks):
        q = linear(queries, w[p + ".q_proj.weight"])
        k = linear(source, w[p + ".k_proj.weight"])
        v = linear(source, w[p + ".v_proj.weight"])
        q = rmsnorm(q.reshape(-1, hd), w[p + ".q_norm.weight"], eps).reshape(q.shape)
        k = rmsnorm(k.reshape(-1, hd), w[p + ".k_norm.weight"], eps).reshape(k.shape)
        return attention(rope(q, H, qc, qs), rope(k, H, kc, ks), v, H)

    for b in range(cfg.blocks):
        p = f"blocks.{b}."
        t = rmsnorm(x, w[p + "norm_self_attn.weight"], eps)
        x = x + linear(attend(p + "self_attn", t, t, cos, sin, cos, sin), w[p + "self_attn.o_proj.weight"])
        t = rmsnorm(x, w[p + "norm_cross_attn.weight"], eps)
        x = x + linear(attend(p + "cross_attn", t, ctx, cos, sin, ccos, csin), w[p + "cross_attn.o_proj.weight"])
        t = rmsnorm(x, w[p + "norm_mlp.weight"], eps)
        h = gelu(linear(t, w[p + "mlp.0.weight"], w.get(p + "mlp.0.bias")))
        x = x + linear(h, w[p + "mlp.2.weight"], w.get(p + "mlp.2.bias"))
    y = linear(x, w["out_proj.weight"], w.get("out_proj.bias"))
    return rmsnorm(y, w["norm.weight"], eps)
