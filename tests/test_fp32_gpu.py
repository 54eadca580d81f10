"""fp32 compute (model_desc.compute == ND_F32) against the fp32 oracle.

The task's fp32 bar: max|d| / max|ref| <= 1e-4 for layer outputs. The GEMMs
run on bf16 hi|lo operand pairs (ND_BF16X2: hi.hi + hi.lo + lo.hi, fp32
accumulation), the attention in fp32 on the CUDA cores; everything else is
fp32. The layer tests hold 1e-5 (a GEMM alone) and the composed steps 1e-4.
"""
import numpy as np
import pytest
import torch

import oracle as O
from naivediffusion_b200 import _lib, ops
from naivediffusion_b200.denoiser import AnimaConfig, Device, build_denoiser, synthetic_weights

pytestmark = pytest.mark.gpu

F32 = _lib.ND_F32


def rel(a, b):
    a = np.asarray(a, np.float64)
    return float(np.abs(a - b).max() / np.abs(b).max())


def _rand(shape, seed, scale=1.0):
    return (np.random.default_rng(seed).standard_normal(shape) * scale).astype(np.float32)


@pytest.mark.parametrize("m,k,n", [(300, 512, 384), (128, 64, 64), (1000, 2048, 2048)])
def test_pair_gemm_store_matches_fp32(cuda, m, k, n):
    x, w, b = _rand((m, k), 1), _rand((n, k), 2, 0.02), _rand((n,), 3, 0.1)
    y = ops.linear(ops.to_pairs(torch.from_numpy(x).cuda()), ops.to_pairs(torch.from_numpy(w).cuda()),
                   torch.from_numpy(b).cuda(), pairs=True)
    torch.cuda.synchronize()
    ref = O.linear(x, w, b)
    assert y.shape == (m, 2 * n)
    assert rel(ops.from_pairs(y).cpu().numpy(), ref) < 1e-5


def test_pair_gemm_epilogues(cuda):
    m, k, n = 256, 256, 512
    x, w, b = _rand((m, k), 4), _rand((2 * n, k), 5, 0.05), _rand((2 * n,), 6, 0.1)
    xp = ops.to_pairs(torch.from_numpy(x).cuda())
    wp = ops.to_pairs(torch.from_numpy(w).cuda())
    ref = np.concatenate([O.linear(x[:128], w[:n], b[:n]), O.linear(x[128:], w[n:], b[n:])])
    # two row groups, exact GELU
    y = ops.linear(xp, wp, torch.from_numpy(b).cuda(), epilogue=_lib.ND_EPI_GELU_ERF, group_split=128, pairs=True)
    # gated fp32 residual
    gate = _rand((2, n), 7)
    res0 = _rand((m, n), 8)
    res = torch.from_numpy(res0.copy()).cuda()
    ops.linear(xp, wp, torch.from_numpy(b).cuda(), epilogue=_lib.ND_EPI_RESIDUAL_GATE, residual=res,
               gate=torch.from_numpy(gate).cuda(), group_split=128, pairs=True)
    y32 = ops.linear(xp, wp, torch.from_numpy(b).cuda(), epilogue=_lib.ND_EPI_STORE_F32, group_split=128, pairs=True)
    torch.cuda.synchronize()
    assert rel(ops.from_pairs(y).cpu().numpy(), O.gelu(ref)) < 1e-5
    g = np.concatenate([np.broadcast_to(gate[0], (128, n)), np.broadcast_to(gate[1], (128, n))])
    assert rel(res.cpu().numpy(), res0 + g * ref) < 1e-5
    assert rel(y32.cpu().numpy(), ref) < 1e-5


def test_pair_gemm_head_norm_rope_writes_fp32(cuda):
    m, k, heads = 200, 256, 2
    D = heads * 128
    x, w = _rand((m, k), 9), _rand((3 * D, k), 10, 0.05)
    qn = (1 + _rand((2, 128), 11, 0.1)).astype(np.float32)
    ang = _rand((m, 64), 12)
    cos_t, sin_t = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    y = ops.linear(ops.to_pairs(torch.from_numpy(x).cuda()), ops.to_pairs(torch.from_numpy(w).cuda()),
                   epilogue=_lib.ND_EPI_QK_NORM_ROPE, qk_norm=torch.from_numpy(qn).cuda(),
                   rope_cos=torch.from_numpy(cos_t).cuda(), rope_sin=torch.from_numpy(sin_t).cuda(),
                   qk_cols=2 * D, pairs=True)
    torch.cuda.synchronize()
    assert y.dtype == torch.float32 and y.shape == (m, 3 * D)
    full = O.linear(x, w)
    q = O.rope(O.rmsnorm(full[:, :D].reshape(m, heads, 128), qn[0], 1e-6).reshape(m, D), heads, cos_t, sin_t)
    kk = O.rope(O.rmsnorm(full[:, D:2 * D].reshape(m, heads, 128), qn[1], 1e-6).reshape(m, D), heads, cos_t, sin_t)
    ref = np.concatenate([q, kk, full[:, 2 * D:]], 1)
    assert rel(y.cpu().numpy(), ref) < 1e-5


@pytest.mark.parametrize("hd,heads,q_rows,kv_rows,batch,causal,key_limit",
                         [(128, 2, 200, 77, 2, False, 0), (64, 3, 130, 130, 1, True, 0),
                          (128, 1, 64, 300, 1, False, 150), (128, 16, 1024, 1024, 1, False, 0)])
def test_fp32_attention_matches_oracle(cuda, hd, heads, q_rows, kv_rows, batch, causal, key_limit):
    W = heads * hd
    q = _rand((batch * q_rows, W), 20, 2.0)
    k = _rand((batch * kv_rows, W), 21, 2.0)
    v = _rand((batch * kv_rows, W), 22)
    out = ops.attention(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), heads,
                        batch=batch, causal=causal, key_limit=key_limit, head_dim=hd)
    pairs = ops.attention(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(),
                          heads, batch=batch, causal=causal, key_limit=key_limit, head_dim=hd, out_pairs=True)
    torch.cuda.synchronize()
    ref = np.concatenate([O.attention(q[b * q_rows:(b + 1) * q_rows], k[b * kv_rows:(b + 1) * kv_rows],
                                      v[b * kv_rows:(b + 1) * kv_rows], heads, causal=causal, key_len=key_limit)
                          for b in range(batch)])
    assert rel(out.cpu().numpy(), ref) < 1e-5
    assert rel(ops.from_pairs(pairs).cpu().numpy(), ref) < 1e-5


def test_modulate_and_gemv_pairs(cuda):
    rows, width = 300, 2048
    x = _rand((rows, width), 30, 3.0)
    sh, sc = _rand((width,), 31, 0.5), _rand((width,), 32, 0.5)
    y = ops.modulate(torch.from_numpy(x).cuda(), torch.from_numpy(sh).cuda(), torch.from_numpy(sc).cuda(),
                     out_dtype="pairs")
    w = _rand((768, 512), 33, 0.05)
    xv = _rand((1, 512), 34)
    g = ops.gemv(ops.to_pairs(torch.from_numpy(w).cuda()), torch.from_numpy(xv).cuda(), w_pairs=True)
    torch.cuda.synchronize()
    assert rel(ops.from_pairs(y).cpu().numpy(), O.modulate(x, sh, sc, 1e-6)) < 1e-5
    assert rel(g.cpu().numpy(), O.linear(xv, w)) < 1e-5


@pytest.fixture(scope="module")
def device(cuda):
    d = Device(0)
    yield d
    d.close()


def _anima_case(cfg, seed):
    w = dict(synthetic_weights(cfg, seed=seed))
    rng = np.random.default_rng(seed)
    lat = rng.standard_normal((cfg.batch, 16, cfg.latent_height, cfg.latent_width)).astype(np.float32)
    ctx = rng.standard_normal((cfg.batch, cfg.context_rows, cfg.context_width)).astype(np.float32)
    return w, lat, ctx


def test_anima_fp32_step_within_1e4(device):
    cfg = AnimaConfig(width=256, heads=2, blocks=2, mlp_width=1024, adaln_rank=64, context_rows=96,
                      context_width=128, latent_height=32, latent_width=32, batch=2, compute=F32)
    w, lat, ctx = _anima_case(cfg, 3)
    with build_denoiser(device, cfg, w) as d:
        y = d.predict(lat, 0.0, 0.6, {"context": ctx})
    ref = O.anima_forward(w, cfg, lat, ctx, 0.6)
    assert rel(y, ref) < 1e-4, rel(y, ref)


def test_anima_fp32_cfg1_block_within_1e4(device):
    """benchmark configuration 1 in full: one Anima block, fp32, D 2048, 16 x 128
    heads, 1024 image tokens with 3-D RoPE, cross-attention to 256 x 1024,
    GELU MLP 8192, low-rank adaLN rank 256 (plus the embedder and final layer
    the denoiser step always runs)."""
    cfg = AnimaConfig(width=2048, heads=16, blocks=1, mlp_width=8192, adaln_rank=256, context_rows=256,
                      context_width=1024, latent_height=64, latent_width=64, batch=1, compute=F32)
    w, lat, ctx = _anima_case(cfg, 0)
    with build_denoiser(device, cfg, w) as d:
        y = d.predict(lat, 0.0, 0.5, {"context": ctx})
    ref = O.anima_forward(w, cfg, lat, ctx, 0.5)
    assert rel(y, ref) < 1e-4, rel(y, ref)


@pytest.mark.parametrize("key_len", [0, 5500])
def test_mmdit_fp32_step_within_1e4(device, key_len):
    """The dual-stream MMDiT step in fp32 compute (joint attention with 2-D
    RoPE, GELU-tanh MLP), with and without the key-count mask."""
    from naivediffusion_b200.denoiser import MMDiTConfig
    cfg = MMDiTConfig(width=256, heads=2, blocks=2, mlp_width=512, context_rows=64, context_width=64,
                      latent_height=16, latent_width=32, compute=F32)
    w = dict(synthetic_weights(cfg, seed=4))
    rng = np.random.default_rng(4)
    lat = rng.standard_normal((1, cfg.latent_channels, cfg.latent_height, cfg.latent_width)).astype(np.float32)
    ctx = rng.standard_normal((1, cfg.context_rows, cfg.context_width)).astype(np.float32)
    M = (cfg.latent_height // 2) * (cfg.latent_width // 2) + cfg.context_rows
    kl = min(key_len, M - 7) if key_len else 0
    cond = {"context": ctx}
    if kl:
        cond["key_length"] = np.array([kl], np.int32)
    with build_denoiser(device, cfg, w) as d:
        y = d.predict(lat, 500.0, 0.5, cond)
    ref = O.mmdit_forward(w, cfg, lat, ctx[0], 0.5, key_len=kl)
    assert rel(y, ref) < 1e-4, rel(y, ref)
