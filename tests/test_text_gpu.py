"""The text towers on the device (nd_text_encode): Qwen3TextModel.Forward and
Anima's LlmAdapter.Forward against the oracle's fp32 compositions
(oracle.qwen3_text_forward / llm_adapter_forward). bf16 compute:
max|d| / max|ref| <= 2e-2 and cosine >= 0.999; fp32 compute <= 1e-4."""
import numpy as np
import pytest
import torch

import oracle as O
from naivediffusion_b200 import _lib, ops
from naivediffusion_b200.denoiser import (Device, LlmAdapterConfig, Qwen3TextConfig, build_denoiser,
                                          synthetic_weights)

pytestmark = pytest.mark.gpu


def rel(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / np.abs(b).max())


def cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


@pytest.fixture(scope="module")
def device(cuda):
    d = Device(0)
    yield d
    d.close()


SMALL_Q = dict(width=256, blocks=2, heads=4, kv_heads=2, mlp_width=384, vocab=1000, context_rows=64)


@pytest.mark.parametrize("rows,final_norm", [(37, True), (64, False), (1, True)])
def test_qwen3_matches_oracle(device, rows, final_norm):
    cfg = Qwen3TextConfig(**SMALL_Q)
    w = dict(synthetic_weights(cfg, seed=1))
    ids = np.random.default_rng(rows).integers(0, cfg.vocab, rows)
    with build_denoiser(device, cfg, w) as d:
        y = d.text_encode(ids, final_norm=final_norm)
        y2 = d.text_encode(ids, final_norm=final_norm)
    ref = O.qwen3_text_forward(w, cfg, ids, final_norm)
    assert np.array_equal(y, y2)
    assert rel(y, ref) < 2e-2, rel(y, ref)
    assert cos(y, ref) > 0.999


def test_qwen3_fp32_within_1e4(device):
    cfg = Qwen3TextConfig(**SMALL_Q, compute=_lib.ND_F32)
    w = dict(synthetic_weights(cfg, seed=2))
    ids = np.random.default_rng(2).integers(0, cfg.vocab, 45)
    with build_denoiser(device, cfg, w) as d:
        y = d.text_encode(ids)
    ref = O.qwen3_text_forward(w, cfg, ids)
    assert rel(y, ref) < 1e-4, rel(y, ref)


def test_qwen3_06b_shapes(device):
    """Qwen3-0.6B's widths (1024, 16 x 128 query heads over 8 key heads,
    SwiGLU 3072, its 151936-row table), four of its 28 layers."""
    cfg = Qwen3TextConfig(blocks=4, context_rows=256)
    w = dict(synthetic_weights(cfg, seed=3))
    ids = np.random.default_rng(3).integers(0, cfg.vocab, 200)
    with build_denoiser(device, cfg, w) as d:
        y = d.text_encode(ids)
    ref = O.qwen3_text_forward(w, cfg, ids)
    assert rel(y, ref) < 2e-2, rel(y, ref)
    assert cos(y, ref) > 0.999


def test_qwen3_errors(device):
    cfg = Qwen3TextConfig(**SMALL_Q)
    w = dict(synthetic_weights(cfg, seed=1))
    with build_denoiser(device, cfg, w) as d:
        with pytest.raises(Exception, match="vocabulary"):
            d.text_encode(np.array([1, cfg.vocab], np.int32))
        with pytest.raises(Exception, match="rows"):
            d.text_encode(np.zeros(cfg.context_rows + 1, np.int32))
        with pytest.raises(Exception, match="nd_text_encode"):
            d.predict(np.zeros((1, 1, 1, 1), np.float32), 0.0, 0.0, {})


SMALL_A = dict(width=256, blocks=2, heads=4, head_dim=64, mlp_width=512, vocab=500, context_rows=64, source_rows=96)


@pytest.mark.parametrize("rows,src", [(37, 30), (64, 96), (5, 1)])
def test_llm_adapter_matches_oracle(device, rows, src):
    cfg = LlmAdapterConfig(**SMALL_A)
    w = dict(synthetic_weights(cfg, seed=4))
    rng = np.random.default_rng(rows + src)
    ids = rng.integers(0, cfg.vocab, rows)
    ctx = rng.standard_normal((src, cfg.width)).astype(np.float32)
    with build_denoiser(device, cfg, w) as d:
        y = d.text_encode(ids, source=ctx)
    ref = O.llm_adapter_forward(w, cfg, ids, ctx)
    assert rel(y, ref) < 2e-2, rel(y, ref)
    assert cos(y, ref) > 0.999


def test_llm_adapter_anima_shapes(device):
    """The adapter's real shape: 6 blocks 1024 wide, 16 x 64 heads, MLP 4096,
    T5's 32128-row table, reading 300 Qwen3 rows."""
    cfg = LlmAdapterConfig()
    w = dict(synthetic_weights(cfg, seed=5))
    rng = np.random.default_rng(5)
    ids = rng.integers(0, cfg.vocab, 120)
    ctx = rng.standard_normal((300, cfg.width)).astype(np.float32)
    with build_denoiser(device, cfg, w) as d:
        y = d.text_encode(ids, source=ctx)
        with pytest.raises(Exception, match="source"):
            d.text_encode(ids)
    ref = O.llm_adapter_forward(w, cfg, ids, ctx)
    assert rel(y, ref) < 2e-2, rel(y, ref)
    assert cos(y, ref) > 0.999


@pytest.mark.parametrize("hd,dtype", [(64, torch.bfloat16), (128, torch.float32), (64, torch.float16)])
def test_head_norm_rope_op(cuda, hd, dtype):
    rows, heads = 77, 3
    rng = np.random.default_rng(hd)
    x = rng.standard_normal((rows, heads * hd + 32)).astype(np.float32)
    wt = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    c, s = O.rope_tables_1d(rows, hd, 1e4)
    t = torch.from_numpy(x).to(dtype).cuda()
    xin = t.float().cpu().numpy()
    ops.head_norm_rope(t, heads, hd, torch.from_numpy(wt).cuda(), torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda())
    torch.cuda.synchronize()
    ref = O.rope(O.rmsnorm(np.ascontiguousarray(xin[:, :heads * hd]).reshape(-1, hd), wt, 1e-6).reshape(rows, -1),
                 heads, c, s)
    got = t.float().cpu().numpy()
    assert rel(got[:, :heads * hd], ref) < (1e-5 if dtype == torch.float32 else 1e-2)
    assert np.array_equal(got[:, heads * hd:], xin[:, heads * hd:])  # columns past the heads untouched


def test_weights_mean_the_same_at_every_float_width(device):
    """CpuMathTests' point on the device (tests/NaiveDiffusion.Tests/CpuMathTests.cs:
    a matrix has to mean the same numbers at every width a checkpoint stores it
    at): the same tower uploaded from fp32 and fp16 host arrays and from bf16
    device tensors -- every value exact at all three widths -- encodes a prompt
    bit-identically (the embedding row gather and every GEMM read the same numbers)."""
    cfg = Qwen3TextConfig(**SMALL_Q)
    w = {}
    for name, a in synthetic_weights(cfg, seed=5):
        v = O.round_bf16(a)
        v[np.abs(v) < 2.0 ** -14] = 0.0   # below fp16's normal range: keep every value exact in fp16
        assert np.array_equal(v.astype(np.float16).astype(np.float32), v)
        w[name] = v
    ids = np.random.default_rng(5).integers(0, cfg.vocab, 29)
    uploads = [w, {k: v.astype(np.float16) for k, v in w.items()},
               {k: torch.from_numpy(v).cuda().bfloat16() for k, v in w.items()}]
    outs = []
    for weights in uploads:
        with build_denoiser(device, cfg, weights) as d:
            outs.append(d.text_encode(ids))
    assert np.isfinite(outs[0]).all()
    assert np.array_equal(outs[0], outs[1])
    assert np.array_equal(outs[0], outs[2])
