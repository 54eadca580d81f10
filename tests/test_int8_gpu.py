"""int8 weight-only path (BlockQuantizer scheme, fused dequant GEMM).

- The widened weights are bit-exact with the oracle's dequantization
  (bf16 / fp16 of the exact fp32 product q * scale).
- The int8 GEMM feeds the tensor cores the same bf16 tiles the bf16 GEMM
  would read from a dequantized copy, so its output is bit-identical to the
  bf16 GEMM over nd_op_dequantize's weights.
- Against the fp32 product of the unquantized weights the error stays under
  QuantProbe's bar: max|d| / max|y| < 2e-2 (NaiveDiffusion.Cli/QuantProbe.cs:52-57).
"""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


def _quant(n, k, group, f16, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    q, s = O.quantize(w, group=group if group else k, scale_f16=f16)
    return w, q, s


def _dev_scales(s):
    if s.dtype == np.uint16:
        return torch.from_numpy(s.view(np.float16)).cuda()
    return torch.from_numpy(s).cuda()


@pytest.mark.parametrize("group,f16,out", [(32, True, torch.bfloat16), (0, False, torch.bfloat16),
                                           (32, True, torch.float16)])
def test_dequantize_bit_exact(cuda, group, f16, out):
    from naivediffusion_b200 import ops
    w, q, s = _quant(300, 512, group, f16, seed=1)
    deq = ops.dequantize(torch.from_numpy(q).cuda(), _dev_scales(s), quant_group=group, out_dtype=out)
    ops.sync()
    ref = O.dequantize(q, s, group=group if group else 512)      # exact fp32 products
    ref_t = torch.from_numpy(ref).to(out)                          # RNE to the storage type
    assert torch.equal(deq.cpu().view(torch.int16), ref_t.view(torch.int16))


@pytest.mark.parametrize("m,n,k,group,f16", [(640, 768, 1024, 32, True), (5632, 3072, 3072, 0, False),
                                             (300, 512, 256, 32, True), (128, 1280, 640, 32, True)])
def test_int8_gemm_matches_dequantized_bf16_gemm(cuda, m, n, k, group, f16):
    from naivediffusion_b200 import ops
    w, q, s = _quant(n, k, group, f16, seed=m + n)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(2)).bfloat16().cuda()
    b = (torch.randn(n, generator=torch.Generator().manual_seed(3)) * 0.1).cuda()
    qd, sd = torch.from_numpy(q).cuda(), _dev_scales(s)
    y8 = ops.linear(x, qd, b, scales=sd, quant_group=group)
    wd = ops.dequantize(qd, sd, quant_group=group)
    y16 = ops.linear(x, wd, b)
    ops.sync()
    assert torch.equal(y8, y16)
    ref = x.float() @ torch.from_numpy(w).cuda().t() + b
    err = ((y8.float() - ref).abs().max() / ref.abs().max()).item()
    assert err < 2e-2, err


def test_int8_gemm_epilogues_and_row_groups(cuda):
    from naivediffusion_b200 import ops, _lib
    m, width, split = 384, 512, 256
    n, k = 3 * width, 256
    w, q, s = _quant(2 * n, k, 32, True, seed=9)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(4)).bfloat16().cuda()
    qd, sd = torch.from_numpy(q).cuda(), _dev_scales(s)
    wd = ops.dequantize(qd, sd, 32)
    norm = (1 + 0.1 * torch.randn(2, 2, 128)).cuda()
    ang = torch.rand(m, 64) * 6.28
    cs, sn = ang.cos().cuda(), ang.sin().cuda()
    kw = dict(epilogue=_lib.ND_EPI_QK_NORM_ROPE, group_split=split, qk_norm=norm, rope_cos=cs,
              rope_sin=sn, qk_cols=2 * width)
    y8 = ops.linear(x, qd, None, scales=sd, quant_group=32, **kw)
    y16 = ops.linear(x, wd, None, **kw)
    r0 = torch.randn(m, n, device="cuda")
    gate = torch.randn(2, n, device="cuda")
    r8, r16 = r0.clone(), r0.clone()
    ops.linear(x, qd, None, scales=sd, quant_group=32, epilogue=_lib.ND_EPI_RESIDUAL_GATE, residual=r8,
               gate=gate, group_split=split)
    ops.linear(x, wd, None, epilogue=_lib.ND_EPI_RESIDUAL_GATE, residual=r16, gate=gate, group_split=split)
    ops.sync()
    assert torch.equal(y8, y16)
    assert torch.equal(r8, r16)


def _quantized_model_weights(cfg, seed):
    """Synthetic bf16 weights, the oracle's BlockQuantizer on each int8
    matrix, and the dequantized bf16 values the GPU's tiles hold."""
    from naivediffusion_b200.denoiser import synthetic_weights
    w = dict(synthetic_weights(cfg, seed=seed))
    q8, deq = {}, {}
    for name, a in w.items():
        if a.ndim == 2 and cfg.quantized(*a.shape):
            g = cfg.quant_group or a.shape[1]
            q, s = O.quantize(a, group=g, scale_f16=cfg.quant_scale_dtype == 1)
            q8[name] = (q, s)
            deq[name] = O.round_bf16(O.dequantize(q, s, group=g))
        else:
            deq[name] = a
    return w, q8, deq


@pytest.mark.parametrize("group,scale_dtype,host_quant", [(32, 1, False), (0, 0, False), (32, 1, True)])
def test_int8_mmdit_step(cuda, group, scale_dtype, host_quant):
    """The whole dual-stream step with int8 weights (device- or host-quantized)
    against the oracle run on the dequantized weights."""
    from naivediffusion_b200 import _lib
    from naivediffusion_b200.denoiser import Device, CudaDenoiser, MMDiTConfig
    cfg = MMDiTConfig(width=256, heads=2, blocks=2, mlp_width=512, context_rows=64, context_width=64,
                      latent_height=16, latent_width=32, weight_dtype=_lib.ND_I8, quant_group=group,
                      quant_scale_dtype=scale_dtype)
    w, q8, deq = _quantized_model_weights(cfg, seed=5)
    assert len(q8) >= 2 * 2 * 6
    rng = np.random.default_rng(5)
    lat = rng.standard_normal((1, 16, 16, 32)).astype(np.float32)
    ctx = rng.standard_normal((1, 64, 64)).astype(np.float32)
    with Device(0) as dev:
        d = CudaDenoiser(dev, cfg.desc())
        try:
            for name, a in w.items():
                if host_quant and name in q8:
                    q, s = q8[name]
                    d.set_weight_q8(name, q, s.view(np.float16) if s.dtype == np.uint16 else s, group)
                else:
                    d.set_weight(name, a)
            d.finalize()
            y = d.predict(lat, 0.0, 0.4, {"context": ctx})
            m = d.memory()
        finally:
            d.close()
    ref = O.mmdit_forward(deq, cfg, lat, ctx[0], 0.4)
    rel = float(np.abs(y - ref).max() / np.abs(ref).max())
    cos = float((y * ref).sum() / np.linalg.norm(y) / np.linalg.norm(ref))
    assert rel < 2e-2 and cos > 0.999, (rel, cos)
    # int8 storage: roughly half the bf16 model's bytes
    full = sum(a.size * (1 if n in q8 else (2 if a.ndim == 2 else 4)) for n, a in w.items())
    assert m.persistent_bytes < 0.75 * sum(a.size * (2 if a.ndim == 2 else 4) for a in w.values()) or full == 0


@pytest.mark.parametrize("group,f16", [(32, True), (0, False), (64, True)])
def test_device_quantizer_matches_block_quantizer_bit_for_bit(cuda, group, f16):
    from naivediffusion_b200 import ops
    rng = np.random.default_rng(group)
    w = (rng.standard_normal((257, 512)) * 0.02).astype(np.float32)
    w[3, :32] = 0.0                       # a zero block: zero scale, zero values
    w[5, 7] = 1e-9                        # a block whose fp16 scale underflows
    w[5, 8:32] = 0.0
    w[9, 40] = 127.0 * 0.5                # exact halves: round half to even
    wb = O.round_bf16(w)
    q, s = ops.quantize(torch.from_numpy(wb).cuda().bfloat16(), group,
                        torch.float16 if f16 else torch.float32)
    ops.sync()
    qo, so = O.quantize(wb, group=group or 512, scale_f16=f16)
    assert np.array_equal(q.cpu().numpy(), qo)
    sg = s.cpu().numpy()
    assert np.array_equal(sg.view(np.uint16) if f16 else sg, so.reshape(sg.shape))
