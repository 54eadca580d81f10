"""The SwiGLU GEMM epilogue (ND_EPI_SWIGLU: y = silu(x Wg^T) * (x Wu^T) from
the fused [gate; up] matrix, QwenImageDit.FeedForward) and single-stream row
groups (shared_weights: one matrix, per-row gate vectors split at any row),
against a torch fp32 reference of the same op (bf16 / fp16: max|d|/max|ref|
<= 2e-2 and cosine >= 0.999), the fp32 oracle for pair operands (<= 1e-5),
and the int8 kernel against the same GEMM on the dequantized weights
(bit-identical: the widening is exact and the accumulation order the same).
"""
import numpy as np
import pytest
import torch

import oracle as O
from naivediffusion_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).abs().max() / b.abs().max()).item()


def _cos(a, b):
    return torch.nn.functional.cosine_similarity(a.double().flatten(), b.double().flatten(), dim=0).item()


def _swiglu_ref(x, w, b=None):
    f = w.shape[0] // 2
    h = x.float() @ w.float().t()
    if b is not None:
        h = h + b
    return torch.nn.functional.silu(h[:, :f]) * h[:, f:]


@pytest.mark.parametrize("m,f,k", [(4352, 12288 // 8, 1024), (300, 384, 256), (128, 128, 64), (77, 640, 512)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_swiglu_matches_torch(cuda, m, f, k, dtype):
    g = torch.Generator().manual_seed(m + f)
    x = torch.randn(m, k, generator=g).to(dtype).cuda()
    w = (torch.randn(2 * f, k, generator=g) * 0.05).to(dtype).cuda()
    b = (torch.randn(2 * f, generator=g) * 0.1).cuda()
    y = ops.linear(x, w, None, epilogue=_lib.ND_EPI_SWIGLU)
    yb = ops.linear(x, w, b, epilogue=_lib.ND_EPI_SWIGLU)
    ops.sync()
    assert y.shape == (m, f)
    ref, refb = _swiglu_ref(x, w), _swiglu_ref(x, w, b)
    assert _rel(y, ref) < 2e-2 and _cos(y, ref) > 0.999
    assert _rel(yb, refb) < 2e-2 and _cos(yb, refb) > 0.999


def test_swiglu_rejects_ragged_width(cuda):
    x = torch.zeros(128, 64, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(2 * 96, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(Exception, match="SWIGLU"):
        ops.linear(x, w, None, epilogue=_lib.ND_EPI_SWIGLU)


def test_swiglu_pairs_matches_fp32_oracle(cuda):
    m, f, k = 300, 256, 512
    rng = np.random.default_rng(3)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (rng.standard_normal((2 * f, k)) * 0.05).astype(np.float32)
    y = ops.linear(ops.to_pairs(torch.from_numpy(x).cuda()), ops.to_pairs(torch.from_numpy(w).cuda()), None,
                   epilogue=_lib.ND_EPI_SWIGLU, pairs=True)
    torch.cuda.synchronize()
    h = O.linear(x, w, None)
    ref = O.silu(np.ascontiguousarray(h[:, :f])) * h[:, f:]
    assert y.shape == (m, 2 * f)
    got = ops.from_pairs(y).cpu().numpy()
    assert float(np.abs(got - ref).max() / np.abs(ref).max()) < 1e-5


def test_swiglu_int8_matches_dequantized(cuda):
    m, f, k = 640, 384, 1024
    g = torch.Generator().manual_seed(5)
    w = (torch.randn(2 * f, k, generator=g) * 0.05).bfloat16()
    q, s = O.quantize(w.float().numpy(), 32, True)
    qd = torch.from_numpy(q).cuda()
    sd = torch.from_numpy(s.view(np.float16)).cuda()
    wd = ops.dequantize(qd, sd, 32)
    x = torch.randn(m, k, generator=g).bfloat16().cuda()
    y8 = ops.linear(x, qd, None, scales=sd, quant_group=32, epilogue=_lib.ND_EPI_SWIGLU)
    y16 = ops.linear(x, wd, None, epilogue=_lib.ND_EPI_SWIGLU)
    ops.sync()
    assert torch.equal(y8, y16)


@pytest.mark.parametrize("m,split", [(4096 + 200, 4096), (300, 77), (5000, 4913)])
def test_shared_weights_row_groups(cuda, m, split):
    """One weight matrix, the gate vector switching at an arbitrary row (the
    single-stream block's image rows vs text rows)."""
    n, k = 512, 384
    g = torch.Generator().manual_seed(split)
    x = torch.randn(m, k, generator=g).bfloat16().cuda()
    w = (torch.randn(n, k, generator=g) * 0.05).bfloat16().cuda()
    gate = torch.randn(2, n, generator=g).cuda()
    r0 = torch.randn(m, n, generator=g).cuda()
    r = r0.clone()
    ops.linear(x, w, None, epilogue=_lib.ND_EPI_RESIDUAL_GATE, residual=r, gate=gate, group_split=split,
               shared_weights=True)
    ops.sync()
    gr = torch.where(torch.arange(m, device="cuda")[:, None] < split, gate[0], gate[1])
    ref = r0 + gr * (x.float() @ w.float().t())
    assert _rel(r, ref) < 2e-2 and _cos(r - r0, ref - r0) > 0.999


def test_shared_weights_qk_norm_uses_one_set(cuda):
    """QK_NORM_ROPE with shared weights: every row uses the first norm set,
    the same result as one group."""
    m, width = 400, 256
    g = torch.Generator().manual_seed(2)
    x = torch.randn(m, width, generator=g).bfloat16().cuda()
    w = (torch.randn(3 * width, width, generator=g) * 0.05).bfloat16().cuda()
    norm = (1 + 0.1 * torch.randn(2, 128, generator=g)).cuda()
    ang = torch.rand(m, 64, generator=g) * 6.28
    kw = dict(epilogue=_lib.ND_EPI_QK_NORM_ROPE, qk_norm=norm, rope_cos=ang.cos().cuda(), rope_sin=ang.sin().cuda(),
              qk_cols=2 * width)
    a = ops.linear(x, w, None, **kw)
    b = ops.linear(x, w, None, group_split=137, shared_weights=True, **kw)
    ops.sync()
    assert torch.equal(a, b)


@pytest.mark.parametrize("m,f,k", [(8192, 2560, 640), (300, 384, 256)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_geglu_epilogue_matches_torch(cuda, m, f, k, dtype):
    """ND_EPI_GEGLU: h * gelu(g) (exact GELU) from the fused [h; g] projection,
    SDXL's feed-forward (UNetLayers.Geglu)."""
    g = torch.Generator().manual_seed(m + f)
    x = torch.randn(m, k, generator=g).to(dtype).cuda()
    w = (torch.randn(2 * f, k, generator=g) * 0.05).to(dtype).cuda()
    b = (torch.randn(2 * f, generator=g) * 0.1).cuda()
    y = ops.linear(x, w, b, epilogue=_lib.ND_EPI_GEGLU)
    ops.sync()
    h = x.float() @ w.float().t() + b
    ref = h[:, :f] * torch.nn.functional.gelu(h[:, f:])
    assert y.shape == (m, f)
    assert _rel(y, ref) < 2e-2 and _cos(y, ref) > 0.999
