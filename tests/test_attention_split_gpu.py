"""The attention kernel's split of the last partial wave along the keys
(nd_attention_args.workspace): the (query-tile pair x head x batch) units past
the last whole wave of SMs run as several CTAs over consecutive key ranges,
and the last of them to finish merges the pieces' (max, sum, O) in piece
order. Against the CPU oracle (CpuMath.Attention, Tensors/CpuMath.cs:203-248,
plus the key-count mask), against the unsplit kernel, and for the properties
the merge must keep: bit-identical output from run to run and a workspace
whose counters are back at zero.

Tolerance (the 16-bit bar): max|d| / max|ref| <= 2e-2 and cosine >= 0.999;
split against unsplit 1e-2 (both round P to 16 bits, in different key
groupings).
"""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

COUNTER_BYTES = 16384


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / np.abs(b).max())


def _cos(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


def _qkv(rows, kv_rows, heads, kv_heads, hd, dtype, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = (torch.randn(rows, heads * hd, generator=g) * 1.5).to(dtype).cuda()
    k = (torch.randn(kv_rows, kv_heads * hd, generator=g) * 1.5).to(dtype).cuda()
    v = torch.randn(kv_rows, kv_heads * hd, generator=g).to(dtype).cuda()
    return q, k, v


def _oracle(q, k, v, heads, kv_heads, batch, key_limit, causal=False):
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    qn, kn, vn = f(q), f(k), f(v)
    qr, kr = qn.shape[0] // batch, kn.shape[0] // batch
    return np.concatenate([O.attention(qn[b * qr:(b + 1) * qr], kn[b * kr:(b + 1) * kr], vn[b * kr:(b + 1) * kr],
                                       heads, kv_heads=kv_heads, causal=causal, key_len=key_limit)
                           for b in range(batch)])


# rows, kv_rows, heads, kv_heads, head_dim, batch, key_limit, dtype
CASES = [
    (1024, 1024, 8, 8, 128, 1, 0, torch.bfloat16),       # 32 units < one wave: all split
    (1100, 1024, 6, 6, 128, 1, 1000, torch.float16),     # ragged query tile, key count inside a tile
    (4096, 4096, 10, 10, 64, 2, 0, torch.float16),       # SDXL level 1: 320 units, a 24-unit tail
    (1024, 1024, 20, 20, 64, 2, 0, torch.float16),       # SDXL level 2: 160 units, a 12-unit tail
    (2048, 1536, 4, 2, 128, 2, 1500, torch.bfloat16),    # grouped-query heads, batch 2, key count
]


@pytest.mark.parametrize("rows,kv_rows,heads,kv_heads,hd,batch,key_limit,dtype", CASES)
def test_split_against_oracle(cuda, rows, kv_rows, heads, kv_heads, hd, batch, key_limit, dtype):
    from naivediffusion_b200 import ops
    q, k, v = _qkv(batch * rows, batch * kv_rows, heads, kv_heads, hd, dtype, seed=rows + heads + hd)
    ws = ops.attention_workspace(hd)
    kw = dict(batch=batch, key_limit=key_limit, head_dim=hd, kv_heads=kv_heads)
    y1 = ops.attention(q, k, v, heads, workspace=ws, **kw)
    y2 = ops.attention(q, k, v, heads, workspace=ws, **kw)
    y0 = ops.attention(q, k, v, heads, **kw)
    ops.sync()
    # the split ran: pieces left their (max, sum) rows in the workspace ...
    assert ws[COUNTER_BYTES:].any(), "no unit was split"
    # ... and the merging pieces put every counter back to zero
    assert not ws[:COUNTER_BYTES].any(), "counters not reset"
    assert torch.equal(y1, y2), "split attention differs between runs"
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    ref = _oracle(q, k, v, heads, kv_heads, batch, key_limit)
    r, c = _rel(f(y1), ref), _cos(f(y1), ref)
    print(f"split vs oracle: max rel {r:.3e}, cosine {c:.7f}")
    assert r <= 2e-2 and c >= 0.999
    assert _rel(f(y1), f(y0)) <= 1e-2


def test_no_split_when_waves_are_whole_or_causal(cuda):
    """148 units (one whole wave) and a causal launch never split: the
    workspace stays all zero and the output equals the unsplit kernel's."""
    from naivediffusion_b200 import ops
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    ws = ops.attention_workspace(128)
    q, k, v = _qkv(256 * sms, 2048, 1, 1, 128, torch.bfloat16, seed=11)
    y1 = ops.attention(q, k, v, 1, workspace=ws)
    y0 = ops.attention(q, k, v, 1)
    ops.sync()
    assert not ws.any() and torch.equal(y1, y0)
    q, k, v = _qkv(1024, 1024, 4, 4, 128, torch.bfloat16, seed=12)
    y1 = ops.attention(q, k, v, 4, causal=True, workspace=ws)
    y0 = ops.attention(q, k, v, 4, causal=True)
    ops.sync()
    assert not ws.any() and torch.equal(y1, y0)


def test_split_in_a_graph(cuda):
    """Captured once, replayed: every replay merges in the same order (the
    counters reset themselves between launches), so replays are identical."""
    from naivediffusion_b200 import ops
    q, k, v = _qkv(2048, 2048, 6, 6, 128, torch.bfloat16, seed=13)
    ws = ops.attention_workspace(128)
    out = torch.empty_like(q)
    ops.attention(q, k, v, 6, out=out, workspace=ws)  # warm-up (configures the kernel)
    ops.sync()
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
        ops.attention(q, k, v, 6, out=out, workspace=ws)
    outs = []
    for _ in range(3):
        g.replay()
        torch.cuda.synchronize()
        outs.append(out.clone())
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    assert not ws[:COUNTER_BYTES].any()
    ref = _oracle(q, k, v, 6, 6, 1, 0)
    assert _rel(outs[0].float().cpu().numpy(), ref) <= 2e-2


def test_workspace_bytes(cuda):
    from naivediffusion_b200 import _lib
    L = _lib.lib()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert L.nd_attention_workspace_bytes(128) == COUNTER_BYTES + 2 * sms * 256 * (8 + 4 * 128)
    assert L.nd_attention_workspace_bytes(64) == COUNTER_BYTES + 2 * sms * 256 * (8 + 4 * 64)
    assert L.nd_attention_workspace_bytes(96) == 0
