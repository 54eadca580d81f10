"""nd_op_group_norm_noalloc (fixed in-library scratch, no allocation) against
nd_op_group_norm (growable scratch), both called through the C ABI.

The file name sorts last so that, in a full run, the no-allocation entry point
is exercised after every other test has used the library (and its growable
scratch) on the same device; it also passes on its own.
"""
import ctypes as C

import pytest
import torch

from naivediffusion_b200 import _lib

pytestmark = pytest.mark.gpu

_ARGS = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
         C.c_float, C.c_int, C.c_void_p]


def _fn(name):
    f = getattr(_lib.lib(), name)
    f.argtypes = _ARGS
    f.restype = C.c_int
    return f


def _call(name, x, y, groups, w, b, eps, silu):
    bsz, pixels, ch = x.shape
    dt = _lib.ND_F16 if x.dtype == torch.float16 else _lib.ND_BF16
    return _fn(name)(x.data_ptr(), y.data_ptr(), dt, bsz, pixels, ch, groups, w.data_ptr(),
                     None if b is None else b.data_ptr(), eps, int(silu),
                     C.c_void_p(torch.cuda.current_stream().cuda_stream))


def _case(bsz, pixels, ch, seed, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(bsz, pixels, ch, generator=g) * 2 + 0.5).to(dtype).cuda()
    w = (1 + 0.1 * torch.randn(ch, generator=g)).cuda()
    b = (0.1 * torch.randn(ch, generator=g)).cuda()
    return x, w, b


def test_noalloc_matches_allocating_entry_point_twice_in_a_row(cuda):
    # Two different shapes back to back: the second call reuses the array the
    # first one filled, so stale partial sums would show up as a mismatch.
    cases = [(_case(2, 4096, 640, 1), 32, 1e-5, True),
             (_case(1, 16384, 320, 2, torch.bfloat16), 32, 1e-6, False)]
    outs = []
    for (x, w, b), groups, eps, silu in cases:
        y = torch.empty_like(x)
        assert _call("nd_op_group_norm_noalloc", x, y, groups, w, b, eps, silu) == _lib.ND_OK
        outs.append(y)
    for ((x, w, b), groups, eps, silu), y in zip(cases, outs):
        ref = torch.empty_like(x)
        assert _call("nd_op_group_norm", x, ref, groups, w, b, eps, silu) == _lib.ND_OK
        torch.cuda.synchronize()
        assert torch.equal(y, ref)


def test_noalloc_leaves_free_memory_unchanged(cuda):
    x, w, b = _case(2, 16384, 960, 3)  # the SDXL UNet's largest GroupNorm at 1024 x 1024
    y = torch.empty_like(x)
    assert _call("nd_op_group_norm_noalloc", x, y, 32, w, b, 1e-5, True) == _lib.ND_OK  # per-device set-up
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(2):
        assert _call("nd_op_group_norm_noalloc", x, y, 32, w, b, 1e-5, True) == _lib.ND_OK
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    ref = torch.empty_like(x)
    assert _call("nd_op_group_norm", x, ref, 32, w, b, 1e-5, True) == _lib.ND_OK
    torch.cuda.synchronize()
    assert torch.equal(y, ref)


def test_noalloc_rejects_shapes_beyond_its_fixed_scratch(cuda):
    # 4 x 8192 x 32 x 8 bytes = 8 MiB of partial sums alone: over the limit.
    x = torch.zeros(4, 262144, 64, dtype=torch.float16, device="cuda")
    w = torch.ones(64, device="cuda")
    y = torch.empty_like(x)
    rc = _call("nd_op_group_norm_noalloc", x, y, 32, w, None, 1e-5, False)
    assert rc == _lib.ND_ERR_INVALID
    assert b"fixed" in _lib.lib().nd_last_error()
