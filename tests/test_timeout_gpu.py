"""The device-timeout path (the library's stand-in for the reference's
DeviceRemovedException, src/NaiveDiffusion/Dml/DeviceExceptions.cs:13-21):
a kernel whose bounded mbarrier wait runs out records a status, returns, and
the host reads ND_ERR_TIMEOUT from nd_op_sync; the CUDA context stays usable.

The wait that runs out is on a barrier nothing arrives on, with a 1 ms limit;
no GPU fault, trap or hang is involved.
"""
import time

import numpy as np
import pytest
import torch

import oracle as O
from naivediffusion_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def test_unarmed_wait_runs_out_and_reports_timeout(cuda):
    ops.sync()  # start from a clean status word
    t0 = time.perf_counter()
    ops.wait_probe(1_000_000, ctas=8)  # 1 ms limit, nothing ever arrives
    with pytest.raises(_lib.NdError) as e:
        ops.sync()
    elapsed = time.perf_counter() - t0
    assert e.value.code == _lib.ND_ERR_TIMEOUT
    assert "0x600" in str(e.value)
    assert elapsed < 5.0, elapsed  # the kernel gave up and returned
    ops.sync()  # the report cleared the status word


def test_armed_wait_completes(cuda):
    ops.wait_probe(1_000_000, ctas=8, armed=True)
    ops.sync()


def test_context_usable_after_timeout(cuda):
    """After a timed-out kernel, the next op on the same context runs and is
    right (the reference's device needs recreating after DeviceRemoved; here
    nothing does)."""
    ops.wait_probe(1_000_000, ctas=2)
    with pytest.raises(_lib.NdError):
        ops.sync()
    rng = np.random.default_rng(3)
    q, k, v = (torch.from_numpy(rng.standard_normal((256, 256)).astype(np.float32)).cuda().bfloat16()
               for _ in range(3))
    y = ops.attention(q, k, v, 2)
    ops.sync()
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    ref = O.attention(f(q), f(k), f(v), 2)
    out = f(y)
    assert np.abs(out - ref).max() / np.abs(ref).max() < 2e-2


def test_probe_rejects_bad_arguments(cuda):
    for args in ((0, 1), (1_000_000, 0), (20_000_000_000, 1), (1_000_000, 5000)):
        with pytest.raises(_lib.NdError) as e:
            ops.wait_probe(*args)
        assert e.value.code == _lib.ND_ERR_INVALID
