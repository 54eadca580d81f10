"""CPU checks of the C ABI boundary: the library loads without a GPU, exports
every entry point include/nd_denoise.h declares, reports errors through
nd_last_error, and the ctypes mirrors match the header's struct layouts."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

from naivediffusion_b200 import _lib
from naivediffusion_b200 import denoiser as D

HEADER = Path(__file__).resolve().parent.parent / "include" / "nd_denoise.h"


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"ND_API\s+[\w\s\*]+?\b(nd_\w+)\s*\(", text)))


def test_every_declared_symbol_is_exported():
    names = declared()
    assert len(names) >= 20
    L = _lib.lib()
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_version_and_error_channel_without_gpu():
    L = _lib.lib()
    assert b"sm_100a" in L.nd_version()
    rc = L.nd_op_linear(None, None)
    assert rc == _lib.ND_ERR_INVALID
    assert b"null args" in L.nd_last_error()


def test_struct_layouts_match_the_header(tmp_path):
    """ctypes mirrors vs the C compiler's view of include/nd_denoise.h."""
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if not cc:
        pytest.skip("no C compiler")
    structs = {"nd_linear_args": _lib.LinearArgs, "nd_conv_args": _lib.ConvArgs,
               "nd_sampler_args": _lib.SamplerArgs,
               "nd_attention_args": _lib.AttentionArgs,
               "nd_modulate_args": _lib.ModulateArgs, "nd_rmsnorm_args": _lib.RmsNormArgs,
               "nd_gemv_args": _lib.GemvArgs, "nd_model_desc": D.ModelDesc,
               "nd_named_tensor": D.NamedTensor, "nd_memory": D.Memory, "nd_kernel_time": D.KernelTime}
    src = tmp_path / "sizes.c"
    lines = []
    for n, cls in structs.items():
        lines.append(f'printf("%zu\\n", sizeof({n}));\n')
        lines += [f'printf("%zu\\n", offsetof({n}, {f[0]}));\n' for f in cls._fields_]
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "nd_denoise.h"\nint main(void){\n' +
                   "".join(lines) + "return 0;}\n")
    exe = tmp_path / "sizes"
    subprocess.run([cc, "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    sizes = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    it = iter(sizes)
    for name, cls in structs.items():
        assert C.sizeof(cls) == next(it), name
        for f in cls._fields_:
            assert getattr(cls, f[0]).offset == next(it), (name, f[0])


def test_weight_table_covers_the_checkpoint_layout():
    cfg = D.MMDiTConfig(blocks=2)
    t = D.weight_table(cfg)
    names = [n for n, *_ in t]
    assert len(names) == len(set(names)) == 13 + 2 * 32
    assert "transformer_blocks.1.attn.add_k_proj.weight" in names
    assert "transformer_blocks.0.txt_mlp.net.2.bias" in names
    shapes = {n: (r, c) for n, r, c, _ in t}
    assert shapes["transformer_blocks.0.img_mod.1.weight"] == (6 * 3072, 3072)
    assert shapes["img_in.weight"] == (3072, 64)
    assert shapes["txt_in.weight"] == (3072, 3584)


def test_cfg3_algorithmic_flops():
    # 99.9 TFLOP per step: GEMMs 76.5 + joint attention 23.4 (+ embeddings).
    f = D.MMDiTConfig().flops_per_step()
    assert 99.8e12 < f < 100.1e12


def test_cfg5_algorithmic_flops():
    # 13.52 TFLOP per SDXL UNet step at batch 2: convolutions, the 70
    # transformer blocks' GEMMs and attention, the time / add embeddings.
    f = D.UNetConfig().flops_per_step()
    assert 13.50e12 < f < 13.54e12
    # linear in the batch; a one-block sample is a small fraction of the step
    assert abs(D.UNetConfig(batch=1).flops_per_step() * 2 - f) < 1e6
    one = D.UNetConfig(depth=(0, 1, 1), batch=1)
    sample = one.resblock_flops(320, 320, 128 * 128) + one.transformer2d_flops(640, 64 * 64, 1)
    assert 50 < f / sample < 100


def test_synthetic_weights_prefix_filter_draws_the_same_values():
    cfg = D.UNetConfig(width=64, depth=(0, 1, 1), latent_height=16, latent_width=16, context_width=128,
                       add_width=256, time_width=64)
    full = dict(D.synthetic_weights(cfg, seed=3))
    part = dict(D.synthetic_weights(cfg, seed=3, only=("down_blocks.1.attentions.0.", "conv_in.")))
    assert part and set(part) == {k for k in full if k.startswith(("down_blocks.1.attentions.0.", "conv_in."))}
    for k, v in part.items():
        np.testing.assert_array_equal(v, full[k])


def test_device_open_fails_cleanly_without_gpu():
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    with pytest.raises(_lib.NdError):
        D.Device(0)
