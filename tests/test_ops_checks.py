"""The op wrappers refuse caller-provided outputs and vectors that cannot
hold what the op writes or reads (the C ABI sees only pointers and row
strides). CPU tensors: every check raises before anything is launched."""
import pytest
import torch

from naivediffusion_b200 import _lib, ops


def test_linear_rejects_a_short_residual_or_output():
    x = torch.zeros(64, 32, dtype=torch.bfloat16)
    w = torch.zeros(48, 32, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="residual"):
        ops.linear(x, w, epilogue=_lib.ND_EPI_RESIDUAL_ADD, residual=torch.zeros(63, 48))
    with pytest.raises(ValueError, match="residual"):
        ops.linear(x, w, epilogue=_lib.ND_EPI_RESIDUAL_ADD, residual=torch.zeros(64, 48, dtype=torch.float16))
    with pytest.raises(ValueError, match="out"):
        ops.linear(x, w, out=torch.zeros(64, 47, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="out"):
        ops.linear(x, w, out=torch.zeros(48, 64, dtype=torch.bfloat16).t())   # column stride 48


def test_attention_rejects_a_short_output():
    q = torch.zeros(128, 256, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="attention: out"):
        ops.attention(q, q, q, 2, out=torch.zeros(127, 256, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="attention: out"):
        ops.attention(q, q, q, 2, out=torch.zeros(128, 256, dtype=torch.float16))


def test_modulate_rejects_short_vectors_and_outputs():
    x = torch.zeros(256, 512)
    sc = torch.zeros(512)
    with pytest.raises(ValueError, match="scale"):
        ops.modulate(x, None, torch.zeros(511))
    with pytest.raises(ValueError, match="scale"):
        ops.modulate(x, None, sc, group_split=128)          # two groups need 2 x 512
    with pytest.raises(ValueError, match="shift"):
        ops.modulate(x, torch.zeros(512, dtype=torch.float16), sc)
    with pytest.raises(ValueError, match="modulate: out"):
        ops.modulate(x, None, sc, out=torch.zeros(256, 511, dtype=torch.bfloat16))


def test_sampler_step_rejects_mismatched_buffers():
    s = torch.zeros(16)
    with pytest.raises(ValueError, match="branches"):
        ops.sampler_step(0, 0, torch.zeros(24), s, sigma=1.0, sigma_next=0.5)
    with pytest.raises(ValueError, match="last"):
        ops.sampler_step(0, 0, torch.zeros(32), s, last=torch.zeros(8), sigma=1.0, sigma_next=0.5)
    with pytest.raises(ValueError, match="next_input"):
        ops.sampler_step(0, 0, s, s, next_input=torch.zeros(16, dtype=torch.float16), sigma=1.0, sigma_next=0.5)
