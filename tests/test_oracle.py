"""Pins the CPU oracle (oracle/nd_oracle.cpp) against the known-answer checks
of the reference's own tests and smoke command, restated here.

The reference is C#; nothing of it can run in this container, so these
restatements are what pins the oracle (its header says so). Sources:
  tests/NaiveDiffusion.Tests/BlockQuantizerTests.cs:10-71
  tests/NaiveDiffusion.Tests/TransformerInputsTests.cs:21-89
  src/NaiveDiffusion.Cli/SmokeTest.cs (Gemm :66-87, MHA :337-387,
    masked attention :393-485, RotateHalf :738-776)
  src/NaiveDiffusion/Tensors/CpuMath.cs (LayerNorm double two-pass, Erf A&S)
"""
import math

import numpy as np
import pytest

import oracle as O


# ---------------------------------------------------------------- BlockQuantizer

def test_quantizer_fits_whole_blocks_only():
    # BlockQuantizerTests.FitsNeedsWholeBlocksPerRow / RefusesAShapeThatDoesNotTile
    O.quantize(np.zeros((4, 64), np.float32))
    with pytest.raises(ValueError):
        O.quantize(np.zeros((4, 48), np.float32))
    with pytest.raises(ValueError):
        O.quantize(np.zeros((1, 48), np.float32))


def test_quantizer_round_trip_within_half_a_step():
    # BlockQuantizerTests.DequantizingComesBackWithinHalfAStep
    rng = np.random.default_rng(1)
    rows, cols = 4, 96
    vals = (rng.random(rows * cols) * 2 - 1) * np.where(rng.integers(0, 4, rows * cols) == 0, 8, 1)
    vals = vals.astype(np.float32).reshape(rows, cols)
    q, s16 = O.quantize(vals)
    assert q.dtype == np.int8 and q.shape == (rows, cols)
    assert s16.shape == (rows, cols // 32)
    s = O.from_f16_bits(s16)
    for r in range(rows):
        for b in range(cols // 32):
            blk = vals[r, b * 32:(b + 1) * 32]
            peak = np.abs(blk).max()
            sc = s[r, b]
            assert abs(sc - peak / 127) <= peak / 127 * 1e-3
            qq = q[r, b * 32:(b + 1) * 32].astype(np.float32)
            assert np.all(np.abs(qq) <= 127)
            assert np.all(np.abs(qq * sc - blk) <= sc * 0.5 + 1e-6)


def test_quantizer_zero_block_has_zero_scale():
    # BlockQuantizerTests.AZeroBlockHasAZeroScale: 1e-9 / 127 underflows fp16.
    v = np.zeros((2, 32), np.float32)
    v.flat[40] = 1e-9
    q, s = O.quantize(v)
    assert np.all(s == 0) and np.all(q == 0)


def test_quantizer_rounds_half_to_even_against_stored_scale():
    # BlockQuantizer.QuantizeBlock uses MathF.Round (banker's rounding) of
    # w * (1 / stored) where stored is the fp16-rounded scale.
    w = np.zeros((1, 32), np.float32)
    w[0, 0] = 127.0       # scale 1.0 exactly
    w[0, 1] = 2.5         # -> 2 (even)
    w[0, 2] = 3.5         # -> 4 (even)
    w[0, 3] = -0.5        # -> -0 (even)
    q, s = O.quantize(w)
    assert O.from_f16_bits(s)[0, 0] == 1.0
    assert list(q[0, :4]) == [127, 2, 4, 0]


def test_per_channel_quantizer_fp32_scales():
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((8, 256)) * 0.02).astype(np.float32)
    q, s = O.quantize(w, group=256, scale_f16=False)
    assert s.dtype == np.float32 and s.shape == (8, 1)
    np.testing.assert_array_equal(s[:, 0], np.abs(w).max(1).astype(np.float32) / np.float32(127))
    deq = O.dequantize(q, s, group=256)
    assert np.all(np.abs(deq - w) <= s * 0.5 + 1e-9)


def test_f16_and_bf16_conversions_round_to_nearest_even():
    x = np.array([1.0, 1 + 2 ** -11, 1 + 3 * 2 ** -11, 65504, 65520, 1e-8, 2 ** -24, -2.5], np.float32)
    rng = np.random.default_rng(0)
    y = (rng.standard_normal(10000) * 10.0 ** rng.integers(-8, 6, 10000)).astype(np.float32)
    with np.errstate(over="ignore"):  # numpy warns on the overflow to inf it performs
        np.testing.assert_array_equal(O.to_f16_bits(x), x.astype(np.float16).view(np.uint16))
        np.testing.assert_array_equal(O.to_f16_bits(y), y.astype(np.float16).view(np.uint16))
        np.testing.assert_array_equal(O.from_f16_bits(O.to_f16_bits(y)), y.astype(np.float16).astype(np.float32))
    b = O.to_bf16_bits(np.array([1.0, 1 + 2 ** -8, 1 + 3 * 2 ** -8], np.float32))
    assert list(O.from_bf16_bits(b)) == [1.0, 1.0, 1 + 2 ** -6]


# ---------------------------------------------------------------- TransformerInputs

def _bf16_truncated(values):
    """NarrowingLossTests.BFloat16 (tests/NaiveDiffusion.Tests/NarrowingLossTests.cs:15-24):
    the top 16 bits of each float32."""
    bits = (np.array(values, np.float32).view(np.uint32) >> 16).astype(np.uint16)
    return O.from_bf16_bits(bits)


def test_bfloat16_inside_the_normal_range_narrows_to_float16_exactly():
    """NarrowingLossTests.BFloat16InsideTheNormalRangeNarrowsExactly (:26-35):
    what the fp16 (SDXL) upload does to a bf16 checkpoint's values."""
    v = _bf16_truncated([1.0, -0.5, 0.0, 1024.0, 1e-3, -60000.0])
    assert np.array_equal(O.round_f16(v), v)


def test_each_way_out_of_the_float16_range():
    """NarrowingLossTests.EachWayOutOfTheRangeIsCountedWithItsEnergy (:37-49):
    1e5 overflows, 1e-5 lands in the subnormal range, 1e-9 flushes to zero, NaN stays NaN."""
    v = _bf16_truncated([1e5, 1e-5, 1e-9, 1.0, float("nan")])
    h = O.round_f16(v)
    assert np.isinf(h[0])
    assert 0 < abs(float(h[1])) < 6.103515625e-05   # below fp16's smallest normal, 2^-14
    assert h[2] == 0.0
    assert h[3] == 1.0
    assert np.isnan(h[4])


def test_sinusoid_is_half_cosines_then_half_sines():
    assert list(O.sinusoid(0.0, 8)) == [1, 1, 1, 1, 0, 0, 0, 0]
    a = O.sinusoid(1.0, 8)
    assert abs(a[0] - math.cos(1)) < 1e-6 and abs(a[1] - math.cos(0.1)) < 1e-6
    assert abs(a[4] - math.sin(1)) < 1e-6 and abs(a[7] - math.sin(0.001)) < 1e-6


def test_qwen_rope_tables_place_text_after_image():
    rows, cols, tlen, ctx = 2, 3, 5, 7
    c, s = O.qwen_rope_tables(rows, cols, tlen, ctx)
    assert c.shape == (rows * cols + ctx, 64)
    assert abs(c[0, 0] - math.cos(tlen)) < 1e-6
    assert s[rows * cols, 0] == 0
    assert abs(s[rows * cols + 3, 0] - math.sin(3)) < 1e-6
    assert abs(s[0, 8] - math.sin(-1)) < 1e-6
    assert abs(s[cols, 8]) < 1e-6
    assert abs(s[0, 36] - math.sin(-2)) < 1e-6
    assert abs(s[2, 36]) < 1e-6
    p = rows * cols + 4
    assert abs(s[p, 8] - math.sin(4)) < 1e-6 and abs(s[p, 36] - math.sin(4)) < 1e-6


def test_anima_rope_tables_leave_temporal_pairs_still():
    c, s = O.anima_rope_tables(2, 2, 128)
    assert c.shape == (4, 64)
    assert np.all(c[:, :22] == 1) and np.all(s[:, :22] == 0)
    assert abs(s[2, 22] - math.sin(1)) < 1e-6
    assert abs(s[1, 22 + 21] - math.sin(1)) < 1e-6
    assert s[1, 22] == 0


# ---------------------------------------------------------------- SmokeTest ops

def test_gemm_known_product():
    # SmokeTest.Gemm: [2,3] x [3,4] with a = 1..6, b = 0..11 (b given [in, out]).
    a = np.arange(1, 7, dtype=np.float32).reshape(2, 3)
    b = np.arange(12, dtype=np.float32).reshape(3, 4)
    y = O.linear(a, b.T.copy())
    np.testing.assert_array_equal(y, a @ b)


def test_linear_reads_every_float_width_alike():
    """CpuMathTests.LinearReadsEveryFloatWidthAlike (tests/NaiveDiffusion.Tests/
    CpuMathTests.cs:40-67): a 5 x 8 matrix of values exact at every width,
    (i % 7 - 3) * 0.25, read from fp32, fp16 and bf16 storage (widened as
    HostTensor does), gives the same product as the float loop."""
    w = np.array([(i % 7 - 3) * 0.25 for i in range(40)], np.float32).reshape(5, 8)
    x = np.sin(np.arange(24, dtype=np.float32)).reshape(3, 8)
    bias = np.array([1, 2, 3, 4, 5], np.float32)
    expected = np.empty((3, 5), np.float32)
    for m in range(3):
        for o in range(5):
            acc = np.float32(bias[o])
            for i in range(8):
                acc = np.float32(acc + x[m, i] * w[o, i])
            expected[m, o] = acc
    for widened in (w, O.from_f16_bits(O.to_f16_bits(w)), O.from_bf16_bits(O.to_bf16_bits(w))):
        assert np.array_equal(widened, w)
        assert np.abs(O.linear(x, widened, bias) - expected).max() <= 1e-5


def test_linear_matches_float64():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((37, 200)).astype(np.float32)
    w = rng.standard_normal((53, 200)).astype(np.float32)
    b = rng.standard_normal(53).astype(np.float32)
    y = O.linear(x, w, b)
    ref = x.astype(np.float64) @ w.T.astype(np.float64) + b
    assert np.abs(y - ref).max() < 1e-4


def test_layernorm_double_two_pass_keeps_nearly_constant_rows():
    # CpuMath.LayerNorm's reason for double: a nearly-constant row.
    x = (1000.0 + np.array([[0, 1e-3, -1e-3, 2e-3]])).astype(np.float32)
    y = O.layernorm(x, 1e-12)
    xd = x.astype(np.float64)
    ref = (xd - xd.mean()) / np.sqrt(xd.var() + 1e-12)
    assert np.abs(y - ref).max() < 1e-5


def test_modulate_and_rmsnorm():
    rng = np.random.default_rng(2)
    x = rng.standard_normal((9, 64)).astype(np.float32)
    sh, sc = rng.standard_normal(64).astype(np.float32), rng.standard_normal(64).astype(np.float32)
    y = O.modulate(x, sh, sc, 1e-6)
    xd = x.astype(np.float64)
    ln = (xd - xd.mean(1, keepdims=True)) / np.sqrt(xd.var(1, keepdims=True) + 1e-6)
    assert np.abs(y - (ln * (1 + sc) + sh)).max() < 1e-5
    w = rng.standard_normal(64).astype(np.float32)
    r = O.rmsnorm(x, w, 1e-6)
    ref = xd / np.sqrt((xd ** 2).mean(1, keepdims=True) + 1e-6) * w
    assert np.abs(r - ref).max() < 1e-5


def test_rotate_half():
    # SmokeTest.RotateHalf: feature i pairs with i + dim/2.
    rng = np.random.default_rng(4)
    rows, heads, dim = 5, 3, 8
    x = rng.standard_normal((rows, heads * dim)).astype(np.float32)
    ang = rng.random((rows, dim // 2)).astype(np.float32) * 6
    c, s = np.cos(ang), np.sin(ang)
    y = O.rope(x, heads, c, s).reshape(rows, heads, dim)
    xv = x.reshape(rows, heads, dim)
    lo, hi = xv[..., :4], xv[..., 4:]
    ref = np.concatenate([lo * c[:, None] - hi * s[:, None], hi * c[:, None] + lo * s[:, None]], -1)
    assert np.abs(y - ref).max() < 1e-6


def _attn_ref(q, k, v, heads, causal=False, key_len=0):
    rows, kr = q.shape[0], k.shape[0]
    d = q.shape[1] // heads
    out = np.zeros_like(q, dtype=np.float64)
    keys = key_len if 0 < key_len < kr else kr
    for h in range(heads):
        qh = q[:, h * d:(h + 1) * d].astype(np.float64)
        kh = k[:keys, h * d:(h + 1) * d].astype(np.float64)
        vh = v[:keys, h * d:(h + 1) * d].astype(np.float64)
        s = qh @ kh.T / math.sqrt(d)
        if causal:
            s = np.where(np.tril(np.ones_like(s)) > 0, s, -np.inf)
        p = np.exp(s - s.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        out[:, h * d:(h + 1) * d] = p @ vh
    return out


@pytest.mark.parametrize("causal,key_len", [(False, 0), (True, 0), (False, 5)])
def test_attention(causal, key_len):
    # SmokeTest.MultiheadAttention / MaskedAttention (masked keys left out).
    rng = np.random.default_rng(5)
    heads, d = 2, 16
    q = rng.standard_normal((9, heads * d)).astype(np.float32)
    k = rng.standard_normal((9, heads * d)).astype(np.float32)
    v = rng.standard_normal((9, heads * d)).astype(np.float32)
    y = O.attention(q, k, v, heads, causal=causal, key_len=key_len)
    assert np.abs(y - _attn_ref(q, k, v, heads, causal, key_len)).max() < 1e-5


def test_gelu_variants():
    x = np.linspace(-6, 6, 1001).astype(np.float32)
    erf = np.array([math.erf(v / math.sqrt(2)) for v in x.astype(np.float64)])
    exact = 0.5 * x * (1 + erf)
    assert np.abs(O.gelu(x) - exact).max() < 1e-5       # A&S 7.1.26: |err| <= 1.5e-7 in erf
    tanh_form = 0.5 * x * (1 + np.tanh(math.sqrt(2 / math.pi) * (x + 0.044715 * x ** 3)))
    assert np.abs(O.gelu_tanh(x) - tanh_form).max() < 1e-5
    assert np.abs(O.silu(x) - x / (1 + np.exp(-x.astype(np.float64)))).max() < 1e-5


def test_group_norm_smoke_recipe():
    # SmokeTest.GroupNormalization (NaiveDiffusion.Cli/SmokeTest.cs:208-239):
    # [1, 4, 1, 3] in two groups, eps 1e-5, double mean / variance.
    data = np.array([1, 2, 3, 4, 5, 6, 0, 0, 0, 1, 1, 4], np.float32)
    y = O.group_norm(data.reshape(4, 1, 3), 2, eps=1e-5).ravel()
    ref = []
    for g in range(2):
        d = data[g * 6:(g + 1) * 6].astype(np.float64)
        ref += list((d - d.mean()) / np.sqrt(d.var() + 1e-5))
    assert np.abs(y - np.array(ref)).max() < 1e-6


def test_convolution_smoke_recipe():
    # SmokeTest.Convolution (SmokeTest.cs:241-281): an identity tap plus 0.5
    # and a 3x3 box sum minus 1 over 0..8, padding 1.
    x = np.arange(9, dtype=np.float32).reshape(1, 3, 3)
    f = np.zeros((2, 1, 3, 3), np.float32)
    f[0, 0, 1, 1] = 1
    f[1] = 1
    y = O.conv2d(x, f, np.array([0.5, -1], np.float32))
    assert np.array_equal(y[0].ravel(), np.arange(9) + 0.5)
    box = np.pad(x[0], 1)
    ref = np.array([[box[r:r + 3, c:c + 3].sum() for c in range(3)] for r in range(3)]) - 1
    assert np.array_equal(y[1], ref)


def test_strided_convolution():
    rng = np.random.default_rng(8)
    x = rng.standard_normal((3, 8, 6)).astype(np.float32)
    w = rng.standard_normal((4, 3, 3, 3)).astype(np.float32)
    y = O.conv2d(x, w, None, stride=2, pad=1)
    assert y.shape == (4, 4, 3)
    xp = np.pad(x, ((0, 0), (1, 1), (1, 1))).astype(np.float64)
    ref = np.zeros((4, 4, 3))
    for o in range(4):
        for r in range(4):
            for c in range(3):
                ref[o, r, c] = (w[o] * xp[:, 2 * r:2 * r + 3, 2 * c:2 * c + 3]).sum()
    assert np.abs(y - ref).max() < 1e-4


# ---------------------------------------------------------------- sampling
# The reference's sampler checks, restated (SchedulersTests.cs:142-205,
# FlowSamplingTests.cs "ASamplerRunsTheLineDownToCleanData"): given perfect
# predictions, every sampler walks the sample down to the clean latent.

def _vp_sigmas(steps, rho=7.0):
    """SDXL's scaled-linear VP levels (beta 0.00085 .. 0.012 over 1000 steps)
    spaced evenly in sigma^(1/rho) (Karras), then 0."""
    import math
    betas = np.linspace(0.00085 ** 0.5, 0.012 ** 0.5, 1000, dtype=np.float64) ** 2
    alphas = np.cumprod(1.0 - betas)
    levels = np.sqrt((1.0 - alphas) / alphas)
    lo, hi = levels[0] ** (1 / rho), levels[-1] ** (1 / rho)
    s = [(hi + i / (steps - 1) * (lo - hi)) ** rho for i in range(steps)]
    return np.array(s + [0.0], dtype=np.float32)


def _flow_sigmas(steps, shift=3.0):
    t = np.linspace(1.0, 0.0, steps + 1)
    return np.array([shift * x / (1 + (shift - 1) * x) for x in t], dtype=np.float32)


@pytest.mark.parametrize("prediction", ["epsilon", "velocity", "flow"])
@pytest.mark.parametrize("sampler", ["euler", "euler_a", "dpmpp_2m", "dpmpp_2m_sde"])
def test_oracle_samplers_land_on_the_clean_latent(sampler, prediction):
    from naivediffusion_b200.sampling import PREDICTIONS, SAMPLERS, StepScalars
    clean = np.sin(np.arange(64) * 0.37).astype(np.float32)
    rng = np.random.default_rng(3)
    sigmas = _flow_sigmas(15) if prediction == "flow" else _vp_sigmas(15)
    sch = StepScalars(sampler, prediction, sigmas)
    sample = (clean + rng.standard_normal(64).astype(np.float32) * sigmas[0]).astype(np.float32)
    last = np.zeros(64, np.float32)
    for step in range(sch.steps):
        s = float(sigmas[step])
        if prediction == "epsilon":
            out = (sample - clean) / np.float32(s)
        elif prediction == "flow":
            out = (sample - clean) / np.float32(s)   # noise - x0 on the line x = (1 - s) x0 + s noise
        else:
            eps = (sample - clean) / np.float32(s)
            out = (eps - np.float32(s) * clean) / np.float32(np.sqrt(s * s + 1))
        d = sch.at(step)
        noise = rng.standard_normal(64).astype(np.float32) if sch.stochastic else None
        sample, last, den = O.sampler_step(SAMPLERS[sampler], PREDICTIONS[prediction], out.astype(np.float32),
                                           sample, last=last, noise=noise, want_denoised=True, **d)
        assert np.abs(den - clean).max() < 2e-3, (step, np.abs(den - clean).max())
    assert np.abs(sample - clean).max() < 2e-3


def test_oracle_guidance_combine_and_euler_arithmetic():
    """Combine then Euler, checked against float32 numpy arithmetic done the
    reference's way (uncond + g * (cond - uncond); sample += d * (sn - s))."""
    rng = np.random.default_rng(0)
    out = rng.standard_normal((2, 1000)).astype(np.float32)
    sample = rng.standard_normal(1000).astype(np.float32)
    g = np.float32(4.5)
    pred = out[0] + g * (out[1] - out[0])
    delta = np.float32(0.25) - np.float32(1.5)
    ref = sample + pred * delta
    got, _ = O.sampler_step(0, 0, out, sample, guidance=float(g), sigma=1.5, sigma_next=0.25)
    assert np.array_equal(got, ref)


def test_causal_table_golden():
    # TransformerInputsTests.TheCausalTableIsATriangleClosedOverThePadding and
    # QwenImagesBranchesArePaddedAndMaskedToTheirOwnLength.
    assert O.causal_table(1, 1).ravel().tolist() == [1]
    assert O.causal_table(2, 4).ravel().tolist() == [1, 0, 0, 0, 1, 1, 0, 0, 1, 1, 0, 0, 1, 1, 0, 0]
    assert O.causal_table(2, 3).ravel().tolist() == [1, 0, 0, 1, 1, 0, 1, 1, 0]
    assert O.causal_table(3, 3).ravel().tolist() == [1, 0, 0, 1, 1, 0, 1, 1, 1]


@pytest.mark.parametrize("real,rows", [(3, 7), (7, 7), (1, 5)])
def test_causal_plus_key_count_is_the_causal_table(real, rows):
    """The text rows' attention under QwenImageConditioning.CausalTable is the
    causal mask with the keys past the real text left out."""
    rng = np.random.default_rng(real * 10 + rows)
    heads, d = 2, 16
    q, k, v = (rng.standard_normal((rows, heads * d)).astype(np.float32) for _ in range(3))
    y = O.attention(q, k, v, heads, causal=True, key_len=real if real < rows else 0)
    mask = O.causal_table(real, rows) > 0
    ref = np.zeros((rows, heads * d))
    for h in range(heads):
        sl = slice(h * d, (h + 1) * d)
        s = q[:, sl].astype(np.float64) @ k[:, sl].astype(np.float64).T / math.sqrt(d)
        s = np.where(mask, s, -np.inf)
        p = np.exp(s - s.max(1, keepdims=True))
        ref[:, sl] = (p / p.sum(1, keepdims=True)) @ v[:, sl]
    assert np.abs(y - ref).max() < 1e-5


def test_pair_rotation_is_rotate_half_on_permuted_features():
    """QwenImageDit.PairsToHalves: rotating adjacent pairs equals rotating
    halves after reordering each head's features (2i, 2i+1) -> (i, 64+i)."""
    rng = np.random.default_rng(9)
    rows, heads, dim = 6, 3, 128
    x = rng.standard_normal((rows, heads * dim)).astype(np.float32)
    ang = rng.random((rows, dim // 2)).astype(np.float32) * 6
    c, s = np.cos(ang), np.sin(ang)
    perm = np.concatenate([np.arange(0, dim, 2), np.arange(1, dim, 2)])  # halves order -> pair source
    xp = x.reshape(rows, heads, dim)[:, :, perm].reshape(rows, heads * dim)
    y_half = O.rope(xp, heads, c, s).reshape(rows, heads, dim)
    y_pair = O.rope_pairs(x, heads, c, s).reshape(rows, heads, dim)
    assert np.array_equal(y_half, y_pair[:, :, perm])
