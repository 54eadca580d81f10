"""ctypes binding of libnd_denoise.so (include/nd_denoise.h).

This is the Python stand-in for the C# P/Invoke layer: the same C entry
points a `[LibraryImport("nd_denoise")]` class would bind. Loading fails
loudly when the library is missing; there is no fallback path.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libnd_denoise.so"

ND_OK = 0
ND_ERR_INVALID = 1
ND_ERR_OOM = 2
ND_ERR_CUDA = 3
ND_ERR_TIMEOUT = 4
ND_ERR_STATE = 5
ND_ERR_UNSUPPORTED = 6
ND_ERR_MISSING_WEIGHT = 7

ND_F32, ND_F16, ND_BF16, ND_I8, ND_I32 = 0, 1, 2, 3, 4
ND_BF16X2 = 5  # fp32 as a bf16 hi|lo pair: [rows, 2 * cols], hi columns then lo
ND_SAMPLER_EULER, ND_SAMPLER_EULER_A, ND_SAMPLER_DPMPP_2M, ND_SAMPLER_DPMPP_2M_SDE = 0, 1, 2, 3
ND_PRED_EPSILON, ND_PRED_VELOCITY, ND_PRED_FLOW = 0, 1, 2

ND_EPI_STORE = 0
ND_EPI_GELU_TANH = 1
ND_EPI_GELU_ERF = 2
ND_EPI_SILU = 3
ND_EPI_RESIDUAL_GATE = 4
ND_EPI_STORE_F32 = 5
ND_EPI_QK_NORM_ROPE = 6
ND_EPI_RESIDUAL_ADD = 7
ND_EPI_ADD_STORE = 8
ND_EPI_SWIGLU = 9
ND_EPI_GEGLU = 10


class NdError(RuntimeError):
    """A nonzero status from the library, with nd_last_error()'s message."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code


class LinearArgs(C.Structure):
    _fields_ = [
        ("dtype", C.c_int), ("epilogue", C.c_int),
        ("rows", C.c_int64), ("in_features", C.c_int64), ("out_features", C.c_int64),
        ("x", C.c_void_p), ("ldx", C.c_int64),
        ("weight", C.c_void_p), ("bias", C.c_void_p), ("group_split", C.c_int64),
        ("y", C.c_void_p), ("ldy", C.c_int64),
        ("residual", C.c_void_p), ("ldr", C.c_int64),
        ("gate", C.c_void_p), ("gate_stride", C.c_int64), ("qk_norm", C.c_void_p),
        ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p),
        ("qk_cols", C.c_int64), ("eps", C.c_float),
        ("weight_dtype", C.c_int), ("scales", C.c_void_p), ("scale_dtype", C.c_int),
        ("quant_group", C.c_int64), ("norm_span", C.c_int64), ("rope_period", C.c_int64),
        ("addend", C.c_void_p), ("ld_add", C.c_int64), ("shared_weights", C.c_int),
    ]


class ConvArgs(C.Structure):
    _fields_ = [
        ("dtype", C.c_int), ("epilogue", C.c_int),
        ("batch", C.c_int), ("height", C.c_int), ("width", C.c_int), ("in_channels", C.c_int),
        ("out_channels", C.c_int), ("stride", C.c_int),
        ("x", C.c_void_p), ("weight", C.c_void_p), ("bias", C.c_void_p), ("per_batch_bias", C.c_int),
        ("bias_stride", C.c_int64),
        ("y", C.c_void_p), ("y_f32", C.c_void_p), ("addend", C.c_void_p),
    ]


class AttentionArgs(C.Structure):
    _fields_ = [
        ("dtype", C.c_int), ("heads", C.c_int), ("head_dim", C.c_int), ("batch", C.c_int),
        ("q_rows", C.c_int64), ("kv_rows", C.c_int64), ("key_limit", C.c_int64),
        ("causal", C.c_int),
        ("q", C.c_void_p), ("ldq", C.c_int64), ("k", C.c_void_p), ("ldk", C.c_int64),
        ("v", C.c_void_p), ("ldv", C.c_int64), ("out", C.c_void_p), ("ldo", C.c_int64),
        ("scale", C.c_float), ("out_dtype", C.c_int), ("kv_heads", C.c_int),
        ("workspace", C.c_void_p), ("workspace_bytes", C.c_int64),
    ]


class ModulateArgs(C.Structure):
    _fields_ = [
        ("x", C.c_void_p), ("ldx", C.c_int64),
        ("y", C.c_void_p), ("ldy", C.c_int64), ("out_dtype", C.c_int),
        ("rows", C.c_int64), ("width", C.c_int64),
        ("shift", C.c_void_p), ("scale", C.c_void_p),
        ("vec_stride", C.c_int64), ("group_split", C.c_int64), ("eps", C.c_float),
        ("affine", C.c_int),
    ]


class RmsNormArgs(C.Structure):
    _fields_ = [
        ("x", C.c_void_p), ("ldx", C.c_int64), ("in_dtype", C.c_int),
        ("y", C.c_void_p), ("ldy", C.c_int64), ("out_dtype", C.c_int),
        ("rows", C.c_int64), ("width", C.c_int64),
        ("weight", C.c_void_p), ("plus_one", C.c_int), ("eps", C.c_float), ("silu", C.c_int),
    ]


class GemvArgs(C.Structure):
    _fields_ = [
        ("w", C.c_void_p), ("w_dtype", C.c_int), ("n", C.c_int64), ("k", C.c_int64),
        ("x", C.c_void_p), ("batch", C.c_int), ("pre_silu", C.c_int),
        ("bias", C.c_void_p), ("act", C.c_int), ("y", C.c_void_p),
        ("scales", C.c_void_p), ("scale_dtype", C.c_int), ("quant_group", C.c_int64),
        ("x_rows_per_vec", C.c_int64), ("bias_period", C.c_int64),
    ]


class SamplerArgs(C.Structure):
    _fields_ = [
        ("sampler", C.c_int), ("prediction", C.c_int), ("n", C.c_int64), ("branches", C.c_int),
        ("out", C.c_void_p), ("guidance", C.c_float), ("sample", C.c_void_p), ("last_denoised", C.c_void_p),
        ("noise", C.c_void_p), ("denoised_out", C.c_void_p), ("next_input", C.c_void_p),
        ("next_input_scale", C.c_float), ("sigma", C.c_float), ("sigma_next", C.c_float),
        ("up", C.c_double), ("down", C.c_double), ("rescale", C.c_double), ("noise_scale", C.c_double),
        ("shrink", C.c_double), ("weight", C.c_double), ("second_order", C.c_int),
    ]


_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(
                f"{LIB_PATH} is missing: build it with `python -m naivediffusion_b200.build`")
        L = C.CDLL(str(LIB_PATH))
        L.nd_last_error.restype = C.c_char_p
        L.nd_version.restype = C.c_char_p
        L.nd_op_linear.argtypes = [C.POINTER(LinearArgs), C.c_void_p]
        L.nd_op_sync.argtypes = [C.c_void_p]
        L.nd_op_wait_probe.argtypes = [C.c_uint64, C.c_int, C.c_int, C.c_void_p]
        L.nd_op_quantize.argtypes = [C.c_void_p, C.c_int, C.c_int64, C.c_int64, C.c_int64, C.c_int,
                                     C.c_void_p, C.c_void_p, C.c_void_p]
        L.nd_op_dequantize.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int64, C.c_int64,
                                       C.c_int64, C.c_void_p, C.c_int, C.c_void_p]
        L.nd_op_group_norm.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                       C.c_void_p, C.c_void_p, C.c_float, C.c_int, C.c_void_p]
        L.nd_op_geglu.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int64, C.c_int64, C.c_void_p]
        L.nd_op_conv2d.argtypes = [C.POINTER(ConvArgs), C.c_void_p]
        L.nd_op_attention.argtypes = [C.POINTER(AttentionArgs), C.c_void_p]
        L.nd_attention_workspace_bytes.argtypes = [C.c_int]
        L.nd_attention_workspace_bytes.restype = C.c_int64
        L.nd_op_sampler_step.argtypes = [C.POINTER(SamplerArgs), C.c_void_p]
        L.nd_op_modulate.argtypes = [C.POINTER(ModulateArgs), C.c_void_p]
        L.nd_op_rmsnorm.argtypes = [C.POINTER(RmsNormArgs), C.c_void_p]
        L.nd_op_head_norm_rope.argtypes = [C.c_void_p, C.c_int, C.c_int64, C.c_int64, C.c_int, C.c_int, C.c_void_p,
                                           C.c_void_p, C.c_void_p, C.c_float, C.c_void_p]
        L.nd_op_gemv.argtypes = [C.POINTER(GemvArgs), C.c_void_p]
        L.nd_op_patchify.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                     C.c_int, C.c_int, C.c_int64, C.c_void_p]
        L.nd_op_unpatchify.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                       C.c_int, C.c_int, C.c_void_p]
        L.nd_op_tile_gather.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                        C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        L.nd_op_tile_blend.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_int,
                                       C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        _lib = L
    return _lib


def check(code: int) -> None:
    if code != ND_OK:
        raise NdError(code, lib().nd_last_error().decode(errors="replace"))
