"""ctypes binding of libvoxcpm_b200.so (the C ABI in include/voxcpm_b200.h).

The shared library is the product: every kernel runs from it. This module
only declares argument types. It raises at import when the library is
missing; there is no fallback path.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_size_t, c_uint, c_uint64, c_void_p
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / "libvoxcpm_b200.so"

VX_OK = 0
VX_UNSUPPORTED = 1
VX_INVALID = 2
VX_CUDA_ERROR = 3
VX_DEVICE_TIMEOUT = 4

WEIGHTS_BF16 = 0
WEIGHTS_BF16_TILES = 1
WEIGHTS_Q8_TILES = 2

OUT_F32 = 0
OUT_BF16 = 1

PRODUCT_ACCUMULATE = 1
PRODUCT_INDEPENDENT = 2

SPREAD_VARIANT = 102

CACHE_F32 = 0
CACHE_BF16 = 1


class WmmaPlan(ctypes.Structure):
    """vx_wmma_plan (replaces WmmaPlan, kernels/wmma_products.hpp:74-81)."""

    _fields_ = [
        ("splits", c_size_t),
        ("blocks_per_split", c_size_t),
        ("partial_floats", c_size_t),
        ("counters", c_size_t),
        ("variant", c_int),
    ]


class VaeConfig(ctypes.Structure):
    """vx_vae_config: the decoder fields of AudioVaeConfig (config.hpp:53-72)."""

    _fields_ = [
        ("latent_dim", c_size_t),
        ("decoder_dim", c_size_t),
        ("decoder_rates", c_size_t * 8),
        ("decoder_rate_count", c_size_t),
        ("out_sample_rate", c_size_t),
        ("sr_bin_boundaries", c_size_t * 8),
        ("sr_bin_boundary_count", c_size_t),
    ]


class MatmulShape(ctypes.Structure):
    """vx_matmul_shape (replaces MatmulShape, gemm.hpp:16-38): column-major
    C[m][n] (+)= op(A)[m][k] * op(B)[k][n], strides in elements."""

    _fields_ = [
        ("transpose_a", c_int),
        ("transpose_b", c_int),
        ("m", c_size_t),
        ("n", c_size_t),
        ("k", c_size_t),
        ("lda", c_size_t),
        ("ldb", c_size_t),
        ("ldc", c_size_t),
        ("stride_a", ctypes.c_int64),
        ("stride_b", ctypes.c_int64),
        ("stride_c", ctypes.c_int64),
        ("batch", c_size_t),
        ("accumulate", c_int),
    ]


def TuningBucket(size: int) -> int:
    """Rounds up to a multiple of 128 (gemm.hpp:74-77)."""
    return (size + 127) // 128 * 128


class SplitScratch(ctypes.Structure):
    """vx_split_scratch (kernels/wmma_products.hpp:62-68)."""

    _fields_ = [
        ("partials", c_void_p),
        ("partial_floats", c_size_t),
        ("counters", c_void_p),
        ("counter_count", c_size_t),
    ]


class StackConfig(ctypes.Structure):
    """vx_stack_config (config.hpp:15-31)."""

    _fields_ = [("hidden", c_int), ("intermediate", c_int), ("layers", c_int), ("heads", c_int),
                ("kv_heads", c_int), ("head_dim", c_int), ("rms_eps", c_float), ("rope", c_int)]


class ProjectionC(ctypes.Structure):
    """vx_projection (weights.hpp:20-26)."""

    _fields_ = [("format", c_int), ("weight", c_void_p), ("bias", c_void_p), ("in_", c_size_t),
                ("out", c_size_t)]


class LayerWeightsC(ctypes.Structure):
    """vx_layer_weights (weights.hpp:28-36)."""

    _fields_ = [("input_norm", c_void_p), ("qkv", ProjectionC), ("o", ProjectionC), ("post_norm", c_void_p),
                ("gate_up", ProjectionC), ("down", ProjectionC)]


class StackWeightsC(ctypes.Structure):
    """vx_stack_weights (weights.hpp:38-42)."""

    _fields_ = [("config", StackConfig), ("layers", POINTER(LayerWeightsC)), ("norm", c_void_p)]


class AttentionLayoutC(ctypes.Structure):
    """vx_attention_layout (transformer.hpp:38-48)."""

    _fields_ = [("positions", c_void_p), ("cache_rows", c_void_p), ("rows_per_sequence", c_size_t),
                ("keys_per_sequence", c_size_t), ("past", c_size_t), ("causal", c_int)]


class StackScratchC(ctypes.Structure):
    """vx_stack_scratch (transformer.hpp:50-58)."""

    _fields_ = [("normed", c_void_p), ("qkv", c_void_p), ("q", c_void_p), ("attention", c_void_p),
                ("gate_up", c_void_p), ("activation", c_void_p)]


class ModelConfig(ctypes.Structure):
    """vx_model_config (config.hpp:78-92)."""

    _fields_ = [("lm", StackConfig), ("residual_lm", StackConfig), ("encoder", StackConfig),
                ("dit", StackConfig), ("rope_theta", ctypes.c_double), ("rope_scaling", ctypes.c_double),
                ("rope_factors", ctypes.c_double * 64), ("patch_size", c_int), ("feat_dim", c_int),
                ("fsq_latent_dim", c_int), ("fsq_scale", c_float), ("max_length", c_int), ("vocab", c_int)]


CHECKPOINT_Q8 = 0
CHECKPOINT_BF16 = 1

# Tensor element types (safetensors.hpp:18) and file components.
DTYPE_F32, DTYPE_BF16, DTYPE_F16, DTYPE_I64, DTYPE_I32, DTYPE_U8, DTYPE_Q8_0 = range(7)
DTYPE_NAMES = ("F32", "BF16", "F16", "I64", "I32", "U8", "Q8_0")
COMPONENT_MODEL = 0
COMPONENT_VAE = 1


class TensorInfo(ctypes.Structure):
    """vx_tensor_info (safetensors.hpp:23-34)."""

    _fields_ = [("name", c_char_p), ("dtype", c_int), ("rank", c_int), ("shape", c_uint64 * 8),
                ("data", c_void_p), ("bytes", c_uint64), ("offset", c_uint64)]

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    "vx_last_error": (c_char_p, []),
    "vx_device_error": (c_int, [POINTER(c_uint)]),
    "vx_version": (c_char_p, []),
    "vx_q8_tiles_bytes": (c_size_t, [c_size_t, c_size_t]),
    "vx_bf16_tiles_bytes": (c_size_t, [c_size_t, c_size_t]),
    "vx_q8_0_to_tiles": (c_int, [c_void_p, c_size_t, c_size_t, c_void_p, c_void_p]),
    "vx_bf16_to_tiles": (c_int, [c_void_p, c_size_t, c_size_t, c_void_p, c_void_p]),
    "vx_q8_tiles_to_bf16": (c_int, [c_void_p, c_size_t, c_size_t, c_void_p, c_void_p]),
    "vx_bf16_tiles_to_rows": (c_int, [c_void_p, c_size_t, c_size_t, c_void_p, c_void_p]),
    "vx_plan_wmma": (WmmaPlan, [c_size_t, c_size_t, c_size_t, c_size_t]),
    "vx_wmma_q8": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_size_t, c_size_t, c_size_t, c_int,
         POINTER(WmmaPlan), POINTER(SplitScratch), c_void_p],
    ),
    "vx_wmma_bf16": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_size_t, c_size_t, c_size_t, c_int,
         POINTER(WmmaPlan), POINTER(SplitScratch), c_void_p],
    ),
    "vx_skinny_gemm": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_size_t, c_size_t, c_size_t, c_int, c_void_p],
    ),
    "vx_skinny_gemm_with": (
        c_int,
        [c_int, c_void_p, c_void_p, c_void_p, c_size_t, c_size_t, c_size_t, c_int, c_void_p],
    ),
    "vx_read_probe": (c_int, [c_void_p, c_size_t, c_uint, c_void_p, c_void_p]),
    "vx_product": (
        c_int,
        [c_int, c_void_p, c_void_p, c_void_p, c_int, c_size_t, c_size_t, c_size_t,
         c_int, POINTER(WmmaPlan), c_void_p],
    ),
    "vx_product_ex": (
        c_int,
        [c_int, c_void_p, c_void_p, c_void_p, c_int, c_size_t, c_size_t, c_size_t,
         c_uint, POINTER(WmmaPlan), c_void_p],
    ),
    "vx_product_host": (
        c_int,
        [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_size_t, c_size_t,
         c_size_t, c_uint, POINTER(WmmaPlan), c_void_p],
    ),
    "vx_stage": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    "vx_set_programmatic_launch": (None, [c_int]),
    "vx_set_product_l2_prefetch": (None, [c_int]),
    "vx_set_tensor_core_products": (None, [c_int]),
    "vx_tensor_core_products": (c_int, []),
    "vx_set_wide_tensor_core_products": (None, [c_int]),
    "vx_wide_tensor_core_products": (c_int, []),
    "vx_product_variants": (c_int, []),
    "vx_product_variant_shape": (
        None, [c_int, POINTER(c_int), POINTER(c_int), POINTER(c_int), POINTER(c_int)]
    ),
    "vx_random_q8_0": (c_int, [c_uint64, c_uint64, c_size_t, c_size_t, c_float, c_void_p]),
    "vx_random_bf16": (c_int, [c_uint64, c_uint64, c_size_t, c_float, c_float, c_void_p]),
    "vx_embed": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_size_t, c_float, c_void_p]),
    "vx_scatter_rows": (c_int, [c_void_p, c_void_p, c_void_p, c_size_t, c_size_t, c_void_p]),
    "vx_gather_rows": (c_int, [c_void_p, c_void_p, c_void_p, c_size_t, c_size_t, c_void_p]),
    "vx_rms_norm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_size_t, c_float, c_void_p]),
    "vx_qkv_rope": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
         c_size_t, c_size_t, c_size_t, c_size_t, c_size_t, c_void_p],
    ),
    "vx_attention": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_size_t, c_size_t, c_size_t, c_size_t,
         c_void_p, c_int, c_size_t, c_size_t, c_size_t, c_size_t, c_size_t, c_void_p],
    ),
    "vx_swiglu": (c_int, [c_void_p, c_void_p, c_size_t, c_size_t, c_void_p]),
    "vx_add_bias": (c_int, [c_void_p, c_void_p, c_size_t, c_size_t, c_void_p]),
    "vx_to_bf16": (c_int, [c_void_p, c_void_p, c_size_t, c_int, c_void_p]),
    "vx_concat_rows": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p, c_void_p, c_size_t, c_void_p,
                               c_size_t, c_void_p]),
    "vx_quantize": (c_int, [c_void_p, c_void_p, c_size_t, c_float, c_void_p]),
    "vx_select_rows": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_size_t, c_void_p]),
    "vx_prepend_special": (c_int, [c_void_p, c_void_p, c_void_p, c_size_t, c_size_t, c_size_t, c_void_p]),
    "vx_assemble_dit": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_size_t,
                                c_void_p]),
    "vx_guided_euler": (c_int, [c_void_p, c_void_p, c_size_t, c_float, c_float, c_void_p]),
    "vx_rope_table": (c_int, [ctypes.c_double, c_size_t, c_void_p, ctypes.c_double, c_size_t, c_void_p]),
    "vx_euler_schedule": (c_size_t, [c_size_t, c_float, c_void_p, c_void_p, c_void_p, c_size_t]),
    "vx_sinusoid": (c_int, [c_float, c_size_t, c_void_p]),
    "vx_model_config_released": (None, [POINTER(ModelConfig)]),
    "vx_generator_create": (c_void_p, [POINTER(ModelConfig), c_uint64, c_int, c_int]),
    "vx_generator_destroy": (None, [c_void_p]),
    "vx_generator_prefill": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t]),
    "vx_generator_step": (c_int, [c_void_p, c_void_p, c_size_t, c_float, c_void_p, c_void_p]),
    "vx_generator_velocity": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_void_p]),
    "vx_generator_dit_patch": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_float, c_void_p]),
    "vx_generator_dit_patch_static": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_float, c_void_p]),
    "vx_generator_replay_dit_patch": (c_int, [c_void_p]),
    "vx_set_dit_stall_for_tests": (None, [c_uint64]),
    "vx_set_persistent_max_ctas": (None, [c_size_t]),
    "vx_set_persistent_cooperative": (None, [c_int]),
    "vx_generator_state": (c_int, [c_void_p, c_char_p, c_void_p, c_size_t]),
    "vx_generator_set_state": (c_int, [c_void_p, c_char_p, c_void_p, c_size_t]),
    "vx_generator_set_graphs": (c_int, [c_void_p, c_int]),
    "vx_generator_set_persistent": (c_int, [c_void_p, c_int]),
    "vx_generator_persistent": (c_int, [c_void_p]),
    "vx_generator_position": (c_size_t, [c_void_p]),
    "vx_generator_latent": (c_void_p, [c_void_p]),
    "vx_generator_latent_event": (c_void_p, [c_void_p]),
    "vx_generator_weight_bytes": (c_size_t, [c_void_p]),
    "vx_generator_stream": (c_void_p, [c_void_p]),
    "vx_generator_batch_create": (c_void_p, [POINTER(ModelConfig), c_uint64, c_int, c_int, c_size_t]),
    "vx_generator_batch_create_from_files": (c_void_p, [POINTER(ModelConfig), c_void_p, c_int, c_size_t]),
    "vx_generator_batch_destroy": (None, [c_void_p]),
    "vx_generator_batch_slots": (c_size_t, [c_void_p]),
    "vx_generator_batch_prefill": (c_int, [c_void_p, c_size_t, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t]),
    "vx_generator_batch_step": (c_int, [c_void_p, c_void_p, c_void_p, c_size_t, c_float, c_void_p, c_void_p]),
    "vx_generator_batch_position": (c_size_t, [c_void_p, c_size_t]),
    "vx_generator_batch_state": (c_int, [c_void_p, c_size_t, c_char_p, c_void_p, c_size_t]),
    "vx_generator_batch_set_graphs": (c_int, [c_void_p, c_int]),
    "vx_generator_batch_stream": (c_void_p, [c_void_p]),
    "vx_vae_config_default": (None, [POINTER(VaeConfig)]),
    "vx_audio_vae_create": (c_void_p, [POINTER(VaeConfig), c_uint64]),
    "vx_audio_vae_destroy": (None, [c_void_p]),
    "vx_audio_vae_decode_hop": (c_size_t, [c_void_p]),
    "vx_audio_vae_stream": (c_void_p, [c_void_p]),
    "vx_audio_vae_reset": (c_int, [c_void_p]),
    "vx_audio_vae_decode": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    "vx_audio_vae_enqueue": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    "vx_audio_vae_collect": (c_int, [c_void_p, c_void_p, c_size_t, POINTER(c_size_t)]),
    "vx_model_files_open": (c_void_p, [c_char_p]),
    "vx_model_files_close": (None, [c_void_p]),
    "vx_model_files_is_voxcpm2_gguf": (c_int, [c_char_p]),
    "vx_model_files_is_gguf": (c_int, [c_void_p]),
    "vx_model_files_config": (c_char_p, [c_void_p]),
    "vx_model_files_tokenizer": (c_char_p, [c_void_p]),
    "vx_model_files_count": (c_size_t, [c_void_p, c_int]),
    "vx_model_files_tensor": (c_int, [c_void_p, c_int, c_size_t, POINTER(TensorInfo)]),
    "vx_model_files_find": (c_int, [c_void_p, c_int, c_char_p, POINTER(TensorInfo)]),
    "vx_parse_config": (c_int, [c_char_p, c_size_t, POINTER(ModelConfig)]),
    "vx_generator_create_from_files": (c_void_p, [POINTER(ModelConfig), c_void_p, c_int]),
    "vx_half_to_bf16": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    "vx_float_to_bf16": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    "vx_q8_0_to_bf16": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    "vx_plan_spread": (WmmaPlan, [c_int, c_size_t, c_size_t, c_size_t]),
    "vx_set_spread_products": (None, [c_int]),
    "vx_spread_products": (c_int, []),
    "vx_gemm_create": (c_void_p, [c_void_p]),
    "vx_gemm_destroy": (None, [c_void_p]),
    "vx_gemm_linear": (
        c_int,
        [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_size_t, c_size_t, c_size_t, c_int],
    ),
    "vx_gemm_linear_ex": (
        c_int,
        [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int, c_size_t, c_size_t, c_size_t, c_uint],
    ),
    "vx_gemm_linear_host": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int, c_size_t, c_size_t,
         c_size_t, c_uint],
    ),
    "vx_matmul": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "vx_gemm_matmul": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "vx_stack_scratch_elements": (c_int, [c_void_p, c_size_t, c_void_p]),
    "vx_kv_cache_create": (c_void_p, [c_void_p, c_size_t, c_int]),
    "vx_kv_cache_destroy": (None, [c_void_p]),
    "vx_kv_cache_capacity": (c_size_t, [c_void_p]),
    "vx_kv_cache_keys": (c_void_p, [c_void_p, c_size_t]),
    "vx_kv_cache_values": (c_void_p, [c_void_p, c_size_t]),
    "vx_forward_stack": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
                                 c_void_p, c_void_p]),
    "vx_project": (c_int, [c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
}

_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """The loaded library with argument types declared (raises if absent)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIBRARY.exists():
        raise ImportError(
            f"{LIBRARY} is missing: build it with `python -m voxcpm_b200.build` "
            "(the CUDA library is the only implementation; there is no fallback)"
        )
    lib = ctypes.CDLL(str(LIBRARY), mode=os.RTLD_NOW | ctypes.RTLD_GLOBAL)
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _lib = lib
    return lib


class VxError(RuntimeError):
    """A failed library call (the reference throws GpuError, device.hpp:16-30)."""

    def __init__(self, status: int, message: str):
        super().__init__(f"status {status}: {message}")
        self.status = status


def check(status: int, unsupported_ok: bool = False) -> bool:
    """Maps a vx_status to True / False (unsupported) / an exception."""
    if status == VX_OK:
        return True
    if status == VX_UNSUPPORTED and unsupported_ok:
        return False
    raise VxError(status, load().vx_last_error().decode(errors="replace"))
