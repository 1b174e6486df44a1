"""ctypes binding of libomnivoice_b200.so (include/ov_*.h).

There is no Python or CPU fallback: if the library is missing or a CUDA
call fails, the functions raise.
"""
from __future__ import annotations

import ctypes
from ctypes import (POINTER, Structure, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t,
                    c_uint16, c_uint32, c_uint64, c_void_p)
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libomnivoice_b200.so")

OV_OK = 0
OV_ERR_INVALID = 1
OV_ERR_CUDA = 2
OV_ERR_OOM = 3
OV_ERR_UNSUPPORTED = 4
OV_ERR_TIMEOUT = 5
OV_ERR_CANCELLED = 6
OV_ERR_IO = 7

OV_DEVICE_WAIT_TIMEOUT = 1
OV_DEVICE_BAD_ARGUMENT = 2

OV_EPI_STORE_F32 = 0
OV_EPI_ACCUM_F32 = 1
OV_EPI_SWIGLU_F16 = 2
OV_EPI_QKNORM_ROPE_F16 = 3
OV_SWIGLU_GROUP = 64

OV_NOISE_NONE = 0
OV_NOISE_DEVICE = 1
OV_NOISE_BUFFER = 2

OV_GEN_NOISE_REFERENCE = 0
OV_GEN_NOISE_DEVICE = 1


class ModelConfig(Structure):
    _fields_ = [("vocab_size", c_size_t), ("hidden_size", c_size_t),
                ("intermediate_size", c_size_t), ("layers", c_size_t), ("heads", c_size_t),
                ("kv_heads", c_size_t), ("head_dim", c_size_t), ("max_positions", c_size_t),
                ("rms_norm_eps", c_float), ("rope_theta", c_float),
                ("audio_codebooks", c_size_t), ("audio_vocab_size", c_size_t),
                ("audio_mask_id", c_uint32)]


class DecodingConfigC(Structure):
    _fields_ = [("steps", c_size_t), ("guidance", c_float), ("t_shift", c_float),
                ("layer_penalty", c_float), ("position_temperature", c_float)]


class ConditionalInputC(Structure):
    _fields_ = [("codebooks", c_size_t), ("length", c_size_t), ("audio_start", c_size_t),
                ("target_frames", c_size_t), ("ids", POINTER(c_int32))]


class GeneratorStats(Structure):
    _fields_ = [("rows", c_size_t), ("steps_run", c_size_t), ("flops_per_step", ctypes.c_double),
                ("kernels_per_step", c_size_t), ("kernels_per_reset", c_size_t),
                ("h2d_bytes", c_size_t), ("d2h_bytes", c_size_t), ("stream", c_void_p)]


class KernelTime(Structure):
    _fields_ = [("name", ctypes.c_char * 32), ("ms", ctypes.c_double), ("launches", c_size_t),
                ("flops", ctypes.c_double), ("bytes", ctypes.c_double)]


class MatmulShape(Structure):
    _fields_ = [("transpose_a", c_int32), ("transpose_b", c_int32), ("m", c_size_t),
                ("n", c_size_t), ("k", c_size_t), ("lda", c_size_t), ("ldb", c_size_t),
                ("ldc", c_size_t), ("stride_a", c_int64), ("stride_b", c_int64),
                ("stride_c", c_int64), ("batch", c_size_t), ("accumulate", c_int32)]


class EpilogueArgs(Structure):
    _fields_ = [("q_norm", c_void_p), ("k_norm", c_void_p), ("positions", c_void_p),
                ("rope_cos", c_void_p), ("rope_sin", c_void_p), ("max_positions", c_int32),
                ("heads", c_int32), ("kv_heads", c_int32), ("head_dim", c_int32),
                ("epsilon", c_float)]


class CodecConfigC(Structure):
    _fields_ = [("codebooks", c_size_t), ("codebook_size", c_size_t),
                ("codebook_dim", c_size_t), ("semantic_hidden", c_size_t),
                ("latent_channels", c_size_t), ("decoder_channels", c_size_t),
                ("upsampling_ratios", c_size_t * 8), ("num_upsampling", c_size_t),
                ("sample_rate", c_uint32)]

class CodecEncoderConfigC(Structure):
    """ov_codec_encoder_config (include/ov_codec.h)."""
    _fields_ = [("sample_rate", c_uint32), ("codebooks", c_size_t), ("codebook_size", c_size_t),
                ("codebook_dim", c_size_t), ("semantic_sample_rate", c_uint32),
                ("hidden_size", c_size_t), ("intermediate_size", c_size_t), ("heads", c_size_t),
                ("layers", c_size_t), ("position_kernel", c_size_t), ("position_groups", c_size_t),
                ("layer_norm_eps", c_float), ("conv_channels", c_size_t * 8),
                ("conv_kernels", c_size_t * 8), ("conv_strides", c_size_t * 8),
                ("num_convs", c_size_t), ("encoder_channels", c_size_t),
                ("latent_channels", c_size_t), ("downsampling_ratios", c_size_t * 8),
                ("num_downsampling", c_size_t)]


CANCEL_FN = ctypes.CFUNCTYPE(c_int, c_void_p)

_P = c_void_p  # device or host pointer passed as an integer address
_S = c_size_t

# name -> (restype, argtypes); every function declared in include/ov_*.h.
SIGNATURES: dict[str, tuple] = {
    # ov_runtime.h
    "ov_last_error": (c_int, [c_char_p, _S]),
    "ov_device_count": (c_int, [POINTER(c_int)]),
    "ov_set_device": (c_int, [c_int]),
    "ov_get_device": (c_int, [POINTER(c_int)]),
    "ov_device_info": (c_int, [c_int, POINTER(c_int), POINTER(c_int), POINTER(c_int)]),
    "ov_malloc": (c_int, [POINTER(c_void_p), _S]),
    "ov_free": (c_int, [_P]),
    "ov_malloc_host": (c_int, [POINTER(c_void_p), _S]),
    "ov_free_host": (c_int, [_P]),
    "ov_memcpy_h2d_async": (c_int, [_P, _P, _S, _P]),
    "ov_memcpy_d2h_async": (c_int, [_P, _P, _S, _P]),
    "ov_memcpy_d2d_async": (c_int, [_P, _P, _S, _P]),
    "ov_memset_async": (c_int, [_P, c_int, _S, _P]),
    "ov_stream_create": (c_int, [POINTER(c_void_p)]),
    "ov_stream_destroy": (c_int, [_P]),
    "ov_stream_sync": (c_int, [_P]),
    "ov_event_create": (c_int, [POINTER(c_void_p)]),
    "ov_event_destroy": (c_int, [_P]),
    "ov_event_record": (c_int, [_P, _P]),
    "ov_event_sync": (c_int, [_P]),
    "ov_event_elapsed_ms": (c_int, [_P, _P, POINTER(c_float)]),
    "ov_graph_capture_begin": (c_int, [_P]),
    "ov_graph_capture_end": (c_int, [_P, POINTER(c_void_p)]),
    "ov_graph_launch": (c_int, [_P, _P]),
    "ov_graph_destroy": (c_int, [_P]),
    "ov_take_device_errors": (c_int, [POINTER(c_uint32), _P]),
    # ov_kernels.h
    "ov_embed": (c_int, [_P, _S, _P, _P, _S, _P, _S, _S, _S, _P, _P, c_float, _P, _P]),
    "ov_rmsnorm": (c_int, [_P, _P, _P, _S, _S, c_float, _P]),
    "ov_gather_rmsnorm": (c_int, [_P, _P, _S, _P, _P, _S, c_float, _P]),
    "ov_rope_tables": (c_int, [c_float, _S, _S, _P, _P]),
    "ov_qknorm_rope": (c_int, [_P, _S, _P, _P, _P, _P, _P, _S, _S, _S, _S, _S, c_float, _P, _S,
                               _P]),
    "ov_swiglu": (c_int, [_P, _S, _S, _P, _P]),
    "ov_gemm_f16": (c_int, [_P, _S, _P, _P, _S, _S, _S, _S, c_int, POINTER(EpilogueArgs), _P,
                            _S, _P]),
    "ov_gemm_workspace_bytes": (c_size_t, [_S, _S, _S, c_int]),
    "ov_interleave_gate_up": (c_int, [_P, _S, _S, _P]),
    "ov_matmul_f16": (c_int, [POINTER(MatmulShape), _P, _P, _P, _P]),
    "ov_gemm_f16_noalloc": (c_int, [_P, _S, _P, _P, _S, _S, _S, _S, c_int, POINTER(EpilogueArgs),
                                    _P]),
    "ov_attention_varlen": (c_int, [_P, _S, _S, _P, _S, _S, _S, _S, _S, c_float, _P, _S, _P]),
    "ov_attention_varlen_items": (c_int, [_P, _S, _S, _P, _S, _S, _P, _S, c_int, _S, _S, _S,
                                          c_float, _P, _S, _P]),
    "ov_score": (c_int, [_P, _S, _S, _S, _S, c_uint32, c_float, _P, _P, _P]),
    "ov_select_positions": (c_int, [_P, _P, _S, _S, _S, c_float, c_float, c_int, _P, c_uint64,
                                    c_int32, c_uint32, _P, _P, _P, _S, _S, _S, _P]),
    "ov_gumbel_from_uniform": (c_float, [c_float]),
    "ov_synthetic_fill": (c_int, [_P, _S, c_uint64, c_uint64, c_float, c_uint64, _P]),
    "ov_synthetic_fill_host": (c_int, [_P, _S, c_uint64, c_uint64, c_float, c_uint64]),
    # ov_generator.h
    "ov_default_model_config": (None, [POINTER(ModelConfig)]),
    "ov_default_decoding_config": (None, [POINTER(DecodingConfigC)]),
    "ov_generator_load": (c_int, [POINTER(ModelConfig), c_char_p, c_int, POINTER(c_void_p)]),
    "ov_generator_create_synthetic": (c_int, [POINTER(ModelConfig), c_uint64, c_int,
                                              POINTER(c_void_p)]),
    "ov_generator_destroy": (None, [_P]),
    "ov_generator_forward": (c_int, [_P, POINTER(ConditionalInputC), _P]),
    "ov_generator_score": (c_int, [_P, POINTER(ConditionalInputC), c_float, _P, _P]),
    "ov_generator_generate": (c_int, [_P, POINTER(ConditionalInputC), POINTER(DecodingConfigC),
                                      c_uint64, c_int, CANCEL_FN, _P, _P, _P]),
    "ov_generator_generate_batch": (c_int, [_P, POINTER(ConditionalInputC), _S,
                                            POINTER(DecodingConfigC), POINTER(c_uint64), c_int,
                                            CANCEL_FN, _P, POINTER(c_void_p), POINTER(c_void_p)]),
    "ov_generator_prepare": (c_int, [_P, POINTER(ConditionalInputC), _S,
                                     POINTER(DecodingConfigC), POINTER(c_uint64), c_int]),
    "ov_generator_run": (c_int, [_P, CANCEL_FN, _P]),
    "ov_generator_fetch": (c_int, [_P, POINTER(c_void_p), POINTER(c_void_p)]),
    "ov_generator_stats_get": (c_int, [_P, POINTER(GeneratorStats)]),
    "ov_generator_profile_step": (c_int, [_P, POINTER(KernelTime), _S, POINTER(c_size_t)]),
    "ov_unmask_schedule": (c_int, [_S, _S, c_float, POINTER(c_size_t)]),
    "ov_build_conditional_input": (c_size_t, [POINTER(c_uint32), _S, POINTER(c_int32), _S, _S,
                                              _S, c_uint32, POINTER(c_int32)]),
    # ov_codec.h
    "ov_codec_default_config": (None, [POINTER(CodecConfigC)]),
    "ov_codec_load": (c_int, [POINTER(CodecConfigC), c_char_p, c_int, POINTER(c_void_p)]),
    "ov_codec_create_synthetic": (c_int, [POINTER(CodecConfigC), c_uint64, c_int,
                                          POINTER(c_void_p)]),
    "ov_codec_free": (None, [_P]),
    "ov_codec_frame_samples": (c_size_t, [_P]),
    "ov_codec_decode": (c_int, [_P, _P, _S, _P]),
    "ov_codec_decode_device": (c_int, [_P, _P, _S, _P, _P]),
    "ov_codec_encoder_default_config": (None, [POINTER(CodecEncoderConfigC)]),
    "ov_codec_encoder_load": (c_int, [POINTER(CodecEncoderConfigC), c_char_p, c_int,
                                      POINTER(c_void_p)]),
    "ov_codec_encoder_create_synthetic": (c_int, [POINTER(CodecEncoderConfigC), c_uint64, c_int,
                                                  POINTER(c_void_p)]),
    "ov_codec_encoder_free": (None, [_P]),
    "ov_codec_encoder_frame_samples": (c_size_t, [_P]),
    "ov_codec_encode": (c_int, [_P, _P, _S, _P, _S, POINTER(c_size_t)]),
}

_lib: ctypes.CDLL | None = None


class OmniVoiceError(RuntimeError):
    """A non-zero status from the library, with its message."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def lib() -> ctypes.CDLL:
    """Loads the native library once; raises if it was not built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run `python -m omnivoice_b200.build` "
                               "(there is no CPU fallback)")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = handle
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(4096)
    lib().ov_last_error(buf, len(buf))
    return buf.value.decode("utf-8", "replace")


def check(status: int) -> None:
    if status != OV_OK:
        raise OmniVoiceError(status, last_error())


def default_model_config() -> ModelConfig:
    cfg = ModelConfig()
    lib().ov_default_model_config(ctypes.byref(cfg))
    return cfg


def default_decoding_config() -> DecodingConfigC:
    cfg = DecodingConfigC()
    lib().ov_default_decoding_config(ctypes.byref(cfg))
    return cfg
