"""ctypes binding of libmarian_cuda.so (declared in include/marian_cuda.h).

The library is the product; there is no fallback.  If it is missing or was
not built for this machine, loading raises, and every caller fails loudly.
"""
from __future__ import annotations

import ctypes as C
import os

from . import build as _build

MC_OK, MC_INVALID_INPUT, MC_MODEL, MC_INFERENCE, MC_DEVICE_TIMEOUT, MC_CUDA = range(6)
STATUS_NAMES = {0: "OK", 1: "INVALID_INPUT", 2: "MODEL", 3: "INFERENCE", 4: "DEVICE_TIMEOUT", 5: "CUDA"}

# Every symbol include/marian_cuda.h declares.
EXPORTS = [
    "mc_config_default", "mc_create", "mc_load_marian_bin", "mc_model_info_get", "mc_destroy",
    "mc_last_error", "mc_is_ready", "mc_translate_token_ids", "mc_submit", "mc_step", "mc_poll",
    "mc_trace_first_step", "mc_stream", "mc_q8_gemm", "mc_op_status", "mc_profile",
    "mc_profile_read", "mc_launch_count", "mc_q8_linear", "mc_q8_linear_noalloc", "mc_q8_linear_ln", "mc_load_shortlist",
    "mc_segment_text", "mc_timeline", "mc_timeline_read", "mc_inspect_marian_bin",
    "mc_encode_token_ids", "mc_replay",
]

# MC_Q8_LINEAR_NOALLOC_MAX_ACTIVATIONS in include/marian_cuda.h
NOALLOC_MAX_ACTIVATIONS = 8 * 1024 * 1024

KERNEL_KINDS = ["embed", "gemm_qkv", "gemm_out", "gemm_ffn1", "gemm_ffn2", "gemm_crosskv",
                "gemm_vocab", "attn_enc", "attn_self", "attn_cross", "layernorm", "ssru", "finalize", "gemm_ln"]


class Config(C.Structure):
    _fields_ = [("device", C.c_int32), ("max_inflight", C.c_uint32), ("max_encode_tokens", C.c_uint32),
                ("page_tokens", C.c_uint32), ("kv_pages", C.c_uint32), ("max_length_factor", C.c_uint32),
                ("lanes", C.c_uint32)]


class TextSegment(C.Structure):
    _fields_ = [("content_start", C.c_uint64), ("content_end", C.c_uint64),
                ("separator_start", C.c_uint64), ("separator_end", C.c_uint64),
                ("source_pieces", C.c_uint64)]


class SegmentError(C.Structure):
    _fields_ = [("kind", C.c_int32), ("start", C.c_uint64), ("end", C.c_uint64),
                ("pieces", C.c_uint64), ("maximum", C.c_uint64), ("message", C.c_char * 256)]


# mc_piece_count_fn
PIECE_COUNT_FN = C.CFUNCTYPE(C.c_int32, C.c_void_p, C.POINTER(C.c_char), C.c_size_t,
                             C.POINTER(C.c_uint64), C.POINTER(C.c_char), C.c_size_t)


class ModelInfo(C.Structure):
    _fields_ = [("dim", C.c_int32), ("heads", C.c_int32), ("ffn_dim", C.c_int32),
                ("encoder_layers", C.c_int32), ("decoder_layers", C.c_int32),
                ("decoder_kind", C.c_int32), ("source_vocab", C.c_int32),
                ("target_vocab", C.c_int32), ("weight_bytes", C.c_uint64)]


class ModelReport(C.Structure):
    _fields_ = [("tensors", C.c_uint64), ("dense_linears", C.c_uint64), ("embeddings", C.c_uint64),
                ("activation_scales", C.c_uint64), ("row_scaled_linears", C.c_uint64),
                ("decoder_output_alpha", C.c_float), ("engine_graph", C.c_int32),
                ("decoder_kind", C.c_int32), ("dim", C.c_int32), ("heads", C.c_int32),
                ("encoder_layers", C.c_int32), ("decoder_layers", C.c_int32)]


class MarianCudaError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


_lib = None


def load(build_if_missing: bool = True):
    global _lib
    if _lib is not None:
        return _lib
    if build_if_missing and not os.path.exists(_build.LIB):
        _build.build()
    raw = C.CDLL(_build.LIB)

    lib = raw
    vp, sz, u32, i32, u64 = C.c_void_p, C.c_size_t, C.c_uint32, C.c_int32, C.c_uint64
    missing = [n for n in EXPORTS if not hasattr(raw, n)]
    if missing:
        for n in missing:
            setattr(raw, n, None)
    if getattr(raw, 'mc_config_default', None) is not None: lib.mc_config_default.argtypes = [C.POINTER(Config)]
    if getattr(raw, 'mc_config_default', None) is not None: lib.mc_config_default.restype = None
    if getattr(raw, 'mc_create', None) is not None: lib.mc_create.argtypes = [C.POINTER(Config), C.POINTER(vp)]
    if getattr(raw, 'mc_load_marian_bin', None) is not None: lib.mc_load_marian_bin.argtypes = [vp, C.c_char_p, sz]
    if getattr(raw, 'mc_model_info_get', None) is not None: lib.mc_model_info_get.argtypes = [vp, C.POINTER(ModelInfo)]
    if getattr(raw, 'mc_destroy', None) is not None: lib.mc_destroy.argtypes = [vp]
    if getattr(raw, 'mc_destroy', None) is not None: lib.mc_destroy.restype = None
    if getattr(raw, 'mc_last_error', None) is not None: lib.mc_last_error.argtypes = [vp, C.c_char_p, sz]
    if getattr(raw, 'mc_last_error', None) is not None: lib.mc_last_error.restype = sz
    if getattr(raw, 'mc_is_ready', None) is not None: lib.mc_is_ready.argtypes = [vp]
    if getattr(raw, 'mc_is_ready', None) is not None: lib.mc_is_ready.restype = i32
    if getattr(raw, 'mc_translate_token_ids', None) is not None: lib.mc_translate_token_ids.argtypes = [vp, vp, sz, vp, u32, vp, vp, vp, sz, vp]
    if getattr(raw, 'mc_submit', None) is not None: lib.mc_submit.argtypes = [vp, u64, vp, u32, u32, u32]
    if getattr(raw, 'mc_step', None) is not None: lib.mc_step.argtypes = [vp, C.POINTER(u32), C.POINTER(u32)]
    if getattr(raw, 'mc_poll', None) is not None: lib.mc_poll.argtypes = [vp, vp, vp, u32, vp, sz, C.POINTER(u32)]
    if getattr(raw, 'mc_trace_first_step', None) is not None: lib.mc_trace_first_step.argtypes = [vp, vp, sz, vp, u32, vp, vp, vp, vp]
    if getattr(raw, 'mc_stream', None) is not None: lib.mc_stream.argtypes = [vp]
    if getattr(raw, 'mc_stream', None) is not None: lib.mc_stream.restype = vp
    if getattr(raw, 'mc_q8_gemm', None) is not None: lib.mc_q8_gemm.argtypes = [vp, vp, i32, i32, i32, vp, vp, vp, vp, i32, i32, vp, vp]
    if getattr(raw, 'mc_op_status', None) is not None: lib.mc_op_status.argtypes = [C.POINTER(u32)]
    lib.mc_q8_linear.argtypes = [vp, i32, i32, vp, i32, C.c_float, C.c_float, vp, vp, vp]
    lib.mc_q8_linear_ln.argtypes = [vp, i32, i32, vp, i32, C.c_float, C.c_float, vp, vp, vp, vp, vp, vp,
                                    C.c_float, vp]
    lib.mc_q8_linear_noalloc.argtypes = [vp, i32, i32, vp, i32, C.c_float, C.c_float, vp, vp, vp,
                                         C.POINTER(u32)]
    lib.mc_profile.argtypes = [vp, i32]
    lib.mc_profile_read.argtypes = [vp, i32, C.POINTER(u64), C.POINTER(C.c_double),
                                    C.POINTER(C.c_double), C.POINTER(C.c_double)]
    lib.mc_load_shortlist.argtypes = [vp, C.c_char_p, sz]
    lib.mc_segment_text.argtypes = [C.c_char_p, sz, u64, PIECE_COUNT_FN, vp, C.POINTER(TextSegment), sz,
                                    C.POINTER(sz), C.POINTER(SegmentError)]
    lib.mc_timeline.argtypes = [vp, i32]
    lib.mc_timeline_read.argtypes = [vp, C.POINTER(u64), C.POINTER(C.c_double), C.POINTER(C.c_double)]
    lib.mc_encode_token_ids.argtypes = [vp, vp, sz, vp, u32, vp]
    lib.mc_replay.argtypes = [vp, vp, sz, vp, u32, vp, vp, vp, vp]
    lib.mc_inspect_marian_bin.argtypes = [C.c_char_p, sz, C.POINTER(ModelReport), C.c_char_p, sz]
    lib.mc_launch_count.argtypes = [vp]
    lib.mc_launch_count.restype = u64
    _lib = lib
    return lib


def check(status, engine=None):
    if status != MC_OK:
        msg = ""
        if engine:
            buf = C.create_string_buffer(1024)
            load().mc_last_error(engine, buf, 1024)
            msg = buf.value.decode(errors="replace")
        raise MarianCudaError(status, msg)
