"""ctypes binding of libdecisive_b200.so (include/decisive_b200.h).

Loading fails loudly: there is no CPU fallback for any entry point.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdecisive_b200.so")

# entry points declared in include/decisive_b200.h: (name, restype, argtypes)
_vp, _sz, _i64, _i32, _f = C.c_void_p, C.c_size_t, C.c_int64, C.c_int, C.c_float
_fp = C.POINTER(C.c_float)


class DbError(C.Structure):
    _fields_ = [("code", C.c_char * 32), ("message", C.c_char * 224)]


class EncoderConfig(C.Structure):
    _fields_ = [("layers", C.c_int32), ("hidden", C.c_int32), ("q_heads", C.c_int32), ("kv_heads", C.c_int32),
                ("head_dim", C.c_int32), ("ffn", C.c_int32), ("vocab", C.c_int32), ("weight_bits", C.c_int32),
                ("rope_theta", C.c_float), ("eps", C.c_float), ("max_sequence_tokens", C.c_int32),
                ("fused", C.c_int32), ("causal", C.c_int32)]


class BertConfig(C.Structure):
    _fields_ = [("layers", C.c_int32), ("hidden", C.c_int32), ("heads", C.c_int32), ("ffn", C.c_int32),
                ("vocab", C.c_int32), ("max_positions", C.c_int32), ("block", C.c_int32), ("eps", C.c_float),
                ("fused", C.c_int32), ("mode", C.c_int32)]


class Parameters(C.Structure):
    _fields_ = [("max_sequence_tokens", C.c_int32)]


_u16pp = C.POINTER(C.POINTER(C.c_uint16))
_fpp = C.POINTER(C.POINTER(C.c_float))


class EncoderWeights(C.Structure):
    _fields_ = [("embedding", C.POINTER(C.c_uint16))] + \
               [(n, _u16pp) for n in ("q", "k", "v", "o", "gate", "up", "down")] + \
               [(n, _fpp) for n in ("input_norm", "post_norm", "q_norm", "k_norm")] + \
               [("final_norm", C.POINTER(C.c_float))]


SIGNATURES = [
    ("db_abi_version", _i32, []),
    ("db_scale_row_stride", _i64, [_i64]),
    ("db_last_error_code", C.c_char_p, []),
    ("db_last_error_message", C.c_char_p, []),
    ("db_device_count", _i32, []),
    ("db_device_error_word", _i32, []),
    ("db_quantize_activations_g64", _i32, [_vp, _i32, _i64, _i64, _i64, _i32, _vp, _i32, _i64, _vp, _vp, _i64, _vp, _vp]),
    ("db_pack_weights_g64", _i32, [_vp, _i64, _i64, _i32, _vp, _vp, _vp]),
    ("db_import_packed", _i32, [_vp, _i64, _i64, _i32, _vp, _vp, _vp]),
    ("db_export_packed", _i32, [_vp, _vp, _i64, _i64, _i32, _vp, _vp]),
    ("db_dequant_rows_g64", _i32, [_vp, _vp, _i64, _i64, _i32, _vp, _i64, _vp, _i64, _vp]),
    ("db_gemm_g64", _i32, [_vp, _i32, _i64, _vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _i32, _i32, _i32, _vp, _i64,
                           _vp, _vp]),
    ("db_gemm_g64_config", _i32, [_vp, _i32, _i64, _vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _i32, _i32, _i32, _vp,
                                  _i64, _vp, _vp, _vp]),
    ("db_gemv_max_rows", _i32, []),
    ("db_decima_quantize_weights", _i32, [_vp, _i64, _i64, _i32, _vp, _vp, _vp]),
    ("db_decima_quantize_activations", _i32, [_vp, _i64, _i64, _i32, _vp, _i32, _i64, _vp, _i64, _vp, _vp]),
    ("db_decima_workspace_bytes", _sz, [_i64, _i64, _i32]),
    ("db_decima_linear", _i32, [_vp, _i64, _i64, _vp, _vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp]),
    ("db_decima_linear_w8a32", _i32, [_vp, _i64, _i64, _vp, _vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp]),
    ("db_gemm_tune", _i32, [_i64, _i64, _i64, _i32, _i32, C.c_char_p, _vp, C.c_char_p, _sz]),
    ("db_linear_workspace_bytes", _sz, [_i64, _i64]),
    ("db_linear_g64", _i32, [_vp, _i64, _i64, _vp, _vp, _i64, _i32, _i32, _i32, _vp, _vp, _vp]),
    ("db_linear_noalloc_scratch_bytes", _sz, []),
    ("db_linear_g64_noalloc", _i32, [_vp, _i64, _i64, _vp, _vp, _i64, _i32, _i32, _i32, _vp, _vp]),
    ("db_linear_noalloc_error_word", _i32, []),
    ("db_project_packed", _i32, [_vp, _i64, _vp, _vp, _i64, _i32, _vp, _vp, _vp]),
    ("db_mlp_g64", _i32, [_vp, _i64, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _i32, _i32, _vp, _i64, _vp, _i64, _vp, _vp]),
    ("db_mlp_g64_natural", _i32, [_vp, _i64, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _i32, _i32, _vp, _i64, _vp, _i64, _vp, _vp]),
    ("db_interleave_gate_up", _i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i32, _vp, _vp, _vp]),
    ("db_attention", _i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _f, _vp, _i64, _vp]),
    ("db_attention_decoder", _i32, [_vp, _vp, _vp, _i64, _i64, _vp, _vp, _i64, C.c_int, _i64, _i64, _i64, _f, _vp,
                                    _i64, _vp]),
    ("db_synthetic_bf16", _i32, [C.c_uint64, C.c_uint64, _i64, _f, _vp, _vp]),
    ("db_model_create", _vp, [_i32, C.POINTER(EncoderConfig), C.POINTER(EncoderWeights), C.POINTER(DbError)]),
    ("db_model_create_synthetic", _vp, [_i32, C.POINTER(EncoderConfig), C.c_uint64, _f, C.POINTER(DbError)]),
    ("db_model_synthetic_weight", _i64, [_vp, C.c_char_p, _i32, _vp, _i64]),
    ("db_model_destroy", None, [_vp]),
    ("db_model_capabilities", _i32, [_vp, C.c_char_p, _sz]),
    ("db_cache_create", _vp, [_vp, _sz, _i32, C.POINTER(DbError)]),
    ("db_cache_clear", _i32, [_vp, _vp, C.POINTER(DbError)]),
    ("db_cache_destroy", None, [_vp]),
    ("db_predict", _i32, [_vp, _vp, _sz, C.POINTER(Parameters), _vp, _vp, _vp, C.POINTER(DbError)]),
    ("db_predict_batch", _i32, [_vp, _vp, _vp, _sz, C.POINTER(Parameters), _vp, _vp, _vp, _vp, _vp,
                                C.POINTER(DbError)]),
    ("db_forward_device", _i32, [_vp, _vp, _i64, _vp, _vp]),
    ("db_bert_create_synthetic", _vp, [_i32, C.POINTER(BertConfig), C.c_uint64, _f, C.POINTER(DbError)]),
    ("db_bert_destroy", None, [_vp]),
    ("db_bert_predict", _i32, [_vp, _vp, _sz, _vp, _vp, C.POINTER(DbError)]),
    ("db_bert_score", _i32, [_vp, _vp, _sz, _vp, _vp, _sz, _vp, _vp, C.POINTER(DbError)]),
    ("db_predict_continuations", _i32, [_vp, _vp, _vp, _sz, _vp, _sz, _sz, _vp, _vp, C.POINTER(DbError)]),
    ("db_score_continuations", _i32, [_vp, _vp, _vp, _sz, _vp, _sz, _sz, _vp, _vp, _vp, C.POINTER(DbError)]),
    ("db_cache_stats", _i32, [_vp, _vp, _vp, _vp]),
    ("db_model_profile", _i32, [_vp, _i32]),
    ("db_model_set_code_layout", _i32, [_vp, _i32]),
    ("db_model_use_graphs", _i32, [_vp, _i32]),
    ("db_model_export_packed", _i32, [_vp, C.c_char_p, C.POINTER(DbError)]),
    ("db_model_set_streaming", _i32, [_vp, _i32, C.POINTER(DbError)]),
    ("db_model_create_packed", _vp, [_i32, C.POINTER(EncoderConfig), C.c_char_p, _i32, C.POINTER(DbError)]),
    ("db_model_tune", _i32, [_vp, _i64, C.c_char_p, C.c_char_p, _sz, C.POINTER(DbError)]),
    ("db_model_profile_read", _i32, [_vp, _vp, _vp, _i32, _i32]),
    ("db_model_profile_name", C.c_char_p, [_i32]),
]

_lib = None


def load(path: str = LIB_PATH):
    """Load the library; raises if it is missing (no fallback path exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(f"decisive_b200: CUDA library not built ({path}); run `python -m decisive_b200.build`")
    lib = C.CDLL(path)
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def last_error() -> tuple[str, str]:
    lib = load()
    return lib.db_last_error_code().decode(), lib.db_last_error_message().decode()


class CudaError(RuntimeError):
    def __init__(self, status: int):
        code, msg = last_error()
        super().__init__(f"{code}: {msg} (status {status})")
        self.status, self.code, self.msg = status, code, msg


def check(status: int) -> None:
    if status != 0:
        raise CudaError(status)
