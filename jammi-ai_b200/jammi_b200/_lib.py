"""ctypes binding of libjammi_b200.so (the C ABI in include/jammi_b200.h).

Loading fails loudly when the library is missing: there is no fallback path.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("JAMMI_B200_LIB", os.path.join(_HERE, "libjammi_b200.so"))

# jb_status
OK, ERR_OOM, ERR_INVALID, ERR_CUDA, ERR_TIMEOUT, ERR_SEQ_TOO_LONG, ERR_IO, ERR_NO_DEVICE = range(8)
STATUS_NAMES = {0: "OK", 1: "OOM", 2: "INVALID", 3: "CUDA", 4: "TIMEOUT", 5: "SEQ_TOO_LONG",
                6: "IO", 7: "NO_DEVICE"}
# jb_format
FMT_F32, FMT_BF16, FMT_INT8, FMT_F16 = 0, 1, 2, 3
FORMATS = {"f32": FMT_F32, "bf16": FMT_BF16, "int8": FMT_INT8, "f16": FMT_F16}
# jb_pooling
POOL_MEAN, POOL_CLS, POOL_MAX, POOL_WEIGHTED_MEAN = 0, 1, 2, 3
# jb_dtype
DT_F32, DT_BF16, DT_S8, DT_S32, DT_F16 = 0, 1, 2, 3, 4
# jb_epilogue
EPI_NONE, EPI_GELU, EPI_QUICK_GELU, EPI_RESIDUAL = 0, 1, 2, 3
# jb_family
FAMILY_BERT, FAMILY_CLIP_VISION, FAMILY_CLIP_TEXT = 0, 1, 2
TEXT_BERT, TEXT_DISTILBERT, TEXT_MODERNBERT = 0, 1, 2


class JbError(RuntimeError):
    """A non-OK jb_status with the library's message.  OOM messages contain
    "out of memory", matching the reference's OOM classifier
    (crates/jammi-ai/src/inference/runner.rs:243-256)."""

    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")


class ModelInfo(ctypes.Structure):
    _fields_ = [("family", ctypes.c_int32), ("format", ctypes.c_int32), ("device", ctypes.c_int32),
                ("hidden", ctypes.c_int32), ("output_dim", ctypes.c_int32), ("layers", ctypes.c_int32),
                ("heads", ctypes.c_int32), ("ffn", ctypes.c_int32), ("max_seq", ctypes.c_int32),
                ("image_size", ctypes.c_int32), ("weight_bytes", ctypes.c_int64),
                ("projection_rank", ctypes.c_int32), ("variant", ctypes.c_int32),
                ("preprocess_mean", ctypes.c_float * 3), ("preprocess_std", ctypes.c_float * 3)]


_lib = None

# (name, restype, argtypes)
_P = ctypes.c_void_p
_I = ctypes.c_int
_SIGS = [
    ("jb_last_error", ctypes.c_char_p, []),
    ("jb_model_load", _I, [ctypes.c_char_p, ctypes.c_char_p, _I, _I, ctypes.POINTER(_P)]),
    ("jb_model_load_family", _I, [ctypes.c_char_p, ctypes.c_char_p, _I, _I, _I, ctypes.POINTER(_P)]),
    ("jb_tokenizer_load", _I, [ctypes.c_char_p, ctypes.POINTER(_P)]),
    ("jb_tokenizer_load_clip_bpe", _I, [ctypes.c_char_p, ctypes.POINTER(_P)]),
    ("jb_tokenize_rows", _I, [_P, _P, _P, ctypes.c_int64, _I, _P, ctypes.c_uint64, _P]),
    ("jb_tokenizer_free", None, [_P]),
    ("jb_tokenize", _I, [_P, _P, _P, ctypes.c_int64, _I, _P, ctypes.c_uint64, _P]),
    ("jb_model_free", None, [_P]),
    ("jb_model_get_info", _I, [_P, ctypes.POINTER(ModelInfo)]),
    ("jb_estimate_batch_bytes", ctypes.c_size_t, [_P, _I, _I]),
    ("jb_model_sync", _I, [_P, _P]),
    ("jb_model_profile_enable", _I, [_P, _I]),
    ("jb_model_set_projection_head", _I, [_P, _P, _P, _I, ctypes.c_double]),
    ("jb_model_load_projection_head", _I, [_P, ctypes.c_char_p, ctypes.c_double]),
    ("jb_model_set_lora", _I, [_P, _I, _I, _P, _P, _I, ctypes.c_double]),
    ("jb_model_load_lora", _I, [_P, ctypes.c_char_p, ctypes.c_double, _I, _P]),
    ("jb_model_profile_read", _I, [_P, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int32)]),
    ("jb_encode_text", _I, [_P, _P, _P, _I, _I, _I, _P, _P]),
    ("jb_encode_text_device", _I, [_P, _P, _P, _I, _I, _I, _P, _P]),
    ("jb_encode_text_device_noalloc", _I, [_P, _P, _P, _I, _I, _I, _P, _P]),
    ("jb_forward_hidden_device", _I, [_P, _P, _P, _I, _I, _P, _P]),
    ("jb_encode_image", _I, [_P, _P, _I, _P, _P]),
    ("jb_encode_image_rgb8", _I, [_P, _P, ctypes.c_size_t, _P, _P, _P, _I, _P, _P]),
    ("jb_op_preprocess_rgb8", _I, [_P, _P, _P, _P, _I, _I, _I, _P, _P, _P, _P]),
    ("jb_encode_image_device", _I, [_P, _P, _I, _P, _P]),
    ("jb_op_sync", _I, [_P]),
    ("jb_op_linear", _I, [_P, _I, _P, _I, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    ("jb_op_linear_s8", _I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    ("jb_op_quantize_rows", _I, [_P, _I, _P, _P, _I, _I, _P]),
    ("jb_op_quantize_rows_act", _I, [_P, _I, _I, _P, _P, _I, _I, _P]),
    ("jb_op_layernorm", _I, [_P, _P, _P, _P, _P, _I, _I, _I, ctypes.c_float, _P]),
    ("jb_op_attention", _I, [_P, _P, _P, _I, _I, _I, _I, _I, _P]),
    ("jb_op_attention_causal", _I, [_P, _P, _P, _I, _I, _I, _I, _I, _P]),
    ("jb_op_attention_rows", _I, [_P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P]),
    ("jb_set_attention_tcgen05", None, [_I]),
    ("jb_op_pool_normalize", _I, [_P, _I, _P, _P, _I, _I, _I, _P]),
    ("jb_op_wait_flag", _I, [_P, _I, _I, _P]),
    ("jb_pooling_from_config", _I, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_int)]),
    ("jb_pooling_from_model_dir", _I, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_int)]),
    ("jb_op_fit_binary_threshold", _I, [_P, ctypes.c_int64, _I, _I, _P, _P]),
    ("jb_op_pack_threshold_bits", _I, [_P, ctypes.c_int64, _I, _P, _P, _P]),
    ("jb_op_exact_search", _I, [_P, ctypes.c_int64, _I, _P, _P, _I, _I, _P, _P, _P, _P]),
    ("jb_sidecar_create", _I, [_I, _I, _I, ctypes.POINTER(_P)]),
    ("jb_sidecar_add", _I, [_P, _P, _P, ctypes.c_int64, _P, _P]),
    ("jb_sidecar_build", _I, [_P, _I, _P]),
    ("jb_sidecar_len", ctypes.c_int64, [_P]),
    ("jb_sidecar_search", _I, [_P, _P, _I, _I, _P, _P]),
    ("jb_sidecar_search_final", _I, [_P, _P, _I, _I, _I, _P, _P]),
    ("jb_sidecar_export", _I, [_P, _P, _P, _P]),
    ("jb_sidecar_free", None, [_P]),
    ("jb_scheduler_new", _P, [ctypes.c_uint64, ctypes.c_double]),
    ("jb_scheduler_new_unlimited", _P, []),
    ("jb_scheduler_for_device", _P, [_I, ctypes.c_double]),
    ("jb_scheduler_free", None, [_P]),
    ("jb_scheduler_is_unlimited", _I, [_P]),
    ("jb_scheduler_available", ctypes.c_uint64, [_P]),
    ("jb_scheduler_try_acquire", _I, [_P, ctypes.c_uint64]),
    ("jb_scheduler_acquire", _I, [_P, ctypes.c_uint64, _I, ctypes.c_int64]),
    ("jb_scheduler_release", None, [_P, ctypes.c_uint64]),
    ("jb_is_oom_message", _I, [ctypes.c_char_p]),
    ("jb_run_chunks", _I, [ctypes.c_int64, ctypes.POINTER(ctypes.c_int), _P, _P]),
    ("jb_generate_embeddings", _I, [_P, _I, _P, _P, ctypes.c_int64, _P, _P, _P, _P]),
]


def lib():
    """The loaded library (loaded on first use)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"libjammi_b200.so not built (expected at {LIB_PATH}); "
                              "run `make -C jammi-ai_b200` or __graft_entry__.build()")
        handle = ctypes.CDLL(LIB_PATH)
        for name, res, args in _SIGS:
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def exported_symbols():
    return [name for name, _, _ in _SIGS]


def check(status: int):
    if status != OK:
        msg = lib().jb_last_error()
        raise JbError(status, msg.decode() if msg else "")
