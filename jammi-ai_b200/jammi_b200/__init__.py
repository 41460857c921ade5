"""jammi_b200: B200 (sm_100a) embedding-generation library -- Python loader.

The compute lives in ``libjammi_b200.so`` (hand-written CUDA for sm_100a
behind the C ABI of ``include/jammi_b200.h``); this package binds it with
ctypes and mirrors the reference's encoder surface for tests and benchmarks.
"""
from ._lib import (JbError, LIB_PATH, lib, check, FMT_F32, FMT_BF16, FMT_INT8, FMT_F16,  # noqa: F401
                   POOL_MEAN, POOL_CLS, POOL_MAX, POOL_WEIGHTED_MEAN,
                   EPI_NONE, EPI_GELU, EPI_QUICK_GELU, EPI_RESIDUAL)
from .tokenizer import Tokenizer  # noqa: F401
from .encoders import (Bert, Model, OpenClipText, OpenClipVisionTransformer, SequenceTooLong,  # noqa: F401
                       load_model, mask_to_lengths)
