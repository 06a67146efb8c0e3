"""LEMA (latest exact match attention) inference hot path for NVIDIA B200 (sm_100a).

A from-scratch B200 implementation of the inference path of
moritzbroe/latest_exact_match_attention, behind the same interfaces as its `code/lema`
package:

    attention   pack_codes, latest_prev_match, lema_hard      (code/lema/attention.py)
    cache       HashStore, LayerStore, LemaCache (in HBM)      (code/lema/cache.py)
    model       ModelConfig, Transformer, Block, Attention     (code/lema/model.py)
    decode      decoder, LemaDecoder (one CUDA graph per step) (code/lema/decode.py)

The kernels live in liblema_b200.so (C ABI: include/lema_b200.h), built by `build.py`.
"""
from .attention import (latest_prev_match, lema_hard, pack_codes, prefill_match,  # noqa: F401
                        proj_codes)
from ._lib import LemaError  # noqa: F401
from .model import ModelConfig, Transformer  # noqa: F401
from .decode import LemaDecoder, decoder  # noqa: F401

__version__ = "0.1.0"
