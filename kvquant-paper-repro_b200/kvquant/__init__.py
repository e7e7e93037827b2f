"""kvquant -- B200 (sm_100a) build of KVQuant's decode-time quantized-KV path.

Mirrors the reference package's public API for this path; the calibration,
sensitivity, model-loading and perplexity tooling of the reference are not
part of this package.
"""
from .quant.kv_quantizer import KVQuantizer
from .attention_patch import patch_model, unpatch_model
from .kv_cache import QuantizedKVCache

__all__ = [
    "KVQuantizer",
    "patch_model",
    "unpatch_model",
    "QuantizedKVCache",
]
