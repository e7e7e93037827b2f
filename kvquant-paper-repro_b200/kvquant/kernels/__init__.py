"""kvquant.kernels -- the reference's kernel host API backed by sm_100a kernels."""
from .rope_fused import apply_rope_elementwise, apply_rope_inplace, rope_inv_freq
from .matvec_ds import dense_matvec_lut, sparse_matvec, sparse_matvec_csr
from .cuda_ops import get_cuda_ops, cuda_available
from .decode import (quantize_keys, quantize_values, qk_scores, qk_scores_stats, softmax,
                     pv_out, pv_out_scores, decode_attention, make_appendable, append_keys,
                     append_values, key_outlier_thresholds, decode_attention_shard,
                     merge_shards, set_decode_kernels)

__all__ = [
    "apply_rope_elementwise",
    "apply_rope_inplace",
    "dense_matvec_lut",
    "sparse_matvec",
    "sparse_matvec_csr",
    "get_cuda_ops",
    "cuda_available",
    "rope_inv_freq",
    "quantize_keys",
    "quantize_values",
    "qk_scores",
    "qk_scores_stats",
    "softmax",
    "pv_out",
    "pv_out_scores",
    "decode_attention",
    "make_appendable",
    "append_keys",
    "append_values",
    "key_outlier_thresholds",
    "decode_attention_shard",
    "merge_shards",
    "set_decode_kernels",
]
