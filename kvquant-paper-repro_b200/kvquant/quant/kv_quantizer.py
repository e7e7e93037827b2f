"""KVQuantizer (drop-in for kvquant/quant/kv_quantizer.py).

Same constructor and methods. quantize_k / quantize_v return the reference's
fake-quant output (quantize, then dequantize to the input dtype) computed by
the sm_100a quantize kernels; on the same inputs the result equals the
reference's bit for bit, except where torch.topk's unspecified order among
equal |n| at the top-k threshold picks a different position (the kernels take
the lower index). pack_k / pack_v return the packed cache dict instead.
"""
from __future__ import annotations

import torch

from ..kernels.cuda_ops import get_cuda_ops
from ..kernels.decode import quantize_keys, quantize_values


def _lut_lookup(x_norm: torch.Tensor, codebook: torch.Tensor):
    """Nearest centroid (first minimum) on the GPU; kv_quantizer.py:7-21."""
    if not x_norm.is_cuda:
        raise RuntimeError("_lut_lookup: kvquant_b200 runs on CUDA tensors only")
    cb = codebook.to(x_norm.device, dtype=torch.float32).reshape(-1).contiguous()
    idx, dq = get_cuda_ops().lut_lookup(x_norm.reshape(-1).float(), cb)
    return idx.reshape(x_norm.shape), dq.reshape(x_norm.shape)


class KVQuantizer:
    def __init__(
        self,
        k_codebooks,
        v_codebooks,
        k_scales,
        k_zeros,
        k_bits: int = 3,
        v_bits: int = 3,
        layer_bits: dict = None,
        outlier_ratio: float = 0.01,
        sink_token: bool = True,
        use_dense_sparse: bool = True,
    ):
        self.k_codebooks = k_codebooks
        self.v_codebooks = v_codebooks
        self.k_scales = k_scales
        self.k_zeros = k_zeros
        self.k_bits = k_bits
        self.v_bits = v_bits
        self.layer_bits = layer_bits
        self.outlier_ratio = outlier_ratio
        self.sink_token = sink_token
        self.use_dense_sparse = use_dense_sparse

    def _get_bits(self, layer_idx: int, is_key: bool) -> int:
        """kv_quantizer.py:49-52."""
        if self.layer_bits is not None and layer_idx in self.layer_bits:
            return self.layer_bits[layer_idx]
        return self.k_bits if is_key else self.v_bits

    @staticmethod
    def _split_sink(x, sink: bool):
        """kv_quantizer.py:55-58."""
        if sink and x.size(1) > 1:
            return x[:, :1, :].contiguous(), x[:, 1:, :].contiguous()
        return None, x

    def _ratio(self) -> float:
        return self.outlier_ratio if self.use_dense_sparse else 0.0

    @staticmethod
    def _codebook_bits(cb) -> int:
        n = int(torch.as_tensor(cb).numel())
        bits = n.bit_length() - 1
        if n != 1 << bits or bits not in (2, 3, 4):
            raise RuntimeError(f"codebook with {n} entries is not a 2/3/4-bit NUQ table")
        return bits

    def pack_k(self, layer_idx: int, k: torch.Tensor, capacity: int | None = None,
               dequant: bool = False) -> dict:
        cb = self.k_codebooks[layer_idx]
        return quantize_keys(k, self.k_scales[layer_idx], self.k_zeros[layer_idx], cb,
                             self._codebook_bits(cb), self._ratio(), self.sink_token,
                             capacity=capacity, dequant=dequant)

    def pack_v(self, layer_idx: int, v: torch.Tensor, capacity: int | None = None,
               dequant: bool = False) -> dict:
        cb = self.v_codebooks[layer_idx]
        return quantize_values(v, cb, self._codebook_bits(cb), self._ratio(), self.sink_token,
                               capacity=capacity, dequant=dequant)

    def quantize_k(self, layer_idx: int, k: torch.Tensor):
        """Pre-RoPE per-channel key fake quant; kv_quantizer.py:72-94."""
        if k.size(1) == 0:
            return k
        return self.pack_k(layer_idx, k, dequant=True)["dequant"].to(k.dtype)

    def quantize_v(self, layer_idx: int, v: torch.Tensor):
        """Per-token value fake quant; kv_quantizer.py:96-122."""
        if v.size(1) == 0:
            return v
        return self.pack_v(layer_idx, v, dequant=True)["dequant"].to(v.dtype)
