"""Dense-and-sparse outlier helpers (drop-in for kvquant/quant/dense_sparse.py).

Tensor utilities with the reference's semantics, written with torch ops (they
run on whatever device the input lives on). The quantize kernels do their own
fused outlier selection; these helpers exist for API compatibility and for
unpacking results. extract_outliers breaks ties at the top-k threshold toward
lower indices, the rule the quantize kernels use.
"""
from __future__ import annotations

import torch


def extract_outliers(x: torch.Tensor, outlier_ratio: float = 0.01, dim: int = -1):
    """dense_sparse.py:4-32: (dense with outliers zeroed, outliers, mask)."""
    if outlier_ratio <= 0:
        mask = torch.zeros_like(x, dtype=torch.bool)
        return x.clone(), torch.zeros_like(x), mask
    n = x.shape[dim]
    k = max(1, min(int(n * outlier_ratio), n))
    abs_x = x.abs()
    # stable descending sort: among equal |x| the lower index comes first
    order = torch.sort(abs_x, dim=dim, descending=True, stable=True).indices
    topk_idx = order.narrow(dim, 0, k)
    mask = torch.zeros_like(x, dtype=torch.bool)
    mask.scatter_(dim, topk_idx, True)
    dense_x = x.masked_fill(mask, 0.0)
    outliers = x - dense_x
    return dense_x, outliers, mask


def pack_csr(x: torch.Tensor):
    """dense_sparse.py:79-88: CSR of a [R, C] matrix's nonzeros."""
    R, C = x.shape
    mask = x != 0
    values = x[mask]
    col_indices = mask.nonzero(as_tuple=False)[:, 1].to(torch.int32)
    row_counts = mask.sum(dim=1)
    row_ptr = torch.zeros(R + 1, dtype=torch.int32, device=x.device)
    row_ptr[1:] = row_counts.cumsum(0).to(torch.int32)
    return values, col_indices, row_ptr


def unpack_csr(values, col_indices, row_ptr, R: int, C: int, device=None,
               dtype=torch.float16):
    """dense_sparse.py:91-101, vectorized (no per-row Python loop)."""
    if device is None:
        device = values.device
    out = torch.zeros(R, C, device=device, dtype=dtype)
    counts = (row_ptr[1:].long() - row_ptr[:-1].long()).to(device)
    rows = torch.repeat_interleave(torch.arange(R, device=device), counts)
    out[rows, col_indices.long().to(device)] = values.to(device, dtype)
    return out
