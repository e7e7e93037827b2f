"""Dense/sparse matvec host API (drop-in for kvquant/kernels/matvec_ds.py).

Same functions, arguments and results as the reference; every call runs an
sm_100a kernel of the kvquant_b200 library. The reference's PyTorch fallbacks
(matvec_ds.py:18-23, 40-49, 69-72) are not part of this library: inputs must be
CUDA tensors.
"""
from __future__ import annotations

import torch

from .cuda_ops import get_cuda_ops


def _cuda_only(name, *ts):
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError(f"{name}: kvquant_b200 runs on CUDA tensors only")


def dense_matvec_lut(x: torch.Tensor, codebook: torch.Tensor):
    """Nearest-centroid snap (quantize + dequantize) of x; matvec_ds.py:6-23.

    x: [..., D]; codebook: [2^b]; returns [..., D] in x's dtype.
    """
    _cuda_only("dense_matvec_lut", x)
    cb = codebook.to(x.device, dtype=torch.float32).reshape(-1).contiguous()
    _, dq = get_cuda_ops().lut_lookup(x.reshape(-1).float(), cb)
    return dq.reshape(x.shape).to(x.dtype)


def sparse_matvec_csr(row_ptr, col_idx, values, x):
    """CSR matrix x vector; matvec_ds.py:26-49. Returns [R] in x's dtype (fp16)."""
    _cuda_only("sparse_matvec_csr", row_ptr, col_idx, values, x)
    R = int(row_ptr.numel()) - 1
    return get_cuda_ops().sparse_matvec_csr(row_ptr, col_idx, values, x, R)


def sparse_matvec(indices: torch.Tensor, values: torch.Tensor, shape, x: torch.Tensor):
    """COO matrix x vector via CSR; matvec_ds.py:52-72."""
    _cuda_only("sparse_matvec", indices, values, x)
    R, C = shape
    rows = indices[:, 0].long()
    cols = indices[:, 1].long()
    order = torch.argsort(rows, stable=True)
    rows_s, cols_s, vals_s = rows[order], cols[order], values[order]
    row_counts = torch.bincount(rows_s, minlength=R)
    row_ptr = torch.zeros(R + 1, dtype=torch.int32, device=x.device)
    row_ptr[1:] = row_counts.cumsum(0).to(torch.int32)
    return get_cuda_ops().sparse_matvec_csr(row_ptr, cols_s.to(torch.int32),
                                            vals_s.contiguous(), x, R)
