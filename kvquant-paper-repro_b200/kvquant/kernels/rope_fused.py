"""RoPE host API (drop-in for kvquant/kernels/rope_fused.py).

Same functions and argument meaning as the reference. The rotation runs in the
sm_100a ``rope_apply`` kernel with fp32 cos/sin tables (the reference's CUDA
semantics, rope_fused.py:29-34); tensors must be CUDA fp16.
"""
from __future__ import annotations

import torch

from .cuda_ops import get_cuda_ops


def _build_cos_sin(seq_len, dim, device, dtype=torch.float32, base=10000.0):
    """rope_fused.py:6-12: fp32 angles outer(t, 1/base^(i/half)), then cos/sin."""
    half = dim // 2
    inv_freq = 1.0 / (base ** (torch.arange(0, half, device=device,
                                             dtype=torch.float32) / half))
    t = torch.arange(seq_len, device=device, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    return freqs.cos().to(dtype), freqs.sin().to(dtype)


def rope_inv_freq(dim: int = 128, base: float = 10000.0) -> torch.Tensor:
    """The fp32 inverse frequencies of rope_fused.py:7-8, computed on the CPU.

    The fused key kernel takes these 64 values and forms each angle as the
    fp32 product t * inv_freq[i] itself, exactly as torch.outer does.
    """
    half = dim // 2
    return 1.0 / (base ** (torch.arange(0, half, dtype=torch.float32) / half))


def apply_rope_elementwise(x: torch.Tensor,
                           position_offset: int = 0,
                           base: float = 10000.0):
    """Rotate-half RoPE of x ([B, S, H] or [B, H, S, D]); rope_fused.py:15-46."""
    assert x.dim() in (3, 4), f"unsupported input shape: {x.shape}"
    if not x.is_cuda or x.dtype != torch.float16:
        raise RuntimeError("apply_rope_elementwise: kvquant_b200 needs a CUDA fp16 tensor")
    orig_dim = x.dim()
    x4 = x.unsqueeze(2) if orig_dim == 3 else x
    B, H, S, D = x4.shape
    cos, sin = _build_cos_sin(S + position_offset, D, x4.device, dtype=torch.float32, base=base)
    out4 = get_cuda_ops().rope_apply(x4.contiguous(), cos.contiguous(), sin.contiguous(),
                                     int(position_offset))
    return out4.squeeze(2) if orig_dim == 3 else out4


def apply_rope_inplace(x: torch.Tensor,
                       position_offset: int = 0,
                       base: float = 10000.0):
    """rope_fused.py:49-54."""
    out = apply_rope_elementwise(x, position_offset=position_offset, base=base)
    x.copy_(out)
    return x
