"""Seeded synthetic decode workloads generated on the GPU.

Distributions of the benchmark configs: keys N(0,1) x per-channel scale drawn
log-uniform in [0.1, 10], values N(0,1), 1% of entries x20, fp16. Every
(layer, token chunk) has its own seed, so any rank regenerates exactly the
same full-width tensors and can keep the heads it owns. Key scale/zero follow
the calibration formula of kvquant/calibration.py:102-105 over the quantized
tokens; codebooks are fit with train_nuq_codebook (kvquant/quant/nuq.py) on a
sample of normalized, clamped, non-outlier values with the calibration's
scale^2 weights (kvquant/calibration.py:114-125, Fisher = 1).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .quant.nuq import train_nuq_codebook


@dataclass(frozen=True)
class Workload:
    name: str
    batch: int
    kv_heads: int
    q_per_kv: int
    tokens: int
    layers: int
    bits: int
    outlier_ratio: float
    rope_base: float
    head_dim: int = 128

    @property
    def channels(self) -> int:
        return self.kv_heads * self.head_dim


WORKLOADS = {
    # LLaMA-2-7B shape, 1M cached tokens x 32 layers, 4-bit, 1% outliers
    "longctx-1m-4bit": Workload("longctx-1m-4bit", 1, 32, 1, 1 << 20, 32, 4, 0.01, 10000.0),
    # one LLaMA-7B attention layer, 4096 tokens, 4-bit
    "layer-4k-4bit": Workload("layer-4k-4bit", 1, 32, 1, 4096, 1, 4, 0.01, 10000.0),
    # context sweep points, 3-bit, 0.5% outliers
    "layer-2k-3bit": Workload("layer-2k-3bit", 1, 32, 1, 2048, 1, 3, 0.005, 10000.0),
    "layer-8k-3bit": Workload("layer-8k-3bit", 1, 32, 1, 8192, 1, 3, 0.005, 10000.0),
    "layer-32k-3bit": Workload("layer-32k-3bit", 1, 32, 1, 32768, 1, 3, 0.005, 10000.0),
    # LLaMA-3-8B GQA shape, batch 16 x 8K, 2-bit
    "gqa-16x8k-2bit": Workload("gqa-16x8k-2bit", 16, 8, 4, 8192, 1, 2, 0.01, 500000.0),
}


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def channel_scales(C: int, layer: int, seed: int, device) -> torch.Tensor:
    g = _gen(seed * 1000003 + layer * 7919 + 17, device)
    u = torch.rand(C, generator=g, device=device, dtype=torch.float32)
    return torch.exp(math.log(0.1) + u * (math.log(10.0) - math.log(0.1)))


def fill_layer(k: torch.Tensor, v: torch.Tensor, layer: int, seed: int = 0,
               chunk: int = 1 << 15, outlier_frac: float = 0.01, outlier_mult: float = 20.0):
    """Fills k, v [B, T, C] fp16 in place with the layer's seeded synthetic data."""
    B, T, C = k.shape
    dev = k.device
    cs = channel_scales(C, layer, seed, dev)
    for b in range(B):
        for c0 in range(0, T, chunk):
            c1 = min(T, c0 + chunk)
            g = _gen(((seed * 131 + layer) * 65599 + b) * 1000003 + c0, dev)
            for dst, scale in ((k, cs), (v, None)):
                x = torch.randn((c1 - c0, C), generator=g, device=dev, dtype=torch.float32)
                if scale is not None:
                    x.mul_(scale)
                m = torch.rand((c1 - c0, C), generator=g, device=dev) < outlier_frac
                x[m] *= outlier_mult
                dst[b, c0:c1].copy_(x)
                del x, m


def key_calibration(k: torch.Tensor, sink: bool = True, chunk: int = 1 << 16):
    """Per-channel scale/zero over tokens 1.. (kvquant/calibration.py:102-105)."""
    B, T, C = k.shape
    lo = torch.full((C,), float("inf"), device=k.device)
    hi = torch.full((C,), float("-inf"), device=k.device)
    t0 = 1 if (sink and T > 1) else 0
    for b in range(B):
        for c0 in range(t0, T, chunk):
            x = k[b, c0:min(T, c0 + chunk)].float()
            lo = torch.minimum(lo, x.amin(0))
            hi = torch.maximum(hi, x.amax(0))
    return (hi - lo) / 2.0, (hi + lo) / 2.0


def fit_codebooks(k: torch.Tensor, v: torch.Tensor, k_scale: torch.Tensor, k_zero: torch.Tensor,
                  bits: int, n_samples: int = 20000, seed: int = 0):
    """NUQ codebooks for keys and values from a random sample of the layer."""
    B, T, C = k.shape
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    rows = torch.randint(1 if T > 1 else 0, T, (min(T, 512),), generator=g)
    b = torch.randint(0, B, (rows.numel(),), generator=g)
    ks = k[b, rows].float().cpu()
    vs = v[b, rows].float().cpu()
    kn = (ks - k_zero.cpu()) / (k_scale.cpu() + 1e-8)
    vmin, vmax = vs.min(-1, keepdim=True).values, vs.max(-1, keepdim=True).values
    vsc, vz = (vmax - vmin) / 2.0, (vmax + vmin) / 2.0
    vn = (vs - vz) / (vsc + 1e-8)
    out = []
    for xn, w in ((kn, (k_scale.cpu() ** 2).expand_as(kn)), (vn, (vsc ** 2).expand_as(vn))):
        keep = xn.abs() <= 1.0  # drop the outlier tail, as the calibration does
        x, wt = xn[keep], w[keep]
        if x.numel() > n_samples:
            idx = torch.randperm(x.numel(), generator=g)[:n_samples]
            x, wt = x[idx], wt[idx]
        # one solver thread: the multi-threaded k-means reductions round
        # differently from run to run, and the synthetic model's codebooks
        # (hence every cached code) should be the same in every process
        from threadpoolctl import threadpool_limits
        with threadpool_limits(limits=1):
            out.append(train_nuq_codebook(x, wt, n_bits=bits))
    return out[0], out[1]


def make_query(B: int, Hq: int, layer: int, seed: int, device, head_dim: int = 128):
    g = _gen(seed * 7 + layer * 104729 + 3, device)
    return torch.randn((B, Hq, head_dim), generator=g, device=device).to(torch.float16)
