"""Seeded synthetic K/V generators with the distributions of the benchmark configs.

Keys: N(0,1) times a per-channel scale drawn log-uniform in [0.1, 10]; values:
N(0,1); 1% of all entries multiplied by 20; fp16. The reference measures on
real model activations (wikitext-2, not available offline); these seeded
inputs stand in for them. Key calibration (scale/zero) follows
kvquant/calibration.py:102-105 over the quantized tokens (1..S-1).
"""
from __future__ import annotations

import numpy as np

F16 = np.float16
F32 = np.float32


def make_kv(B: int, S: int, C: int, seed: int = 0, outlier_frac: float = 0.01,
            outlier_mult: float = 20.0):
    rng = np.random.default_rng(seed)
    ch_scale = np.exp(rng.uniform(np.log(0.1), np.log(10.0), size=C)).astype(F32)
    k = rng.standard_normal((B, S, C), dtype=F32) * ch_scale[None, None, :]
    v = rng.standard_normal((B, S, C), dtype=F32)
    for x in (k, v):
        m = rng.random(x.shape) < outlier_frac
        x[m] *= outlier_mult
    return k.astype(F16), v.astype(F16)


def key_calibration(k: np.ndarray, sink: bool = True):
    """Per-channel scale/zero (calibration.py:102-105) over tokens 1.. (or all)."""
    x = k[:, 1:, :] if (sink and k.shape[1] > 1) else k
    flat = x.reshape(-1, x.shape[-1]).astype(F32)
    kmin, kmax = flat.min(axis=0), flat.max(axis=0)
    scale = ((kmax - kmin) / F32(2.0)).astype(F32)
    zero = ((kmax + kmin) / F32(2.0)).astype(F32)
    return scale, zero


def make_query(B: int, Hq: int, D: int = 128, seed: int = 1):
    rng = np.random.default_rng(seed)
    return rng.standard_normal((B, Hq, D), dtype=F32).astype(F16)
