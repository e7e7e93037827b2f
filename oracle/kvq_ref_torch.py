"""CPU port of the reference's decode path over the reference's own cache format,
in torch on the host cores: the timed CPU baseline of bench.py.

Test/measurement infrastructure, not product code: only bench.py's CPU legs use it.

The reference stores a layer's quantized cache as kvquant/kv_cache.py:4-44 does:
one code per byte (q_idx uint8 [B, S, C]), the outliers as CSR over token rows
(values fp16, cols int32, row_ptr int32; dense_sparse.py:79-88), per-channel
key scale/zero and per-token value scale/zero, and the fp16 sink token. It has
no decode attention of its own; the decode step restated here is the one the
fake-quant path feeds to the model's attention:

* dequantization (cb[q] + o) * s + z in fp32, rounded to fp16
  (kv_quantizer.py:89 keys, :117 values), the outliers scattered from the CSR;
* RoPE on the dequantized keys with the fp32 angle tables of
  rope_fused.py:6-12 (rotate-half, rope_fused.py:40-44), in fp32;
* scores q . K, softmax(scores / sqrt(128)), output p . V in fp32
  (torch.matmul / torch.softmax).

Every step is a torch op over the whole layer, multithreaded by torch.
"""
from __future__ import annotations

import math

import numpy as np
import torch

HEAD_DIM = 128


def make_reference_cache(T: int, n_kv_heads: int, bits: int, ratio: float, seed: int = 0,
                         base: float = 10000.0) -> dict:
    """A seeded layer cache in the reference's format (batch 1, T tokens with a
    sink at token 0). Codes are uniform; outlier counts follow
    dense_sparse.py:22-23 (keys: top-k per channel along tokens, k =
    int((T-1)*ratio); values: top-k per token along channels, k = int(C*ratio))
    at random positions. The decode's cost does not depend on the values."""
    g = np.random.default_rng(seed)
    C = n_kv_heads * HEAD_DIM
    S = T - 1
    out = {"T": T, "C": C, "H": n_kv_heads, "bits": bits, "base": base}
    for kind in ("k", "v"):
        q_idx = g.integers(0, 1 << bits, size=(S, C), dtype=np.uint8)
        if kind == "k":
            kk = max(1, min(int(S * ratio), S))
            rows = np.concatenate([g.choice(S, kk, replace=False) for _ in range(C)])
            cols = np.repeat(np.arange(C, dtype=np.int32), kk)
            order = np.lexsort((cols, rows))
            rows, cols = rows[order], cols[order]
        else:
            kk = max(1, min(int(C * ratio), C))
            rows = np.repeat(np.arange(S), kk)
            cols = np.concatenate([np.sort(g.choice(C, kk, replace=False)) for _ in range(S)])
        row_ptr = np.zeros(S + 1, np.int64)
        np.add.at(row_ptr, rows + 1, 1)
        row_ptr = np.cumsum(row_ptr).astype(np.int32)
        vals = g.uniform(-2, 2, size=rows.size).astype(np.float16)
        cb = np.sort(g.uniform(-1, 1, 1 << bits)).astype(np.float32)
        if kind == "k":
            scale = np.exp(g.uniform(np.log(0.1), np.log(10.0), C)).astype(np.float32)
            zero = g.normal(0, 0.1, C).astype(np.float32)
        else:
            scale = g.uniform(1, 3, S).astype(np.float32)
            zero = g.normal(0, 0.1, S).astype(np.float32)
        out[kind] = {
            "q_idx": torch.from_numpy(q_idx), "codebook": torch.from_numpy(cb),
            "outlier_values": torch.from_numpy(vals), "outlier_cols": torch.from_numpy(cols),
            "outlier_rowptr": torch.from_numpy(row_ptr), "scale": torch.from_numpy(scale),
            "zero": torch.from_numpy(zero),
            "sink": torch.from_numpy(g.standard_normal(C).astype(np.float16)),
        }
    out["q"] = torch.from_numpy(g.standard_normal((n_kv_heads, HEAD_DIM)).astype(np.float16))
    return out


def _dequant(c: dict, per_channel: bool) -> torch.Tensor:
    """(cb[q] + o) * s + z -> fp16 [S, C] (kv_quantizer.py:89,117), CSR outliers scattered."""
    S, C = c["q_idx"].shape
    x = c["codebook"][c["q_idx"].long()]                          # cb[q], fp32
    counts = (c["outlier_rowptr"][1:] - c["outlier_rowptr"][:-1]).long()
    rows = torch.repeat_interleave(torch.arange(S), counts)
    flat = rows * C + c["outlier_cols"].long()
    x.view(-1).index_add_(0, flat, c["outlier_values"].float())  # + o
    if per_channel:
        x.mul_(c["scale"]).add_(c["zero"])
    else:
        x.mul_(c["scale"][:, None]).add_(c["zero"][:, None])
    return x.half()


def _cos_sin(T: int, base: float):
    """rope_fused.py:6-12: fp32 angles outer(t, inv_freq)."""
    inv = 1.0 / (base ** (torch.arange(0, HEAD_DIM, 2, dtype=torch.float32) / HEAD_DIM))
    ang = torch.outer(torch.arange(T, dtype=torch.float32), inv)
    return torch.cos(ang), torch.sin(ang)


def decode_step(cache: dict) -> torch.Tensor:
    """One decode step of one layer: fp16 output [H, 128]."""
    T, H = cache["T"], cache["H"]
    kd = torch.cat([cache["k"]["sink"][None], _dequant(cache["k"], True)])   # [T, C] fp16
    vd = torch.cat([cache["v"]["sink"][None], _dequant(cache["v"], False)])
    cos, sin = _cos_sin(T, cache["base"])
    K = kd.float().view(T, H, HEAD_DIM).transpose(0, 1)                     # [H, T, D]
    k1, k2 = K[..., :HEAD_DIM // 2], K[..., HEAD_DIM // 2:]
    Kr = torch.cat([k1 * cos - k2 * sin, k1 * sin + k2 * cos], dim=-1)  # position 0: identity
    q = cache["q"].float()
    s = torch.matmul(Kr, q[:, :, None])[..., 0]                            # [H, T]
    p = torch.softmax(s / math.sqrt(HEAD_DIM), dim=-1)
    V = vd.float().view(T, H, HEAD_DIM).transpose(0, 1)
    return torch.matmul(p[:, None, :], V)[:, 0].half()
