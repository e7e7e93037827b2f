"""Fused decode-path ops of kvquant_b200 (added beside the reference's ops).

quantize_keys / quantize_values
    Quantize-on-append of a prefill block with the semantics of
    KVQuantizer.quantize_k / quantize_v (kvquant/quant/kv_quantizer.py:72-122),
    returning the packed per-layer dict stored in QuantizedKVCache
    (kvquant/kv_cache.py:38-43 keys plus layout fields).
qk_scores
    Fused key kernel: packed codes -> LUT -> outliers -> RoPE -> q.K.
softmax, pv_out, decode_attention
    Softmax over tokens, value kernel (p.V), and the whole decode step.

All tensors are CUDA tensors; work is launched on the current stream.
"""
from __future__ import annotations

import math

import torch

from .cuda_ops import _check, _ptr, _stream, ceil_div, get_cuda_ops

TILE_TOKENS = 32
HEAD_DIM = 128


def tile_bytes(bits: int) -> int:
    return TILE_TOKENS * HEAD_DIM * bits // 8


def _tiles(n: int) -> int:
    return -(-n // TILE_TOKENS)


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def _quantize(kind: str, x: torch.Tensor, codebook: torch.Tensor, bits: int,
              outlier_ratio: float, sink: bool, scale=None, zero=None, h0: int = 0,
              n_heads: int | None = None, capacity: int | None = None,
              dequant: bool = False) -> dict:
    if not x.is_cuda:
        raise RuntimeError(f"quantize_{kind}: kvquant_b200 runs on CUDA tensors only")
    if x.dim() != 3:
        raise RuntimeError(f"quantize_{kind}: expected [B, S, C], got {tuple(x.shape)}")
    if bits not in (2, 3, 4):
        raise RuntimeError(f"quantize_{kind}: bits must be 2, 3 or 4")
    lib = get_cuda_ops().lib
    dev = x.device
    xc = x.to(torch.float16).contiguous()
    B, S, C_full = xc.shape
    if C_full % HEAD_DIM:
        raise RuntimeError(f"quantize_{kind}: C={C_full} is not a multiple of {HEAD_DIM}")
    H = C_full // HEAD_DIM - h0 if n_heads is None else int(n_heads)
    cap = max(S, int(capacity or S))
    nt_cap = _tiles(cap)
    cb = codebook.to(dev, torch.float32).reshape(-1).contiguous()
    if cb.numel() != (1 << bits):
        raise RuntimeError(f"quantize_{kind}: codebook has {cb.numel()} entries, need {1 << bits}")
    U = B * H
    # CSR row pointer over (unit, tile, 16-token block): 2 rows per tile
    out_ptr = torch.empty(2 * U * nt_cap + 1, dtype=torch.int32, device=dev)
    nnz_dev = torch.zeros(1, dtype=torch.int64, device=dev)
    codes = torch.empty((U, nt_cap, tile_bytes(bits)), dtype=torch.uint8, device=dev)
    sink_t = torch.empty((B, H * HEAD_DIM), dtype=torch.float16, device=dev) \
        if (sink and S > 1) else None
    deq = torch.empty((B, S, H * HEAD_DIM), dtype=torch.float16, device=dev) if dequant else None
    with torch.cuda.device(dev):
        st = _stream(xc)
        if kind == "k":
            sc = scale.to(dev, torch.float32).reshape(-1).contiguous()
            ze = zero.to(dev, torch.float32).reshape(-1).contiguous()
            if sc.numel() != C_full or ze.numel() != C_full:
                raise RuntimeError("quantize_keys: scale/zero must have C entries")
            ws = _workspace(lib.kvq_quantize_keys_workspace(B, S, H), dev)
            _check(lib.kvq_quantize_keys_plan(_ptr(xc), B, S, C_full, h0, H, _ptr(sc), _ptr(ze),
                                              float(outlier_ratio), int(sink), _ptr(out_ptr),
                                              nt_cap, _ptr(nnz_dev), _ptr(ws), ws.numel(), st),
                   lib)
            nnz = int(nnz_dev.item())
            ent = torch.empty(max(nnz, 1), dtype=torch.int32, device=dev)
            _check(lib.kvq_quantize_keys_emit(_ptr(xc), B, S, C_full, h0, H, _ptr(sc), _ptr(ze),
                                              _ptr(cb), bits, float(outlier_ratio), int(sink),
                                              _ptr(codes), nt_cap, _ptr(out_ptr), _ptr(ent), nnz,
                                              _ptr(sink_t), _ptr(deq), _ptr(ws), ws.numel(), st),
                   lib)
            scale_out, zero_out = sc[h0 * HEAD_DIM:(h0 + H) * HEAD_DIM].clone(), \
                ze[h0 * HEAD_DIM:(h0 + H) * HEAD_DIM].clone()
        else:
            vs = torch.zeros((B, cap), dtype=torch.float32, device=dev)
            vz = torch.zeros((B, cap), dtype=torch.float32, device=dev)
            ws = _workspace(lib.kvq_quantize_values_workspace(B, S, H), dev)
            _check(lib.kvq_quantize_values_plan(_ptr(xc), B, S, C_full, h0, H,
                                                float(outlier_ratio), int(sink), _ptr(vs),
                                                _ptr(vz), cap, _ptr(out_ptr), nt_cap,
                                                _ptr(nnz_dev), _ptr(ws), ws.numel(), st), lib)
            nnz = int(nnz_dev.item())
            ent = torch.empty(max(nnz, 1), dtype=torch.int32, device=dev)
            _check(lib.kvq_quantize_values_emit(_ptr(xc), B, S, C_full, h0, H, _ptr(cb), bits,
                                                float(outlier_ratio), int(sink), _ptr(vs),
                                                _ptr(vz), cap, _ptr(codes), nt_cap,
                                                _ptr(out_ptr), _ptr(ent), nnz, _ptr(sink_t),
                                                _ptr(deq), _ptr(ws), ws.numel(), st), lib)
            scale_out, zero_out = vs, vz
    pairs = ent.view(torch.int16).view(-1, 2)
    packed = {
        "q_idx": codes,
        # one int32 per outlier: low half = (token_in_tile << 7) | channel, high
        # half = fp16 value; the two halves are also exposed as strided views
        "outlier_entries": ent,
        "outlier_values": pairs[:nnz, 1].view(torch.float16),
        "outlier_cols": pairs[:nnz, 0],
        "outlier_rowptr": out_ptr,
        "scale": scale_out,
        "zero": zero_out,
        "sink": sink_t,
        "codebook": cb,
        "bits": int(bits),
        "kind": kind,
        "batch": B,
        "n_heads": H,
        "h0": int(h0),
        "length": S,
        "capacity": nt_cap * TILE_TOKENS,
        "nnz": nnz,
    }
    if dequant:
        packed["dequant"] = deq
    return packed


def quantize_keys(k: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor,
                  codebook: torch.Tensor, bits: int, outlier_ratio: float = 0.01,
                  sink: bool = True, h0: int = 0, n_heads: int | None = None,
                  capacity: int | None = None, dequant: bool = False) -> dict:
    """Pre-RoPE per-channel key quantization of k [B, S, C] (kv_quantizer.py:72-94)."""
    return _quantize("k", k, codebook, bits, outlier_ratio, sink, scale, zero, h0, n_heads,
                     capacity, dequant)


def quantize_values(v: torch.Tensor, codebook: torch.Tensor, bits: int,
                    outlier_ratio: float = 0.01, sink: bool = True, h0: int = 0,
                    n_heads: int | None = None, capacity: int | None = None,
                    dequant: bool = False) -> dict:
    """Per-token value quantization of v [B, S, C] (kv_quantizer.py:96-122)."""
    return _quantize("v", v, codebook, bits, outlier_ratio, sink, None, None, h0, n_heads,
                     capacity, dequant)


def _group(q: torch.Tensor, packed: dict) -> int:
    B, Hq, D = q.shape
    if D != HEAD_DIM or B != packed["batch"] or Hq % packed["n_heads"]:
        raise RuntimeError(f"q {tuple(q.shape)} does not match the cache "
                           f"(B={packed['batch']}, heads={packed['n_heads']}, D={HEAD_DIM})")
    return Hq // packed["n_heads"]


def qk_scores(q: torch.Tensor, packed_k: dict, inv_freq: torch.Tensor,
              length: int | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Raw scores q . RoPE_t(Khat_t), fp32 [B, Hq, T]; q fp16 [B, Hq, 128]."""
    lib = get_cuda_ops().lib
    qc = q.to(torch.float16).contiguous()
    G = _group(qc, packed_k)
    T = int(length or packed_k["length"])
    B, Hq, _ = qc.shape
    f = inv_freq.to(qc.device, torch.float32).contiguous()
    scores = out if out is not None else torch.empty((B, Hq, T), dtype=torch.float32,
                                                      device=qc.device)
    with torch.cuda.device(qc.device):
        _check(lib.kvq_key_scores(_ptr(packed_k["q_idx"]), _ptr(packed_k["outlier_entries"]),
                                  _ptr(packed_k["outlier_rowptr"]),
                                  _ptr(packed_k["scale"]), _ptr(packed_k["zero"]),
                                  _ptr(packed_k["sink"]), _ptr(packed_k["codebook"]),
                                  packed_k["bits"], _ptr(qc), _ptr(f), B, packed_k["n_heads"], G,
                                  T, packed_k["q_idx"].shape[1], _ptr(scores), _stream(qc)), lib)
    return scores


def softmax(scores: torch.Tensor, scale: float | None = None) -> torch.Tensor:
    """softmax(scores * scale) over the last axis (fp32); scale defaults to 1/sqrt(128)."""
    lib = get_cuda_ops().lib
    s = scores.contiguous()
    T = s.shape[-1]
    rows = s.numel() // T
    scale = 1.0 / math.sqrt(HEAD_DIM) if scale is None else float(scale)
    probs = torch.empty_like(s)
    with torch.cuda.device(s.device):
        ws = _workspace(lib.kvq_softmax_workspace(rows, T), s.device)
        _check(lib.kvq_softmax(_ptr(s), rows, T, scale, _ptr(probs), _ptr(ws), ws.numel(),
                               _stream(s)), lib)
    return probs


def pv_out(probs: torch.Tensor, packed_v: dict, length: int | None = None) -> torch.Tensor:
    """Value kernel: out[b, hq] = sum_t probs[b, hq, t] * Vhat_t; fp16 [B, Hq, 128]."""
    lib = get_cuda_ops().lib
    p = probs.to(torch.float32).contiguous()
    B, Hq, T = p.shape
    if length is not None and int(length) != T:
        raise RuntimeError("pv_out: probs length differs from `length`")
    H = packed_v["n_heads"]
    if B != packed_v["batch"] or Hq % H:
        raise RuntimeError("pv_out: probs do not match the value cache")
    G = Hq // H
    out = torch.empty((B, Hq, HEAD_DIM), dtype=torch.float16, device=p.device)
    with torch.cuda.device(p.device):
        ws = _workspace(lib.kvq_value_output_workspace(B, H, G, T), p.device)
        _check(lib.kvq_value_output(_ptr(packed_v["q_idx"]), _ptr(packed_v["outlier_entries"]),
                                    _ptr(packed_v["outlier_rowptr"]), _ptr(packed_v["scale"]),
                                    _ptr(packed_v["zero"]), packed_v["scale"].shape[1],
                                    _ptr(packed_v["sink"]), _ptr(packed_v["codebook"]),
                                    packed_v["bits"], _ptr(p), B, H, G, T,
                                    packed_v["q_idx"].shape[1], _ptr(out), _ptr(ws), ws.numel(),
                                    _stream(p)), lib)
    return out


def qk_scores_stats(q: torch.Tensor, packed_k: dict, inv_freq: torch.Tensor,
                    length: int | None = None, scale: float | None = None,
                    out: torch.Tensor | None = None, stats_out: torch.Tensor | None = None):
    """qk_scores plus the key kernel's softmax partials of softmax(scores * scale).

    Returns (scores fp32 [B, Hq, T], stats fp32 [B*Hq, ceil(T/256), 2]) where
    stats[row, k] = (max over the k-th 256-token chunk of scores * scale,
    sum over that chunk of exp(scores * scale - max)). pv_out_scores turns the
    pair back into the softmax of the whole row.
    """
    lib = get_cuda_ops().lib
    qc = q.to(torch.float16).contiguous()
    G = _group(qc, packed_k)
    T = int(length or packed_k["length"])
    B, Hq, _ = qc.shape
    scale = 1.0 / math.sqrt(HEAD_DIM) if scale is None else float(scale)
    f = inv_freq.to(qc.device, torch.float32).contiguous()
    scores = out if out is not None else torch.empty((B, Hq, T), dtype=torch.float32,
                                                      device=qc.device)
    n_chunks = ceil_div(T, 256)
    if lib.kvq_key_stats_size(B * Hq, T) != B * Hq * n_chunks * 8:
        raise RuntimeError("qk_scores_stats: library disagrees on the stats size")
    stats = stats_out if stats_out is not None else torch.empty(
        (B * Hq, n_chunks, 2), dtype=torch.float32, device=qc.device)
    if (scores.shape != (B, Hq, T) or scores.dtype != torch.float32
            or not scores.is_contiguous() or stats.numel() != B * Hq * n_chunks * 2
            or stats.dtype != torch.float32 or not stats.is_contiguous()):
        raise RuntimeError("qk_scores_stats: out / stats_out do not match the shapes")
    with torch.cuda.device(qc.device):
        _check(lib.kvq_key_scores_stats(
            _ptr(packed_k["q_idx"]), _ptr(packed_k["outlier_entries"]),
            _ptr(packed_k["outlier_rowptr"]), _ptr(packed_k["scale"]), _ptr(packed_k["zero"]),
            _ptr(packed_k["sink"]), _ptr(packed_k["codebook"]), packed_k["bits"], _ptr(qc),
            _ptr(f), B, packed_k["n_heads"], G, T, packed_k["q_idx"].shape[1], _ptr(scores),
            scale, _ptr(stats), _stream(qc)), lib)
    return scores, stats


def pv_out_scores(scores: torch.Tensor, stats: torch.Tensor, packed_v: dict,
                  scale: float | None = None) -> torch.Tensor:
    """Value kernel on raw scores: sum_t softmax(scores * scale)[t] * Vhat_t, fp16 [B, Hq, 128].

    `stats` comes from qk_scores_stats with the same scale.
    """
    lib = get_cuda_ops().lib
    s = scores.contiguous()
    if s.dtype != torch.float32:
        raise RuntimeError("pv_out_scores: scores must be fp32")
    B, Hq, T = s.shape
    H = packed_v["n_heads"]
    if B != packed_v["batch"] or Hq % H:
        raise RuntimeError("pv_out_scores: scores do not match the value cache")
    G = Hq // H
    scale = 1.0 / math.sqrt(HEAD_DIM) if scale is None else float(scale)
    st = stats.contiguous()
    if st.dtype != torch.float32 or st.numel() * 4 != lib.kvq_key_stats_size(B * Hq, T):
        raise RuntimeError("pv_out_scores: stats do not match the scores")
    out = torch.empty((B, Hq, HEAD_DIM), dtype=torch.float16, device=s.device)
    with torch.cuda.device(s.device):
        ws = _workspace(lib.kvq_value_output_scores_workspace(B, H, G, T), s.device)
        _check(lib.kvq_value_output_scores(
            _ptr(packed_v["q_idx"]), _ptr(packed_v["outlier_entries"]),
            _ptr(packed_v["outlier_rowptr"]), _ptr(packed_v["scale"]), _ptr(packed_v["zero"]),
            packed_v["scale"].shape[1], _ptr(packed_v["sink"]), _ptr(packed_v["codebook"]),
            packed_v["bits"], _ptr(s), _ptr(st), scale, B, H, G, T, packed_v["q_idx"].shape[1],
            _ptr(out), _ptr(ws), ws.numel(), _stream(s)), lib)
    return out


class DecodeWorkspace:
    """Reusable scratch for decode_attention (one per stream)."""

    def __init__(self):
        self.buf = None

    def get(self, nbytes: int, device) -> torch.Tensor:
        if self.buf is None or self.buf.numel() < nbytes or self.buf.device != device:
            self.buf = _workspace(nbytes, device)
        return self.buf


def decode_attention(q: torch.Tensor, packed_k: dict, packed_v: dict, inv_freq: torch.Tensor,
                     length: int | None = None, out: torch.Tensor | None = None,
                     workspace: DecodeWorkspace | None = None,
                     scores_out: torch.Tensor | None = None,
                     probs_out: torch.Tensor | None = None) -> torch.Tensor:
    """One decode step over the quantized cache: fp16 [B, Hq, 128]."""
    lib = get_cuda_ops().lib
    qc = q.to(torch.float16).contiguous()
    G = _group(qc, packed_k)
    if packed_k["bits"] != packed_v["bits"]:
        raise RuntimeError("decode_attention: keys and values must use the same bit width")
    T = int(length or packed_k["length"])
    B, Hq, _ = qc.shape
    H = packed_k["n_heads"]
    f = inv_freq.to(qc.device, torch.float32).contiguous()
    o = out if out is not None else torch.empty((B, Hq, HEAD_DIM), dtype=torch.float16,
                                                device=qc.device)
    need = lib.kvq_decode_attention_workspace(B, H, G, T)
    ws = (workspace or DecodeWorkspace()).get(need, qc.device)
    with torch.cuda.device(qc.device):
        _check(lib.kvq_decode_attention(
            _ptr(packed_k["q_idx"]), _ptr(packed_k["outlier_entries"]),
            _ptr(packed_k["outlier_rowptr"]),
            _ptr(packed_k["scale"]), _ptr(packed_k["zero"]), _ptr(packed_k["sink"]),
            _ptr(packed_k["codebook"]), _ptr(packed_v["q_idx"]), _ptr(packed_v["outlier_entries"]),
            _ptr(packed_v["outlier_rowptr"]),
            _ptr(packed_v["scale"]), _ptr(packed_v["zero"]), packed_v["scale"].shape[1],
            _ptr(packed_v["sink"]), _ptr(packed_v["codebook"]), packed_k["bits"], _ptr(qc), _ptr(f),
            B, H, G, T, packed_k["q_idx"].shape[1], _ptr(o), _ptr(scores_out), _ptr(probs_out),
            _ptr(ws), ws.numel(), _stream(qc)), lib)
    return o
