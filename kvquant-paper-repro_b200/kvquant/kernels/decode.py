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
make_appendable, append_keys, append_values, key_outlier_thresholds
    Decode-time append of new tokens into a packed cache (O(new tokens) per
    call): values exactly as one-token calls of quantize_v, keys with
    calibrated per-channel outlier thresholds.

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
        # half = the fp16 dequantized value (cb[c0] + n) * s + z at that position
        # (kv_quantizer.py:89,117); the two halves are also exposed as strided views
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
        "C_full": C_full,
        "n_heads": H,
        "h0": int(h0),
        "length": S,
        "capacity": nt_cap * TILE_TOKENS,
        "nnz": nnz,
        "outlier_ratio": float(outlier_ratio),
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
                    out: torch.Tensor | None = None, stats_out: torch.Tensor | None = None,
                    pos0: int = 0):
    """qk_scores plus the key kernel's softmax partials of softmax(scores * scale).

    Returns (scores fp32 [B, Hq, T], stats fp32 [B*Hq, ceil(T/16), 2]) where
    stats[row, k] = (max over the k-th 16-token block of scores * scale,
    sum over that block of exp(scores * scale - max)). pv_out_scores turns the
    pair back into the softmax of the whole row. pos0: RoPE position of the
    cache's token 0 (a token-range shard of a longer context).
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
    n_chunks = ceil_div(T, 16)
    if lib.kvq_key_stats_size(B * Hq, T) != B * Hq * n_chunks * 8:
        raise RuntimeError("qk_scores_stats: library disagrees on the stats size")
    stats = stats_out if stats_out is not None else torch.empty(
        (B * Hq, n_chunks, 2), dtype=torch.float32, device=qc.device)
    if (scores.shape != (B, Hq, T) or scores.dtype != torch.float32
            or not scores.is_contiguous() or stats.numel() != B * Hq * n_chunks * 2
            or stats.dtype != torch.float32 or not stats.is_contiguous()):
        raise RuntimeError("qk_scores_stats: out / stats_out do not match the shapes")
    with torch.cuda.device(qc.device):
        if pos0:
            _check(lib.kvq_key_scores_stats_at(
                _ptr(packed_k["q_idx"]), _ptr(packed_k["outlier_entries"]),
                _ptr(packed_k["outlier_rowptr"]), _ptr(packed_k["scale"]),
                _ptr(packed_k["zero"]), _ptr(packed_k["sink"]), _ptr(packed_k["codebook"]),
                packed_k["bits"], _ptr(qc), _ptr(f), B, packed_k["n_heads"], G, T,
                packed_k["q_idx"].shape[1], int(pos0), _ptr(scores), scale, _ptr(stats),
                _stream(qc)), lib)
        else:
            _check(lib.kvq_key_scores_stats(
                _ptr(packed_k["q_idx"]), _ptr(packed_k["outlier_entries"]),
                _ptr(packed_k["outlier_rowptr"]), _ptr(packed_k["scale"]),
                _ptr(packed_k["zero"]), _ptr(packed_k["sink"]), _ptr(packed_k["codebook"]),
                packed_k["bits"], _ptr(qc), _ptr(f), B, packed_k["n_heads"], G, T,
                packed_k["q_idx"].shape[1], _ptr(scores), scale, _ptr(stats), _stream(qc)), lib)
    return scores, stats


def pv_out_scores(scores: torch.Tensor, stats: torch.Tensor, packed_v: dict,
                  scale: float | None = None, ml_out: torch.Tensor | None = None,
                  out: torch.Tensor | None = None,
                  workspace: "DecodeWorkspace | None" = None) -> torch.Tensor:
    """Value kernel on raw scores: sum_t softmax(scores * scale)[t] * Vhat_t, fp16 [B, Hq, 128].

    `stats` comes from qk_scores_stats with the same scale. ml_out (fp32
    [B*Hq, 2], optional) receives each row's softmax stats (M, 1/L), which
    merge_shards needs to combine token-range shards.
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
    if out is None:
        out = torch.empty((B, Hq, HEAD_DIM), dtype=torch.float16, device=s.device)
    if ml_out is not None and (ml_out.dtype != torch.float32 or not ml_out.is_contiguous()
                               or ml_out.numel() != B * Hq * 2):
        raise RuntimeError("pv_out_scores: ml_out must be contiguous fp32 [B*Hq, 2]")
    with torch.cuda.device(s.device):
        need = lib.kvq_value_output_scores_workspace(B, H, G, T)
        ws = workspace.get(need, s.device) if workspace is not None else _workspace(need, s.device)
        args = (_ptr(packed_v["q_idx"]), _ptr(packed_v["outlier_entries"]),
                _ptr(packed_v["outlier_rowptr"]), _ptr(packed_v["scale"]), _ptr(packed_v["zero"]),
                packed_v["scale"].shape[1], _ptr(packed_v["sink"]), _ptr(packed_v["codebook"]),
                packed_v["bits"], _ptr(s), _ptr(st), scale, B, H, G, T,
                packed_v["q_idx"].shape[1], _ptr(out))
        if ml_out is None:
            _check(lib.kvq_value_output_scores(*args, _ptr(ws), ws.numel(), _stream(s)), lib)
        else:
            _check(lib.kvq_value_output_scores_ml(*args, _ptr(ml_out), _ptr(ws), ws.numel(),
                                                  _stream(s)), lib)
    return out


def decode_attention_shard(q: torch.Tensor, packed_k: dict, packed_v: dict,
                           inv_freq: torch.Tensor, pos0: int, scores: torch.Tensor | None = None,
                           stats: torch.Tensor | None = None, out: torch.Tensor | None = None,
                           ml_out: torch.Tensor | None = None,
                           workspace: "DecodeWorkspace | None" = None):
    """One decode step over a token-range shard: the cache holds the tokens at
    positions [pos0, pos0 + length) (its token 0 is the sink only when pos0 == 0).
    Returns (o fp16 [B, Hq, 128] normalized over the shard's tokens, ml fp32
    [B*Hq, 2] = the shard's softmax row stats); merge_shards combines shards."""
    qc = q.to(torch.float16).contiguous()
    B, Hq, _ = qc.shape
    if ml_out is None:
        ml_out = torch.empty((B * Hq, 2), dtype=torch.float32, device=qc.device)
    sc, st = qk_scores_stats(qc, packed_k, inv_freq, out=scores, stats_out=stats, pos0=pos0)
    o = pv_out_scores(sc, st, packed_v, ml_out=ml_out, out=out, workspace=workspace)
    return o, ml_out


def merge_shards(o_shards: torch.Tensor, ml_shards: torch.Tensor,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """Output over the whole context from n token-range shards.

    o_shards fp16 [n, B, Hq, 128] and ml_shards fp32 [n, B*Hq, 2] as returned
    by decode_attention_shard on each shard (e.g. all-gathered across ranks).
    """
    lib = get_cuda_ops().lib
    o = o_shards.contiguous()
    ml = ml_shards.contiguous()
    if o.dtype != torch.float16 or ml.dtype != torch.float32 or o.shape[-1] != HEAD_DIM:
        raise RuntimeError("merge_shards: expected fp16 outputs [n, ..., 128] and fp32 stats")
    n = o.shape[0]
    rows = o[0].numel() // HEAD_DIM
    if ml.numel() != n * rows * 2:
        raise RuntimeError("merge_shards: stats do not match the outputs")
    if out is None:
        out = torch.empty(o.shape[1:], dtype=torch.float16, device=o.device)
    with torch.cuda.device(o.device):
        _check(lib.kvq_merge_shards(_ptr(o), _ptr(ml), n, rows, _ptr(out), _stream(o)), lib)
    return out


_KERNELS = {"mma": 0, "tc": 1}


def set_decode_kernels(key: str | None = None, value: str | None = None) -> tuple[str, str]:
    """Selects the decode kernels process-wide and returns the previous choice.

    "mma" = warp-level mma.sync kernels (the default), "tc" = tcgen05 kernels
    with TMEM accumulators (the key one serves one query head per KV head);
    None keeps the current one. Both compute the same values up to fp32
    summation order."""
    lib = get_cuda_ops().lib
    cur = lib.kvq_decode_kernels()
    names = {v: k for k, v in _KERNELS.items()}
    prev = (names[cur & 1], names[(cur >> 1) & 1])
    for x in (key, value):
        if x is not None and x not in _KERNELS:
            raise ValueError(f"decode kernel must be one of {sorted(_KERNELS)}, got {x!r}")
    _check(lib.kvq_set_decode_kernels(_KERNELS.get(key, -1), _KERNELS.get(value, -1)), lib)
    return prev


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


# ---------------------------------------------------------------------------
# Decode-time append
# ---------------------------------------------------------------------------
def make_appendable(packed: dict, extra_tokens: int,
                    entries_per_token: int | None = None) -> dict:
    """Copy of a packed cache laid out for appending up to `extra_tokens` tokens.

    The prefill layout packs every unit's outlier entries back to back, so a
    unit's CSR rows cannot grow. This copy gives each unit (b, head) its own
    entry segment of `ent_stride` entries (its current entries plus
    extra_tokens * entries_per_token free slots) and one spare code tile after
    the last appendable token; the decode kernels read it unchanged. Default
    entries_per_token: 128 for keys (every channel of a token may be an outlier,
    as with thresholds = 0), min(128, k) for values (k = the per-token top-k).
    The `nnz` field keeps the count at the time of the copy.
    """
    if extra_tokens < 0:
        raise RuntimeError("make_appendable: extra_tokens must be >= 0")
    dev = packed["q_idx"].device
    U, nt_cap, tb = packed["q_idx"].shape
    T = int(packed["length"])
    nt = _tiles(T)
    new_cap = _tiles(T + extra_tokens) + 1
    if entries_per_token is None:
        if packed["kind"] == "k":
            entries_per_token = HEAD_DIM
        else:
            C_full = packed.get("C_full", packed["n_heads"] * HEAD_DIM)
            r = packed.get("outlier_ratio", 0.01)
            entries_per_token = min(HEAD_DIM, max(1, int(C_full * r))) if r > 0 else 0
    codes = torch.zeros((U, new_cap, tb), dtype=torch.uint8, device=dev)
    codes[:, :nt] = packed["q_idx"][:, :nt]
    ptr = packed["outlier_rowptr"].to(torch.int64)
    R, R2 = 2 * nt_cap, 2 * new_cap
    rows = torch.arange(U, device=dev) * R
    starts = ptr[rows].cpu().tolist()
    ends = ptr[rows + 2 * nt].cpu().tolist()
    used = [e - s for s, e in zip(starts, ends)]
    stride = max(used + [0]) + extra_tokens * int(entries_per_token)
    stride = max(64, -(-stride // 64) * 64)
    if U * stride >= 2 ** 31:
        raise RuntimeError("make_appendable: the entry segments exceed int32 indexing")
    ent = torch.zeros(U * stride, dtype=torch.int32, device=dev)
    new_ptr = torch.empty(U * R2 + 1, dtype=torch.int32, device=dev)
    old_ent = packed["outlier_entries"]
    for u in range(U):
        s, n = starts[u], used[u]
        if n:
            ent[u * stride:u * stride + n] = old_ent[s:s + n]
        seg = ptr[u * R:u * R + 2 * nt + 1] - s + u * stride
        new_ptr[u * R2:u * R2 + 2 * nt + 1] = seg.to(torch.int32)
        new_ptr[u * R2 + 2 * nt + 1:(u + 1) * R2] = u * stride + n
    new_ptr[U * R2] = U * stride
    out = dict(packed)
    pairs = ent.view(torch.int16).view(-1, 2)
    out.update({
        "q_idx": codes,
        "outlier_entries": ent,
        "outlier_values": pairs[:, 1].view(torch.float16),
        "outlier_cols": pairs[:, 0],
        "outlier_rowptr": new_ptr,
        "capacity": (new_cap - 1) * TILE_TOKENS,
        "ent_stride": stride,
        "appendable": True,
        # reused by every append call: the status word and the values' scratch
        "append_status": torch.zeros(1, dtype=torch.int32, device=dev),
        "append_workspace": None,
    })
    if packed["kind"] == "v":
        B = packed["batch"]
        for key in ("scale", "zero"):
            st = torch.zeros((B, new_cap * TILE_TOKENS), dtype=torch.float32, device=dev)
            st[:, :T] = packed[key][:, :T]
            out[key] = st
    return out


def _append_status(status: torch.Tensor, what: str, check: bool) -> None:
    # The status word only ever gets bits set (by a unit that had no room), so
    # it is cleared only after a failure is read; an unchecked call's failure
    # is reported by the next checked one.
    if check and int(status.item()) != 0:
        status.zero_()
        raise RuntimeError(f"{what}: a unit's outlier segment is full (nothing was appended "
                           "for that unit); rebuild with make_appendable and more "
                           "entries_per_token")


def _append_prologue(kind: str, packed: dict, x: torch.Tensor):
    if not packed.get("appendable"):
        raise RuntimeError(f"append_{kind}: the cache is not appendable (see make_appendable)")
    if not x.is_cuda or x.dim() != 3:
        raise RuntimeError(f"append_{kind}: expected a CUDA tensor [B, S_new, C]")
    xc = x.to(torch.float16).contiguous()
    if xc.shape[0] != packed["batch"]:
        raise RuntimeError(f"append_{kind}: batch {xc.shape[0]} != cache batch {packed['batch']}")
    if packed["length"] + xc.shape[1] > packed["capacity"]:
        raise RuntimeError(f"append_{kind}: {packed['length']} + {xc.shape[1]} tokens exceed the "
                           f"appendable capacity {packed['capacity']}")
    return xc


def append_keys(packed_k: dict, k_new: torch.Tensor, thresholds: torch.Tensor | None,
                check: bool = True) -> dict:
    """Appends k_new [B, S_new, C] (pre-RoPE keys) to an appendable key cache, in place.

    thresholds: fp32 [n_heads*128] per-channel outlier thresholds on the
    normalized |n| (key_outlier_thresholds), or None for no outliers; zeros
    reproduce the reference's quantize_k on one-token blocks. check=True reads
    the status back (one host sync) and raises if a unit ran out of room (in
    this call or in an earlier call made with check=False).
    """
    lib = get_cuda_ops().lib
    kc = _append_prologue("keys", packed_k, k_new)
    B, S, C_full = kc.shape
    H, dev = packed_k["n_heads"], kc.device
    thr = None
    if thresholds is not None:
        thr = thresholds.to(dev, torch.float32).reshape(-1).contiguous()
        if thr.numel() != H * HEAD_DIM:
            raise RuntimeError("append_keys: thresholds must have n_heads*128 entries")
    status = packed_k["append_status"]
    with torch.cuda.device(dev):
        _check(lib.kvq_append_keys(
            _ptr(kc), B, S, C_full, packed_k["h0"], H, _ptr(packed_k["scale"]),
            _ptr(packed_k["zero"]), _ptr(thr), _ptr(packed_k["codebook"]), packed_k["bits"],
            packed_k["length"], _ptr(packed_k["q_idx"]), packed_k["q_idx"].shape[1],
            _ptr(packed_k["outlier_rowptr"]), _ptr(packed_k["outlier_entries"]),
            packed_k["ent_stride"], _ptr(status), _stream(kc)), lib)
    _append_status(status, "append_keys", check)
    packed_k["length"] += S
    return packed_k


def append_values(packed_v: dict, v_new: torch.Tensor, check: bool = True) -> dict:
    """Appends v_new [B, S_new, C] to an appendable value cache, in place.

    Every new token is quantized as a one-token call of quantize_v would
    (kv_quantizer.py:96-122): per-token scale/zero and top-k outliers over all
    C channels of v_new, with the cache's outlier ratio.
    """
    lib = get_cuda_ops().lib
    vc = _append_prologue("values", packed_v, v_new)
    B, S, C_full = vc.shape
    dev = vc.device
    need = lib.kvq_append_values_workspace(B, S)
    ws = packed_v.get("append_workspace")
    if ws is None or ws.numel() < need:
        ws = packed_v["append_workspace"] = _workspace(need, dev)
    status = packed_v["append_status"]
    with torch.cuda.device(dev):
        _check(lib.kvq_append_values(
            _ptr(vc), B, S, C_full, packed_v["h0"], packed_v["n_heads"],
            float(packed_v.get("outlier_ratio", 0.01)), _ptr(packed_v["codebook"]),
            packed_v["bits"], packed_v["length"], _ptr(packed_v["scale"]),
            _ptr(packed_v["zero"]), packed_v["scale"].shape[1], _ptr(packed_v["q_idx"]),
            packed_v["q_idx"].shape[1], _ptr(packed_v["outlier_rowptr"]),
            _ptr(packed_v["outlier_entries"]), packed_v["ent_stride"], _ptr(ws), ws.numel(),
            _ptr(status), _stream(vc)), lib)
    _append_status(status, "append_values", check)
    packed_v["length"] += S
    return packed_v


def key_outlier_thresholds(k: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor,
                           outlier_ratio: float = 0.01, sink: bool = True, h0: int = 0,
                           n_heads: int | None = None) -> torch.Tensor:
    """Per-channel thresholds on |n| from a calibration block k [B, S, C] (offline).

    n = (k - zero) / (scale + 1e-8) over the block's tokens (the sink token
    excluded, as quantize_k does); the threshold of a channel is the m-th
    largest |n| over all B * S' values, m = max(1, int(B * S' * ratio)), so the
    calibration block itself has about the reference's outlier share.
    Returns fp32 [n_heads*128] for heads [h0, h0 + n_heads).
    """
    B, S, C_full = k.shape
    H = C_full // HEAD_DIM - h0 if n_heads is None else int(n_heads)
    c0, c1 = h0 * HEAD_DIM, (h0 + H) * HEAD_DIM
    x = k[:, 1:] if (sink and S > 1) else k
    sc = scale.to(k.device, torch.float32).reshape(-1)[c0:c1]
    ze = zero.to(k.device, torch.float32).reshape(-1)[c0:c1]
    n = ((x[:, :, c0:c1].float() - ze) / (sc + 1e-8)).abs().reshape(-1, c1 - c0)
    m = max(1, int(n.shape[0] * outlier_ratio))
    return torch.topk(n.t(), m, dim=1).values[:, -1].contiguous()
