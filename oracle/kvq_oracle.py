"""CPU oracle for KVQuant's decode-time quantized-KV attention path.

TEST INFRASTRUCTURE ONLY. Nothing in the product (the package under
``kvquant-paper-repro_b200/``) imports this module. It is used by ``tests/`` as
the checker, by ``__graft_entry__.smoke()`` to check one small GPU run, and by
``bench.py``'s ``cpu_baseline`` leg / ``--impl reference`` arm as the timed CPU
port of the reference path.

It restates, in numpy, the reference's algorithm for the path. Every function
cites the reference file and lines it follows (paths relative to the
KVQuant-Paper-Repro project root). Parity of this restatement is pinned by
``tests/test_oracle_golden.py`` against golden vectors produced by running the
reference's own PyTorch code (``tests/golden/make_golden.py``).

Packed-format helpers (``pack_codes``/``unpack_codes``/``tile_outliers``) define
the library's HBM layout for the quantized cache; the reference stores one code
per byte and has no bit packing, so the format is new and is checked here by
round trips to the reference's indices.
"""
from __future__ import annotations

import math

import numpy as np

F16 = np.float16
F32 = np.float32

TILE_TOKENS = 32     # tokens per code tile
HEAD_DIM = 128       # channels per head (LLaMA head_dim)
ROPE_PAIRS = HEAD_DIM // 2
EPS = F32(1e-8)      # kv_quantizer.py:82,110 `scale + 1e-8` (fp32 add)


# --------------------------------------------------------------------------
# Nearest-centroid lookup and dense-and-sparse outliers
# --------------------------------------------------------------------------
def lut_lookup(x: np.ndarray, codebook: np.ndarray):
    """Nearest centroid, first minimum wins.

    kvquant/quant/kv_quantizer.py:15-21 (CPU branch) and
    kvquant/kernels/csrc/kvquant_ops.cu:132-151 (`d < best_d`, strict).
    Returns (idx int64, dequant fp32) with x's shape.
    """
    cb = np.asarray(codebook, dtype=F32).reshape(-1)
    flat = np.asarray(x, dtype=F32).reshape(-1)
    idx = np.empty(flat.shape, dtype=np.int64)
    step = 1 << 20
    for s in range(0, flat.size, step):
        d = np.abs(flat[s:s + step, None] - cb[None, :])
        idx[s:s + step] = d.argmin(axis=1)
    return idx.reshape(np.shape(x)), cb[idx].reshape(np.shape(x))


def outlier_count(n: int, ratio: float) -> int:
    """k = max(1, min(int(n * ratio), n)) -- kvquant/quant/dense_sparse.py:22-23."""
    return max(1, min(int(n * ratio), n))


def topk_mask(xabs: np.ndarray, k: int, axis: int) -> np.ndarray:
    """Top-k mask of |x| along `axis` (kvquant/quant/dense_sparse.py:25-28).

    torch.topk leaves the order of equal values unspecified; the library fixes
    it: among values equal to the k-th largest, lower indices win.
    """
    order = np.argsort(-xabs, axis=axis, kind="stable")
    sel = np.take(order, np.arange(k), axis=axis)
    mask = np.zeros(xabs.shape, dtype=bool)
    np.put_along_axis(mask, sel, True, axis=axis)
    return mask


def extract_outliers(x: np.ndarray, outlier_ratio: float = 0.01, dim: int = -1):
    """kvquant/quant/dense_sparse.py:4-32: (dense with outliers zeroed, outliers, mask)."""
    x = np.asarray(x, dtype=F32)
    if outlier_ratio <= 0:
        return x.copy(), np.zeros_like(x), np.zeros(x.shape, dtype=bool)
    k = outlier_count(x.shape[dim], outlier_ratio)
    mask = topk_mask(np.abs(x), k, dim % x.ndim)
    dense = np.where(mask, F32(0.0), x).astype(F32)
    outliers = (x - dense).astype(F32)
    return dense, outliers, mask


def pack_csr(x: np.ndarray):
    """kvquant/quant/dense_sparse.py:79-88: CSR of nonzeros of a [R, C] matrix."""
    mask = x != 0
    values = x[mask]
    cols = np.nonzero(mask)[1].astype(np.int32)
    row_ptr = np.zeros(x.shape[0] + 1, dtype=np.int32)
    row_ptr[1:] = np.cumsum(mask.sum(axis=1)).astype(np.int32)
    return values, cols, row_ptr


def unpack_csr(values, cols, row_ptr, R: int, C: int, dtype=F16):
    """kvquant/quant/dense_sparse.py:91-101."""
    out = np.zeros((R, C), dtype=dtype)
    for r in range(R):
        s, e = int(row_ptr[r]), int(row_ptr[r + 1])
        if e > s:
            out[r, cols[s:e]] = values[s:e].astype(dtype)
    return out


# --------------------------------------------------------------------------
# KVQuantizer.quantize_k / quantize_v (fake quant: quantize then dequantize)
# --------------------------------------------------------------------------
def _split_sink(x, sink: bool):
    """kvquant/quant/kv_quantizer.py:55-58: token 0 stays fp16 when S > 1."""
    if sink and x.shape[1] > 1:
        return x[:, :1, :], x[:, 1:, :]
    return None, x


def _split_outliers(x_norm_raw, ratio, dim, use_dense_sparse=True):
    """kvquant/quant/kv_quantizer.py:60-70: outliers on raw values, then clamp."""
    if use_dense_sparse and ratio > 0:
        dense_raw, outliers, mask = extract_outliers(x_norm_raw, ratio, dim)
    else:
        dense_raw = x_norm_raw
        outliers = np.zeros_like(x_norm_raw)
        mask = np.zeros(x_norm_raw.shape, dtype=bool)
    return np.clip(dense_raw, F32(-1.0), F32(1.0)).astype(F32), outliers, mask


def quantize_k(k: np.ndarray, codebook, scale, zero, outlier_ratio=0.01,
               sink_token=True, use_dense_sparse=True):
    """kvquant/quant/kv_quantizer.py:72-94 (pre-RoPE, per-channel keys).

    k: [B, S, C] fp16. scale/zero: [C] fp32. Returns a dict with
    ``dequant`` ([B,S,C] fp16, the reference's output), ``idx`` ([B,S',C]
    centroid indices of the quantized tokens), ``mask`` (outlier positions),
    ``norm`` (normalized raw values) and ``has_sink``.
    """
    k = np.asarray(k, dtype=F16)
    cb = np.asarray(codebook, dtype=F32).reshape(-1)
    scale = np.asarray(scale, dtype=F32)
    zero = np.asarray(zero, dtype=F32)
    k_sink, rest = _split_sink(k, sink_token)
    if rest.size == 0:
        return dict(dequant=k.copy(), idx=None, mask=None, norm=None, has_sink=False)
    n = ((rest.astype(F32) - zero) / (scale + EPS)).astype(F32)
    dense, outl, mask = _split_outliers(n, outlier_ratio, 1, use_dense_sparse)
    idx, q = lut_lookup(dense, cb)
    deq = (((q + outl).astype(F32) * scale).astype(F32) + zero).astype(F32)
    out = deq.astype(F16)
    if k_sink is not None:
        out = np.concatenate([k_sink, out], axis=1)
    return dict(dequant=out, idx=idx, mask=mask, norm=n, has_sink=k_sink is not None)


def quantize_k_thresholds(k: np.ndarray, codebook, scale, zero, thresholds):
    """Keys of appended tokens with per-channel outlier thresholds on |n|.

    The reference has no threshold path (the KVQuant paper's calibrated
    thresholds, section 3.4, are not in its code): its quantize_k on a
    one-token block (kvquant/quant/kv_quantizer.py:72-94 with k =
    max(1, int(1 * r)) = 1 per channel, dense_sparse.py:22-23) makes every
    channel an outlier, which is thresholds = 0 here. Normalization, dense
    clamp, first-minimum centroid and dequantization follow
    kv_quantizer.py:82-89 and dense_sparse.py:25-31 (outlier = x - dense).
    k: [B, S, C] fp16 (no sink); thresholds: [C] fp32. Same dict keys as
    quantize_k.
    """
    k = np.asarray(k, dtype=F16)
    cb = np.asarray(codebook, dtype=F32).reshape(-1)
    scale = np.asarray(scale, dtype=F32)
    zero = np.asarray(zero, dtype=F32)
    n = ((k.astype(F32) - zero) / (scale + EPS)).astype(F32)
    mask = np.abs(n) >= np.asarray(thresholds, dtype=F32)
    dense_raw = np.where(mask, F32(0), n).astype(F32)
    outl = (n - dense_raw).astype(F32)
    dense = np.clip(dense_raw, F32(-1.0), F32(1.0)).astype(F32)
    idx, q = lut_lookup(dense, cb)
    deq = (((q + outl).astype(F32) * scale).astype(F32) + zero).astype(F32)
    return dict(dequant=deq.astype(F16), idx=idx, mask=mask, norm=n, has_sink=False)


def value_token_stats(v_rest: np.ndarray):
    """kvquant/quant/kv_quantizer.py:103-107: per-token scale/zero over all C channels."""
    vf = v_rest.astype(F32)
    vmin = vf.min(axis=-1, keepdims=True)
    vmax = vf.max(axis=-1, keepdims=True)
    scale = ((vmax - vmin) / F32(2.0)).astype(F32)
    zero = ((vmax + vmin) / F32(2.0)).astype(F32)
    return scale, zero


def quantize_v(v: np.ndarray, codebook, outlier_ratio=0.01, sink_token=True,
               use_dense_sparse=True):
    """kvquant/quant/kv_quantizer.py:96-122 (per-token values)."""
    v = np.asarray(v, dtype=F16)
    cb = np.asarray(codebook, dtype=F32).reshape(-1)
    v_sink, rest = _split_sink(v, sink_token)
    if rest.size == 0:
        return dict(dequant=v.copy(), idx=None, mask=None, norm=None, has_sink=False,
                    scale=None, zero=None)
    vf = rest.astype(F32)
    scale, zero = value_token_stats(rest)
    n = ((vf - zero) / (scale + EPS)).astype(F32)
    dense, outl, mask = _split_outliers(n, outlier_ratio, -1, use_dense_sparse)
    idx, q = lut_lookup(dense, cb)
    deq = (((q + outl).astype(F32) * scale).astype(F32) + zero).astype(F32)
    out = deq.astype(F16)
    if v_sink is not None:
        out = np.concatenate([v_sink, out], axis=1)
    return dict(dequant=out, idx=idx, mask=mask, norm=n, has_sink=v_sink is not None,
                scale=scale[..., 0], zero=zero[..., 0])


# --------------------------------------------------------------------------
# RoPE
# --------------------------------------------------------------------------
def rope_inv_freq(dim: int, base: float) -> np.ndarray:
    """kvquant/kernels/rope_fused.py:7-8: 1 / base^(i/half) in fp32.

    The exponent i/half is an fp32 division; the power is the correctly
    rounded fp32 value (an fp64 power rounded once), which is what torch's fp32
    pow returns for these arguments (numpy's float32 power is off by up to two
    ulps); the reciprocal is an IEEE fp32 division.
    """
    half = dim // 2
    e = (np.arange(0, half, dtype=F32) / F32(half)).astype(F32)
    p = np.power(np.float64(base), e.astype(np.float64)).astype(F32)
    return (F32(1.0) / p).astype(F32)


def rope_cos_sin(seq_len: int, dim: int, base: float = 10000.0, inv_freq=None):
    """kvquant/kernels/rope_fused.py:6-12: fp32 angles outer(t, inv_freq), fp32 cos/sin."""
    f = rope_inv_freq(dim, base) if inv_freq is None else np.asarray(inv_freq, F32)
    t = np.arange(seq_len, dtype=F32)
    ang = (t[:, None] * f[None, :]).astype(F32)
    return np.cos(ang).astype(F32), np.sin(ang).astype(F32)


def rope_apply(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, pos_offset: int = 0):
    """kvquant/kernels/csrc/kvquant_ops.cu:27-55 (rotate-half, fp32 tables, fp16 out).

    x: [B, H, S, D] fp16; cos/sin: [S_total, D/2] fp32. Computed in float64 and
    rounded once to fp16.
    """
    x = np.asarray(x, dtype=F16)
    B, H, S, D = x.shape
    half = D // 2
    c = cos[pos_offset:pos_offset + S].astype(np.float64)[None, None]
    s = sin[pos_offset:pos_offset + S].astype(np.float64)[None, None]
    x1 = x[..., :half].astype(np.float64)
    x2 = x[..., half:].astype(np.float64)
    return np.concatenate([x1 * c - x2 * s, x1 * s + x2 * c], axis=-1).astype(F16)


# --------------------------------------------------------------------------
# The reference's matvec ops
# --------------------------------------------------------------------------
def lut_matvec(qmat, lut, scale, zero, vec, per_channel: bool):
    """kvquant/kernels/csrc/kvquant_ops.cu:62-100 (+ host :184-216).

    out[i] = sum_j (lut[q[i,j]] * scale[s] + zero[s]) * vec[j], s = j if
    per_channel else i; fp16 tables, exact accumulation, fp16 out.
    """
    q = np.asarray(qmat).astype(np.int64) & 0xFF
    lut = np.asarray(lut, dtype=F16).astype(np.float64)
    sc = np.asarray(scale, dtype=F16).astype(np.float64)
    zc = np.asarray(zero, dtype=F16).astype(np.float64)
    v = np.asarray(vec, dtype=F16).astype(np.float64)
    deq = lut[q]
    if per_channel:
        deq = deq * sc[None, :] + zc[None, :]
    else:
        deq = deq * sc[:, None] + zc[:, None]
    return (deq @ v).astype(F16)


def sparse_matvec_csr(row_ptr, col_idx, values, vec):
    """kvquant/kernels/csrc/kvquant_ops.cu:106-127 (+ host :218-241)."""
    rp = np.asarray(row_ptr, dtype=np.int64)
    ci = np.asarray(col_idx, dtype=np.int64)
    va = np.asarray(values, dtype=F16).astype(np.float64)
    v = np.asarray(vec, dtype=F16).astype(np.float64)
    R = rp.size - 1
    out = np.zeros(R, dtype=np.float64)
    prod = va * v[ci] if ci.size else np.zeros(0)
    for r in range(R):
        out[r] = prod[rp[r]:rp[r + 1]].sum()
    return out.astype(F16)


# --------------------------------------------------------------------------
# Decode attention restated on the reference's dequantized cache
# --------------------------------------------------------------------------
def key_scores(q, k_hat, n_kv_heads: int, inv_freq, pos0: int = 0):
    """Raw scores s[b,h,t] = q[b,h] . RoPE_{pos0+t}(K_hat[b,t,kvh]) in float64.

    K_hat is the reference's fake-quant output (kv_quantizer.py:72-94, fp16),
    RoPE uses the fp32 angle tables of rope_fused.py:6-12 (the CUDA-path
    semantics, rope_fused.py:30-34). GQA: query head h reads KV head
    h // (Hq // Hkv). q is taken as already position-rotated.
    """
    q = np.asarray(q, dtype=F16).astype(np.float64)
    B, Hq, D = q.shape
    T = k_hat.shape[1]
    half = D // 2
    cos, sin = rope_cos_sin(pos0 + T, D, inv_freq=inv_freq)
    c = cos[pos0:].astype(np.float64)[None, :, None, :]
    s = sin[pos0:].astype(np.float64)[None, :, None, :]
    K = np.asarray(k_hat, dtype=F16).astype(np.float64).reshape(B, T, n_kv_heads, D)
    k1, k2 = K[..., :half], K[..., half:]
    Kr = np.concatenate([k1 * c - k2 * s, k1 * s + k2 * c], axis=-1)  # [B,T,Hkv,D]
    G = Hq // n_kv_heads
    kv_of = np.arange(Hq) // G
    return np.einsum("bhd,bthd->bht", q, Kr[:, :, kv_of, :])


def softmax_probs(scores, head_dim: int = HEAD_DIM):
    """p = softmax(s / sqrt(D)) along tokens (float64)."""
    z = scores / math.sqrt(head_dim)
    z = z - z.max(axis=-1, keepdims=True)
    e = np.exp(z)
    return e / e.sum(axis=-1, keepdims=True)


def value_output(p, v_hat, n_kv_heads: int):
    """o[b,h,:] = sum_t p[b,h,t] V_hat[b,t,kvh,:] (V_hat from kv_quantizer.py:96-122)."""
    B, Hq, T = p.shape
    D = v_hat.shape[-1] // n_kv_heads
    V = np.asarray(v_hat, dtype=F16).astype(np.float64).reshape(B, T, n_kv_heads, D)
    G = Hq // n_kv_heads
    kv_of = np.arange(Hq) // G
    return np.einsum("bht,bthd->bhd", p, V[:, :, kv_of, :])


def decode_attention(q, k_hat, v_hat, n_kv_heads: int, inv_freq):
    s = key_scores(q, k_hat, n_kv_heads, inv_freq)
    p = softmax_probs(s, q.shape[-1])
    return s, p, value_output(p, v_hat, n_kv_heads)


def decode_shard(q, k_hat, v_hat, n_kv_heads: int, inv_freq, pos0: int):
    """Decode over the tokens at positions [pos0, pos0 + T) only (restated; the
    reference has no decode attention): (o normalized over the range, M, L)
    with M = max of s/sqrt(D) and L = sum of exp(s/sqrt(D) - M) per row."""
    s = key_scores(q, k_hat, n_kv_heads, inv_freq, pos0)
    z = s / math.sqrt(q.shape[-1])
    m = z.max(axis=-1, keepdims=True)
    e = np.exp(z - m)
    l = e.sum(axis=-1, keepdims=True)
    return value_output(e / l, v_hat, n_kv_heads), m[..., 0], l[..., 0]


def decode_fp16_path(q, k_hat, v_hat, n_kv_heads: int, inv_freq, pos0: int = 0):
    """The reference's own precision for a decode step, as the yardstick of a
    row's conditioning: K_hat (fp16, kv_quantizer.py:72-94) rotated by the
    reference's RoPE op, whose output is fp16 (kvquant_ops.cu:27-55, via
    rope_fused.py:29-34; rope_apply above), then scores, softmax and p.V in fp32
    as an attention kernel keeps them, output rounded to fp16.

    Returns (scores fp32 [B, Hq, T], output fp16 [B, Hq, D]). Where a row's
    softmax falls on a few tokens, its output moves with the last bits of its
    scores; this path's distance from the float64 decode measures that."""
    q = np.asarray(q, dtype=F16)
    B, Hq, D = q.shape
    T = k_hat.shape[1]
    cos, sin = rope_cos_sin(pos0 + T, D, inv_freq=inv_freq)
    K = np.asarray(k_hat, dtype=F16).reshape(B, T, n_kv_heads, D).transpose(0, 2, 1, 3)
    Kr = rope_apply(K, cos, sin, pos0).astype(F32)  # [B, Hkv, T, D]
    G = Hq // n_kv_heads
    kv_of = np.arange(Hq) // G
    s = np.einsum("bhd,bhtd->bht", q.astype(F32), Kr[:, kv_of]).astype(F32)
    z = s * F32(1.0 / math.sqrt(D))
    z = z - z.max(axis=-1, keepdims=True)
    e = np.exp(z)
    p = e / e.sum(axis=-1, keepdims=True)
    V = np.asarray(v_hat, dtype=F16).reshape(B, T, n_kv_heads, D).astype(F32)
    o = np.einsum("bht,bthd->bhd", p, V[:, :, kv_of]).astype(F16)
    return s, o


def merge_shards(os_, ms, ls):
    """Softmax merge of range shards: sum_i w_i o_i / sum_i w_i, w_i = L_i e^(M_i - M)."""
    m = np.max(np.stack(ms), axis=0)
    w = [l * np.exp(mi - m) for mi, l in zip(ms, ls)]
    num = sum(wi[..., None] * oi for wi, oi in zip(w, os_))
    return num / sum(w)[..., None]


# --------------------------------------------------------------------------
# Packed cache format (the library's layout; round-trips to reference indices)
# --------------------------------------------------------------------------
def slab_map(kind: str):
    """Layout of one 32-token code tile: (block, lane, pair slot) -> elements.

    A tile is 2 blocks of 16 tokens; each block holds one slab per lane
    (lane = 4*g + c, g = lane >> 2, c = lane & 3) of 32 code pairs, ordered so
    that a lane's slab is exactly its share of the tensor-core fragments of
    the decode kernels. Returns int arrays [2, 32, 32] (block, lane, slot q):
    (token_a, ch_a, token_b, ch_b) -- the pair's first and second code.

    keys (m16n8k8 A fragments: rows = tokens, k = RoPE pair halves):
        kb = q >> 1, r = q & 1: token 16*block + g + 8r, pair p = 4*kb + c,
        first = channel p, second = channel p + 64 (rotate-half partners);
    values (m16n8k16 A fragments of V^T: rows = channels, k = tokens):
        mb = q >> 2, i = q & 3: channel 16*mb + g + 8*(i & 1),
        first = token 16*block + 2c + 8*(i >> 1), second = that token + 1.
    """
    blk, lane, q = np.meshgrid(np.arange(2), np.arange(32), np.arange(32), indexing="ij")
    g, c = lane >> 2, lane & 3
    if kind == "k":
        kb, r = q >> 1, q & 1
        tok = 16 * blk + g + 8 * r
        p = 4 * kb + c
        return tok, p, tok, p + 64
    mb, i = q >> 2, q & 3
    ch = 16 * mb + g + 8 * (i & 1)
    t0 = 16 * blk + 2 * c + 8 * (i >> 1)
    return t0, ch, t0 + 1, ch


def tile_bytes(bits: int) -> int:
    return TILE_TOKENS * HEAD_DIM * bits // 8


def _slabs_to_tile(slabs: np.ndarray, bits: int) -> np.ndarray:
    """Lane slabs [..., 2, 32, 8*bits] -> tile bytes [..., 512*bits].

    Each 16-token block is stored structure-of-arrays: first bytes 0..15 of
    all 32 lane slabs (512 B), then the remaining 8*bits-16 bytes of all
    lanes, so that every copy of a lane's bytes is coalesced across the warp.
    """
    lead = slabs.shape[:-2]
    r0 = slabs[..., :16].reshape(*lead[:-1], 2, 32 * 16)
    r1 = slabs[..., 16:].reshape(*lead[:-1], 2, 32 * (8 * bits - 16))
    return np.concatenate([r0, r1], axis=-1).reshape(*lead[:-1], 512 * bits)


def _tile_to_slabs(tiles: np.ndarray, bits: int) -> np.ndarray:
    """Inverse of _slabs_to_tile: [..., 512*bits] -> [..., 2, 32, 8*bits]."""
    lead = tiles.shape[:-1]
    blocks = tiles.reshape(*lead, 2, 256 * bits)
    r0 = blocks[..., :512].reshape(*lead, 2, 32, 16)
    r1 = blocks[..., 512:].reshape(*lead, 2, 32, 8 * bits - 16)
    return np.concatenate([r0, r1], axis=-1)


def pack_codes(idx: np.ndarray, bits: int, kind: str) -> np.ndarray:
    """Pack codes [U, T, 128] -> [U, ceil(T/32), 512*bits] uint8.

    Tile = 2 blocks of 16 tokens; each block holds one slab per lane of
    8*bits bytes (stored structure-of-arrays, see _slabs_to_tile). Slot q of a
    lane's slab is the code pair of slab_map at bits [2*bits*q, 2*bits*q +
    2*bits) of the slab's little-endian bit stream, first code in the low
    `bits` bits.
    """
    idx = np.asarray(idx, dtype=np.int64)
    U, T, D = idx.shape
    assert D == HEAD_DIM
    nt = (T + TILE_TOKENS - 1) // TILE_TOKENS
    codes = np.zeros((U, nt * TILE_TOKENS, D), dtype=np.int64)
    codes[:, :T] = idx
    codes = codes.reshape(U, nt, TILE_TOKENS, D)
    ta, ca, tb, cb = slab_map(kind)
    first = codes[:, :, ta, ca]                                  # [U, nt, 2, 32, 32]
    second = codes[:, :, tb, cb]
    slots = np.stack([first, second], axis=-1).reshape(U, nt, 2, 32, 64)
    bitsarr = (slots[..., None] >> np.arange(bits)) & 1          # [.., 64, bits]
    flat = bitsarr.reshape(U, nt, 2, 32, 64 * bits).astype(np.uint8)
    slabs = np.packbits(flat, axis=-1, bitorder="little")       # [.., 8*bits]
    return _slabs_to_tile(slabs, bits)


def unpack_codes(packed: np.ndarray, bits: int, kind: str, T: int) -> np.ndarray:
    """Inverse of pack_codes: [U, nt, 512*bits] uint8 -> [U, T, 128] int64."""
    packed = np.asarray(packed, dtype=np.uint8)
    U, nt, _ = packed.shape
    slabs = _tile_to_slabs(packed, bits)
    bitsarr = np.unpackbits(slabs, axis=-1, bitorder="little").astype(np.int64)
    vals = (bitsarr.reshape(U, nt, 2, 32, 64, bits) << np.arange(bits)).sum(axis=-1)
    vals = vals.reshape(U, nt, 2, 32, 32, 2)
    out = np.empty((U, nt, TILE_TOKENS, HEAD_DIM), dtype=np.int64)
    ta, ca, tb, cb = slab_map(kind)
    out[:, :, ta, ca] = vals[..., 0]
    out[:, :, tb, cb] = vals[..., 1]
    return out.reshape(U, nt * TILE_TOKENS, HEAD_DIM)[:, :T]


def tile_outliers(mask: np.ndarray, values: np.ndarray):
    """Outliers of [U, T, 128] -> CSR over rows (unit, tile, 16-token block).

    Row r = 2 * (u * nt + tile) + blk holds the outliers of tokens
    16*blk .. 16*blk + 15 of the tile, so a tile's entries are rows 2r', 2r'+1
    back to back. Returns (values fp16 [nnz], pos uint16 [nnz] =
    (token_in_tile << 7) | d, row_ptr int32 [2*U*nt + 1]); entries of a row are
    ordered by (token, d).
    """
    U, T, D = mask.shape
    nt = (T + TILE_TOKENS - 1) // TILE_TOKENS
    half = TILE_TOKENS // 2
    m = np.zeros((U, nt * TILE_TOKENS, D), dtype=bool)
    m[:, :T] = mask
    v = np.zeros((U, nt * TILE_TOKENS, D), dtype=F32)
    v[:, :T] = values
    m = m.reshape(U * nt * 2, half * D)
    v = v.reshape(U * nt * 2, half * D)
    counts = m.sum(axis=1)
    row_ptr = np.zeros(U * nt * 2 + 1, dtype=np.int32)
    row_ptr[1:] = np.cumsum(counts)
    r, flatpos = np.nonzero(m)
    pos = (r % 2) * (half * D) + flatpos       # position within the 32-token tile
    return v[r, flatpos].astype(F16), pos.astype(np.uint16), row_ptr


def pack_entries(vals, pos) -> np.ndarray:
    """One uint32 per outlier: position in the low 16 bits, fp16 value bits high."""
    v = np.asarray(vals, dtype=F16).view(np.uint16).astype(np.uint32)
    return (np.asarray(pos, dtype=np.uint32) & 0xFFFF) | (v << 16)


def unpack_entries(ent):
    """Inverse of pack_entries: (fp16 values, uint16 positions)."""
    e = np.asarray(ent).astype(np.uint32)
    return (e >> 16).astype(np.uint16).view(F16), (e & 0xFFFF).astype(np.uint16)


def untile_outliers(vals, pos, row_ptr, U: int, T: int):
    """Inverse of tile_outliers: dense [U, T, 128] fp32 outlier matrix and mask."""
    nt = (T + TILE_TOKENS - 1) // TILE_TOKENS
    dense = np.zeros((U * nt, TILE_TOKENS * HEAD_DIM), dtype=F32)
    mask = np.zeros_like(dense, dtype=bool)
    rows = np.repeat(np.arange(U * nt * 2), np.diff(np.asarray(row_ptr, np.int64))) // 2
    p = np.asarray(pos, dtype=np.int64)
    dense[rows, p] = np.asarray(vals, dtype=F16).astype(F32)
    mask[rows, p] = True
    dense = dense.reshape(U, nt * TILE_TOKENS, HEAD_DIM)[:, :T]
    mask = mask.reshape(U, nt * TILE_TOKENS, HEAD_DIM)[:, :T]
    return dense, mask


def units_view(x_btc: np.ndarray, n_kv_heads: int) -> np.ndarray:
    """[B, T, Hkv*D] -> [B*Hkv, T, D] (unit u = b*Hkv + h)."""
    B, T, C = x_btc.shape
    D = C // n_kv_heads
    return np.ascontiguousarray(
        x_btc.reshape(B, T, n_kv_heads, D).transpose(0, 2, 1, 3).reshape(B * n_kv_heads, T, D))


def cache_from_reference_quant(kq: dict, vq: dict, k: np.ndarray, v: np.ndarray,
                               n_kv_heads: int, bits: int):
    """Expected packed cache for a prefill block, from quantize_k/quantize_v results.

    Token 0 is the fp16 sink (its code slots hold 0); tokens 1.. hold the
    reference's centroid indices. An outlier entry holds the reference's fp16
    dequantized value at its position (kv_quantizer.py:89,117: (cb[c0] + n) *
    s + z with n the normalized outlier of dense_sparse.py:31 and c0 the code
    of a dense 0), which a decoder uses in place of the dense code's value.
    """
    B, S, C = k.shape
    out = {}
    for name, qd, x in (("k", kq, k), ("v", vq, v)):
        idx = np.zeros((B, S, C), dtype=np.int64)
        mask = np.zeros((B, S, C), dtype=bool)
        val = np.zeros((B, S, C), dtype=F32)
        off = 1 if qd["has_sink"] else 0
        idx[:, off:] = qd["idx"]
        mask[:, off:] = qd["mask"]
        val[:, off:] = np.where(qd["mask"], qd["dequant"][:, off:].astype(F32), 0)
        iu = units_view(idx, n_kv_heads)
        mu = units_view(mask, n_kv_heads)
        vu = units_view(val, n_kv_heads)
        out[name + "_codes"] = pack_codes(iu, bits, name)
        ov, op, orp = tile_outliers(mu, vu)
        out[name + "_out_vals"], out[name + "_out_pos"], out[name + "_out_ptr"] = ov, op, orp
        out[name + "_out_ent"] = pack_entries(ov, op)
        out[name + "_sink"] = x[:, 0, :].copy() if qd["has_sink"] else None
    return out


# --------------------------------------------------------------------------
# CPU decode over the packed cache (the timed CPU port of the reference path)
# --------------------------------------------------------------------------
def dequant_packed(codes, out_ent, out_ptr, scale, zero, codebook, bits: int,
                   kind: str, T: int, sink=None):
    """Packed cache of U units -> K_hat / V_hat [U, T, 128] fp16, the reference's
    fake-quant dequantization cb[q] * s + z (kv_quantizer.py:89,117) at dense
    positions and the entries' fp16 dequantized values at outliers. Keys:
    scale/zero [U, 128] per channel; values: scale/zero [U, T] per token. sink:
    [U, 128] fp16 or None.
    """
    U = codes.shape[0]
    idx = unpack_codes(codes, bits, kind, T)
    cb = np.asarray(codebook, F32)
    q = cb[idx]
    out_vals, out_pos = unpack_entries(out_ent)
    o, mask = untile_outliers(out_vals, out_pos, out_ptr, U, T)
    s = np.asarray(scale, F32)
    z = np.asarray(zero, F32)
    if kind == "k":
        s, z = s[:, None, :], z[:, None, :]
    else:
        s, z = s[:, :T, None], z[:, :T, None]
    deq = ((((q + F32(0)).astype(F32)) * s).astype(F32) + z).astype(F16)
    deq = np.where(mask, o.astype(F16), deq)
    if sink is not None:
        deq[:, 0, :] = np.asarray(sink, F16)
    return deq


def decode_packed(q, k_hat_units, v_hat_units, inv_freq, group: int = 1):
    """Decode attention per unit (fp32 numpy, BLAS matmuls) on dequantized units.

    q: [U*group, 128] fp16; k_hat_units / v_hat_units: [U, T, 128] fp16.
    RoPE with fp32 angle tables (rope_fused.py:6-12), softmax(s / sqrt(128)),
    then p . V. Returns fp32 [U*group, 128].
    """
    U, T, D = k_hat_units.shape
    cos, sin = rope_cos_sin(T, D, inv_freq=inv_freq)
    out = np.empty((U * group, D), F32)
    for u in range(U):
        K = k_hat_units[u].astype(F32)
        k1, k2 = K[:, :D // 2], K[:, D // 2:]
        Kr = np.concatenate([k1 * cos - k2 * sin, k1 * sin + k2 * cos], axis=1)
        qs = q[u * group:(u + 1) * group].astype(F32)
        sc = (qs @ Kr.T) / np.float32(math.sqrt(D))
        sc -= sc.max(axis=1, keepdims=True)
        p = np.exp(sc)
        p /= p.sum(axis=1, keepdims=True)
        out[u * group:(u + 1) * group] = p @ v_hat_units[u].astype(F32)
    return out


# --------------------------------------------------------------------------
# NUQ codebook fitting (offline calibration)
# --------------------------------------------------------------------------
def codebook_degenerate(x, n_bits: int):
    """train_nuq_codebook's rules for empty input, fewer samples than clusters and
    fewer distinct values than clusters (kvquant/quant/nuq.py:20-37); None when the
    reference would run KMeans."""
    K = 2 ** n_bits
    x = np.asarray(x, dtype=F32).reshape(-1)
    if x.size == 0:
        return np.zeros(K, dtype=F32)
    if x.size < K:
        c = np.sort(x)
        return np.sort(np.concatenate([c, np.full(K - c.size, c[-1])])).astype(F32)
    u = np.unique(x)
    if u.size < K:
        return np.sort(np.concatenate([u, np.full(K - u.size, u[-1])])).astype(F32)
    return None


def kmeans_1d_inertia(x, w, centres) -> float:
    """sum_i w_i min_k (x_i - c_k)^2 in float64: the objective of the reference's
    weighted KMeans (kvquant/quant/nuq.py:39-42)."""
    x = np.asarray(x, dtype=np.float64).reshape(-1, 1)
    w = np.asarray(w, dtype=np.float64).reshape(-1)
    c = np.asarray(centres, dtype=np.float64).reshape(1, -1)
    return float(np.sum(w * np.min((x - c) ** 2, axis=1)))


def kmeans_1d_optimal(x, w, K: int) -> np.ndarray:
    """Global optimum of the weighted 1-D k-means objective (kvquant/quant/nuq.py:39-42).

    The optimal clusters are intervals of the sorted distinct values; dynamic
    programming over them, O(K n^2) time and O(n^2) memory: small n only.
    Returns the K centres ascending (fewer if there are fewer distinct values).
    """
    x = np.asarray(x, dtype=np.float64).reshape(-1)
    w = np.asarray(w, dtype=np.float64).reshape(-1)
    u, inv = np.unique(x, return_inverse=True)
    wu = np.bincount(inv, weights=w, minlength=u.size)
    n = u.size
    PW = np.concatenate([[0.0], np.cumsum(wu)])
    PS = np.concatenate([[0.0], np.cumsum(wu * u)])
    i = np.arange(n + 1)[:, None]
    j = np.arange(n + 1)[None, :]
    Wij = PW[j] - PW[i]
    Sij = PS[j] - PS[i]
    with np.errstate(divide="ignore", invalid="ignore"):
        gain = np.where(Wij > 0, Sij * Sij / np.where(Wij > 0, Wij, 1.0), 0.0)
    gain = np.where(i <= j, gain, -np.inf)
    D = gain[0].copy()
    args = []
    for _ in range(2, min(K, n) + 1):
        tot = D[:, None] + gain
        a = np.argmax(tot, axis=0)
        D = tot[a, np.arange(n + 1)]
        args.append(a)
    centres = []
    jj = n
    for a in reversed(args):
        ii = int(a[jj])
        centres.append((PS[jj] - PS[ii]) / (PW[jj] - PW[ii]) if PW[jj] > PW[ii] else np.nan)
        jj = ii
    centres.append(PS[jj] / PW[jj] if PW[jj] > 0 else np.nan)
    c = np.array(centres[::-1])
    return c[~np.isnan(c)]
