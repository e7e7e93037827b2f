"""Generates the golden fixtures under tests/golden/ by running the reference.

Run in a container where the reference project is mounted (read-only) at
/root/reference:

    python tests/golden/make_golden.py [--ref /root/reference]

It imports the reference's own PyTorch code on the CPU and records, for seeded
synthetic inputs (tests/synth.py), what the reference computes:
  * KVQuantizer.quantize_k / quantize_v outputs (fake-quant fp16), plus the
    centroid indices, outlier masks and normalized values they come from
    (kvquant/quant/kv_quantizer.py:72-122, dense_sparse.py:4-32);
  * NUQ codebooks fit by train_nuq_codebook (kvquant/quant/nuq.py:6-44) with
    the calibration weighting of kvquant/calibration.py:114-125 (Fisher = 1);
  * _lut_lookup, extract_outliers, pack_csr, the CPU fallbacks of
    dense_matvec_lut / sparse_matvec_csr, the RoPE tables of _build_cos_sin
    and the CPU path of apply_rope_elementwise;
  * decode attention restated in float64 on the reference's K_hat/V_hat with
    the reference's fp32 RoPE tables (the reference has no decode attention).
The product never reads these files; tests compare the oracle and the GPU
kernels against them.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))  # tests/ for synth

import synth  # noqa: E402

QUANT_CASES = [
    # name, B, S, C(=Hkv*128), G, bits, ratio, sink, seed, kind of data, rope base
    ("cfg0_4bit", 1, 161, 256, 1, 4, 0.01, True, 0, "normal", 10000.0),
    ("cfg1_3bit", 1, 300, 256, 1, 3, 0.005, True, 1, "normal", 10000.0),
    ("cfg2_2bit_gqa", 2, 97, 256, 4, 2, 0.01, True, 2, "normal", 500000.0),
    ("ties_4bit", 1, 129, 256, 1, 4, 0.03, True, 3, "ties", 10000.0),
    ("nosink_4bit", 1, 70, 128, 1, 4, 0.02, False, 4, "normal", 10000.0),
    ("s2_4bit", 1, 2, 128, 1, 4, 0.01, True, 5, "normal", 10000.0),
    ("s1_4bit", 1, 1, 128, 1, 4, 0.01, True, 6, "normal", 10000.0),
    ("noout_3bit", 1, 65, 128, 1, 3, 0.0, True, 7, "normal", 10000.0),
]


def tie_data(B, S, C, seed):
    rng = np.random.default_rng(seed)
    k = rng.integers(-3, 4, size=(B, S, C)).astype(np.float16)
    v = rng.integers(-3, 4, size=(B, S, C)).astype(np.float16)
    return k, v


def fit_codebooks(ref, torch, k, v, scale, zero, bits, ratio, sink):
    """Codebooks as kvquant/calibration.py:107-125 and :133-155 would fit them."""
    from kvquant.quant.dense_sparse import extract_outliers
    from kvquant.quant.nuq import train_nuq_codebook

    off = 1 if (sink and k.shape[1] > 1) else 0
    kt = torch.from_numpy(k[:, off:].astype(np.float32)).reshape(-1, k.shape[-1])
    vt = torch.from_numpy(v[:, off:].astype(np.float32)).reshape(-1, v.shape[-1])
    sc = torch.from_numpy(scale)
    ze = torch.from_numpy(zero)
    kn = (kt - ze) / (sc + 1e-8)
    dense_raw, _, kmask = extract_outliers(kn, outlier_ratio=max(ratio, 1e-9), dim=0)
    dense_k = torch.clamp(dense_raw, -1.0, 1.0)
    wk = (sc ** 2).unsqueeze(0).expand_as(dense_k)
    ktr, wktr = dense_k[~kmask], wk[~kmask]
    vmin = vt.min(dim=-1, keepdim=True).values
    vmax = vt.max(dim=-1, keepdim=True).values
    vs, vz = (vmax - vmin) / 2.0, (vmax + vmin) / 2.0
    vn = (vt - vz) / (vs + 1e-8)
    dense_raw_v, _, vmask = extract_outliers(vn, outlier_ratio=max(ratio, 1e-9), dim=-1)
    dense_v = torch.clamp(dense_raw_v, -1.0, 1.0)
    wv = (vs ** 2).expand_as(dense_v)
    vtr, wvtr = dense_v[~vmask], wv[~vmask]
    rng = np.random.default_rng(123)

    def sub(x, w, n=20000):
        if x.numel() > n:
            idx = torch.from_numpy(rng.choice(x.numel(), n, replace=False))
            return x[idx], w[idx]
        return x, w

    cbk = train_nuq_codebook(*sub(ktr, wktr), n_bits=bits).numpy().astype(np.float32)
    cbv = train_nuq_codebook(*sub(vtr, wvtr), n_bits=bits).numpy().astype(np.float32)
    return cbk, cbv


def quant_case(ref, torch, case):
    from kvquant.quant.kv_quantizer import KVQuantizer
    from kvquant.quant.dense_sparse import extract_outliers
    from kvquant.kernels.rope_fused import _build_cos_sin

    name, B, S, C, G, bits, ratio, sink, seed, kind, base = case
    if kind == "ties":
        k, v = tie_data(B, S, C, seed)
    else:
        k, v = synth.make_kv(B, S, C, seed=seed)
    if S > 1:
        scale, zero = synth.key_calibration(k, sink)
    else:
        scale, zero = synth.key_calibration(k, False)
    cbk, cbv = fit_codebooks(ref, torch, k, v, scale, zero, bits, ratio, sink)
    qz = KVQuantizer([torch.from_numpy(cbk)], [torch.from_numpy(cbv)],
                     [torch.from_numpy(scale)], [torch.from_numpy(zero)],
                     k_bits=bits, v_bits=bits, outlier_ratio=ratio, sink_token=sink,
                     use_dense_sparse=True)
    kt, vt = torch.from_numpy(k), torch.from_numpy(v)
    k_deq = qz.quantize_k(0, kt).numpy()
    v_deq = qz.quantize_v(0, vt).numpy()
    out = dict(k=k, v=v, scale=scale, zero=zero, cb_k=cbk, cb_v=cbv,
               meta=np.array([B, S, C, G, bits, int(sink)], dtype=np.int64),
               ratio=np.float64(ratio), base=np.float64(base),
               k_dequant=k_deq, v_dequant=v_deq)
    # Intermediates, recomputed exactly as quantize_k / quantize_v do.
    _, k_rest = KVQuantizer._split_sink(kt, sink)
    _, v_rest = KVQuantizer._split_sink(vt, sink)
    if k_rest.numel():
        kn = (k_rest.float() - torch.from_numpy(zero)) / (torch.from_numpy(scale) + 1e-8)
        vf = v_rest.float()
        vmin = vf.min(dim=-1, keepdim=True).values
        vmax = vf.max(dim=-1, keepdim=True).values
        vs, vz = (vmax - vmin) / 2.0, (vmax + vmin) / 2.0
        vn = (vf - vz) / (vs + 1e-8)
        for tag, xn, dim in (("k", kn, 1), ("v", vn, -1)):
            if ratio > 0:
                dense_raw, _, mask = extract_outliers(xn, outlier_ratio=ratio, dim=dim)
            else:
                dense_raw, mask = xn, torch.zeros_like(xn, dtype=torch.bool)
            dense = torch.clamp(dense_raw, -1.0, 1.0)
            from kvquant.quant.kv_quantizer import _lut_lookup
            idx, _ = _lut_lookup(dense, torch.from_numpy(cbk if tag == "k" else cbv))
            out[f"{tag}_idx"] = idx.numpy().astype(np.uint8)
            out[f"{tag}_mask"] = np.packbits(mask.numpy().reshape(-1))
            out[f"{tag}_norm_at_mask"] = xn.numpy()[mask.numpy()].astype(np.float32)
        out["v_scale"] = vs.numpy()[..., 0]
        out["v_zero"] = vz.numpy()[..., 0]
        # pack_csr of the key outlier matrix of batch 0 (token-major CSR)
        kmask = np.unpackbits(out["k_mask"])[:kn.numel()].reshape(kn.shape).astype(bool)
        om = np.where(kmask, kn.numpy(), 0).astype(np.float32)[0]
        from kvquant.quant.dense_sparse import pack_csr
        vals, cols, rp = pack_csr(torch.from_numpy(om))
        out["csr_vals"], out["csr_cols"], out["csr_rowptr"] = vals.numpy(), cols.numpy(), rp.numpy()
    # Decode attention on the reference's K_hat / V_hat (float64).
    Hkv = C // 128
    Hq = Hkv * G
    q = synth.make_query(B, Hq, 128, seed=seed + 100)
    cos, sin = _build_cos_sin(S, 128, "cpu", dtype=torch.float32, base=base)
    c = cos.numpy().astype(np.float64)[None, :, None, :]
    s = sin.numpy().astype(np.float64)[None, :, None, :]
    K = k_deq.astype(np.float64).reshape(B, S, Hkv, 128)
    Kr = np.concatenate([K[..., :64] * c - K[..., 64:] * s, K[..., :64] * s + K[..., 64:] * c], -1)
    kv_of = np.arange(Hq) // G
    scores = np.einsum("bhd,bthd->bht", q.astype(np.float64), Kr[:, :, kv_of, :])
    z = scores / np.sqrt(128.0)
    p = np.exp(z - z.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    V = v_deq.astype(np.float64).reshape(B, S, Hkv, 128)
    o = np.einsum("bht,bthd->bhd", p, V[:, :, kv_of, :])
    out.update(q=q, scores=scores, probs=p, attn_out=o)
    return name, out


def misc(ref, torch):
    from kvquant.kernels.rope_fused import _build_cos_sin, apply_rope_elementwise
    from kvquant.kernels.matvec_ds import dense_matvec_lut, sparse_matvec_csr
    from kvquant.quant.kv_quantizer import _lut_lookup
    from kvquant.quant.dense_sparse import extract_outliers

    out = {}
    rows = np.array([0, 1, 2, 31, 32, 1000, 4095, 8191, 32767, 65535, 131071,
                     524287, 1048575], dtype=np.int64)
    for base in (10000.0, 500000.0):
        cos, sin = _build_cos_sin(1 << 20, 128, "cpu", dtype=torch.float32, base=base)
        tag = f"b{int(base)}"
        out[f"cos_{tag}"] = cos.numpy()[rows]
        out[f"sin_{tag}"] = sin.numpy()[rows]
        half = 64
        inv = 1.0 / (base ** (torch.arange(0, half, dtype=torch.float32) / half))
        out[f"inv_freq_{tag}"] = inv.numpy()
        del cos, sin
    out["rope_rows"] = rows
    rng = np.random.default_rng(11)
    x = rng.standard_normal((2, 3, 5, 128), dtype=np.float32).astype(np.float16)
    out["rope_x"] = x
    out["rope_cpu_out"] = apply_rope_elementwise(torch.from_numpy(x), position_offset=7).numpy()
    # lut lookup with exact ties (midpoints) and values equal to centroids
    cb = np.sort(rng.uniform(-1, 1, 16)).astype(np.float32)
    mids = ((cb[1:] + cb[:-1]) / 2).astype(np.float32)
    xs = np.concatenate([rng.uniform(-1.2, 1.2, 5000).astype(np.float32), cb, mids,
                         np.array([0.0, -0.0, 1.0, -1.0], np.float32)])
    idx, dq = _lut_lookup(torch.from_numpy(xs), torch.from_numpy(cb))
    out.update(lut_cb=cb, lut_x=xs, lut_idx=idx.numpy(), lut_dq=dq.numpy())
    dq2 = dense_matvec_lut(torch.from_numpy(xs.reshape(-1, 5)), torch.from_numpy(cb))
    out["dense_matvec_lut_out"] = dq2.numpy()
    # extract_outliers on data without ties
    y = rng.standard_normal((3, 40, 12), dtype=np.float32)
    for dim in (1, -1):
        _, o, m = extract_outliers(torch.from_numpy(y), outlier_ratio=0.1, dim=dim)
        out[f"eo_mask_dim{dim}"] = m.numpy()
    out["eo_x"] = y
    # sparse matvec (CPU fallback of the reference)
    R, Cc = 50, 64
    dense = np.where(rng.random((R, Cc)) < 0.1, rng.standard_normal((R, Cc)), 0).astype(np.float16)
    dense[7] = 0  # an empty row
    mask = dense != 0
    vals = dense[mask]
    cols = np.nonzero(mask)[1].astype(np.int32)
    rp = np.zeros(R + 1, np.int32)
    rp[1:] = np.cumsum(mask.sum(1))
    vec = rng.standard_normal(Cc).astype(np.float16)
    sm = sparse_matvec_csr(torch.from_numpy(rp), torch.from_numpy(cols), torch.from_numpy(vals),
                           torch.from_numpy(vec))
    out.update(sp_rowptr=rp, sp_cols=cols, sp_vals=vals, sp_vec=vec, sp_out=sm.numpy())
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    import torch
    import kvquant  # the reference package

    torch.manual_seed(0)
    for case in QUANT_CASES:
        name, out = quant_case(kvquant, torch, case)
        np.savez_compressed(HERE / f"quant_{name}.npz", **out)
        print("wrote", name)
    np.savez_compressed(HERE / "misc.npz", **misc(kvquant, torch))
    print("wrote misc")


if __name__ == "__main__":
    main()
