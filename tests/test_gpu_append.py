"""GPU parity of decode-time append (kvq_append_keys / kvq_append_values).

Values: appending tokens one call at a time must give bit for bit the cache
that quantizing the whole sequence at once gives (quantize_v is per token,
kvquant/quant/kv_quantizer.py:96-122). Keys: the appended tokens must match the
oracle's threshold quantizer bit for bit, and with zero thresholds the
reference's quantize_k on a one-token block. Decode over the grown cache must
match the oracle within the decode tolerance.
"""
import numpy as np
import pytest
import torch

from oracle import kvq_oracle as O
from cache_read import read_packed
import synth

pytestmark = pytest.mark.gpu

TOL = 2e-3


def t(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def rel_l2(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)


def chunks(T0, T1, sizes=(1, 1, 13, 2, 31, 40)):
    """Append calls covering [T0, T1): single tokens and blocks across tiles."""
    out, t0, i = [], T0, 0
    while t0 < T1:
        n = min(sizes[i % len(sizes)], T1 - t0)
        out.append((t0, t0 + n))
        t0 += n
        i += 1
    return out


@pytest.mark.parametrize("bits", [4, 3, 2])
def test_append_values_equals_whole_sequence(cuda, bits):
    from kvquant.kernels import quantize_values, make_appendable, append_values
    B, H, T0, T1, ratio = 2, 2, 70, 181, 0.01
    _, v = synth.make_kv(B, T1, H * 128, seed=11 + bits)
    cb = t(np.sort(np.random.default_rng(bits).uniform(-1, 1, 1 << bits)).astype(np.float32), cuda)
    full = quantize_values(t(v, cuda), cb, bits, ratio, True)
    pv = make_appendable(quantize_values(t(v[:, :T0], cuda), cb, bits, ratio, True), T1 - T0)
    for a, b in chunks(T0, T1):
        append_values(pv, t(v[:, a:b], cuda))
    assert pv["length"] == T1
    for g_, w_ in zip(read_packed(pv), read_packed(full)):
        np.testing.assert_array_equal(g_, w_)
    np.testing.assert_array_equal(pv["scale"][:, :T1].cpu().numpy(), full["scale"][:, :T1].cpu().numpy())
    np.testing.assert_array_equal(pv["zero"][:, :T1].cpu().numpy(), full["zero"][:, :T1].cpu().numpy())


def _key_case(cuda, bits, B=2, H=2, T0=45, T1=150, ratio=0.01, seed=21, calib_all=False):
    from kvquant.kernels import quantize_keys, make_appendable, key_outlier_thresholds
    k, v = synth.make_kv(B, T1, H * 128, seed=seed)
    # calibration on the prefill block (appended keys may leave its range) or on
    # the whole sequence (a calibration set that covers the later tokens)
    scale, zero = synth.key_calibration(k if calib_all else k[:, :T0])
    cb = np.sort(np.random.default_rng(seed).uniform(-1, 1, 1 << bits)).astype(np.float32)
    pk0 = quantize_keys(t(k[:, :T0], cuda), t(scale, cuda), t(zero, cuda), t(cb, cuda), bits,
                        ratio, True)
    thr = key_outlier_thresholds(t(k[:, :T0], cuda), t(scale, cuda), t(zero, cuda), ratio)
    return k, v, scale, zero, cb, pk0, thr, make_appendable(pk0, T1 - T0)


@pytest.mark.parametrize("bits", [4, 3, 2])
def test_append_keys_threshold_parity(cuda, bits):
    from kvquant.kernels import append_keys
    T0, T1 = 45, 150
    k, _, scale, zero, cb, pk0, thr, pk = _key_case(cuda, bits, T0=T0, T1=T1)
    old = read_packed(pk0)
    for a, b in chunks(T0, T1):
        append_keys(pk, t(k[:, a:b], cuda), thr)
    idx, mask, vals = read_packed(pk)
    H = pk["n_heads"]
    exp = O.quantize_k_thresholds(k[:, T0:], cb, scale, zero, thr.cpu().numpy())
    e_idx = O.units_view(exp["idx"], H)
    e_mask = O.units_view(exp["mask"], H)
    # an entry holds the dequantized key at its position
    e_val = O.units_view(np.where(exp["mask"], exp["dequant"].astype(np.float32), 0), H)
    for g_, o_ in zip((idx, mask, vals), old):  # the prefill part is untouched
        np.testing.assert_array_equal(g_[:, :T0], o_)
    np.testing.assert_array_equal(idx[:, T0:], e_idx)
    np.testing.assert_array_equal(mask[:, T0:], e_mask)
    np.testing.assert_array_equal(vals[:, T0:], e_val)
    assert 0 < e_mask.mean() < 0.05  # calibrated thresholds keep about the outlier share


def test_append_keys_zero_thresholds_is_reference_one_token(cuda):
    """thresholds = 0: every channel of the new token is an outlier, as in the
    reference's quantize_k on the one-token block of a decode step."""
    from kvquant.kernels import append_keys
    T0 = 64
    k, _, scale, zero, cb, _, _, pk = _key_case(cuda, 4, T0=T0, T1=T0 + 2)
    zeros = torch.zeros(pk["n_heads"] * 128, device=cuda)
    for a in (T0, T0 + 1):
        append_keys(pk, t(k[:, a:a + 1], cuda), zeros)
        ref = O.quantize_k(k[:, a:a + 1], cb, scale, zero, 0.01, True)
        idx, mask, vals = read_packed(pk)
        np.testing.assert_array_equal(idx[:, a:a + 1], O.units_view(ref["idx"], pk["n_heads"]))
        assert mask[:, a].all()
        np.testing.assert_array_equal(
            vals[:, a:a + 1], O.units_view(ref["dequant"].astype(np.float32), pk["n_heads"]))


def test_decode_after_appends(cuda):
    """decode_attention (and the key scores) over a prefill + appended cache
    against the oracle. The key calibration covers the whole sequence, as a
    calibration set would, and the query is scaled by 1/4: with N(0,1) queries
    this synthetic layer's scores reach +-600 and the softmax puts > 0.99 on one
    token, where the 1e-3 score error of the fp16 kernels (the same for the
    prefill and the appended tokens) turns into output errors near 2e-3 even for
    a cache built in one prefill block."""
    from kvquant.kernels import (quantize_values, make_appendable, append_keys, append_values,
                                 decode_attention, qk_scores, rope_inv_freq)
    B, H, G, T0, T1, bits, ratio = 1, 2, 2, 200, 333, 4, 0.01
    k, v, scale, zero, cb, _, thr, pk = _key_case(cuda, bits, B=B, H=H, T0=T0, T1=T1, seed=31,
                                                  calib_all=True)
    pv = make_appendable(quantize_values(t(v[:, :T0], cuda), t(cb, cuda), bits, ratio, True),
                         T1 - T0)
    for a, b in chunks(T0, T1):
        append_keys(pk, t(k[:, a:b], cuda), thr)
        append_values(pv, t(v[:, a:b], cuda))
    q = (synth.make_query(B, H * G, 128, seed=3).astype(np.float32) * 0.25).astype(np.float16)
    out = decode_attention(t(q, cuda), pk, pv, rope_inv_freq(128, 10000.0)).cpu().numpy()
    scores = qk_scores(t(q, cuda), pk, rope_inv_freq(128, 10000.0)).cpu().numpy()
    k_hat = np.concatenate([O.quantize_k(k[:, :T0], cb, scale, zero, ratio, True)["dequant"],
                            O.quantize_k_thresholds(k[:, T0:], cb, scale, zero,
                                                    thr.cpu().numpy())["dequant"]], axis=1)
    v_hat = O.quantize_v(v, cb, ratio, True)["dequant"]
    ref_s, _, ref = O.decode_attention(q, k_hat, v_hat, H, O.rope_inv_freq(128, 10000.0))
    assert rel_l2(scores, ref_s) <= TOL, rel_l2(scores, ref_s)
    assert rel_l2(out, ref) <= TOL, rel_l2(out, ref)


def test_full_segment_is_reported_and_left_alone(cuda):
    from kvquant.kernels import quantize_keys, make_appendable, append_keys
    k, _ = synth.make_kv(1, 40, 256, seed=41)
    scale, zero = synth.key_calibration(k)
    cb = t(np.linspace(-1, 1, 16).astype(np.float32), cuda)
    pk = make_appendable(quantize_keys(t(k[:, :32], cuda), t(scale, cuda), t(zero, cuda), cb, 4,
                                       0.01, True), 8, entries_per_token=1)
    before = (pk["q_idx"].clone(), pk["outlier_rowptr"].clone(), pk["outlier_entries"].clone())
    with pytest.raises(RuntimeError, match="segment is full"):
        append_keys(pk, t(k[:, 32:40], cuda), torch.zeros(256, device=cuda))
    assert pk["length"] == 32
    for a, b in zip(before, (pk["q_idx"], pk["outlier_rowptr"], pk["outlier_entries"])):
        assert torch.equal(a, b)
    # without outliers the same append fits
    append_keys(pk, t(k[:, 32:40], cuda), None)
    assert pk["length"] == 40


def test_regrow_and_append_again(cuda):
    """make_appendable on a grown cache gives more room; values stay identical
    to quantizing the whole sequence at once."""
    from kvquant.kernels import quantize_values, make_appendable, append_values
    B, H, bits, ratio = 1, 3, 4, 0.02
    _, v = synth.make_kv(B, 120, H * 128, seed=51)
    cb = t(np.linspace(-1, 1, 16).astype(np.float32), cuda)
    pv = make_appendable(quantize_values(t(v[:, :40], cuda), cb, bits, ratio, True), 10)
    append_values(pv, t(v[:, 40:50], cuda))
    with pytest.raises(RuntimeError, match="capacity"):
        append_values(pv, t(v[:, 50:120], cuda))
    pv = make_appendable(pv, 70)
    append_values(pv, t(v[:, 50:51], cuda))
    append_values(pv, t(v[:, 51:120], cuda))
    full = quantize_values(t(v, cuda), cb, bits, ratio, True)
    for g_, w_ in zip(read_packed(pv), read_packed(full)):
        np.testing.assert_array_equal(g_, w_)
