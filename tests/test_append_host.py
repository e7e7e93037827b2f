"""Decode-time append, host side (no GPU): the oracle's threshold quantizer
against the reference semantics, the appendable layout copy, and argument
checks of the C ABI."""
import numpy as np
import torch

from oracle import kvq_oracle as O
from cache_read import read_cache
import synth


def test_zero_thresholds_are_the_reference_one_token_quantize_k():
    """quantize_k on a one-token block (kv_quantizer.py:72-94) keeps every
    channel as an outlier (k = max(1, int(1 * r)) = 1); thresholds = 0 does too."""
    k, _ = synth.make_kv(2, 1, 256, seed=5)
    scale, zero = synth.key_calibration(synth.make_kv(2, 64, 256, seed=6)[0])
    cb = np.sort(np.random.default_rng(0).uniform(-1, 1, 16)).astype(np.float32)
    ref = O.quantize_k(k, cb, scale, zero, 0.01, True)
    thr = O.quantize_k_thresholds(k, cb, scale, zero, np.zeros(256, np.float32))
    assert ref["mask"].all() and thr["mask"].all()
    np.testing.assert_array_equal(ref["idx"], thr["idx"])
    np.testing.assert_array_equal(ref["dequant"], thr["dequant"])
    np.testing.assert_array_equal(ref["norm"], thr["norm"])


def test_thresholds_select_large_values_only():
    k, _ = synth.make_kv(1, 40, 128, seed=7)
    scale, zero = synth.key_calibration(k)
    cb = np.linspace(-1, 1, 8).astype(np.float32)
    thr = np.full(128, 0.5, np.float32)
    r = O.quantize_k_thresholds(k, cb, scale, zero, thr)
    np.testing.assert_array_equal(r["mask"], np.abs(r["norm"]) >= 0.5)
    # the dense part of an outlier is 0, so its code is the centroid nearest 0
    q0, _ = O.lut_lookup(np.zeros(1, np.float32), cb)
    assert np.all(r["idx"][r["mask"]] == q0[0])


def _torch_packed(kind, exp, B, H, T, bits):
    return {"q_idx": torch.from_numpy(exp[kind + "_codes"]),
            "outlier_entries": torch.from_numpy(exp[kind + "_out_ent"].view(np.int32)),
            "outlier_rowptr": torch.from_numpy(exp[kind + "_out_ptr"]),
            "kind": kind, "bits": bits, "batch": B, "n_heads": H, "h0": 0, "length": T,
            "C_full": H * 128, "outlier_ratio": 0.01,
            "scale": torch.ones((B, 32 * exp[kind + "_codes"].shape[1])),
            "zero": torch.zeros((B, 32 * exp[kind + "_codes"].shape[1]))}


def test_make_appendable_keeps_the_cache():
    """The per-unit segment copy decodes to the same codes and outliers."""
    from kvquant.kernels import make_appendable
    B, H, T, bits = 2, 3, 77, 3
    k, v = synth.make_kv(B, T, H * 128, seed=9)
    scale, zero = synth.key_calibration(k)
    cb = np.sort(np.random.default_rng(1).uniform(-1, 1, 1 << bits)).astype(np.float32)
    kq = O.quantize_k(k, cb, scale, zero, 0.02, True)
    vq = O.quantize_v(v, cb, 0.02, True)
    exp = O.cache_from_reference_quant(kq, vq, k, v, H, bits)
    for kind in ("k", "v"):
        p = _torch_packed(kind, exp, B, H, T, bits)
        a = make_appendable(p, extra_tokens=50)
        assert a["appendable"] and a["capacity"] >= T + 50
        assert a["q_idx"].shape[1] * 32 >= a["capacity"] + 32  # a spare tile
        got = read_cache(a["q_idx"].numpy(), a["outlier_rowptr"].numpy(),
                         a["outlier_entries"].numpy(), bits, kind, T)
        want = read_cache(exp[kind + "_codes"], exp[kind + "_out_ptr"], exp[kind + "_out_ent"],
                          bits, kind, T)
        for g_, w_ in zip(got, want):
            np.testing.assert_array_equal(g_, w_)
        ptr = a["outlier_rowptr"].numpy().astype(np.int64)
        R = 2 * a["q_idx"].shape[1]
        nt = -(-T // 32)
        for u in range(B * H):  # unit u's rows stay inside its own segment
            seg = ptr[u * R:u * R + 2 * nt + 1]
            assert seg[0] == u * a["ent_stride"] and seg[-1] <= (u + 1) * a["ent_stride"]


def test_append_rejects_bad_arguments_before_any_launch():
    from kvquant.kernels.cuda_ops import load_library
    lib = load_library()
    # T_old = 0: nothing to append behind
    rc = lib.kvq_append_keys(None, 1, 1, 128, 0, 1, None, None, None, None, 4, 0, None, 4, None,
                             None, 64, None, None)
    assert rc == 1 and b"T_old" in lib.kvq_last_error()
    # no spare tile after the new tokens
    rc = lib.kvq_append_values(None, 1, 1, 128, 0, 1, 0.01, None, 4, 95, None, None, 128, None,
                               3, None, None, 64, None, 0, None, None)
    assert rc == 1 and b"spare tile" in lib.kvq_last_error()
    rc = lib.kvq_append_keys(None, 1, 1, 128, 0, 1, None, None, None, None, 5, 1, None, 4, None,
                             None, 64, None, None)
    assert rc == 3


def test_cache_container_append_needs_a_stored_layer():
    import pytest
    from kvquant.kv_cache import QuantizedKVCache
    c = QuantizedKVCache()
    c.k_cache, c.v_cache = [None], [None]
    with pytest.raises(RuntimeError, match="holds no cache"):
        c.append_tokens(0, None, None)
