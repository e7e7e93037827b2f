"""GPU parity of quantize-on-append: codes, outlier positions and values bit-exact.

Checked against (a) the reference's own outputs (golden fixtures) and (b) the
oracle's packed cache for the same inputs.
"""
import numpy as np
import pytest
import torch

from oracle import kvq_oracle as O
from goldens import QUANT_CASES, load_quant
import synth

pytestmark = pytest.mark.gpu


def t(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def run_quant(g, cuda, capacity=None):
    from kvquant.kernels import quantize_keys, quantize_values
    pk = quantize_keys(t(g["k"], cuda), t(g["scale"], cuda), t(g["zero"], cuda),
                       t(g["cb_k"], cuda), g["bits"], g["ratio"], g["sink"],
                       capacity=capacity, dequant=True)
    pv = quantize_values(t(g["v"], cuda), t(g["cb_v"], cuda), g["bits"], g["ratio"], g["sink"],
                         capacity=capacity, dequant=True)
    return pk, pv


def expected_cache(g):
    kq = O.quantize_k(g["k"], g["cb_k"], g["scale"], g["zero"], g["ratio"], g["sink"])
    vq = O.quantize_v(g["v"], g["cb_v"], g["ratio"], g["sink"])
    exp = O.cache_from_reference_quant(kq, vq, g["k"], g["v"], g["C"] // 128, g["bits"])
    return kq, vq, exp


def check_packed(p, exp, tag, nt):
    codes = p["q_idx"].cpu().numpy()
    U, nt_cap = codes.shape[:2]
    np.testing.assert_array_equal(codes[:, :nt], exp[f"{tag}_codes"])
    rp = p["outlier_rowptr"].cpu().numpy()
    if nt_cap != nt:
        rp = _compact_rowptr(rp, U, nt_cap, nt)
    np.testing.assert_array_equal(rp, exp[f"{tag}_out_ptr"])
    np.testing.assert_array_equal(p["outlier_values"].cpu().numpy().view(np.uint16),
                                  exp[f"{tag}_out_vals"].view(np.uint16))
    np.testing.assert_array_equal(p["outlier_cols"].cpu().numpy().view(np.uint16),
                                  exp[f"{tag}_out_pos"])
    nnz = p["nnz"]
    np.testing.assert_array_equal(p["outlier_entries"].cpu().numpy()[:nnz].view(np.uint32),
                                  exp[f"{tag}_out_ent"])


def _compact_rowptr(rp, U, nt_cap, nt):
    """Row pointer over (unit, tile < nt, block) from one over (unit, tile < nt_cap, block)."""
    out = [0]
    for u in range(U):
        for r in range(2 * u * nt_cap, 2 * (u * nt_cap + nt)):
            out.append(out[-1] + rp[r + 1] - rp[r])
    return np.array(out, dtype=np.int32)


@pytest.mark.parametrize("name", QUANT_CASES)
def test_quantize_matches_reference_and_oracle(cuda, name):
    g = load_quant(name)
    pk, pv = run_quant(g, cuda)
    kq, vq, exp = expected_cache(g)
    nt = -(-g["S"] // 32)
    # fake-quant output: the oracle shares the tie rule; the reference matches
    # wherever its (unspecified) tie order agrees, i.e. in every non-tie case
    for p, q, tag in ((pk, kq, "k"), (pv, vq, "v")):
        got = p["dequant"].cpu().numpy()
        np.testing.assert_array_equal(got.view(np.uint16), q["dequant"].view(np.uint16))
        if not name.startswith("ties"):
            np.testing.assert_array_equal(got.view(np.uint16), g[f"{tag}_dequant"].view(np.uint16))
        check_packed(p, exp, tag, nt)
    if g["S"] > 1 and g["sink"]:
        np.testing.assert_array_equal(pk["sink"].cpu().numpy(), g["k"][:, 0])
        np.testing.assert_array_equal(pv["sink"].cpu().numpy(), g["v"][:, 0])
    if vq["scale"] is not None:
        off = g["off"]
        np.testing.assert_array_equal(pv["scale"].cpu().numpy()[:, off:g["S"]], vq["scale"])
        np.testing.assert_array_equal(pv["zero"].cpu().numpy()[:, off:g["S"]], vq["zero"])


def test_quantize_with_capacity(cuda):
    g = load_quant("cfg0_4bit")
    pk, pv = run_quant(g, cuda, capacity=1000)
    _, _, exp = expected_cache(g)
    nt = -(-g["S"] // 32)
    assert pk["q_idx"].shape[1] == 32
    check_packed(pk, exp, "k", nt)
    check_packed(pv, exp, "v", nt)
    assert int(pk["q_idx"][:, nt:].abs().sum()) == 0


def test_kvquantizer_drop_in_bit_exact(cuda):
    from kvquant import KVQuantizer
    for name in ("cfg0_4bit", "cfg1_3bit", "cfg2_2bit_gqa", "s1_4bit", "noout_3bit"):
        g = load_quant(name)
        qz = KVQuantizer([t(g["cb_k"], cuda)], [t(g["cb_v"], cuda)], [t(g["scale"], cuda)],
                         [t(g["zero"], cuda)], k_bits=g["bits"], v_bits=g["bits"],
                         outlier_ratio=g["ratio"], sink_token=g["sink"])
        k = qz.quantize_k(0, t(g["k"], cuda)).cpu().numpy()
        v = qz.quantize_v(0, t(g["v"], cuda)).cpu().numpy()
        np.testing.assert_array_equal(k.view(np.uint16), g["k_dequant"].view(np.uint16))
        np.testing.assert_array_equal(v.view(np.uint16), g["v_dequant"].view(np.uint16))


@pytest.mark.parametrize("bits,ratio,B,S,H,h0,nh", [(4, 0.01, 1, 4096, 4, 0, 4),
                                                    (3, 0.005, 1, 2048, 4, 1, 2),
                                                    (2, 0.01, 3, 517, 2, 0, 2)])
def test_quantize_larger_blocks(cuda, bits, ratio, B, S, H, h0, nh):
    """Bigger blocks and a head sub-range (as one rank of a head-sharded run sees it)."""
    from kvquant.kernels import quantize_keys, quantize_values
    C = H * 128
    k, v = synth.make_kv(B, S, C, seed=bits)
    scale, zero = synth.key_calibration(k)
    cb = np.sort(np.random.default_rng(bits).uniform(-1, 1, 1 << bits)).astype(np.float32)
    pk = quantize_keys(t(k, cuda), t(scale, cuda), t(zero, cuda), t(cb, cuda), bits, ratio, True,
                       h0=h0, n_heads=nh, dequant=True)
    pv = quantize_values(t(v, cuda), t(cb, cuda), bits, ratio, True, h0=h0, n_heads=nh,
                         dequant=True)
    cs = slice(h0 * 128, (h0 + nh) * 128)
    kq = O.quantize_k(k[:, :, cs], cb, scale[cs], zero[cs], ratio, True)
    vq = O.quantize_v(v, cb, ratio, True)  # per-token stats span all channels
    np.testing.assert_array_equal(pk["dequant"].cpu().numpy().view(np.uint16),
                                  kq["dequant"].view(np.uint16))
    np.testing.assert_array_equal(pv["dequant"].cpu().numpy().view(np.uint16),
                                  vq["dequant"][:, :, cs].view(np.uint16))
    # packed codes round-trip to the reference indices
    nt = -(-S // 32)
    codes = O.unpack_codes(pk["q_idx"].cpu().numpy(), bits, "k", S)
    idx = np.zeros((B, S, nh * 128), np.int64)
    idx[:, 1:] = kq["idx"]
    np.testing.assert_array_equal(codes, O.units_view(idx, nh))
    vcodes = O.unpack_codes(pv["q_idx"].cpu().numpy(), bits, "v", S)
    vidx = np.zeros((B, S, C), np.int64)
    vidx[:, 1:] = vq["idx"]
    np.testing.assert_array_equal(vcodes, O.units_view(vidx[:, :, cs], nh))
    # outlier positions and fp16 values
    d, m = O.untile_outliers(pk["outlier_values"].cpu().numpy(),
                             pk["outlier_cols"].cpu().numpy().view(np.uint16),
                             pk["outlier_rowptr"].cpu().numpy(), B * nh, S)
    kmask = np.zeros((B, S, nh * 128), bool)
    kmask[:, 1:] = kq["mask"]
    np.testing.assert_array_equal(m, O.units_view(kmask, nh))
    assert pk["nnz"] == B * nh * 128 * O.outlier_count(S - 1, ratio)
    assert nt == pk["q_idx"].shape[1]
