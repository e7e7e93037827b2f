"""GPU parity of the decode path (key kernel, softmax, value kernel).

Reference: fp32/float64 attention restated on the reference's own fake-quant
K_hat / V_hat (the oracle, pinned to the reference by test_oracle_golden.py).
Tolerance: relative L2 error <= 2e-3 for scores and outputs (fp16 cache
values and fp32 math against a float64 reference).
"""
import numpy as np
import pytest
import torch

from oracle import kvq_oracle as O
from goldens import QUANT_CASES, load_quant
import synth

pytestmark = pytest.mark.gpu

TOL = 2e-3


def t(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def rel_l2(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)


def build(cuda, k, v, scale, zero, cbk, cbv, bits, ratio, sink=True, capacity=None):
    from kvquant.kernels import quantize_keys, quantize_values
    pk = quantize_keys(t(k, cuda), t(scale, cuda), t(zero, cuda), t(cbk, cuda), bits, ratio, sink,
                       capacity=capacity)
    pv = quantize_values(t(v, cuda), t(cbv, cuda), bits, ratio, sink, capacity=capacity)
    return pk, pv


@pytest.mark.parametrize("name", QUANT_CASES)
def test_decode_golden_cases(cuda, name):
    from kvquant.kernels import qk_scores, softmax, pv_out, decode_attention, rope_inv_freq
    g = load_quant(name)
    pk, pv = build(cuda, g["k"], g["v"], g["scale"], g["zero"], g["cb_k"], g["cb_v"], g["bits"],
                   g["ratio"], g["sink"])
    inv = rope_inv_freq(128, g["base"])
    q = t(g["q"], cuda)
    s = qk_scores(q, pk, inv).cpu().numpy()
    assert rel_l2(s, g["scores"]) <= TOL, rel_l2(s, g["scores"])
    p = softmax(torch.from_numpy(g["scores"].astype(np.float32)).to(cuda)).cpu().numpy()
    assert rel_l2(p, g["probs"]) <= 1e-5
    o = pv_out(torch.from_numpy(g["probs"].astype(np.float32)).to(cuda), pv).cpu().numpy()
    assert rel_l2(o, g["attn_out"]) <= TOL, rel_l2(o, g["attn_out"])
    o2 = decode_attention(q, pk, pv, inv).cpu().numpy()
    assert rel_l2(o2, g["attn_out"]) <= TOL, rel_l2(o2, g["attn_out"])


def _config_case(cuda, B, Hkv, G, T, bits, ratio, base, seed, heads_checked=None):
    from kvquant.kernels import qk_scores, decode_attention, rope_inv_freq
    C = Hkv * 128
    k, v = synth.make_kv(B, T, C, seed=seed)
    scale, zero = synth.key_calibration(k)
    rng = np.random.default_rng(seed)
    cbk = np.sort(rng.uniform(-1, 1, 1 << bits)).astype(np.float32)
    cbv = np.sort(rng.uniform(-1, 1, 1 << bits)).astype(np.float32)
    pk, pv = build(cuda, k, v, scale, zero, cbk, cbv, bits, ratio)
    q = synth.make_query(B, Hkv * G, 128, seed=seed + 1)
    inv = rope_inv_freq(128, base)
    s = qk_scores(t(q, cuda), pk, inv).cpu().numpy()
    o = decode_attention(t(q, cuda), pk, pv, inv).cpu().numpy()
    # oracle on a subset of KV heads (keys are per channel; value stats need all C)
    hs = list(range(Hkv)) if heads_checked is None else heads_checked
    cs = np.concatenate([np.arange(h * 128, (h + 1) * 128) for h in hs])
    kq = O.quantize_k(k[:, :, cs], cbk, scale[cs], zero[cs], ratio, True)
    vq = O.quantize_v(v, cbv, ratio, True)
    qh = np.concatenate([np.arange(h * G, (h + 1) * G) for h in hs])
    rs, _, ro = O.decode_attention(q[:, qh], kq["dequant"], vq["dequant"][:, :, cs], len(hs),
                                   O.rope_inv_freq(128, base))
    es, eo = rel_l2(s[:, qh], rs), rel_l2(o[:, qh], ro)
    assert es <= TOL and eo <= TOL, (es, eo)
    return es, eo


def test_cfg0_full(cuda):
    """LLaMA-7B layer: B1, 32 heads, T=4096, 4-bit, 1% outliers, theta 10000."""
    _config_case(cuda, 1, 32, 1, 4096, 4, 0.01, 10000.0, 0, heads_checked=[0, 7, 31])


@pytest.mark.parametrize("T", [2048, 8192])
def test_cfg1_sweep(cuda, T):
    """3-bit, 0.5% outliers, 32 heads."""
    _config_case(cuda, 1, 32, 1, T, 3, 0.005, 10000.0, 1, heads_checked=[3, 30])


def test_cfg2_gqa_2bit(cuda):
    """GQA: 4 query heads per KV head, 2-bit, theta 500000 (B reduced for the oracle)."""
    _config_case(cuda, 4, 8, 4, 1024, 2, 0.01, 500000.0, 2, heads_checked=[0, 5])


@pytest.mark.parametrize("G", [1, 2, 8])
def test_group_sizes(cuda, G):
    _config_case(cuda, 2, 2, G, 333, 4, 0.01, 10000.0, 3)


def test_long_context_positions(cuda):
    """Positions up to 2^17: fp32 angle rounding must follow the reference."""
    _config_case(cuda, 1, 1, 1, 131072 + 17, 4, 0.01, 10000.0, 4)
