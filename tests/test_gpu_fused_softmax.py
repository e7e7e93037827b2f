"""GPU parity of the fused-softmax decode path.

The key kernel leaves per-(row, 16-token block) softmax partials (max, sum of
exp) beside the raw scores and the value kernel forms the probabilities from
the raw scores itself (kvq_key_scores_stats + kvq_value_output_scores, the
default of kvq_decode_attention when no probabilities are requested). The
result must be the reference's softmax -> p.V: the oracle's output within the
decode tolerance (relative L2 <= 2e-3; for the value side, on the kernel's own
scores), the explicit-softmax path within the same bound, and the partials equal
to the ones numpy computes from the scores the kernel returned (relative 1e-5:
fp32 exp of the same values).

Why the two GPU paths are not compared more tightly: both round each token's
weight p * s to fp16 for the tensor-core p.V (the reference likewise rounds the
probabilities to fp16 before p @ V). Probabilities that agree to 1e-7 can land
on two sides of an fp16 rounding tie; with one dominant token (p ~ 1) that is a
2^-11 step of its whole weight, amplified where s * cb and the zero point
cancel -- 1.4e-3 relative on one head of the 4096-token case below.
"""
import numpy as np
import pytest
import torch

from oracle import kvq_oracle as O
import synth

pytestmark = pytest.mark.gpu

TOL = 2e-3
SCALE = 1.0 / np.sqrt(128.0)


def t(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def rel_l2(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)


def _case(cuda, B, Hkv, G, T, bits, ratio, seed, sink=True, base=10000.0, want_v=False):
    from kvquant.kernels import quantize_keys, quantize_values
    C = Hkv * 128
    k, v = synth.make_kv(B, T, C, seed=seed)
    scale, zero = synth.key_calibration(k)
    rng = np.random.default_rng(seed)
    cbk = np.sort(rng.uniform(-1, 1, 1 << bits)).astype(np.float32)
    cbv = np.sort(rng.uniform(-1, 1, 1 << bits)).astype(np.float32)
    pk = quantize_keys(t(k, cuda), t(scale, cuda), t(zero, cuda), t(cbk, cuda), bits, ratio, sink)
    pv = quantize_values(t(v, cuda), t(cbv, cuda), bits, ratio, sink)
    q = synth.make_query(B, Hkv * G, 128, seed=seed + 1)
    kq = O.quantize_k(k, cbk, scale, zero, ratio, sink)
    vq = O.quantize_v(v, cbv, ratio, sink)
    ref = O.decode_attention(q, kq["dequant"], vq["dequant"], Hkv, O.rope_inv_freq(128, base))
    return (pk, pv, q, ref, vq["dequant"]) if want_v else (pk, pv, q, ref)


def _chunk_stats(scores):
    """(max, sum exp(x - max)) of scores * SCALE per 16-token block, float64."""
    rows = scores.reshape(-1, scores.shape[-1]).astype(np.float64) * np.float32(SCALE)
    T = rows.shape[1]
    n = (T + 15) // 16
    out = np.zeros((rows.shape[0], n, 2))
    for k in range(n):
        x = rows[:, 16 * k:16 * (k + 1)]
        m = x.max(axis=1)
        out[:, k, 0] = m
        out[:, k, 1] = np.exp(x - m[:, None]).sum(axis=1)
    return out


@pytest.mark.parametrize("B,Hkv,G,T,bits", [
    (1, 4, 1, 4096, 4),
    (2, 2, 2, 333, 3),
    (1, 2, 4, 1000, 2),
    (2, 1, 8, 257, 4),
])
def test_fused_ops_match_oracle(cuda, B, Hkv, G, T, bits):
    from kvquant.kernels import (qk_scores, qk_scores_stats, pv_out_scores, pv_out, softmax,
                                 rope_inv_freq)
    pk, pv, q, (rs, rp, ro), vh = _case(cuda, B, Hkv, G, T, bits, 0.01, 11 + T, want_v=True)
    inv = rope_inv_freq(128, 10000.0)
    qd = t(q, cuda)
    s, st = qk_scores_stats(qd, pk, inv)
    # the scores are the plain key kernel's, bit for bit
    s_plain = qk_scores(qd, pk, inv)
    assert torch.equal(s, s_plain)
    assert rel_l2(s.cpu().numpy(), rs) <= TOL
    want = _chunk_stats(s.cpu().numpy())
    got = st.cpu().numpy().astype(np.float64)
    np.testing.assert_allclose(got[..., 0], want[..., 0], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(got[..., 1], want[..., 1], rtol=1e-5)
    o = pv_out_scores(s, st, pv).cpu().numpy()
    # value side against the oracle on the kernel's own scores (as the golden
    # decode cases check pv_out on the reference's probabilities)
    sk = s.cpu().numpy().astype(np.float64)
    ro_k = O.value_output(O.softmax_probs(sk, 128), vh, Hkv)
    assert rel_l2(o, ro_k) <= TOL, rel_l2(o, ro_k)
    # and against the explicit softmax -> p.V of the same scores
    o_explicit = pv_out(softmax(s), pv).cpu().numpy()
    assert rel_l2(o, o_explicit) <= TOL, rel_l2(o, o_explicit)


@pytest.mark.parametrize("T", [1, 31, 256, 2049])
def test_fused_vs_explicit_softmax(cuda, T):
    """decode_attention with and without probs_out: the same attention."""
    from kvquant.kernels import decode_attention, rope_inv_freq
    pk, pv, q, (rs, rp, ro), vh = _case(cuda, 1, 2, 2, T, 4, 0.01, 5 + T, want_v=True)
    inv = rope_inv_freq(128, 10000.0)
    qd = t(q, cuda)
    s = torch.empty((1, 4, T), dtype=torch.float32, device=cuda)
    fused = decode_attention(qd, pk, pv, inv, scores_out=s).cpu().numpy()
    assert rel_l2(s.cpu().numpy(), rs) <= TOL
    ro_k = O.value_output(O.softmax_probs(s.cpu().numpy().astype(np.float64), 128), vh, 2)
    probs = torch.empty((1, 4, T), dtype=torch.float32, device=cuda)
    explicit = decode_attention(qd, pk, pv, inv, probs_out=probs).cpu().numpy()
    assert rel_l2(fused, ro_k) <= TOL, rel_l2(fused, ro_k)
    assert rel_l2(explicit, ro_k) <= TOL
    assert rel_l2(fused, explicit) <= TOL


@pytest.mark.parametrize("T", [32769, 70001])
def test_fused_long_context_chunked_merge(cuda, T):
    """Past 32,768 tokens a row has more than 2048 softmax partials, which the value
    prep merges in 2048-partial chunks over many blocks (the block that completes a
    row's last chunk folds the chunk pairs): (M, 1/L) against float64 over the
    scores, the output against the explicit softmax path and the oracle, on two
    calls in a row (the merge counts are cleared per call)."""
    from kvquant.kernels import qk_scores_stats, pv_out_scores, pv_out, softmax, rope_inv_freq
    pk, pv, q, (rs, rp, ro), vh = _case(cuda, 1, 2, 2, T, 4, 0.01, 23 + T, want_v=True)
    inv = rope_inv_freq(128, 10000.0)
    s, st = qk_scores_stats(t(q, cuda), pk, inv)
    assert rel_l2(s.cpu().numpy(), rs) <= TOL
    x = s.cpu().numpy().reshape(4, T).astype(np.float64) * np.float32(SCALE)
    m = x.max(axis=1)
    inv_l = 1.0 / np.exp(x - m[:, None]).sum(axis=1)
    ro_k = O.value_output(O.softmax_probs(s.cpu().numpy().astype(np.float64), 128), vh, 2)
    o_explicit = pv_out(softmax(s), pv).cpu().numpy()
    for _ in range(2):
        ml = torch.full((4, 2), float("nan"), dtype=torch.float32, device=cuda)
        o = pv_out_scores(s, st, pv, ml_out=ml).cpu().numpy()
        got = ml.cpu().numpy().astype(np.float64)
        np.testing.assert_allclose(got[:, 0], m, rtol=1e-6, atol=1e-6)
        np.testing.assert_allclose(got[:, 1], inv_l, rtol=3e-5)
        assert rel_l2(o, o_explicit) <= TOL, rel_l2(o, o_explicit)
        assert rel_l2(o, ro_k) <= TOL, rel_l2(o, ro_k)


def test_fused_without_sink(cuda):
    from kvquant.kernels import decode_attention, rope_inv_freq
    pk, pv, q, (rs, rp, ro), vh = _case(cuda, 1, 2, 1, 700, 3, 0.01, 9, sink=False, want_v=True)
    s = torch.empty((1, 2, 700), dtype=torch.float32, device=cuda)
    o = decode_attention(t(q, cuda), pk, pv, rope_inv_freq(128, 10000.0),
                         scores_out=s).cpu().numpy()
    assert rel_l2(s.cpu().numpy(), rs) <= TOL
    ro_k = O.value_output(O.softmax_probs(s.cpu().numpy().astype(np.float64), 128), vh, 2)
    assert rel_l2(o, ro_k) <= TOL


def test_fused_rejects_bad_stats(cuda):
    from kvquant.kernels import pv_out_scores
    pk, pv, q, _ = _case(cuda, 1, 1, 1, 64, 4, 0.01, 1)
    s = torch.zeros((1, 1, 64), dtype=torch.float32, device=cuda)
    with pytest.raises(RuntimeError):
        pv_out_scores(s, torch.zeros((1, 2, 2), dtype=torch.float32, device=cuda), pv)
