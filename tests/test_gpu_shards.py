"""GPU parity of token-range shards of a decode step (position offset, row
stats, merge) against the oracle's decode over the whole context."""
import numpy as np
import pytest
import torch

from oracle import kvq_oracle as O
import synth

pytestmark = pytest.mark.gpu

TOL = 2e-3


def t(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def rel_l2(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)


def _shards(cuda, G, bits, cuts, seed):
    """Shards quantized as their own blocks (the first with the sink) and decoded
    at their positions; also the oracle's dequantization of the same blocks."""
    from kvquant.kernels import (quantize_keys, quantize_values, decode_attention_shard,
                                 merge_shards, rope_inv_freq)
    B, Hkv, ratio = 1, 2, 0.01
    T = cuts[-1]
    k, v = synth.make_kv(B, T, Hkv * 128, seed=seed)
    scale, zero = synth.key_calibration(k)
    rng = np.random.default_rng(bits)
    cbk = np.sort(rng.uniform(-1, 1, 1 << bits)).astype(np.float32)
    cbv = np.sort(rng.uniform(-1, 1, 1 << bits)).astype(np.float32)
    q = (synth.make_query(B, Hkv * G, 128, seed=5).astype(np.float32) * 0.25).astype(np.float16)
    inv = rope_inv_freq(128, 10000.0)
    os_, mls, k_hat, v_hat = [], [], [], []
    for a, b in zip(cuts, cuts[1:]):
        sink = a == 0
        pk = quantize_keys(t(k[:, a:b], cuda), t(scale, cuda), t(zero, cuda), t(cbk, cuda), bits,
                           ratio, sink)
        pv = quantize_values(t(v[:, a:b], cuda), t(cbv, cuda), bits, ratio, sink)
        o, ml = decode_attention_shard(t(q, cuda), pk, pv, inv, pos0=a)
        os_.append(o)
        mls.append(ml)
        k_hat.append(O.quantize_k(k[:, a:b], cbk, scale, zero, ratio, sink)["dequant"])
        v_hat.append(O.quantize_v(v[:, a:b], cbv, ratio, sink)["dequant"])
    return q, Hkv, os_, mls, k_hat, v_hat


@pytest.mark.parametrize("G,bits,cuts", [(1, 4, (0, 256, 700)), (2, 4, (0, 300, 512, 833)),
                                         (4, 4, (0, 131072, 131072 + 999))])
def test_shards_merge_to_the_whole_decode(cuda, G, bits, cuts):
    """Merged shards against the oracle's decode of the whole context. Each
    shard is a decode held to the 2e-3 bar; the merged output combines fp16
    shard outputs (each rounded once more, 2^-11) whose errors add, so the
    whole-context bar here is 3e-3; the merge itself is checked to fp16
    rounding in test_merge_kernel_is_the_softmax_merge."""
    from kvquant.kernels import merge_shards
    q, Hkv, os_, mls, k_hat, v_hat = _shards(cuda, G, bits, cuts, 61 + G)
    out = merge_shards(torch.stack(os_), torch.stack(mls)).cpu().numpy()
    _, _, ref = O.decode_attention(q, np.concatenate(k_hat, 1), np.concatenate(v_hat, 1), Hkv,
                                   O.rope_inv_freq(128, 10000.0))
    assert rel_l2(out, ref) <= 1.5 * TOL, rel_l2(out, ref)
    for (a, b), o, ml, kh, vh in zip(zip(cuts, cuts[1:]), os_, mls, k_hat, v_hat):
        ro, rm, rl = O.decode_shard(q, kh, vh, Hkv, O.rope_inv_freq(128, 10000.0), a)
        assert rel_l2(o.cpu().numpy(), ro) <= 1.5 * TOL, (a, b, rel_l2(o.cpu().numpy(), ro))
        # the row's log-sum-exp M + log L (what the merge weights encode)
        m = ml.cpu().numpy().astype(np.float64)
        lse, rlse = m[:, 0] - np.log(m[:, 1]), (rm + np.log(rl)).reshape(-1)
        assert np.abs(lse - rlse).max() <= 2e-3 * np.abs(rlse).max() + 1e-3, (lse, rlse)


@pytest.mark.parametrize("G,bits,cuts", [(2, 3, (0, 300, 512, 833)), (4, 2, (0, 4096, 5095))])
def test_merge_kernel_is_the_softmax_merge(cuda, G, bits, cuts):
    """merge_shards on the GPU's own shard outputs and row stats against the
    float64 merge of the same numbers (fp16 output rounding only)."""
    from kvquant.kernels import merge_shards
    _, _, os_, mls, _, _ = _shards(cuda, G, bits, cuts, 71 + G)
    out = merge_shards(torch.stack(os_), torch.stack(mls)).cpu().numpy()
    o = [x.cpu().numpy().astype(np.float64) for x in os_]
    B, Hq = o[0].shape[:2]
    ms = [m.cpu().numpy().astype(np.float64)[:, 0].reshape(B, Hq) for m in mls]
    ls = [1.0 / m.cpu().numpy().astype(np.float64)[:, 1].reshape(B, Hq) for m in mls]
    ref = O.merge_shards(o, ms, ls)
    assert rel_l2(out, ref) <= 5e-4, rel_l2(out, ref)


def test_single_shard_at_zero_is_decode_attention(cuda):
    from kvquant.kernels import (quantize_keys, quantize_values, decode_attention,
                                 decode_attention_shard, merge_shards, rope_inv_freq)
    k, v = synth.make_kv(2, 300, 256, seed=71)
    scale, zero = synth.key_calibration(k)
    cb = t(np.linspace(-1, 1, 16).astype(np.float32), cuda)
    pk = quantize_keys(t(k, cuda), t(scale, cuda), t(zero, cuda), cb, 4, 0.01, True)
    pv = quantize_values(t(v, cuda), cb, 4, 0.01, True)
    q = t(synth.make_query(2, 2, 128, seed=2), cuda)
    inv = rope_inv_freq(128, 10000.0)
    full = decode_attention(q, pk, pv, inv)
    o, ml = decode_attention_shard(q, pk, pv, inv, pos0=0)
    # the same kernels; the value kernel's shared-memory float atomics may order
    # the outlier sums differently, so the fp16 outputs agree to rounding
    assert rel_l2(o.cpu().numpy(), full.cpu().numpy()) <= 1e-3
    merged = merge_shards(o[None], ml[None])
    assert rel_l2(merged.cpu().numpy(), o.cpu().numpy()) <= 5e-4
