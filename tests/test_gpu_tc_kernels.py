"""The tcgen05 decode kernels (selected with set_decode_kernels("tc", "tc")) on
the decode parity cases, and against the default mma.sync kernels on the same
cache: both compute the same values up to fp32 summation order."""
import numpy as np
import pytest
import torch

import synth
from goldens import QUANT_CASES

pytestmark = pytest.mark.gpu


@pytest.fixture
def tc(cuda):
    from kvquant.kernels import set_decode_kernels
    prev = set_decode_kernels("tc", "tc")
    yield cuda
    set_decode_kernels(*prev)


@pytest.mark.parametrize("name", QUANT_CASES)
def test_tc_golden_cases(tc, name):
    import test_gpu_decode as D
    D.test_decode_golden_cases(tc, name)


def test_tc_cfg1_32k(tc):
    import test_gpu_parity_full as P
    P.test_cfg1_32k(tc)


@pytest.mark.parametrize("G", [1, 4])
def test_tc_positions_near_2_20(tc, G):
    import test_gpu_parity_full as P
    P.test_positions_near_2_20(tc, G)


def test_tc_group_sizes(tc):
    import test_gpu_decode as D
    D.test_group_sizes(tc, 8)


@pytest.mark.parametrize("bits", [2, 3, 4])
def test_tc_matches_mma(cuda, bits):
    """65536 tokens, 8 KV heads: scores of the two kernel pairs agree to 2e-3 and
    outputs to 5e-3 (relative L2, every row). The tcgen05 key kernel keeps single
    fp16 code values and constants where the mma.sync one splits them into high
    and low parts; rows whose softmax sits on a few tokens turn that score
    difference into a larger output difference."""
    from kvquant.kernels import (quantize_keys, quantize_values, qk_scores, decode_attention,
                                 rope_inv_freq, set_decode_kernels)
    B, Hkv, T = 1, 8, 65536
    k, v = synth.make_kv(B, T, Hkv * 128, seed=40 + bits)
    scale, zero = synth.key_calibration(k)
    rng = np.random.default_rng(41)
    cbk = np.sort(rng.uniform(-1, 1, 1 << bits)).astype(np.float32)
    cbv = np.sort(rng.uniform(-1, 1, 1 << bits)).astype(np.float32)
    f = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(cuda)
    pk = quantize_keys(f(k), f(scale), f(zero), f(cbk), bits, 0.01, True)
    pv = quantize_values(f(v), f(cbv), bits, 0.01, True)
    q = f((synth.make_query(B, Hkv, 128, seed=42).astype(np.float32) * 0.25).astype(np.float16))
    inv = rope_inv_freq(128, 10000.0)
    res = {}
    for kern in ("mma", "tc"):
        prev = set_decode_kernels(kern, kern)
        try:
            res[kern] = (qk_scores(q, pk, inv).double().cpu(),
                         decode_attention(q, pk, pv, inv).double().cpu())
        finally:
            set_decode_kernels(*prev)
    for i in range(2):
        a, b = res["tc"][i].reshape(-1, res["tc"][i].shape[-1]), \
            res["mma"][i].reshape(-1, res["mma"][i].shape[-1])
        err = (a - b).norm(dim=1) / b.norm(dim=1).clamp_min(1e-30)
        assert err.max().item() < (2e-3, 5e-3)[i], (bits, i, err.max().item())


def test_selector_rejects_unknown(cuda):
    from kvquant.kernels import set_decode_kernels
    with pytest.raises(ValueError):
        set_decode_kernels("wgmma")
