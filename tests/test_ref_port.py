"""The torch CPU port of the reference's decode (oracle/kvq_ref_torch.py, the
bench's CPU baseline) against the oracle's float64 decode on the same cache in
the reference's format. No GPU."""
import numpy as np
import torch

from oracle import kvq_oracle as O
from oracle import kvq_ref_torch as R


def _dense(c, S, C, per_channel):
    x = c["codebook"].numpy()[c["q_idx"].numpy().astype(np.int64)]
    rp, cols, vals = (c[k].numpy() for k in ("outlier_rowptr", "outlier_cols", "outlier_values"))
    for r in range(S):
        x[r, cols[rp[r]:rp[r + 1]]] += vals[rp[r]:rp[r + 1]].astype(np.float32)
    s, z = c["scale"].numpy(), c["zero"].numpy()
    x = x * s + z if per_channel else x * s[:, None] + z[:, None]
    return x.astype(np.float16)


def test_port_decode_matches_the_oracle():
    T, H = 300, 2
    c = R.make_reference_cache(T, H, 4, 0.01, seed=3)
    C = H * 128
    kh = np.concatenate([c["k"]["sink"].numpy()[None], _dense(c["k"], T - 1, C, True)])[None]
    vh = np.concatenate([c["v"]["sink"].numpy()[None], _dense(c["v"], T - 1, C, False)])[None]
    q = (c["q"].float() * 0.1).half()
    c["q"] = q
    _, _, ref = O.decode_attention(q.numpy()[None], kh, vh, H, O.rope_inv_freq(128, 10000.0))
    got = R.decode_step(c).numpy()
    assert np.linalg.norm(got - ref[0]) / np.linalg.norm(ref[0]) < 2e-3
    # outlier counts of the reference's format (dense_sparse.py:22-23)
    assert int(c["k"]["outlier_rowptr"][-1]) == C * int((T - 1) * 0.01 or 1)
    assert int(c["v"]["outlier_rowptr"][-1]) == (T - 1) * max(1, int(C * 0.01))
