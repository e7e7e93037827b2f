"""Reads a packed cache (prefill layout or the appendable one with per-unit
outlier segments) back into dense numpy arrays, checking the CSR invariants."""
from __future__ import annotations

import numpy as np

from oracle import kvq_oracle as O


def read_cache(codes, out_ptr, out_ent, bits: int, kind: str, T: int):
    """-> (idx int64 [U, T, 128], mask bool [U, T, 128], vals fp32 [U, T, 128])."""
    codes = np.asarray(codes)
    U, nt_cap = codes.shape[:2]
    ptr = np.asarray(out_ptr).astype(np.int64)
    ent = np.asarray(out_ent)
    nt = -(-T // 32)
    idx = O.unpack_codes(codes, bits, kind, T)
    vals = np.zeros((U, nt * 32, 128), np.float32)
    mask = np.zeros((U, nt * 32, 128), bool)
    for u in range(U):
        r0 = u * 2 * nt_cap
        assert np.all(np.diff(ptr[r0:r0 + 2 * nt + 1]) >= 0), "row pointers decrease"
        for r in range(2 * nt):
            s, e = ptr[r0 + r], ptr[r0 + r + 1]
            v, pos = O.unpack_entries(ent[s:e])
            pos = pos.astype(np.int64)
            tok, ch = pos >> 7, pos & 127
            assert np.all((tok >= 16 * (r % 2)) & (tok < 16 * (r % 2) + 16)), "entry outside its row"
            key = tok * 128 + ch
            assert np.all(np.diff(key) > 0), "row entries not in (token, channel) order"
            t = (r // 2) * 32 + tok
            vals[u, t, ch] = v.astype(np.float32)
            mask[u, t, ch] = True
    return idx, mask[:, :T], vals[:, :T]


def read_packed(p: dict, T: int | None = None):
    """read_cache on a packed dict of torch tensors."""
    T = int(p["length"]) if T is None else T
    return read_cache(p["q_idx"].cpu().numpy(), p["outlier_rowptr"].cpu().numpy(),
                      p["outlier_entries"].cpu().numpy(), p["bits"],
                      "k" if p["kind"] == "k" else "v", T)
