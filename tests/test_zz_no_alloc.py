"""kvq_value_output_noalloc: the value kernel with library-owned scratch.

Called through the C ABI and compared with kvq_value_output (caller workspace)
on the same packed cache and probabilities, twice in a row so the second call
runs on scratch the first one left behind. Tolerance: relative L2 <= 2e-3, the
decode tests' bar (the two calls run the same kernels, so they agree far
closer than that).
"""
import ctypes

import numpy as np
import pytest
import torch

import synth

pytestmark = pytest.mark.gpu

TOL = 2e-3


def rel_l2(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)


def _noalloc(lib, pv, p, out):
    B, Hq, T = p.shape
    H = pv["n_heads"]
    return lib.kvq_value_output_noalloc(
        pv["q_idx"].data_ptr(), pv["outlier_entries"].data_ptr(),
        pv["outlier_rowptr"].data_ptr(), pv["scale"].data_ptr(), pv["zero"].data_ptr(),
        pv["scale"].shape[1], pv["sink"].data_ptr(), pv["codebook"].data_ptr(), pv["bits"],
        p.data_ptr(), B, H, Hq // H, T, pv["q_idx"].shape[1], out.data_ptr(),
        torch.cuda.current_stream(p.device).cuda_stream)


@pytest.mark.parametrize("B,Hkv,G,T,bits", [(2, 4, 2, 3000, 4), (1, 8, 1, 20000, 3)])
def test_noalloc_matches_workspace_entry(cuda, B, Hkv, G, T, bits):
    from kvquant.kernels import pv_out, quantize_values
    from kvquant.kernels.cuda_ops import get_cuda_ops
    lib = get_cuda_ops().lib
    _, v = synth.make_kv(B, T, Hkv * 128, seed=7)
    rng = np.random.default_rng(7)
    cbv = np.sort(rng.uniform(-1, 1, 1 << bits)).astype(np.float32)
    pv = quantize_values(torch.from_numpy(v).to(cuda), torch.from_numpy(cbv).to(cuda), bits,
                         0.01, True)
    logits = torch.from_numpy(rng.standard_normal((B, Hkv * G, T)).astype(np.float32) * 3)
    p = torch.softmax(logits, dim=-1).to(cuda).contiguous()
    ref = pv_out(p, pv).cpu().numpy()
    with torch.cuda.device(cuda):
        for _ in range(2):
            out = torch.full((B, Hkv * G, 128), float("nan"), dtype=torch.float16, device=cuda)
            rc = _noalloc(lib, pv, p, out)
            assert rc == 0, lib.kvq_last_error().decode()
            got = out.cpu().numpy()
            assert np.isfinite(got).all()
            assert rel_l2(got, ref) <= TOL, rel_l2(got, ref)


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda):
    from kvquant.kernels.cuda_ops import get_cuda_ops
    lib = get_cuda_ops().lib
    B, H, G, T = 1024, 8, 8, 32  # 8192 units x 8 heads x 129 partial floats > 4 MiB
    assert lib.kvq_value_output_workspace(B, H, G, T) > 4 << 20
    with torch.cuda.device(cuda):
        rc = lib.kvq_value_output_noalloc(None, None, None, None, None, T, None, None, 4, None,
                                          B, H, G, T, 1, None, None)
    assert rc == 1  # KVQ_ERR_INVALID, nothing launched
    assert "scratch" in lib.kvq_last_error().decode()
