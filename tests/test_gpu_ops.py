"""GPU parity of the reference's four ops (kvquant_ops.cu:265-270) against the oracle."""
import numpy as np
import pytest
import torch

from oracle import kvq_oracle as O
from goldens import load_misc

pytestmark = pytest.mark.gpu


def t(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


@pytest.mark.parametrize("shape,pos", [((2, 3, 5, 128), 7), ((1, 32, 64, 128), 0),
                                       ((1, 2, 1, 64), 4095), ((1, 1, 3, 2), 0)])
def test_rope_apply(cuda, shape, pos):
    from kvquant.kernels import get_cuda_ops
    rng = np.random.default_rng(0)
    x = rng.standard_normal(shape, dtype=np.float32).astype(np.float16)
    S, D = shape[2], shape[3]
    cos, sin = O.rope_cos_sin(S + pos, D, 10000.0)
    got = get_cuda_ops().rope_apply(t(x, cuda), t(cos, cuda), t(sin, cuda), pos).cpu().numpy()
    ref = O.rope_apply(x, cos, sin, pos)
    # fp32 math rounded once to fp16 on both sides; allow one fp16 ulp
    assert np.max(np.abs(got.astype(np.float32) - ref.astype(np.float32)) /
                  np.maximum(np.abs(ref.astype(np.float32)), 2 ** -14)) <= 2 ** -10


def test_apply_rope_elementwise_api(cuda):
    from kvquant.kernels import apply_rope_elementwise, apply_rope_inplace
    m = load_misc()
    x = t(m["rope_x"], cuda)
    out = apply_rope_elementwise(x, position_offset=7).cpu().numpy()
    np.testing.assert_allclose(out.astype(np.float32), m["rope_cpu_out"].astype(np.float32),
                               rtol=4e-3, atol=4e-3)
    x3 = t(m["rope_x"][:, 0, :, :].reshape(2, 5, 128), cuda)
    assert apply_rope_elementwise(x3, 3).shape == x3.shape
    y = x.clone()
    apply_rope_inplace(y, 7)
    assert torch.equal(y, apply_rope_elementwise(x, 7))


@pytest.mark.parametrize("N,D,per_channel", [(100, 128, True), (100, 128, False),
                                             (7, 100, True), (33, 4096, False), (1, 16, True)])
def test_lut_matvec(cuda, N, D, per_channel):
    from kvquant.kernels import get_cuda_ops
    rng = np.random.default_rng(N + D)
    q = rng.integers(0, 16, size=(N, D)).astype(np.uint8)
    lut = np.sort(rng.uniform(-1, 1, 16)).astype(np.float16)
    n_s = D if per_channel else N
    scale = rng.uniform(0.1, 2, n_s).astype(np.float16)
    zero = rng.uniform(-0.5, 0.5, n_s).astype(np.float16)
    vec = rng.standard_normal(D).astype(np.float16)
    got = get_cuda_ops().lut_matvec(t(q, cuda), t(lut, cuda), t(scale, cuda), t(zero, cuda),
                                    t(vec, cuda), per_channel).cpu().numpy().astype(np.float32)
    ref = O.lut_matvec(q, lut, scale, zero, vec, per_channel).astype(np.float32)
    np.testing.assert_allclose(got, ref, rtol=2e-3, atol=2e-3 * np.abs(ref).max())


def test_sparse_matvec_csr(cuda):
    from kvquant.kernels import sparse_matvec_csr, sparse_matvec
    m = load_misc()
    got = sparse_matvec_csr(t(m["sp_rowptr"], cuda), t(m["sp_cols"], cuda), t(m["sp_vals"], cuda),
                            t(m["sp_vec"], cuda)).cpu().numpy()
    np.testing.assert_allclose(got.astype(np.float32), m["sp_out"].astype(np.float32),
                               rtol=1e-3, atol=1e-3)
    assert got[7] == 0
    # COO entry point on the same matrix, entries shuffled
    rows = np.repeat(np.arange(len(m["sp_rowptr"]) - 1), np.diff(m["sp_rowptr"]))
    perm = np.random.default_rng(0).permutation(len(rows))
    idx = np.stack([rows, m["sp_cols"]], 1)[perm]
    got2 = sparse_matvec(t(idx, cuda), t(m["sp_vals"][perm], cuda), (50, 64),
                         t(m["sp_vec"], cuda)).cpu().numpy()
    np.testing.assert_allclose(got2.astype(np.float32), m["sp_out"].astype(np.float32),
                               rtol=1e-3, atol=1e-3)


def test_sparse_matvec_bad_column_is_reported(cuda):
    from kvquant.kernels import get_cuda_ops
    ops = get_cuda_ops()
    rp = torch.tensor([0, 2], dtype=torch.int32, device=cuda)
    col = torch.tensor([0, 99], dtype=torch.int32, device=cuda)
    val = torch.ones(2, dtype=torch.float16, device=cuda)
    vec = torch.ones(4, dtype=torch.float16, device=cuda)
    out = ops.sparse_matvec_csr(rp, col, val, vec, 1)
    with pytest.raises(RuntimeError, match="out of range"):
        ops.check_status(cuda)
    assert out.item() == 1.0  # the in-range entry was still added
    ops.check_status(cuda)    # status was cleared


def test_lut_lookup_bit_exact(cuda):
    from kvquant.kernels import get_cuda_ops, dense_matvec_lut
    m = load_misc()
    idx, dq = get_cuda_ops().lut_lookup(t(m["lut_x"], cuda), t(m["lut_cb"], cuda))
    np.testing.assert_array_equal(idx.cpu().numpy(), m["lut_idx"])
    np.testing.assert_array_equal(dq.cpu().numpy(), m["lut_dq"])
    got = dense_matvec_lut(t(m["lut_x"].reshape(-1, 5), cuda), t(m["lut_cb"], cuda))
    np.testing.assert_array_equal(got.cpu().numpy(), m["dense_matvec_lut_out"])
    # large random input against the oracle
    rng = np.random.default_rng(5)
    x = rng.uniform(-1.5, 1.5, 3_000_001).astype(np.float32)
    cb = np.sort(rng.uniform(-1, 1, 8)).astype(np.float32)
    idx, dq = get_cuda_ops().lut_lookup(t(x, cuda), t(cb, cuda))
    ri, rd = O.lut_lookup(x, cb)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_array_equal(dq.cpu().numpy(), rd)


def test_normalize_matches_ieee_division_for_every_fp16_input(cuda):
    """The quantizers' n = (x - z) / (s + 1e-8) (kv_quantizer.py:82,104), computed by
    the kernels from the reciprocal of the divisor, equals numpy's IEEE fp32
    quotient bit for bit for all 65536 fp16 inputs and per-column (zero, scale)
    pairs spanning the guarded range and beyond it (tiny, huge and zero scales,
    tiny and huge offsets, divisors whose mantissa is all ones)."""
    from kvquant.kernels import get_cuda_ops
    x = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16)
    rng = np.random.default_rng(5)
    allones = np.array([(e << 23) | 0x7FFFFF for e in (100, 120, 126, 127, 128, 135)],
                       np.uint32).view(np.float32)
    scale = np.concatenate([rng.uniform(1e-3, 50, 40).astype(np.float32),
                            np.exp(rng.uniform(-30, 30, 20)).astype(np.float32), allones,
                            np.array([0, 1e-8, 1e-30, 1e12, 3e38], np.float32)])
    zero = np.concatenate([rng.standard_normal(scale.size - 12).astype(np.float32) * 10,
                           np.array([0, -0.0, 1e-20, -1e-38, 1e-45, 2e20, -7e30, 65504,
                                     -65504, 0.5, 1.0, -3.0], np.float32)])
    rows = x.reshape(-1, 1).repeat(scale.size, 1)          # [65536, n_pairs] fp16
    got = get_cuda_ops().normalize(t(rows, cuda), t(zero, cuda), t(scale, cuda),
                                   True).cpu().numpy()
    with np.errstate(all="ignore"):
        ref = ((rows.astype(np.float32) - zero) / (scale + np.float32(1e-8))).astype(np.float32)
    same = (got.view(np.uint32) == ref.view(np.uint32)) | (np.isnan(got) & np.isnan(ref))
    assert same.all(), (int((~same).sum()), np.argwhere(~same)[:5])
    # per-row (values) orientation
    vr = rng.standard_normal((64, 512)).astype(np.float16)
    vz = rng.standard_normal(64).astype(np.float32)
    vs = rng.uniform(0.5, 30, 64).astype(np.float32)
    got = get_cuda_ops().normalize(t(vr, cuda), t(vz, cuda), t(vs, cuda), False).cpu().numpy()
    ref = ((vr.astype(np.float32) - vz[:, None]) / (vs[:, None] + np.float32(1e-8))).astype(np.float32)
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))
