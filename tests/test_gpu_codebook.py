"""NUQ codebook fitting on the GPU (kvq_fit_codebook) against the oracle's exact
1-D k-means and the reference's solver (kvquant/quant/nuq.py:6-44).

Parity for a k-means fit is its objective: the GPU centres must reach the
global optimum the oracle computes (small cases) and never do worse than the
reference's KMeans local search (large cases); the reference's degenerate-input
rules must hold exactly."""
import numpy as np
import pytest
import torch

from oracle import kvq_oracle as O

pytestmark = pytest.mark.gpu


def _data(seed, n, kind="normal"):
    rng = np.random.default_rng(seed)
    if kind == "normal":
        x = np.clip(rng.normal(0.0, 0.4, n), -1.0, 1.0)
    elif kind == "bimodal":
        x = np.clip(np.concatenate([rng.normal(-0.5, 0.1, n // 2), rng.normal(0.4, 0.2, n - n // 2)]),
                    -1.0, 1.0)
    else:
        x = rng.uniform(-1.0, 1.0, n)
    w = rng.gamma(2.0, 1.0, n)
    return x.astype(np.float32), w.astype(np.float32)


def _fit(x, w, bits, dev, **kw):
    from kvquant.quant.nuq import fit_nuq_codebook_cuda
    c = fit_nuq_codebook_cuda(torch.from_numpy(x).to(dev), torch.from_numpy(w).to(dev), bits, **kw)
    assert c.is_cuda and c.dtype == torch.float32 and c.numel() == 2 ** bits
    return c.cpu().numpy()


@pytest.mark.parametrize("seed,bits,kind", [(0, 1, "normal"), (1, 2, "bimodal"), (2, 3, "normal"),
                                            (3, 4, "uniform"), (4, 4, "normal"), (5, 4, "bimodal")])
def test_small_fit_reaches_the_global_optimum(cuda, seed, bits, kind):
    x, w = _data(seed, 1500, kind)
    wn = w / w.sum()
    got = _fit(x, w, bits, cuda)
    opt = O.kmeans_1d_optimal(x, wn, 2 ** bits)
    assert np.all(np.diff(got) >= 0)
    assert O.kmeans_1d_inertia(x, wn, got) <= O.kmeans_1d_inertia(x, wn, opt) * (1 + 1e-5)
    np.testing.assert_allclose(got, opt, rtol=0, atol=2e-4)


@pytest.mark.parametrize("seed,bits", [(10, 2), (11, 3), (12, 4)])
def test_large_fit_is_never_worse_than_the_reference_solver(cuda, seed, bits):
    from threadpoolctl import threadpool_limits
    from kvquant.quant.nuq import train_nuq_codebook

    x, w = _data(seed, 100_000, "bimodal" if seed % 2 else "normal")
    wn = w / w.sum()
    with threadpool_limits(limits=1):
        ref = train_nuq_codebook(torch.from_numpy(x), torch.from_numpy(w), n_bits=bits).numpy()
    got = _fit(x, w, bits, cuda)
    assert O.kmeans_1d_inertia(x, wn, got) <= O.kmeans_1d_inertia(x, wn, ref) * (1 + 1e-5)


def test_lloyd_refinement_never_raises_the_objective(cuda):
    x, w = _data(20, 300_000, "normal")
    wn = w / w.sum()
    vals = [O.kmeans_1d_inertia(x, wn, _fit(x, w, 4, cuda, refine_iters=r)) for r in (0, 1, 4)]
    assert vals[1] <= vals[0] * (1 + 1e-7) and vals[2] <= vals[1] * (1 + 1e-7)


def test_unaligned_and_odd_sized_inputs(cuda):
    """Buffers off the 16-byte boundary and a length that is not a multiple of
    four take the scalar loads; the fit is the same."""
    from kvquant.quant.nuq import fit_nuq_codebook_cuda

    x, w = _data(30, 50_003, "normal")
    xb = torch.zeros(x.size + 1, device=cuda)
    wb = torch.zeros(x.size + 1, device=cuda)
    xb[1:] = torch.from_numpy(x).to(cuda)
    wb[1:] = torch.from_numpy(w).to(cuda)
    a = fit_nuq_codebook_cuda(xb[1:], wb[1:], 3).cpu().numpy()
    b = _fit(x, w, 3, cuda)
    np.testing.assert_allclose(a, b, rtol=0, atol=1e-5)


def test_degenerate_inputs_follow_the_reference(cuda):
    cases = [np.zeros(0, np.float32), np.array([0.3, -0.2, 0.7], np.float32),
             np.array([0.1, 0.1, 0.5, 0.5, 0.5, -0.4] * 3, np.float32),
             np.full(40, 0.25, np.float32)]
    for x in cases:
        got = _fit(x, np.ones_like(x), 3, cuda)
        np.testing.assert_array_equal(got, O.codebook_degenerate(x, 3))


def test_values_bunched_below_the_bin_width_are_reported(cuda):
    x = np.concatenate([np.float32(0.5) + np.arange(20, dtype=np.float32) * np.float32(1e-6),
                        np.float32([1000.0])]).astype(np.float32)
    with pytest.raises(RuntimeError, match="histogram bins"):
        _fit(x, np.ones_like(x), 3, cuda)


def test_train_nuq_codebook_runs_on_the_device_for_cuda_tensors(cuda):
    from kvquant.quant.nuq import train_nuq_codebook

    x, w = _data(40, 20_000, "normal")
    c = train_nuq_codebook(torch.from_numpy(x).to(cuda), torch.from_numpy(w).to(cuda), n_bits=2)
    # a CPU tensor, as the reference returns (calibration pickles the codebooks)
    assert not c.is_cuda and c.dtype == torch.float32
    np.testing.assert_allclose(c.numpy(), _fit(x, w, 2, cuda), rtol=0, atol=1e-6)


def test_train_nuq_codebook_bunched_values_use_the_reference_solver(cuda):
    """Where the GPU fit reports bunched values, train_nuq_codebook returns
    the reference solver's codebook instead of raising."""
    from kvquant.quant.nuq import train_nuq_codebook
    x = np.concatenate([np.float32(0.5) + np.arange(20, dtype=np.float32) * np.float32(1e-6),
                        np.float32([1000.0])]).astype(np.float32)
    w = np.ones_like(x)
    got = train_nuq_codebook(torch.from_numpy(x).to(cuda), torch.from_numpy(w).to(cuda), n_bits=3)
    ref = train_nuq_codebook(torch.from_numpy(x), torch.from_numpy(w), n_bits=3)
    assert not got.is_cuda
    np.testing.assert_array_equal(got.numpy(), ref.numpy())


def test_zero_weights_are_ignored(cuda):
    """Samples of weight 0 move no centre (the reference passes the weights to
    KMeans as sample_weight)."""
    x, w = _data(50, 1500, "bimodal")
    w[np.random.default_rng(51).random(x.size) < 0.4] = 0.0
    wn = w / w.sum()
    got = _fit(x, w, 3, cuda)
    opt = O.kmeans_1d_optimal(x[w > 0], wn[w > 0], 8)
    assert O.kmeans_1d_inertia(x, wn, got) <= O.kmeans_1d_inertia(x, wn, opt) * (1 + 1e-5)
    np.testing.assert_allclose(got, opt, rtol=0, atol=2e-4)


def test_non_finite_samples_and_bad_weights_raise(cuda):
    x, w = _data(60, 5000, "normal")
    for bad_x, bad_w in ((np.nan, None), (np.inf, None), (None, np.inf), (None, -1.0),
                         (None, np.nan)):
        xx, ww = x.copy(), w.copy()
        if bad_x is not None:
            xx[1234] = bad_x
        if bad_w is not None:
            ww[4321] = bad_w
        with pytest.raises(ValueError):
            _fit(xx, ww, 3, cuda)
    _fit(x, w, 3, cuda)  # a clean call after the flagged ones


def test_sixteen_million_samples_on_few_values_reach_the_optimum(cuda):
    """16,777,216 samples on 400 distinct values (each far from the others in bin
    terms) with gamma weights: every CTA adds about 113K samples into few bins, the
    case where fp32 bin sums lose 1e-4..1e-3 relative. The fit must reach the
    exact optimum of the aggregated (value, weight) problem."""
    rng = np.random.default_rng(16)
    vals = np.sort(rng.uniform(-1, 1, 400)).astype(np.float32)
    n = 1 << 24
    x = vals[rng.integers(0, vals.size, n)]
    w = rng.gamma(2.0, 1.0, n).astype(np.float32)
    got = _fit(x, w, 4, cuda)
    agg = np.bincount(np.searchsorted(vals, x), weights=w.astype(np.float64), minlength=vals.size)
    opt = O.kmeans_1d_optimal(vals, agg, 16)
    assert O.kmeans_1d_inertia(vals, agg, got) <= O.kmeans_1d_inertia(vals, agg, opt) * (1 + 1e-6)
