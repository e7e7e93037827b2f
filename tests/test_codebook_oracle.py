"""NUQ codebook fitting on the CPU: the oracle's exact 1-D k-means and the
reference's rules (kvquant/quant/nuq.py), the C ABI's argument checks, and the
host wrapper's device rule. No GPU needed."""
import ctypes
import itertools

import numpy as np
import pytest
import torch

from oracle import kvq_oracle as O


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


def _brute_force(x, w, K):
    """Best inertia over every split of the sorted distinct values into K intervals."""
    u = np.unique(x)
    best = np.inf
    for cuts in itertools.combinations(range(1, u.size), K - 1):
        bounds = [0, *cuts, u.size]
        cs = []
        for a, b in zip(bounds[:-1], bounds[1:]):
            m = (x >= u[a]) & (x <= u[b - 1])
            cs.append(np.sum(w[m] * x[m]) / np.sum(w[m]))
        best = min(best, O.kmeans_1d_inertia(x, w, cs))
    return best


@pytest.mark.parametrize("seed,K", [(0, 2), (1, 3), (2, 4)])
def test_oracle_optimum_matches_exhaustive_search(seed, K):
    x, w = _data(seed, 11)
    c = O.kmeans_1d_optimal(x, w, K)
    assert c.size == K and np.all(np.diff(c) > 0)
    assert O.kmeans_1d_inertia(x, w, c) == pytest.approx(_brute_force(x, w, K), rel=1e-12)


@pytest.mark.parametrize("seed,bits,kind", [(0, 1, "normal"), (1, 2, "bimodal"), (2, 3, "normal"),
                                            (3, 4, "uniform"), (4, 4, "normal")])
def test_oracle_optimum_is_never_worse_than_the_reference_solver(seed, bits, kind):
    """The reference's solver (train_nuq_codebook on CPU tensors: weighted
    KMeans, n_init=10) reaches a local optimum; the oracle's is global."""
    from threadpoolctl import threadpool_limits
    from kvquant.quant.nuq import train_nuq_codebook

    x, w = _data(seed, 1200, kind)
    wn = w / w.sum()
    with threadpool_limits(limits=1):
        ref = train_nuq_codebook(torch.from_numpy(x), torch.from_numpy(w), n_bits=bits).numpy()
    opt = O.kmeans_1d_optimal(x, wn, 2 ** bits)
    assert np.all(np.diff(opt) > 0)
    assert O.kmeans_1d_inertia(x, wn, opt) <= O.kmeans_1d_inertia(x, wn, ref) * (1 + 1e-12)


def test_degenerate_rules_follow_the_reference():
    from kvquant.quant.nuq import train_nuq_codebook

    cases = [np.zeros(0, np.float32), np.array([0.3, -0.2, 0.7], np.float32),
             np.array([0.1, 0.1, 0.5, 0.5, 0.5, -0.4] * 3, np.float32),
             np.full(40, 0.25, np.float32)]
    for x in cases:
        w = np.ones_like(x)
        got = train_nuq_codebook(torch.from_numpy(x), torch.from_numpy(w), n_bits=3).numpy()
        np.testing.assert_array_equal(got, O.codebook_degenerate(x, 3))
    assert O.codebook_degenerate(_data(0, 100)[0], 3) is None


def test_fit_entry_point_rejects_bad_arguments():
    from kvquant.kernels.cuda_ops import load_library

    lib = load_library()
    p = ctypes.c_void_p(256)
    assert lib.kvq_fit_codebook(p, p, 0, 3, 2, p, p, 1 << 30, p, None) == 1
    assert lib.kvq_fit_codebook(p, p, 100, 5, 2, p, p, 1 << 30, p, None) == 3
    assert b"bits" in lib.kvq_last_error()
    assert lib.kvq_fit_codebook(p, p, 100, 3, 65, p, p, 1 << 30, p, None) == 1
    need = lib.kvq_fit_codebook_workspace(100)
    assert need > 8192 * 16
    rc = lib.kvq_fit_codebook(p, p, 100, 3, 2, p, p, need - 1, p, None)
    assert rc == 1 and b"workspace" in lib.kvq_last_error()
    rc = lib.kvq_fit_codebook(p, p, 100, 3, 2, p, ctypes.c_void_p(264), need, p, None)
    assert rc == 1 and b"aligned" in lib.kvq_last_error()
    # the per-CTA partial histograms grow with n up to one CTA per SM
    assert lib.kvq_fit_codebook_workspace(1 << 30) > lib.kvq_fit_codebook_workspace(100)


def test_gpu_fit_rejects_host_tensors():
    from kvquant.quant.nuq import fit_nuq_codebook_cuda

    with pytest.raises(RuntimeError, match="CUDA"):
        fit_nuq_codebook_cuda(torch.zeros(10), torch.ones(10), 2)


def test_padding_helper_matches_the_reference_rule():
    """The host helper that applies nuq.py:26-37 to the GPU path's inputs."""
    from kvquant.quant.nuq import _pad_sorted

    for x in (np.array([0.3, -0.2, 0.7], np.float32), np.array([0.5], np.float32),
              np.array([-1.0, 1.0, 0.0, 0.25], np.float32)):
        got = _pad_sorted(torch.from_numpy(x), 8).numpy()
        np.testing.assert_array_equal(got, O.codebook_degenerate(x, 3))


def test_oracle_optimum_is_equivariant():
    """Scaling the weights leaves the optimum; shifting / scaling the samples moves
    it with them (properties of the weighted 1-D k-means objective)."""
    x, w = _data(7, 400, "bimodal")
    base = O.kmeans_1d_optimal(x, w, 4)
    # a power-of-two weight scale is exact in fp32, so the optimum must not move at all
    np.testing.assert_array_equal(O.kmeans_1d_optimal(x, w * np.float32(32.0), 4), base)
    np.testing.assert_allclose(O.kmeans_1d_optimal(x.astype(np.float64) * 2.0 + 0.5, w, 4),
                               base * 2.0 + 0.5, rtol=1e-12, atol=1e-12)
    # mirrored samples give mirrored centres
    np.testing.assert_allclose(O.kmeans_1d_optimal(-x.astype(np.float64), w, 4), -base[::-1],
                               rtol=1e-12, atol=1e-12)
