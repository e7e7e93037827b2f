"""NUQ codebook fitting (drop-in for kvquant/quant/nuq.py).

Offline calibration, not part of the decode path. ``train_nuq_codebook`` keeps
the reference's signature and rules:

* CPU tensors: the reference's solver, a Fisher-weighted scikit-learn KMeans
  with its settings (n_init=10, max_iter=100, random_state=0; nuq.py:39-44)
  and its degenerate-input rules (nuq.py:20-37);
* CUDA tensors: ``fit_nuq_codebook_cuda``, the same objective solved on the GPU
  by the library's exact 1-D method (weighted histogram, optimal interval split,
  Lloyd refinement; ``kvq_fit_codebook``), with the same degenerate-input rules.
  The centres come back as a CPU tensor, as the reference's do (its calibration
  pickles them, so a codebook must not be tied to a device index). Values
  bunched into fewer histogram bins than clusters go to the reference's solver.

``fit_nuq_codebook_cuda`` keeps its centres on the device for callers that feed
them straight to the quantize kernels.
"""
from __future__ import annotations

import numpy as np
import torch


class CodebookBinsError(RuntimeError):
    """At least 2^n_bits distinct values fall into fewer than 2^n_bits of the
    GPU fit's histogram bins (values bunched far below the bin width)."""


def _pad_sorted(vals: torch.Tensor, n_clusters: int) -> torch.Tensor:
    """Sorted values padded with their maximum to n_clusters (nuq.py:26-37)."""
    c = torch.sort(vals.reshape(-1)).values
    pad = c[-1:].expand(n_clusters - c.numel())
    return torch.sort(torch.cat([c, pad])).values


def fit_nuq_codebook_cuda(activations: torch.Tensor, fisher: torch.Tensor, n_bits: int = 3,
                          refine_iters: int = 2) -> torch.Tensor:
    """Weighted 1-D k-means of activations [N] (CUDA) with weights fisher [N] (>= 0)
    -> sorted fp32 centres [2^n_bits] on the same device.

    Minimises the objective of nuq.py:39-42 (the weights' normalisation to sum 1,
    nuq.py:23, does not move the centres). n_bits 1..4. Raises ValueError for NaN or
    infinite activations (as the reference's KMeans input check does) and for weights
    that are negative or not finite; RuntimeError when the library is missing, and
    when at least 2^n_bits distinct values fall into
    fewer than 2^n_bits of the 8192 histogram bins (values bunched far below the
    bin width of their range), which the GPU method does not resolve.
    """
    from ..kernels.cuda_ops import _check, _ptr, _stream, get_cuda_ops

    if not activations.is_cuda:
        raise RuntimeError("fit_nuq_codebook_cuda: activations must be a CUDA tensor")
    lib = get_cuda_ops().lib
    n_clusters = 2 ** int(n_bits)
    x = activations.reshape(-1).to(torch.float32).contiguous()
    w = fisher.reshape(-1).to(device=x.device, dtype=torch.float32).contiguous()
    if w.numel() != x.numel():
        raise ValueError(f"fisher has {w.numel()} values for {x.numel()} activations")
    n = x.numel()
    if n == 0:
        return torch.zeros(n_clusters, dtype=torch.float32, device=x.device)
    if n < n_clusters:
        return _pad_sorted(x, n_clusters)
    ws = torch.empty(max(int(lib.kvq_fit_codebook_workspace(n)), 1), dtype=torch.uint8,
                     device=x.device)
    status = torch.zeros(2, dtype=torch.int32, device=x.device)
    out = torch.empty(n_clusters, dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        _check(lib.kvq_fit_codebook(_ptr(x), _ptr(w), n, int(n_bits), int(refine_iters),
                                    _ptr(out), _ptr(ws), ws.numel(), _ptr(status),
                                    _stream(x)), lib)
    flag, occupied = (int(v) for v in status.cpu())
    if flag & 2:
        raise ValueError("activations contain NaN or infinity")
    if flag & 4:
        raise ValueError("fisher weights must be finite and non-negative")
    if flag:
        uniq = torch.unique(x)
        if uniq.numel() < n_clusters:
            return _pad_sorted(uniq, n_clusters)
        raise CodebookBinsError(
            f"fit_nuq_codebook_cuda: {uniq.numel()} distinct values fall into {occupied} "
            f"of the 8192 histogram bins, fewer than the {n_clusters} clusters")
    return out


def train_nuq_codebook(activations: torch.Tensor, fisher: torch.Tensor, n_bits: int = 3):
    """activations [N] in [-1, 1], fisher [N] weights -> sorted fp32 centers [2^n_bits]."""
    if activations.is_cuda:
        try:
            return fit_nuq_codebook_cuda(activations, fisher, n_bits).cpu()
        except CodebookBinsError:
            activations, fisher = activations.cpu(), fisher.cpu()
    from sklearn.cluster import KMeans

    n_clusters = 2 ** n_bits
    X = activations.reshape(-1).float().cpu().numpy()
    w = fisher.reshape(-1).float().cpu().numpy()
    if X.size == 0:
        return torch.zeros(n_clusters, dtype=torch.float32)
    w = w / (w.sum() + 1e-8)
    if X.size < n_clusters:
        centers = np.sort(X)
        pad = np.full(n_clusters - centers.size, centers[-1])
        return torch.tensor(np.sort(np.concatenate([centers, pad])), dtype=torch.float32)
    uniq = np.unique(X)
    if uniq.size < n_clusters:
        pad = np.full(n_clusters - uniq.size, uniq[-1])
        return torch.tensor(np.sort(np.concatenate([uniq, pad])), dtype=torch.float32)
    kmeans = KMeans(n_clusters=n_clusters, n_init=10, max_iter=100, random_state=0)
    kmeans.fit(X.reshape(-1, 1), sample_weight=w)
    centers = torch.tensor(kmeans.cluster_centers_.flatten(), dtype=torch.float32)
    return torch.sort(centers).values
