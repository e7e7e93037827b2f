"""NUQ codebook fitting (drop-in for kvquant/quant/nuq.py).

Offline calibration, not part of the decode path: a Fisher-weighted 1-D
k-means with the reference's settings (n_init=10, max_iter=100,
random_state=0; nuq.py:39-44) and its degenerate-input rules (nuq.py:20-37),
using the same third-party solver (scikit-learn KMeans).
"""
from __future__ import annotations

import numpy as np
import torch


def train_nuq_codebook(activations: torch.Tensor, fisher: torch.Tensor, n_bits: int = 3):
    """activations [N] in [-1, 1], fisher [N] weights -> sorted fp32 centers [2^n_bits]."""
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
