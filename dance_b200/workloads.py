"""Seeded synthetic workloads with the shapes of BASELINE.json's configs.

The reference's public datasets (DEEP1B, SIFT/BIGANN, YFCC) are not used;
these generators reproduce the stated shapes and value distributions:
  cfg0  N=1e6,  d=96  float32: 1000-centroid Gaussian mixture, centroids
        N(0,1), per-cluster sigma 0.3, rows L2-normalised
  cfg1  N=1e7,  d=128 uint8: 4096 centroids U[0,255], per-dim noise N(0,20),
        clipped to [0,255] and rounded
  cfg2  cfg0 vectors + 1..5 labels per point from a 1000-label vocabulary,
        drawn without replacement with Zipf(s=1) popularity
  cfg3  cfg0 vectors + exactly one label per point from 100 labels with
        Zipf(s=1) label sizes
  cfg4  N=1e8, d=96 float32 with 16384 centroids (cfg0 recipe)
Generation runs on any torch device (CUDA for the full sizes) with a
torch.Generator seeded by `seed`; the same (device, seed, n) gives the same
data.  Ground truth is brute force (exact integer arithmetic for uint8,
float64 for float32).
"""
from __future__ import annotations

import numpy as np
import torch


def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    return g


def gaussian_mixture_f32(n: int, dim: int = 96, centroids: int = 1000, sigma: float = 0.3, seed: int = 42,
                         device="cpu", chunk: int = 1 << 20, normalize: bool = True,
                         stream_offset: int = 0) -> torch.Tensor:
    """Normalised Gaussian-mixture float32 vectors (cfg0/cfg2/cfg3/cfg4 recipe).

    `stream_offset` selects an independent stream of points from the same
    mixture (queries use offset 1)."""
    g = _gen(device, seed)
    cent = torch.randn((centroids, dim), generator=g, device=device, dtype=torch.float32)
    gp = _gen(device, seed * 1000003 + 17 + stream_offset)
    out = torch.empty((n, dim), dtype=torch.float32, device=device)
    for b in range(0, n, chunk):
        e = min(n, b + chunk)
        a = torch.randint(0, centroids, (e - b,), generator=gp, device=device)
        x = cent[a] + sigma * torch.randn((e - b, dim), generator=gp, device=device, dtype=torch.float32)
        if normalize:
            x = x / torch.linalg.vector_norm(x, dim=1, keepdim=True).clamp_min(1e-30)
        out[b:e] = x
    return out


def clustered_u8(n: int, dim: int = 128, centroids: int = 4096, noise: float = 20.0, seed: int = 42, device="cpu",
                 chunk: int = 1 << 20, stream_offset: int = 0) -> torch.Tensor:
    """uint8 mixture: centroids U[0,255], N(0, noise^2) per dimension, clip, round (cfg1)."""
    g = _gen(device, seed)
    cent = torch.rand((centroids, dim), generator=g, device=device, dtype=torch.float32) * 255.0
    gp = _gen(device, seed * 1000003 + 29 + stream_offset)
    out = torch.empty((n, dim), dtype=torch.uint8, device=device)
    for b in range(0, n, chunk):
        e = min(n, b + chunk)
        a = torch.randint(0, centroids, (e - b,), generator=gp, device=device)
        x = cent[a] + noise * torch.randn((e - b, dim), generator=gp, device=device, dtype=torch.float32)
        out[b:e] = torch.round(x.clamp_(0.0, 255.0)).to(torch.uint8)
    return out


def zipf_multilabels(n: int, vocab: int = 1000, min_labels: int = 1, max_labels: int = 5, seed: int = 42):
    """Per-point label sets (cfg2): count ~ U{min..max}, labels without
    replacement with P(label rank r) proportional to 1/r.  Returns a CSR
    (offsets[n+1], labels) with every row strictly increasing."""
    rng = np.random.default_rng(seed)
    p = 1.0 / np.arange(1, vocab + 1)
    p /= p.sum()
    counts = rng.integers(min_labels, max_labels + 1, size=n)
    offsets = np.zeros(n + 1, dtype=np.uint32)
    offsets[1:] = np.cumsum(counts)
    labels = np.empty(int(offsets[-1]), dtype=np.uint32)
    # Gumbel-top-k sampling without replacement
    for c in range(min_labels, max_labels + 1):
        rows = np.nonzero(counts == c)[0]
        if len(rows) == 0:
            continue
        keys = np.log(p)[None, :] - np.log(-np.log(rng.random((len(rows), vocab))))
        top = np.argpartition(-keys, c - 1, axis=1)[:, :c]
        top.sort(axis=1)
        for j, r in enumerate(rows):
            labels[offsets[r]:offsets[r] + c] = top[j]
    return offsets, labels


def zipf_partition_labels(n: int, num_labels: int = 100, seed: int = 42) -> np.ndarray:
    """Exactly one label per point (cfg3) with Zipf(s=1) label sizes."""
    rng = np.random.default_rng(seed)
    p = 1.0 / np.arange(1, num_labels + 1)
    p /= p.sum()
    return rng.choice(num_labels, size=n, p=p).astype(np.uint32)


def brute_force_knn(base: torch.Tensor, queries: torch.Tensor, k: int = 10, qchunk: int = 1024,
                    bchunk: int = 1 << 20):
    """Exact top-k by squared L2, ties broken by id.  uint8 uses exact integer
    dot products (float32 sums of integers below 2^24); float uses float64.
    Tiled over queries and base so the distance tile stays a few GB."""
    dev = base.device
    exact_f32 = base.dtype == torch.uint8
    ct = torch.float32 if exact_f32 else torch.float64
    kk = min(base.shape[0], k + 16)
    prev = None
    if dev.type == "cuda":
        prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
    try:
        out_i = torch.empty((queries.shape[0], k), dtype=torch.int64, device=dev)
        out_d = torch.empty((queries.shape[0], k), dtype=torch.float64, device=dev)
        for qb in range(0, queries.shape[0], qchunk):
            q = queries[qb:qb + qchunk].to(ct)
            qn = (q * q).sum(1)
            best_d = None
            best_i = None
            for bb in range(0, base.shape[0], bchunk):
                B = base[bb:bb + bchunk].to(ct)
                d = (B * B).sum(1)[None, :] - 2.0 * (q @ B.T) + qn[:, None]
                kc = min(kk, B.shape[0])
                v, i = torch.topk(d, kc, dim=1, largest=False)
                v = v.to(torch.float64)
                i = i + bb
                if best_d is None:
                    best_d, best_i = v, i
                else:
                    cd = torch.cat([best_d, v], 1)
                    ci = torch.cat([best_i, i], 1)
                    v2, j = torch.topk(cd, min(kk, cd.shape[1]), dim=1, largest=False)
                    best_d, best_i = v2, torch.gather(ci, 1, j)
            # order the candidates by (distance, id)
            o = torch.argsort(best_i, dim=1)
            d2 = torch.gather(best_d, 1, o)
            i2 = torch.gather(best_i, 1, o)
            o2 = torch.argsort(d2, dim=1, stable=True)
            out_i[qb:qb + qchunk] = torch.gather(i2, 1, o2)[:, :k]
            out_d[qb:qb + qchunk] = torch.gather(d2, 1, o2)[:, :k]
        return out_i, out_d
    finally:
        if prev is not None:
            torch.backends.cuda.matmul.allow_tf32 = prev
