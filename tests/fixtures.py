"""Shared seeded test workloads (small enough for the CPU oracle)."""
from __future__ import annotations

import copy
import functools

import numpy as np
import torch

from gofann import _abi as A, index_build, planner, synth


@functools.lru_cache(maxsize=None)
def cfg1_small(n=6000, n_labels=16, n_queries=160, threshold=400, degree=32, pq_dim=32, seed=0, dim=128):
    w = synth.config1(seed=seed, n=n, n_labels=n_labels, n_queries=n_queries, dim=dim)
    idx = index_build.build_index(w, threshold=threshold, degree=degree, pq_dim=pq_dim, seed=seed)
    plan = planner.plan_queries(idx, w.query_labels)
    return w, idx, plan


@functools.lru_cache(maxsize=None)
def cfg2_small(n=5000, vocab=120, n_queries=160, threshold=300, degree=64, pq_dim=48, seed=1):
    w = synth.config2_small(seed=seed, n=n, vocab=vocab, n_queries=n_queries)
    idx = index_build.build_index(w, threshold=threshold, degree=degree, pq_dim=pq_dim, seed=seed)
    plan = planner.plan_queries(idx, w.query_labels)
    return w, idx, plan


@functools.lru_cache(maxsize=None)
def cfg2_small_u8cb(pq_dim=48):
    """cfg2_small with its codebook rounded to integers in 0..255 and the
    codes re-encoded against it: the preconditions of GOFANN_PQ_U8."""
    from oracle import oracle as O
    w, idx, plan = cfg2_small(pq_dim=pq_dim)
    cent = np.clip(np.rint(idx.pq_centroids), 0, 255).astype(np.float32)
    idx2 = copy.copy(idx)
    idx2.pq_centroids = cent
    idx2.pq_codes = O.pq_encode(w.base.astype(np.float32), cent, idx.pq_codes.shape[1])
    return w, idx2, plan


def random_orthogonal(p: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    q, r = np.linalg.qr(rng.standard_normal((p, p)))
    q *= np.sign(np.diag(r))
    return q.astype(np.float32)


@functools.lru_cache(maxsize=None)
def rabitq_artifacts(n=6000, n_labels=16, n_queries=160, n_anchors=16, seed=3, dim=128):
    """RaBitQ codes for a config-1 style workload of `dim` dimensions:
    rotation, anchors, 1-bit codes and factors from the oracle's encoder;
    rotated queries."""
    from oracle import oracle as O
    w, idx, plan = cfg1_small(n=n, n_labels=n_labels, n_queries=n_queries, dim=dim)
    rng = np.random.default_rng(seed)
    p = ((w.dim + 63) // 64) * 64
    rot = random_orthogonal(p, seed)
    pad = lambda x: np.pad(x.astype(np.float32), ((0, 0), (0, p - x.shape[1])))
    xr = pad(w.base) @ rot
    anchors = xr[rng.choice(w.n, n_anchors, replace=False)]
    anchor_ids = np.argmin(((xr[:, None, :] - anchors[None]) ** 2).sum(-1), axis=1).astype(np.uint32)
    codes, factors = O.rabitq_encode(xr - anchors[anchor_ids], anchors, anchor_ids)
    qr = (pad(w.queries) @ rot).astype(np.float32)
    return w, idx, plan, {"rq_codes": codes, "rq_factors": factors, "rq_anchor_ids": anchor_ids,
                          "num_anchors": n_anchors}, anchors.astype(np.float32), qr


def dev(a, device="cuda"):
    """numpy -> torch device tensor (unsigned views as signed of equal width)."""
    if a is None:
        return None
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint64:
        a = a.view(np.int64)
    elif a.dtype == np.uint32:
        a = a.view(np.int32)
    elif a.dtype == np.uint16:
        a = a.view(np.int16)
    elif a.dtype.fields is not None:
        a = a.view(np.uint8).reshape(-1)
    return torch.from_numpy(a).to(device)


def dev_dict(d: dict, device="cuda") -> dict:
    return {k: (dev(v, device) if isinstance(v, np.ndarray) else v) for k, v in d.items()}


def host(t: torch.Tensor, dtype) -> np.ndarray:
    return t.cpu().numpy().view(dtype)


def fbits(x) -> np.ndarray:
    return np.ascontiguousarray(x, np.float32).view(np.uint32)
