"""Seeded synthetic workloads standing in for the reference's datasets.

The reference measures on YFCC10M / arxiv / LAION (not available offline);
these generators reproduce the shapes, sizes and value distributions that
the benchmark configurations name: Gaussian-mixture vectors, Zipf label
frequencies, single-label or AND-of-tags queries.  Everything is a pure
function of the seed.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


def zipf_probs(n: int, s: float) -> np.ndarray:
    w = 1.0 / np.arange(1, n + 1, dtype=np.float64) ** s
    return w / w.sum()


def gaussian_mixture(rng: np.random.Generator, n: int, dim: int, centres: np.ndarray, sigma: float):
    """Samples n points; returns (points f32, component ids)."""
    comp = rng.integers(0, centres.shape[0], size=n)
    x = centres[comp] + sigma * rng.standard_normal((n, dim), dtype=np.float32)
    return x.astype(np.float32), comp.astype(np.int32)


def csr_from_lists(rows: list[np.ndarray]):
    indptr = np.zeros(len(rows) + 1, np.uint64)
    indptr[1:] = np.cumsum([len(r) for r in rows], dtype=np.uint64)
    indices = np.concatenate(rows).astype(np.uint32) if rows else np.zeros(0, np.uint32)
    return indptr, indices


@dataclass
class Workload:
    """Base vectors, labels and labelled queries of one configuration."""
    name: str
    base: np.ndarray                 # [n, dim] f32 or u8
    dtype: str                       # "f32" | "u8" | "f16"
    label_indptr: np.ndarray         # [n+1] u64, sorted unique labels per row
    label_indices: np.ndarray        # [nnz] u32
    n_labels: int
    queries: np.ndarray              # [q, dim] same dtype as base (f32 for f16)
    query_labels: list               # per query: np.ndarray of labels (AND)
    k: int = 10
    extra: dict = field(default_factory=dict)

    @property
    def n(self) -> int:
        return int(self.base.shape[0])

    @property
    def dim(self) -> int:
        return int(self.base.shape[1])

    def label_cardinality(self) -> np.ndarray:
        return np.bincount(self.label_indices, minlength=self.n_labels).astype(np.int64)


def config1(seed: int = 0, n: int = 100_000, dim: int = 128, n_centres: int = 64, sigma: float = 0.3,
            n_labels: int = 100, zipf_s: float = 1.0, n_queries: int = 1000) -> Workload:
    """BASELINE config 1 (CPU-runnable): Gaussian mixture f32, one Zipf label per
    vector, single-label equality queries drawn from the same mixture."""
    rng = np.random.default_rng(seed)
    centres = rng.standard_normal((n_centres, dim), dtype=np.float32)
    base, _ = gaussian_mixture(rng, n, dim, centres, sigma)
    p = zipf_probs(n_labels, zipf_s)
    labels = rng.choice(n_labels, size=n, p=p).astype(np.uint32)
    indptr = np.arange(n + 1, dtype=np.uint64)
    queries, _ = gaussian_mixture(rng, n_queries, dim, centres, sigma)
    qlab = rng.choice(n_labels, size=n_queries, p=p).astype(np.uint32)
    return Workload("config1", base, "f32", indptr, labels, n_labels, queries, [np.array([l], np.uint32) for l in qlab])


def config2_small(seed: int = 0, n: int = 20_000, dim: int = 192, n_centres: int = 64, vocab: int = 400,
                  zipf_s: float = 1.1, max_tags: int = 20, n_queries: int = 200) -> Workload:
    """Scaled-down BASELINE config 2 shape: uint8 mixture, 1..max_tags Zipf tags
    per vector, queries AND of 1-2 tags (used by parity tests)."""
    rng = np.random.default_rng(seed)
    centres = rng.uniform(40, 215, size=(n_centres, dim)).astype(np.float32)
    x, _ = gaussian_mixture(rng, n, dim, centres, 18.0)
    base = np.clip(np.rint(x), 0, 255).astype(np.uint8)
    p = zipf_probs(vocab, zipf_s)
    rows = []
    for _ in range(n):
        t = rng.integers(1, max_tags + 1)
        rows.append(np.unique(rng.choice(vocab, size=t, p=p)).astype(np.uint32))
    indptr, indices = csr_from_lists(rows)
    qx, _ = gaussian_mixture(rng, n_queries, dim, centres, 18.0)
    queries = np.clip(np.rint(qx), 0, 255).astype(np.uint8)
    qlabels = []
    for i in range(n_queries):
        # AND of 1-2 tags, both present on one sampled base row so the
        # conjunction is satisfiable
        r = rows[rng.integers(0, n)]
        m = 1 if (len(r) < 2 or rng.random() < 0.5) else 2
        qlabels.append(np.sort(rng.choice(r, size=m, replace=False)).astype(np.uint32))
    return Workload("config2_small", base, "u8", indptr, indices, vocab, queries, qlabels)
