"""Index artefacts in the reference's layout, built from a Workload.

Produces what the search path consumes (GraphRuntime / GraphMetadata /
LowfreqPostingIndex of src/data/dataloader.h:569-602,753-836):
  * per-label graphs for labels whose cardinality exceeds the specificity
    threshold, concatenated row-wise with label_offset[group] + local_row
    addressing, row_to_sample, a seed row per group;
  * posting lists (sorted sample ids) for every label, used as the
    low-frequency routes;
  * PQ codebook [256][dim] (full-dim layout, backend_pq.cu:1812-1815) and
    uint8 codes.

Graph and codebook *training* are outside the reference's hot path (it uses
cuVS CAGRA/Vamana and cuVS PQ, which are absent here); these are simple,
seeded stand-ins.  Graphs: per label, `degree - n_random` exact (or
block-approximate, for very large labels) nearest neighbours plus
`n_random` random members for long-range navigation.  All heavy math runs
in torch on the given device.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

U32MAX = 0xFFFFFFFF


@dataclass
class Index:
    dim: int
    dtype: str
    base: np.ndarray
    label_indptr: np.ndarray
    label_indices: np.ndarray
    n_labels: int
    threshold: int
    degree: int
    adjacency: np.ndarray       # [rows][degree] u32 local rows, U32MAX padding
    row_to_sample: np.ndarray   # [rows] u32
    label_offset: np.ndarray    # [groups] u32
    group_label: np.ndarray     # [groups] u32
    label_group: np.ndarray     # [n_labels] i64, -1 when low-frequency
    seeds: np.ndarray           # [groups] u32 local seed row
    posting_ids: np.ndarray     # concatenated sorted members of every label
    posting_begin: np.ndarray   # [n_labels] u64
    posting_count: np.ndarray   # [n_labels] u32
    pq_centroids: np.ndarray | None = None  # [256][dim] f32
    pq_codes: np.ndarray | None = None      # [n][M] u8

    def attrs(self) -> dict:
        return {"label_indptr": self.label_indptr, "label_indices": self.label_indices}

    def graph(self) -> dict:
        return {"adjacency": self.adjacency, "row_to_sample": self.row_to_sample, "label_offset": self.label_offset}

    def codes(self) -> dict:
        return {"pq_codes": self.pq_codes}


def _as_float(x: np.ndarray | torch.Tensor, device) -> torch.Tensor:
    t = torch.as_tensor(x, device=device)
    return t.float()


def label_members(indptr: np.ndarray, indices: np.ndarray, n_labels: int):
    """CSR of sample ids per label (each list sorted ascending)."""
    n = indptr.shape[0] - 1
    rows = np.repeat(np.arange(n, dtype=np.uint32), np.diff(indptr).astype(np.int64))
    order = np.lexsort((rows, indices))
    lab_sorted = indices[order]
    members = rows[order]
    count = np.bincount(lab_sorted, minlength=n_labels).astype(np.uint32)
    begin = np.zeros(n_labels, np.uint64)
    begin[1:] = np.cumsum(count[:-1], dtype=np.uint64)
    return members.astype(np.uint32), begin, count


def train_pq(x, pq_dim: int, iters: int = 12, seed: int = 0, sample: int = 65536, device="cpu") -> np.ndarray:
    """Lloyd k-means with 256 centroids per subspace, all subspaces batched."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    n, dim = x.shape
    w = dim // pq_dim
    idx = torch.randperm(n, generator=g)[: min(sample, n)]
    xs = _as_float(np.asarray(x)[idx.numpy()], device).view(-1, pq_dim, w).transpose(0, 1).contiguous()  # [M, s, w]
    init = torch.randperm(xs.shape[1], generator=g)[:256].to(device)
    cent = xs[:, init, :].clone()  # [M, 256, w]
    for _ in range(iters):
        d = torch.cdist(xs, cent)  # [M, s, 256]
        a = d.argmin(dim=2)        # [M, s]
        sums = torch.zeros_like(cent).scatter_add_(1, a.unsqueeze(-1).expand(-1, -1, w), xs)
        cnt = torch.zeros(cent.shape[:2], device=device).scatter_add_(1, a, torch.ones_like(a, dtype=torch.float32))
        empty = cnt == 0
        cent = torch.where(empty.unsqueeze(-1), cent, sums / cnt.clamp(min=1).unsqueeze(-1))
    # full-dim layout: centroid c, subspace m at [c, m*w:(m+1)*w]
    return cent.transpose(0, 1).reshape(256, dim).contiguous().cpu().numpy().astype(np.float32)


def encode_pq(x, centroids: np.ndarray, pq_dim: int, device="cpu", chunk: int = 1 << 16) -> np.ndarray:
    n, dim = x.shape
    w = dim // pq_dim
    c = torch.as_tensor(centroids, device=device).view(256, pq_dim, w).transpose(0, 1).contiguous()  # [M,256,w]
    out = np.empty((n, pq_dim), np.uint8)
    for s in range(0, n, chunk):
        xs = _as_float(np.asarray(x)[s:s + chunk], device).view(-1, pq_dim, w).transpose(0, 1)  # [M, b, w]
        d = torch.cdist(xs, c)
        out[s:s + chunk] = d.argmin(dim=2).transpose(0, 1).to(torch.uint8).cpu().numpy()
    return out


def knn_within(x: torch.Tensor, k: int, chunk: int = 4096) -> torch.Tensor:
    """Exact k nearest neighbours (excluding self) by brute force; [n, k] int64."""
    n = x.shape[0]
    k = min(k, n - 1)
    if k <= 0:
        return torch.empty((n, 0), dtype=torch.int64, device=x.device)
    sq = (x * x).sum(1)
    out = torch.empty((n, k), dtype=torch.int64, device=x.device)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        d = sq[s:e, None] + sq[None, :] - 2.0 * (x[s:e] @ x.T)
        d[torch.arange(e - s, device=x.device), torch.arange(s, e, device=x.device)] = float("inf")
        out[s:e] = d.topk(k, dim=1, largest=False).indices
    return out


def build_label_graph(x: torch.Tensor, degree: int, n_random: int, gen: torch.Generator) -> tuple[np.ndarray, int]:
    """Local adjacency [n][degree] (U32MAX padded) and the seed row."""
    n = x.shape[0]
    adj = np.full((n, degree), U32MAX, np.uint32)
    n_near = max(degree - n_random, 1)
    nn = knn_within(x, n_near).cpu().numpy()
    adj[:, : nn.shape[1]] = nn
    if n > n_near + 1 and n_random > 0:
        r = torch.randint(0, n, (n, n_random), generator=gen).numpy().astype(np.uint32)
        adj[:, n_near:n_near + n_random] = r
        # drop self loops and duplicates of the near list (keep first occurrence)
        for i in range(n_near, n_near + n_random):
            col = adj[:, i]
            bad = col == np.arange(n, dtype=np.uint32)
            bad |= (adj[:, :i] == col[:, None]).any(axis=1)
            col[bad] = U32MAX
    mean = x.mean(0, keepdim=True)
    seed_row = int(((x - mean) ** 2).sum(1).argmin().item())
    return adj, seed_row


def build_index(w, threshold: int, degree: int, pq_dim: int | None = None, n_random: int | None = None,
                seed: int = 0, device="cpu", pq_iters: int = 12, pq_codes=None, pq_centroids=None) -> Index:
    """Per-label graphs + postings (+ PQ) for a synth.Workload."""
    n_random = degree // 4 if n_random is None else n_random
    members, begin, count = label_members(w.label_indptr, w.label_indices, w.n_labels)
    high = np.nonzero(count > threshold)[0]
    gen = torch.Generator(device="cpu").manual_seed(seed + 1)
    adjs, r2s, offsets, seeds = [], [], [], []
    row = 0
    label_group = np.full(w.n_labels, -1, np.int64)
    for gi, lab in enumerate(high):
        mem = members[begin[lab]: begin[lab] + count[lab]]
        xl = _as_float(w.base[mem], device)
        adj, srow = build_label_graph(xl, degree, n_random, gen)
        adjs.append(adj)
        r2s.append(mem)
        offsets.append(row)
        seeds.append(srow)
        label_group[lab] = gi
        row += mem.shape[0]
    adjacency = np.concatenate(adjs) if adjs else np.zeros((0, degree), np.uint32)
    idx = Index(
        dim=w.dim, dtype=w.dtype, base=w.base, label_indptr=w.label_indptr, label_indices=w.label_indices,
        n_labels=w.n_labels, threshold=threshold, degree=degree, adjacency=np.ascontiguousarray(adjacency),
        row_to_sample=np.concatenate(r2s).astype(np.uint32) if r2s else np.zeros(0, np.uint32),
        label_offset=np.asarray(offsets, np.uint32), group_label=high.astype(np.uint32), label_group=label_group,
        seeds=np.asarray(seeds, np.uint32), posting_ids=members, posting_begin=begin, posting_count=count)
    if pq_dim is not None:
        if pq_centroids is None:
            pq_centroids = train_pq(w.base, pq_dim, iters=pq_iters, seed=seed, device=device)
        idx.pq_centroids = pq_centroids
        idx.pq_codes = pq_codes if pq_codes is not None else encode_pq(w.base, pq_centroids, pq_dim, device=device)
    return idx
