"""Multi-GPU layout of the filtered-search path: the base set is split into
contiguous id ranges, one per rank; every rank holds its own per-label
graphs, postings, codes and rerank store (the specificity threshold applies
per shard), runs the whole route set of the replicated query batch, and the
ranks exchange only their per-query top-k: one all-gather of
[queries][k] ids and distances, then a (dist, id) merge on every rank
(rabitq_lowfreq_merge.h:800-806 order).  The reference is single-GPU; this
is the one exchange step the path has.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _abi as A


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Rows [lo, hi) of an n-row base set owned by `rank` of `world`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    return rank * n // world, (rank + 1) * n // world


def shard_data(data: dict, lo: int, hi: int, device) -> dict:
    """Rows [lo, hi) of a generated workload (base vectors, sample-major label
    CSR, per-label postings) re-indexed to local ids 0..hi-lo-1.  Queries are
    shared, not copied."""
    if not 0 <= lo <= hi <= data["n"]:
        raise ValueError(f"shard [{lo}, {hi}) outside [0, {data['n']})")
    if hi - lo >= 1 << 24:
        raise ValueError("a shard holds fewer than 2^24 rows (posting sort key)")
    ip = data["label_indptr"]
    a, b = int(ip[lo]), int(ip[hi])
    indptr = ip[lo:hi + 1] - a
    indices = data["label_indices"][a:b]
    base = data["base"][lo:hi]
    vocab = data["vocab"]
    rows = torch.repeat_interleave(torch.arange(hi - lo, device=device, dtype=torch.int64), indptr[1:] - indptr[:-1])
    key = torch.sort((indices.to(torch.int64) << 24) | rows).values
    pid = (key & ((1 << 24) - 1)).to(torch.int32)
    card = torch.bincount(indices, minlength=vocab).cpu().numpy().astype(np.int64)
    begin = np.zeros(vocab, np.int64)
    begin[1:] = np.cumsum(card)[:-1]
    return dict(base=base, label_indptr=indptr, label_indices=indices, posting_ids=pid, card=card, begin=begin,
                queries=data["queries"], vocab=vocab, dim=data["dim"], n=hi - lo)


class ShardExchange:
    """Per-batch exchange of each rank's top-k.  Buffers are allocated once;
    every rank calls exchange() in the same order (one all-gather of ids, one
    of distances)."""

    def __init__(self, world: int, n_queries: int, k: int, device, group=None):
        self.world, self.n_queries, self.k, self.group = world, n_queries, k, group
        self.all_ids = torch.empty((world, n_queries, k), dtype=torch.int32, device=device)
        self.all_dists = torch.empty((world, n_queries, k), dtype=torch.float32, device=device)
        self.ids = torch.empty((n_queries, k), dtype=torch.int32, device=device)
        self.dists = torch.empty((n_queries, k), dtype=torch.float32, device=device)

    def gather(self, ids: torch.Tensor, dists: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """All-gather of [queries][k] global ids + distances into
        [world][queries][k] (rank-major, the layout gofann_shard_merge reads)."""
        import torch.distributed as dist
        if ids.shape != (self.n_queries, self.k) or dists.shape != (self.n_queries, self.k):
            raise ValueError(f"expected [{self.n_queries}, {self.k}] ids and distances")
        dist.all_gather_into_tensor(self.all_ids.view(-1), ids.reshape(-1).contiguous(), group=self.group)
        dist.all_gather_into_tensor(self.all_dists.view(-1), dists.reshape(-1).contiguous(), group=self.group)
        return self.all_ids, self.all_dists

    def exchange(self, ids: torch.Tensor, dists: torch.Tensor, shard_base: int,
                 stream: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Local top-k (local ids) -> merged global top-k on every rank:
        gofann_offset_ids, all-gather, gofann_shard_merge (device kernels)."""
        L = A.lib()
        A.check(L.gofann_offset_ids(A.ptr(ids), ids.numel(), shard_base, stream), "offset_ids")
        self.gather(ids, dists)
        A.check(L.gofann_shard_merge(A.ptr(self.all_ids), A.ptr(self.all_dists), self.world, self.n_queries,
                                     self.k, A.ptr(self.ids), A.ptr(self.dists), stream), "shard_merge")
        return self.ids, self.dists
