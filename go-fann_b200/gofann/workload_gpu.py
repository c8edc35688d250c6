"""BASELINE configuration 2 built on the GPU: synthetic data, index, ground truth.

Stand-in for the reference's YFCC10M categorical workload (10M x 192 uint8,
~200k tags, AND-of-tags queries; the dataset is not available offline):

  * base: 10M x 192 uint8 from a 1,024-centre Gaussian mixture (centres
    N(0,1), sigma 0.5), mapped by 128 + 40 x and clipped to 0..255;
  * tags: 1..20 per vector from a 200k vocabulary with Zipf(1.1)
    frequencies (duplicates within a row collapse);
  * queries: 100k mixture samples; half one tag, half an AND of two tags
    that co-occur on some base row; the first tag is the one whose
    selectivity is closest to a log-uniform target in [1e-5, 0.3];
  * index: PQ 48 x 256, per-label graphs of degree 64 for labels above the
    specificity threshold (2,000, the reference default), postings for all
    labels;
  * ground truth: exact filtered top-10 by brute force on a query sample.

Graph construction (outside the hot path; the reference uses cuVS
CAGRA/Vamana) is a window k-NN: each label's members are ordered by coarse
cluster and a random projection, tiles of 1,024 rows take their 24 nearest
inside a 2,048-row window (TF32 GEMMs, exact for uint8 inputs), plus 40
random long-range edges per row (on the 10M workload this mix reached
recall@10 0.957 at queue 256, against 0.946 with 48 near + 16 random).
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _abi as A


def _log(msg: str, t0: float) -> None:
    print(f"[workload {time.time() - t0:7.1f}s] {msg}", flush=True)


@dataclass
class GpuIndex:
    """Device-resident index with the same fields DeviceIndex/planner read."""
    dim: int
    dtype: str
    n: int
    base: torch.Tensor              # [n, dim] u8
    label_indptr: torch.Tensor      # [n+1] i64
    label_indices: torch.Tensor     # [nnz] i32
    n_labels: int
    threshold: int
    degree: int
    adjacency: torch.Tensor         # [rows, degree] i32 (local rows, -1 padding)
    row_to_sample: torch.Tensor     # [rows] i32
    label_offset: np.ndarray        # [groups] u32
    group_label: np.ndarray         # [groups] u32
    label_group: np.ndarray         # [n_labels] i64
    seeds: np.ndarray               # [groups] u32
    posting_ids: torch.Tensor       # [nnz] i32
    posting_begin: np.ndarray       # [n_labels] u64
    posting_count: np.ndarray       # [n_labels] u32
    pq_centroids: torch.Tensor      # [256, dim] f32
    pq_codes: torch.Tensor          # [n, M] u8
    stats: dict = field(default_factory=dict)


@dataclass
class Queries:
    vectors: torch.Tensor           # [q, dim] u8 (device)
    labels: list                    # per query np.ndarray of tags (AND)
    selectivity: np.ndarray         # [q] fraction of base rows passing


def zipf_cdf(vocab: int, s: float, device) -> torch.Tensor:
    w = 1.0 / torch.arange(1, vocab + 1, dtype=torch.float64, device=device) ** s
    c = torch.cumsum(w, 0)
    return c / c[-1]


def generate(device="cuda", seed=0, n=10_000_000, dim=192, n_centres=1024, vocab=200_000, zipf_s=1.1,
             max_tags=20, n_queries=100_000, sel_lo=1e-5, sel_hi=0.3, sigma=0.5, scale=40.0, t0=None):
    t0 = t0 or time.time()
    g = torch.Generator(device=device).manual_seed(seed)
    centres = torch.randn((n_centres, dim), generator=g, device=device)
    base = torch.empty((n, dim), dtype=torch.uint8, device=device)
    chunk = 1 << 20
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        comp = torch.randint(0, n_centres, (e - s,), generator=g, device=device)
        x = centres[comp] + sigma * torch.randn((e - s, dim), generator=g, device=device)
        base[s:e] = (128.0 + scale * x).round_().clamp_(0, 255).to(torch.uint8)
    _log(f"base {n} x {dim} u8", t0)
    # tags
    cdf = zipf_cdf(vocab, zipf_s, device)
    per_row = torch.randint(1, max_tags + 1, (n,), generator=g, device=device)
    total = int(per_row.sum())
    rows = torch.repeat_interleave(torch.arange(n, device=device, dtype=torch.int64), per_row)
    u = torch.rand(total, generator=g, device=device, dtype=torch.float64)
    tags = torch.searchsorted(cdf, u).clamp_(max=vocab - 1)
    key = torch.unique((rows << 18) | tags)  # sorted, duplicates within a row collapse
    del rows, tags, u
    rows_u = key >> 18
    tags_u = (key & ((1 << 18) - 1)).to(torch.int32)
    counts = torch.bincount(rows_u, minlength=n)
    indptr = torch.zeros(n + 1, dtype=torch.int64, device=device)
    indptr[1:] = torch.cumsum(counts, 0)
    # postings: members of each tag in ascending row order
    key2 = torch.sort((tags_u.to(torch.int64) << 24) | rows_u).values
    posting_ids = (key2 & ((1 << 24) - 1)).to(torch.int32)
    card = torch.bincount(tags_u, minlength=vocab)
    del key2, key, rows_u
    _log(f"tags: {int(tags_u.numel())} memberships, max card {int(card.max())}", t0)
    card_h = card.cpu().numpy().astype(np.int64)
    begin_h = np.zeros(vocab, np.int64)
    begin_h[1:] = np.cumsum(card_h)[:-1]
    # queries
    qc = torch.randint(0, n_centres, (n_queries,), generator=g, device=device)
    qx = centres[qc] + sigma * torch.randn((n_queries, dim), generator=g, device=device)
    qv = (128.0 + scale * qx).round_().clamp_(0, 255).to(torch.uint8)
    rng = np.random.default_rng(seed + 7)
    target = 10 ** rng.uniform(np.log10(sel_lo), np.log10(sel_hi), size=n_queries) * n
    order = np.argsort(card_h)
    sorted_card = card_h[order]
    nz = np.searchsorted(sorted_card, 1)
    pos = np.clip(np.searchsorted(sorted_card, target), nz, vocab - 1)
    lower = np.clip(pos - 1, nz, vocab - 1)
    pick = np.where(np.abs(sorted_card[lower] - target) < np.abs(sorted_card[pos] - target), lower, pos)
    tag1 = order[pick]
    two = rng.random(n_queries) < 0.5
    # second tag: another tag of a random member of tag1
    mem_pos = begin_h[tag1] + (rng.random(n_queries) * card_h[tag1]).astype(np.int64)
    mem_pos_d = torch.from_numpy(mem_pos).to(device)
    row = posting_ids[mem_pos_d].to(torch.int64)
    deg = (indptr[row + 1] - indptr[row])
    r = (torch.rand(n_queries, generator=g, device=device, dtype=torch.float64) * (deg - 1).clamp(min=0)).floor().to(torch.int64)
    p2 = indptr[row] + r
    t2 = tags_u[p2].to(torch.int64)
    t1d = torch.from_numpy(tag1).to(device)
    t2 = torch.where(t2 == t1d, tags_u[indptr[row + 1] - 1].to(torch.int64), t2)
    t2_h = t2.cpu().numpy()
    deg_h = deg.cpu().numpy()
    labels = []
    for i in range(n_queries):
        if two[i] and deg_h[i] > 1:
            labels.append(np.sort(np.array([tag1[i], t2_h[i]], np.uint32)))
        else:
            labels.append(np.array([tag1[i]], np.uint32))
    _log(f"{n_queries} queries ({int(sum(len(x) == 2 for x in labels))} two-tag)", t0)
    return dict(base=base, label_indptr=indptr, label_indices=tags_u, posting_ids=posting_ids, card=card_h,
                begin=begin_h, queries=Queries(qv, labels, np.zeros(n_queries)), vocab=vocab, dim=dim, n=n)


def train_pq_gpu(base: torch.Tensor, pq_dim: int, seed=0, sample=262_144, iters=10) -> torch.Tensor:
    n, dim = base.shape
    w = dim // pq_dim
    g = torch.Generator(device=base.device).manual_seed(seed + 3)
    idx = torch.randint(0, n, (sample,), generator=g, device=base.device)
    xs = base[idx].float().view(sample, pq_dim, w).transpose(0, 1).contiguous()  # [M, s, w]
    cent = xs[:, torch.randperm(sample, generator=g, device=base.device)[:256], :].clone()
    for _ in range(iters):
        a = torch.cdist(xs, cent).argmin(2)
        sums = torch.zeros_like(cent).scatter_add_(1, a.unsqueeze(-1).expand(-1, -1, w), xs)
        cnt = torch.zeros(cent.shape[:2], device=base.device).scatter_add_(1, a, torch.ones_like(a, dtype=torch.float32))
        cent = torch.where((cnt == 0).unsqueeze(-1), cent, sums / cnt.clamp(min=1).unsqueeze(-1))
    return cent.transpose(0, 1).reshape(256, dim).contiguous()


def coarse_assign(base: torch.Tensor, k=1024, seed=0, sample=262_144, iters=8) -> torch.Tensor:
    n, dim = base.shape
    g = torch.Generator(device=base.device).manual_seed(seed + 5)
    xs = base[torch.randint(0, n, (sample,), generator=g, device=base.device)].float()
    cent = xs[torch.randperm(sample, generator=g, device=base.device)[:k]].clone()
    for _ in range(iters):
        a = (xs.square().sum(1, keepdim=True) - 2 * xs @ cent.T + cent.square().sum(1)).argmin(1)
        sums = torch.zeros_like(cent).index_add_(0, a, xs)
        cnt = torch.bincount(a, minlength=k).float()
        cent = torch.where((cnt == 0).unsqueeze(1), cent, sums / cnt.clamp(min=1).unsqueeze(1))
    out = torch.empty(n, dtype=torch.int64, device=base.device)
    cn = cent.square().sum(1)
    for s in range(0, n, 1 << 20):
        x = base[s:s + (1 << 20)].float()
        out[s:s + x.shape[0]] = (cn - 2 * x @ cent.T).argmin(1)
    return out


def window_knn(x: torch.Tensor, k: int, tile=1024, window=2048, chunk_tiles=96, with_dist=False):
    """[n, k] label-local neighbour rows (-1 where fewer than k exist), and
    their squared distances (inf for missing) when with_dist."""
    n, dim = x.shape
    dev = x.device
    out = torch.full((n, k), -1, dtype=torch.int64, device=dev)
    outd = torch.full((n, k), float("inf"), device=dev) if with_dist else None
    sq = x.square().sum(1)
    if n <= window:
        d = sq[:, None] + sq[None, :] - 2.0 * (x @ x.T)
        d.fill_diagonal_(float("inf"))
        kk = min(k, n - 1)
        if kk > 0:
            tk = d.topk(kk, dim=1, largest=False)
            out[:, :kk] = tk.indices
            if with_dist:
                outd[:, :kk] = tk.values
        return (out, outd) if with_dist else out
    half = (window - tile) // 2
    n_tiles = (n + tile - 1) // tile
    padded = n_tiles * tile + 2 * half
    xp = torch.zeros((padded, dim), dtype=x.dtype, device=dev)
    xp[half:half + n] = x
    sqp = torch.full((padded,), float("inf"), device=dev)
    sqp[half:half + n] = sq
    ar = torch.arange(tile, device=dev)
    for t0 in range(0, n_tiles, chunk_tiles):
        t1 = min(n_tiles, t0 + chunk_tiles)
        c = t1 - t0
        q = xp.as_strided((c, tile, dim), (tile * dim, dim, 1), (half + t0 * tile) * dim)
        wv = xp.as_strided((c, window, dim), (tile * dim, dim, 1), t0 * tile * dim)
        qn = sqp.as_strided((c, tile), (tile, 1), half + t0 * tile)
        wn = sqp.as_strided((c, window), (tile, 1), t0 * tile)
        d = torch.baddbmm(qn.unsqueeze(2) + wn.unsqueeze(1), q, wv.transpose(1, 2), beta=1.0, alpha=-2.0)
        d[:, ar, ar + half] = float("inf")  # self
        tk = d.topk(k, dim=2, largest=False)  # window positions
        glob = tk.indices + (torch.arange(t0, t1, device=dev) * tile - half).view(c, 1, 1)
        lo, hi = t0 * tile, min(n, t1 * tile)
        out[lo:hi] = glob.view(c * tile, k)[: hi - lo]
        if with_dist:
            outd[lo:hi] = tk.values.view(c * tile, k)[: hi - lo]
    return (out, outd) if with_dist else out


def merge_candidates(ids: torch.Tensor, dist: torch.Tensor, k: int) -> torch.Tensor:
    """Per row, the k nearest distinct ids among the candidate columns."""
    order = torch.argsort(ids, dim=1)
    sid = torch.gather(ids, 1, order)
    sd = torch.gather(dist, 1, order)
    dup = torch.zeros_like(sid, dtype=torch.bool)
    dup[:, 1:] = sid[:, 1:] == sid[:, :-1]
    sd = torch.where(dup | (sid < 0), torch.full_like(sd, float("inf")), sd)
    tk = sd.topk(k, dim=1, largest=False)
    res = torch.gather(sid, 1, tk.indices)
    return torch.where(torch.isinf(tk.values), torch.full_like(res, -1), res)


def build_index(data: dict, threshold=2000, degree=64, n_random=40, pq_dim=48, seed=0, t0=None,
                torch_encode=False, passes=1, window=2048, float_codebook=False) -> GpuIndex:
    """passes > 1: each pass orders the label's members by coarse cluster and
    a different random projection; the window k-NN lists of all passes are
    merged (nearest distinct ids), which widens every row's candidate pool.
    float_codebook: keep the trained float centroids (the reference's
    artefacts are float pivots + mean), which the table and direct PQ modes
    score; by default they are rounded to integers for GOFANN_PQ_U8."""
    t0 = t0 or time.time()
    dev = data["base"].device
    base = data["base"]
    n, dim = base.shape
    prev_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True  # exact for uint8 inputs
    try:
        # codebook values rounded to integers in 0..255: with u8 queries every
        # table entry and ADC sum is then an exact integer (GOFANN_PQ_U8)
        cent = train_pq_gpu(base, pq_dim, seed)
        if not float_codebook:
            cent = cent.round_().clamp_(0, 255)
        codes = torch.empty((n, pq_dim), dtype=torch.uint8, device=dev)
        if torch_encode:
            w = dim // pq_dim
            c3 = cent.view(256, pq_dim, w).transpose(0, 1).contiguous()
            for s in range(0, n, 1 << 20):
                xs = base[s:s + (1 << 20)].float().view(-1, pq_dim, w).transpose(0, 1)
                codes[s:s + xs.shape[1]] = torch.cdist(xs, c3).argmin(2).transpose(0, 1).to(torch.uint8)
        else:
            L = A.lib()
            A.check(L.gofann_pq_encode(A.ptr(base), A.DTYPE_U8, n, dim, A.ptr(cent), pq_dim, A.ptr(codes),
                                       torch.cuda.current_stream().cuda_stream), "gofann_pq_encode")
        torch.cuda.synchronize()
        _log(f"PQ {pq_dim}x256 trained and encoded", t0)
        coarse = coarse_assign(base, seed=seed)
        gproj = torch.Generator(device=dev).manual_seed(seed + 11)
        vs = torch.randn((dim, passes), generator=gproj, device=dev)
        projs = torch.empty((n, passes), device=dev)
        for s0 in range(0, n, 1 << 21):
            projs[s0:s0 + (1 << 21)] = base[s0:s0 + (1 << 21)].float() @ vs
        card, begin = data["card"], data["begin"]
        high = np.nonzero(card > threshold)[0]
        total_rows = int(card[high].sum())
        adjacency = torch.full((total_rows, degree), -1, dtype=torch.int32, device=dev)
        row_to_sample = torch.empty(total_rows, dtype=torch.int32, device=dev)
        label_offset = np.zeros(len(high), np.uint32)
        seeds = np.zeros(len(high), np.uint32)
        label_group = np.full(data["vocab"], -1, np.int64)
        grand = torch.Generator(device=dev).manual_seed(seed + 13)
        n_near = degree - n_random
        row = 0
        pid = data["posting_ids"]
        for gi, lab in enumerate(high):
            m = pid[int(begin[lab]): int(begin[lab]) + int(card[lab])].to(torch.int64)
            def order_by(pi):
                pr = projs[m, pi].double()
                return torch.argsort(coarse[m].double() * 1e7 + (pr - pr.min()))
            o0 = order_by(0)
            rows = m[o0]
            nl = rows.shape[0]
            row_to_sample[row:row + nl] = rows.to(torch.int32)
            x = base[rows].float()
            if passes == 1 or nl <= window:
                nn = window_knn(x, n_near, window=window)
            else:
                inv0 = torch.empty(nl, dtype=torch.int64, device=dev)
                inv0[o0] = torch.arange(nl, device=dev)
                cand_i, cand_d = [], []
                for pi in range(passes):
                    # pass-pi order expressed as positions in the pass-0 row order
                    perm = torch.arange(nl, device=dev) if pi == 0 else inv0[order_by(pi)]
                    ii, dd = window_knn(x[perm], n_near, window=window, with_dist=True)
                    glob = torch.where(ii >= 0, perm[ii.clamp(min=0)], torch.full_like(ii, -1))
                    pass_ids = torch.full_like(glob, -1)
                    pass_d = torch.full_like(dd, float("inf"))
                    pass_ids[perm] = glob
                    pass_d[perm] = dd
                    cand_i.append(pass_ids)
                    cand_d.append(pass_d)
                nn = merge_candidates(torch.cat(cand_i, 1), torch.cat(cand_d, 1), n_near)
            adj = adjacency[row:row + nl]
            adj[:, :n_near] = nn.to(torch.int32)
            # long-range edges: distinct per row (sorted, repeats dropped), never
            # the row itself or one of its near edges
            rnd = torch.randint(0, nl, (nl, n_random), generator=grand, device=dev).sort(dim=1).values
            dup = torch.zeros_like(rnd, dtype=torch.bool)
            dup[:, 1:] = rnd[:, 1:] == rnd[:, :-1]
            dup |= (rnd.unsqueeze(2) == nn.unsqueeze(1)).any(2) | (rnd == torch.arange(nl, device=dev).unsqueeze(1))
            adj[:, n_near:] = torch.where(dup, torch.full_like(rnd, -1), rnd).to(torch.int32)
            mean = x.mean(0)
            seeds[gi] = int((x - mean).square().sum(1).argmin())
            label_offset[gi] = row
            label_group[lab] = gi
            row += nl
        torch.cuda.synchronize()
        _log(f"{len(high)} label graphs, {total_rows} rows, degree {degree}", t0)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev_tf32
    return GpuIndex(dim=dim, dtype="u8", n=n, base=base, label_indptr=data["label_indptr"],
                    label_indices=data["label_indices"], n_labels=data["vocab"], threshold=threshold, degree=degree,
                    adjacency=adjacency, row_to_sample=row_to_sample, label_offset=label_offset,
                    group_label=high.astype(np.uint32), label_group=label_group, seeds=seeds,
                    posting_ids=data["posting_ids"], posting_begin=begin.astype(np.uint64),
                    posting_count=card.astype(np.uint32), pq_centroids=cent, pq_codes=codes,
                    stats=dict(groups=len(high), graph_rows=total_rows))


def ground_truth(data: dict, q: Queries, sample: np.ndarray, k=10) -> np.ndarray:
    """Exact filtered top-k (uint8 L2 as exact integers, ties by id) for the
    queries in `sample`; [len(sample), k] ids with UINT32_MAX fill."""
    base, pid = data["base"], data["posting_ids"]
    card, begin = data["card"], data["begin"]
    dev = base.device
    n = base.shape[0]
    out = np.full((len(sample), k), A.U32MAX, np.uint32)
    mask = torch.zeros(n, dtype=torch.bool, device=dev)
    for j, qi in enumerate(sample):
        labs = q.labels[qi]
        lab = labs[np.argmin(card[labs])]
        cand = pid[int(begin[lab]): int(begin[lab]) + int(card[lab])].to(torch.int64)
        for other in labs:
            if other == lab:
                continue
            om = pid[int(begin[other]): int(begin[other]) + int(card[other])].to(torch.int64)
            mask[om] = True
            cand = cand[mask[cand]]
            mask[om] = False
        if cand.numel() == 0:
            continue
        qv = q.vectors[qi].to(torch.int32)
        best = None
        for s in range(0, cand.numel(), 1 << 21):
            c = cand[s:s + (1 << 21)]
            diff = base[c].to(torch.int32) - qv
            d = diff.square().sum(1).to(torch.int64)
            keyv = (d << 24) | c
            kk = min(k, keyv.numel())
            top = keyv.topk(kk, largest=False).values
            best = top if best is None else torch.cat([best, top]).topk(min(k, best.numel() + kk), largest=False).values
        best = torch.sort(best).values[:k]
        ids = (best & ((1 << 24) - 1)).cpu().numpy()
        out[j, :ids.shape[0]] = ids
    return out


def recall_at_k(pred: np.ndarray, gt: np.ndarray, k=10) -> float:
    """scripts/evaluate.py:163-196: mean over queries with non-empty truth of
    |truth & prediction| / |truth| on the first k slots."""
    tot, m = 0.0, 0
    for p, t in zip(pred, gt):
        ts = set(int(x) for x in t[:k] if x != A.U32MAX)
        if not ts:
            continue
        ps = set(int(x) for x in p[:k] if x != A.U32MAX)
        tot += len(ts & ps) / len(ts)
        m += 1
    return tot / m if m else float("nan")
