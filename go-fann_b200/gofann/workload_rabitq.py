"""BASELINE configuration 3 built on the GPU: a 1-bit RaBitQ workload.

Stand-in for the reference's arxiv workloads (2.7M x 4096 f32 embeddings,
RaBitQ-1bit, range and set-membership filters; the dataset is not available
offline):

  * base: n x 4096 f32 from a 4,096-centre Gaussian mixture (centres N(0,1);
    each component's covariance is spread^2 = 16 on a rank-32 subspace --
    one of 64 random orthonormal bases -- plus 0.01 I), every vector
    L2-normalised; kept as the f32 rerank store (44 GB at n = 2.7M).  The
    low-rank components give neighbourhoods structure, as embeddings have:
    with isotropic 4096-d components the members of a component are nearly
    equidistant and recall@10 is decided by noise;
  * attributes: one numeric value uniform in [0, 1e9) (float32, the
    reference's range semantics, range_filter.cuh:28-45) and one set of 1..8
    values from a 10k vocabulary (uniform);
  * queries: mixture samples, half with a range predicate of selectivity
    0.001 / 0.01 / 0.1 / 0.5, half with a membership predicate (one value
    held by some base vector);
  * index: random orthogonal rotation R (4096 x 4096), anchors = the
    normalised mixture centres (the reference trains them with cuVS
    balanced k-means), nearest-anchor assignment, residuals r = (x - c) R
    on the tensor cores (gofann_rabitq_rotate, one TF32 pass: index time),
    codes and factors by gofann_rabitq_encode; a global graph of degree 32
    (window k-NN along a coarse-cluster + projection order for 24 near edges;
    8 long-range edges, 6 into members of the 16 components nearest to the
    row's own and 2 uniformly random, so that greedy routing can move from
    component to component); postings per membership value; the base ids
    ordered by the numeric attribute (the reference's ordered range
    postings, range_posting_index.h:12-104);
  * routing (the reference's categorical / range access split,
    dataloader.cpp:11862 plan_graph_range_access): a membership query scans
    its value's posting; a range query whose rows are at most
    `range_scan_rows` scans its slice of the attribute order, a wider one
    runs the graph traversal with the range as a DNF atom;
  * ground truth: exact filtered top-10 (FP32 GEMM over the candidates).
"""
from __future__ import annotations

import ctypes as C
import os
import tempfile
import time
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _abi as A
from . import range_postings as RP

SELECTIVITIES = (0.001, 0.01, 0.1, 0.5)
RANGE_MAX = 1e9


def _log(msg: str, t0: float) -> None:
    print(f"[config3 {time.time() - t0:7.1f}s] {msg}", flush=True)


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


@dataclass
class RqQueries:
    vectors: torch.Tensor        # [q, dim] f32 (device)
    kind: np.ndarray             # [q] 0 = membership, 1 = range
    value: np.ndarray            # [q] membership value (kind 0)
    lower: np.ndarray            # [q] f32 range bounds (kind 1): lower <= v < upper
    upper: np.ndarray
    selectivity: np.ndarray      # [q] target selectivity (range) or posting fraction


@dataclass
class RqIndex:
    n: int
    dim: int
    padded_dim: int
    base: torch.Tensor           # [n, dim] f32
    attr: torch.Tensor           # [n, 1] f32 numeric attribute
    set_indptr: torch.Tensor     # [n+1] i64
    set_indices: torch.Tensor    # [nnz] i32
    rotation: torch.Tensor       # [dim, padded_dim] f32
    anchors: torch.Tensor        # [A, padded_dim] f32 (rotated)
    codes: torch.Tensor          # [n, padded_dim/8] u8
    factors: torch.Tensor        # [n, 3] f32
    anchor_ids: torch.Tensor     # [n] i32
    adjacency: torch.Tensor      # [n, degree] i32
    seed: int
    anchor_entry: torch.Tensor   # [A] i32: the member of each anchor's cluster nearest to it (seed if empty)
    posting_ids: torch.Tensor    # [nnz + n] i32: membership postings, then the attribute order
    posting_begin: np.ndarray    # [vocab] u64 (membership)
    posting_count: np.ndarray    # [vocab] u32
    order_base: int              # offset of the attribute order in posting_ids
    range_index: object          # the FARPIDX1 range postings (range_postings.Index)
    stats: dict = field(default_factory=dict)
    extra_attrs: dict = field(default_factory=dict)  # further gofann_attrs arrays (strings, int64 values)


def _mixture(g, centres, bases, comp, spread, noise):
    """Samples of components `comp`: centre + spread * (a rank-r orthonormal
    basis shared by every 64th component) . z + isotropic noise."""
    n, dim = comp.shape[0], centres.shape[1]
    r = bases.shape[2]
    x = centres[comp] + noise * torch.randn((n, dim), generator=g, device=centres.device)
    z = torch.randn((n, r), generator=g, device=centres.device)
    grp = comp % bases.shape[0]
    for b in range(bases.shape[0]):
        rows = torch.nonzero(grp == b).squeeze(1)
        if rows.numel():
            x[rows] += spread * (z[rows] @ bases[b].T)
    return x


def generate(device="cuda", seed=0, n=2_700_000, dim=4096, n_centres=4096, rank=32, spread=4.0, noise=0.1,
             vocab=10_000, max_vals=8, n_queries=10_000, t0=None):
    t0 = t0 or time.time()
    g = torch.Generator(device=device).manual_seed(seed)
    centres = torch.randn((n_centres, dim), generator=g, device=device)
    # component covariance: spread^2 on a rank-`rank` subspace plus noise^2 I
    # (an isotropic 4096-d component leaves its members almost equidistant)
    bases = torch.linalg.qr(torch.randn((64, dim, rank), generator=g, device=device))[0].contiguous()
    base = torch.empty((n, dim), dtype=torch.float32, device=device)
    comp_all = torch.empty(n, dtype=torch.int64, device=device)
    chunk = 1 << 17
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        comp = torch.randint(0, n_centres, (e - s,), generator=g, device=device)
        base[s:e] = torch.nn.functional.normalize(_mixture(g, centres, bases, comp, spread, noise), dim=1)
        comp_all[s:e] = comp
    _log(f"base {n} x {dim} f32 ({base.numel() * 4 / 1e9:.1f} GB)", t0)
    attr = (torch.rand((n, 1), generator=g, device=device, dtype=torch.float64) * RANGE_MAX).to(torch.float32)
    # membership sets: 1..8 distinct values per row
    per = torch.randint(1, max_vals + 1, (n,), generator=g, device=device)
    rows = torch.repeat_interleave(torch.arange(n, device=device, dtype=torch.int64), per)
    vals = torch.randint(0, vocab, (rows.numel(),), generator=g, device=device)
    key = torch.unique((rows << 14) | vals)
    rows_u, vals_u = key >> 14, (key & ((1 << 14) - 1)).to(torch.int32)
    indptr = torch.zeros(n + 1, dtype=torch.int64, device=device)
    indptr[1:] = torch.cumsum(torch.bincount(rows_u, minlength=n), 0)
    key2 = torch.sort((vals_u.to(torch.int64) << 32) | rows_u).values
    postings = (key2 & 0xffffffff).to(torch.int32)
    card = torch.bincount(vals_u, minlength=vocab).cpu().numpy().astype(np.int64)
    begin = np.zeros(vocab, np.int64)
    begin[1:] = np.cumsum(card)[:-1]
    _log(f"{int(vals_u.numel())} memberships over {vocab} values (mean card {card.mean():.0f})", t0)
    # queries
    qc = torch.randint(0, n_centres, (n_queries,), generator=g, device=device)
    qv = torch.nn.functional.normalize(_mixture(g, centres, bases, qc, spread, noise), dim=1)
    rng = np.random.default_rng(seed + 17)
    kind = (rng.random(n_queries) < 0.5).astype(np.int32)  # 1 = range
    sel = np.asarray(SELECTIVITIES)[rng.integers(0, len(SELECTIVITIES), n_queries)]
    lower = (rng.random(n_queries) * (1.0 - sel) * RANGE_MAX).astype(np.float32)
    upper = (lower.astype(np.float64) + sel * RANGE_MAX).astype(np.float32)
    host_row = rng.integers(0, n, n_queries)
    ip = indptr.cpu().numpy()
    pick = ip[host_row] + (rng.random(n_queries) * (ip[host_row + 1] - ip[host_row])).astype(np.int64)
    value = vals_u[torch.from_numpy(pick).to(device)].cpu().numpy().astype(np.int64)
    msel = card[value] / n
    q = RqQueries(qv, kind, value, lower, upper, np.where(kind == 1, sel, msel))
    _log(f"{n_queries} queries ({int(kind.sum())} range, {int((kind == 0).sum())} membership)", t0)
    return dict(base=base, comp=comp_all, centres=centres, attr=attr, set_indptr=indptr, set_indices=vals_u,
                postings=postings, card=card, begin=begin, queries=q, vocab=vocab, n=n, dim=dim)


def random_rotation(p: int, seed: int, device) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed + 7)
    m = torch.randn((p, p), generator=g, device=device, dtype=torch.float64)
    q, r = torch.linalg.qr(m)
    q = q * torch.sign(torch.diagonal(r)).unsqueeze(0)
    return q.to(torch.float32).contiguous()


def rotate(x: torch.Tensor, rot: torch.Tensor, precision: int) -> torch.Tensor:
    """x [m, dim] . rot [dim, p] on the tensor cores (library GEMM)."""
    L = A.lib()
    m, d = x.shape
    p = rot.shape[1]
    out = torch.empty((m, p), dtype=torch.float32, device=x.device)
    nb = int(L.gofann_rabitq_gemm_scratch_bytes(m, d, p, precision))
    scratch = torch.empty(max(nb, 256), dtype=torch.uint8, device=x.device)
    status = torch.zeros(1, dtype=torch.int32, device=x.device)
    A.check(L.gofann_rabitq_rotate(A.ptr(x), m, d, A.ptr(rot), p, precision, A.ptr(out), A.ptr(scratch), nb,
                                   A.ptr(status), _stream()), "gofann_rabitq_rotate")
    if int(status.item()) != 0:
        raise A.GofannError(int(status.item()), "gofann_rabitq_rotate (device)")
    return out


def _window_knn(base: torch.Tensor, order: torch.Tensor, k: int, tile=1024, window=2048) -> torch.Tensor:
    """[n, k] approximate nearest neighbours (as positions in `order`) of the
    rows base[order], from exact distances inside a sliding window of the
    order (rows gathered per window, no full reordered copy)."""
    n = order.shape[0]
    dev = base.device
    out = torch.full((n, k), -1, dtype=torch.int64, device=dev)
    half = (window - tile) // 2
    for q0 in range(0, n, tile):
        q1 = min(n, q0 + tile)
        w0, w1 = max(0, q0 - half), min(n, q1 + half)
        xw = base[order[w0:w1]].float()
        sq = xw.square().sum(1)
        xq, sqq = xw[q0 - w0:q1 - w0], sq[q0 - w0:q1 - w0]
        d = sqq[:, None] + sq[None, :] - 2.0 * (xq @ xw.T)
        ar = torch.arange(q1 - q0, device=dev)
        d[ar, ar + (q0 - w0)] = float("inf")
        kk = min(k, w1 - w0 - 1)
        out[q0:q1, :kk] = d.topk(kk, dim=1, largest=False).indices + w0
    return out


def build_index(data: dict, degree=32, n_random=8, seed=0, t0=None, chunk=1 << 18, normalize_anchors=True,
                range_postings=True) -> RqIndex:
    """RaBitQ index of data["base"] (f32, or f16 read in f32 chunks): anchors
    = the mixture centres (normalised when the base is), codes, factors,
    graph, membership postings and (range_postings) the FARPIDX1 order of the
    float attribute."""
    t0 = t0 or time.time()
    base = data["base"]
    n, dim = base.shape
    dev = base.device
    p = ((dim + 63) // 64) * 64
    rot = random_rotation(p, seed, dev)[:dim].contiguous()  # [dim][p]
    anchors = torch.nn.functional.normalize(data["centres"], dim=1) if normalize_anchors else data["centres"]
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        # nearest anchor (an orthogonal rotation keeps distances)
        an = anchors.square().sum(1)
        aid = torch.empty(n, dtype=torch.int64, device=dev)
        for s in range(0, n, chunk):
            aid[s:s + chunk] = (an - 2.0 * base[s:s + chunk].float() @ anchors.T).argmin(1)
        ranchors = rotate(anchors, rot, A.GEMM_TF32X3)
        codes = torch.empty((n, p // 8), dtype=torch.uint8, device=dev)
        factors = torch.empty((n, 3), dtype=torch.float32, device=dev)
        L = A.lib()
        aid32 = aid.to(torch.int32)
        for s in range(0, n, chunk):
            e = min(n, s + chunk)
            res = rotate(base[s:e].float().contiguous(), rot, A.GEMM_TF32)
            res -= ranchors[aid[s:e]]
            A.check(L.gofann_rabitq_encode(A.ptr(res), A.ptr(ranchors), A.ptr(aid32[s:e]), e - s, p,
                                           A.ptr(codes[s:e]), A.ptr(factors[s:e]), _stream()), "gofann_rabitq_encode")
            del res
        torch.cuda.synchronize()
        _log(f"rotation, anchors ({anchors.shape[0]}), RaBitQ 1-bit codes ({p // 8} B) and factors", t0)
        # global graph: order by anchor then a random projection, window k-NN
        gp = torch.Generator(device=dev).manual_seed(seed + 11)
        rvec = torch.randn((dim, 1), generator=gp, device=dev)
        proj = torch.cat([base[s0:s0 + chunk].float() @ rvec for s0 in range(0, n, chunk)])
        pr = proj.squeeze(1).double()
        order = torch.argsort(aid.double() * 1e3 + (pr - pr.min()))
        inv = torch.empty_like(order)
        inv[order] = torch.arange(n, device=dev)
        n_near = degree - n_random
        nn = _window_knn(base, order, n_near)
        near = torch.where(nn >= 0, order[nn.clamp(min=0)], torch.full_like(nn, -1))
        adj = torch.full((n, degree), -1, dtype=torch.int32, device=dev)
        adj[order, :n_near] = near.to(torch.int32)  # row i = vector i
        # long-range edges: most into members of the 16 components nearest to
        # the row's own (the anchors' k-NN), so that greedy routing moves
        # between neighbouring components, two uniformly random
        na = anchors.shape[0]
        ad = an[:, None] + an[None, :] - 2.0 * anchors @ anchors.T
        ad.fill_diagonal_(float("inf"))
        near_c = ad.topk(16, dim=1, largest=False).indices           # [A, 16]
        by_anchor = torch.argsort(aid)                               # rows grouped by anchor
        cnt = torch.bincount(aid, minlength=na)
        start = torch.cumsum(cnt, 0) - cnt
        n_local = n_random - 2
        pick = near_c[aid][torch.arange(n, device=dev)[:, None],
                           torch.randint(0, 16, (n, n_local), generator=gp, device=dev)]  # [n, n_local] components
        pos = start[pick] + (torch.rand((n, n_local), generator=gp, device=dev) * cnt[pick]).long()
        local = torch.where(cnt[pick] > 0, by_anchor[pos.clamp(max=n - 1)], torch.zeros_like(pos))
        far = torch.randint(0, n, (n, 2), generator=gp, device=dev)
        rnd = torch.cat([local, far], 1).sort(dim=1).values
        dup = torch.zeros_like(rnd, dtype=torch.bool)
        dup[:, 1:] = rnd[:, 1:] == rnd[:, :-1]
        dup |= (rnd.unsqueeze(2) == adj[:, :n_near].to(torch.int64).unsqueeze(1)).any(2)
        dup |= rnd == torch.arange(n, device=dev).unsqueeze(1)
        adj[:, n_near:] = torch.where(dup, torch.full_like(rnd, -1), rnd).to(torch.int32)
        mean = base.mean(0, dtype=torch.float32)
        dm = torch.cat([(base[s0:s0 + chunk].float() - mean).square().sum(1) for s0 in range(0, n, chunk)])
        seed_row = int(dm.argmin())
        del dm
        # entry row per anchor: its nearest member
        dist_a = torch.empty(n, device=dev)
        for s0 in range(0, n, chunk):
            x = base[s0:s0 + chunk].float()
            dist_a[s0:s0 + chunk] = (x - anchors[aid[s0:s0 + chunk]]).square().sum(1)
        key = aid.double() * 1e6 + dist_a.double()
        first = torch.argsort(key)[start[cnt > 0]] if bool((cnt > 0).any()) else torch.zeros(0, dtype=torch.int64)
        anchor_entry = torch.full((na,), seed_row, dtype=torch.int64, device=dev)
        anchor_entry[torch.nonzero(cnt > 0).squeeze(1)] = first
        anchor_entry = anchor_entry.to(torch.int32)
        torch.cuda.synchronize()
        _log(f"global graph {n} rows, degree {degree}", t0)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    # ordered range postings: written as a FARPIDX1 file and loaded back the
    # way the reference maps its ordered_postings.bin
    attr = data.get("attr")
    rindex = None
    posting_ids = data["postings"]
    if range_postings:
        rdir = tempfile.mkdtemp(prefix="gofann_rp_")
        rpath = os.path.join(rdir, "ordered_postings.bin")
        RP.write(rpath, attr.cpu().numpy())
        rindex = RP.load(rpath)
        order_attr = torch.from_numpy(rindex.dimensions[0].sample_ids.astype(np.int64)).to(dev)
        posting_ids = torch.cat([data["postings"], order_attr.to(torch.int32)])
        _log(f"range postings {rpath}: {rindex.dimensions[0].unique_values.shape[0]} distinct values", t0)
    return RqIndex(n=n, dim=dim, padded_dim=p, base=base, attr=attr, set_indptr=data["set_indptr"],
                   set_indices=data["set_indices"], rotation=rot, anchors=ranchors, codes=codes, factors=factors,
                   anchor_ids=aid32, adjacency=adj, seed=seed_row, anchor_entry=anchor_entry, posting_ids=posting_ids,
                   posting_begin=data["begin"].astype(np.uint64), posting_count=data["card"].astype(np.uint32),
                   order_base=int(data["postings"].numel()), range_index=rindex,
                   stats=dict(graph_rows=n, anchors=int(anchors.shape[0])))


@dataclass
class RqPlan:
    graph_routes: dict
    graph_query: np.ndarray
    posting_routes: dict
    posting_query: np.ndarray
    posting_begin: np.ndarray
    posting_count: np.ndarray
    n_queries: int


def _routes(qidx, n_range_atoms, lower=None, upper=None, start=0):
    n = len(qidx)
    r = {"query_row": np.asarray(qidx, np.uint32), "group_id": np.zeros(n, np.uint32),
         "start_local": np.full(n, start, np.uint32)}
    if n_range_atoms:
        clauses = np.zeros(n, A.CLAUSE_DTYPE)
        clauses["range_begin"] = np.arange(n, dtype=np.uint32)
        clauses["range_end"] = np.arange(1, n + 1, dtype=np.uint32)
        atoms = np.zeros(n, A.RANGE_ATOM_DTYPE)
        atoms["dimension"], atoms["mode"] = 0, 3
        atoms["lower"], atoms["upper"] = lower, upper
        r.update(pred_offsets=np.arange(n + 1, dtype=np.uint32), clauses=clauses,
                 pred_handles=np.zeros(1, np.uint32), pred_ranges=atoms, pred_enabled=np.ones(n, np.uint8))
    return r


def plan_queries(idx: RqIndex, q: RqQueries, range_scan_rows=30_000) -> RqPlan:
    """Membership -> posting scan; range -> slice scan of the attribute order
    when it holds at most range_scan_rows rows, else graph traversal with the
    range as a DNF atom."""
    nq = q.kind.shape[0]
    modes = np.where(q.kind == 1, 3, 0).astype(np.uint8).reshape(nq, 1)
    sl = RP.choose_smallest_slice(idx.range_index, modes, q.lower.reshape(nq, 1), q.upper.reshape(nq, 1))
    g_q, p_q, p_b, p_c = [], [], [], []
    for i in range(nq):
        if q.kind[i] == 0:
            p_q.append(i); p_b.append(int(idx.posting_begin[q.value[i]])); p_c.append(int(idx.posting_count[q.value[i]]))
        elif sl.count[i] <= range_scan_rows:  # RP.eligible_for_scan
            p_q.append(i); p_b.append(idx.order_base + int(sl.begin[i])); p_c.append(int(sl.count[i]))
        else:
            g_q.append(i)
    g_q = np.asarray(g_q, np.int64)
    graph = _routes(g_q, 1, q.lower[g_q], q.upper[g_q], start=idx.seed)
    post = _routes(p_q, 0)
    return RqPlan(graph, g_q.astype(np.uint32), post, np.asarray(p_q, np.uint32), np.asarray(p_b, np.uint64),
                  np.asarray(p_c, np.uint32), int(q.kind.shape[0]))


def ground_truth(idx: RqIndex, data: dict, q: RqQueries, sample: np.ndarray, k=10, chunk=1 << 19) -> np.ndarray:
    """Exact filtered top-k (FP32 distances, ties by id) for the queries in
    `sample`: [len(sample), k] ids, UINT32_MAX fill."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        base = idx.base
        n = base.shape[0]
        out = np.full((len(sample), k), A.U32MAX, np.uint32)
        qv = q.vectors[torch.from_numpy(np.asarray(sample)).to(base.device)]
        bn = None
        # range queries: all at once, chunk by chunk over the base
        rs = np.nonzero(q.kind[sample] == 1)[0]
        if rs.size:
            lo = torch.from_numpy(q.lower[sample][rs]).to(base.device)
            hi = torch.from_numpy(q.upper[sample][rs]).to(base.device)
            best_d = torch.full((rs.size, k), float("inf"), device=base.device)
            best_i = torch.full((rs.size, k), -1, dtype=torch.int64, device=base.device)
            qq = qv[torch.from_numpy(rs).to(base.device)]
            qn = qq.square().sum(1, keepdim=True)
            for s in range(0, n, chunk):
                b = base[s:s + chunk]
                d = qn + b.square().sum(1)[None, :] - 2.0 * qq @ b.T
                v = idx.attr[s:s + chunk, 0][None, :]
                d = torch.where((v >= lo[:, None]) & (v < hi[:, None]), d, torch.full_like(d, float("inf")))
                kk = min(k, d.shape[1])
                tk = d.topk(kk, dim=1, largest=False)
                cd = torch.cat([best_d, tk.values], 1)
                ci = torch.cat([best_i, tk.indices + s], 1)
                o = cd.topk(k, dim=1, largest=False)
                best_d, best_i = o.values, torch.gather(ci, 1, o.indices)
            bi = best_i.cpu().numpy()
            bd = best_d.cpu().numpy()
            for j, r in enumerate(rs):
                ok = np.isfinite(bd[j])
                ids = bi[j][ok]
                dd = bd[j][ok]
                o = np.lexsort((ids, dd))
                out[r, :len(o)] = ids[o]
        ms = np.nonzero(q.kind[sample] == 0)[0]
        for r in ms:
            v = q.value[sample[r]]
            b0, c0 = int(idx.posting_begin[v]), int(idx.posting_count[v])
            cand = idx.posting_ids[b0:b0 + c0].to(torch.int64)
            x = qv[r]
            d = (base[cand] - x).square().sum(1)
            kk = min(k, cand.numel())
            tk = d.topk(kk, largest=False)
            ids = cand[tk.indices].cpu().numpy()
            dd = tk.values.cpu().numpy()
            o = np.lexsort((ids, dd))
            out[r, :kk] = ids[o]
        return out
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
