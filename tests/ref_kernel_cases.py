"""Seeded traversal cases shaped for the reference's own PQ search kernel.

The reference's device-resident PQ traversal compiles only for pq_dim 16 or
64, u8 queries of at most 192 dimensions and queue capacities 64..512
(src/search/pq/backend_pq.cu:71-75, 530-538, 2772-2799).  These cases stay
inside that envelope and are built with numpy alone (integer distances,
stable sorts, PCG64 streams), so the same seed gives the same inputs on
any machine: the reference kernel's outputs recorded on a B200
(tests/golden/make_ref_kernel_golden.py) can be replayed against the CPU
oracle here, and the GPU test rebuilds identical inputs on the box.

Per case: a Gaussian-mixture u8 base, 1-3 labels per sample from 5 labels,
one label graph per label (exact integer k-NN plus seeded long-range
edges), a PQ codebook (float, or rounded to integers for the cases that
exercise tie resolution), single-label and two-label AND queries routed to
the rarer label with the other label as a residual DNF clause.
"""
from __future__ import annotations

import functools
import hashlib

import numpy as np

U32MAX = 0xFFFFFFFF

# (name, pq_dim, dim, queue_size, predicate_bias, early_stop_mode, int_codebook, full_label_check, result_width)
CASES = [
    ("pq16_q64_bias_adaptive", 16, 128, 64, 1, 2, False, 0, 100),
    ("pq16_q128_nobias_fixed", 16, 128, 128, 0, 0, False, 1, 64),
    ("pq64_q64_bias_adaptive", 64, 128, 64, 1, 2, False, 0, 100),
    ("pq64_q256_nobias_off", 64, 128, 256, 0, 1, False, 0, 50),
    ("pq16_q64_int_bias_adaptive", 16, 128, 64, 1, 2, True, 0, 100),
    ("pq16_q128_int_nobias_adaptive", 16, 128, 128, 0, 2, True, 1, 100),
    ("pq64_q96_int_bias_fixed", 64, 128, 96, 1, 0, True, 0, 32),
    ("pq16_q512_int_bias_adaptive", 16, 128, 512, 1, 2, True, 0, 200),
]
CASE_NAMES = [c[0] for c in CASES]


def case_params(name: str) -> dict:
    c = dict(zip(("name", "pq_dim", "dim", "queue_size", "predicate_bias", "early_stop_mode", "int_codebook",
                  "full_label_check", "result_width"), next(x for x in CASES if x[0] == name)))
    return c


def _knn_graph(x: np.ndarray, members: np.ndarray, degree: int, n_random: int, rng) -> np.ndarray:
    """[len(members), degree] local rows: exact integer-L2 nearest (ties by
    row), then distinct random long-range rows; UINT32_MAX padding."""
    m = members.shape[0]
    xi = x[members].astype(np.int64)
    sq = (xi * xi).sum(1)
    d = sq[:, None] + sq[None, :] - 2 * (xi @ xi.T)
    np.fill_diagonal(d, np.iinfo(np.int64).max)
    n_near = min(degree - n_random, m - 1)
    order = np.argsort(d, axis=1, kind="stable")[:, :n_near]
    adj = np.full((m, degree), U32MAX, np.uint32)
    adj[:, :n_near] = order
    for r in range(m):
        cand = rng.permutation(m)[: n_random + n_near + 1]
        taken = set(order[r].tolist()) | {r}
        extra = [c for c in cand.tolist() if c not in taken][:n_random]
        adj[r, n_near:n_near + len(extra)] = extra
    return adj


@functools.lru_cache(maxsize=None)
def _data(seed: int, dim: int, n: int, n_labels: int, degree: int, n_random: int):
    """Base vectors, labels and per-label graphs (shared by the cases of one dim)."""
    rng = np.random.default_rng(seed + dim)
    centres = rng.normal(0, 1, size=(24, dim))
    comp = rng.integers(0, 24, size=n)
    base = np.clip(np.rint(128 + 30 * (centres[comp] + 0.6 * rng.normal(0, 1, size=(n, dim)))), 0, 255).astype(np.uint8)
    # labels: 1..3 per sample, skewed
    freq = np.array([0.45, 0.3, 0.2, 0.12, 0.08])[:n_labels]
    rows = []
    for i in range(n):
        k = 1 + int(rng.integers(0, 3))
        labs = np.unique(rng.choice(n_labels, size=k, p=freq / freq.sum()))
        rows.append(labs.astype(np.uint32))
    indptr = np.zeros(n + 1, np.uint64)
    indptr[1:] = np.cumsum([len(r) for r in rows])
    indices = np.concatenate(rows).astype(np.uint32)
    members = [np.nonzero([lab in r for r in rows])[0].astype(np.uint32) for lab in range(n_labels)]
    # per-label graphs, rows grouped by label
    adj_parts, r2s_parts, offs, seeds = [], [], [], []
    off = 0
    for lab in range(n_labels):
        mem = members[lab]
        adj_parts.append(_knn_graph(base, mem, degree, n_random, rng))
        r2s_parts.append(mem)
        offs.append(off)
        xm = base[mem].astype(np.int64)
        seeds.append(int(np.argmin(((xm - xm.mean(0)) ** 2).sum(1))))
        off += mem.shape[0]
    graph = {"adjacency": np.concatenate(adj_parts), "row_to_sample": np.concatenate(r2s_parts),
             "label_offset": np.asarray(offs, np.uint32)}
    attrs = {"label_indptr": indptr, "label_indices": indices}
    card = np.array([m.shape[0] for m in members])
    return base, centres, graph, attrs, card, np.asarray(seeds, np.uint32)


def build_case(name: str, seed: int = 11, n: int = 2400, n_labels: int = 5, n_routes: int = 64,
               degree: int = 32, n_random: int = 8):
    """Inputs of one case as numpy arrays in the gofann_* descriptor layouts."""
    from oracle import oracle as O  # the oracle's encoder (argmin, lowest centroid on ties)
    p = case_params(name)
    dim, pq_dim = p["dim"], p["pq_dim"]
    base, centres, graph, attrs, card, seeds = _data(seed, dim, n, n_labels, degree, n_random)
    rng = np.random.default_rng([seed, CASE_NAMES.index(name)])
    # codebook: 256 base rows (+ noise unless integer)
    cent = base[rng.choice(n, 256, replace=False)].astype(np.float32)
    if not p["int_codebook"]:
        cent = (cent + rng.normal(0, 3.0, size=cent.shape)).astype(np.float32)
    codes = O.pq_encode(base.astype(np.float32), cent, pq_dim)
    # queries and routes
    qc = rng.integers(0, centres.shape[0], size=n_routes)
    queries = np.clip(np.rint(128 + 30 * (centres[qc] + 0.6 * rng.normal(0, 1, size=(n_routes, dim)))), 0,
                      255).astype(np.uint8)
    qlabels = []
    for r in range(n_routes):
        a = int(rng.integers(0, n_labels))
        if rng.random() < 0.5:
            b = int(rng.integers(0, n_labels))
            qlabels.append(np.unique(np.array([a, b], np.uint32)))
        else:
            qlabels.append(np.array([a], np.uint32))
    primary = np.array([int(l[np.argmin(card[l])]) for l in qlabels], np.uint32)
    qptr = np.zeros(n_routes + 1, np.uint64)
    qptr[1:] = np.cumsum([len(l) for l in qlabels])
    qind = np.concatenate(qlabels).astype(np.uint32)
    residual = [np.array([x for x in l if x != pr], np.uint32) for l, pr in zip(qlabels, primary)]
    hptr = np.zeros(n_routes + 1, np.uint32)
    hptr[1:] = np.cumsum([len(x) for x in residual])
    handles = np.concatenate(residual + [np.zeros(1, np.uint32)]).astype(np.uint32)
    clauses = np.zeros((n_routes, 4), np.uint32)
    clauses[:, 0] = hptr[:-1]
    clauses[:, 1] = hptr[1:]
    routes = {
        "query_row": np.arange(n_routes, dtype=np.uint32),
        "group_id": primary.copy(),
        "start_local": seeds[primary].astype(np.uint32),
        "qlabel_indptr": qptr,
        "qlabel_indices": qind,
        "primary_label": primary,
        "pred_offsets": np.arange(n_routes + 1, dtype=np.uint32),
        "clauses": clauses,
        "pred_handles": handles,
        "pred_enabled": np.array([len(x) > 0 for x in residual], np.uint8),
    }
    params = dict(queue_size=p["queue_size"], predicate_bias=p["predicate_bias"],
                  early_stop_mode=p["early_stop_mode"], full_label_check=p["full_label_check"],
                  result_width=p["result_width"], finish_limit=40, stop_width=10, alpha=0.15)
    return dict(params=params, graph=graph, attrs=attrs, codes={"pq_codes": codes}, centroids=cent,
                queries=queries, routes=routes, base=base)


def case_digest(c: dict) -> str:
    """SHA-256 over every input array of a case (detects generator drift)."""
    h = hashlib.sha256()
    for grp in ("graph", "attrs", "codes", "routes"):
        for k in sorted(c[grp]):
            h.update(k.encode())
            h.update(np.ascontiguousarray(c[grp][k]).tobytes())
    for k in ("centroids", "queries"):
        h.update(np.ascontiguousarray(c[k]).tobytes())
    return h.hexdigest()
