"""Route planning: labelled queries -> graph routes and posting routes.

Mirrors the reference's categorical routing (validate_and_prepare_queries,
src/data/dataloader.cpp:10972; routing mode greedy_min_posting,
dataloader.cpp:7833-7836) and its compiled predicate
(route_predicate::compile, src/planning/route_predicate_plan.h:175-315):
  * an AND query picks the label with the smallest posting as its route;
  * a label with a graph group becomes a graph route seeded at the group's
    seed row; otherwise the label's posting list is scanned;
  * the full conjunction is compiled as one DNF clause and enabled whenever
    it says more than the route's own label (a residual).
Route tables are returned as numpy arrays in the gofann_routes layout.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _abi as A


@dataclass
class Plan:
    graph_routes: dict           # gofann_routes arrays for the beam search
    graph_query: np.ndarray      # [n_graph_routes] original query index
    posting_routes: dict         # gofann_routes arrays for the posting scan
    posting_query: np.ndarray
    posting_begin: np.ndarray    # [n_posting_routes] u64 offsets into posting_ids
    posting_count: np.ndarray    # [n_posting_routes] u32
    n_queries: int

    @property
    def n_routes(self) -> int:
        return int(self.graph_query.shape[0] + self.posting_query.shape[0])

    def merge_tables(self):
        """CSR of routes per original query over the concatenation
        [graph routes ; posting routes] (route_to_original_query)."""
        r2q = np.concatenate([self.graph_query, self.posting_query]).astype(np.int64)
        order = np.argsort(r2q, kind="stable").astype(np.uint32)
        counts = np.bincount(r2q, minlength=self.n_queries)
        qoff = np.zeros(self.n_queries + 1, np.uint32)
        qoff[1:] = np.cumsum(counts)
        return qoff, order


def _residual_clauses(lab, primary):
    """One DNF clause per route with the query labels other than the route's
    own label, which every row of the route carries (its graph group or its
    posting list): the compiled residual of the conjunction."""
    res = [np.asarray([x for x in l if x != p], np.uint32) for l, p in zip(lab, primary)]
    n = len(res)
    rptr = np.zeros(n + 1, np.uint64)
    rptr[1:] = np.cumsum([len(x) for x in res], dtype=np.uint64)
    handles = np.concatenate(res).astype(np.uint32) if n else np.zeros(0, np.uint32)
    if handles.size == 0:  # keep a valid (unreferenced) array: empty arrays map to NULL
        handles = np.zeros(1, np.uint32)
    clauses = np.zeros(n, A.CLAUSE_DTYPE)
    clauses["label_begin"] = rptr[:-1].astype(np.uint32)
    clauses["label_end"] = rptr[1:].astype(np.uint32)
    enabled = np.array([len(x) > 0 for x in res], np.uint8)
    return clauses, handles, enabled


def _route_tables(qidx, labels_of, primary, group, start):
    n = len(qidx)
    indptr = np.zeros(n + 1, np.uint64)
    lab = [labels_of[q] for q in qidx]
    indptr[1:] = np.cumsum([len(x) for x in lab], dtype=np.uint64)
    indices = np.concatenate(lab).astype(np.uint32) if n else np.zeros(0, np.uint32)
    primary = np.asarray(primary, np.uint32)
    clauses, handles, enabled = _residual_clauses(lab, primary)
    return {
        "query_row": np.asarray(qidx, np.uint32),
        "group_id": np.asarray(group, np.uint32),
        "start_local": np.asarray(start, np.uint32),
        "qlabel_indptr": indptr,
        "qlabel_indices": indices,
        "primary_label": primary,
        "pred_offsets": np.arange(n + 1, dtype=np.uint32),
        "clauses": clauses,
        "pred_handles": handles,
        "pred_enabled": enabled,
    }


def plan_queries(index, query_labels: list) -> Plan:
    """greedy_min_posting routing of AND-of-labels queries."""
    card = index.posting_count
    g_q, g_p, g_grp, g_start = [], [], [], []
    p_q, p_p, p_b, p_c = [], [], [], []
    for qi, labs in enumerate(query_labels):
        labs = np.asarray(labs, np.uint32)
        lab = int(labs[np.argmin(card[labs])])
        grp = int(index.label_group[lab])
        if grp >= 0:
            g_q.append(qi); g_p.append(lab); g_grp.append(grp); g_start.append(int(index.seeds[grp]))
        else:
            p_q.append(qi); p_p.append(lab)
            p_b.append(int(index.posting_begin[lab])); p_c.append(int(index.posting_count[lab]))
    labels_of = [np.asarray(x, np.uint32) for x in query_labels]
    graph = _route_tables(g_q, labels_of, g_p, g_grp, g_start)
    post = _route_tables(p_q, labels_of, p_p, np.zeros(len(p_q), np.uint32), np.zeros(len(p_q), np.uint32))
    return Plan(graph, np.asarray(g_q, np.uint32), post, np.asarray(p_q, np.uint32),
                np.asarray(p_b, np.uint64), np.asarray(p_c, np.uint32), len(query_labels))


def plan_queries_native(index, query_labels) -> Plan:
    """plan_queries through the library's host planner
    (gofann_plan_categorical): the same tables, built in C++ for the whole
    batch.  query_labels: a list of label arrays, or (indptr u64, labels u32)."""
    if isinstance(query_labels, tuple):
        qptr, qlab = (np.ascontiguousarray(query_labels[0], np.uint64),
                      np.ascontiguousarray(query_labels[1], np.uint32))
    else:
        qptr = np.zeros(len(query_labels) + 1, np.uint64)
        qptr[1:] = np.cumsum([len(x) for x in query_labels])
        qlab = (np.concatenate([np.asarray(x, np.uint32) for x in query_labels]) if len(query_labels)
                else np.zeros(0, np.uint32))
    nq, nnz = qptr.shape[0] - 1, int(qptr[-1])
    card = np.ascontiguousarray(index.posting_count, np.uint32)
    group = np.ascontiguousarray(index.label_group, np.int64)
    seeds = np.ascontiguousarray(index.seeds, np.uint32)
    pbeg = np.ascontiguousarray(index.posting_begin, np.uint64)
    bufs = []
    for _ in range(2):
        b = dict(query=np.empty(nq, np.uint32), group_id=np.empty(nq, np.uint32),
                 start_local=np.empty(nq, np.uint32), primary_label=np.empty(nq, np.uint32),
                 qlabel_indptr=np.empty(nq + 1, np.uint64), qlabel_indices=np.empty(max(nnz, 1), np.uint32),
                 pred_handles=np.empty(max(nnz, 1), np.uint32), clauses=np.zeros(max(nq, 1), A.CLAUSE_DTYPE),
                 pred_enabled=np.empty(max(nq, 1), np.uint8), posting_begin=np.empty(max(nq, 1), np.uint64),
                 posting_count=np.empty(max(nq, 1), np.uint32))
        t = A.PlanTables(**{k: A.ptr(v) for k, v in b.items()})
        bufs.append((b, t))
    A.check(A.lib().gofann_plan_categorical(A.ptr(qptr), A.ptr(qlab), nq, A.ptr(card), A.ptr(group), A.ptr(seeds),
                                            A.ptr(pbeg), card.shape[0], seeds.shape[0], C.byref(bufs[0][1]),
                                            C.byref(bufs[1][1])), "gofann_plan_categorical")

    def tables(b, t):
        n, nl, nh = t.n_routes, t.n_labels, t.n_handles
        return {"query_row": b["query"][:n].copy(), "group_id": b["group_id"][:n].copy(),
                "start_local": b["start_local"][:n].copy(), "qlabel_indptr": b["qlabel_indptr"][:n + 1].copy(),
                "qlabel_indices": b["qlabel_indices"][:nl].copy(), "primary_label": b["primary_label"][:n].copy(),
                "pred_offsets": np.arange(n + 1, dtype=np.uint32), "clauses": b["clauses"][:n].copy(),
                "pred_handles": b["pred_handles"][:nh].copy() if nh else np.zeros(1, np.uint32),
                "pred_enabled": b["pred_enabled"][:n].copy()}, b["posting_begin"][:n].copy(), \
            b["posting_count"][:n].copy()

    g, _, _ = tables(*bufs[0])
    p, pb, pc = tables(*bufs[1])
    p["group_id"][:] = 0
    p["start_local"][:] = 0
    return Plan(g, g["query_row"].copy(), p, p["query_row"].copy(), pb, pc, nq)


def subset_routes(routes: dict, sel: np.ndarray) -> dict:
    """Route tables restricted to the routes `sel` (label CSR re-based)."""
    sel = np.asarray(sel, np.int64)
    out = {}
    for k in ("query_row", "group_id", "start_local", "primary_label", "pred_enabled"):
        out[k] = np.ascontiguousarray(routes[k][sel])
    ip = routes["qlabel_indptr"]
    lab = [routes["qlabel_indices"][ip[i]:ip[i + 1]] for i in sel]
    n = len(sel)
    indptr = np.zeros(n + 1, np.uint64)
    indptr[1:] = np.cumsum([len(x) for x in lab], dtype=np.uint64)
    indices = np.concatenate(lab).astype(np.uint32) if n else np.zeros(0, np.uint32)
    clauses, handles, enabled = _residual_clauses(lab, out["primary_label"])
    out.update(qlabel_indptr=indptr, qlabel_indices=indices, pred_offsets=np.arange(n + 1, dtype=np.uint32),
               clauses=clauses, pred_handles=handles, pred_enabled=enabled)
    return out


def concat_routes(a: dict, b: dict) -> dict:
    """Route tables of `a` followed by those of `b`."""
    na, nb = a["query_row"].shape[0], b["query_row"].shape[0]
    both = subset_routes(a, np.arange(na))
    sb = subset_routes(b, np.arange(nb))
    out = {}
    for k in ("query_row", "group_id", "start_local", "primary_label", "pred_enabled"):
        out[k] = np.concatenate([both[k], sb[k]])
    ip = np.concatenate([both["qlabel_indptr"], sb["qlabel_indptr"][1:] + both["qlabel_indptr"][-1]])
    ind = np.concatenate([both["qlabel_indices"], sb["qlabel_indices"]]).astype(np.uint32)
    n = na + nb
    lab = [ind[ip[i]:ip[i + 1]] for i in range(n)]
    clauses, handles, enabled = _residual_clauses(lab, out["primary_label"])
    out.update(qlabel_indptr=ip.astype(np.uint64), qlabel_indices=ind, pred_offsets=np.arange(n + 1, dtype=np.uint32),
               clauses=clauses, pred_handles=handles, pred_enabled=enabled)
    return out


def order_by_work(plan: Plan, index) -> Plan:
    """The same plan with its graph routes reordered longest-expected first.

    Persistent warps take routes in table order, so a long route taken last
    keeps its warp busy after the others have run dry.  A route's length
    grows as its predicate's pass rate falls (the stop rule counts only
    passing expansions), so routes are ordered by the pass rate estimated from
    label frequencies: the product over the residual labels of card / n, the
    labels taken as independent.  Ties go to the larger graph first.  Results
    do not depend on the order: every route writes its own output row, and
    the route -> query merge reads the plan's tables."""
    routes = plan.graph_routes
    n_routes = routes["query_row"].shape[0]
    if n_routes == 0:
        return plan
    card = np.asarray(index.posting_count, np.float64)
    n = float(max(1, getattr(index, "n", card.max())))
    ip, ind, prim = routes["qlabel_indptr"].astype(np.int64), routes["qlabel_indices"], routes["primary_label"]
    owner = np.repeat(np.arange(n_routes), np.diff(ip))
    resid = ind != prim[owner]
    logp = np.zeros(n_routes)
    np.add.at(logp, owner[resid], np.log(np.maximum(card[ind[resid]], 1e-300) / n))
    rate = np.exp(logp)
    size = card[prim]
    perm = np.lexsort((-size, rate)).astype(np.int64)
    out = subset_routes(routes, perm)
    return Plan(out, plan.graph_query[perm], plan.posting_routes, plan.posting_query, plan.posting_begin,
                plan.posting_count, plan.n_queries)
