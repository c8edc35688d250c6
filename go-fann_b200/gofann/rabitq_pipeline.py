"""Device pipeline of one RaBitQ filtered-search batch (configuration 3 shape).

Query preparation on the tensor cores (rotation q' = q . R and the centroid
distances, both FP32-accurate 3xTF32 GEMMs; int8 quantisation; each graph
route's entry row = the entry row of its query's nearest anchor), then the
1-bit RaBitQ traversal over the graph routes, RaBitQ posting scans over the
membership postings and the attribute-order slices, exact f32 rerank of
each route's shortlist and the route -> query merge -- the B200
counterpart of the reference's RaBitQ batch (init_prepared_query_state and
execute_rabitq_iteration, src/search/rabitq/backend_rabitq.cu:7800,
13762-13776).  Every computation is one of the library's kernels.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _abi as A
from . import range_postings as RP
from .engine import _t, stream_handle
from .workload_rabitq import RqIndex, RqPlan


PER_ROUTE = ("query_row", "group_id", "start_local", "filter_bits", "primary_label", "pred_enabled",
             "route_compiled")


def _segment_routes(routes: dict, sel: np.ndarray) -> dict:
    """Route tables of the segments, segment j scanning for route sel[j]:
    per-route arrays gathered; with one DNF clause per route (pred_offsets =
    0..n) the clauses and their extensions gathered as well, the atom arrays
    they index shared."""
    out = {}
    one_clause = "pred_offsets" in routes and np.array_equal(routes["pred_offsets"],
                                                             np.arange(routes["query_row"].shape[0] + 1))
    if "pred_offsets" in routes and not one_clause:
        raise ValueError("segmented scans need one predicate clause per route")
    for k, v in routes.items():
        if k in PER_ROUTE or (one_clause and k in ("clauses", "pred_ext")):
            out[k] = np.ascontiguousarray(v[sel])
        elif k == "pred_offsets":
            out[k] = np.arange(sel.shape[0] + 1, dtype=np.uint32)
        else:
            out[k] = v
    return out


class RabitqPipeline:
    def __init__(self, idx: RqIndex, plan: RqPlan, queue_size: int, shortlist: int = 200, topk: int = 10,
                 alpha: float = 0.15, entries: bool = True, segment_rows: int = 0):
        self.L = A.lib()
        d = idx.base.device
        self.idx, self.plan = idx, plan
        self.topk, self.shortlist = topk, shortlist
        self.entries = entries  # start graph routes near the query (else at the graph's seed row)
        nq, ng, npo = plan.n_queries, int(plan.graph_query.shape[0]), int(plan.posting_query.shape[0])
        self.nq, self.ng, self.npo = nq, ng, npo
        p, na = idx.padded_dim, int(idx.anchors.shape[0])
        self.graph = {"adjacency": idx.adjacency, "row_to_sample": torch.arange(idx.n, dtype=torch.int32, device=d),
                      "label_offset": torch.zeros(1, dtype=torch.int32, device=d)}
        self.attrs = {"label_indptr": idx.set_indptr, "label_indices": idx.set_indices, "range_values": idx.attr}
        self.attrs.update(idx.extra_attrs)
        self.base_dtype = A.DTYPE_F16 if idx.base.dtype == torch.float16 else A.DTYPE_F32
        self.codes = {"rq_codes": idx.codes, "rq_factors": idx.factors, "rq_anchor_ids": idx.anchor_ids,
                      "num_anchors": na}
        self.gs, self.at, self.cs = A.fill_graph(self.graph), A.fill_attrs(self.attrs), A.fill_codes(self.codes)
        self.groutes = {k: _t(v, d) for k, v in plan.graph_routes.items()}
        self.proutes = {k: _t(v, d) for k, v in plan.posting_routes.items()}
        self.grs, self.prs = A.fill_routes(self.groutes), A.fill_routes(self.proutes)
        self.p_begin, self.p_count = _t(plan.posting_begin, d), _t(plan.posting_count, d)
        # segmented scans (posting_segments::make_plan): slices longer than
        # segment_rows are scanned as near-equal segments, one block each, and
        # their shortlists merged per route
        self.seg = None
        if segment_rows and npo:
            sp = RP.make_plan(np.arange(npo), plan.posting_begin, plan.posting_count, segment_rows)
            sel = sp.query_positions.astype(np.int64)
            seg_routes = {k: _t(v, d) for k, v in _segment_routes(plan.posting_routes, sel).items()}
            nseg = int(sel.shape[0])
            self.seg = {"routes": seg_routes, "rs": A.fill_routes(seg_routes), "n": nseg,
                        "begin": _t(sp.offsets, d), "count": _t(sp.sizes.astype(np.uint32), d),
                        "indptr": _t(sp.query_indptr, d),
                        "ids": torch.empty((nseg, shortlist), dtype=torch.int32, device=d),
                        "d": torch.empty((nseg, shortlist), dtype=torch.float32, device=d)}
        r2q = np.concatenate([plan.graph_query, plan.posting_query]).astype(np.int64)
        order = np.argsort(r2q, kind="stable").astype(np.uint32)
        qoff = np.zeros(nq + 1, np.uint32)
        qoff[1:] = np.cumsum(np.bincount(r2q, minlength=nq))
        self.qoff, self.qroutes = _t(qoff, d), _t(order, d)
        # prepared state
        self.rotated = torch.empty((nq, p), dtype=torch.float32, device=d)
        self.q8 = torch.empty((nq, p), dtype=torch.int8, device=d)
        self.scale = torch.empty(nq, dtype=torch.float32, device=d)
        self.k1 = torch.empty(nq, dtype=torch.float32, device=d)
        self.gdist = torch.empty((nq, na), dtype=torch.float32, device=d)
        self.prep = {"rq_q8": self.q8, "rq_scale": self.scale, "rq_k1xsumq": self.k1,
                     "rq_centroid_dist": self.gdist}
        self.ps = A.fill_prepared(self.prep)
        nb = max(int(self.L.gofann_rabitq_gemm_scratch_bytes(nq, idx.dim, p, A.GEMM_TF32X3)),
                 int(self.L.gofann_rabitq_gemm_scratch_bytes(nq, p, na, A.GEMM_TF32X3)))
        self.gemm_scratch = torch.empty(nb, dtype=torch.uint8, device=d)
        self.status = torch.zeros(1, dtype=torch.int32, device=d)
        # outputs
        rw = shortlist
        self.g_ids = torch.empty((max(ng, 1), rw), dtype=torch.int32, device=d)
        self.g_d = torch.empty((max(ng, 1), rw), dtype=torch.float32, device=d)
        self.g_steps = torch.empty(max(ng, 1), dtype=torch.int32, device=d)
        self.g_counters = torch.zeros((max(ng, 1), 4), dtype=torch.int32, device=d)
        self.p_ids = torch.empty((max(npo, 1), rw), dtype=torch.int32, device=d)
        self.p_d = torch.empty((max(npo, 1), rw), dtype=torch.float32, device=d)
        self.r_ids = torch.empty((ng + npo + 1, topk), dtype=torch.int32, device=d)
        self.r_d = torch.empty((ng + npo + 1, topk), dtype=torch.float32, device=d)
        self.out_ids = torch.empty((nq, topk), dtype=torch.int32, device=d)
        self.out_d = torch.empty((nq, topk), dtype=torch.float32, device=d)
        self.scratch_bytes = int(self.L.gofann_beam_search_scratch_bytes(max(ng, 1)))
        self.scratch = torch.empty(self.scratch_bytes, dtype=torch.uint8, device=d)
        self.params = A.fill_params(queue_size=queue_size, stop_width=10, result_width=rw, finish_limit=100,
                                    early_stop_mode=A.EARLY_STOP_ADAPTIVE, scorer=A.SCORER_RABITQ, predicate_bias=1,
                                    alpha=alpha)
        self.out_s = A.SearchOut(ids=A.ptr(self.g_ids), dists=A.ptr(self.g_d), steps=A.ptr(self.g_steps),
                                 counters=A.ptr(self.g_counters), status=A.ptr(self.status))
        self.launches_per_run = 2 * (1 if ng else 0) + 2 * (1 if npo else 0) + 1 + (1 if self.seg else 0)

    def prepare(self, queries: torch.Tensor, stream=None):
        """Rotation, int8 quantisation and centroid distances (the reference
        runs these before its QPS window)."""
        s = stream_handle(stream)
        L, idx = self.L, self.idx
        nb = self.gemm_scratch.numel()
        A.check(L.gofann_rabitq_rotate(A.ptr(queries), self.nq, idx.dim, A.ptr(idx.rotation), idx.padded_dim,
                                       A.GEMM_TF32X3, A.ptr(self.rotated), A.ptr(self.gemm_scratch), nb,
                                       A.ptr(self.status), s), "gofann_rabitq_rotate")
        A.check(L.gofann_rabitq_quantize(A.ptr(self.rotated), self.nq, idx.padded_dim, A.ptr(self.q8),
                                         A.ptr(self.scale), A.ptr(self.k1), s), "gofann_rabitq_quantize")
        A.check(L.gofann_rabitq_centroid_dist_tc(A.ptr(self.rotated), self.nq, A.ptr(idx.anchors),
                                                 int(idx.anchors.shape[0]), idx.padded_dim, A.GEMM_TF32X3,
                                                 A.ptr(self.gdist), A.ptr(self.gemm_scratch), nb, A.ptr(self.status),
                                                 s), "gofann_rabitq_centroid_dist_tc")
        if self.ng and self.entries:
            # graph routes start at the entry row of their query's nearest anchor
            A.check(L.gofann_rabitq_route_entries(A.ptr(self.gdist), int(idx.anchors.shape[0]),
                                                  A.ptr(self.groutes["query_row"]), self.ng, A.ptr(idx.anchor_entry),
                                                  A.ptr(self.groutes["start_local"]), s),
                    "gofann_rabitq_route_entries")

    def beam_search(self, stream=None):
        if not self.ng:
            return
        A.check(self.L.gofann_beam_search(C.byref(self.gs), C.byref(self.at), C.byref(self.cs), C.byref(self.ps),
                                          C.byref(self.grs), C.byref(self.params), C.byref(self.out_s),
                                          A.ptr(self.scratch), self.scratch_bytes, stream_handle(stream)),
                "gofann_beam_search")

    def posting_scan(self, stream=None):
        if not self.npo:
            return
        if self.seg:
            g = self.seg
            A.check(self.L.gofann_posting_scan(C.byref(self.cs), C.byref(self.ps), C.byref(self.at), C.byref(g["rs"]),
                                               A.SCORER_RABITQ, A.ptr(self.idx.posting_ids), A.ptr(g["begin"]),
                                               A.ptr(g["count"]), self.shortlist, 1, A.PQ_LUT_GLOBAL, A.ptr(g["ids"]),
                                               A.ptr(g["d"]), A.ptr(self.status), stream_handle(stream)),
                    "gofann_posting_scan(segments)")
            A.check(self.L.gofann_segment_merge(A.ptr(g["indptr"]), self.npo, A.ptr(g["ids"]), A.ptr(g["d"]),
                                                self.shortlist, A.ptr(self.p_ids), A.ptr(self.p_d),
                                                stream_handle(stream)), "gofann_segment_merge")
            return
        A.check(self.L.gofann_posting_scan(C.byref(self.cs), C.byref(self.ps), C.byref(self.at), C.byref(self.prs),
                                           A.SCORER_RABITQ, A.ptr(self.idx.posting_ids), A.ptr(self.p_begin),
                                           A.ptr(self.p_count), self.shortlist, 1, A.PQ_LUT_GLOBAL, A.ptr(self.p_ids),
                                           A.ptr(self.p_d), A.ptr(self.status), stream_handle(stream)),
                "gofann_posting_scan")

    def rerank(self, queries: torch.Tensor, stream=None):
        s = stream_handle(stream)
        idx, k = self.idx, self.topk
        if self.ng:
            A.check(self.L.gofann_rerank(A.ptr(idx.base), self.base_dtype, idx.n, idx.dim, A.ptr(queries),
                                         C.byref(self.at), C.byref(self.grs), A.ptr(self.g_ids), self.shortlist, k,
                                         A.ptr(self.r_ids),
                                         A.ptr(self.r_d), s), "gofann_rerank(graph)")
        if self.npo:
            A.check(self.L.gofann_rerank(A.ptr(idx.base), self.base_dtype, idx.n, idx.dim, A.ptr(queries),
                                         C.byref(self.at), C.byref(self.prs), A.ptr(self.p_ids), self.shortlist, k,
                                         A.ptr(self.r_ids[self.ng:]), A.ptr(self.r_d[self.ng:]), s),
                    "gofann_rerank(posting)")

    def merge(self, stream=None):
        A.check(self.L.gofann_route_merge(A.ptr(self.r_ids), A.ptr(self.r_d), self.topk, A.ptr(self.qoff),
                                          A.ptr(self.qroutes), self.nq, self.topk, A.ptr(self.out_ids),
                                          A.ptr(self.out_d), stream_handle(stream)), "gofann_route_merge")

    def search(self, queries: torch.Tensor, stream=None):
        """The timed part of a batch (after prepare)."""
        self.beam_search(stream)
        self.posting_scan(stream)
        self.rerank(queries, stream)
        self.merge(stream)
        return self.out_ids, self.out_d

    def run(self, queries: torch.Tensor, stream=None):
        self.prepare(queries, stream)
        return self.search(queries, stream)
