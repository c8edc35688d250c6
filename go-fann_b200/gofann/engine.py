"""Device pipeline of one filtered search batch, driven through the C ABI.

One batch = per-query LUT build -> graph beam search over graph routes ->
posting scans over low-frequency routes -> exact rerank of every route's
shortlist -> route-to-query merge.  This is the B200 counterpart of the
reference's execute_graph_batch + run_lowfreq_pq_search_with_context +
highfreq rerank + merge_route_results_to_original
(src/search/pq/backend_pq.cu:9740-10185, 10769, 2479-2592, 13205-13226).

torch supplies device memory and the stream; every computation is one of
the library's kernels (there is no CPU or torch fallback: a missing
libgofann_b200.so raises).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _abi as A
from .planner import Plan

DTYPES = {"u8": A.DTYPE_U8, "f32": A.DTYPE_F32, "f16": A.DTYPE_F16}


def _t(a, device):
    if a is None:
        return None
    if isinstance(a, torch.Tensor):
        return a.to(device).contiguous()
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint64:
        a = a.view(np.int64)
    elif a.dtype == np.uint32:
        a = a.view(np.int32)
    elif a.dtype.fields is not None:  # clause / range-atom records
        a = a.view(np.uint8).reshape(-1)
    elif a.dtype == np.float16:
        a = a.view(np.int16)
    return torch.from_numpy(a).to(device)


def stream_handle(stream: torch.cuda.Stream | None = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


@dataclass
class SearchConfig:
    queue_size: int = 64
    stop_width: int = 10
    result_width: int = 100
    finish_limit: int = 100
    early_stop_mode: int = A.EARLY_STOP_ADAPTIVE
    max_steps: int = 0
    predicate_bias: int = 1
    alpha: float = 0.15
    pq_mode: int = A.PQ_LUT_GLOBAL
    resident_warps: int = 0
    lowfreq_shortlist: int = 100
    topk: int = 10

    def params(self, scorer=A.SCORER_PQ) -> A.SearchParams:
        return A.fill_params(queue_size=self.queue_size, stop_width=self.stop_width, result_width=self.result_width,
                             finish_limit=self.finish_limit, early_stop_mode=self.early_stop_mode,
                             max_steps=self.max_steps, scorer=scorer, predicate_bias=self.predicate_bias,
                             alpha=self.alpha, pq_mode=self.pq_mode, resident_warps=self.resident_warps)


class DeviceIndex:
    """Index arrays resident in HBM."""

    def __init__(self, index, device="cuda", row_records: bool = True):
        self.device = torch.device(device)
        d = self.device
        self.dim = index.dim
        self.dtype = index.dtype
        self.n = int(index.base.shape[0])
        self.graph = {"adjacency": _t(index.adjacency, d), "row_to_sample": _t(index.row_to_sample, d),
                      "label_offset": _t(index.label_offset, d)}
        self.attrs = {"label_indptr": _t(index.label_indptr, d), "label_indices": _t(index.label_indices, d)}
        self.codes = {"pq_codes": _t(index.pq_codes, d)}
        self.pq_dim = int(index.pq_codes.shape[1])
        self.pq_centroids = _t(index.pq_centroids, d)
        self.base = _t(index.base, d)
        self.posting_ids = _t(index.posting_ids, d)
        self.graph_s = A.fill_graph(self.graph)
        self.graph_s.degree = int(index.adjacency.shape[1])
        self.attrs_s = A.fill_attrs(self.attrs)
        self.codes_s = A.fill_codes(self.codes)
        if row_records:
            self.build_row_records()

    def build_row_records(self) -> None:
        """Per-row records (code row + sample + label-row range, one line per
        graph row) read by the traversal instead of row -> sample -> code."""
        L = A.lib()
        stride = int(L.gofann_row_record_stride(self.pq_dim))
        rows = int(self.graph_s.total_rows)
        rec = torch.empty((max(rows, 1), stride), dtype=torch.uint8, device=self.device)
        status = torch.zeros(1, dtype=torch.int32, device=self.device)
        A.check(L.gofann_build_row_records(C.byref(self.graph_s), C.byref(self.attrs_s), C.byref(self.codes_s),
                                           A.ptr(rec), A.ptr(status), stream_handle()), "gofann_build_row_records")
        if int(status.item()) != 0:
            raise A.GofannError(int(status.item()), "gofann_build_row_records (device)")
        self.graph["records"] = rec
        self.graph_s.records = A.ptr(rec)
        self.graph_s.record_stride = stride

    def hbm_bytes(self) -> int:
        ts = list(self.graph.values()) + list(self.attrs.values()) + [self.codes["pq_codes"], self.base,
                                                                      self.posting_ids]
        return int(sum(t.numel() * t.element_size() for t in ts if t is not None))


class DevicePlan:
    def __init__(self, plan: Plan, device):
        d = torch.device(device)
        self.plan = plan
        self.graph = {k: _t(v, d) for k, v in plan.graph_routes.items()}
        self.post = {k: _t(v, d) for k, v in plan.posting_routes.items()}
        self.post_begin = _t(plan.posting_begin, d)
        self.post_count = _t(plan.posting_count, d)
        qoff, order = plan.merge_tables()
        self.qoff = _t(qoff, d)
        self.qroutes = _t(order, d)
        self.graph_s = A.fill_routes(self.graph)
        self.post_s = A.fill_routes(self.post)
        self.n_graph = int(plan.graph_query.shape[0])
        self.n_post = int(plan.posting_query.shape[0])
        self.n_queries = plan.n_queries


class Pipeline:
    """Workspace + launch sequence for one batch shape."""

    def __init__(self, dindex: DeviceIndex, dplan: DevicePlan, cfg: SearchConfig):
        self.L = A.lib()
        self.di, self.dp, self.cfg = dindex, dplan, cfg
        d = dindex.device
        nq, ng, npo = dplan.n_queries, dplan.n_graph, dplan.n_post
        rw, sl, k = cfg.result_width, cfg.lowfreq_shortlist, cfg.topk
        # a per-query table batch is only materialised for the table modes
        self.lut = (torch.empty((nq, dindex.pq_dim, A.PQ_CENTROIDS), dtype=torch.float32, device=d)
                    if cfg.pq_mode in A.TABLE_MODES else None)
        self.g_ids = torch.empty((max(ng, 1), rw), dtype=torch.int32, device=d)
        self.g_d = torch.empty((max(ng, 1), rw), dtype=torch.float32, device=d)
        self.g_steps = torch.empty(max(ng, 1), dtype=torch.int32, device=d)
        self.g_counters = torch.zeros((max(ng, 1), 4), dtype=torch.int32, device=d)
        self.p_ids = torch.empty((max(npo, 1), sl), dtype=torch.int32, device=d)
        self.p_d = torch.empty((max(npo, 1), sl), dtype=torch.float32, device=d)
        self.r_ids = torch.empty((ng + npo + 1, k), dtype=torch.int32, device=d)
        self.r_d = torch.empty((ng + npo + 1, k), dtype=torch.float32, device=d)
        self.out_ids = torch.empty((nq, k), dtype=torch.int32, device=d)
        self.out_d = torch.empty((nq, k), dtype=torch.float32, device=d)
        self.status = torch.zeros(1, dtype=torch.int32, device=d)
        self.scratch_bytes = int(self.L.gofann_beam_search_scratch_bytes(max(ng, 1)))
        self.scratch = torch.empty(self.scratch_bytes, dtype=torch.uint8, device=d)
        self.prep = {"pq_lut": self.lut}
        self.prep_s = A.fill_prepared(self.prep)
        self.queries = None
        self.params = cfg.params(A.SCORER_PQ)
        self.out_s = A.SearchOut(ids=A.ptr(self.g_ids), dists=A.ptr(self.g_d), steps=A.ptr(self.g_steps),
                                 counters=A.ptr(self.g_counters), status=A.ptr(self.status))
        self.launches_per_run = ((1 if cfg.pq_mode in A.TABLE_MODES else 0) + 2 * (1 if ng else 0) +
                                 2 * (1 if npo else 0) + 1)

    # -- individual stages (device pointers, current stream) --------------
    def set_queries(self, queries: torch.Tensor):
        """Points the prepared state at this batch's query rows."""
        if queries is self.queries:
            return
        self.queries = queries
        if self.cfg.pq_mode not in A.TABLE_MODES:
            self.prep = {"pq_query": queries, "pq_centroids": self.di.pq_centroids}
        else:
            self.prep = {"pq_lut": self.lut}
        self.prep_s = A.fill_prepared(self.prep)

    def build_lut(self, queries: torch.Tensor, stream=None):
        """Table build for the table modes (a no-op in PQ_DIRECT and PQ_U8)."""
        self.set_queries(queries)
        if self.lut is None:
            return
        s = stream_handle(stream)
        dt = A.DTYPE_U8 if queries.dtype == torch.uint8 else A.DTYPE_F32
        A.check(self.L.gofann_pq_build_lut(A.ptr(queries), dt, queries.shape[0], queries.shape[1],
                                           A.ptr(self.di.pq_centroids), self.di.pq_dim, A.ptr(self.lut), s),
                "gofann_pq_build_lut")

    def beam_search(self, stream=None):
        if not self.dp.n_graph:
            return
        s = stream_handle(stream)
        A.check(self.L.gofann_beam_search(C.byref(self.di.graph_s), C.byref(self.di.attrs_s),
                                          C.byref(self.di.codes_s), C.byref(self.prep_s), C.byref(self.dp.graph_s),
                                          C.byref(self.params), C.byref(self.out_s), A.ptr(self.scratch),
                                          self.scratch_bytes, s), "gofann_beam_search")

    def posting_scan(self, stream=None):
        if not self.dp.n_post:
            return
        s = stream_handle(stream)
        A.check(self.L.gofann_posting_scan(C.byref(self.di.codes_s), C.byref(self.prep_s), C.byref(self.di.attrs_s),
                                           C.byref(self.dp.post_s), A.SCORER_PQ, A.ptr(self.di.posting_ids),
                                           A.ptr(self.dp.post_begin), A.ptr(self.dp.post_count),
                                           self.cfg.lowfreq_shortlist, 1, self.cfg.pq_mode, A.ptr(self.p_ids),
                                           A.ptr(self.p_d), A.ptr(self.status), s),
                "gofann_posting_scan")

    def rerank(self, queries: torch.Tensor, stream=None):
        s = stream_handle(stream)
        dt = DTYPES[self.di.dtype]
        k = self.cfg.topk
        ng = self.dp.n_graph
        if ng:
            A.check(self.L.gofann_rerank(A.ptr(self.di.base), dt, self.di.n, self.di.dim, A.ptr(queries),
                                         C.byref(self.di.attrs_s), C.byref(self.dp.graph_s), A.ptr(self.g_ids),
                                         self.cfg.result_width, k, A.ptr(self.r_ids), A.ptr(self.r_d), s),
                    "gofann_rerank(graph)")
        if self.dp.n_post:
            A.check(self.L.gofann_rerank(A.ptr(self.di.base), dt, self.di.n, self.di.dim, A.ptr(queries),
                                         C.byref(self.di.attrs_s), C.byref(self.dp.post_s), A.ptr(self.p_ids),
                                         self.cfg.lowfreq_shortlist, k, A.ptr(self.r_ids[ng:]), A.ptr(self.r_d[ng:]),
                                         s), "gofann_rerank(posting)")

    def merge(self, stream=None):
        s = stream_handle(stream)
        A.check(self.L.gofann_route_merge(A.ptr(self.r_ids), A.ptr(self.r_d), self.cfg.topk, A.ptr(self.dp.qoff),
                                          A.ptr(self.dp.qroutes), self.dp.n_queries, self.cfg.topk,
                                          A.ptr(self.out_ids), A.ptr(self.out_d), s), "gofann_route_merge")

    def run(self, queries: torch.Tensor, stream=None):
        """Whole batch on device; returns (ids, dists) device tensors [Q][k]."""
        self.build_lut(queries, stream)
        self.beam_search(stream)
        self.posting_scan(stream)
        self.rerank(queries, stream)
        self.merge(stream)
        return self.out_ids, self.out_d


class ExactPipeline:
    """The Full-GPU exact-distance mode for one batch shape
    (run_full_gpu_search, src/search/full_gpu/backend_full_gpu.cu:5387):
    graph routes are traversed with exact distances of the HBM-resident base
    vectors (gofann_exact_search), posting routes are scanned exactly
    (gofann_exact_posting_scan), both emit their top-k directly, and the
    routes are merged per query.  No codes, no tables, no rerank."""

    def __init__(self, dindex: DeviceIndex, dplan: DevicePlan, cfg: SearchConfig):
        self.L = A.lib()
        self.di, self.dp, self.cfg = dindex, dplan, cfg
        d = dindex.device
        nq, ng, npo, k = dplan.n_queries, dplan.n_graph, dplan.n_post, cfg.topk
        self.r_ids = torch.empty((ng + npo + 1, k), dtype=torch.int32, device=d)
        self.r_d = torch.empty((ng + npo + 1, k), dtype=torch.float32, device=d)
        self.g_steps = torch.empty(max(ng, 1), dtype=torch.int32, device=d)
        self.g_counters = torch.zeros((max(ng, 1), 4), dtype=torch.int32, device=d)
        self.out_ids = torch.empty((nq, k), dtype=torch.int32, device=d)
        self.out_d = torch.empty((nq, k), dtype=torch.float32, device=d)
        self.status = torch.zeros(1, dtype=torch.int32, device=d)
        self.scratch_bytes = int(self.L.gofann_exact_search_scratch_bytes(max(ng, 1)))
        self.scratch = torch.empty(self.scratch_bytes, dtype=torch.uint8, device=d)
        self.params = A.fill_params(queue_size=cfg.queue_size, result_width=k, finish_limit=cfg.finish_limit,
                                    early_stop_mode=cfg.early_stop_mode, max_steps=cfg.max_steps,
                                    resident_warps=cfg.resident_warps)
        self.out_s = A.SearchOut(ids=A.ptr(self.r_ids), dists=A.ptr(self.r_d), steps=A.ptr(self.g_steps),
                                 counters=A.ptr(self.g_counters), status=A.ptr(self.status))
        self.launches_per_run = (1 if ng else 0) + (1 if npo else 0) + 1

    def beam_search(self, queries: torch.Tensor, stream=None):
        if not self.dp.n_graph:
            return
        A.check(self.L.gofann_exact_search(C.byref(self.di.graph_s), None, C.byref(self.di.attrs_s),
                                           A.ptr(self.di.base), DTYPES[self.di.dtype], self.di.dim, A.ptr(queries),
                                           C.byref(self.dp.graph_s), C.byref(self.params), C.byref(self.out_s),
                                           A.ptr(self.scratch), self.scratch_bytes, stream_handle(stream)),
                "gofann_exact_search")

    def posting_scan(self, queries: torch.Tensor, stream=None):
        if not self.dp.n_post:
            return
        ng = self.dp.n_graph
        A.check(self.L.gofann_exact_posting_scan(A.ptr(self.di.base), DTYPES[self.di.dtype], self.di.n, self.di.dim,
                                                 A.ptr(queries), C.byref(self.di.attrs_s), C.byref(self.dp.post_s),
                                                 A.ptr(self.di.posting_ids), A.ptr(self.dp.post_begin),
                                                 A.ptr(self.dp.post_count), self.cfg.topk, A.ptr(self.r_ids[ng:]),
                                                 A.ptr(self.r_d[ng:]), stream_handle(stream)),
                "gofann_exact_posting_scan")

    def merge(self, stream=None):
        k = self.cfg.topk
        A.check(self.L.gofann_route_merge(A.ptr(self.r_ids), A.ptr(self.r_d), k, A.ptr(self.dp.qoff),
                                          A.ptr(self.dp.qroutes), self.dp.n_queries, k, A.ptr(self.out_ids),
                                          A.ptr(self.out_d), stream_handle(stream)), "gofann_route_merge")

    def run(self, queries: torch.Tensor, stream=None):
        """Whole batch on device; returns (ids, dists) device tensors [Q][k]."""
        self.beam_search(queries, stream)
        self.posting_scan(queries, stream)
        self.merge(stream)
        return self.out_ids, self.out_d


def to_numpy_ids(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy().view(np.uint32)
