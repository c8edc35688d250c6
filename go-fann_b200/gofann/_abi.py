"""ctypes mirror of include/gofann.h and the loader of libgofann_b200.so.

The structs here are byte-for-byte the C descriptors.  `fill_*` helpers
build them from dicts of arrays that are either numpy arrays (host pointers)
or torch tensors (device pointers when on CUDA); the caller keeps the arrays
alive for as long as the struct is used.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

PKG_ROOT = Path(__file__).resolve().parents[1]          # go-fann_b200/
LIB_PATH = PKG_ROOT / "libgofann_b200.so"

OK = 0
ERR_INVALID, ERR_CUDA, ERR_UNSUPPORTED, ERR_CAPACITY, ERR_TIMEOUT = -1, -2, -3, -4, -5
EARLY_STOP_FIXED, EARLY_STOP_OFF, EARLY_STOP_ADAPTIVE = 0, 1, 2
SCORER_PQ, SCORER_RABITQ = 0, 1
DTYPE_U8, DTYPE_F32, DTYPE_F16 = 0, 1, 2
PQ_LUT_GLOBAL, PQ_LUT_SHARED, PQ_DIRECT, PQ_U8 = 0, 1, 2, 3
TABLE_MODES = (PQ_LUT_GLOBAL, PQ_LUT_SHARED)  # modes that read a per-query table batch
GEMM_TF32, GEMM_TF32X3 = 0, 1
MAX_DEGREE, MAX_QUEUE, MAX_TOPK, MAX_RESULT_WIDTH, MAX_SHORTLIST = 64, 512, 10, 512, 400
PQ_CENTROIDS, HASH_CAPACITY = 256, 4096
U32MAX = 0xFFFFFFFF
FLT_MAX = float(np.finfo(np.float32).max)

P = C.c_void_p
U32 = C.c_uint32
I32 = C.c_int32


class Clause(C.Structure):
    _fields_ = [("label_begin", U32), ("label_end", U32), ("range_begin", U32), ("range_end", U32)]


class RangeAtom(C.Structure):
    _fields_ = [("dimension", U32), ("mode", U32), ("lower", C.c_float), ("upper", C.c_float)]


STRING_EXACT, STRING_FUZZY, FUZZY_MAX_LENGTH = 0, 1, 32
CLAUSE_EXT_DTYPE = np.dtype([("string_begin", "<u4"), ("string_end", "<u4"), ("int_begin", "<u4"),
                             ("int_end", "<u4")])
STRING_ATOM_DTYPE = np.dtype([("kind", "<u4"), ("max_edits", "<u4"), ("offset", "<u4"), ("length", "<u4")])
INT_ATOM_DTYPE = np.dtype([("dimension", "<u4"), ("mode", "<u4"), ("lower", "<i8"), ("upper", "<i8")])
CLAUSE_DTYPE = np.dtype([("label_begin", "<u4"), ("label_end", "<u4"), ("range_begin", "<u4"), ("range_end", "<u4")])
RANGE_ATOM_DTYPE = np.dtype([("dimension", "<u4"), ("mode", "<u4"), ("lower", "<f4"), ("upper", "<f4")])


class Graph(C.Structure):
    _fields_ = [("adjacency", P), ("row_to_sample", P), ("row_filter_mask", P), ("label_offset", P),
                ("total_rows", U32), ("degree", U32), ("group_count", U32), ("reserved", U32),
                ("records", P), ("record_stride", U32), ("reserved2", U32)]


class Attrs(C.Structure):
    _fields_ = [("label_indptr", P), ("label_indices", P), ("range_values", P),
                ("n_samples", U32), ("range_count", U32), ("string_offsets", P), ("string_bytes", P),
                ("int_values", P), ("int_count", U32), ("reserved", U32)]


class Codes(C.Structure):
    _fields_ = [("pq_codes", P), ("pq_dim", U32), ("n_samples", U32), ("rq_codes", P), ("rq_factors", P),
                ("rq_anchor_ids", P), ("padded_dim", U32), ("num_anchors", U32)]


class Prepared(C.Structure):
    _fields_ = [("pq_lut", P), ("rq_q8", P), ("rq_scale", P), ("rq_k1xsumq", P), ("rq_centroid_dist", P),
                ("n_rows", U32), ("reserved", U32), ("pq_query", P), ("pq_centroids", P), ("pq_query_dtype", I32),
                ("dim", U32)]


class Routes(C.Structure):
    _fields_ = [("n_routes", U32), ("range_count", U32), ("query_row", P), ("group_id", P), ("start_local", P),
                ("filter_bits", P), ("range_modes", P), ("range_lower", P), ("range_upper", P),
                ("qlabel_indptr", P), ("qlabel_indices", P), ("primary_label", P), ("pred_offsets", P),
                ("clauses", P), ("pred_handles", P), ("pred_ranges", P), ("pred_enabled", P),
                ("route_compiled", P), ("pred_ext", P), ("pred_strings", P), ("pred_string_bytes", P),
                ("pred_string_peq", P), ("pred_ints", P)]


class PlanTables(C.Structure):
    _fields_ = [(n, P) for n in ("query", "group_id", "start_local", "primary_label", "qlabel_indptr",
                                 "qlabel_indices", "pred_handles", "clauses", "pred_enabled", "posting_begin",
                                 "posting_count")] + [("n_routes", U32), ("n_labels", U32), ("n_handles", U32),
                                                      ("reserved", U32)]


class SearchParams(C.Structure):
    _fields_ = [("queue_size", I32), ("stop_width", I32), ("result_width", I32), ("finish_limit", I32),
                ("early_stop_mode", I32), ("max_steps", I32), ("scorer", I32), ("predicate_bias", I32),
                ("alpha", C.c_float), ("pending_base_stop", I32), ("full_label_check", I32),
                ("pq_mode", I32), ("resident_warps", I32)]


class Index(C.Structure):
    _fields_ = [("graph", Graph), ("attrs", Attrs), ("codes", Codes), ("pq_centroids", P), ("base", P),
                ("base_dtype", I32), ("dim", U32), ("posting_ids", P), ("rq_rotation", P), ("rq_anchors", P),
                ("rq_anchor_entry", P)]


class Batch(C.Structure):
    _fields_ = [("queries", P), ("n_queries", U32), ("reserved", U32), ("graph_routes", Routes),
                ("posting_routes", Routes), ("posting_begin", P), ("posting_count", P),
                ("query_route_offsets", P), ("query_routes", P)]


class BatchParams(C.Structure):
    _fields_ = [("search", SearchParams), ("posting_shortlist", I32), ("topk", I32), ("rq_entries", I32),
                ("reserved", I32)]


class SearchOut(C.Structure):
    _fields_ = [("ids", P), ("dists", P), ("steps", P), ("counters", P), ("status", P), ("trace", P),
                ("trace_width", U32), ("reserved", U32)]


def ptr(x) -> int | None:
    """Address of a numpy array or torch tensor (None -> NULL)."""
    if x is None:
        return None
    if isinstance(x, np.ndarray):
        if not x.flags["C_CONTIGUOUS"]:
            raise ValueError("array must be C-contiguous")
        return x.ctypes.data
    if hasattr(x, "data_ptr"):
        if not x.is_contiguous():
            raise ValueError("tensor must be contiguous")
        return x.data_ptr()
    raise TypeError(f"cannot take the address of {type(x)!r}")


def _get(d, key):
    return d.get(key) if d is not None else None


def fill_graph(g: dict) -> Graph:
    s = Graph()
    s.adjacency = ptr(g["adjacency"])
    s.row_to_sample = ptr(g["row_to_sample"])
    s.row_filter_mask = ptr(g.get("row_filter_mask"))
    s.label_offset = ptr(g["label_offset"])
    s.total_rows = int(g["adjacency"].shape[0])
    s.degree = int(g["adjacency"].shape[1])
    s.group_count = int(g["label_offset"].shape[0])
    rec = g.get("records")
    if rec is not None:
        s.records = ptr(rec)
        s.record_stride = int(rec.shape[1])
    return s


def fill_attrs(a: dict) -> Attrs:
    s = Attrs()
    s.label_indptr = ptr(a["label_indptr"])
    s.label_indices = ptr(a["label_indices"])
    s.range_values = ptr(a.get("range_values"))
    s.n_samples = int(a["label_indptr"].shape[0] - 1)
    rv = a.get("range_values")
    s.range_count = int(rv.shape[1]) if rv is not None else 0
    s.string_offsets = ptr(a.get("string_offsets"))
    s.string_bytes = ptr(a.get("string_bytes"))
    iv = a.get("int_values")
    s.int_values = ptr(iv)
    s.int_count = int(iv.shape[1]) if iv is not None else 0
    return s


def fill_codes(c: dict) -> Codes:
    s = Codes()
    if c.get("pq_codes") is not None:
        s.pq_codes = ptr(c["pq_codes"])
        s.pq_dim = int(c["pq_codes"].shape[1])
        s.n_samples = int(c["pq_codes"].shape[0])
    if c.get("rq_codes") is not None:
        s.rq_codes = ptr(c["rq_codes"])
        s.rq_factors = ptr(c["rq_factors"])
        s.rq_anchor_ids = ptr(c["rq_anchor_ids"])
        s.padded_dim = int(c["rq_codes"].shape[1] * 8)
        s.num_anchors = int(c["num_anchors"])
        s.n_samples = int(c["rq_codes"].shape[0])
    return s


def fill_prepared(p: dict) -> Prepared:
    s = Prepared()
    s.pq_lut = ptr(p.get("pq_lut"))
    s.rq_q8 = ptr(p.get("rq_q8"))
    s.rq_scale = ptr(p.get("rq_scale"))
    s.rq_k1xsumq = ptr(p.get("rq_k1xsumq"))
    s.rq_centroid_dist = ptr(p.get("rq_centroid_dist"))
    q = p.get("pq_query")
    if q is not None:
        s.pq_query = ptr(q)
        s.pq_centroids = ptr(p["pq_centroids"])
        s.dim = int(q.shape[1])
        s.pq_query_dtype = DTYPE_U8 if str(q.dtype).endswith("uint8") else DTYPE_F32
    for key in ("pq_lut", "rq_q8", "pq_query"):
        if p.get(key) is not None:
            s.n_rows = int(p[key].shape[0])
    return s


ROUTE_KEYS = ("query_row", "group_id", "start_local", "filter_bits", "range_modes", "range_lower",
              "range_upper", "qlabel_indptr", "qlabel_indices", "primary_label", "pred_offsets", "clauses",
              "pred_handles", "pred_ranges", "pred_enabled", "route_compiled", "pred_ext", "pred_strings",
              "pred_string_bytes", "pred_string_peq", "pred_ints")


def fill_routes(r: dict) -> Routes:
    s = Routes()
    s.n_routes = int(r["query_row"].shape[0])
    rm = r.get("range_modes")
    s.range_count = int(rm.shape[1]) if rm is not None and rm.ndim == 2 else 0
    for k in ROUTE_KEYS:
        setattr(s, k, ptr(r.get(k)))
    return s


def fill_params(**kw) -> SearchParams:
    s = SearchParams()
    defaults = dict(queue_size=64, stop_width=10, result_width=100, finish_limit=100,
                    early_stop_mode=EARLY_STOP_ADAPTIVE, max_steps=0, scorer=SCORER_PQ, predicate_bias=0,
                    alpha=0.15, pending_base_stop=0, full_label_check=0, pq_mode=PQ_LUT_GLOBAL,
                    resident_warps=0)
    defaults.update(kw)
    for k, v in defaults.items():
        setattr(s, k, v)
    return s


_LIB = None


def lib() -> C.CDLL:
    """Loads libgofann_b200.so (built in-tree) and declares the signatures."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is not built; run __graft_entry__.build() or `make -C go-fann_b200`")
    L = C.CDLL(str(LIB_PATH))
    sp = C.c_void_p
    L.gofann_abi_version.restype = C.c_int
    L.gofann_last_error.restype = C.c_char_p
    L.gofann_device_sm_count.restype = C.c_int
    sig = {
        "gofann_pq_build_lut": [sp, C.c_int, U32, U32, sp, U32, sp, sp],
        "gofann_pq_adc": [sp, U32, sp, sp, sp, U32, sp, sp],
        "gofann_pq_encode": [sp, C.c_int, U32, U32, sp, U32, sp, sp],
        "gofann_rabitq_quantize": [sp, U32, U32, sp, sp, sp, sp],
        "gofann_rabitq_centroid_dist": [sp, U32, sp, U32, U32, sp, sp],
        "gofann_rabitq_rotate": [sp, U32, U32, sp, U32, C.c_int, sp, sp, C.c_size_t, sp, sp],
        "gofann_rabitq_encode": [sp, sp, sp, U32, U32, sp, sp, sp],
        "gofann_rabitq_route_entries": [sp, U32, sp, U32, sp, sp, sp],
        "gofann_rabitq_centroid_dist_tc": [sp, U32, sp, U32, U32, C.c_int, sp, sp, C.c_size_t, sp, sp],
        "gofann_rabitq_score": [C.POINTER(Codes), C.POINTER(Prepared), sp, sp, U32, sp, sp, sp],
        "gofann_beam_search": [C.POINTER(Graph), C.POINTER(Attrs), C.POINTER(Codes), C.POINTER(Prepared),
                               C.POINTER(Routes), C.POINTER(SearchParams), C.POINTER(SearchOut), sp, C.c_size_t,
                               sp],
        "gofann_beam_search_noalloc": [C.POINTER(Graph), C.POINTER(Attrs), C.POINTER(Codes), C.POINTER(Prepared),
                                       C.POINTER(Routes), C.POINTER(SearchParams), C.POINTER(SearchOut), sp],
        "gofann_search_batch_scratch_bytes": [C.POINTER(Index), C.POINTER(Batch), C.POINTER(BatchParams)],
        "gofann_search_batch": [C.POINTER(Index), C.POINTER(Batch), C.POINTER(BatchParams), sp, C.c_size_t, sp, sp,
                                sp, sp],
        "gofann_segment_merge": [sp, U32, sp, sp, I32, sp, sp, sp],
        "gofann_predicate_pass_masks": [C.POINTER(Graph), C.POINTER(Attrs), C.POINTER(Routes), sp, sp, U32, sp, sp,
                                        sp],
        "gofann_posting_scan": [C.POINTER(Codes), C.POINTER(Prepared), C.POINTER(Attrs), C.POINTER(Routes),
                                C.c_int, sp, sp, sp, I32, I32, I32, sp, sp, sp, sp],
        "gofann_rerank": [sp, C.c_int, U32, U32, sp, C.POINTER(Attrs), C.POINTER(Routes), sp, U32, I32, sp, sp,
                          sp],
        "gofann_route_merge": [sp, sp, U32, sp, sp, U32, I32, sp, sp, sp],
        "gofann_shard_merge": [sp, sp, U32, U32, I32, sp, sp, sp],
        "gofann_offset_ids": [sp, C.c_size_t, U32, sp],
        "gofann_build_row_records": [C.POINTER(Graph), C.POINTER(Attrs), C.POINTER(Codes), sp, sp, sp],
        "gofann_exact_search": [C.POINTER(Graph), sp, C.POINTER(Attrs), sp, C.c_int, U32, sp, C.POINTER(Routes),
                                C.POINTER(SearchParams), C.POINTER(SearchOut), sp, C.c_size_t, sp],
        "gofann_exact_posting_scan": [sp, C.c_int, U32, U32, sp, C.POINTER(Attrs), C.POINTER(Routes), sp, sp, sp,
                                      I32, sp, sp, sp],
    }
    for name, args in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = C.c_int
    L.gofann_beam_search_scratch_bytes.argtypes = [U32]
    L.gofann_beam_search_scratch_bytes.restype = C.c_size_t
    L.gofann_rabitq_gemm_scratch_bytes.argtypes = [U32, U32, U32, C.c_int]
    L.gofann_rabitq_gemm_scratch_bytes.restype = C.c_size_t
    L.gofann_plan_categorical.argtypes = [sp, sp, U32, sp, sp, sp, sp, U32, U32, C.POINTER(PlanTables),
                                          C.POINTER(PlanTables)]
    L.gofann_plan_categorical.restype = C.c_int
    L.gofann_string_peq.argtypes = [sp, U32, sp]
    L.gofann_string_peq.restype = C.c_int
    L.gofann_exact_search_scratch_bytes.argtypes = [U32]
    L.gofann_exact_search_scratch_bytes.restype = C.c_size_t
    L.gofann_row_record_stride.argtypes = [U32]
    L.gofann_row_record_stride.restype = C.c_size_t
    L.gofann_search_batch_scratch_bytes.restype = C.c_size_t
    _LIB = L
    return L


class GofannError(RuntimeError):
    def __init__(self, status: int, where: str):
        msg = lib().gofann_last_error().decode(errors="replace")
        super().__init__(f"{where} failed with status {status}: {msg}")
        self.status = status


def check(status: int, where: str) -> None:
    if status != OK:
        raise GofannError(status, where)


EXPORTED = ("gofann_abi_version", "gofann_last_error", "gofann_device_sm_count", "gofann_pq_build_lut",
            "gofann_pq_adc", "gofann_pq_encode", "gofann_rabitq_quantize", "gofann_rabitq_centroid_dist",
            "gofann_rabitq_score", "gofann_rabitq_gemm_scratch_bytes", "gofann_rabitq_rotate",
            "gofann_rabitq_centroid_dist_tc", "gofann_rabitq_encode", "gofann_rabitq_route_entries",
            "gofann_beam_search_scratch_bytes", "gofann_beam_search",
            "gofann_beam_search_noalloc",
            "gofann_posting_scan", "gofann_segment_merge", "gofann_predicate_pass_masks", "gofann_search_batch_scratch_bytes",
            "gofann_search_batch", "gofann_rerank", "gofann_route_merge", "gofann_shard_merge",
            "gofann_row_record_stride", "gofann_build_row_records", "gofann_offset_ids",
            "gofann_exact_search_scratch_bytes", "gofann_exact_search", "gofann_exact_posting_scan",
            "gofann_string_peq", "gofann_plan_categorical")


def header_symbols(header: str | os.PathLike | None = None) -> list[str]:
    """Function names declared in include/gofann.h."""
    import re
    h = Path(header) if header else PKG_ROOT.parent / "include" / "gofann.h"
    return re.findall(r"^GOFANN_API\s+[\w\s\*]+?\b(gofann_\w+)\(", h.read_text(), flags=re.M)
