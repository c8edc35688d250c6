"""TEST INFRASTRUCTURE ONLY — ctypes front end of the CPU parity oracle.

Loads oracle/liboracle.so (the C restatement of the reference's search path)
and, where built, oracle/_ref/libgofann_ref.so (the reference's own headers
driven by ref_harness.cpp).  Imported only by tests/, __graft_entry__.smoke()
and bench.py's CPU legs; the product never imports this module.

All arrays are numpy (host) arrays laid out exactly as the C ABI descriptors
of include/gofann.h; the descriptor structs come from the product's ctypes
mirror so both sides read identical layouts.
"""
from __future__ import annotations

import ctypes as C
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
sys.path.insert(0, str(ROOT / "go-fann_b200"))
from gofann import _abi as A  # noqa: E402

ORACLE_LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libgofann_ref.so"

_O = None
_R = None


def build(ref_root: str = "/root/reference") -> None:
    """Runs oracle/Makefile (the _ref harness only when the reference tree exists)."""
    import subprocess
    subprocess.run(["make", "-s", "-C", str(HERE), f"REF={ref_root}"], check=True)


def olib() -> C.CDLL:
    global _O
    if _O is None:
        if not ORACLE_LIB.exists():
            build()
        L = C.CDLL(str(ORACLE_LIB))
        sp = C.c_void_p
        U32, I32 = C.c_uint32, C.c_int32
        L.oracle_warp_sum.argtypes = [sp]
        L.oracle_warp_sum.restype = C.c_float
        L.oracle_pq_build_lut.argtypes = [sp, U32, U32, sp, U32, sp]
        L.oracle_pq_adc.argtypes = [sp, U32, sp, sp, sp, U32, sp]
        L.oracle_pq_encode.argtypes = [sp, U32, U32, sp, U32, sp]
        L.oracle_rabitq_quantize.argtypes = [sp, U32, U32, sp, sp, sp]
        L.oracle_rabitq_score.argtypes = [C.POINTER(A.Codes), C.POINTER(A.Prepared), sp, sp, U32, sp, sp]
        L.oracle_rabitq_encode.argtypes = [sp, sp, U32, U32, sp, sp, sp]
        L.oracle_beam_search.argtypes = [C.POINTER(A.Graph), C.POINTER(A.Attrs), C.POINTER(A.Codes),
                                         C.POINTER(A.Prepared), C.POINTER(A.Routes), C.POINTER(A.SearchParams),
                                         sp, sp, sp, sp, C.c_int]
        L.oracle_beam_search_traced.argtypes = L.oracle_beam_search.argtypes + [sp, U32]
        L.oracle_beam_search_traced.restype = C.c_int
        L.oracle_posting_scan.argtypes = [C.POINTER(A.Codes), C.POINTER(A.Prepared), C.POINTER(A.Attrs),
                                          C.POINTER(A.Routes), C.c_int, sp, sp, sp, C.c_int, C.c_int, sp, sp]
        L.oracle_rerank.argtypes = [sp, C.c_int, U32, U32, sp, C.POINTER(A.Attrs), C.POINTER(A.Routes), sp, U32,
                                    C.c_int, sp, sp]
        L.oracle_route_merge.argtypes = [sp, sp, U32, sp, sp, U32, C.c_int, sp, sp]
        L.oracle_shard_merge.argtypes = [sp, sp, U32, U32, C.c_int, sp, sp]
        L.oracle_filtered_topk.argtypes = [sp, C.c_int, U32, U32, sp, C.POINTER(A.Attrs), C.POINTER(A.Routes),
                                           C.c_int, sp, sp]
        L.oracle_seq_smmh.argtypes = [sp, sp, sp, C.c_int, sp, sp, sp]
        L.oracle_seq_smmh.restype = C.c_int
        L.oracle_seq_result_heap.argtypes = [sp, sp, C.c_int, C.c_int, sp, sp]
        L.oracle_seq_result_heap.restype = C.c_int
        L.oracle_seq_hash.argtypes = [sp, C.c_int, sp, sp]
        L.oracle_sl_insert.argtypes = [C.c_float, U32, sp, sp, C.c_int]
        L.oracle_sl_sort.argtypes = [sp, sp, C.c_int]
        L.oracle_hash_test.argtypes = [sp, U32]
        L.oracle_pickup_index.argtypes = [sp, sp, C.c_int]
        L.oracle_rabitq_encode_f32.argtypes = [sp, sp, U32, U32, sp, sp, sp]
        L.oracle_pickup_index.restype = C.c_int
        L.oracle_pred_matches.argtypes = [C.POINTER(A.Routes), C.POINTER(A.Attrs), U32, U32]
        L.oracle_pred_enabled.argtypes = [C.POINTER(A.Routes), U32]
        L.oracle_labels_match.argtypes = [C.POINTER(A.Routes), C.POINTER(A.Attrs), U32, U32]
        L.oracle_levenshtein.argtypes = [sp, U32, sp, U32]
        L.oracle_levenshtein.restype = U32
        L.oracle_full_pickup_index.argtypes = [sp, sp, C.c_int]
        L.oracle_full_pickup_index.restype = C.c_int
        L.oracle_full_l2.argtypes = [sp, C.c_int, U32, U32, sp, U32]
        L.oracle_full_l2.restype = C.c_float
        L.oracle_exact_search.argtypes = [C.POINTER(A.Graph), sp, C.POINTER(A.Attrs), sp, C.c_int, U32, sp,
                                          C.POINTER(A.Routes), C.POINTER(A.SearchParams), sp, sp, sp, sp, U32,
                                          C.c_int]
        L.oracle_exact_posting_scan.argtypes = [sp, C.c_int, U32, sp, C.POINTER(A.Attrs), C.POINTER(A.Routes), sp,
                                                sp, sp, C.c_int, sp, sp]
        for fn in ("oracle_exact_search", "oracle_exact_posting_scan", "oracle_beam_search", "oracle_posting_scan", "oracle_rerank", "oracle_route_merge",
                   "oracle_shard_merge", "oracle_filtered_topk"):
            getattr(L, fn).restype = C.c_int
        _O = L
    return _O


def rlib() -> C.CDLL | None:
    """The reference-header harness, or None where it was not built."""
    global _R
    if _R is None and REF_LIB.exists():
        L = C.CDLL(str(REF_LIB))
        sp = C.c_void_p
        U32 = C.c_uint32
        L.ref_seq_smmh.argtypes = [sp, sp, sp, C.c_int, sp, sp, sp]
        L.ref_seq_smmh.restype = C.c_int
        L.ref_seq_result_heap.argtypes = [sp, sp, C.c_int, C.c_int, sp, sp]
        L.ref_seq_result_heap.restype = C.c_int
        L.ref_seq_hash.argtypes = [sp, C.c_int, sp, sp]
        L.ref_shortlist.argtypes = [sp, sp, C.c_int, C.c_int, C.c_int, sp, sp]
        L.ref_pred_matches.argtypes = [sp, U32, sp, sp, sp, sp, U32, sp, sp, U32, sp, sp, U32, sp]
        L.ref_priority.argtypes = [sp, sp, U32, C.c_float, sp]
        L.ref_route_merge.argtypes = [sp, U32, U32, sp, sp, U32, U32, sp, sp]
        L.ref_route_merge.restype = C.c_int
        L.ref_fp16_l2.argtypes = [sp, sp, U32, U32, sp]
        L.ref_fp16_decode.argtypes = [C.c_uint16]
        L.ref_fp16_decode.restype = C.c_float
        L.ref_graph_write.argtypes = [C.c_char_p, sp, C.c_uint64, U32, C.c_char_p, C.c_int]
        L.ref_graph_write.restype = C.c_int
        L.ref_graph_load.argtypes = [C.c_char_p, sp, C.c_uint64, sp, sp, C.c_char_p, C.c_int]
        L.ref_graph_load.restype = C.c_int
        _R = L
    return _R


P = A.ptr


def _c(x, dtype):
    return np.ascontiguousarray(x, dtype=dtype)


# ------------------------------------------------------------------ stages
def pq_build_lut(queries, centroids, pq_dim):
    q = _c(queries, np.float32)
    c = _c(centroids, np.float32)
    n, dim = q.shape
    out = np.empty((n, pq_dim, A.PQ_CENTROIDS), np.float32)
    olib().oracle_pq_build_lut(P(q), n, dim, P(c), pq_dim, P(out))
    return out


def pq_adc(lut, codes, pair_row, pair_sample):
    lut = _c(lut, np.float32)
    codes = _c(codes, np.uint8)
    r = _c(pair_row, np.uint32)
    s = _c(pair_sample, np.uint32)
    out = np.empty(r.shape[0], np.float32)
    olib().oracle_pq_adc(P(lut), codes.shape[1], P(codes), P(r), P(s), r.shape[0], P(out))
    return out


def pq_encode(vectors, centroids, pq_dim):
    v = _c(vectors, np.float32)
    c = _c(centroids, np.float32)
    out = np.empty((v.shape[0], pq_dim), np.uint8)
    olib().oracle_pq_encode(P(v), v.shape[0], v.shape[1], P(c), pq_dim, P(out))
    return out


def rabitq_quantize(rotated):
    r = _c(rotated, np.float32)
    n, pd = r.shape
    q8 = np.empty((n, pd), np.int8)
    scale = np.empty(n, np.float32)
    k1 = np.empty(n, np.float32)
    olib().oracle_rabitq_quantize(P(r), n, pd, P(q8), P(scale), P(k1))
    return q8, scale, k1


def rabitq_score(codes: dict, prep: dict, pair_row, pair_sample):
    cs, ps = A.fill_codes(codes), A.fill_prepared(prep)
    r = _c(pair_row, np.uint32)
    s = _c(pair_sample, np.uint32)
    out = np.empty(r.shape[0], np.float32)
    ip = np.empty(r.shape[0], np.int32)
    olib().oracle_rabitq_score(C.byref(cs), C.byref(ps), P(r), P(s), r.shape[0], P(out), P(ip))
    return out, ip


def rabitq_encode(residual, rotated_centroids, anchor_ids):
    r = _c(residual, np.float32)
    c = _c(rotated_centroids, np.float32)
    a = _c(anchor_ids, np.uint32)
    n, pd = r.shape
    codes = np.empty((n, pd // 8), np.uint8)
    factors = np.empty((n, 3), np.float32)
    olib().oracle_rabitq_encode(P(r), P(c), n, pd, P(a), P(codes), P(factors))
    return codes, factors


def beam_search(graph: dict, attrs: dict | None, codes: dict, prep: dict, routes: dict, threads: int = 1,
                trace_width: int = 0, **params):
    g = A.fill_graph(graph)
    at = A.fill_attrs(attrs) if attrs is not None else A.Attrs()
    cs, ps, rs = A.fill_codes(codes), A.fill_prepared(prep), A.fill_routes(routes)
    sp = A.fill_params(**params)
    n, rw = rs.n_routes, sp.result_width
    ids = np.empty((n, rw), np.uint32)
    d = np.empty((n, rw), np.float32)
    steps = np.empty(n, np.int32)
    counters = np.empty((n, 4), np.uint32)
    trace = np.empty((n, trace_width), np.uint32) if trace_width else None
    st = olib().oracle_beam_search_traced(C.byref(g), C.byref(at), C.byref(cs), C.byref(ps), C.byref(rs),
                                          C.byref(sp), P(ids), P(d), P(steps), P(counters), threads, P(trace),
                                          trace_width)
    if st != 0:
        raise RuntimeError(f"oracle_beam_search status {st}")
    if trace_width:
        return ids, d, steps, counters, trace
    return ids, d, steps, counters


def posting_scan(codes: dict, prep: dict, attrs: dict | None, routes: dict, scorer: int, posting_ids, route_begin,
                 route_count, k: int, score_first: int = 0):
    cs, ps, rs = A.fill_codes(codes), A.fill_prepared(prep), A.fill_routes(routes)
    at = A.fill_attrs(attrs) if attrs is not None else A.Attrs()
    pid = _c(posting_ids, np.uint32)
    rb = _c(route_begin, np.uint64)
    rc = _c(route_count, np.uint32)
    n = rs.n_routes
    ids = np.empty((n, k), np.uint32)
    d = np.empty((n, k), np.float32)
    st = olib().oracle_posting_scan(C.byref(cs), C.byref(ps), C.byref(at), C.byref(rs), scorer, P(pid), P(rb), P(rc),
                                    k, score_first, P(ids), P(d))
    if st != 0:
        raise RuntimeError(f"oracle_posting_scan status {st}")
    return ids, d


def rerank(base, dtype: int, queries, attrs: dict | None, routes: dict, cand, k: int):
    base = np.ascontiguousarray(base)
    queries = np.ascontiguousarray(queries)
    cand = _c(cand, np.uint32)
    rs = A.fill_routes(routes)
    at = A.fill_attrs(attrs) if attrs is not None else None
    n = rs.n_routes
    ids = np.empty((n, k), np.uint32)
    d = np.empty((n, k), np.float32)
    st = olib().oracle_rerank(P(base), dtype, base.shape[0], base.shape[1], P(queries),
                              C.byref(at) if at is not None else None, C.byref(rs), P(cand), cand.shape[1], k,
                              P(ids), P(d))
    if st != 0:
        raise RuntimeError(f"oracle_rerank status {st}")
    return ids, d


def route_merge(ids, d, qoff, qroutes, k: int):
    ids = _c(ids, np.uint32)
    d = _c(d, np.float32)
    qoff = _c(qoff, np.uint32)
    qr = _c(qroutes, np.uint32)
    nq = qoff.shape[0] - 1
    oi = np.empty((nq, k), np.uint32)
    od = np.empty((nq, k), np.float32)
    olib().oracle_route_merge(P(ids), P(d), ids.shape[1], P(qoff), P(qr), nq, k, P(oi), P(od))
    return oi, od


def shard_merge(ids, d, k: int):
    ids = _c(ids, np.uint32)
    d = _c(d, np.float32)
    s, nq, _ = ids.shape
    oi = np.empty((nq, k), np.uint32)
    od = np.empty((nq, k), np.float32)
    olib().oracle_shard_merge(P(ids), P(d), s, nq, k, P(oi), P(od))
    return oi, od


def filtered_topk(base, dtype: int, queries, attrs: dict, routes: dict, k: int):
    base = np.ascontiguousarray(base)
    queries = np.ascontiguousarray(queries)
    rs, at = A.fill_routes(routes), A.fill_attrs(attrs)
    n = rs.n_routes
    ids = np.empty((n, k), np.uint32)
    d = np.empty((n, k), np.float64)
    olib().oracle_filtered_topk(P(base), dtype, base.shape[0], base.shape[1], P(queries), C.byref(at), C.byref(rs),
                                k, P(ids), P(d))
    return ids, d


def exact_search(graph: dict, attrs: dict, base, dtype: int, queries, routes: dict, label_size=None,
                 threads: int = 1, trace_width: int = 0, **params):
    """Full-GPU exact-distance traversal (run_full_gpu_highfreq_route,
    backend_full_gpu.cu:1682-2043): per route the top-k sample ids and
    distances, step counts and (optionally) the expansion trace."""
    g, at, rs = A.fill_graph(graph), A.fill_attrs(attrs), A.fill_routes(routes)
    sp = A.fill_params(**params)
    base = np.ascontiguousarray(base)
    queries = np.ascontiguousarray(queries)
    ls = None if label_size is None else _c(label_size, np.uint32)
    n, k = rs.n_routes, sp.result_width
    ids = np.empty((n, k), np.uint32)
    d = np.empty((n, k), np.float32)
    steps = np.empty(n, np.int32)
    trace = np.empty((n, trace_width), np.uint32) if trace_width else None
    st = olib().oracle_exact_search(C.byref(g), P(ls), C.byref(at), P(base), dtype, base.shape[1], P(queries),
                                    C.byref(rs), C.byref(sp), P(ids), P(d), P(steps), P(trace), trace_width, threads)
    if st != 0:
        raise RuntimeError(f"oracle_exact_search status {st}")
    if trace_width:
        return ids, d, steps, trace
    return ids, d, steps


def exact_posting_scan(base, dtype: int, queries, attrs: dict, routes: dict, posting_ids, route_begin, route_count,
                       k: int):
    """Full-GPU exact posting scan (full_gpu_lowfreq_kernel, backend_full_gpu.cu:2124-2260)."""
    base = np.ascontiguousarray(base)
    queries = np.ascontiguousarray(queries)
    at, rs = A.fill_attrs(attrs), A.fill_routes(routes)
    pid, rb, rc = _c(posting_ids, np.uint32), _c(route_begin, np.uint64), _c(route_count, np.uint32)
    n = rs.n_routes
    ids = np.empty((n, k), np.uint32)
    d = np.empty((n, k), np.float32)
    st = olib().oracle_exact_posting_scan(P(base), dtype, base.shape[1], P(queries), C.byref(at), C.byref(rs), P(pid),
                                          P(rb), P(rc), k, P(ids), P(d))
    if st != 0:
        raise RuntimeError(f"oracle_exact_posting_scan status {st}")
    return ids, d


def full_l2(base, dtype: int, queries, pair_row, pair_sample):
    base = np.ascontiguousarray(base)
    queries = np.ascontiguousarray(queries)
    L = olib()
    return np.array([L.oracle_full_l2(P(base), dtype, base.shape[1], int(s), P(queries), int(r))
                     for r, s in zip(pair_row, pair_sample)], np.float32)


# ------------------------------------------------------ structure probes
def seq_smmh(op, key, payload, use_ref=False):
    op = _c(op, np.int32)
    key = _c(key, np.float32)
    payload = _c(payload, np.uint32)
    n = op.shape[0]
    f = np.zeros(n + 2, np.float32)
    s = np.zeros(n + 2, np.uint32)
    popped = np.full(n, A.U32MAX, np.uint32)
    L = rlib() if use_ref else olib()
    fn = L.ref_seq_smmh if use_ref else L.oracle_seq_smmh
    size = fn(P(op), P(key), P(payload), n, P(f), P(s), P(popped))
    return f[:size], s[:size], popped


def seq_result_heap(key, payload, cap, use_ref=False):
    key = _c(key, np.float32)
    payload = _c(payload, np.uint32)
    n = key.shape[0]
    f = np.zeros(cap + 2, np.float32)
    s = np.zeros(cap + 2, np.uint32)
    L = rlib() if use_ref else olib()
    fn = L.ref_seq_result_heap if use_ref else L.oracle_seq_result_heap
    size = fn(P(key), P(payload), n, cap, P(f), P(s))
    return f[:size], s[:size]


def seq_hash(values, use_ref=False):
    v = _c(values, np.uint32)
    t = np.zeros(A.HASH_CAPACITY, np.uint32)
    out = np.zeros(v.shape[0], np.int32)
    if use_ref:
        rlib().ref_seq_hash(P(v), v.shape[0], P(t), P(out))
    else:
        olib().oracle_seq_hash(P(v), v.shape[0], P(t), P(out))
    return t, out


def shortlist(dist, ids, k, sort=True, use_ref=False):
    dist = _c(dist, np.float32)
    ids = _c(ids, np.uint32)
    if use_ref:
        od = np.empty(k, np.float32)
        oi = np.empty(k, np.uint32)
        rlib().ref_shortlist(P(dist), P(ids), dist.shape[0], k, 1 if sort else 0, P(od), P(oi))
        return od, oi
    od = np.full(k, A.FLT_MAX, np.float32)
    oi = np.full(k, A.U32MAX, np.uint32)
    L = olib()
    for x, y in zip(dist.tolist(), ids.tolist()):
        L.oracle_sl_insert(C.c_float(x), y, P(od), P(oi), k)
    if sort:
        L.oracle_sl_sort(P(od), P(oi), k)
    return od, oi


def pred_matches(routes: dict, attrs: dict, pair_route, pair_sample):
    rs, at = A.fill_routes(routes), A.fill_attrs(attrs)
    L = olib()
    return np.array([L.oracle_pred_matches(C.byref(rs), C.byref(at), int(r), int(s))
                     for r, s in zip(pair_route, pair_sample)], np.uint8)


def predicate_pass_masks(graph: dict, attrs: dict, routes: dict, cand_route, cand_rows) -> np.ndarray:
    """Pass bitmap of candidate rows (prepare_candidate_pass_masks,
    src/predicates/gpu_predicate_parallel.cuh:21-42): bit i % 32 of word i / 32
    = candidate i (local row cand_rows[i] of route cand_route[i]'s graph
    group) matches the route's DNF predicate, or the route has none enabled.
    Loops in Python over oracle_pred_matches: small cases only."""
    rs, at = A.fill_routes(routes), A.fill_attrs(attrs)
    L = olib()
    cand_route = np.asarray(cand_route, np.uint32)
    cand_rows = np.asarray(cand_rows, np.uint32)
    n = cand_route.shape[0]
    bits = np.zeros(((n + 31) // 32) * 32, np.uint8)
    off, r2s, grp = graph["label_offset"], graph["row_to_sample"], routes["group_id"]
    for i, (r, row) in enumerate(zip(cand_route.tolist(), cand_rows.tolist())):
        s = int(r2s[int(off[grp[r]]) + row])
        bits[i] = L.oracle_pred_matches(C.byref(rs), C.byref(at), r, s) if L.oracle_pred_enabled(C.byref(rs), r) \
            else 1
    return np.packbits(bits.reshape(-1, 32)[:, ::-1], axis=1, bitorder="big").view(">u4").astype(np.uint32).ravel()


def rabitq_encode_f32(residual, rotated_centroids, anchor_ids):
    """The device encoder's FP32 arithmetic: codes [n][padded_dim/8] (u8,
    words little-endian) and factors [n][3]."""
    r = _c(residual, np.float32)
    c = _c(rotated_centroids, np.float32)
    a = _c(anchor_ids, np.uint32)
    n, pd = r.shape
    words = np.empty((n, pd // 32), np.uint32)
    factors = np.empty((n, 3), np.float32)
    olib().oracle_rabitq_encode_f32(P(r), P(c), n, pd, P(a), P(words), P(factors))
    return words.view(np.uint8).reshape(n, pd // 8), factors


def pickup_index(keys, vals, size: int) -> int:
    """The frontier entry the traversal's pickup takes (index, or -1)."""
    k = _c(keys, np.float32)
    v = _c(vals, np.uint32)
    return int(olib().oracle_pickup_index(P(k), P(v), int(size)))


def full_pickup_index(keys, vals, size: int) -> int:
    """The frontier entry the Full-GPU traversal's pickup takes (index, or -1)."""
    k = _c(keys, np.float32)
    v = _c(vals, np.uint32)
    return int(olib().oracle_full_pickup_index(P(k), P(v), int(size)))


def levenshtein(a: bytes, b: bytes) -> int:
    pa = np.frombuffer(a, np.uint8) if a else np.zeros(1, np.uint8)
    pb = np.frombuffer(b, np.uint8) if b else np.zeros(1, np.uint8)
    return int(olib().oracle_levenshtein(P(pa), len(a), P(pb), len(b)))


def cpu_count() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
