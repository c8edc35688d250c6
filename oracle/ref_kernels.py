"""TEST INFRASTRUCTURE ONLY — ctypes front end of oracle/_ref/libgofann_ref_kernels.so.

That library is the reference's own PQ search backend (putatio13/GO-FANN
src/search/pq/backend_pq.cu) compiled in place for sm_100a by
oracle/Makefile (`make refkernels`), with oracle/ref_kernels.cu launching its
device-resident traversal kernel.  `run_reference_pq` runs one seeded case
(tests/ref_kernel_cases.py layout) on the current CUDA device and returns
the reference's ids, distances, step counts, expansion trace and the PQ
table its kernel built.  Imported only by tests and the golden-vector
generator; the product never loads it.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_ref" / "libgofann_ref_kernels.so"
U32MAX = 0xFFFFFFFF

_P = C.c_void_p
_U32, _I32 = C.c_uint32, C.c_int32


class RefPqArgs(C.Structure):
    """Byte-for-byte gofann_ref_pq_args of oracle/ref_kernels.cu."""
    _fields_ = [(n, _P) for n in (
        "codes", "centroids", "queries", "adjacency", "row_to_sample", "label_offset", "zero_groups",
        "data_indptr", "data_indptr32", "data_indices", "group_id", "start_local", "filter_bits",
        "qlabel_indptr", "qlabel_indices", "primary_label", "pred_offsets", "clauses", "pred_handles",
        "pred_enabled", "out_ids", "out_dists", "pq_table", "hash", "time_per_block", "datadist", "trace_rows",
        "trace_slots", "trace_counters")] + \
        [(n, _U32) for n in ("trace_width", "n_samples", "dim", "pq_dim", "degree", "n_routes")] + \
        [(n, _I32) for n in ("queue_size", "finish_limit", "early_stop_mode", "max_steps", "stop_width",
                             "result_width", "predicate_bias", "full_label_check", "pending_base_stop")] + \
        [("alpha", C.c_float)]


_L = None


def available() -> bool:
    return LIB.exists()


def lib() -> C.CDLL:
    global _L
    if _L is None:
        L = C.CDLL(str(LIB))
        L.gofann_ref_pq_search.argtypes = [C.POINTER(RefPqArgs)]
        L.gofann_ref_pq_search.restype = C.c_int
        L.gofann_ref_pq_args_size.restype = C.c_size_t
        if L.gofann_ref_pq_args_size() != C.sizeof(RefPqArgs):
            raise RuntimeError("gofann_ref_pq_args layout mismatch")
        L.gofann_ref_pickup_cases.argtypes = [_P, _P, C.c_int, C.c_int, _P]
        L.gofann_ref_pickup_cases.restype = C.c_int
        L.gofann_ref_result_heap_cases.argtypes = [_P, _P, C.c_int, C.c_int, C.c_int, _P, _P]
        L.gofann_ref_result_heap_cases.restype = C.c_int
        _L = L
    return _L


def run_reference_pq(case: dict, trace_width: int = 64, device="cuda") -> dict:
    """The reference kernel on `case` (route r searches query row r)."""
    import torch
    p = case["params"]
    routes, graph, attrs = case["routes"], case["graph"], case["attrs"]
    n_routes = int(routes["query_row"].shape[0])
    rw = int(p["result_width"])
    pq_dim = int(case["codes"]["pq_codes"].shape[1])
    dim = int(case["queries"].shape[1])
    n_samples = int(attrs["label_indptr"].shape[0] - 1)

    keep = []

    def d(a, dtype=None):
        a = np.ascontiguousarray(a if dtype is None else a.astype(dtype))
        if a.dtype == np.uint64:
            a = a.view(np.int64)
        elif a.dtype == np.uint32:
            a = a.view(np.int32)
        t = torch.from_numpy(a).to(device)
        keep.append(t)
        return t.data_ptr()

    def zeros(shape, dtype):
        t = torch.zeros(shape, dtype=dtype, device=device)
        keep.append(t)
        return t

    a = RefPqArgs()
    a.codes = d(case["codes"]["pq_codes"])
    a.centroids = d(case["centroids"], np.float32)
    a.queries = d(case["queries"][routes["query_row"].astype(np.int64)])
    a.adjacency = d(graph["adjacency"])
    a.row_to_sample = d(graph["row_to_sample"])
    a.label_offset = d(graph["label_offset"])
    a.zero_groups = d(np.zeros(graph["label_offset"].shape[0], np.uint32))
    a.data_indptr = d(attrs["label_indptr"])
    a.data_indptr32 = d(attrs["label_indptr"].astype(np.uint32))
    a.data_indices = d(attrs["label_indices"])
    a.group_id = d(routes["group_id"])
    a.start_local = d(routes["start_local"])
    a.filter_bits = d(routes.get("filter_bits", np.full(n_routes, np.uint64(0xFFFFFFFFFFFFFFFF), np.uint64)))
    a.qlabel_indptr = d(routes["qlabel_indptr"])
    a.qlabel_indices = d(routes["qlabel_indices"])
    a.primary_label = d(routes["primary_label"])
    if routes.get("pred_offsets") is not None:
        a.pred_offsets = d(routes["pred_offsets"])
        a.clauses = d(np.ascontiguousarray(routes["clauses"]).view(np.uint8).reshape(-1))
        a.pred_handles = d(routes["pred_handles"])
        a.pred_enabled = d(routes["pred_enabled"])
    ids = zeros((n_routes, rw), torch.int64)
    dist = zeros((n_routes, rw), torch.float32)
    table = zeros((n_routes, pq_dim, 256), torch.float32)
    a.out_ids, a.out_dists, a.pq_table = ids.data_ptr(), dist.data_ptr(), table.data_ptr()
    a.hash = zeros((n_routes, 4096), torch.int32).data_ptr()
    tpb = zeros((n_routes, 6), torch.float32)
    a.time_per_block = tpb.data_ptr()
    a.datadist = zeros((n_routes, 64), torch.float32).data_ptr()
    trace = None
    if trace_width:
        trace = torch.full((n_routes, trace_width), -1, dtype=torch.int32, device=device)
        keep.append(trace)
        a.trace_rows = trace.data_ptr()
        a.trace_slots = d(np.arange(n_routes, dtype=np.uint32))
        a.trace_counters = zeros((n_routes, 3), torch.int32).data_ptr()
        a.trace_width = trace_width
    a.n_samples, a.dim, a.pq_dim = n_samples, dim, pq_dim
    a.degree = int(graph["adjacency"].shape[1])
    a.n_routes = n_routes
    a.queue_size = int(p["queue_size"])
    a.finish_limit = int(p.get("finish_limit", 100))
    a.early_stop_mode = int(p.get("early_stop_mode", 2))
    a.max_steps = int(p.get("max_steps", 0))
    a.stop_width = int(p.get("stop_width", 10))
    a.result_width = rw
    a.predicate_bias = int(p.get("predicate_bias", 0))
    a.full_label_check = int(p.get("full_label_check", 0))
    a.pending_base_stop = int(p.get("pending_base_stop", 0))
    a.alpha = float(p.get("alpha", 0.15))
    st = lib().gofann_ref_pq_search(C.byref(a))
    if st != 0:
        raise RuntimeError(f"gofann_ref_pq_search returned {st}")
    torch.cuda.synchronize()
    out_ids = ids.cpu().numpy()
    res = {
        "ids": np.where(out_ids == U32MAX, U32MAX, out_ids).astype(np.uint32),
        "dists": dist.cpu().numpy(),
        "steps": tpb.cpu().numpy()[:, 4].astype(np.int32),
        "pq_table": table.cpu().numpy(),
    }
    if trace is not None:
        res["trace"] = trace.cpu().numpy().view(np.uint32)
    del keep
    return res


def pickup_cases(keys: np.ndarray, used: np.ndarray, sizes: np.ndarray, device="cuda") -> np.ndarray:
    """The reference's cooperative pickup on frontiers keys[c][:sizes[c]]
    (index 0 unused; used[c][i] marks expanded entries): the index it picks
    per frontier, -1 when every entry is used."""
    import torch
    n, stride = keys.shape
    f = np.zeros((n, stride, 3), np.uint32)
    f[:, :, 0] = np.ascontiguousarray(keys, np.float32).view(np.uint32)
    f[:, :, 1] = np.arange(stride, dtype=np.uint32)[None, :] | (used.astype(np.uint32) << 31)
    f[:, :, 2] = f[:, :, 0]
    df = torch.from_numpy(f.view(np.int32)).to(device)
    ds = torch.from_numpy(np.ascontiguousarray(sizes, np.int32)).to(device)
    out = torch.empty(n, dtype=torch.int32, device=device)
    st = lib().gofann_ref_pickup_cases(df.data_ptr(), ds.data_ptr(), n, stride, out.data_ptr())
    if st != 0:
        raise RuntimeError(f"gofann_ref_pickup_cases returned {st}")
    torch.cuda.synchronize()
    return out.cpu().numpy()


def result_heap_cases(keys: np.ndarray, payloads: np.ndarray, cap: int, device="cuda"):
    """The reference's result heap fed keys[c] in order (capacity cap), then
    emptied into ascending slots: (firsts, payloads) [n_cases][cap]."""
    import torch
    n, m = keys.shape
    dk = torch.from_numpy(np.ascontiguousarray(keys, np.float32)).to(device)
    dp = torch.from_numpy(np.ascontiguousarray(payloads, np.uint32).view(np.int32)).to(device)
    of = torch.empty((n, cap), dtype=torch.float32, device=device)
    os_ = torch.empty((n, cap), dtype=torch.int32, device=device)
    st = lib().gofann_ref_result_heap_cases(dk.data_ptr(), dp.data_ptr(), n, m, cap, of.data_ptr(), os_.data_ptr())
    if st != 0:
        raise RuntimeError(f"gofann_ref_result_heap_cases returned {st}")
    torch.cuda.synchronize()
    return of.cpu().numpy(), os_.cpu().numpy().view(np.uint32)


# ------------------------------------------------- the Full-GPU backend
FULL_LIB = HERE / "_ref" / "libgofann_ref_full_gpu.so"


class RefFullArgs(C.Structure):
    """Byte-for-byte gofann_ref_full_args of oracle/ref_full_gpu.cu."""
    _fields_ = [(n, _P) for n in (
        "base", "queries", "graph", "active_ids", "query_vector_ids", "group_ids", "start_local", "label_size",
        "label_offset", "row_to_sample", "row_filter_mask", "filter_bits", "filter_modes", "single_extra",
        "active_range_counts", "qlabel_indptr", "qlabel_indices", "sample_indptr", "sample_indices",
        "range_modes", "range_lower", "range_upper", "base_ranges", "low_sample_ids", "results", "distances",
        "steps")] + \
        [(n, _U32) for n in ("base_rows", "dim", "degree", "n_routes", "range_count", "finish_count", "max_steps",
                             "topk")] + \
        [(n, _I32) for n in ("early_stop_mode", "queue_size", "dtype", "reserved")]


_F = None


def full_available() -> bool:
    return FULL_LIB.exists()


def full_lib() -> C.CDLL:
    global _F
    if _F is None:
        L = C.CDLL(str(FULL_LIB))
        for fn in ("gofann_ref_full_highfreq", "gofann_ref_full_lowfreq"):
            getattr(L, fn).argtypes = [C.POINTER(RefFullArgs)]
            getattr(L, fn).restype = C.c_int
        L.gofann_ref_full_args_size.restype = C.c_size_t
        if L.gofann_ref_full_args_size() != C.sizeof(RefFullArgs):
            raise RuntimeError("gofann_ref_full_args layout mismatch")
        L.gofann_ref_block_pickup_cases.argtypes = [_P, _P, C.c_int, C.c_int, _P]
        L.gofann_ref_block_pickup_cases.restype = C.c_int
        _F = L
    return _F


def _full_common(a: RefFullArgs, case: dict, routes: dict, d, device):
    """Fills the arguments both Full-GPU kernels share: vectors, the route's
    residual labels (every query label but its own, filter mode
    GenericWithRange = 5: active ranges, then the labels), filter bits and
    ranges."""
    attrs = case["attrs"]
    n = int(routes["query_row"].shape[0])
    base, queries = case["base"], case["queries"]
    a.base, a.queries = d(base), d(queries)
    a.base_rows, a.dim, a.dtype = int(base.shape[0]), int(base.shape[1]), int(case["dtype"])
    a.active_ids = d(np.arange(n, dtype=np.uint32))
    a.query_vector_ids = d(routes["query_row"])
    a.n_routes = n
    ip, ind, prim = routes["qlabel_indptr"], routes["qlabel_indices"], routes["primary_label"]
    res = [np.array([x for x in ind[ip[r]:ip[r + 1]] if x != prim[r]], np.uint32) for r in range(n)]
    rp = np.zeros(n + 1, np.uint32)
    rp[1:] = np.cumsum([len(x) for x in res])
    a.qlabel_indptr = d(rp)
    a.qlabel_indices = d(np.concatenate(res + [np.zeros(1, np.uint32)]).astype(np.uint32))
    a.sample_indptr = d(attrs["label_indptr"].astype(np.uint32))
    a.sample_indices = d(attrs["label_indices"])
    a.filter_bits = d(routes.get("filter_bits", np.full(n, np.uint64(0xFFFFFFFFFFFFFFFF), np.uint64)))
    a.filter_modes = d(np.full(n, 5, np.uint8))
    a.single_extra = d(np.full(n, U32MAX, np.uint32))
    rm = routes.get("range_modes")
    if rm is not None:
        a.range_count = int(rm.shape[1])
        a.range_modes, a.range_lower, a.range_upper = d(rm), d(routes["range_lower"]), d(routes["range_upper"])
        a.base_ranges = d(attrs["range_values"])
        a.active_range_counts = d((rm != 0).sum(1).astype(np.uint32))
    else:
        a.active_range_counts = d(np.zeros(n, np.uint32))


def run_reference_full(case: dict, device="cuda") -> dict:
    """The reference's graph-route kernel on a tests/ref_full_cases.py case:
    per route the top-k sample ids, distances and step counts."""
    import torch
    keep = []

    def d(x):
        x = np.ascontiguousarray(x)
        if x.dtype == np.uint64:
            x = x.view(np.int64)
        elif x.dtype == np.uint32:
            x = x.view(np.int32)
        elif x.dtype == np.uint16:
            x = x.view(np.int16)
        t = torch.from_numpy(x).to(device)
        keep.append(t)
        return t.data_ptr()

    p, g, routes = case["params"], case["graph"], case["routes"]
    a = RefFullArgs()
    _full_common(a, case, routes, d, device)
    n, k = a.n_routes, int(p["result_width"])
    rows = int(g["adjacency"].shape[0])
    off = g["label_offset"].astype(np.int64)
    a.graph, a.degree = d(g["adjacency"]), int(g["adjacency"].shape[1])
    a.label_offset = d(g["label_offset"])
    a.label_size = d(np.diff(np.append(off, rows)).astype(np.uint32))
    a.row_to_sample = d(g["row_to_sample"])
    a.row_filter_mask = d(g.get("row_filter_mask", np.full(rows, np.uint64(0xFFFFFFFFFFFFFFFF), np.uint64)))
    a.group_ids, a.start_local = d(routes["group_id"]), d(routes["start_local"])
    a.finish_count, a.max_steps, a.topk = int(p["finish_limit"]), int(p["max_steps"]), k
    a.early_stop_mode, a.queue_size = int(p["early_stop_mode"]), int(p["queue_size"])
    ids = torch.full((n, k), -1, dtype=torch.int64, device=device)
    dist = torch.full((n, k), float(np.finfo(np.float32).max), dtype=torch.float32, device=device)
    steps = torch.zeros(n, dtype=torch.int32, device=device)
    a.results, a.distances, a.steps = ids.data_ptr(), dist.data_ptr(), steps.data_ptr()
    st = full_lib().gofann_ref_full_highfreq(C.byref(a))
    if st != 0:
        raise RuntimeError(f"gofann_ref_full_highfreq returned {st}")
    torch.cuda.synchronize()
    out = ids.cpu().numpy().astype(np.uint64)
    res = {"ids": np.where(out > U32MAX, U32MAX, out).astype(np.uint32), "dists": dist.cpu().numpy(),
           "steps": steps.cpu().numpy()}
    del keep
    return res


def run_reference_full_low(case: dict, device="cuda") -> dict:
    """The reference's posting-route kernel on a build_low_case case: each
    route is its own low-frequency group (its slice of posting_ids), every
    posting entry's row mask all ones."""
    import torch
    keep = []

    def d(x):
        x = np.ascontiguousarray(x)
        if x.dtype == np.uint64:
            x = x.view(np.int64)
        elif x.dtype == np.uint32:
            x = x.view(np.int32)
        elif x.dtype == np.uint16:
            x = x.view(np.int16)
        t = torch.from_numpy(x).to(device)
        keep.append(t)
        return t.data_ptr()

    routes = case["routes"]
    a = RefFullArgs()
    _full_common(a, case, routes, d, device)
    n, k = a.n_routes, int(case["topk"])
    a.group_ids = d(np.arange(n, dtype=np.uint32))
    a.label_offset = d(case["begin"].astype(np.uint32))
    a.label_size = d(case["count"])
    a.low_sample_ids = d(case["posting_ids"])
    a.row_filter_mask = d(np.full(case["posting_ids"].shape[0], np.uint64(0xFFFFFFFFFFFFFFFF), np.uint64))
    a.topk = k
    ids = torch.full((n, k), -1, dtype=torch.int64, device=device)
    dist = torch.full((n, k), float(np.finfo(np.float32).max), dtype=torch.float32, device=device)
    steps = torch.zeros(n, dtype=torch.int32, device=device)
    a.results, a.distances, a.steps = ids.data_ptr(), dist.data_ptr(), steps.data_ptr()
    st = full_lib().gofann_ref_full_lowfreq(C.byref(a))
    if st != 0:
        raise RuntimeError(f"gofann_ref_full_lowfreq returned {st}")
    torch.cuda.synchronize()
    out = ids.cpu().numpy().astype(np.uint64)
    res = {"ids": np.where(out > U32MAX, U32MAX, out).astype(np.uint32), "dists": dist.cpu().numpy()}
    del keep
    return res


def block_pickup_cases(keys: np.ndarray, used: np.ndarray, sizes: np.ndarray, device="cuda") -> np.ndarray:
    """The Full-GPU backend's block pickup (128 threads) on frontiers
    keys[c][:sizes[c]]: the index it picks per frontier, -1 when all used."""
    import torch
    n, stride = keys.shape
    f = np.zeros((n, stride, 2), np.uint32)
    f[:, :, 0] = np.ascontiguousarray(keys, np.float32).view(np.uint32)
    f[:, :, 1] = np.arange(stride, dtype=np.uint32)[None, :] | (used.astype(np.uint32) << 31)
    df = torch.from_numpy(f.view(np.int32)).to(device)
    ds = torch.from_numpy(np.ascontiguousarray(sizes, np.int32)).to(device)
    out = torch.empty(n, dtype=torch.int32, device=device)
    st = full_lib().gofann_ref_block_pickup_cases(df.data_ptr(), ds.data_ptr(), n, stride, out.data_ptr())
    if st != 0:
        raise RuntimeError(f"gofann_ref_block_pickup_cases returned {st}")
    torch.cuda.synchronize()
    return out.cpu().numpy()


# ------------------------------------------------- the RaBitQ estimator
RQ_LIB = HERE / "_ref" / "libgofann_ref_rabitq.so"
_Q = None


def rq_available() -> bool:
    return RQ_LIB.exists()


def run_reference_rq_score(case: dict, device="cuda") -> np.ndarray:
    """The reference's score_rabitq_code_device<true> on a
    tests/ref_rabitq_cases.py case: one estimate per (row, point) pair."""
    import torch
    global _Q
    if _Q is None:
        L = C.CDLL(str(RQ_LIB))
        L.gofann_ref_rq_score.argtypes = [_P] * 9 + [_U32, _U32, _U32, _P]
        L.gofann_ref_rq_score.restype = C.c_int
        _Q = L
    keep = []

    def d(x):
        x = np.ascontiguousarray(x)
        if x.dtype == np.uint32:
            x = x.view(np.int32)
        t = torch.from_numpy(x).to(device)
        keep.append(t)
        return t.data_ptr()

    n = int(case["pair_row"].shape[0])
    out = torch.empty(n, dtype=torch.float32, device=device)
    st = _Q.gofann_ref_rq_score(d(case["anchor_ids"]), d(case["codes"]), d(case["factors"]), d(case["k1"]),
                                d(case["gdist"]), d(case["q8"]), d(case["scale"]), d(case["pair_row"]),
                                d(case["pair_point"]), n, int(case["num_anchors"]), int(case["padded_dim"]),
                                out.data_ptr())
    if st != 0:
        raise RuntimeError(f"gofann_ref_rq_score returned {st}")
    torch.cuda.synchronize()
    res = out.cpu().numpy()
    del keep
    return res
