"""Full-GPU exact-distance mode on the GPU against the CPU oracle: the
traversal (gofann_exact_search, run_full_gpu_highfreq_route,
src/search/full_gpu/backend_full_gpu.cu:1682-2043) and the exact posting
scan (gofann_exact_posting_scan, full_gpu_lowfreq_kernel :2124-2260).

u8 distances are integers, so ids, distance bits, step counts and expansion
traces must match exactly; f32 / f16 distances follow the reference's lane
order and tree in both implementations, so they must match bit for bit too.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from fixtures import cfg1_small, cfg2_small, dev, dev_dict, fbits, host, with_predicates
from gofann import _abi as A
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    assert torch.cuda.is_available()
    return A.lib()


def stream():
    return torch.cuda.current_stream().cuda_stream


def run_exact(L, graph, attrs, base, dtype, queries, routes, trace_width=0, label_size=None, **params):
    dg, da, dr = dev_dict(graph), dev_dict(attrs), dev_dict(routes)
    gs, at, rs = A.fill_graph(dg), A.fill_attrs(da), A.fill_routes(dr)
    gs.degree = int(graph["adjacency"].shape[1])
    sp = A.fill_params(**params)
    n, k = rs.n_routes, sp.result_width
    ids = torch.empty((n, k), dtype=torch.int32, device="cuda")
    d = torch.empty((n, k), dtype=torch.float32, device="cuda")
    steps = torch.empty(n, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    trace = torch.empty((n, max(trace_width, 1)), dtype=torch.int32, device="cuda")
    out = A.SearchOut(ids=A.ptr(ids), dists=A.ptr(d), steps=A.ptr(steps), status=A.ptr(status),
                      trace=A.ptr(trace) if trace_width else None, trace_width=trace_width)
    nbytes = L.gofann_exact_search_scratch_bytes(n)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    db, dq = dev(base), dev(queries)
    ls = dev(label_size) if label_size is not None else None
    A.check(L.gofann_exact_search(C.byref(gs), A.ptr(ls), C.byref(at), A.ptr(db), dtype, base.shape[1], A.ptr(dq),
                                  C.byref(rs), C.byref(sp), C.byref(out), A.ptr(scratch), nbytes, stream()),
            "exact_search")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    res = (host(ids, np.uint32), d.cpu().numpy(), steps.cpu().numpy())
    if trace_width:
        return res + (host(trace, np.uint32),)
    return res


def _check(got, want):
    for name, g, o in zip(("ids", "dists", "steps", "trace"), got, want):
        if name == "dists":
            g, o = fbits(g), fbits(o)
        assert np.array_equal(g, o), f"{name} differ in {np.count_nonzero(np.any(np.atleast_2d(g != o), axis=-1))} routes"


VARIANTS = [
    dict(queue_size=64, early_stop_mode=A.EARLY_STOP_ADAPTIVE, result_width=10),
    dict(queue_size=16, early_stop_mode=A.EARLY_STOP_FIXED, finish_limit=20, result_width=10),
    dict(queue_size=200, early_stop_mode=A.EARLY_STOP_FIXED, finish_limit=100, result_width=7),
    dict(queue_size=512, early_stop_mode=A.EARLY_STOP_OFF, max_steps=300, result_width=10),
    dict(queue_size=2, early_stop_mode=A.EARLY_STOP_ADAPTIVE, result_width=1),
    dict(queue_size=96, early_stop_mode=A.EARLY_STOP_ADAPTIVE, result_width=10, max_steps=40),
]


def _workload(wl):
    """(workload, index, plan, base, queries, dtype) of a small case:
    cfg2 u8 192-d, cfg1 f32 128-d, or cfg1 converted to f16."""
    if wl == "u8":
        w, idx, plan = cfg2_small()
        return w, idx, plan, w.base, w.queries, A.DTYPE_U8
    w, idx, plan = cfg1_small()
    if wl == "f32":
        return w, idx, plan, w.base.astype(np.float32), w.queries.astype(np.float32), A.DTYPE_F32
    return w, idx, plan, w.base.astype(np.float16).view(np.uint16), w.queries.astype(np.float16).view(np.uint16), \
        A.DTYPE_F16


@pytest.mark.parametrize("wl", ["u8", "f32", "f16"])
@pytest.mark.parametrize("vi", range(len(VARIANTS)))
def test_exact_search_bitexact(L, wl, vi):
    w, idx, plan, base, q, dt = _workload(wl)
    params = VARIANTS[vi]
    want = O.exact_search(idx.graph(), idx.attrs(), base, dt, q, plan.graph_routes, threads=8, trace_width=64,
                          **params)
    got = run_exact(L, idx.graph(), idx.attrs(), base, dt, q, plan.graph_routes, trace_width=64, **params)
    _check(got, want)


def test_exact_search_filters_bitexact(L):
    """Filter bits against row masks, range modes 0-3 and residual labels on
    the expanded node (candidate_passes_device, backend_full_gpu.cu:
    1015-1092)."""
    w, idx, plan = cfg2_small()
    attrs, graph, _, legacy = with_predicates(w, idx, plan.graph_routes, seed=5)
    params = dict(queue_size=64, early_stop_mode=A.EARLY_STOP_ADAPTIVE, result_width=10)
    want = O.exact_search(graph, attrs, w.base, A.DTYPE_U8, w.queries, legacy, threads=8, trace_width=64, **params)
    got = run_exact(L, graph, attrs, w.base, A.DTYPE_U8, w.queries, legacy, trace_width=64, **params)
    _check(got, want)
    assert (want[2] > 0).all()


def test_exact_search_label_size_and_bad_routes(L):
    """Explicit group sizes give the same results as sizes derived from the
    offsets; routes with an out-of-range group or seed return no results and
    zero steps."""
    w, idx, plan = cfg2_small()
    g = idx.graph()
    off = g["label_offset"].astype(np.int64)
    sizes = np.diff(np.append(off, g["adjacency"].shape[0])).astype(np.uint32)
    routes = {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in plan.graph_routes.items()}
    routes["group_id"][0] = 0xFFFFFFFF
    routes["start_local"][1] = sizes[routes["group_id"][1]]
    params = dict(queue_size=48, early_stop_mode=A.EARLY_STOP_ADAPTIVE, result_width=10)
    want = O.exact_search(g, idx.attrs(), w.base, A.DTYPE_U8, w.queries, routes, threads=8, **params)
    got1 = run_exact(L, g, idx.attrs(), w.base, A.DTYPE_U8, w.queries, routes, **params)
    got2 = run_exact(L, g, idx.attrs(), w.base, A.DTYPE_U8, w.queries, routes, label_size=sizes, **params)
    _check(got1, want)
    _check(got2, want)
    assert want[2][0] == 0 and want[2][1] == 0 and (want[0][:2] == A.U32MAX).all()


def _chain(n=6000, degree=64, dim=64, seed=4):
    """One group whose rows link forward: routes admit thousands of rows, so
    their visited tables fill; some rows list an id twice."""
    rng = np.random.default_rng(seed)
    adj = ((np.arange(n)[:, None] + 1 + rng.integers(0, 200, size=(n, degree))) % n).astype(np.uint32)
    adj[:, 5] = adj[:, 0]
    base = rng.integers(0, 256, size=(n, dim)).astype(np.uint8)
    q = rng.integers(0, 256, size=(24, dim)).astype(np.uint8)
    graph = {"adjacency": adj, "row_to_sample": np.arange(n, dtype=np.uint32),
             "label_offset": np.zeros(1, np.uint32)}
    attrs = {"label_indptr": np.zeros(n + 1, np.uint64), "label_indices": np.zeros(1, np.uint32)}
    routes = {"query_row": np.arange(24, dtype=np.uint32), "group_id": np.zeros(24, np.uint32),
              "start_local": rng.integers(0, n, size=24).astype(np.uint32)}
    return graph, attrs, base, q, routes


@pytest.mark.parametrize("queue_size", [64, 512])
def test_exact_search_visited_table_fills(L, queue_size):
    graph, attrs, base, q, routes = _chain()
    params = dict(queue_size=queue_size, early_stop_mode=A.EARLY_STOP_OFF, max_steps=400, result_width=10)
    want = O.exact_search(graph, attrs, base, A.DTYPE_U8, q, routes, threads=8, trace_width=64, **params)
    got = run_exact(L, graph, attrs, base, A.DTYPE_U8, q, routes, trace_width=64, **params)
    _check(got, want)


@pytest.mark.parametrize("wl", ["u8", "f32", "f16"])
@pytest.mark.parametrize("k", [1, 10, 100])
def test_exact_posting_scan_bitexact(L, wl, k):
    w, idx, plan, base, q, dt = _workload(wl)
    attrs, _, dnf, _ = with_predicates(w, idx, plan.posting_routes, seed=2)
    pr = dnf
    want = O.exact_posting_scan(base, dt, q, attrs, pr, idx.posting_ids, plan.posting_begin, plan.posting_count, k)
    dr, da = dev_dict(pr), dev_dict(attrs)
    rs, at = A.fill_routes(dr), A.fill_attrs(da)
    n = rs.n_routes
    ids = torch.empty((n, k), dtype=torch.int32, device="cuda")
    d = torch.empty((n, k), dtype=torch.float32, device="cuda")
    db, dq = dev(base), dev(q)
    pid, pb, pc = dev(idx.posting_ids), dev(plan.posting_begin), dev(plan.posting_count)
    A.check(L.gofann_exact_posting_scan(A.ptr(db), dt, base.shape[0], base.shape[1], A.ptr(dq), C.byref(at),
                                        C.byref(rs), A.ptr(pid), A.ptr(pb), A.ptr(pc), k, A.ptr(ids), A.ptr(d),
                                        stream()), "exact_posting_scan")
    torch.cuda.synchronize()
    assert np.array_equal(host(ids, np.uint32), want[0])
    assert np.array_equal(fbits(d.cpu().numpy()), fbits(want[1]))


@pytest.mark.parametrize("wl", ["cfg1", "cfg2"])
def test_exact_pipeline_matches_oracle_and_recall(L, wl):
    from gofann.engine import DeviceIndex, DevicePlan, ExactPipeline, SearchConfig
    w, idx, plan = cfg1_small() if wl == "cfg1" else cfg2_small()
    dt = A.DTYPE_U8 if w.dtype == "u8" else A.DTYPE_F32
    cfg = SearchConfig(queue_size=64)
    pipe = ExactPipeline(DeviceIndex(idx, row_records=False), DevicePlan(plan, "cuda"), cfg)
    gi, gd = pipe.run(dev(w.queries))
    torch.cuda.synchronize()
    gi, gd = host(gi, np.uint32), gd.cpu().numpy()
    params = dict(queue_size=cfg.queue_size, result_width=cfg.topk, finish_limit=cfg.finish_limit,
                  early_stop_mode=cfg.early_stop_mode)
    bi, bd, _ = O.exact_search(idx.graph(), idx.attrs(), w.base, dt, w.queries, plan.graph_routes, threads=8,
                               **params)
    pi, pd = O.exact_posting_scan(w.base, dt, w.queries, idx.attrs(), plan.posting_routes, idx.posting_ids,
                                  plan.posting_begin, plan.posting_count, cfg.topk)
    qoff, order = plan.merge_tables()
    wi, wd = O.route_merge(np.concatenate([bi, pi]), np.concatenate([bd, pd]), qoff, order, cfg.topk)
    assert np.array_equal(gi, wi)
    assert np.array_equal(fbits(gd), fbits(wd))
    from gofann.planner import _route_tables
    labs = [np.asarray(x, np.uint32) for x in w.query_labels]
    gt_routes = _route_tables(list(range(len(labs))), labs, [x[0] for x in labs], [0] * len(labs), [0] * len(labs))
    gt_routes["pred_enabled"][:] = 0
    ti, _ = O.filtered_topk(w.base, dt, w.queries, idx.attrs(), gt_routes, 10)
    rec = np.mean([len((set(gi[i].tolist()) & set(ti[i].tolist())) - {A.U32MAX}) /
                   max(1, len(set(ti[i].tolist()) - {A.U32MAX})) for i in range(gi.shape[0])])
    assert rec >= 0.95, rec
