"""Predicate kinds beyond the AND of labels, on the GPU against the oracle.

Fixtures (tests/fixtures.with_predicates) add float range attributes in two
dimensions, per-row filter masks, and two predicate forms to the planner's
routes:
  * compiled DNF: 1-3 OR-ed clauses of label atoms and range atoms in modes
    1-3 (gpu_predicate_index.cuh:100-136, range_filter.cuh:28-77), some
    routes with the predicate disabled;
  * the legacy per-route filters: query filter bits against row filter masks
    (backend_pq.cu:4394-4397), range modes 0-3 with bounds
    (range_filter.cuh:47-98), compiled-route flags, the resident residual
    label check.
Traversal ids, distances, steps, counters and traces, posting-scan
shortlists and the predicate pass bitmaps must equal the oracle's bit for
bit.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from fixtures import cfg1_small, cfg2_small_u8cb, dev, dev_dict, fbits, host, rabitq_artifacts, with_predicates
from gofann import _abi as A
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return A.lib()


def stream():
    return torch.cuda.current_stream().cuda_stream


def _cfg1():
    w, idx, plan = cfg1_small()
    attrs, graph, dnf, legacy = with_predicates(w, idx, plan.graph_routes, seed=5)
    return w, idx, plan, attrs, graph, dnf, legacy


def _beam(L, graph, attrs, codes, prep, routes, trace_width, **params):
    from test_gpu_parity import run_gpu_beam
    return run_gpu_beam(L, graph, attrs, codes, prep, routes, trace_width=trace_width, **params)


def _check(got, want):
    for name, g, o in zip(("ids", "dists", "steps", "counters", "trace"), got, want):
        if name == "dists":
            g, o = fbits(g), fbits(o)
        assert np.array_equal(g, o), f"{name} differ in {np.count_nonzero(np.any(np.atleast_2d(g != o), axis=-1))} routes"


VARIANTS = [
    dict(queue_size=64, predicate_bias=1, early_stop_mode=A.EARLY_STOP_ADAPTIVE, result_width=100,
         pq_mode=A.PQ_LUT_GLOBAL),
    dict(queue_size=32, predicate_bias=0, early_stop_mode=A.EARLY_STOP_FIXED, finish_limit=20, result_width=50,
         pq_mode=A.PQ_DIRECT),
    dict(queue_size=128, predicate_bias=1, early_stop_mode=A.EARLY_STOP_OFF, result_width=200, max_steps=300,
         pq_mode=A.PQ_LUT_SHARED, alpha=0.4),
]


@pytest.mark.parametrize("form", ["dnf", "legacy", "legacy_full_label"])
@pytest.mark.parametrize("vi", range(len(VARIANTS)))
def test_beam_search_predicates_bitexact(L, form, vi):
    w, idx, plan, attrs, graph, dnf, legacy = _cfg1()
    params = dict(VARIANTS[vi], scorer=A.SCORER_PQ)
    if form != "dnf":
        params["predicate_bias"] = 0  # the bias needs a DNF predicate
    if form == "legacy_full_label":
        params["full_label_check"] = 1
    routes = dnf if form == "dnf" else legacy
    lut = O.pq_build_lut(w.queries.astype(np.float32), idx.pq_centroids, idx.pq_codes.shape[1])
    want = O.beam_search(graph, attrs, idx.codes(), {"pq_lut": lut}, routes, threads=8, trace_width=64, **params)
    if params["pq_mode"] in (A.PQ_DIRECT, A.PQ_U8):
        prep = {"pq_query": dev(w.queries), "pq_centroids": dev(idx.pq_centroids)}
    else:
        prep = {"pq_lut": dev(lut)}
    got = _beam(L, graph, attrs, idx.codes(), prep, routes, 64, **params)
    _check(got, want)
    # the predicates must bite: some route returns fewer results than without them
    assert np.any((want[0] != A.U32MAX).sum(1) < params["result_width"])


@pytest.mark.parametrize("form", ["dnf", "legacy"])
def test_beam_search_predicates_u8_records_bitexact(L, form):
    """PQ_U8 traversal over per-row records (sample, label row and signature
    read from the record) under both predicate forms."""
    from test_gpu_parity import _with_records
    w, idx, plan = cfg2_small_u8cb(48)
    attrs, graph, dnf, legacy = with_predicates(w, idx, plan.graph_routes, seed=9)
    routes = dnf if form == "dnf" else legacy
    params = dict(queue_size=64, predicate_bias=1 if form == "dnf" else 0, early_stop_mode=A.EARLY_STOP_ADAPTIVE,
                  result_width=100, pq_mode=A.PQ_U8, scorer=A.SCORER_PQ)
    lut = O.pq_build_lut(w.queries.astype(np.float32), idx.pq_centroids, idx.pq_codes.shape[1])
    want = O.beam_search(graph, attrs, idx.codes(), {"pq_lut": lut}, routes, threads=8, trace_width=64, **params)
    g, _ = _with_records(L, graph, attrs, idx.codes())
    prep = {"pq_query": dev(w.queries), "pq_centroids": dev(idx.pq_centroids)}
    _check(_beam(L, g, attrs, idx.codes(), prep, routes, 64, **params), want)


def test_beam_search_predicates_rabitq_bitexact(L):
    from test_gpu_parity import _rq_prepared
    w, idx, plan, rq, anchors, qr = rabitq_artifacts(dim=480)
    attrs, graph, dnf, legacy = with_predicates(w, idx, plan.graph_routes, seed=13)
    dprep, hprep = _rq_prepared(L, qr, anchors)
    params = dict(queue_size=64, predicate_bias=1, early_stop_mode=A.EARLY_STOP_ADAPTIVE, result_width=100,
                  scorer=A.SCORER_RABITQ)
    want = O.beam_search(graph, attrs, rq, hprep, dnf, threads=8, trace_width=64, **params)
    _check(_beam(L, graph, attrs, rq, dprep, dnf, 64, **params), want)


@pytest.mark.parametrize("scorer", ["pq_lut", "pq_u8", "rabitq"])
def test_posting_scan_dnf_bitexact(L, scorer):
    """Posting scans under OR-ed clauses with range atoms, over the planner's
    postings and long slices of a random order of the base."""
    from test_gpu_parity import _rq_prepared, run_gpu_posting
    if scorer == "rabitq":
        w, idx, plan, rq, anchors, qr = rabitq_artifacts(dim=992, n_queries=64)
        codes = rq
        dprep, hprep = _rq_prepared(L, qr, anchors)
        sc, mode = A.SCORER_RABITQ, A.PQ_LUT_GLOBAL
    else:
        w, idx, plan = cfg2_small_u8cb(48) if scorer == "pq_u8" else cfg1_small()
        codes = idx.codes()
        lut = O.pq_build_lut(w.queries.astype(np.float32), idx.pq_centroids, idx.pq_codes.shape[1])
        hprep = {"pq_lut": lut}
        if scorer == "pq_u8":
            dprep = {"pq_query": dev(w.queries), "pq_centroids": dev(idx.pq_centroids)}
            mode = A.PQ_U8
        else:
            dprep, mode = {"pq_lut": dev(lut)}, A.PQ_LUT_GLOBAL
        sc = A.SCORER_PQ
    attrs, graph, dnf, legacy = with_predicates(w, idx, plan.graph_routes, seed=17)
    n = dnf["query_row"].shape[0]
    rng = np.random.default_rng(1)
    order = rng.permutation(w.n).astype(np.uint32)
    pids = np.concatenate([idx.posting_ids, order]).astype(np.uint32)
    lab = dnf["primary_label"]
    begin = idx.posting_begin[lab].astype(np.uint64)
    count = idx.posting_count[lab].astype(np.uint32)
    half = np.arange(n) % 2 == 1  # odd routes scan a long slice of the order instead
    lo = rng.integers(0, w.n // 2, size=n)
    begin[half] = (idx.posting_ids.shape[0] + lo[half]).astype(np.uint64)
    count[half] = rng.integers(1000, w.n - lo[half]).astype(np.uint32)
    for k in (10, 100):
        want = O.posting_scan(codes, hprep, attrs, dnf, sc, pids, begin, count, k)
        got = run_gpu_posting(L, codes, dprep, attrs, dnf, sc, pids, begin, count, k, pq_mode=mode)
        assert np.array_equal(got[0], want[0])
        assert np.array_equal(fbits(got[1]), fbits(want[1]))
    assert np.any((want[0] == A.U32MAX).any(1))  # some shortlists come out short


def _masks(L, graph, attrs, routes, cand_route, cand_rows, expect_status=0):
    dg, da, dr = dev_dict(graph), dev_dict(attrs), dev_dict(routes)
    gs, at, rs = A.fill_graph(dg), A.fill_attrs(da), A.fill_routes(dr)
    n = cand_route.shape[0]
    out = torch.full(((n + 31) // 32,), -1, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    d_route, d_rows = dev(cand_route), dev(cand_rows)  # alive until the kernel has run
    A.check(L.gofann_predicate_pass_masks(C.byref(gs), C.byref(at), C.byref(rs), A.ptr(d_route), A.ptr(d_rows), n,
                                          A.ptr(out), A.ptr(status), stream()), "predicate_pass_masks")
    torch.cuda.synchronize()
    assert int(status.item()) == expect_status
    return host(out, np.uint32)


@pytest.mark.parametrize("n", [1, 31, 32, 33, 5000, 100_003])
def test_predicate_pass_masks_bitexact(L, n):
    w, idx, plan, attrs, graph, dnf, legacy = _cfg1()
    rng = np.random.default_rng(n)
    nr = dnf["query_row"].shape[0]
    cr = rng.integers(0, nr, size=n).astype(np.uint32)
    grp = dnf["group_id"][cr]
    sizes = np.diff(np.append(graph["label_offset"], graph["adjacency"].shape[0]))
    rows = (rng.random(n) * sizes[grp]).astype(np.uint32)
    got = _masks(L, graph, attrs, dnf, cr, rows)
    sel = slice(0, min(n, 6000))  # the oracle loops in Python: check a prefix, then the popcount of the rest
    m = min(n, 6000)
    want = O.predicate_pass_masks(graph, attrs, dnf, cr[sel], rows[sel])
    full = m // 32
    assert np.array_equal(got[:full], want[:full])
    if m % 32 and n == m:
        assert got[full] == want[full]
    bits = np.unpackbits(got.view(np.uint8), bitorder="little")[:n]
    if n >= 5000:
        assert 0 < bits.sum() < n  # some pass, some fail


def test_predicate_pass_masks_rejects_bad_rows(L):
    w, idx, plan, attrs, graph, dnf, legacy = _cfg1()
    cr = np.array([0, 1, dnf["query_row"].shape[0] + 3], np.uint32)  # third route out of range
    rows = np.array([0, 1 << 30, 0], np.uint32)                     # second row out of range
    got = _masks(L, graph, attrs, dnf, cr, rows, expect_status=A.ERR_INVALID)
    assert got[0] & 0b110 == 0
