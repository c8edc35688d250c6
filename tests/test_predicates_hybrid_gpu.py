"""The config-4 predicate kinds on the GPU against the oracle: DNF clauses
whose atoms include exact strings, fuzzy strings (Levenshtein distance up to
max_edits, the device's bit-parallel check against the oracle's dynamic
programme) and int64 ranges, besides the labels
(tests/fixtures.with_hybrid_predicates).  Traversal results, posting-scan
shortlists (code and exact scorers) and pass bitmaps must be equal bit for
bit."""
import numpy as np
import pytest
import torch

from fixtures import cfg2_small, cfg2_small_u8cb, dev, fbits, with_hybrid_predicates
from gofann import _abi as A
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    assert torch.cuda.is_available()
    return A.lib()


@pytest.mark.parametrize("records", [False, True])
@pytest.mark.parametrize("bias", [1, 0])
def test_beam_search_hybrid_bitexact(L, records, bias):
    from test_gpu_parity import _with_records, run_gpu_beam
    w, idx, plan = cfg2_small_u8cb(48)
    attrs, routes = with_hybrid_predicates(w, idx, plan.graph_routes, seed=21)
    params = dict(queue_size=64, predicate_bias=bias, early_stop_mode=A.EARLY_STOP_ADAPTIVE, result_width=100,
                  pq_mode=A.PQ_U8, scorer=A.SCORER_PQ)
    lut = O.pq_build_lut(w.queries.astype(np.float32), idx.pq_centroids, idx.pq_codes.shape[1])
    want = O.beam_search(idx.graph(), attrs, idx.codes(), {"pq_lut": lut}, routes, threads=8, trace_width=64,
                         **params)
    graph = idx.graph()
    if records:
        graph, _ = _with_records(L, graph, attrs, idx.codes())
    prep = {"pq_query": dev(w.queries), "pq_centroids": dev(idx.pq_centroids)}
    got = run_gpu_beam(L, graph, attrs, idx.codes(), prep, routes, trace_width=64, **params)
    for name, g, o in zip(("ids", "dists", "steps", "counters", "trace"), got, want):
        if name == "dists":
            g, o = fbits(g), fbits(o)
        assert np.array_equal(g, o), name
    assert np.any((want[0] != A.U32MAX).sum(1) < params["result_width"])


@pytest.mark.parametrize("scorer", ["pq_lut", "exact"])
def test_posting_scan_hybrid_bitexact(L, scorer):
    import ctypes as C
    from fixtures import dev_dict, host
    from test_gpu_parity import run_gpu_posting
    w, idx, plan = cfg2_small()
    attrs, routes = with_hybrid_predicates(w, idx, plan.graph_routes, seed=23)
    n = routes["query_row"].shape[0]
    rng = np.random.default_rng(2)
    order = rng.permutation(w.n).astype(np.uint32)
    begin = rng.integers(0, w.n // 2, size=n).astype(np.uint64)
    count = rng.integers(500, w.n // 2, size=n).astype(np.uint32)
    k = 10
    if scorer == "pq_lut":
        lut = O.pq_build_lut(w.queries.astype(np.float32), idx.pq_centroids, idx.pq_codes.shape[1])
        want = O.posting_scan(idx.codes(), {"pq_lut": lut}, attrs, routes, A.SCORER_PQ, order, begin, count, k)
        got = run_gpu_posting(L, idx.codes(), {"pq_lut": dev(lut)}, attrs, routes, A.SCORER_PQ, order, begin, count,
                              k, pq_mode=A.PQ_LUT_GLOBAL)
        gi, gd = got[0], got[1]
    else:
        want = O.exact_posting_scan(w.base, A.DTYPE_U8, w.queries, attrs, routes, order, begin, count, k)
        dr, da = dev_dict(routes), dev_dict(attrs)
        rs, at = A.fill_routes(dr), A.fill_attrs(da)
        ids = torch.empty((n, k), dtype=torch.int32, device="cuda")
        d = torch.empty((n, k), dtype=torch.float32, device="cuda")
        db, dq, pid, pb, pc = dev(w.base), dev(w.queries), dev(order), dev(begin), dev(count)
        A.check(L.gofann_exact_posting_scan(A.ptr(db), A.DTYPE_U8, w.n, w.base.shape[1], A.ptr(dq), C.byref(at),
                                            C.byref(rs), A.ptr(pid), A.ptr(pb), A.ptr(pc), k, A.ptr(ids), A.ptr(d),
                                            torch.cuda.current_stream().cuda_stream), "exact_posting_scan")
        torch.cuda.synchronize()
        gi, gd = host(ids, np.uint32), d.cpu().numpy()
    assert np.array_equal(gi, want[0])
    assert np.array_equal(fbits(gd), fbits(want[1]))
    assert np.any((want[0] == A.U32MAX).any(1)) and np.any((want[0] != A.U32MAX).all(1))


def test_predicate_pass_masks_hybrid_bitexact(L):
    from test_predicates_gpu import _masks
    w, idx, plan = cfg2_small()
    attrs, routes = with_hybrid_predicates(w, idx, plan.graph_routes, seed=25)
    graph = idx.graph()
    rng = np.random.default_rng(5)
    n = 6000
    nr = routes["query_row"].shape[0]
    cr = rng.integers(0, nr, size=n).astype(np.uint32)
    sizes = np.diff(np.append(graph["label_offset"], graph["adjacency"].shape[0]))
    rows = (rng.random(n) * sizes[routes["group_id"][cr]]).astype(np.uint32)
    got = _masks(L, graph, attrs, routes, cr, rows)
    want = O.predicate_pass_masks(graph, attrs, routes, cr, rows)
    assert np.array_equal(got[: n // 32], want[: n // 32])
    bits = np.unpackbits(got.view(np.uint8), bitorder="little")[:n]
    assert 0 < bits.sum() < n
