"""The allocation-free traversal entry point against the allocating one.

gofann_beam_search_noalloc serves callers that cannot allocate device
memory (their host runtime owns the allocator, they run while a stream is
being captured, or they cannot afford an allocation on the serving path):
its scratch lives in a static device array inside the library.  Its results
must equal gofann_beam_search's exactly (traversal ids, distances, steps and
counters are bit-exact everywhere in this suite), on two calls in a row --
the second call finds the array holding the first call's state -- for the
PQ table mode (4-warp blocks), the integer-codebook mode (24-warp blocks,
capped at 42 blocks by the array's 1,024 tables) and the RaBitQ scorer.  A
batch of more routes than the array has visited tables checks the capped
grid.

This file sorts last so a run that stops at the first failure has already
run every other test; it also passes alone in a fresh process (the first
call performs the per-device set-up).
"""
import ctypes as C

import numpy as np
import pytest
import torch

from fixtures import cfg1_small, cfg2_small_u8cb, dev, dev_dict, fbits, rabitq_artifacts
from gofann import _abi as A
from gofann.planner import concat_routes
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _outputs(n, rw):
    t = dict(ids=torch.empty((n, rw), dtype=torch.int32, device="cuda"),
             d=torch.empty((n, rw), dtype=torch.float32, device="cuda"),
             steps=torch.empty(n, dtype=torch.int32, device="cuda"),
             cnt=torch.empty((n, 4), dtype=torch.int32, device="cuda"),
             status=torch.zeros(1, dtype=torch.int32, device="cuda"))
    s = A.SearchOut(ids=A.ptr(t["ids"]), dists=A.ptr(t["d"]), steps=A.ptr(t["steps"]), counters=A.ptr(t["cnt"]),
                    status=A.ptr(t["status"]))
    return t, s


def _host(t):
    return (t["ids"].cpu().numpy(), fbits(t["d"].cpu().numpy()), t["steps"].cpu().numpy(), t["cnt"].cpu().numpy(),
            int(t["status"].item()))


def _prepared(L, wl, w, idx, stream):
    """Device prepared state of a workload: the PQ table batch (cfg1, table
    mode), u8 query rows + integer codebook (cfg2 in GOFANN_PQ_U8), or the
    RaBitQ int8 queries, scales and centroid distances."""
    if wl == "cfg1":
        return {"pq_lut": dev(O.pq_build_lut(w.queries, idx.pq_centroids, idx.pq_codes.shape[1]))}
    if wl == "cfg2_u8":
        return {"pq_query": dev(w.queries), "pq_centroids": dev(idx.pq_centroids)}
    _, _, _, rq, anchors, qr = rabitq_artifacts()
    n, pd = qr.shape
    q8 = torch.empty((n, pd), dtype=torch.int8, device="cuda")
    sc = torch.empty(n, dtype=torch.float32, device="cuda")
    k1 = torch.empty(n, dtype=torch.float32, device="cuda")
    gd = torch.empty((n, anchors.shape[0]), dtype=torch.float32, device="cuda")
    dq, da = dev(qr), dev(anchors)
    A.check(L.gofann_rabitq_quantize(A.ptr(dq), n, pd, A.ptr(q8), A.ptr(sc), A.ptr(k1), stream), "quantize")
    A.check(L.gofann_rabitq_centroid_dist(A.ptr(dq), n, A.ptr(da), anchors.shape[0], pd, A.ptr(gd), stream), "gdist")
    torch.cuda.synchronize()
    return {"rq_q8": q8, "rq_scale": sc, "rq_k1xsumq": k1, "rq_centroid_dist": gd}


# (workload, scorer, PQ mode): the 4-warp table mode, the 24-warp integer
# codebook mode (42 blocks under the 1,024-table cap) and the RaBitQ scorer
WORKLOADS = [("cfg1", A.SCORER_PQ, A.PQ_LUT_GLOBAL), ("cfg2_u8", A.SCORER_PQ, A.PQ_U8),
             ("rabitq", A.SCORER_RABITQ, A.PQ_LUT_GLOBAL)]


@pytest.mark.parametrize("wl,scorer,mode", WORKLOADS)
@pytest.mark.parametrize("tile", [1, 12])
def test_noalloc_matches_allocating_entry_point(wl, scorer, mode, tile):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    L = A.lib()
    stream = torch.cuda.current_stream().cuda_stream
    if wl == "cfg1":
        w, idx, plan = cfg1_small()
        codes = idx.codes()
    elif wl == "cfg2_u8":
        w, idx, plan = cfg2_small_u8cb()
        codes = idx.codes()
    else:
        w, idx, plan, codes, _, _ = rabitq_artifacts()
    routes = plan.graph_routes
    for _ in range(tile - 1):  # tile=12: more routes than the 1,024 static visited tables
        routes = concat_routes(routes, plan.graph_routes)
    prep = _prepared(L, wl, w, idx, stream)
    dg, da, dc, dr = dev_dict(idx.graph()), dev_dict(idx.attrs()), dev_dict(codes), dev_dict(routes)
    gs, at, cs, ps, rs = A.fill_graph(dg), A.fill_attrs(da), A.fill_codes(dc), A.fill_prepared(prep), A.fill_routes(dr)
    sp = A.fill_params(queue_size=64, predicate_bias=1, early_stop_mode=A.EARLY_STOP_ADAPTIVE, result_width=100,
                       scorer=scorer, pq_mode=mode)
    n = rs.n_routes

    want_t, want_s = _outputs(n, 100)
    nbytes = L.gofann_beam_search_scratch_bytes(n)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    A.check(L.gofann_beam_search(C.byref(gs), C.byref(at), C.byref(cs), C.byref(ps), C.byref(rs), C.byref(sp),
                                 C.byref(want_s), A.ptr(scratch), nbytes, stream), "gofann_beam_search")
    torch.cuda.synchronize()
    want = _host(want_t)
    assert want[4] == 0

    for call in range(2):
        got_t, got_s = _outputs(n, 100)
        A.check(L.gofann_beam_search_noalloc(C.byref(gs), C.byref(at), C.byref(cs), C.byref(ps), C.byref(rs),
                                             C.byref(sp), C.byref(got_s), stream), "gofann_beam_search_noalloc")
        torch.cuda.synchronize()
        got = _host(got_t)
        for name, g, o in zip(("ids", "dists", "steps", "counters", "status"), got, want):
            assert np.array_equal(g, o), f"call {call}: {name} differ"
