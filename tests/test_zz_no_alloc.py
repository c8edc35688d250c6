"""The allocation-free traversal entry point against the allocating one.

gofann_beam_search_noalloc serves callers that cannot allocate device
memory (their host runtime owns the allocator, they run while a stream is
being captured, or they cannot afford an allocation on the serving path):
its scratch lives in a static device array inside the library.  Its results
must equal gofann_beam_search's exactly (traversal ids, distances, steps and
counters are bit-exact everywhere in this suite), on two calls in a row --
the second call finds the array holding the first call's state.  A batch of
more routes than the array has visited tables checks the capped grid.

This file sorts last so a run that stops at the first failure has already
run every other test; it also passes alone in a fresh process (the first
call performs the per-device set-up).
"""
import ctypes as C

import numpy as np
import pytest
import torch

from fixtures import cfg1_small, dev, dev_dict, fbits
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


@pytest.mark.parametrize("tile", [1, 12])
def test_noalloc_matches_allocating_entry_point(tile):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    L = A.lib()
    w, idx, plan = cfg1_small()
    routes = plan.graph_routes
    for _ in range(tile - 1):  # tile=12: more routes than the 1,024 static visited tables
        routes = concat_routes(routes, plan.graph_routes)
    lut = dev(O.pq_build_lut(w.queries, idx.pq_centroids, idx.pq_codes.shape[1]))
    dg, da, dc, dr = dev_dict(idx.graph()), dev_dict(idx.attrs()), dev_dict(idx.codes()), dev_dict(routes)
    prep = {"pq_lut": lut}
    gs, at, cs, ps, rs = A.fill_graph(dg), A.fill_attrs(da), A.fill_codes(dc), A.fill_prepared(prep), A.fill_routes(dr)
    sp = A.fill_params(queue_size=64, predicate_bias=1, early_stop_mode=A.EARLY_STOP_ADAPTIVE, result_width=100,
                       pq_mode=A.PQ_LUT_GLOBAL)
    n = rs.n_routes
    stream = torch.cuda.current_stream().cuda_stream

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
