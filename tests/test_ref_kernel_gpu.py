"""The reference's own device traversal against the oracle and this library.

oracle/_ref/libgofann_ref_kernels.so is the reference's PQ search backend
(src/search/pq/backend_pq.cu) compiled in place for sm_100a; its
device-resident kernel runs here on the seeded cases of
tests/ref_kernel_cases.py.  Every output it produces must equal the CPU
oracle's and this library's bit for bit: the per-route PQ table its kernel
builds (computePQTable, backend_pq.cu:1999-2022) against the oracle's
table, and the traversal's shortlist ids, float distances, step counts and
expansion order against the oracle's restatement and against
gofann_beam_search in every PQ scoring mode the case admits.  The cases with
an integer codebook make equal distances common, so the heap layouts and the
cooperative pickup's tie rule decide the ids.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from fixtures import dev, dev_dict, fbits, host
from gofann import _abi as A
from oracle import oracle as O
from oracle import ref_kernels as RK
import ref_kernel_cases as R

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if not RK.available():
        pytest.skip("oracle/_ref/libgofann_ref_kernels.so not built (needs the reference tree at build time)")
    return A.lib()


def run_library(L, case, mode, lut):
    p = case["params"]
    dg, da, dc, dr = (dev_dict(case["graph"]), dev_dict(case["attrs"]), dev_dict(case["codes"]),
                      dev_dict(case["routes"]))
    if mode == A.PQ_LUT_GLOBAL:
        prep = {"pq_lut": dev(lut)}
    else:
        prep = {"pq_query": dev(case["queries"]), "pq_centroids": dev(case["centroids"])}
    gs, at, cs, ps, rs = A.fill_graph(dg), A.fill_attrs(da), A.fill_codes(dc), A.fill_prepared(prep), A.fill_routes(dr)
    sp = A.fill_params(scorer=A.SCORER_PQ, pq_mode=mode, **p)
    n, rw = rs.n_routes, sp.result_width
    ids = torch.empty((n, rw), dtype=torch.int32, device="cuda")
    d = torch.empty((n, rw), dtype=torch.float32, device="cuda")
    steps = torch.empty(n, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    trace = torch.empty((n, 64), dtype=torch.int32, device="cuda")
    out = A.SearchOut(ids=A.ptr(ids), dists=A.ptr(d), steps=A.ptr(steps), status=A.ptr(status), trace=A.ptr(trace),
                      trace_width=64)
    nbytes = L.gofann_beam_search_scratch_bytes(n)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    A.check(L.gofann_beam_search(C.byref(gs), C.byref(at), C.byref(cs), C.byref(ps), C.byref(rs), C.byref(sp),
                                 C.byref(out), A.ptr(scratch), nbytes, torch.cuda.current_stream().cuda_stream),
            "gofann_beam_search")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return {"ids": host(ids, np.uint32), "dists": d.cpu().numpy(), "steps": steps.cpu().numpy(),
            "trace": host(trace, np.uint32)}


def assert_same(name, got, want):
    for k in ("ids", "dists", "steps", "trace"):
        g, w = got[k], want[k]
        if k == "dists":
            g, w = fbits(g), fbits(w)
        bad = np.nonzero(np.any(np.atleast_2d(g != w), axis=-1) if g.ndim > 1 else g != w)[0]
        assert bad.size == 0, f"{name}: {k} differ in {bad.size} routes (first {bad[:5].tolist()})"


@pytest.mark.parametrize("name", R.CASE_NAMES)
def test_reference_kernel_matches_oracle_and_library(L, name):
    case = R.build_case(name)
    ref = RK.run_reference_pq(case, trace_width=64)
    pq_dim = case["codes"]["pq_codes"].shape[1]
    lut = O.pq_build_lut(case["queries"].astype(np.float32), case["centroids"], pq_dim)
    assert np.array_equal(fbits(ref["pq_table"]), fbits(lut)), "reference computePQTable != oracle table"
    want = O.beam_search(case["graph"], case["attrs"], case["codes"], {"pq_lut": lut}, case["routes"], threads=8,
                         trace_width=64, scorer=A.SCORER_PQ, **case["params"])
    ora = dict(zip(("ids", "dists", "steps", "counters", "trace"), want))
    assert_same(f"{name} reference vs oracle", ref, ora)
    modes = [A.PQ_LUT_GLOBAL, A.PQ_DIRECT]
    if R.case_params(name)["int_codebook"] and (case["queries"].shape[1] // pq_dim) % 4 == 0:
        modes.append(A.PQ_U8)
    for mode in modes:
        assert_same(f"{name} library mode {mode} vs reference", run_library(L, case, mode, lut), ref)
