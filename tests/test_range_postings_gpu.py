"""Segmented slice scans on the GPU: gofann_posting_scan over the segments of
a make_plan split, then gofann_segment_merge, must return what one scan of
each whole slice returns (and the oracle), bit for bit -- RaBitQ and PQ_U8,
under OR-ed DNF predicates with range atoms, slices of 0 to 6,000 rows."""
import ctypes as C

import numpy as np
import pytest
import torch

from fixtures import cfg2_small_u8cb, dev, fbits, host, rabitq_artifacts, with_predicates
from gofann import _abi as A
from gofann import range_postings as RP
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return A.lib()


def repeat_routes(r: dict, sel: np.ndarray) -> dict:
    """Route tables of the routes `sel` (repeats allowed), predicate CSRs re-based."""
    out = {}
    for k in ("query_row", "group_id", "start_local", "primary_label", "pred_enabled", "filter_bits",
              "route_compiled", "range_modes", "range_lower", "range_upper"):
        if r.get(k) is not None:
            out[k] = np.ascontiguousarray(r[k][sel])
    ip, ind = r["qlabel_indptr"], r["qlabel_indices"]
    rows = [ind[ip[i]:ip[i + 1]] for i in sel]
    out["qlabel_indptr"] = np.concatenate([[0], np.cumsum([len(x) for x in rows])]).astype(np.uint64)
    out["qlabel_indices"] = (np.concatenate(rows) if rows else np.zeros(0)).astype(np.uint32)
    if r.get("pred_offsets") is not None:
        off = r["pred_offsets"]
        cl = [r["clauses"][off[i]:off[i + 1]] for i in sel]
        out["pred_offsets"] = np.concatenate([[0], np.cumsum([len(x) for x in cl])]).astype(np.uint32)
        out["clauses"] = np.concatenate(cl)
        out["pred_handles"], out["pred_ranges"] = r["pred_handles"], r["pred_ranges"]
    return out


@pytest.mark.parametrize("scorer,target", [("rabitq", 700), ("rabitq", 2048), ("pq_u8", 333)])
def test_segmented_scan_and_merge_equal_one_scan(L, scorer, target):
    from test_gpu_parity import _rq_prepared, run_gpu_posting
    if scorer == "rabitq":
        w, idx, plan, codes, anchors, qr = rabitq_artifacts(dim=992, n_queries=64)
        dprep, hprep = _rq_prepared(L, qr, anchors)
        sc, mode = A.SCORER_RABITQ, A.PQ_LUT_GLOBAL
    else:
        w, idx, plan = cfg2_small_u8cb(48)
        codes = idx.codes()
        hprep = {"pq_lut": O.pq_build_lut(w.queries.astype(np.float32), idx.pq_centroids, 48)}
        dprep = {"pq_query": dev(w.queries), "pq_centroids": dev(idx.pq_centroids)}
        sc, mode = A.SCORER_PQ, A.PQ_U8
    attrs, graph, dnf, _ = with_predicates(w, idx, plan.graph_routes, seed=23)
    n = dnf["query_row"].shape[0]
    rng = np.random.default_rng(target)
    order = rng.permutation(w.n).astype(np.uint32)
    lo = rng.integers(0, w.n // 2, size=n).astype(np.uint64)
    cnt = rng.integers(0, min(6000, w.n // 2), size=n).astype(np.uint64)
    cnt[0] = 0
    k = 100
    want = O.posting_scan(codes, hprep, attrs, dnf, sc, order, lo, cnt.astype(np.uint32), k)
    whole = run_gpu_posting(L, codes, dprep, attrs, dnf, sc, order, lo, cnt.astype(np.uint32), k, pq_mode=mode)
    sp = RP.make_plan(np.arange(n), lo, cnt, target)
    segs = repeat_routes(dnf, sp.query_positions.astype(np.int64))
    seg_i, seg_d = run_gpu_posting(L, codes, dprep, attrs, segs, sc, order, sp.offsets, sp.sizes.astype(np.uint32), k,
                                   pq_mode=mode)
    d_ind, d_si, d_sd = dev(sp.query_indptr), dev(seg_i), dev(seg_d)
    out_i = torch.empty((n, k), dtype=torch.int32, device="cuda")
    out_d = torch.empty((n, k), dtype=torch.float32, device="cuda")
    A.check(L.gofann_segment_merge(A.ptr(d_ind), n, A.ptr(d_si), A.ptr(d_sd), k, A.ptr(out_i), A.ptr(out_d),
                                   torch.cuda.current_stream().cuda_stream), "segment_merge")
    torch.cuda.synchronize()
    gi, gd = host(out_i, np.uint32), out_d.cpu().numpy()
    assert sp.route_ids.shape[0] > n  # slices really were split
    assert np.array_equal(gi, want[0]) and np.array_equal(fbits(gd), fbits(want[1]))
    assert np.array_equal(gi, whole[0]) and np.array_equal(fbits(gd), fbits(whole[1]))
