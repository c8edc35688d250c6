"""bench.py's CPU legs run without a GPU.

The config-2 CPU baseline (host_index + cpu_search: the oracle restatement
of LUT build, traversal, posting scans, u8 rerank and merge over a query
sample) is the part of the default bench run that executes on host cores;
it runs here on a small config-2 shaped index and must give the same merged
top-10 as the oracle pipeline run on all queries, row for row.
"""
import sys
from pathlib import Path

import numpy as np

from fixtures import cfg2_small
from gofann import _abi as A
from oracle import oracle as O

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402


def test_cpu_search_sample_matches_full_oracle_pipeline():
    w, idx, plan = cfg2_small()
    hidx = bench.host_index(idx)
    sel = np.arange(0, w.queries.shape[0], 3)
    res = bench.cpu_search(hidx, plan, w.queries, sel, 64, 2)
    lut = O.pq_build_lut(w.queries.astype(np.float32), idx.pq_centroids, idx.pq_codes.shape[1])
    bi, _, _, _ = O.beam_search(idx.graph(), idx.attrs(), idx.codes(), {"pq_lut": lut}, plan.graph_routes, threads=2,
                                queue_size=64, result_width=100, predicate_bias=1, alpha=0.15,
                                early_stop_mode=A.EARLY_STOP_ADAPTIVE)
    ri, rd = O.rerank(w.base, A.DTYPE_U8, w.queries, idx.attrs(), plan.graph_routes, bi, 10)
    pi, _ = O.posting_scan(idx.codes(), {"pq_lut": lut}, idx.attrs(), plan.posting_routes, A.SCORER_PQ,
                           idx.posting_ids, plan.posting_begin, plan.posting_count, 100)
    rpi, rpd = O.rerank(w.base, A.DTYPE_U8, w.queries, idx.attrs(), plan.posting_routes, pi, 10)
    qoff, order = plan.merge_tables()
    wi, wd = O.route_merge(np.concatenate([ri, rpi]), np.concatenate([rd, rpd]), qoff, order, 10)
    assert np.array_equal(res["final_ids"], wi[sel])
    assert np.array_equal(res["final_d"].view(np.uint32), wd[sel].view(np.uint32))


def test_route_order_by_work_keeps_results():
    """Graph routes reordered longest-expected first (planner.order_by_work):
    the CPU path gives the same merged top-10 per query as in plan order."""
    from gofann import planner
    w, idx, plan = cfg2_small()
    hidx = bench.host_index(idx)
    sel = np.arange(w.queries.shape[0])
    a = bench.cpu_search(hidx, plan, w.queries, sel, 64, 2)
    b = bench.cpu_search(hidx, planner.order_by_work(plan, idx), w.queries, sel, 64, 2)
    assert np.array_equal(a["final_ids"], b["final_ids"])
    assert np.array_equal(a["final_d"].view(np.uint32), b["final_d"].view(np.uint32))


def test_profiled_traffic_record_is_consistent():
    """roofline.traffic of the config-2 line scales the committed capture's
    DRAM-bytes-per-algorithmic-byte ratio; the ratio must match the bytes it
    was computed from, and a launch moves at least its algorithmic bytes."""
    t = bench.profiled_traffic()
    assert t is not None and t["kernel"] == "beam_search_kernel"
    ratio = t["dram_bytes"] / t["algorithmic_bytes"]
    assert abs(ratio - t["traffic_per_algorithmic_byte"]) < 5e-4
    assert ratio >= 1.0
