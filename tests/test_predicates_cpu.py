"""The oracle's predicate forms against a direct numpy statement of their
semantics, on the fixtures the GPU predicate tests use (no GPU).

DNF (gpu_predicate_index.cuh:100-136): a route passes a sample when some
clause holds, a clause holds when the sample carries every label atom and
satisfies every range atom; range modes (range_filter.cuh:28-45) 0 any, 1
v > lower, 2 v < upper, 3 lower <= v < upper.  The pass bitmap keeps
candidate order, 32 candidates per word, candidate i at bit i % 32.
"""
import numpy as np
import pytest

from fixtures import cfg1_small, with_predicates
from oracle import oracle as O


def _range_ok(mode, lo, hi, v):
    return {0: True, 1: v > lo, 2: v < hi, 3: lo <= v < hi}.get(int(mode), False)


def _dnf(routes, attrs, route, sample):
    ip, ind, vals = attrs["label_indptr"], attrs["label_indices"], attrs["range_values"]
    row = set(ind[ip[sample]:ip[sample + 1]].tolist())
    off = routes["pred_offsets"]
    for c in routes["clauses"][off[route]:off[route + 1]]:
        labs = routes["pred_handles"][c["label_begin"]:c["label_end"]]
        ok = all(int(x) in row for x in labs)
        for a in routes["pred_ranges"][c["range_begin"]:c["range_end"]]:
            ok = ok and _range_ok(a["mode"], a["lower"], a["upper"], vals[sample, a["dimension"]])
        if ok:
            return True
    return False


def test_oracle_dnf_and_pass_masks_match_semantics():
    w, idx, plan = cfg1_small(n=1500, n_queries=64)
    attrs, graph, dnf, legacy = with_predicates(w, idx, plan.graph_routes, seed=5)
    rng = np.random.default_rng(0)
    n = 2000
    nr = dnf["query_row"].shape[0]
    cr = rng.integers(0, nr, size=n).astype(np.uint32)
    grp = dnf["group_id"][cr]
    sizes = np.diff(np.append(graph["label_offset"], graph["adjacency"].shape[0]))
    rows = (rng.random(n) * sizes[grp]).astype(np.uint32)
    samples = graph["row_to_sample"][graph["label_offset"][grp] + rows]
    want = np.array([(not dnf["pred_enabled"][r]) or _dnf(dnf, attrs, r, s) for r, s in zip(cr, samples)], bool)
    assert 0 < want.sum() < n
    assert np.array_equal(O.pred_matches(dnf, attrs, cr, samples).astype(bool) | (dnf["pred_enabled"][cr] == 0),
                          want)
    masks = O.predicate_pass_masks(graph, attrs, dnf, cr, rows)
    bits = np.unpackbits(masks.view(np.uint8), bitorder="little")[:n].astype(bool)
    assert np.array_equal(bits, want)


@pytest.mark.parametrize("wl", ["cfg1", "cfg2"])
def test_native_planner_equals_python_planner(wl):
    """gofann_plan_categorical (host C++) builds the same route tables as
    planner.plan_queries: route split, seeds, posting slices, label lists,
    residual clauses and their enable flags."""
    from fixtures import cfg1_small, cfg2_small
    from gofann import planner
    w, idx, plan = cfg1_small() if wl == "cfg1" else cfg2_small()
    nat = planner.plan_queries_native(idx, w.query_labels)
    for a, b in ((plan.graph_routes, nat.graph_routes), (plan.posting_routes, nat.posting_routes)):
        assert sorted(a) == sorted(b)
        for k in a:
            assert np.array_equal(np.asarray(a[k]).view(np.uint8), np.asarray(b[k]).view(np.uint8)), k
    for k in ("graph_query", "posting_query", "posting_begin", "posting_count"):
        assert np.array_equal(getattr(plan, k), getattr(nat, k)), k


def test_native_planner_rejects_bad_labels():
    from fixtures import cfg2_small
    from gofann import _abi as A, planner
    w, idx, plan = cfg2_small()
    with pytest.raises(A.GofannError):
        planner.plan_queries_native(idx, [np.array([10 ** 7], np.uint32)])
    with pytest.raises(A.GofannError):
        planner.plan_queries_native(idx, [np.array([], np.uint32)])
