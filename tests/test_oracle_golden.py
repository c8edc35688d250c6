"""The CPU oracle replays every golden case produced by the reference's own
headers (tests/golden/make_golden.py) and must agree bit for bit."""
import numpy as np
import pytest

from oracle import oracle as O
from gofann import _abi as A

G = np.load(Path := __import__("pathlib").Path(__file__).resolve().parent / "golden" / "reference_structures.npz")


def bits(x):
    return np.asarray(x, np.float32).view(np.uint32)


@pytest.mark.parametrize("case", range(12))
def test_smmh_sequences(case):
    f, s, popped = O.seq_smmh(G[f"smmh{case}_op"], G[f"smmh{case}_key"], G[f"smmh{case}_payload"])
    assert np.array_equal(bits(f), bits(G[f"smmh{case}_first"]))
    assert np.array_equal(s, G[f"smmh{case}_second"])
    assert np.array_equal(popped, G[f"smmh{case}_popped"])


@pytest.mark.parametrize("case", range(8))
def test_result_heap_sequences(case):
    f, s = O.seq_result_heap(G[f"rheap{case}_key"], G[f"rheap{case}_payload"], int(G[f"rheap{case}_cap"]))
    assert np.array_equal(bits(f), bits(G[f"rheap{case}_first"]))
    assert np.array_equal(s, G[f"rheap{case}_second"])


@pytest.mark.parametrize("case", range(3))
def test_visited_hash(case):
    table, outcome = O.seq_hash(G[f"hash{case}_values"])
    assert np.array_equal(table, G[f"hash{case}_table"])
    assert np.array_equal((outcome == 1).astype(np.int32), G[f"hash{case}_found_before"])


@pytest.mark.parametrize("case", range(8))
@pytest.mark.parametrize("srt", [0, 1])
def test_shortlist_heap(case, srt):
    od, oi = O.shortlist(G[f"sl{case}_in_d"], G[f"sl{case}_in_i"], int(G[f"sl{case}_k"]), sort=bool(srt))
    assert np.array_equal(bits(od), bits(G[f"sl{case}_{srt}_d"]))
    assert np.array_equal(oi, G[f"sl{case}_{srt}_i"])


def test_dnf_predicate():
    ranges = np.zeros(G["pred_ranges"].shape[0], A.RANGE_ATOM_DTYPE)
    r = G["pred_ranges"]
    ranges["dimension"], ranges["mode"] = r[:, 0], r[:, 1]
    ranges["lower"], ranges["upper"] = r[:, 2].view(np.float32), r[:, 3].view(np.float32)
    clauses = np.zeros(G["pred_clauses"].shape[0], A.CLAUSE_DTYPE)
    c = G["pred_clauses"]
    for i, f in enumerate(("label_begin", "label_end", "range_begin", "range_end")):
        clauses[f] = c[:, i]
    routes = {"query_row": np.zeros(len(G["pred_route_off"]) - 1, np.uint32), "pred_offsets": G["pred_route_off"],
              "clauses": clauses, "pred_handles": G["pred_handles"], "pred_ranges": ranges}
    attrs = {"label_indptr": G["pred_csr_off"].astype(np.uint64), "label_indices": G["pred_csr_lab"],
             "range_values": G["pred_base_ranges"]}
    got = O.pred_matches(routes, attrs, G["pred_qr"], G["pred_qs"])
    assert np.array_equal(got, G["pred_out"])


@pytest.mark.parametrize("case", range(3))
def test_predicate_priority(case):
    from oracle.oracle import olib
    import ctypes as C
    L = olib()
    # the oracle's priority is exercised through its static helper via the
    # traversal; here it is restated with numpy float32 arithmetic
    base, passv, pen = G["prio_base"], G["prio_pass"], np.float32(G[f"prio{case}_pen"])
    out = base.copy()
    with np.errstate(all="ignore"):
        for i in range(base.shape[0]):
            b = base[i]
            if passv[i] or pen == 0 or not np.isfinite(b) or b == np.finfo(np.float32).max:
                out[i] = b
            elif b > np.float32(np.finfo(np.float32).max - pen):
                out[i] = np.finfo(np.float32).max
            else:
                out[i] = np.float32(b + pen)
    assert np.array_equal(bits(out), bits(G[f"prio{case}_out"]))


@pytest.mark.parametrize("case", range(7))
def test_route_merge(case):
    r2q = G[f"rm{case}_r2q"].astype(np.int64)
    n_q = G[f"rm{case}_oi"].shape[0]
    order = np.argsort(r2q, kind="stable").astype(np.uint32)
    qoff = np.zeros(n_q + 1, np.uint32)
    qoff[1:] = np.cumsum(np.bincount(r2q, minlength=n_q))
    oi, od = O.route_merge(G[f"rm{case}_ids"], G[f"rm{case}_d"], qoff, order, 10)
    assert np.array_equal(oi, G[f"rm{case}_oi"])
    assert np.array_equal(bits(od), bits(G[f"rm{case}_od"]))


def test_fp16_decode_and_l2():
    import ctypes as C
    from oracle.oracle import olib
    h = G["f16_bits"]
    # the oracle's f16 decode is reached through exact_l2 against a zero query
    base = h.reshape(-1, 1).astype(np.uint16)
    L = olib()
    L.oracle_exact_l2.argtypes = [C.c_void_p, C.c_int, C.c_uint32, C.c_uint32, C.c_void_p, C.c_uint32]
    L.oracle_exact_l2.restype = C.c_float
    q = np.zeros(1, np.float32)
    dec = G["f16_decoded"]
    for i in range(0, h.shape[0], 97):
        got = L.oracle_exact_l2(O.P(base), A.DTYPE_F16, 1, i, O.P(q), 0)
        want = np.float32(dec[i]) * np.float32(dec[i]) if np.isfinite(dec[i]) else np.float32(np.inf)
        if np.isnan(dec[i]):
            assert np.isnan(got)
        else:
            assert bits(got) == bits(np.float32(0.0) + want) or (np.isinf(want) and np.isinf(got))
    rows = G["f16_rows"]
    for r in range(rows.shape[0]):
        got = L.oracle_exact_l2(O.P(rows), A.DTYPE_F16, rows.shape[1], r, O.P(G["f16_query"]), 0)
        # reference scalar loop accumulates without fma: relative 1e-6 agreement
        assert abs(got - G["f16_l2"][r]) <= 1e-5 * max(1.0, abs(G["f16_l2"][r]))


# ------------------------------------------------ reference device traversal
# tests/golden/reference_pq_kernel.npz holds the outputs of the reference's
# own device-resident PQ traversal (backend_pq.cu compiled in place for
# sm_100a, run on a B200 by tests/golden/make_ref_kernel_golden.py) on the
# numpy-built cases of tests/ref_kernel_cases.py.  The oracle's traversal
# restatement must reproduce every one of them bit for bit, and its PQ table
# must hash to the table the reference kernel built.
import hashlib  # noqa: E402

import ref_kernel_cases as RC  # noqa: E402

_KG = Path.parent / "reference_pq_kernel.npz"  # Path: tests/golden/reference_structures.npz


@pytest.mark.skipif(not _KG.exists(), reason="reference kernel golden vectors not recorded yet")
@pytest.mark.parametrize("name", RC.CASE_NAMES)
def test_oracle_replays_reference_kernel(name):
    K = np.load(_KG)
    case = RC.build_case(name)
    assert RC.case_digest(case) == bytes(K[f"{name}/digest"]).hex(), "case generator drifted from the recording"
    pq_dim = case["codes"]["pq_codes"].shape[1]
    lut = O.pq_build_lut(case["queries"].astype(np.float32), case["centroids"], pq_dim)
    assert hashlib.sha256(np.ascontiguousarray(lut, np.float32).tobytes()).digest() == bytes(K[f"{name}/table_sha256"])
    ids, d, steps, _, trace = O.beam_search(case["graph"], case["attrs"], case["codes"], {"pq_lut": lut},
                                            case["routes"], threads=8, trace_width=64, scorer=A.SCORER_PQ,
                                            **case["params"])
    assert np.array_equal(ids, K[f"{name}/ids"])
    assert np.array_equal(bits(d), K[f"{name}/dist_bits"])
    assert np.array_equal(steps, K[f"{name}/steps"])
    assert np.array_equal(trace, K[f"{name}/trace"])


@pytest.mark.skipif(not _KG.exists(), reason="reference kernel golden vectors not recorded yet")
def test_oracle_pickup_matches_reference_device_pickup():
    """The reference's cooperative pickup, run on a B200 on 600 frontiers of
    2..520 entries with keys from six values (many ties) and 30 % of the
    entries used: the oracle picks the same entry every time."""
    K = np.load(_KG)
    keys, used, sizes, picked = K["pickup/keys"], K["pickup/used"], K["pickup/sizes"], K["pickup/picked"]
    vals = (np.arange(keys.shape[1], dtype=np.uint32)[None, :] | (used.astype(np.uint32) << 31)).astype(np.uint32)
    got = np.array([O.pickup_index(keys[c], vals[c], int(sizes[c])) for c in range(keys.shape[0])])
    assert np.array_equal(got, picked)


@pytest.mark.skipif(not _KG.exists(), reason="reference kernel golden vectors not recorded yet")
@pytest.mark.parametrize("cap", [1, 10, 33, 100, 200])
def test_oracle_result_heap_matches_reference_device_heap(cap):
    """The reference's binary result heap on the device (push / pop of
    bin_heap.h, then emptied into ascending slots) against the oracle's."""
    K = np.load(_KG)
    hk, f, p = K[f"rheap{cap}/keys"], K[f"rheap{cap}/first"], K[f"rheap{cap}/payload"]
    for c in range(hk.shape[0]):
        of, op = O.seq_result_heap(hk[c], np.arange(hk.shape[1], dtype=np.uint32), cap)
        assert np.array_equal(bits(of[:cap][::-1]), bits(f[c])) and np.array_equal(op[:cap][::-1], p[c])


# ---- the reference's Full-GPU kernels, recorded on a B200
# (tests/golden/make_ref_full_gpu_golden.py over tests/ref_full_cases.py)
FG = np.load(Path.parent / "reference_full_gpu.npz")


def _full_cases():
    import ref_full_cases as R
    return R


@pytest.mark.parametrize("name", _full_cases().CASE_NAMES)
def test_oracle_replays_reference_full_gpu_kernel(name):
    """Exact-distance traversal: ids, distance bits and step counts of the
    reference's full_gpu_highfreq_kernel on u8 / f32 / f16 cases with many
    distance ties, filter bits, row masks and range modes."""
    R = _full_cases()
    c = R.build_case(name)
    assert bytes(FG[f"{name}/digest"]).hex() == R.case_digest(c), "case inputs drifted from the golden file"
    ids, d, steps = O.exact_search(c["graph"], c["attrs"], c["base"], c["dtype"], c["queries"], c["routes"],
                                   threads=4, **c["params"])
    assert np.array_equal(ids, FG[f"{name}/ids"])
    assert np.array_equal(bits(d), FG[f"{name}/dist_bits"])
    assert np.array_equal(steps, FG[f"{name}/steps"])


@pytest.mark.parametrize("name", _full_cases().LOW_NAMES)
def test_oracle_replays_reference_full_gpu_posting_kernel(name):
    R = _full_cases()
    c = R.build_low_case(name)
    assert bytes(FG[f"{name}/digest"]).hex() == R.case_digest(c)
    ids, d = O.exact_posting_scan(c["base"], c["dtype"], c["queries"], c["attrs"], c["routes"], c["posting_ids"],
                                  c["begin"], c["count"], c["topk"])
    assert np.array_equal(ids, FG[f"{name}/ids"])
    assert np.array_equal(bits(d), FG[f"{name}/dist_bits"])


def test_oracle_full_pickup_matches_reference_block_pickup():
    """The block pickup's choice (smallest distance, then smallest index) on
    600 tie-heavy frontiers."""
    keys, used, sizes = FG["pickup/keys"], FG["pickup/used"], FG["pickup/sizes"]
    vals = np.arange(keys.shape[1], dtype=np.uint32)[None, :] | (used.astype(np.uint32) << 31)
    mine = np.array([O.full_pickup_index(keys[c], vals[c], int(sizes[c])) for c in range(keys.shape[0])])
    assert np.array_equal(mine, FG["pickup/picked"])


# ---- the reference's 1-bit RaBitQ estimator, recorded on a B200
# (tests/golden/make_ref_rabitq_golden.py over tests/ref_rabitq_cases.py)
RQ = np.load(Path.parent / "reference_rabitq_score.npz")


@pytest.mark.parametrize("pd", (128, 512, 4096))
def test_oracle_replays_reference_rabitq_estimator(pd):
    """The oracle's combine order, fma(f_rescale, fma(ip, scale, k1xsumq),
    f_add + gdist), gives the reference kernel's estimate bits on 6,000
    pairs per padded dim."""
    import ref_rabitq_cases as R
    c = R.build_case(pd)
    assert bytes(RQ[f"pd{pd}/digest"]).hex() == R.case_digest(c)
    est, _ = O.rabitq_score(R.codes_dict(c), R.prep_dict(c), c["pair_row"], c["pair_point"])
    assert np.array_equal(bits(est), RQ[f"pd{pd}/est_bits"])
