"""GPU parity: every CUDA stage against the CPU oracle on the same seeded
inputs, called through the C ABI (libgofann_b200.so).

Bit-exact: PQ LUT / ADC / codes, RaBitQ int8 query, scale, k1xsumq, integer
inner products and estimates, traversal ids + distances + steps + counters,
posting shortlists, uint8 rerank, merges.  Tolerance: f32 rerank 1e-5
relative, f16 rerank 1e-3 relative (ids compared up to ties within that
tolerance), centroid distances 1e-3 + 2e-5 x against FP64
(rabitq_query_rotation_test.cu:48-50).
"""
import ctypes as C

import numpy as np
import pytest
import torch

from fixtures import cfg1_small, cfg2_small, cfg2_small_u8cb, dev, dev_dict, fbits, host, rabitq_artifacts
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


_KEEP = []


def dptr(a):
    """Device copy of a numpy array, kept alive until the test module ends."""
    t = dev(a)
    _KEEP.append(t)
    return A.ptr(t)


@pytest.fixture(autouse=True)
def _release():
    yield
    torch.cuda.synchronize()
    _KEEP.clear()


# ------------------------------------------------------------------ PQ stages
@pytest.mark.parametrize("dim,pq_dim,qdtype", [(128, 32, "f32"), (192, 48, "u8"), (96, 16, "f32"), (64, 64, "u8"),
                                               (256, 128, "f32")])
def test_pq_lut_bitexact(L, dim, pq_dim, qdtype):
    rng = np.random.default_rng(dim + pq_dim)
    n = 37
    if qdtype == "u8":
        q = rng.integers(0, 256, size=(n, dim)).astype(np.uint8)
        cent = rng.uniform(0, 255, size=(256, dim)).astype(np.float32)
    else:
        q = rng.standard_normal((n, dim)).astype(np.float32)
        cent = rng.standard_normal((256, dim)).astype(np.float32)
    want = O.pq_build_lut(q.astype(np.float32), cent, pq_dim)
    lut = torch.empty((n, pq_dim, 256), dtype=torch.float32, device="cuda")
    A.check(L.gofann_pq_build_lut(dptr((q)), A.DTYPE_U8 if qdtype == "u8" else A.DTYPE_F32, n, dim,
                                  dptr((cent)), pq_dim, A.ptr(lut), stream()), "lut")
    torch.cuda.synchronize()
    assert np.array_equal(fbits(lut.cpu().numpy()), fbits(want))


@pytest.mark.parametrize("pq_dim", [16, 24, 32, 48, 64, 96, 128])
def test_pq_adc_bitexact(L, pq_dim):
    rng = np.random.default_rng(pq_dim)
    n_rows, n_samples, n_pairs = 11, 500, 4000
    lut = rng.uniform(0, 100, size=(n_rows, pq_dim, 256)).astype(np.float32)
    codes = rng.integers(0, 256, size=(n_samples, pq_dim)).astype(np.uint8)
    pr = rng.integers(0, n_rows, size=n_pairs).astype(np.uint32)
    ps = rng.integers(0, n_samples, size=n_pairs).astype(np.uint32)
    want = O.pq_adc(lut, codes, pr, ps)
    out = torch.empty(n_pairs, dtype=torch.float32, device="cuda")
    A.check(L.gofann_pq_adc(dptr((lut)), pq_dim, dptr((codes)), dptr((pr)), dptr((ps)), n_pairs,
                            A.ptr(out), stream()), "adc")
    assert np.array_equal(fbits(out.cpu().numpy()), fbits(want))


@pytest.mark.parametrize("dim,pq_dim,dtype", [(128, 32, "f32"), (192, 48, "u8")])
def test_pq_encode_bitexact(L, dim, pq_dim, dtype):
    rng = np.random.default_rng(7)
    n = 3000
    x = (rng.integers(0, 256, size=(n, dim)).astype(np.uint8) if dtype == "u8"
         else rng.standard_normal((n, dim)).astype(np.float32))
    cent = x[rng.choice(n, 256, replace=False)].astype(np.float32)
    want = O.pq_encode(x.astype(np.float32), cent, pq_dim)
    out = torch.empty((n, pq_dim), dtype=torch.uint8, device="cuda")
    A.check(L.gofann_pq_encode(dptr((x)), A.DTYPE_U8 if dtype == "u8" else A.DTYPE_F32, n, dim,
                               dptr((cent)), pq_dim, A.ptr(out), stream()), "encode")
    assert np.array_equal(out.cpu().numpy(), want)


# -------------------------------------------------------------- RaBitQ
@pytest.mark.parametrize("pd", [64, 512, 4096])
def test_rabitq_quantize_bitexact(L, pd):
    rng = np.random.default_rng(pd)
    n = 29
    r = rng.standard_normal((n, pd)).astype(np.float32)
    r[3] = 0.0  # zero query -> scale 1
    r[4, :5] = [127.5, -127.5, 0.5, -0.5, 1.5]
    q8, scale, k1 = O.rabitq_quantize(r)
    gq8 = torch.empty((n, pd), dtype=torch.int8, device="cuda")
    gs = torch.empty(n, dtype=torch.float32, device="cuda")
    gk = torch.empty(n, dtype=torch.float32, device="cuda")
    A.check(L.gofann_rabitq_quantize(dptr((r)), n, pd, A.ptr(gq8), A.ptr(gs), A.ptr(gk), stream()), "quantize")
    assert np.array_equal(gq8.cpu().numpy(), q8)
    assert np.array_equal(fbits(gs.cpu().numpy()), fbits(scale))
    assert np.array_equal(fbits(gk.cpu().numpy()), fbits(k1))


def test_rabitq_centroid_dist_tolerance(L):
    rng = np.random.default_rng(5)
    n, a, pd = 17, 33, 512
    q = rng.standard_normal((n, pd)).astype(np.float32)
    c = rng.standard_normal((a, pd)).astype(np.float32)
    want = ((q[:, None, :].astype(np.float64) - c[None].astype(np.float64)) ** 2).sum(-1)
    out = torch.empty((n, a), dtype=torch.float32, device="cuda")
    A.check(L.gofann_rabitq_centroid_dist(dptr((q)), n, dptr((c)), a, pd, A.ptr(out), stream()), "gdist")
    got = out.cpu().numpy().astype(np.float64)
    assert np.all(np.abs(got - want) <= 1e-3 + 2e-5 * np.abs(want))


def _rq_prepared(L, qr, anchors):
    n, pd = qr.shape
    gq8 = torch.empty((n, pd), dtype=torch.int8, device="cuda")
    gs = torch.empty(n, dtype=torch.float32, device="cuda")
    gk = torch.empty(n, dtype=torch.float32, device="cuda")
    gd = torch.empty((n, anchors.shape[0]), dtype=torch.float32, device="cuda")
    A.check(L.gofann_rabitq_quantize(dptr((qr)), n, pd, A.ptr(gq8), A.ptr(gs), A.ptr(gk), stream()), "quantize")
    A.check(L.gofann_rabitq_centroid_dist(dptr((qr)), n, dptr((anchors)), anchors.shape[0], pd, A.ptr(gd),
                                          stream()), "gdist")
    torch.cuda.synchronize()
    dprep = {"rq_q8": gq8, "rq_scale": gs, "rq_k1xsumq": gk, "rq_centroid_dist": gd}
    hprep = {"rq_q8": gq8.cpu().numpy(), "rq_scale": gs.cpu().numpy(), "rq_k1xsumq": gk.cpu().numpy(),
             "rq_centroid_dist": gd.cpu().numpy()}
    return dprep, hprep


def test_rabitq_score_bitexact(L):
    w, idx, plan, rq, anchors, qr = rabitq_artifacts()
    dprep, hprep = _rq_prepared(L, qr, anchors)
    rng = np.random.default_rng(11)
    n_pairs = 5000
    pr = rng.integers(0, qr.shape[0], size=n_pairs).astype(np.uint32)
    ps = rng.integers(0, w.n, size=n_pairs).astype(np.uint32)
    want, want_ip = O.rabitq_score(rq, hprep, pr, ps)
    dcodes = dev_dict(rq)
    cs, pp = A.fill_codes(dcodes), A.fill_prepared(dprep)
    out = torch.empty(n_pairs, dtype=torch.float32, device="cuda")
    ip = torch.empty(n_pairs, dtype=torch.int32, device="cuda")
    A.check(L.gofann_rabitq_score(C.byref(cs), C.byref(pp), dptr((pr)), dptr((ps)), n_pairs, A.ptr(out),
                                  A.ptr(ip), stream()), "rq score")
    assert np.array_equal(ip.cpu().numpy(), want_ip)
    assert np.array_equal(fbits(out.cpu().numpy()), fbits(want))


# ----------------------------------------------------------- traversal
def run_gpu_beam(L, graph, attrs, codes, prep, routes, trace_width=0, expect_status=0, **params):
    dg, da, dc, dp, dr = dev_dict(graph), dev_dict(attrs), dev_dict(codes), prep, dev_dict(routes)
    gs, at, cs, ps, rs = A.fill_graph(dg), A.fill_attrs(da), A.fill_codes(dc), A.fill_prepared(dp), A.fill_routes(dr)
    sp = A.fill_params(**params)
    n, rw = rs.n_routes, sp.result_width
    ids = torch.empty((n, rw), dtype=torch.int32, device="cuda")
    d = torch.empty((n, rw), dtype=torch.float32, device="cuda")
    steps = torch.empty(n, dtype=torch.int32, device="cuda")
    cnt = torch.empty((n, 4), dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    trace = torch.empty((n, max(trace_width, 1)), dtype=torch.int32, device="cuda")
    out = A.SearchOut(ids=A.ptr(ids), dists=A.ptr(d), steps=A.ptr(steps), counters=A.ptr(cnt), status=A.ptr(status),
                      trace=A.ptr(trace) if trace_width else None, trace_width=trace_width)
    nbytes = L.gofann_beam_search_scratch_bytes(n)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    A.check(L.gofann_beam_search(C.byref(gs), C.byref(at), C.byref(cs), C.byref(ps), C.byref(rs), C.byref(sp),
                                 C.byref(out), A.ptr(scratch), nbytes, stream()), "beam_search")
    torch.cuda.synchronize()
    assert int(status.item()) == expect_status
    res = (host(ids, np.uint32), d.cpu().numpy(), steps.cpu().numpy(), host(cnt, np.uint32))
    if trace_width:
        return res + (host(trace, np.uint32),)
    return res


BEAM_VARIANTS = [
    dict(queue_size=64, predicate_bias=1, early_stop_mode=A.EARLY_STOP_ADAPTIVE, result_width=100,
         pq_mode=A.PQ_DIRECT),
    dict(queue_size=16, predicate_bias=0, early_stop_mode=A.EARLY_STOP_FIXED, finish_limit=20, result_width=50,
         pq_mode=A.PQ_LUT_GLOBAL),
    dict(queue_size=200, predicate_bias=1, early_stop_mode=A.EARLY_STOP_FIXED, finish_limit=100, result_width=512,
         pq_mode=A.PQ_LUT_SHARED),
    dict(queue_size=512, predicate_bias=0, early_stop_mode=A.EARLY_STOP_OFF, max_steps=300, result_width=100,
         pq_mode=A.PQ_DIRECT),
    dict(queue_size=2, predicate_bias=1, early_stop_mode=A.EARLY_STOP_ADAPTIVE, stop_width=1, result_width=1,
         pq_mode=A.PQ_DIRECT),
    dict(queue_size=96, predicate_bias=1, early_stop_mode=A.EARLY_STOP_ADAPTIVE, pending_base_stop=1,
         full_label_check=1, alpha=0.3, pq_mode=A.PQ_LUT_GLOBAL),
    dict(queue_size=384, predicate_bias=1, early_stop_mode=A.EARLY_STOP_ADAPTIVE, result_width=100,
         pq_mode=A.PQ_LUT_GLOBAL),
]


def pq_prep(w, idx, mode):
    """Device prepared state for a PQ mode: the LUT batch, or query rows + codebook."""
    if mode in (A.PQ_DIRECT, A.PQ_U8):
        return {"pq_query": dev(w.queries), "pq_centroids": dev(idx.pq_centroids)}
    return {"pq_lut": dev(O.pq_build_lut(w.queries.astype(np.float32), idx.pq_centroids, idx.pq_codes.shape[1]))}


@pytest.mark.parametrize("wl", ["cfg1", "cfg2"])
@pytest.mark.parametrize("vi", range(len(BEAM_VARIANTS)))
def test_beam_search_pq_bitexact(L, wl, vi):
    w, idx, plan = cfg1_small() if wl == "cfg1" else cfg2_small()
    params = dict(BEAM_VARIANTS[vi], scorer=A.SCORER_PQ)
    lut = O.pq_build_lut(w.queries.astype(np.float32), idx.pq_centroids, idx.pq_codes.shape[1])
    want = O.beam_search(idx.graph(), idx.attrs(), idx.codes(), {"pq_lut": lut}, plan.graph_routes, threads=8,
                         trace_width=64, **params)
    got = run_gpu_beam(L, idx.graph(), idx.attrs(), idx.codes(), pq_prep(w, idx, params["pq_mode"]),
                       plan.graph_routes, trace_width=64, **params)
    for name, g, o in zip(("ids", "dists", "steps", "counters", "trace"), got, want):
        if name == "dists":
            g, o = fbits(g), fbits(o)
        assert np.array_equal(g, o), f"{name} differ in {np.count_nonzero(np.any(np.atleast_2d(g != o), axis=-1))} routes"


@pytest.mark.parametrize("vi,pq_dim", [(v, 48) for v in range(len(BEAM_VARIANTS))] + [(1, 24), (6, 24)])
def test_beam_search_pq_u8_bitexact(L, vi, pq_dim):
    """GOFANN_PQ_U8 (integer codebook, u8 queries) against the oracle's float
    table + float ADC on the same codebook: the same bits.  Integer
    distances tie often, which the reference heap resolves by its layout.
    pq_dim 48 takes the 16-byte-chunk scorer, 24 (8-byte subvectors) the
    generic one."""
    w, idx, plan = cfg2_small_u8cb(pq_dim)
    params = dict(BEAM_VARIANTS[vi], scorer=A.SCORER_PQ, pq_mode=A.PQ_U8)
    lut = O.pq_build_lut(w.queries.astype(np.float32), idx.pq_centroids, idx.pq_codes.shape[1])
    want = O.beam_search(idx.graph(), idx.attrs(), idx.codes(), {"pq_lut": lut}, plan.graph_routes, threads=8,
                         trace_width=64, **params)
    got = run_gpu_beam(L, idx.graph(), idx.attrs(), idx.codes(), pq_prep(w, idx, A.PQ_U8), plan.graph_routes,
                       trace_width=64, **params)
    for name, g, o in zip(("ids", "dists", "steps", "counters", "trace"), got, want):
        if name == "dists":
            g, o = fbits(g), fbits(o)
        assert np.array_equal(g, o), f"{name} differ in {np.count_nonzero(np.any(np.atleast_2d(g != o), axis=-1))} routes"


def _with_records(L, graph, attrs, codes):
    """graph dict + per-row records built on the device."""
    dg, da, dc = dev_dict(graph), dev_dict(attrs), dev_dict(codes)
    gs, at, cs = A.fill_graph(dg), A.fill_attrs(da), A.fill_codes(dc)
    stride = int(L.gofann_row_record_stride(cs.pq_dim))
    rec = torch.empty((gs.total_rows, stride), dtype=torch.uint8, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    A.check(L.gofann_build_row_records(C.byref(gs), C.byref(at), C.byref(cs), A.ptr(rec), A.ptr(status), stream()),
            "build_row_records")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return dict(graph, records=rec), rec


def test_row_records_layout(L):
    """Record r = code row of sample row_to_sample[r], then (sample, label
    start, label length, label signature) at GOFANN_RECORD_META(pq_dim), then
    the label row itself when it has at most 16 labels."""
    w, idx, plan = cfg2_small()
    g, rec = _with_records(L, idx.graph(), idx.attrs(), idx.codes())
    rec = rec.cpu().numpy()
    m = idx.pq_codes.shape[1]
    meta = ((m + 15) // 16) * 16
    r2s = idx.graph()["row_to_sample"].astype(np.int64)
    ip = idx.attrs()["label_indptr"].astype(np.int64)
    assert np.array_equal(rec[:, :m], idx.pq_codes[r2s])
    words = rec[:, meta:meta + 16].copy().view(np.uint32)
    assert np.array_equal(words[:, 0], r2s)
    assert np.array_equal(words[:, 1], ip[r2s])
    assert np.array_equal(words[:, 2], ip[r2s + 1] - ip[r2s])
    ind = idx.attrs()["label_indices"].astype(np.uint64)
    bit = (np.uint64(1) << (((ind * np.uint64(0x9E3779B1)) & np.uint64(0xFFFFFFFF)) >> np.uint64(27))).astype(np.uint32)
    sig = np.bitwise_or.reduceat(bit, ip[:-1].astype(np.int64)) if ind.size else np.zeros(0, np.uint32)
    sig = np.where(ip[1:] > ip[:-1], sig, 0).astype(np.uint32)
    assert np.array_equal(words[:, 3], sig[r2s]), "label signature word"
    assert rec.shape[1] == meta + 16 + 4 * 16
    labels = rec[:, meta + 16:meta + 16 + 64].copy().view(np.uint32)
    ind = idx.attrs()["label_indices"]
    checked = 0
    for r in range(0, rec.shape[0], max(1, rec.shape[0] // 500)):
        n_lab = int(ip[r2s[r] + 1] - ip[r2s[r]])
        if n_lab <= 16:
            assert np.array_equal(labels[r, :n_lab], ind[ip[r2s[r]]:ip[r2s[r] + 1]])
            assert not labels[r, n_lab:].any()
            checked += 1
    assert checked > 0


@pytest.mark.parametrize("vi,mode", [(0, A.PQ_U8), (5, A.PQ_U8), (6, A.PQ_U8), (1, A.PQ_LUT_GLOBAL),
                                     (2, A.PQ_LUT_SHARED), (3, A.PQ_DIRECT)])
def test_beam_search_row_records_bitexact(L, vi, mode):
    """The traversal reading per-row records returns what the oracle (and
    the record-less path) returns."""
    w, idx, plan = cfg2_small_u8cb()
    params = dict(BEAM_VARIANTS[vi], scorer=A.SCORER_PQ, pq_mode=mode)
    lut = O.pq_build_lut(w.queries.astype(np.float32), idx.pq_centroids, idx.pq_codes.shape[1])
    want = O.beam_search(idx.graph(), idx.attrs(), idx.codes(), {"pq_lut": lut}, plan.graph_routes, threads=8,
                         trace_width=64, **params)
    g, _ = _with_records(L, idx.graph(), idx.attrs(), idx.codes())
    got = run_gpu_beam(L, g, idx.attrs(), idx.codes(), pq_prep(w, idx, mode), plan.graph_routes, trace_width=64,
                       **params)
    for name, gv, o in zip(("ids", "dists", "steps", "counters", "trace"), got, want):
        if name == "dists":
            gv, o = fbits(gv), fbits(o)
        assert np.array_equal(gv, o), name


def test_beam_search_pq_u8_rejects_fractional_codebook(L):
    """A codebook value that is not an integer in 0..255 sets the status word
    to GOFANN_ERR_INVALID (checked on the device) instead of searching."""
    w, idx, plan = cfg2_small_u8cb()
    cent = idx.pq_centroids.copy()
    cent[17, 5] += 0.5
    params = dict(BEAM_VARIANTS[1], scorer=A.SCORER_PQ, pq_mode=A.PQ_U8)
    run_gpu_beam(L, idx.graph(), idx.attrs(), idx.codes(), {"pq_query": dev(w.queries), "pq_centroids": dev(cent)},
                 plan.graph_routes, expect_status=A.ERR_INVALID, **params)


@pytest.mark.parametrize("share", [2, 20])
@pytest.mark.parametrize("vi", [0, 2, 5, 6])
def test_beam_search_pq_ties_bitexact(L, share, vi):
    """Equal priorities: samples share PQ codes (every 2nd, or every 20th,
    sample copies its neighbour's code row), so candidates tie exactly and the
    order among equal entries is decided by the reference heap's layout."""
    w, idx, plan = cfg2_small()
    codes = idx.codes()
    pq = codes["pq_codes"].copy()
    rows = np.arange(pq.shape[0])
    dup = rows[(rows % share) == 1]
    pq[dup] = pq[dup - 1]
    codes = dict(codes, pq_codes=pq)
    params = dict(BEAM_VARIANTS[vi], scorer=A.SCORER_PQ)
    lut = O.pq_build_lut(w.queries.astype(np.float32), idx.pq_centroids, pq.shape[1])
    want = O.beam_search(idx.graph(), idx.attrs(), codes, {"pq_lut": lut}, plan.graph_routes, threads=8,
                         trace_width=64, **params)
    got = run_gpu_beam(L, idx.graph(), idx.attrs(), codes, pq_prep(w, idx, params["pq_mode"]), plan.graph_routes,
                       trace_width=64, **params)
    for name, g, o in zip(("ids", "dists", "steps", "counters", "trace"), got, want):
        if name == "dists":
            g, o = fbits(g), fbits(o)
        assert np.array_equal(g, o), f"{name} differ in {np.count_nonzero(np.any(np.atleast_2d(g != o), axis=-1))} routes"


def _chain_graph(n=12000, fwd=48, back=16):
    """Row r scores 65535 - r (codes (r >> 8, r & 255) against a table whose
    entries are exact integers) and links the next `fwd` and the previous
    `back` rows: every expansion admits fresh rows, so a route admits far
    more than 4,096 rows, and the backward links meet rows whose inserts a
    full visited table dropped."""
    deg = fwd + back
    r = np.arange(n, dtype=np.int64)[:, None]
    off = np.concatenate([np.arange(1, fwd + 1), -np.arange(1, back + 1)])[None, :]
    adj = r + off
    adj = np.where((adj >= 0) & (adj < n), adj, 0xFFFFFFFF).astype(np.uint32)
    graph = {"adjacency": adj, "row_to_sample": np.arange(n, dtype=np.uint32),
             "label_offset": np.zeros(1, np.uint32)}
    attrs = {"label_indptr": np.arange(n + 1, dtype=np.uint64), "label_indices": np.zeros(n, np.uint32)}
    codes = {"pq_codes": np.stack([np.arange(n) >> 8, np.arange(n) & 255], 1).astype(np.uint8)}
    lut = np.zeros((1, 2, 256), np.float32)
    lut[0, 0] = 256.0 * (255 - np.arange(256))
    lut[0, 1] = 255 - np.arange(256)
    starts = np.array([0, 5, 300, 1000], np.uint32)
    routes = {"query_row": np.zeros(len(starts), np.uint32), "group_id": np.zeros(len(starts), np.uint32),
              "start_local": starts}
    return graph, attrs, codes, lut, routes


@pytest.mark.parametrize("queue_size", [64, 512])
def test_beam_search_visited_table_fills(L, queue_size):
    """Routes that admit more than 4,096 rows: the visited table fills and
    drops later inserts exactly as the reference's does."""
    graph, attrs, codes, lut, routes = _chain_graph()
    params = dict(queue_size=queue_size, predicate_bias=0, early_stop_mode=A.EARLY_STOP_OFF, max_steps=400,
                  result_width=100, scorer=A.SCORER_PQ, pq_mode=A.PQ_LUT_GLOBAL)
    want = O.beam_search(graph, attrs, codes, {"pq_lut": lut}, routes, threads=4, trace_width=64, **params)
    assert want[3][:, 3].min() > 4096, "a route did not fill its visited table"
    got = run_gpu_beam(L, graph, attrs, codes, {"pq_lut": dev(lut)}, routes, trace_width=64, **params)
    for name, g, o in zip(("ids", "dists", "steps", "counters", "trace"), got, want):
        if name == "dists":
            g, o = fbits(g), fbits(o)
        assert np.array_equal(g, o), name


@pytest.mark.parametrize("queue_size", [64, 512])
def test_beam_search_repeated_neighbour_ids(L, queue_size):
    """Adjacency rows that list an id twice: both copies pass the step's
    visited test and enter the frontier, as in the reference, but the visited
    table takes the id once -- so the table fills (routes admit more than
    4,096 rows) at exactly the reference's point."""
    graph, attrs, codes, lut, routes = _chain_graph()
    adj = graph["adjacency"].copy()
    adj[:, 5] = adj[:, 0]          # a forward neighbour listed twice
    adj[::3, 40] = adj[::3, 2]     # and another on every third row
    graph = dict(graph, adjacency=adj)
    params = dict(queue_size=queue_size, predicate_bias=0, early_stop_mode=A.EARLY_STOP_OFF, max_steps=400,
                  result_width=100, scorer=A.SCORER_PQ, pq_mode=A.PQ_LUT_GLOBAL)
    want = O.beam_search(graph, attrs, codes, {"pq_lut": lut}, routes, threads=4, trace_width=64, **params)
    assert want[3][:, 3].min() > 4096, "a route did not fill its visited table"
    got = run_gpu_beam(L, graph, attrs, codes, {"pq_lut": dev(lut)}, routes, trace_width=64, **params)
    for name, g, o in zip(("ids", "dists", "steps", "counters", "trace"), got, want):
        if name == "dists":
            g, o = fbits(g), fbits(o)
        assert np.array_equal(g, o), name


def test_row_records_reject_out_of_range_sample(L):
    """A row whose row -> sample entry is past the attribute table gets an
    all-zero record and the status word reports GOFANN_ERR_INVALID."""
    w, idx, plan = cfg2_small()
    g = dict(idx.graph())
    r2s = g["row_to_sample"].copy()
    r2s[7] = w.n + 3
    g["row_to_sample"] = r2s
    dg, da, dc = dev_dict(g), dev_dict(idx.attrs()), dev_dict(idx.codes())
    gs, at, cs = A.fill_graph(dg), A.fill_attrs(da), A.fill_codes(dc)
    stride = int(L.gofann_row_record_stride(cs.pq_dim))
    rec = torch.full((gs.total_rows, stride), 0xAB, dtype=torch.uint8, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    A.check(L.gofann_build_row_records(C.byref(gs), C.byref(at), C.byref(cs), A.ptr(rec), A.ptr(status), stream()),
            "build_row_records")
    torch.cuda.synchronize()
    assert int(status.item()) == A.ERR_INVALID
    r = rec.cpu().numpy()
    assert not r[7].any()
    assert r[8].any()


@pytest.mark.parametrize("pd", [64, 512, 4096])
def test_rabitq_encode_bitexact(L, pd):
    """Device 1-bit encoder against the oracle's restatement of its FP32
    order, given the residuals: codes and factor bits equal (exact zeros and
    -0.0 give bit 0; a vector of zeros takes the rxu = 0 guard)."""
    rng = np.random.default_rng(pd)
    n, a = 777, 13
    r = rng.standard_normal((n, pd)).astype(np.float32)
    r[5, ::3] = 0.0
    r[6, 1::4] = -0.0
    r[7] = 0.0
    c = rng.standard_normal((a, pd)).astype(np.float32)
    aid = rng.integers(0, a, size=n).astype(np.uint32)
    want_c, want_f = O.rabitq_encode_f32(r, c, aid)
    codes = torch.empty((n, pd // 8), dtype=torch.uint8, device="cuda")
    f = torch.empty((n, 3), dtype=torch.float32, device="cuda")
    A.check(L.gofann_rabitq_encode(dptr(r), dptr(c), dptr(aid), n, pd, A.ptr(codes), A.ptr(f), stream()), "encode")
    torch.cuda.synchronize()
    assert np.array_equal(codes.cpu().numpy(), want_c)
    assert np.array_equal(fbits(f.cpu().numpy()), fbits(want_f))


def test_rabitq_route_entries(L):
    """Each route starts at the entry row of its query's nearest anchor
    (lowest anchor on equal distances)."""
    rng = np.random.default_rng(4)
    rows, na, nr = 50, 300, 777
    g = rng.integers(0, 40, size=(rows, na)).astype(np.float32)  # many ties
    qr = rng.integers(0, rows, size=nr).astype(np.uint32)
    entry = rng.permutation(100000)[:na].astype(np.uint32)
    out = torch.empty(nr, dtype=torch.int32, device="cuda")
    A.check(L.gofann_rabitq_route_entries(dptr(g), na, dptr(qr), nr, dptr(entry), A.ptr(out), stream()), "entries")
    torch.cuda.synchronize()
    assert np.array_equal(host(out, np.uint32), entry[np.argmin(g[qr], axis=1)])


@pytest.mark.parametrize("vi,dim", [(0, 128), (1, 128), (3, 128), (0, 512), (1, 4096)])
def test_beam_search_rabitq_bitexact(L, vi, dim):
    """RaBitQ traversal at padded dims 128, 512 and 4096 (64- and 512-byte
    codes, the config-4 and config-3 widths)."""
    w, idx, plan, rq, anchors, qr = rabitq_artifacts(n=6000 if dim == 128 else 2500, dim=dim)
    dprep, hprep = _rq_prepared(L, qr, anchors)
    params = dict(BEAM_VARIANTS[vi], scorer=A.SCORER_RABITQ, pq_mode=A.PQ_LUT_GLOBAL)
    want = O.beam_search(idx.graph(), idx.attrs(), rq, hprep, plan.graph_routes, threads=8, **params)
    got = run_gpu_beam(L, idx.graph(), idx.attrs(), rq, dprep, plan.graph_routes, **params)
    for name, g, o in zip(("ids", "dists", "steps", "counters"), got, want):
        if name == "dists":
            g, o = fbits(g), fbits(o)
        assert np.array_equal(g, o), name


def test_beam_search_edge_cases(L):
    """Seed-only graphs (all neighbours padding), a seed whose neighbours are
    all visited, and a zero-route batch."""
    w, idx, plan = cfg1_small()
    g = idx.graph()
    adj = g["adjacency"].copy()
    adj[: adj.shape[0] // 2] = A.U32MAX
    g = dict(g, adjacency=adj)
    lut = O.pq_build_lut(w.queries, idx.pq_centroids, idx.pq_codes.shape[1])
    params = dict(queue_size=32, predicate_bias=1)
    want = O.beam_search(g, idx.attrs(), idx.codes(), {"pq_lut": lut}, plan.graph_routes, **params)
    got = run_gpu_beam(L, g, idx.attrs(), idx.codes(), {"pq_lut": dev(lut)}, plan.graph_routes, **params)
    assert np.array_equal(got[0], want[0]) and np.array_equal(got[2], want[2])
    empty = {k: v[:0] if k not in ("qlabel_indptr", "pred_offsets") else v[:1] for k, v in plan.graph_routes.items()}
    dg, da, dc = dev_dict(idx.graph()), dev_dict(idx.attrs()), dev_dict(idx.codes())
    dr = dev_dict({k: v if v.size else np.zeros(1, v.dtype) for k, v in empty.items()})
    gs, at, cs, rs = A.fill_graph(dg), A.fill_attrs(da), A.fill_codes(dc), A.fill_routes(dr)
    rs.n_routes = 0
    dl = {"pq_lut": dev(lut)}
    ps = A.fill_prepared(dl)
    sp = A.fill_params(**params)
    buf = torch.empty(16, dtype=torch.int32, device="cuda")
    out = A.SearchOut(ids=A.ptr(buf), dists=A.ptr(buf))
    assert L.gofann_beam_search(C.byref(gs), C.byref(at), C.byref(cs), C.byref(ps), C.byref(rs), C.byref(sp),
                                C.byref(out), A.ptr(buf), 64, stream()) == 0


# ----------------------------------------------------------- postings
def run_gpu_posting(L, codes, prep, attrs, routes, scorer, pids, begin, count, k, pq_mode=A.PQ_LUT_GLOBAL,
                    expect_status=0):
    dc, da, dr = dev_dict(codes), dev_dict(attrs), dev_dict(routes)
    cs, pp, at, rs = A.fill_codes(dc), A.fill_prepared(prep), A.fill_attrs(da), A.fill_routes(dr)
    n = rs.n_routes
    ids = torch.empty((n, k), dtype=torch.int32, device="cuda")
    d = torch.empty((n, k), dtype=torch.float32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    A.check(L.gofann_posting_scan(C.byref(cs), C.byref(pp), C.byref(at), C.byref(rs), scorer, dptr((pids)),
                                  dptr((begin)), dptr((count)), k, 1, pq_mode, A.ptr(ids), A.ptr(d), A.ptr(status),
                                  stream()), "posting")
    torch.cuda.synchronize()
    assert int(status.item()) == expect_status
    return host(ids, np.uint32), d.cpu().numpy()


@pytest.mark.parametrize("k,fused", [(1, False), (10, True), (100, False), (100, True), (400, True)])
def test_posting_scan_pq_bitexact(L, k, fused):
    from gofann.planner import concat_routes, subset_routes
    w, idx, plan = cfg2_small()
    lut = O.pq_build_lut(w.queries.astype(np.float32), idx.pq_centroids, idx.pq_codes.shape[1])
    # the planner's low-frequency routes, plus scans of the three largest
    # postings (several sort rounds) and one empty posting
    big = np.argsort(idx.posting_count)[-3:]
    extra = subset_routes(plan.graph_routes, np.arange(4))
    routes = concat_routes(plan.posting_routes, extra)
    begin = np.concatenate([plan.posting_begin, idx.posting_begin[big], [0]]).astype(np.uint64)
    count = np.concatenate([plan.posting_count, idx.posting_count[big], [0]]).astype(np.uint32)
    want = O.posting_scan(idx.codes(), {"pq_lut": lut}, idx.attrs(), routes, A.SCORER_PQ, idx.posting_ids, begin,
                          count, k)
    prep = pq_prep(w, idx, A.PQ_DIRECT if fused else A.PQ_LUT_GLOBAL)  # fused: table built in the scan
    got = run_gpu_posting(L, idx.codes(), prep, idx.attrs(), routes, A.SCORER_PQ, idx.posting_ids, begin, count, k)
    assert np.array_equal(got[0], want[0])
    assert np.array_equal(fbits(got[1]), fbits(want[1]))


@pytest.mark.parametrize("k,pq_dim", [(10, 48), (100, 48), (400, 48), (100, 24)])
def test_posting_scan_pq_u8_codebook_bitexact(L, k, pq_dim):
    """The index's integer codebook with u8 queries and no prebuilt table (the
    traversal's GOFANN_PQ_U8 inputs).  4-byte subvectors run the PQ_U8 scorer
    (persistent blocks, packed integer codebook), 8-byte ones the table the
    scan builds itself; both match the oracle's float table + sequential
    float ADC bit for bit, over multi-round postings and an empty posting."""
    from gofann.planner import concat_routes, subset_routes
    w, idx, plan = cfg2_small_u8cb(pq_dim)
    lut = O.pq_build_lut(w.queries.astype(np.float32), idx.pq_centroids, idx.pq_codes.shape[1])
    big = np.argsort(idx.posting_count)[-3:]
    extra = subset_routes(plan.graph_routes, np.arange(4))
    routes = concat_routes(plan.posting_routes, extra)
    begin = np.concatenate([plan.posting_begin, idx.posting_begin[big], [0]]).astype(np.uint64)
    count = np.concatenate([plan.posting_count, idx.posting_count[big], [0]]).astype(np.uint32)
    want = O.posting_scan(idx.codes(), {"pq_lut": lut}, idx.attrs(), routes, A.SCORER_PQ, idx.posting_ids, begin,
                          count, k)
    mode = A.PQ_U8 if pq_dim == 48 else A.PQ_DIRECT
    got = run_gpu_posting(L, idx.codes(), pq_prep(w, idx, A.PQ_U8), idx.attrs(), routes, A.SCORER_PQ,
                          idx.posting_ids, begin, count, k, pq_mode=mode)
    assert np.array_equal(got[0], want[0])
    assert np.array_equal(fbits(got[1]), fbits(want[1]))


def test_posting_scan_pq_u8_rejects_fractional_codebook(L):
    """A codebook value that is not an integer: the PQ_U8 scan sets the status
    word and returns empty shortlists (no scoring on a wrong codebook)."""
    w, idx, plan = cfg2_small_u8cb(48)
    prep = pq_prep(w, idx, A.PQ_U8)
    cent = prep["pq_centroids"].clone()
    cent[3, 5] += 0.5
    prep = dict(prep, pq_centroids=cent)
    routes = plan.posting_routes
    ids, d = run_gpu_posting(L, idx.codes(), prep, idx.attrs(), routes, A.SCORER_PQ, idx.posting_ids,
                             plan.posting_begin, plan.posting_count, 10, pq_mode=A.PQ_U8,
                             expect_status=A.ERR_INVALID)
    assert np.all(ids == A.U32MAX) and np.all(d == np.float32(np.finfo(np.float32).max))


@pytest.mark.parametrize("dim", [128, 4096])
def test_posting_scan_rabitq_bitexact(L, dim):
    w, idx, plan, rq, anchors, qr = rabitq_artifacts(n=6000 if dim == 128 else 2500, dim=dim)
    dprep, hprep = _rq_prepared(L, qr, anchors)
    routes = plan.graph_routes  # scan each graph route's label posting
    lab = routes["primary_label"]
    begin, count = idx.posting_begin[lab], idx.posting_count[lab]
    want = O.posting_scan(rq, hprep, idx.attrs(), routes, A.SCORER_RABITQ, idx.posting_ids, begin, count, 100)
    got = run_gpu_posting(L, rq, dprep, idx.attrs(), routes, A.SCORER_RABITQ,
                          idx.posting_ids, begin, count, 100)
    assert np.array_equal(got[0], want[0])
    assert np.array_equal(fbits(got[1]), fbits(want[1]))


@pytest.mark.parametrize("dim,k", [(128, 100), (160, 10), (480, 400), (992, 100)])
def test_posting_scan_rabitq_long_slices(L, dim, k):
    """Slices of a random order of the whole base (the attribute-order range
    scans): thousands of candidates per route, so the running top-k merges
    several times; lanes per candidate 1, none (padded_dim 192 is not a
    multiple of 128), 4 and 8; UINT32_MAX padding and repeated ids inside the
    slices; the planner's DNF predicates on half of the routes."""
    w, idx, plan, rq, anchors, qr = rabitq_artifacts(n=6000, dim=dim, n_queries=48)
    dprep, hprep = _rq_prepared(L, qr, anchors)
    rng = np.random.default_rng(dim)
    order = rng.permutation(w.n).astype(np.uint32)
    order[rng.random(w.n) < 0.01] = A.U32MAX
    order[100:110] = order[200:210]
    routes = {kk: v.copy() for kk, v in plan.graph_routes.items()}
    n = routes["query_row"].shape[0]
    routes["pred_enabled"] = (np.arange(n) % 2).astype(np.uint8)
    lo = rng.integers(0, w.n // 2, size=n)
    cnt = rng.integers(1, w.n - lo).astype(np.uint32)
    cnt[0], lo[0] = w.n, 0   # the whole order
    cnt[1] = 0               # an empty slice
    begin = lo.astype(np.uint64)
    want = O.posting_scan(rq, hprep, idx.attrs(), routes, A.SCORER_RABITQ, order, begin, cnt, k)
    got = run_gpu_posting(L, rq, dprep, idx.attrs(), routes, A.SCORER_RABITQ, order, begin, cnt, k)
    assert np.array_equal(got[0], want[0])
    assert np.array_equal(fbits(got[1]), fbits(want[1]))


# --------------------------------------------------------------- rerank
def _ties_equivalent(gi, gd, wi, wd, rtol):
    """Ids equal, or differing only inside a run of distances equal within rtol."""
    if np.array_equal(gi, wi):
        return True
    for r in range(gi.shape[0]):
        if np.array_equal(gi[r], wi[r]):
            continue
        if not np.allclose(gd[r], wd[r], rtol=rtol, atol=0):
            return False
        for j in np.nonzero(gi[r] != wi[r])[0]:
            near = np.abs(wd[r] - gd[r, j]) <= rtol * np.abs(gd[r, j])
            if gi[r, j] not in wi[r][near] and gi[r, j] != A.U32MAX:
                return False
    return True


@pytest.mark.parametrize("dtype", ["u8", "f32", "f16"])
def test_rerank(L, dtype):
    if dtype == "u8":
        w, idx, plan = cfg2_small()
        base, queries = w.base, w.queries
    else:
        w, idx, plan = cfg1_small()
        base = w.base if dtype == "f32" else w.base.astype(np.float16)
        queries = w.queries
    dt = {"u8": A.DTYPE_U8, "f32": A.DTYPE_F32, "f16": A.DTYPE_F16}[dtype]
    rng = np.random.default_rng(3)
    routes = plan.graph_routes
    n = routes["query_row"].shape[0]
    width = 100
    cand = rng.integers(0, w.n, size=(n, width)).astype(np.uint32)
    cand[:, 5] = cand[:, 3]  # duplicates
    cand[rng.random(cand.shape) < 0.05] = A.U32MAX
    cand[0, :] = A.U32MAX    # empty shortlist
    cand[1, 7] = w.n + 5     # out of range id
    want_i, want_d = O.rerank(base, dt, queries, idx.attrs(), routes, cand, 10)
    bt = dev(base.view(np.uint16) if dtype == "f16" else base)
    ids = torch.empty((n, 10), dtype=torch.int32, device="cuda")
    d = torch.empty((n, 10), dtype=torch.float32, device="cuda")
    da, dr = dev_dict(idx.attrs()), dev_dict(routes)
    at, rs = A.fill_attrs(da), A.fill_routes(dr)
    A.check(L.gofann_rerank(A.ptr(bt), dt, w.n, w.dim, dptr((queries)), C.byref(at), C.byref(rs),
                            dptr((cand)), width, 10, A.ptr(ids), A.ptr(d), stream()), "rerank")
    gi, gd = host(ids, np.uint32), d.cpu().numpy()
    if dtype == "u8":
        assert np.array_equal(gi, want_i) and np.array_equal(fbits(gd), fbits(want_d))
    else:
        rtol = 1e-5 if dtype == "f32" else 1e-3
        valid = want_i != A.U32MAX
        assert np.array_equal(gi == A.U32MAX, ~valid)
        assert np.all(np.abs(gd[valid] - want_d[valid]) <= rtol * np.abs(want_d[valid]))
        assert _ties_equivalent(gi, gd, want_i, want_d, rtol)


# --------------------------------------------------------------- merges
def test_route_merge_bitexact(L):
    rng = np.random.default_rng(9)
    n_routes, n_q, width = 700, 300, 10
    r2q = rng.integers(0, n_q, size=n_routes)
    ids = rng.integers(0, 500, size=(n_routes, width)).astype(np.uint32)
    ids[rng.random(ids.shape) < 0.1] = A.U32MAX
    d = rng.integers(0, 50, size=(n_routes, width)).astype(np.float32)
    order = np.argsort(r2q, kind="stable").astype(np.uint32)
    qoff = np.zeros(n_q + 1, np.uint32)
    qoff[1:] = np.cumsum(np.bincount(r2q, minlength=n_q))
    wi, wd = O.route_merge(ids, d, qoff, order, 10)
    oi = torch.empty((n_q, 10), dtype=torch.int32, device="cuda")
    od = torch.empty((n_q, 10), dtype=torch.float32, device="cuda")
    A.check(L.gofann_route_merge(dptr((ids)), dptr((d)), width, dptr((qoff)), dptr((order)), n_q, 10,
                                 A.ptr(oi), A.ptr(od), stream()), "route merge")
    assert np.array_equal(host(oi, np.uint32), wi) and np.array_equal(fbits(od.cpu().numpy()), fbits(wd))


@pytest.mark.parametrize("shards", [1, 2, 8])
def test_shard_merge_bitexact(L, shards):
    rng = np.random.default_rng(shards)
    nq, k = 257, 10
    ids = np.empty((shards, nq, k), np.uint32)
    d = np.empty((shards, nq, k), np.float32)
    for s in range(shards):
        # each shard's list is sorted by (dist, id) with unique, shard-disjoint ids
        dd = rng.integers(0, 30, size=(nq, k)).astype(np.float32)
        ii = np.stack([s * 1000 + rng.permutation(1000)[:k] for _ in range(nq)]).astype(np.uint32)
        for q in range(nq):
            o = np.lexsort((ii[q], dd[q]))
            ids[s, q], d[s, q] = ii[q][o], dd[q][o]
    ids[0, 0, 5:] = A.U32MAX
    d[0, 0, 5:] = A.FLT_MAX
    wi, wd = O.shard_merge(ids, d, k)
    oi = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    od = torch.empty((nq, k), dtype=torch.float32, device="cuda")
    A.check(L.gofann_shard_merge(dptr((ids)), dptr((d)), shards, nq, k, A.ptr(oi), A.ptr(od), stream()), "shard")
    assert np.array_equal(host(oi, np.uint32), wi) and np.array_equal(fbits(od.cpu().numpy()), fbits(wd))


def test_offset_ids(L):
    x = np.array([0, 5, A.U32MAX, 7], np.uint32)
    t = dev(x)
    A.check(L.gofann_offset_ids(A.ptr(t), 4, 100, stream()), "offset")
    assert np.array_equal(host(t, np.uint32), np.array([100, 105, A.U32MAX, 107], np.uint32))


# ------------------------------------------------------------ end to end
@pytest.mark.parametrize("wl", ["cfg1", "cfg2"])
def test_pipeline_matches_oracle_and_recall(L, wl):
    from gofann.engine import DeviceIndex, DevicePlan, Pipeline, SearchConfig
    w, idx, plan = cfg1_small() if wl == "cfg1" else cfg2_small()
    cfg = SearchConfig(queue_size=64, result_width=100)
    pipe = Pipeline(DeviceIndex(idx), DevicePlan(plan, "cuda"), cfg)
    q = dev(w.queries)
    gi, gd = pipe.run(q)
    torch.cuda.synchronize()
    gi = host(gi, np.uint32)
    # oracle pipeline on the same inputs
    dt = A.DTYPE_U8 if w.dtype == "u8" else A.DTYPE_F32
    lut = O.pq_build_lut(w.queries.astype(np.float32), idx.pq_centroids, idx.pq_codes.shape[1])
    bi, _, _, _ = O.beam_search(idx.graph(), idx.attrs(), idx.codes(), {"pq_lut": lut}, plan.graph_routes, threads=8,
                                **{k: getattr(cfg, k) for k in ("queue_size", "stop_width", "result_width",
                                                                "finish_limit", "early_stop_mode", "predicate_bias",
                                                                "alpha")})
    ri, rd = O.rerank(w.base, dt, w.queries, idx.attrs(), plan.graph_routes, bi, 10)
    pi, _ = O.posting_scan(idx.codes(), {"pq_lut": lut}, idx.attrs(), plan.posting_routes, A.SCORER_PQ,
                           idx.posting_ids, plan.posting_begin, plan.posting_count, cfg.lowfreq_shortlist)
    rpi, rpd = O.rerank(w.base, dt, w.queries, idx.attrs(), plan.posting_routes, pi, 10)
    qoff, order = plan.merge_tables()
    wi, wd = O.route_merge(np.concatenate([ri, rpi]), np.concatenate([rd, rpd]), qoff, order, 10)
    if w.dtype == "u8":
        assert np.array_equal(gi, wi)
    else:
        assert _ties_equivalent(gi, gd.cpu().numpy(), wi, wd, 1e-5)
    # recall against exhaustive filtered top-k (FP64)
    from gofann.planner import _route_tables
    labs = [np.asarray(x, np.uint32) for x in w.query_labels]
    gt_routes = _route_tables(list(range(len(labs))), labs, [x[0] for x in labs], [0] * len(labs), [0] * len(labs))
    gt_routes["pred_enabled"][:] = 0  # filter = every query label (residual check + primary)
    ti, _ = O.filtered_topk(w.base, dt, w.queries, idx.attrs(), gt_routes, 10)
    rec = np.mean([len((set(gi[i].tolist()) & set(ti[i].tolist())) - {A.U32MAX}) /
                   max(1, len(set(ti[i].tolist()) - {A.U32MAX})) for i in range(gi.shape[0])])
    assert rec >= 0.95, rec
