"""The whole-batch C entry point, driven from C++ (tests/cpp/batch_driver.cpp).

The driver is compiled with g++ against include/gofann.h and
libgofann_b200.so only; it reads a batch written here, runs
gofann_search_batch and writes the per-query top-k.  CPU tests: the driver
compiles and links, the batch scratch size is a host computation and bad
shapes are rejected without a GPU.  GPU tests: its results equal the
per-stage pipeline's and the oracle pipeline's bit for bit, for the PQ table
mode, the PQ_U8 mode with predicates, and RaBitQ with tensor-core query
preparation.
"""
import ctypes as C
import subprocess
from pathlib import Path

import numpy as np
import pytest

from gofann import _abi as A

ROOT = Path(__file__).resolve().parents[1]
DRIVER_SRC = ROOT / "tests" / "cpp" / "batch_driver.cpp"


def build_driver(out_dir: Path) -> Path:
    exe = out_dir / "batch_driver"
    subprocess.run(["g++", "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror", "-I", str(ROOT / "include"),
                    "-I", "/usr/local/cuda/include", str(DRIVER_SRC), "-L", str(A.LIB_PATH.parent), "-lgofann_b200",
                    "-L", "/usr/local/cuda/lib64", "-lcudart", f"-Wl,-rpath,{A.LIB_PATH.parent}", "-o", str(exe)],
                   check=True)
    return exe


def test_driver_compiles_and_links(tmp_path):
    exe = build_driver(tmp_path)
    out = subprocess.run(["nm", "-u", str(exe)], capture_output=True, text=True, check=True).stdout
    for sym in ("gofann_search_batch", "gofann_search_batch_scratch_bytes", "gofann_abi_version"):
        assert sym in out


def test_batch_scratch_and_validation_without_gpu():
    L = A.lib()
    ix, b, p = A.Index(), A.Batch(), A.BatchParams()
    assert L.gofann_search_batch_scratch_bytes(C.byref(ix), C.byref(b), C.byref(p)) == 0  # topk 0
    assert b"topk" in L.gofann_last_error()
    p.topk, p.posting_shortlist = 10, 100
    p.search = A.fill_params(result_width=100, pq_mode=A.PQ_LUT_GLOBAL)
    b.n_queries = 1000
    b.graph_routes.n_routes, b.posting_routes.n_routes = 700, 300
    for name in ("queries", "query_route_offsets", "query_routes", "posting_begin", "posting_count"):
        setattr(b, name, 256)
    ix.base, ix.dim, ix.posting_ids, ix.pq_centroids = 256, 128, 256, 256
    ix.codes.pq_dim = 32
    n = L.gofann_search_batch_scratch_bytes(C.byref(ix), C.byref(b), C.byref(p))
    lut = 1000 * 32 * 256 * 4
    routes = 700 * 100 * 8 + 300 * 100 * 8 + 1000 * 10 * 8
    assert n >= lut + routes + L.gofann_beam_search_scratch_bytes(700)
    assert n % 256 == 0
    # the same call with a too-small scratch is refused before any launch
    st = L.gofann_search_batch(C.byref(ix), C.byref(b), C.byref(p), C.c_void_p(256), n - 256, C.c_void_p(256),
                               C.c_void_p(256), None, None)
    assert st == A.ERR_INVALID and b"scratch" in L.gofann_last_error()
    p.search.scorer = A.SCORER_RABITQ
    assert L.gofann_search_batch_scratch_bytes(C.byref(ix), C.byref(b), C.byref(p)) == 0  # f32 base + rotation


# ---------------------------------------------------------------- GPU
def _raw(a: np.ndarray) -> bytes:
    a = np.ascontiguousarray(a)
    return a.tobytes()


def write_batch(d: Path, arrays: dict, scalars: dict):
    d.mkdir(parents=True, exist_ok=True)
    lines = []
    for name, a in arrays.items():
        if a is None:
            continue
        raw = _raw(a)
        (d / f"{name}.bin").write_bytes(raw)
        lines.append(f"array {name} {len(raw)}")
    for name, v in scalars.items():
        lines.append(f"scalar {name} {v!r}")
    (d / "manifest.txt").write_text("\n".join(lines) + "\n")


def _routes(prefix: str, r: dict) -> tuple[dict, dict]:
    arrays = {prefix + k: r.get(k) for k in A.ROUTE_KEYS}
    rm = r.get("range_modes")
    scalars = {prefix + "n_routes": int(r["query_row"].shape[0]),
               prefix + "range_count": int(rm.shape[1]) if rm is not None else 0}
    return arrays, scalars


def batch_inputs(w, idx, plan, attrs=None, graph=None, graph_routes=None, posting_routes=None):
    graph = graph or idx.graph()
    attrs = attrs or idx.attrs()
    g_arrays, g_scalars = _routes("g.", graph_routes or plan.graph_routes)
    p_arrays, p_scalars = _routes("p.", posting_routes or plan.posting_routes)
    qoff, order = plan.merge_tables()
    rv = attrs.get("range_values")
    arrays = {"graph.adjacency": graph["adjacency"], "graph.row_to_sample": graph["row_to_sample"],
              "graph.row_filter_mask": graph.get("row_filter_mask"), "graph.label_offset": graph["label_offset"],
              "attrs.label_indptr": attrs["label_indptr"], "attrs.label_indices": attrs["label_indices"],
              "attrs.range_values": rv, "codes.pq_codes": idx.pq_codes, "pq_centroids": idx.pq_centroids,
              "base": w.base, "posting_ids": idx.posting_ids, "queries": w.queries,
              "posting_begin": plan.posting_begin, "posting_count": plan.posting_count,
              "query_route_offsets": qoff, "query_routes": order, **g_arrays, **p_arrays}
    scalars = {"graph.total_rows": int(graph["adjacency"].shape[0]), "graph.degree": int(graph["adjacency"].shape[1]),
               "graph.group_count": int(graph["label_offset"].shape[0]),
               "attrs.n_samples": int(attrs["label_indptr"].shape[0] - 1),
               "attrs.range_count": int(rv.shape[1]) if rv is not None else 0,
               "codes.pq_dim": int(idx.pq_codes.shape[1]),
               "base_dtype": A.DTYPE_U8 if w.base.dtype == np.uint8 else A.DTYPE_F32, "dim": int(w.dim),
               "n_queries": int(w.queries.shape[0]), **g_scalars, **p_scalars}
    return arrays, scalars


def run_driver(tmp_path: Path, arrays: dict, scalars: dict, nq: int, k: int = 10):
    exe = build_driver(tmp_path)
    d = tmp_path / "batch"
    write_batch(d, arrays, scalars)
    r = subprocess.run([str(exe), str(d)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    ids = np.fromfile(d / "out_ids.bin", np.uint32).reshape(nq, k)
    dists = np.fromfile(d / "out_dists.bin", np.float32).reshape(nq, k)
    return ids, dists


def _oracle_pipeline(w, idx, plan, attrs, graph, groutes, proutes, lut, params, shortlist):
    from oracle import oracle as O
    dt = A.DTYPE_U8 if w.base.dtype == np.uint8 else A.DTYPE_F32
    bi, _, _, _ = O.beam_search(graph, attrs, idx.codes(), {"pq_lut": lut}, groutes, threads=8, **params)
    ri, rd = O.rerank(w.base, dt, w.queries, attrs, groutes, bi, 10)
    pi, _ = O.posting_scan(idx.codes(), {"pq_lut": lut}, attrs, proutes, A.SCORER_PQ, idx.posting_ids,
                           plan.posting_begin, plan.posting_count, shortlist)
    rpi, rpd = O.rerank(w.base, dt, w.queries, attrs, proutes, pi, 10)
    qoff, order = plan.merge_tables()
    return O.route_merge(np.concatenate([ri, rpi]), np.concatenate([rd, rpd]), qoff, order, 10)


@pytest.mark.gpu
@pytest.mark.parametrize("wl", ["cfg2_u8", "cfg2_u8_predicates", "cfg1_lut"])
def test_batch_driver_matches_oracle(tmp_path, wl):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from fixtures import cfg1_small, cfg2_small_u8cb, fbits, with_predicates
    from oracle import oracle as O
    w, idx, plan = cfg1_small() if wl == "cfg1_lut" else cfg2_small_u8cb(48)
    attrs, graph, groutes, proutes = idx.attrs(), idx.graph(), plan.graph_routes, plan.posting_routes
    if wl == "cfg2_u8_predicates":
        attrs, graph, groutes, _ = with_predicates(w, idx, plan.graph_routes, seed=3)
        _, _, proutes, _ = with_predicates(w, idx, plan.posting_routes, seed=4)
    mode = A.PQ_LUT_GLOBAL if wl == "cfg1_lut" else A.PQ_U8
    params = dict(queue_size=64, stop_width=10, result_width=100, finish_limit=100,
                  early_stop_mode=A.EARLY_STOP_ADAPTIVE, predicate_bias=1, alpha=0.15)
    arrays, scalars = batch_inputs(w, idx, plan, attrs, graph, groutes, proutes)
    scalars.update(params, pq_mode=mode, posting_shortlist=100, topk=10, scorer=A.SCORER_PQ)
    ids, dists = run_driver(tmp_path, arrays, scalars, w.queries.shape[0])
    lut = O.pq_build_lut(w.queries.astype(np.float32), idx.pq_centroids, idx.pq_codes.shape[1])
    wi, wd = _oracle_pipeline(w, idx, plan, attrs, graph, groutes, proutes, lut, params, 100)
    if w.base.dtype == np.uint8:
        assert np.array_equal(ids, wi) and np.array_equal(fbits(dists), fbits(wd))
    else:
        from test_gpu_parity import _ties_equivalent
        assert _ties_equivalent(ids, dists, wi, wd, 1e-5)
    assert (ids != A.U32MAX).sum() > 0.9 * ids.size


@pytest.mark.gpu
@pytest.mark.parametrize("entries", [0, 1])
def test_batch_driver_rabitq(tmp_path, entries):
    """RaBitQ batch: rotation and centroid distances on the tensor cores
    inside the call.  Against the oracle traversal, posting scans, rerank and
    merge run on the prepared state the library's preparation kernels give
    (the same calls, so the same bits)."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from fixtures import dev, random_orthogonal, rabitq_artifacts
    from oracle import oracle as O
    w, idx, plan, rq, anchors, qr = rabitq_artifacts(dim=480, n_queries=96)
    pd = qr.shape[1]
    rot = random_orthogonal(pd, 3)[: w.dim].astype(np.float32)  # the fixture's rotation, rows of the real dims
    L = A.lib()
    # prepared state through the library's own preparation kernels
    dq = dev(w.queries.astype(np.float32))
    rotated = torch.empty((w.queries.shape[0], pd), dtype=torch.float32, device="cuda")
    nb = max(L.gofann_rabitq_gemm_scratch_bytes(w.queries.shape[0], w.dim, pd, A.GEMM_TF32X3),
             L.gofann_rabitq_gemm_scratch_bytes(w.queries.shape[0], pd, anchors.shape[0], A.GEMM_TF32X3))
    scratch = torch.empty(nb, dtype=torch.uint8, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    d_rot, d_anchors = dev(rot), dev(anchors)  # alive until the kernels have run
    A.check(L.gofann_rabitq_rotate(A.ptr(dq), w.queries.shape[0], w.dim, A.ptr(d_rot), pd, A.GEMM_TF32X3,
                                   A.ptr(rotated), A.ptr(scratch), nb, A.ptr(status), s), "rotate")
    n = w.queries.shape[0]
    q8 = torch.empty((n, pd), dtype=torch.int8, device="cuda")
    sc, k1 = torch.empty(n, device="cuda"), torch.empty(n, device="cuda")
    gd = torch.empty((n, anchors.shape[0]), device="cuda")
    A.check(L.gofann_rabitq_quantize(A.ptr(rotated), n, pd, A.ptr(q8), A.ptr(sc), A.ptr(k1), s), "quantize")
    A.check(L.gofann_rabitq_centroid_dist_tc(A.ptr(rotated), n, A.ptr(d_anchors), anchors.shape[0], pd,
                                             A.GEMM_TF32X3, A.ptr(gd), A.ptr(scratch), nb, A.ptr(status), s), "gd")
    torch.cuda.synchronize()
    hprep = {"rq_q8": q8.cpu().numpy(), "rq_scale": sc.cpu().numpy(), "rq_k1xsumq": k1.cpu().numpy(),
             "rq_centroid_dist": gd.cpu().numpy()}
    groutes = {k: v.copy() for k, v in plan.graph_routes.items()}
    # with entry points on, every graph route starts at its nearest anchor's
    # entry row: local row 0 of its group here (the seed rows differ)
    anchor_entry = np.zeros(anchors.shape[0], np.uint32)
    if entries:
        best = hprep["rq_centroid_dist"][groutes["query_row"]].argmin(1)
        groutes["start_local"] = anchor_entry[best]
    params = dict(queue_size=64, stop_width=10, result_width=100, finish_limit=100,
                  early_stop_mode=A.EARLY_STOP_ADAPTIVE, predicate_bias=1, alpha=0.15, scorer=A.SCORER_RABITQ)
    bi, _, _, _ = O.beam_search(idx.graph(), idx.attrs(), rq, hprep, groutes, threads=8, **params)
    ri, rd = O.rerank(w.base, A.DTYPE_F32, w.queries, idx.attrs(), groutes, bi, 10)
    pi, _ = O.posting_scan(rq, hprep, idx.attrs(), plan.posting_routes, A.SCORER_RABITQ, idx.posting_ids,
                           plan.posting_begin, plan.posting_count, 100)
    rpi, rpd = O.rerank(w.base, A.DTYPE_F32, w.queries, idx.attrs(), plan.posting_routes, pi, 10)
    qoff, order = plan.merge_tables()
    wi, wd = O.route_merge(np.concatenate([ri, rpi]), np.concatenate([rd, rpd]), qoff, order, 10)

    arrays, scalars = batch_inputs(w, idx, plan)
    arrays.update({"codes.rq_codes": rq["rq_codes"], "codes.rq_factors": rq["rq_factors"],
                   "codes.rq_anchor_ids": rq["rq_anchor_ids"], "rq_rotation": rot, "rq_anchors": anchors,
                   "rq_anchor_entry": anchor_entry, "queries": w.queries.astype(np.float32),
                   "base": w.base.astype(np.float32)})
    scalars.update({k: v for k, v in params.items()}, pq_mode=0, posting_shortlist=100, topk=10,
                   rq_entries=entries, base_dtype=A.DTYPE_F32)
    scalars["codes.padded_dim"], scalars["codes.num_anchors"] = pd, int(anchors.shape[0])
    ids, dists = run_driver(tmp_path, arrays, scalars, n)
    from test_gpu_parity import _ties_equivalent
    assert _ties_equivalent(ids, dists, wi, wd, 1e-5)
    assert np.array_equal(ids == A.U32MAX, wi == A.U32MAX)
    assert np.all(np.abs(dists[wi != A.U32MAX] - wd[wi != A.U32MAX]) <= 1e-5 * np.abs(wd[wi != A.U32MAX]))
