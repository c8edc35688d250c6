"""On-disk formats (go-fann_b200/gofann/formats.py): round trips, the
reference loaders' checks, and -- where oracle/_ref is built -- FDRG files
exchanged with the reference's own graph_file_format.cpp in both
directions."""
import struct

import numpy as np
import pytest

from gofann import formats as F
from oracle import oracle as O


def _adj(rows, degree, seed=0):
    rng = np.random.default_rng(seed)
    a = rng.integers(0, max(rows, 1), size=(rows, degree)).astype(np.uint32)
    a[:, -1] = 0xFFFFFFFF
    return a


@pytest.mark.parametrize("rows,degree", [(0, 32), (1, 32), (31, 32), (32, 32), (33, 32), (1000, 64), (77, 24),
                                         (5, 1024)])
def test_graph_round_trip(tmp_path, rows, degree):
    a = _adj(rows, degree, rows)
    p = tmp_path / "g.bin"
    h = F.write_graph(p, a)
    assert h.rows_per_block == 4096 // (4 * degree)
    assert p.stat().st_size == 4096 * (1 + -(-rows // h.rows_per_block))
    assert F.has_graph_magic(p)
    got = F.load_graph(p)
    assert got.shape == (rows, degree) and np.array_equal(got, a)
    if rows:
        r = rows - 1
        with open(p, "rb") as f:
            f.seek(F.graph_row_offset(h, r))
            assert np.array_equal(np.frombuffer(f.read(4 * degree), np.uint32), a[r])


def test_graph_checks(tmp_path):
    p = tmp_path / "g.bin"
    F.write_graph(p, _adj(10, 32))
    raw = bytearray(p.read_bytes())
    for off, val, msg in [(0, 1, "invalid magic"), (4, 2, "unsupported graph file version"),
                          (8, 1024, "unexpected block/header size"), (24, 0, "degree must be > 0"),
                          (28, 12, "row_size_bytes does not match"), (32, 7, "rows_per_block is invalid")]:
        bad = bytearray(raw)
        struct.pack_into("<I", bad, off, val)
        q = tmp_path / "bad.bin"
        q.write_bytes(bytes(bad))
        with pytest.raises(F.FormatError, match=msg):
            F.load_graph(q)
    with pytest.raises(F.FormatError, match="degree too large"):
        F.write_graph(tmp_path / "x.bin", np.zeros((2, 1025), np.uint32))


def test_legacy_graph_conversion(tmp_path):
    a = _adj(300, 32, 3)
    leg = tmp_path / "legacy.bin"
    with open(leg, "wb") as f:
        f.write(struct.pack("<QQ", 300, 32))
        f.write(a.tobytes())
    F.convert_legacy_graph(leg, tmp_path / "g.bin")
    assert np.array_equal(F.load_graph(tmp_path / "g.bin"), a)


@pytest.mark.skipif(O.rlib() is None, reason="reference harness not built (oracle/_ref)")
@pytest.mark.parametrize("rows,degree", [(1, 32), (1000, 32), (513, 64)])
def test_graph_files_interchange_with_reference(tmp_path, rows, degree):
    import ctypes as C
    L = O.rlib()
    a = _adj(rows, degree, 7)
    err = C.create_string_buffer(512)
    ref_path = str(tmp_path / "ref.bin").encode()
    assert L.ref_graph_write(ref_path, a.ctypes.data, rows, degree, err, 512) == 0, err.value
    ours = tmp_path / "ours.bin"
    F.write_graph(ours, a)
    assert (tmp_path / "ref.bin").read_bytes() == ours.read_bytes()  # byte-identical files
    out = np.zeros(rows * degree, np.uint32)
    r, c = C.c_uint64(), C.c_uint64()
    assert L.ref_graph_load(str(ours).encode(), out.ctypes.data, out.shape[0], C.byref(r), C.byref(c), err, 512) == 0
    assert (r.value, c.value) == (rows, degree) and np.array_equal(out.reshape(rows, degree), a)
    assert np.array_equal(F.load_graph(tmp_path / "ref.bin"), a)


def test_spmat_round_trip_sorts_and_dedups(tmp_path):
    rows = [[5, 1, 5], [], [3], [9, 0, 2, 2, 9]]
    indptr = np.zeros(len(rows) + 1, np.uint64)
    indptr[1:] = np.cumsum([len(r) for r in rows])
    ind = np.concatenate([np.asarray(r, np.uint32) for r in rows])
    p = tmp_path / "l.spmat"
    F.write_spmat(p, indptr, ind, 10)
    ip, ix, cols = F.load_spmat(p)
    assert cols == 10
    assert ip.tolist() == [0, 2, 2, 3, 6] and ix.tolist() == [1, 5, 3, 0, 2, 9]
    ip2, ix2, _ = F.load_spmat(p, row_limit=2)
    assert ip2.tolist() == [0, 2, 2] and ix2.tolist() == [1, 5]


def test_spmat_checks(tmp_path):
    def w(indptr, ind, cols, nnz=None):
        p = tmp_path / "b.spmat"
        with open(p, "wb") as f:
            f.write(struct.pack("<QQQ", len(indptr) - 1, cols, len(ind) if nnz is None else nnz))
            f.write(np.asarray(indptr, np.uint64).tobytes())
            f.write(np.asarray(ind, np.uint32).tobytes())
        return p
    with pytest.raises(F.FormatError, match="must start at 0"):
        F.load_spmat(w([1, 2], [0, 0], 4))
    with pytest.raises(F.FormatError, match="not monotonic"):
        F.load_spmat(w([0, 2, 1], [0, 1], 4))
    with pytest.raises(F.FormatError, match="exceeds nnz"):
        F.load_spmat(w([0, 3], [0, 1], 4, nnz=2))
    with pytest.raises(F.FormatError, match="out of range"):
        F.load_spmat(w([0, 2], [0, 4], 4))


def test_rabitq_artifact_round_trip_and_checks(tmp_path):
    rng = np.random.default_rng(0)
    dim, n, A = 100, 50, 4
    c = F.rq_codec(dim)
    pd = c["padded_dim"]
    assert pd == 128 and c["short_code_words"] == 4
    anchors = rng.normal(size=(A, pd)).astype(np.float32)
    rot = rng.normal(size=(pd, pd)).astype(np.float32)
    ids = rng.integers(0, A, size=n).astype(np.uint32)
    codes = rng.integers(0, 256, size=(n, pd // 8)).astype(np.uint8)
    fac = rng.normal(size=(n, 3)).astype(np.float32)
    p = tmp_path / "rq.bin"
    F.write_rabitq_artifact(p, dim, anchors, rot, ids, codes, fac)
    a = F.load_rabitq_artifact(p)
    assert a["header"]["num_points"] == n and a["header"]["code_bytes"] == 16
    for k, v in (("anchors", anchors), ("rotation", rot), ("anchor_ids", ids), ("codes", codes), ("factors", fac)):
        assert np.array_equal(a[k], v), k
    raw = bytearray(p.read_bytes())
    bad = bytearray(raw)
    struct.pack_into("<I", bad, 0, 3)
    (tmp_path / "b1").write_bytes(bytes(bad))
    with pytest.raises(F.FormatError, match="unsupported artifact version"):
        F.load_rabitq_artifact(tmp_path / "b1")
    bad = bytearray(raw)
    struct.pack_into("<I", bad, 24 + 16, 0)  # layout flags
    (tmp_path / "b2").write_bytes(bytes(bad))
    with pytest.raises(F.FormatError, match="layout_flags"):
        F.load_rabitq_artifact(tmp_path / "b2")
    ids2 = ids.copy()
    ids2[3] = A
    F.write_rabitq_artifact(tmp_path / "b3", dim, anchors, rot, ids2, codes, fac)
    with pytest.raises(F.FormatError, match="out-of-range anchor"):
        F.load_rabitq_artifact(tmp_path / "b3")
    F.write_rabitq_artifact(tmp_path / "b4", dim, anchors, rot, ids, codes[:-1], fac)
    with pytest.raises(F.FormatError, match="sizes do not match"):
        F.load_rabitq_artifact(tmp_path / "b4")


def test_pq_pivots_and_codes(tmp_path):
    rng = np.random.default_rng(1)
    dim, M = 192, 48
    piv = rng.normal(size=(256, dim)).astype(np.float32)
    cen = rng.normal(size=dim).astype(np.float32)
    co = np.arange(0, dim + 1, dim // M, dtype=np.uint32)
    p = tmp_path / "pivots.bin"
    F.write_pq_pivots(p, piv, cen, co)
    got = F.load_pq_pivots(p, M)
    assert np.array_equal(got["pivots"], piv) and np.array_equal(got["centroid"], cen)
    assert np.array_equal(got["chunk_offsets"], co)
    assert np.array_equal(got["codebook"], piv + cen[None, :])
    with pytest.raises(F.FormatError, match="chunk offsets shape"):
        F.load_pq_pivots(p, M + 1)
    codes = rng.integers(0, 256, size=(1000, M)).astype(np.uint8)
    F.write_pq_codes(tmp_path / "c.bin", codes)
    assert np.array_equal(F.load_pq_codes(tmp_path / "c.bin", 1000), codes)
    assert np.array_equal(F.load_pq_codes(tmp_path / "c.bin", 10), codes[:10])
    with pytest.raises(F.FormatError, match="do not match expected rows"):
        F.load_pq_codes(tmp_path / "c.bin", 2000)
