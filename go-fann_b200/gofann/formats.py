"""On-disk index formats of the reference, so that its prepared datasets can
be loaded into the device index directly.

Each reader makes the checks the reference's loader makes (and fails with
FormatError); each writer produces files the reference reads.

  * graph.bin, "FDRG" block format (src/index/graph_file_format.h:10-25,
    graph_file_format.cpp:60-170): a 4096-byte header block (magic
    0x47524446, version 1, block size 4096, header size 4096, rows, degree,
    row bytes = 4 * degree, rows per block = 4096 // row bytes), then
    4096-byte blocks each packing rows_per_block adjacency rows of uint32,
    the last block zero-padded.  The legacy layout (u64 rows, u64 degree,
    rows x degree uint32) converts to it (graph_file_format.cpp:180-250).
  * .spmat label matrices (load_spmat_labels, src/data/dataloader.cpp:
    6663-6777): u64 rows, u64 cols, u64 nnz, indptr u64[rows + 1], indices
    u32[nnz]; indptr starts at 0, is monotonic and bounded by nnz, every
    label is below cols; rows are sorted and de-duplicated on load (a row
    limit reads a prefix).
  * the native RaBitQ artifact (save_rabitq_index / load_rabitq_index,
    src/search/rabitq/backend_rabitq.cu:2748-2847, header and codec structs
    backend_rabitq.cuh:16-32, checks :1213-1250): a 24-byte header (version
    2, dim, num_anchors, code bytes, u64 points), a 28-byte codec spec
    (padded dim, bits per dim, short code words, long code bytes, layout
    flags, 3 short and 2 extra factors), then eight u64-length-prefixed
    vectors: anchors f32, rotation f32, query scaling factors f32[2], anchor
    ids u32, codes u8, long codes u8, factors f32, extra factors f32.
  * PQ pivots and codes in the DiskANN bin layout (load_pq_pivots_local,
    src/search/pq/backend_pq.cu:1717-1795; pq.codes.bin,
    tools/quantization/pq_builder.cu:123): a bin block is an int32 row count,
    an int32 column count and the row-major payload; the pivots file starts
    with a bin block of 4 (or, old layout, 5) u64 offsets locating the
    256 x dim pivot table, the dim-long centroid and the chunk offsets
    (num_chunks + 1 rows of u32).  The codebook the search uses is pivots +
    centroid (backend_pq.cu:1812-1815).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass

import numpy as np


class FormatError(ValueError):
    pass


# ------------------------------------------------------------------ FDRG graph
GRAPH_MAGIC = 0x47524446  # "FDRG"
GRAPH_VERSION = 1
GRAPH_BLOCK = 4096
GRAPH_HEADER = struct.Struct("<IIIIQIIQ")  # 40 bytes, then zero padding to 4096


@dataclass
class GraphHeader:
    rows: int
    degree: int
    row_size_bytes: int
    rows_per_block: int


def _gfail(msg):
    raise FormatError("graph file format failed: " + msg)


def write_graph(path, adjacency: np.ndarray) -> GraphHeader:
    """FDRG file of adjacency [rows][degree] (uint32)."""
    adj = np.ascontiguousarray(adjacency, np.uint32)
    if adj.ndim != 2 or adj.shape[1] == 0:
        _gfail(f"degree must be > 0 for graph file output {path}")
    rows, degree = adj.shape
    row_bytes = degree * 4
    rpb = GRAPH_BLOCK // row_bytes if row_bytes <= GRAPH_BLOCK else 0
    if rpb == 0:
        _gfail(f"degree too large for 4KB block packing in {path}")
    blocks = (rows + rpb - 1) // rpb
    payload = np.zeros((blocks, GRAPH_BLOCK), np.uint8)
    if rows:
        padded = np.zeros((blocks * rpb, degree), np.uint32)
        padded[:rows] = adj
        payload[:, :rpb * row_bytes] = padded.reshape(blocks, rpb * degree).view(np.uint8)
    header = bytearray(GRAPH_BLOCK)
    GRAPH_HEADER.pack_into(header, 0, GRAPH_MAGIC, GRAPH_VERSION, GRAPH_BLOCK, GRAPH_BLOCK, rows, degree, row_bytes,
                           rpb)
    with open(path, "wb") as f:
        f.write(header)
        f.write(payload.tobytes())
    return GraphHeader(rows, degree, row_bytes, rpb)


def read_graph_header(path) -> GraphHeader:
    with open(path, "rb") as f:
        raw = f.read(GRAPH_HEADER.size)
    if len(raw) < GRAPH_HEADER.size:
        _gfail(f"failed to read graph file header from {path}")
    magic, version, block, hsize, rows, degree, row_bytes, rpb = GRAPH_HEADER.unpack(raw)
    if magic != GRAPH_MAGIC:
        _gfail(f"invalid magic in graph file {path}")
    if version != GRAPH_VERSION:
        _gfail(f"unsupported graph file version in {path}")
    if block != GRAPH_BLOCK or hsize != GRAPH_BLOCK:
        _gfail(f"unexpected block/header size in {path}")
    if degree == 0:
        _gfail(f"degree must be > 0 in {path}")
    if row_bytes != degree * 4:
        _gfail(f"row_size_bytes does not match degree in {path}")
    want = GRAPH_BLOCK // row_bytes if row_bytes <= GRAPH_BLOCK else 0
    if want == 0 or rpb != want:
        _gfail(f"rows_per_block is invalid in {path}")
    return GraphHeader(rows, degree, row_bytes, rpb)


def has_graph_magic(path) -> bool:
    with open(path, "rb") as f:
        raw = f.read(4)
    if len(raw) < 4:
        _gfail(f"unable to read format marker from {path}")
    return struct.unpack("<I", raw)[0] == GRAPH_MAGIC


def graph_row_offset(h: GraphHeader, row: int) -> int:
    """Byte offset of a row in the file (graph_file_row_offset_bytes)."""
    return GRAPH_BLOCK + (row // h.rows_per_block) * GRAPH_BLOCK + (row % h.rows_per_block) * h.row_size_bytes


def load_graph(path) -> np.ndarray:
    """adjacency [rows][degree] uint32 of an FDRG file (every block read in
    full, as load_graph_file_as_contiguous_matrix does)."""
    h = read_graph_header(path)
    blocks = (h.rows + h.rows_per_block - 1) // h.rows_per_block
    raw = np.fromfile(path, np.uint8, count=blocks * GRAPH_BLOCK, offset=GRAPH_BLOCK) if blocks else \
        np.zeros(0, np.uint8)
    if raw.shape[0] != blocks * GRAPH_BLOCK:
        _gfail(f"failed reading graph file block from {path}")
    rows = raw.reshape(blocks, GRAPH_BLOCK)[:, :h.rows_per_block * h.row_size_bytes]
    return np.ascontiguousarray(rows).view(np.uint32).reshape(-1, h.degree)[:h.rows].copy()


def load_legacy_graph(path) -> np.ndarray:
    with open(path, "rb") as f:
        hdr = f.read(16)
        if len(hdr) < 16:
            _gfail(f"failed to read legacy graph header from {path}")
        rows, cols = struct.unpack("<QQ", hdr)
        if cols == 0 or cols > 0xFFFFFFFF:
            _gfail(f"invalid degree in legacy graph {path}")
        data = np.fromfile(f, np.uint32, count=rows * cols)
    if data.shape[0] != rows * cols:
        _gfail(f"failed reading row payload from {path}")
    return data.reshape(rows, cols)


def convert_legacy_graph(legacy_path, graph_path) -> GraphHeader:
    return write_graph(graph_path, load_legacy_graph(legacy_path))


# ------------------------------------------------------------- .spmat labels
def _sfail(msg):
    raise FormatError("graph load failed: " + msg)


def write_spmat(path, indptr: np.ndarray, indices: np.ndarray, cols: int) -> None:
    indptr = np.ascontiguousarray(indptr, np.uint64)
    indices = np.ascontiguousarray(indices, np.uint32)
    with open(path, "wb") as f:
        f.write(struct.pack("<QQQ", indptr.shape[0] - 1, cols, indices.shape[0]))
        f.write(indptr.tobytes())
        f.write(indices.tobytes())


def load_spmat(path, row_limit: int = 0):
    """(indptr u64 [rows+1], indices u32, cols) with every row sorted and
    de-duplicated; a row limit reads the first row_limit rows."""
    with open(path, "rb") as f:
        hdr = f.read(24)
        if len(hdr) < 24:
            _sfail(f"invalid spmat header in {path}")
        rows, cols, nnz = struct.unpack("<QQQ", hdr)
        if rows > 0xFFFFFFFF:
            _sfail(f"spmat row count exceeds uint32 range in {path}")
        if cols > 0xFFFFFFFF:
            _sfail(f"spmat label count exceeds uint32 range in {path}")
        eff = row_limit if 0 < row_limit < rows else rows
        indptr = np.fromfile(f, np.uint64, count=eff + 1)
        if indptr.shape[0] != eff + 1:
            _sfail(f"failed to read spmat indptr from {path}")
        if indptr[0] != 0:
            _sfail(f"spmat indptr must start at 0 in {path}")
        if np.any(indptr[:-1] > indptr[1:]):
            _sfail(f"spmat indptr is not monotonic in {path}")
        if np.any(indptr[1:] > nnz):
            _sfail(f"spmat indptr exceeds nnz in {path}")
        f.seek(24 + (rows + 1) * 8)
        n_eff = int(indptr[eff])
        indices = np.fromfile(f, np.uint32, count=n_eff)
    if indices.shape[0] != n_eff:
        _sfail(f"failed to read spmat indices from {path}")
    if n_eff and int(indices.max()) >= cols:
        _sfail(f"spmat label index out of range in {path}")
    row_of = np.repeat(np.arange(eff, dtype=np.int64), np.diff(indptr).astype(np.int64))
    order = np.lexsort((indices, row_of))
    r, lab = row_of[order], indices[order]
    keep = np.ones(lab.shape[0], bool)
    keep[1:] = (r[1:] != r[:-1]) | (lab[1:] != lab[:-1])
    r, lab = r[keep], lab[keep]
    out_ptr = np.zeros(eff + 1, np.uint64)
    out_ptr[1:] = np.cumsum(np.bincount(r, minlength=eff))
    return out_ptr, lab.astype(np.uint32), int(cols)


# ------------------------------------------------------- native RaBitQ artifact
RQ_VERSION = 2
RQ_HEADER = struct.Struct("<IIIIQ")          # 24 bytes
RQ_CODEC = struct.Struct("<IIIIIII")         # 28 bytes
RQ_LAYOUT_SAMPLE_MAJOR, RQ_LAYOUT_MSB32, RQ_LAYOUT_CUVS_FACTORS = 1, 2, 4
RQ_FIELDS = (("anchors", np.float32), ("rotation", np.float32), ("query_scaling_factors", np.float32),
             ("anchor_ids", np.uint32), ("codes", np.uint8), ("long_codes", np.uint8), ("factors", np.float32),
             ("ex_factors", np.float32))


def _rfail(msg):
    raise FormatError("rabitq backend failed: " + msg)


def rq_codec(dim: int, bits_per_dim: int = 1) -> dict:
    """make_codec_spec (backend_rabitq.cu:1196-1211)."""
    if bits_per_dim == 0 or bits_per_dim > 9:
        _rfail("bits_per_dim must be in [1, 9]")
    pd = (dim + 63) // 64 * 64
    return dict(padded_dim=pd, bits_per_dim=bits_per_dim, short_code_words=(pd + 31) // 32,
                long_code_bytes=0 if bits_per_dim <= 1 else pd * (bits_per_dim - 1) // 8,
                layout_flags=RQ_LAYOUT_SAMPLE_MAJOR | RQ_LAYOUT_MSB32 | RQ_LAYOUT_CUVS_FACTORS,
                short_factor_count=3, ex_factor_count=2)


def _rq_validate(h: dict, c: dict) -> None:
    if h["version"] != RQ_VERSION:
        _rfail("unsupported artifact version")
    if h["dim"] == 0 or h["num_anchors"] == 0 or h["num_points"] == 0:
        _rfail("artifact header contains zero-sized fields")
    pd = c["padded_dim"]
    if pd < h["dim"] or pd % 64:
        _rfail("artifact codec padded_dim is invalid")
    if c["bits_per_dim"] == 0 or c["bits_per_dim"] > 9:
        _rfail("artifact codec bits_per_dim is invalid")
    if c["short_code_words"] != (pd + 31) // 32:
        _rfail("artifact codec short_code_words is invalid")
    if c["long_code_bytes"] != (0 if c["bits_per_dim"] <= 1 else pd * (c["bits_per_dim"] - 1) // 8):
        _rfail("artifact codec long_code_bytes is invalid")
    req = RQ_LAYOUT_SAMPLE_MAJOR | RQ_LAYOUT_MSB32 | RQ_LAYOUT_CUVS_FACTORS
    if c["layout_flags"] & req != req:
        _rfail("artifact codec layout_flags are invalid")
    if c["short_factor_count"] != 3 or c["ex_factor_count"] != 2:
        _rfail("artifact codec factor counts are invalid")
    if h["code_bytes"] != 4 * ((pd + 31) // 32):
        _rfail("artifact header code_bytes does not match dim")


def write_rabitq_artifact(path, dim: int, anchors, rotation, anchor_ids, codes, factors,
                          query_scaling_factors=(1.0, 1.0), long_codes=None, ex_factors=None) -> None:
    """Native RaBitQ artifact of a 1-bit index: anchors [A][padded_dim],
    rotation [padded_dim][padded_dim], codes [n][padded_dim / 8] (32-bit
    words, dimension d at bit 31 - d % 32 of word d / 32), factors [n][3]."""
    c = rq_codec(dim)
    n = int(np.asarray(anchor_ids).shape[0])
    h = dict(version=RQ_VERSION, dim=dim, num_anchors=int(np.asarray(anchors).shape[0]), code_bytes=4 *
             c["short_code_words"], num_points=n)
    _rq_validate(h, c)
    vals = dict(anchors=anchors, rotation=rotation, query_scaling_factors=np.asarray(query_scaling_factors),
                anchor_ids=anchor_ids, codes=codes,
                long_codes=np.zeros(0, np.uint8) if long_codes is None else long_codes, factors=factors,
                ex_factors=np.zeros(n * 2, np.float32) if ex_factors is None else ex_factors)
    with open(path, "wb") as f:
        f.write(RQ_HEADER.pack(h["version"], h["dim"], h["num_anchors"], h["code_bytes"], h["num_points"]))
        f.write(RQ_CODEC.pack(*(c[k] for k in ("padded_dim", "bits_per_dim", "short_code_words", "long_code_bytes",
                                               "layout_flags", "short_factor_count", "ex_factor_count"))))
        for name, dt in RQ_FIELDS:
            a = np.ascontiguousarray(vals[name], dt).reshape(-1)
            f.write(struct.pack("<Q", a.shape[0]))
            f.write(a.tobytes())


def load_rabitq_artifact(path) -> dict:
    """Header, codec and arrays of a native RaBitQ artifact, shaped: anchors
    [A][padded_dim], rotation [padded_dim][padded_dim], anchor_ids [n], codes
    [n][code_bytes], factors [n][3], ex_factors [n][2]."""
    with open(path, "rb") as f:
        raw = f.read(RQ_HEADER.size)
        if len(raw) < RQ_HEADER.size:
            _rfail("failed to read artifact header")
        h = dict(zip(("version", "dim", "num_anchors", "code_bytes", "num_points"), RQ_HEADER.unpack(raw)))
        raw = f.read(RQ_CODEC.size)
        if len(raw) < RQ_CODEC.size:
            _rfail("failed to read artifact codec spec")
        c = dict(zip(("padded_dim", "bits_per_dim", "short_code_words", "long_code_bytes", "layout_flags",
                      "short_factor_count", "ex_factor_count"), RQ_CODEC.unpack(raw)))
        _rq_validate(h, c)
        out = {}
        for name, dt in RQ_FIELDS:
            raw = f.read(8)
            if len(raw) < 8:
                _rfail("failed to read artifact payload")
            size = struct.unpack("<Q", raw)[0]
            a = np.fromfile(f, dt, count=size)
            if a.shape[0] != size:
                _rfail("failed to read artifact payload")
            out[name] = a
    n, pd, A = h["num_points"], c["padded_dim"], h["num_anchors"]
    want = dict(anchors=A * pd, rotation=pd * pd, query_scaling_factors=2, anchor_ids=n, codes=n * h["code_bytes"],
                long_codes=n * c["long_code_bytes"], factors=n * 3, ex_factors=n * 2)
    if any(out[k].shape[0] != v for k, v in want.items()):
        _rfail("artifact payload sizes do not match header")
    if n and int(out["anchor_ids"].max()) >= A:
        _rfail("artifact anchor_ids contain an out-of-range anchor id")
    out["anchors"] = out["anchors"].reshape(A, pd)
    out["rotation"] = out["rotation"].reshape(pd, pd)
    out["codes"] = out["codes"].reshape(n, h["code_bytes"])
    out["factors"] = out["factors"].reshape(n, 3)
    out["ex_factors"] = out["ex_factors"].reshape(n, 2)
    return dict(header=h, codec=c, **out)


# ------------------------------------------------------ PQ pivots and codes
def _pfail(msg):
    raise FormatError("pq backend failed: " + msg)


def _bin_block(arr: np.ndarray) -> bytes:
    a = np.ascontiguousarray(arr)
    r, c = (a.shape[0], a.shape[1]) if a.ndim == 2 else (a.shape[0], 1)
    return struct.pack("<ii", r, c) + a.tobytes()


def _read_bin(f, dtype, offset: int = 0, max_rows: int | None = None):
    f.seek(offset)
    raw = f.read(8)
    if len(raw) < 8:
        _pfail(f"failed to read bin header from {f.name}")
    r, c = struct.unpack("<ii", raw)
    r, c = max(0, r), max(0, c)
    n = r if max_rows is None else min(r, max_rows)
    a = np.fromfile(f, dtype, count=n * c)
    if a.shape[0] != n * c:
        _pfail(f"failed to read bin payload from {f.name}")
    return a.reshape(n, c)


def write_pq_pivots(path, pivots: np.ndarray, centroid: np.ndarray, chunk_offsets: np.ndarray) -> None:
    """Pivots file: the 4-offset table, then the bin blocks of pivots
    [256][dim] f32, centroid [dim][1] f32 and chunk offsets [M+1][1] u32."""
    blocks = [_bin_block(np.asarray(pivots, np.float32)),
              _bin_block(np.asarray(centroid, np.float32).reshape(-1, 1)),
              _bin_block(np.asarray(chunk_offsets, np.uint32).reshape(-1, 1))]
    table_len = 8 + 4 * 8
    offs, o = [], table_len
    for b in blocks:
        offs.append(o)
        o += len(b)
    offs.append(o)  # file end
    with open(path, "wb") as f:
        f.write(_bin_block(np.asarray(offs, np.uint64).reshape(-1, 1)))
        for b in blocks:
            f.write(b)


def load_pq_pivots(path, num_chunks: int = 0) -> dict:
    """(pivots [256][dim], centroid [dim], chunk_offsets [M+1], codebook =
    pivots + centroid [256][dim]) of a pivots file, as load_pq_pivots_local
    reads it (4 or 5 offsets; the old 5-offset layout keeps the chunk offsets
    at index 3)."""
    with open(path, "rb") as f:
        offs = _read_bin(f, np.uint64)
        if offs.shape[0] not in (4, 5):
            _pfail("unexpected pq pivots offset table size")
        old = offs.shape[0] == 5
        pivots = _read_bin(f, np.float32, int(offs[0, 0]))
        dim = pivots.shape[1]
        centroid = _read_bin(f, np.float32, int(offs[1, 0])).reshape(-1)
        co = _read_bin(f, np.uint32, int(offs[3 if old else 2, 0]))
    if co.shape[1] != 1 or (co.shape[0] != num_chunks + 1 and num_chunks != 0):
        _pfail("unexpected pq chunk offsets shape")
    if pivots.shape[0] != 256 or centroid.shape[0] != dim:
        _pfail("unexpected pq pivots shape")
    return dict(pivots=pivots, centroid=centroid, chunk_offsets=co.reshape(-1),
                codebook=(pivots + centroid[None, :]).astype(np.float32))


def write_pq_codes(path, codes: np.ndarray) -> None:
    """Compressed codes in the bin layout (int32 rows, int32 pq_dim, u8 payload)."""
    with open(path, "wb") as f:
        f.write(_bin_block(np.asarray(codes, np.uint8)))


def load_pq_codes(path, expected_rows: int | None = None) -> np.ndarray:
    """Codes [rows][pq_dim] (load_bin_prefix_local: at most expected_rows rows,
    which must all be present)."""
    with open(path, "rb") as f:
        codes = _read_bin(f, np.uint8, 0, expected_rows)
    if expected_rows is not None and codes.shape[0] != expected_rows:
        _pfail("compressed codes rows do not match expected rows")
    return codes
