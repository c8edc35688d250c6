"""Ordered range postings: the FARPIDX1 file, slice selection and segment plans.

Format (the reference's range posting index, src/index/range_posting_index.h:
12-50, loader range_posting_index.cpp:147-260): a 40-byte packed header
(magic "FARPIDX1", version 1, header bytes, file bytes, row count, range
count, reserved) followed by one 72-byte descriptor per range dimension
(range index, reserved, unique count, row count, then offset and byte size of
the dimension's unique values (f32, strictly increasing), value offsets (u64,
unique count + 1, from 0 to row count) and sample ids (u32, a permutation of
the rows ordered by value)).  The file is memory-mapped read-only; every
check the reference's loader makes is made here, with the same messages.

choose_smallest_slice (range_posting_index.cpp:270-310): for every active
range dimension of a query the rows satisfying its atom are one contiguous
slice of that dimension's sample ids -- mode 1 (v > lower) from
upper_bound(lower), mode 2 (v < upper) up to lower_bound(upper), mode 3
(lower <= v < upper) from lower_bound(lower) to the first value >= upper
after it -- and the query scans the smallest one (ties: the lowest
dimension).

make_plan (src/execution/posting_segment_plan.h:20-52): a slice is split into
ceil(rows / target) segments of near-equal size (sizes differ by at most
one; an empty slice keeps one empty segment), each scanned separately; the
union of the segments' shortlists contains the slice's shortlist, which
gofann_segment_merge recovers.
"""
from __future__ import annotations

import mmap
import os
import struct
from dataclasses import dataclass

import numpy as np

MAGIC = b"FARPIDX1"
VERSION = 1
HEADER = struct.Struct("<8sIIQQII")              # 40 bytes
DESCRIPTOR = struct.Struct("<IIQQQQQQQQ")        # 72 bytes
ALIGN = 64


class RangePostingError(ValueError):
    pass


def _fail(msg: str):
    raise RangePostingError("range posting index failed: " + msg)


def _align(x: int) -> int:
    return (x + ALIGN - 1) // ALIGN * ALIGN


def write(path, values: np.ndarray) -> None:
    """FARPIDX1 file of the attribute matrix values [rows][range_count]
    (float32): per dimension the unique values, their offsets and the sample
    ids ordered by (value, id)."""
    values = np.ascontiguousarray(values, np.float32)
    if values.ndim != 2 or values.shape[0] == 0 or values.shape[1] == 0:
        _fail("values must be a non-empty [rows][range_count] matrix")
    rows, rc = values.shape
    if not np.all(np.isfinite(values)):
        _fail("attribute values must be finite")
    dims = []
    for d in range(rc):
        col = values[:, d]
        ids = np.lexsort((np.arange(rows), col)).astype(np.uint32)
        uniq, counts = np.unique(col, return_counts=True)
        offs = np.zeros(uniq.shape[0] + 1, np.uint64)
        offs[1:] = np.cumsum(counts, dtype=np.uint64)
        dims.append((uniq.astype(np.float32), offs, ids))
    header_bytes = HEADER.size + rc * DESCRIPTOR.size
    cursor = _align(header_bytes)
    descs, blobs = [], []
    for d, (u, o, ids) in enumerate(dims):
        vo = cursor
        cursor = _align(cursor + u.nbytes)
        oo = cursor
        cursor = _align(cursor + o.nbytes)
        so = cursor
        cursor = _align(cursor + ids.nbytes)
        descs.append(DESCRIPTOR.pack(d, 0, u.shape[0], rows, vo, oo, so, u.nbytes, o.nbytes, ids.nbytes))
        blobs += [(vo, u), (oo, o), (so, ids)]
    buf = bytearray(cursor)
    buf[:HEADER.size] = HEADER.pack(MAGIC, VERSION, header_bytes, cursor, rows, rc, 0)
    for i, dsc in enumerate(descs):
        buf[HEADER.size + i * DESCRIPTOR.size: HEADER.size + (i + 1) * DESCRIPTOR.size] = dsc
    for off, arr in blobs:
        buf[off: off + arr.nbytes] = arr.tobytes()
    with open(path, "wb") as f:
        f.write(buf)


@dataclass
class Dimension:
    range_index: int
    unique_values: np.ndarray   # f32 [unique]
    offsets: np.ndarray         # u64 [unique + 1]
    sample_ids: np.ndarray      # u32 [rows]


@dataclass
class Index:
    row_count: int
    dimensions: list
    _map: object = None

    @property
    def range_count(self) -> int:
        return len(self.dimensions)


def _array(mm, offset: int, nbytes: int, count: int, dtype, file_bytes: int, name: str) -> np.ndarray:
    item = np.dtype(dtype).itemsize
    if nbytes != count * item:
        _fail(f"{name} byte count does not match element count")
    if offset % item != 0 or offset > file_bytes or nbytes > file_bytes - offset:
        _fail(f"{name} region is unaligned or outside the file")
    return np.frombuffer(mm, dtype=dtype, count=count, offset=offset)


def load(path) -> Index:
    """Memory-maps and validates a FARPIDX1 file."""
    file_bytes = os.path.getsize(path)
    if file_bytes < HEADER.size:
        _fail("file is too small or exceeds the host address range")
    with open(path, "rb") as f:
        mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
    magic, version, header_bytes, hdr_file_bytes, rows, rc, _ = HEADER.unpack_from(mm, 0)
    if magic != MAGIC:
        _fail("magic mismatch")
    if version != VERSION:
        _fail(f"unsupported version {version}")
    if hdr_file_bytes != file_bytes:
        _fail("header file size does not match the actual file")
    if rows == 0 or rows > 0xFFFFFFFF:
        _fail("row count must fit nonzero uint32 sample ids")
    if rc == 0:
        _fail("range count must be nonzero")
    desc_bytes = rc * DESCRIPTOR.size
    if header_bytes != HEADER.size + desc_bytes or desc_bytes > file_bytes - HEADER.size:
        _fail("descriptor table size is invalid")
    dims = []
    for d in range(rc):
        (ri, reserved, uc, rcount, vo, oo, so, vb, ob, sb) = DESCRIPTOR.unpack_from(mm, HEADER.size + d * DESCRIPTOR.size)
        if ri != d or reserved != 0:
            _fail("dimension descriptors must be dense, ordered, and reserved-zero")
        if rcount != rows or uc == 0 or uc > rcount:
            _fail("dimension row count mismatch or invalid value-domain size")
        vals = _array(mm, vo, vb, uc, np.float32, file_bytes, "unique values")
        offs = _array(mm, oo, ob, uc + 1, np.uint64, file_bytes, "value offsets")
        ids = _array(mm, so, sb, rcount, np.uint32, file_bytes, "sample ids")
        if not np.all(np.isfinite(vals)) or (uc > 1 and not np.all(vals[1:] > vals[:-1])):
            _fail("unique values must be finite and strictly increasing")
        if offs[0] != 0 or offs[-1] != rcount:
            _fail("value offsets must begin at zero and end at row_count")
        if np.any(offs[1:] < offs[:-1]) or np.any(offs > rcount):
            _fail("value offsets must be monotonic and in range")
        if np.any(ids >= rcount):
            _fail("sample id is outside the base row range")
        if np.unique(ids).shape[0] != rcount:
            _fail("sample ids must form a permutation without duplicates")
        dims.append(Dimension(d, vals, offs, ids))
    return Index(int(rows), dims, mm)


@dataclass
class Slices:
    has_active_range: np.ndarray      # bool [queries]
    active_dimension_count: np.ndarray
    range_index: np.ndarray           # u32, UINT32_MAX when inactive
    begin: np.ndarray                 # u64
    count: np.ndarray                 # u64 (0 when inactive)


def slice_bounds(dim: Dimension, mode: np.ndarray, lower: np.ndarray, upper: np.ndarray):
    """[begin, end) rows of dim.sample_ids satisfying each query's atom."""
    v = dim.unique_values
    n = v.shape[0]
    first = np.zeros(mode.shape[0], np.int64)
    last = np.full(mode.shape[0], n, np.int64)
    m1, m2, m3 = mode == 1, mode == 2, mode == 3
    first[m1] = np.searchsorted(v, lower[m1], side="right")
    last[m2] = np.searchsorted(v, upper[m2], side="left")
    first[m3] = np.searchsorted(v, lower[m3], side="left")
    last[m3] = np.maximum(first[m3], np.searchsorted(v, upper[m3], side="left"))
    bad = (mode != 0) & ~(m1 | m2 | m3)
    if bad.any():
        _fail(f"unknown active query range mode {int(mode[bad][0])}")
    return dim.offsets[first], dim.offsets[last]


def choose_smallest_slice(index: Index, modes: np.ndarray, lower: np.ndarray, upper: np.ndarray) -> Slices:
    """Per query (rows of the [queries][range_count] tables) the smallest
    slice among its active range dimensions (ties: lowest dimension)."""
    modes = np.asarray(modes, np.uint8)
    nq, rc = modes.shape
    if rc != index.range_count:
        _fail("query and posting range counts do not match")
    best_count = np.full(nq, np.iinfo(np.uint64).max, np.uint64)
    best_begin = np.zeros(nq, np.uint64)
    best_dim = np.full(nq, 0xFFFFFFFF, np.uint32)
    active = np.zeros(nq, np.uint32)
    for d in range(rc):
        m = modes[:, d]
        on = m != 0
        if not on.any():
            continue
        active += on
        b, e = slice_bounds(index.dimensions[d], m, np.asarray(lower, np.float32)[:, d],
                            np.asarray(upper, np.float32)[:, d])
        cnt = (e - b).astype(np.uint64)
        take = on & (cnt < best_count)  # strict: equal counts keep the lower dimension
        best_count[take] = cnt[take]
        best_begin[take] = b[take]
        best_dim[take] = d
    has = active > 0
    best_count[~has] = 0
    best_begin[~has] = 0
    best_dim[~has] = 0xFFFFFFFF
    return Slices(has, active, best_dim, best_begin, best_count)


@dataclass
class SegmentPlan:
    route_ids: np.ndarray        # u32 [segments]
    query_positions: np.ndarray  # u32 [segments]: position of the segment's slice in the input
    offsets: np.ndarray          # u64 [segments]
    sizes: np.ndarray            # u64 [segments]
    query_indptr: np.ndarray     # u32 [slices + 1]


def make_plan(route_ids, offsets, sizes, target_rows: int) -> SegmentPlan:
    """Near-equal segments of at most target_rows rows per slice."""
    route_ids = np.asarray(route_ids, np.uint32)
    offsets = np.asarray(offsets, np.uint64)
    sizes = np.asarray(sizes, np.uint64)
    if target_rows <= 0 or not (route_ids.shape == offsets.shape == sizes.shape):
        raise ValueError("invalid posting segment plan inputs")
    if np.any(offsets > np.iinfo(np.uint64).max - sizes):
        raise OverflowError("posting segment offset overflow")
    rows = sizes.astype(object)  # exact for any u64
    count = np.array([1 if r == 0 else 1 + (r - 1) // target_rows for r in rows], dtype=object)
    if int(count.sum()) > 0xFFFFFFFF:
        raise OverflowError("posting segment count exceeds uint32 range")
    cnt = count.astype(np.int64)
    seg_q = np.repeat(np.arange(route_ids.shape[0], dtype=np.int64), cnt)
    part = np.arange(seg_q.shape[0], dtype=np.int64) - np.repeat(np.cumsum(cnt) - cnt, cnt)
    width = (sizes // cnt.astype(np.uint64))[seg_q]
    rem = (sizes % cnt.astype(np.uint64))[seg_q]
    p = part.astype(np.uint64)
    seg_off = offsets[seg_q] + p * width + np.minimum(p, rem)
    seg_size = width + (p < rem).astype(np.uint64)
    indptr = np.zeros(route_ids.shape[0] + 1, np.uint32)
    indptr[1:] = np.cumsum(cnt)
    return SegmentPlan(route_ids[seg_q], seg_q.astype(np.uint32), seg_off, seg_size, indptr)
