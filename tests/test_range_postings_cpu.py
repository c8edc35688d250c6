"""Ordered range postings (FARPIDX1), slice selection and segment plans (no GPU).

Known answers are the reference's own (tests/native/range_posting_index_test.cpp:
the 6-row, 2-dimension index and its five query slices, and the corrupt
files its loader must reject; tests/native/posting_segment_test.cpp: the
segment plan of routes {7, 3, 11, 5} and the invalid inputs).  The
segmented scan is checked the way the reference checks it: the shortlist
of the merged segment shortlists equals the shortlist of the whole slice.
"""
import numpy as np
import pytest

from gofann import range_postings as RP
from oracle import oracle as O

# dimension 0: values {1, 2, 4}, rows in value order 0..5; dimension 1:
# values {10, 20, 30} held by rows {5}, {3, 4}, {0, 1, 2}
VALUES = np.array([[1, 30], [1, 30], [2, 30], [2, 20], [4, 20], [4, 10]], np.float32)


@pytest.fixture
def index_path(tmp_path):
    p = tmp_path / "valid.bin"
    RP.write(p, VALUES)
    return p


def test_layout_matches_the_reference_fixture(index_path):
    ix = RP.load(index_path)
    assert ix.row_count == 6 and ix.range_count == 2
    d0, d1 = ix.dimensions
    assert d0.unique_values.tolist() == [1.0, 2.0, 4.0] and d0.offsets.tolist() == [0, 2, 4, 6]
    assert d0.sample_ids.tolist() == [0, 1, 2, 3, 4, 5]
    assert d1.unique_values.tolist() == [10.0, 20.0, 30.0] and d1.offsets.tolist() == [0, 1, 3, 6]
    assert d1.sample_ids.tolist() == [5, 3, 4, 0, 1, 2]
    raw = index_path.read_bytes()
    assert raw[:8] == b"FARPIDX1" and len(raw) % 64 == 0


def test_choose_smallest_slice_known_answers(index_path):
    ix = RP.load(index_path)
    modes = np.zeros((5, 2), np.uint8)
    lo = np.zeros((5, 2), np.float32)
    hi = np.zeros((5, 2), np.float32)
    modes[0, 0], lo[0, 0] = 1, 2.0
    modes[1, 1], hi[1, 1] = 2, 20.0
    modes[2, 0], lo[2, 0], hi[2, 0] = 3, 2.0, 4.0
    modes[3, 0], lo[3, 0], hi[3, 0] = 3, 1.0, 4.0
    modes[3, 1], lo[3, 1], hi[3, 1] = 3, 10.0, 20.0
    s = RP.choose_smallest_slice(ix, modes, lo, hi)
    assert (s.range_index[0], s.begin[0], s.count[0]) == (0, 4, 2)
    assert (s.range_index[1], s.begin[1], s.count[1]) == (1, 0, 1)
    assert (s.range_index[2], s.begin[2], s.count[2]) == (0, 2, 2)
    assert s.active_dimension_count[3] == 2 and (s.range_index[3], s.begin[3], s.count[3]) == (1, 0, 1)
    assert not s.has_active_range[4] and s.count[4] == 0
    # the rows of each slice satisfy the atom (and the others do not)
    for q in range(4):
        d = s.range_index[q]
        rows = ix.dimensions[d].sample_ids[s.begin[q]:s.begin[q] + s.count[q]]
        v = VALUES[:, d]
        m, a, b = modes[q, d], lo[q, d], hi[q, d]
        want = {1: v > a, 2: v < b, 3: (v >= a) & (v < b)}[int(m)]
        assert sorted(rows.tolist()) == np.nonzero(want)[0].tolist()


def _patched(src, dst, offset, data):
    raw = bytearray(src.read_bytes())
    raw[offset:offset + len(data)] = data
    dst.write_bytes(bytes(raw))


def test_loader_rejects_corrupt_files(index_path, tmp_path):
    ix = RP.load(index_path)
    d0_desc = RP.HEADER.size
    cases = []
    p = tmp_path / "bad-magic.bin"
    _patched(index_path, p, 0, b"X")
    cases.append((p, "magic mismatch"))
    p = tmp_path / "bad-unique-count.bin"
    _patched(index_path, p, d0_desc + 8, np.uint64(7).tobytes())  # unique_count = row_count + 1
    cases.append((p, "value-domain size"))
    so = RP.DESCRIPTOR.unpack_from(index_path.read_bytes(), d0_desc)[6]
    p = tmp_path / "bad-id.bin"
    _patched(index_path, p, so + 5 * 4, np.uint32(6).tobytes())
    cases.append((p, "sample id"))
    p = tmp_path / "duplicate-id.bin"
    _patched(index_path, p, so + 5 * 4, np.uint32(0).tobytes())
    cases.append((p, "permutation"))
    p = tmp_path / "truncated.bin"
    p.write_bytes(index_path.read_bytes()[:-1])
    cases.append((p, "file size"))
    for path, needle in cases:
        with pytest.raises(RP.RangePostingError, match=needle):
            RP.load(path)
    assert ix.row_count == 6


def test_segment_plan_matches_reference_rules():
    routes = [7, 3, 11, 5]
    offsets = [0, 100, 1000, 30000]
    sizes = [0, 31, 20001, 8]
    plan = RP.make_plan(routes, offsets, sizes, 1024)
    for q in range(4):
        a, b = plan.query_indptr[q], plan.query_indptr[q + 1]
        assert b > a
        assert np.all(plan.route_ids[a:b] == routes[q])
        cursor = offsets[q]
        for p in range(a, b):
            assert plan.offsets[p] == cursor and plan.sizes[p] <= 1024
            cursor += int(plan.sizes[p])
        assert cursor == offsets[q] + sizes[q]
        assert int(plan.sizes[a:b].max()) - int(plan.sizes[a:b].min()) <= 1
    with pytest.raises(OverflowError):
        RP.make_plan([1], [np.iinfo(np.uint64).max], [1], 32)
    with pytest.raises(ValueError):
        RP.make_plan([1], [0], [1], 0)
    with pytest.raises(OverflowError):
        RP.make_plan([1], [0], [np.iinfo(np.uint64).max], 1)


@pytest.mark.parametrize("k", [10, 100, 400])
@pytest.mark.parametrize("target", [32, 1024])
def test_merged_segment_shortlists_equal_the_slice_shortlist(k, target):
    """The reference's segment property on its own tie-heavy scores
    (integers 0..399 for 21,007 ids), through the oracle's shortlist heap."""
    rng = np.random.default_rng(7123)
    scores = rng.integers(0, 400, size=21007).astype(np.float32)
    for rows in (0, 17, 21007):
        plan = RP.make_plan([0], [0], [rows], target)
        full_d, full_i = O.shortlist(scores[:rows], np.arange(rows, dtype=np.uint32), k)
        parts_d, parts_i = [], []
        for off, size in zip(plan.offsets, plan.sizes):
            ids = np.arange(int(off), int(off + size), dtype=np.uint32)
            d, i = O.shortlist(scores[ids], ids, k)
            parts_d.append(d)
            parts_i.append(i)
        md, mi = O.shortlist(np.concatenate(parts_d), np.concatenate(parts_i), k)
        assert np.array_equal(mi, full_i) and np.array_equal(md.view(np.uint32), full_d.view(np.uint32))
