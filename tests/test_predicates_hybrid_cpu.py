"""Config-4 predicate kinds on the CPU: the bit-parallel edit distance the
device runs (Myers 1999 in Hyyro's global form, restated here line for line
from go-fann_b200/csrc/common.cuh:myers_edit_distance) against the oracle's
dynamic programme, the library's match-table helper, and the oracle's
string / int64 atoms."""
import ctypes as C

import numpy as np
import pytest

from fixtures import cfg2_small, with_hybrid_predicates
from gofann import _abi as A
from oracle import oracle as O


def myers(pattern: bytes, text: bytes) -> int:
    m = len(pattern)
    if m == 0:
        return len(text)
    M32 = 0xFFFFFFFF
    peq = [0] * 128
    for i, ch in enumerate(pattern):
        peq[ch] |= 1 << i
    last = 1 << (m - 1)
    pv, mv, score = (M32 if m == 32 else (1 << m) - 1), 0, m
    for c in text:
        eq = peq[c] if c < 128 else 0
        xv = eq | mv
        xh = ((((eq & pv) + pv) & M32) ^ pv) | eq
        ph = (mv | (~(xh | pv) & M32)) & M32
        mh = pv & xh
        if ph & last:
            score += 1
        elif mh & last:
            score -= 1
        ph = ((ph << 1) | 1) & M32
        mh = (mh << 1) & M32
        pv = (mh | (~(xv | ph) & M32)) & M32
        mv = ph & xv
    return score


def test_myers_equals_dynamic_programme():
    rng = np.random.default_rng(0)
    alphabet = [b"ab", b"abc", b"abcdefghijklmnopqrstuvwxyz"]
    for trial in range(3000):
        al = alphabet[trial % 3]
        m = int(rng.integers(0, 33))
        n = int(rng.integers(0, 48))
        p = rng.choice(list(al), size=m).astype(np.uint8).tobytes()
        t = rng.choice(list(al) + [200], size=n).astype(np.uint8).tobytes()
        assert myers(p, t) == O.levenshtein(p, t), (p, t)


def test_string_peq_helper():
    L = A.lib()
    out = np.zeros(128, np.uint32)
    pat = np.frombuffer(b"abca", np.uint8).copy()
    assert L.gofann_string_peq(A.ptr(pat), 4, A.ptr(out)) == 0
    assert out[ord("a")] == 0b1001 and out[ord("b")] == 0b10 and out[ord("c")] == 0b100 and out.sum() == 0b1111
    long = np.frombuffer(b"x" * 33, np.uint8).copy()
    assert L.gofann_string_peq(A.ptr(long), 33, A.ptr(out)) == A.ERR_UNSUPPORTED
    bad = np.frombuffer(b"ab\xc3", np.uint8).copy()
    assert L.gofann_string_peq(A.ptr(bad), 3, A.ptr(out)) == A.ERR_UNSUPPORTED


def test_oracle_hybrid_atoms():
    """The oracle's string and int64 atoms against a direct Python reading of
    the same clauses."""
    w, idx, plan = cfg2_small()
    attrs, routes = with_hybrid_predicates(w, idx, plan.graph_routes, seed=3)
    off, data = attrs["string_offsets"], attrs["string_bytes"]
    iv = attrs["int_values"]
    ip, ind = attrs["label_indptr"], attrs["label_indices"]
    rng = np.random.default_rng(1)
    n_routes = routes["query_row"].shape[0]
    pr = rng.integers(0, n_routes, size=1500)
    ps = rng.integers(0, w.n, size=1500)
    got = O.pred_matches(routes, attrs, pr, ps)

    def clause_ok(ci, s):
        c, x = routes["clauses"][ci], routes["pred_ext"][ci]
        row = set(ind[ip[s]:ip[s + 1]].tolist())
        if any(int(h) not in row for h in routes["pred_handles"][c["label_begin"]:c["label_end"]]):
            return False
        for a in routes["pred_ints"][x["int_begin"]:x["int_end"]]:
            v = int(iv[s, a["dimension"]])
            mode, lo, hi = int(a["mode"]), int(a["lower"]), int(a["upper"])
            if mode == 1 and not v > lo or mode == 2 and not v < hi or mode == 3 and not (lo <= v < hi):
                return False
        text = bytes(data[off[s]:off[s + 1]])
        for a in routes["pred_strings"][x["string_begin"]:x["string_end"]]:
            q = bytes(routes["pred_string_bytes"][a["offset"]:a["offset"] + a["length"]])
            if a["kind"] == A.STRING_EXACT and text != q:
                return False
            if a["kind"] == A.STRING_FUZZY and myers(q, text) > a["max_edits"]:
                return False
        return True

    want = [any(clause_ok(ci, int(s)) for ci in range(routes["pred_offsets"][r], routes["pred_offsets"][r + 1]))
            for r, s in zip(pr, ps)]
    assert np.array_equal(got.astype(bool), np.array(want))
    assert 0 < got.sum() < len(got)
