"""Shared seeded test workloads (small enough for the CPU oracle)."""
from __future__ import annotations

import copy
import functools

import numpy as np
import torch

from gofann import _abi as A, index_build, planner, synth


@functools.lru_cache(maxsize=None)
def cfg1_small(n=6000, n_labels=16, n_queries=160, threshold=400, degree=32, pq_dim=32, seed=0, dim=128):
    w = synth.config1(seed=seed, n=n, n_labels=n_labels, n_queries=n_queries, dim=dim)
    idx = index_build.build_index(w, threshold=threshold, degree=degree, pq_dim=pq_dim, seed=seed)
    plan = planner.plan_queries(idx, w.query_labels)
    return w, idx, plan


@functools.lru_cache(maxsize=None)
def cfg2_small(n=5000, vocab=120, n_queries=160, threshold=300, degree=64, pq_dim=48, seed=1):
    w = synth.config2_small(seed=seed, n=n, vocab=vocab, n_queries=n_queries)
    idx = index_build.build_index(w, threshold=threshold, degree=degree, pq_dim=pq_dim, seed=seed)
    plan = planner.plan_queries(idx, w.query_labels)
    return w, idx, plan


@functools.lru_cache(maxsize=None)
def cfg2_small_u8cb(pq_dim=48):
    """cfg2_small with its codebook rounded to integers in 0..255 and the
    codes re-encoded against it: the preconditions of GOFANN_PQ_U8."""
    from oracle import oracle as O
    w, idx, plan = cfg2_small(pq_dim=pq_dim)
    cent = np.clip(np.rint(idx.pq_centroids), 0, 255).astype(np.float32)
    idx2 = copy.copy(idx)
    idx2.pq_centroids = cent
    idx2.pq_codes = O.pq_encode(w.base.astype(np.float32), cent, idx.pq_codes.shape[1])
    return w, idx2, plan


def random_orthogonal(p: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    q, r = np.linalg.qr(rng.standard_normal((p, p)))
    q *= np.sign(np.diag(r))
    return q.astype(np.float32)


@functools.lru_cache(maxsize=None)
def rabitq_artifacts(n=6000, n_labels=16, n_queries=160, n_anchors=16, seed=3, dim=128):
    """RaBitQ codes for a config-1 style workload of `dim` dimensions:
    rotation, anchors, 1-bit codes and factors from the oracle's encoder;
    rotated queries."""
    from oracle import oracle as O
    w, idx, plan = cfg1_small(n=n, n_labels=n_labels, n_queries=n_queries, dim=dim)
    rng = np.random.default_rng(seed)
    p = ((w.dim + 63) // 64) * 64
    rot = random_orthogonal(p, seed)
    pad = lambda x: np.pad(x.astype(np.float32), ((0, 0), (0, p - x.shape[1])))
    xr = pad(w.base) @ rot
    anchors = xr[rng.choice(w.n, n_anchors, replace=False)]
    anchor_ids = np.argmin(((xr[:, None, :] - anchors[None]) ** 2).sum(-1), axis=1).astype(np.uint32)
    codes, factors = O.rabitq_encode(xr - anchors[anchor_ids], anchors, anchor_ids)
    qr = (pad(w.queries) @ rot).astype(np.float32)
    return w, idx, plan, {"rq_codes": codes, "rq_factors": factors, "rq_anchor_ids": anchor_ids,
                          "num_anchors": n_anchors}, anchors.astype(np.float32), qr


def dev(a, device="cuda"):
    """numpy -> torch device tensor (unsigned views as signed of equal width)."""
    if a is None:
        return None
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint64:
        a = a.view(np.int64)
    elif a.dtype == np.uint32:
        a = a.view(np.int32)
    elif a.dtype == np.uint16:
        a = a.view(np.int16)
    elif a.dtype.fields is not None:
        a = a.view(np.uint8).reshape(-1)
    return torch.from_numpy(a).to(device)


def dev_dict(d: dict, device="cuda") -> dict:
    return {k: (dev(v, device) if isinstance(v, np.ndarray) else v) for k, v in d.items()}


def host(t: torch.Tensor, dtype) -> np.ndarray:
    return t.cpu().numpy().view(dtype)


def fbits(x) -> np.ndarray:
    return np.ascontiguousarray(x, np.float32).view(np.uint32)


def with_predicates(w, idx, routes: dict, seed=0, range_count=2):
    """Range attributes, row filter masks and two predicate forms for the
    routes of a small workload:
      * dnf: 1-3 OR-ed clauses per route -- the route's residual labels, a
        label of a random sample, float range atoms in modes 1-3 over two
        dimensions (gpu_predicate_index.cuh:100-136, range_filter.cuh:28-77)
        -- and a few routes with the predicate disabled;
      * legacy: no DNF; per-route filter bits against per-row masks
        (backend_pq.cu:4394-4397), per-route range modes 0-3 with bounds
        (range_filter.cuh:47-98), a quarter of the routes marked compiled.
    Returns (attrs, graph, dnf_routes, legacy_routes)."""
    from gofann import _abi as A
    rng = np.random.default_rng(seed)
    attrs = dict(idx.attrs())
    vals = rng.uniform(0.0, 1000.0, size=(w.n, range_count)).astype(np.float32)
    vals[::97, 0] = 500.0  # exact bound hits
    attrs["range_values"] = vals
    graph = dict(idx.graph())
    rows = graph["adjacency"].shape[0]
    mask = np.zeros(rows, np.uint64)
    for _ in range(8):
        mask |= np.uint64(1) << rng.integers(0, 64, size=rows).astype(np.uint64)
    graph["row_filter_mask"] = mask
    n = routes["query_row"].shape[0]
    ip, ind = attrs["label_indptr"], attrs["label_indices"]

    def atom(dim):
        mode = int(rng.integers(1, 4))
        lo, hi = np.sort(rng.uniform(0, 1000, size=2)).astype(np.float32)
        if rng.random() < 0.2:
            lo = np.float32(500.0)
        return (dim, mode, lo, hi)

    offs, clauses, handles, ranges = [0], [], [], []
    rip, rind = routes["qlabel_indptr"], routes["qlabel_indices"]
    for r in range(n):
        prim = routes["primary_label"][r]
        for c in range(int(rng.integers(1, 4))):
            lb, rb = len(handles), len(ranges)
            if c == 0:
                handles += [int(x) for x in rind[rip[r]:rip[r + 1]] if x != prim]
            else:
                s = int(rng.integers(0, w.n))
                row = ind[ip[s]:ip[s + 1]]
                if row.size and rng.random() < 0.7:
                    handles.append(int(row[rng.integers(0, row.size)]))
            for _ in range(int(rng.integers(0 if c == 0 else 1, 3))):
                ranges.append(atom(int(rng.integers(0, range_count))))
            clauses.append((lb, len(handles), rb, len(ranges)))
        offs.append(len(clauses))
    cl = np.zeros(len(clauses), A.CLAUSE_DTYPE)
    for i, (a, b, c, d) in enumerate(clauses):
        cl[i] = (a, b, c, d)
    ra = np.zeros(max(1, len(ranges)), A.RANGE_ATOM_DTYPE)
    for i, x in enumerate(ranges):
        ra[i] = x
    dnf = dict(routes)
    dnf.update(pred_offsets=np.asarray(offs, np.uint32), clauses=cl,
               pred_handles=np.asarray(handles if handles else [0], np.uint32), pred_ranges=ra,
               pred_enabled=(rng.random(n) < 0.9).astype(np.uint8))
    legacy = {k: v for k, v in routes.items()
              if k not in ("pred_offsets", "clauses", "pred_handles", "pred_ranges", "pred_enabled")}
    fb = np.zeros(n, np.uint64)
    for _ in range(4):
        fb |= np.uint64(1) << rng.integers(0, 64, size=n).astype(np.uint64)
    fb[::11] = 0
    fb[1::13] = np.uint64(0xFFFFFFFFFFFFFFFF)
    legacy["filter_bits"] = fb
    legacy["range_modes"] = rng.integers(0, 4, size=(n, range_count)).astype(np.uint8)
    lo = rng.uniform(0, 400, size=(n, range_count)).astype(np.float32)
    legacy["range_lower"] = lo
    legacy["range_upper"] = (lo + rng.uniform(300, 900, size=(n, range_count))).astype(np.float32)
    legacy["route_compiled"] = (rng.random(n) < 0.25).astype(np.uint8)
    return attrs, graph, dnf, legacy


def string_table(strings):
    """Per-sample strings as (offsets u64 [n+1], bytes u8)."""
    enc = [s.encode() for s in strings]
    off = np.zeros(len(enc) + 1, np.uint64)
    off[1:] = np.cumsum([len(e) for e in enc])
    data = np.frombuffer(b"".join(enc), np.uint8).copy() if off[-1] else np.zeros(1, np.uint8)
    return off, data


def synth_strings(n, rng, vocab_size=300):
    """ASCII strings of 8-32 bytes built from Zipf-distributed 3-gram tokens
    (the config-4 string attribute); some strings repeat exactly."""
    letters = np.frombuffer(b"abcdefghijklmnopqrstuvwxyz", np.uint8)
    vocab = [bytes(rng.choice(letters, size=3)).decode() for _ in range(vocab_size)]
    p = 1.0 / np.arange(1, vocab_size + 1) ** 1.1
    p /= p.sum()
    out = []
    for _ in range(n):
        target = int(rng.integers(8, 33))
        s = ""
        while len(s) < target:
            s += vocab[int(rng.choice(vocab_size, p=p))]
        out.append(s[:target])
    return out


def mutate(s: str, edits: int, rng) -> str:
    """s with `edits` random insertions, deletions or substitutions."""
    letters = "abcdefghijklmnopqrstuvwxyz"
    s = list(s)
    for _ in range(edits):
        op = int(rng.integers(0, 3))
        i = int(rng.integers(0, max(1, len(s))))
        if op == 0 and len(s) < 32:
            s.insert(i, letters[int(rng.integers(0, 26))])
        elif op == 1 and len(s) > 1:
            del s[i]
        elif s:
            s[i] = letters[int(rng.integers(0, 26))]
    return "".join(s)


def with_hybrid_predicates(w, idx, routes: dict, seed=0, int_count=2):
    """The config-4 predicate kinds on a small workload: every sample gets a
    string and int64 attributes; each route gets 1-3 OR-ed clauses mixing its
    residual labels, an exact-string atom (a sample's string), a fuzzy atom
    (a sample's string with 0-3 edits, max_edits 0-2) and int64 range atoms
    in modes 0-3; some routes keep only label clauses.
    Returns (attrs, routes) with the extended DNF."""
    from gofann import _abi as A
    rng = np.random.default_rng(seed)
    attrs = dict(idx.attrs())
    strings = synth_strings(w.n, rng)
    attrs["string_offsets"], attrs["string_bytes"] = string_table(strings)
    iv = rng.integers(-(1 << 40), 1 << 40, size=(w.n, int_count), dtype=np.int64)
    iv[::53, 0] = 1 << 33  # exact bound hits
    attrs["int_values"] = iv
    n = routes["query_row"].shape[0]
    rip, rind = routes["qlabel_indptr"], routes["qlabel_indices"]
    offs, clauses, handles, ext, satoms, sbytes, iatoms = [0], [], [], [], [], bytearray(), []
    peq_rows = []
    for r in range(n):
        prim = routes["primary_label"][r]
        for c in range(int(rng.integers(1, 4))):
            lb = len(handles)
            if c == 0:
                handles += [int(x) for x in rind[rip[r]:rip[r + 1]] if x != prim]
            sb, ib = len(satoms), len(iatoms)
            kind = int(rng.integers(0, 4))
            if kind in (1, 3):  # a string atom
                s = strings[int(rng.integers(0, w.n))]
                fuzzy = rng.random() < 0.6
                if fuzzy:
                    s = mutate(s, int(rng.integers(0, 4)), rng)
                b = s.encode()
                satoms.append((A.STRING_FUZZY if fuzzy else A.STRING_EXACT, int(rng.integers(0, 3)), len(sbytes),
                               len(b)))
                sbytes += b
                peq = np.zeros(128, np.uint32)
                if fuzzy:
                    for i, ch in enumerate(b):
                        peq[ch] |= np.uint32(1 << i)
                peq_rows.append(peq)
            if kind in (2, 3):  # int64 atoms
                for _ in range(int(rng.integers(1, 3))):
                    lo, hi = np.sort(rng.integers(-(1 << 40), 1 << 40, size=2))
                    if rng.random() < 0.2:
                        lo = 1 << 33
                    iatoms.append((int(rng.integers(0, int_count)), int(rng.integers(0, 4)), int(lo), int(hi)))
            clauses.append((lb, len(handles), 0, 0))
            ext.append((sb, len(satoms), ib, len(iatoms)))
        offs.append(len(clauses))
    cl = np.zeros(len(clauses), A.CLAUSE_DTYPE)
    for i, x in enumerate(clauses):
        cl[i] = x
    ex = np.zeros(len(ext), A.CLAUSE_EXT_DTYPE)
    for i, x in enumerate(ext):
        ex[i] = x
    sa = np.zeros(max(1, len(satoms)), A.STRING_ATOM_DTYPE)
    for i, x in enumerate(satoms):
        sa[i] = x
    ia = np.zeros(max(1, len(iatoms)), A.INT_ATOM_DTYPE)
    for i, x in enumerate(iatoms):
        ia[i] = x
    out = dict(routes)
    out.update(pred_offsets=np.asarray(offs, np.uint32), clauses=cl,
               pred_handles=np.asarray(handles if handles else [0], np.uint32),
               pred_enabled=(rng.random(n) < 0.95).astype(np.uint8), pred_ext=ex, pred_strings=sa,
               pred_string_bytes=np.frombuffer(bytes(sbytes) if sbytes else b"\0", np.uint8).copy(),
               pred_string_peq=np.stack(peq_rows) if peq_rows else np.zeros((1, 128), np.uint32),
               pred_ints=ia)
    out.pop("pred_ranges", None)
    return attrs, out
