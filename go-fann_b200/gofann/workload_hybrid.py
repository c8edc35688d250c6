"""BASELINE configuration 4 built on the GPU: the large hybrid-predicate case.

Stand-in for the reference's LAION100M workloads (512-d FP16 embeddings,
1-bit RaBitQ, categorical / range / exact-string / fuzzy-string / hybrid
predicates; the dataset is not available offline).  One GPU holds one shard
of the 100M-vector case -- 100M / 8 = 12.5M vectors by default, the per-GPU
share when the base set is split by contiguous id range over 8 B200s:

  * base: n x 512 from a 16,384-centre Gaussian mixture (centres N(0,1);
    each component spread on a rank-32 subspace, as in configuration 3),
    stored as FP16 -- the exact rerank store (12.8 GB at n = 12.5M);
  * attributes per vector: 1-10 tags from a 50k vocabulary with Zipf(1.1)
    frequencies (the label CSR); one int64 value, uniform; one ASCII string
    of 8-32 bytes built from Zipf-distributed 3-gram tokens, drawn from a
    dictionary of `n_strings` distinct strings whose use is Zipf(1.1) over
    rows (captions repeat);
  * index: the configuration-3 builder at padded dim 512 (64-byte 1-bit
    RaBitQ codes, anchors = the mixture centres, a global graph of degree
    32); postings per tag, the rows ordered by the int64 value, and the rows
    grouped by string;
  * queries: mixture samples, 25 % categorical (one tag), 20 % int64 range
    (selectivity 1e-5 ... 0.5), 15 % exact string, 15 % fuzzy string (a
    dictionary string with 1-2 random edits, matched at edit distance <= 2),
    25 % hybrid AND (a tag and an int64 range);
  * planning (the reference's categorical / range access split,
    dataloader.cpp:11862, and its fuzzy rewrite into an OR of exact terms,
    dataloader.cpp:2973-3010): a term whose rows number at most `scan_rows`
    is scanned, a more frequent one runs the global graph with the term as
    a DNF atom.  A tag scans its posting, a range its slice of the int64
    order.  A string term is first resolved to dictionary strings -- the
    exact string, or for a fuzzy term the strings within the edit distance,
    found on the device (gofann_predicate_pass_masks runs the bit-parallel
    check over the dictionary) -- whose row groups are scanned, one posting
    route each, merged per query (the rows match, so no residual), or, when
    they hold more than `scan_rows` rows, the graph runs with the exact or
    fuzzy atom.  A hybrid query scans the smaller of its tag posting and
    range slice (the other atom as the residual) when that side is short,
    or when the conjunction is expected to match fewer than `selective_rows`
    rows and the side has at most `max_scan_rows`; otherwise the graph runs
    with both atoms;
  * several GPUs: rank r holds shard r (its own rows, index and plan; the
    shared centres, dictionary and queries come from the common seed), and
    the per-shard top-10 are exchanged and merged (gofann_shard_merge), so
    8 ranks hold the 100M-vector case;
  * ground truth: exact filtered top-10 of FP32 distances over the FP16 base.
"""
from __future__ import annotations

import ctypes as C
import time
from dataclasses import dataclass

import numpy as np
import torch

from . import _abi as A
from . import workload_rabitq as WR

SELECTIVITIES = (1e-5, 1e-4, 1e-3, 1e-2, 0.1, 0.5)
KIND_NAMES = ("categorical", "range", "exact_string", "fuzzy_string", "hybrid")
INT_SPAN = 1 << 40


def _log(msg: str, t0: float) -> None:
    print(f"[config4 {time.time() - t0:7.1f}s] {msg}", flush=True)


@dataclass
class HyQueries:
    vectors: torch.Tensor      # [q, dim] f32
    kind: np.ndarray           # index into KIND_NAMES
    tag: np.ndarray            # categorical / hybrid
    lower: np.ndarray          # int64 range lower <= v < upper
    upper: np.ndarray
    string: list               # bytes per query (exact / fuzzy), b"" otherwise


def _zipf_probs(k: int, s: float, device) -> torch.Tensor:
    p = 1.0 / torch.arange(1, k + 1, dtype=torch.float64, device=device) ** s
    return (p / p.sum()).to(torch.float32)


def _dictionary(g, n_strings: int, device, n_tokens=4096):
    """n_strings distinct ASCII strings of 8-32 bytes from Zipf(1.1) 3-gram
    tokens: (bytes u8 [n_strings][32], lengths)."""
    letters = torch.tensor(list(b"abcdefghijklmnopqrstuvwxyz"), dtype=torch.uint8, device=device)
    tokens = letters[torch.randint(0, 26, (n_tokens, 3), generator=g, device=device)]
    pz = _zipf_probs(n_tokens, 1.1, device)
    out_b, out_l, seen, have = [], [], set(), 0
    while have < n_strings:
        m = 2 * (n_strings - have) + 1024
        t = torch.multinomial(pz, m * 11, replacement=True, generator=g).view(m, 11)
        raw = tokens[t].view(m, 33)[:, :32]
        ln = torch.randint(8, 33, (m,), generator=g, device=device)
        raw = torch.where(torch.arange(32, device=device)[None, :] < ln[:, None], raw, torch.zeros_like(raw))
        rb, rl = raw.cpu().numpy(), ln.cpu().numpy()
        for i in range(m):
            key = rb[i, :rl[i]].tobytes()
            if key in seen:
                continue
            seen.add(key)
            out_b.append(rb[i])
            out_l.append(rl[i])
            have += 1
            if have == n_strings:
                break
    return np.stack(out_b), np.asarray(out_l, np.int64)


def _mutate(s: bytes, edits: int, rng) -> bytes:
    b = bytearray(s)
    for _ in range(edits):
        op = int(rng.integers(0, 3))
        i = int(rng.integers(0, max(1, len(b))))
        c = int(rng.integers(97, 123))
        if op == 0 and len(b) < 32:
            b.insert(i, c)
        elif op == 1 and len(b) > 1:
            del b[i]
        elif b:
            b[i] = c
    return bytes(b)


def generate(device="cuda", seed=0, n=12_500_000, dim=512, n_centres=16_384, rank=32, spread=4.0, noise=0.1,
             vocab=50_000, max_tags=10, n_strings=200_000, n_queries=100_000, t0=None, shard=0):
    """Shard `shard` (n rows) of the workload.  Everything shared by the
    shards -- mixture centres, the string dictionary and its popularity,
    the queries -- comes from a generator seeded with `seed` alone, so every
    rank builds the same queries; the shard's rows come from a generator
    seeded with (seed, shard)."""
    t0 = t0 or time.time()
    g = torch.Generator(device=device).manual_seed(seed)
    gs = torch.Generator(device=device).manual_seed(seed * 1_000_003 + 7919 * (shard + 1))
    centres = torch.randn((n_centres, dim), generator=g, device=device)
    bases = torch.linalg.qr(torch.randn((64, dim, rank), generator=g, device=device))[0].contiguous()
    base = torch.empty((n, dim), dtype=torch.float16, device=device)
    chunk = 1 << 18
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        comp = torch.randint(0, n_centres, (e - s,), generator=gs, device=device)
        base[s:e] = WR._mixture(gs, centres, bases, comp, spread, noise).to(torch.float16)
    _log(f"base {n} x {dim} f16 ({base.numel() * 2 / 1e9:.1f} GB), shard {shard}", t0)
    # tags: 1..max_tags per row, Zipf(1.1) over the vocabulary
    pz = _zipf_probs(vocab, 1.1, device)
    per = torch.randint(1, max_tags + 1, (n,), generator=gs, device=device)
    rows = torch.repeat_interleave(torch.arange(n, device=device, dtype=torch.int64), per)
    vals = torch.cat([torch.multinomial(pz, int(min(1 << 24, rows.numel() - s)), replacement=True, generator=gs)
                      for s in range(0, rows.numel(), 1 << 24)])
    key = torch.unique((rows << 16) | vals)
    rows_u, vals_u = key >> 16, (key & 0xFFFF).to(torch.int32)
    del rows, vals, key
    indptr = torch.zeros(n + 1, dtype=torch.int64, device=device)
    indptr[1:] = torch.cumsum(torch.bincount(rows_u, minlength=n), 0)
    key2 = torch.sort((vals_u.to(torch.int64) << 32) | rows_u).values
    postings = (key2 & 0xFFFFFFFF).to(torch.int32)
    del key2, rows_u
    card = torch.bincount(vals_u, minlength=vocab).cpu().numpy().astype(np.int64)
    begin = np.zeros(vocab, np.int64)
    begin[1:] = np.cumsum(card)[:-1]
    _log(f"{int(vals_u.numel())} tags over {vocab} values", t0)
    # int64 attribute
    ival = torch.randint(0, INT_SPAN, (n, 1), generator=gs, device=device, dtype=torch.int64)
    # strings: a dictionary, each row one of its strings (Zipf over rows)
    dict_b, dict_l = _dictionary(g, n_strings, device)
    pstr = _zipf_probs(n_strings, 1.1, device)
    perm = torch.randperm(n_strings, generator=g, device=device)  # popularity independent of dictionary order
    sid = perm[torch.multinomial(pstr, n, replacement=True, generator=gs)]
    lens = torch.from_numpy(dict_l).to(device)[sid]
    soff = torch.zeros(n + 1, dtype=torch.int64, device=device)
    soff[1:] = torch.cumsum(lens, 0)
    db = torch.from_numpy(dict_b).to(device)
    sbytes = db[sid][torch.arange(32, device=device)[None, :] < lens[:, None]]
    _log(f"strings: {n_strings} distinct, {int(soff[-1]) / 1e9:.2f} GB of bytes", t0)
    # queries (shared by every shard): tags and strings drawn by the rows'
    # own popularity distributions
    rng = np.random.default_rng(seed + 29)
    qc = torch.randint(0, n_centres, (n_queries,), generator=g, device=device)
    qv = WR._mixture(g, centres, bases, qc, spread, noise)
    kind = rng.choice(5, size=n_queries, p=[0.25, 0.20, 0.15, 0.15, 0.25])
    # a row carries a tag about once per draw: its frequency follows pz
    tag = torch.multinomial(pz, n_queries, replacement=True, generator=g).cpu().numpy().astype(np.int64)
    sel = np.asarray(SELECTIVITIES)[rng.integers(0, len(SELECTIVITIES), n_queries)]
    lower = (rng.random(n_queries) * (1.0 - sel) * INT_SPAN).astype(np.int64)
    upper = lower + np.maximum(1, (sel * INT_SPAN).astype(np.int64))
    sid_h = perm[torch.multinomial(pstr, n_queries, replacement=True, generator=g)].cpu().numpy()
    strings = []
    for i in range(n_queries):
        if kind[i] in (2, 3):
            s = dict_b[sid_h[i], :dict_l[sid_h[i]]].tobytes()
            strings.append(_mutate(s, int(rng.integers(1, 3)), rng) if kind[i] == 3 else s)
        else:
            strings.append(b"")
    q = HyQueries(qv, kind, tag, lower, upper, strings)
    _log(f"{n_queries} queries: " + ", ".join(f"{int((kind == k).sum())} {nm}" for k, nm in enumerate(KIND_NAMES)),
         t0)
    return dict(base=base, centres=centres, set_indptr=indptr, set_indices=vals_u, postings=postings, card=card,
                begin=begin, ival=ival, sid=sid, soff=soff, sbytes=sbytes, dict_bytes=dict_b, dict_len=dict_l,
                queries=q, vocab=vocab, n=n, dim=dim)


def build_index(data: dict, seed=0, t0=None) -> WR.RqIndex:
    """The RaBitQ index at padded dim 512 with a degree-32 global graph, plus
    the int64 order and the string groups appended to the postings array."""
    t0 = t0 or time.time()
    idx = WR.build_index(data, degree=32, seed=seed, t0=t0, chunk=1 << 16, normalize_anchors=False,
                         range_postings=False)
    dev = data["base"].device
    n = data["n"]
    iorder = torch.argsort(data["ival"][:, 0], stable=True)
    sorder = torch.argsort(data["sid"], stable=True)
    base_ids = idx.posting_ids.numel()
    idx.posting_ids = torch.cat([idx.posting_ids, iorder.to(torch.int32), sorder.to(torch.int32)])
    scount = torch.bincount(data["sid"], minlength=len(data["dict_len"])).cpu().numpy().astype(np.int64)
    sbegin = np.zeros_like(scount)
    sbegin[1:] = np.cumsum(scount)[:-1]
    idx.stats.update(int_order_base=base_ids, string_order_base=base_ids + n, string_begin=sbegin,
                     string_count=scount, int_sorted=data["ival"][iorder, 0].cpu().numpy())
    idx.extra_attrs = {"string_offsets": data["soff"], "string_bytes": data["sbytes"], "int_values": data["ival"]}
    idx.attr = None
    _log(f"postings: tags, int64 order, {len(scount)} string groups", t0)
    return idx


def _string_peq(b: bytes) -> np.ndarray:
    peq = np.zeros(128, np.uint32)
    for i, ch in enumerate(b):
        peq[ch] |= np.uint32(1 << i)
    return peq


def fuzzy_rewrite(data: dict, strings: list, max_edits: int = 2, device="cuda") -> list:
    """Dictionary string ids within max_edits of each query string: the
    fuzzy atom evaluated on the device (gofann_predicate_pass_masks) for
    every (query, dictionary string) pair whose lengths differ by at most
    max_edits -- the planner's rewrite of a fuzzy term into exact terms."""
    L = A.lib()
    dl = data["dict_len"]
    nd = dl.shape[0]
    db = data["dict_bytes"]
    by_len = {ln: np.nonzero(dl == ln)[0] for ln in range(8, 33)}
    # the dictionary as samples: string attributes, no labels
    off = np.zeros(nd + 1, np.uint64)
    off[1:] = np.cumsum(dl)
    sb = db[np.arange(32)[None, :] < dl[:, None]]
    attrs = {"label_indptr": torch.zeros(nd + 1, dtype=torch.int64, device=device),
             "label_indices": torch.zeros(1, dtype=torch.int32, device=device),
             "string_offsets": torch.from_numpy(off.view(np.int64)).to(device),
             "string_bytes": torch.from_numpy(sb).to(device)}
    graph = {"adjacency": torch.zeros((nd, 1), dtype=torch.int32, device=device),
             "row_to_sample": torch.arange(nd, dtype=torch.int32, device=device),
             "label_offset": torch.zeros(1, dtype=torch.int32, device=device)}
    nq = len(strings)
    out = [[] for _ in range(nq)]
    qs = [i for i in range(nq) if strings[i]]
    step = 256
    for c0 in range(0, len(qs), step):
        cq = qs[c0:c0 + step]
        n = len(cq)
        clauses = np.zeros(n, A.CLAUSE_DTYPE)
        ext = np.zeros(n, A.CLAUSE_EXT_DTYPE)
        ext["string_begin"], ext["string_end"] = np.arange(n), np.arange(1, n + 1)
        sa = np.zeros(n, A.STRING_ATOM_DTYPE)
        qb = b"".join(strings[i] for i in cq)
        lens = np.array([len(strings[i]) for i in cq], np.uint32)
        sa["kind"], sa["max_edits"], sa["length"] = A.STRING_FUZZY, max_edits, lens
        sa["offset"] = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.uint32)
        peq = np.stack([_string_peq(strings[i]) for i in cq])
        routes = {"query_row": np.arange(n, dtype=np.uint32), "group_id": np.zeros(n, np.uint32),
                  "start_local": np.zeros(n, np.uint32), "pred_offsets": np.arange(n + 1, dtype=np.uint32),
                  "clauses": clauses, "pred_handles": np.zeros(1, np.uint32), "pred_ext": ext, "pred_strings": sa,
                  "pred_string_bytes": np.frombuffer(qb, np.uint8).copy(), "pred_string_peq": peq}
        cr, cand = [], []
        for j, i in enumerate(cq):
            ln = len(strings[i])
            ids = np.concatenate([by_len.get(x, np.zeros(0, np.int64)) for x in range(ln - max_edits,
                                                                                      ln + max_edits + 1)])
            cr.append(np.full(ids.shape[0], j, np.uint32))
            cand.append(ids.astype(np.uint32))
        cr, cand = np.concatenate(cr), np.concatenate(cand)
        from .engine import _t
        dr = {k: _t(v, device) for k, v in routes.items()}
        gs, at, rs = A.fill_graph(graph), A.fill_attrs(attrs), A.fill_routes(dr)
        m = cr.shape[0]
        masks = torch.zeros((m + 31) // 32, dtype=torch.int32, device=device)
        d_cr, d_cand = _t(cr, device), _t(cand, device)
        A.check(L.gofann_predicate_pass_masks(C.byref(gs), C.byref(at), C.byref(rs), A.ptr(d_cr), A.ptr(d_cand), m,
                                              A.ptr(masks), None, torch.cuda.current_stream().cuda_stream),
                "gofann_predicate_pass_masks(fuzzy rewrite)")
        hit = np.nonzero(np.unpackbits(masks.cpu().numpy().view(np.uint8), bitorder="little")[:m])[0]
        cuts = np.searchsorted(cr[hit], np.arange(n + 1))  # cr is grouped by query
        for j, i in enumerate(cq):
            out[i] = cand[hit[cuts[j]:cuts[j + 1]]].astype(np.int64)
    return out


@dataclass
class HyPlan:
    graph_routes: dict
    graph_query: np.ndarray
    posting_routes: dict
    posting_query: np.ndarray
    posting_begin: np.ndarray
    posting_count: np.ndarray
    n_queries: int
    matches: list                  # per query: dictionary ids of its string term(s)
    rewrite_ms: float = 0.0
    graph_rows: list = None        # route descriptions (query, start, labels, int atoms, string atoms)
    posting_rows: list = None

    def subset(self, sel: np.ndarray):
        """Route tables of the queries `sel`, re-based onto rows 0..len(sel)-1
        of the sample: (graph routes, graph route positions, posting routes,
        posting route positions)."""
        pos = np.full(self.n_queries, -1, np.int64)
        pos[sel] = np.arange(len(sel))
        gsel = np.nonzero(pos[self.graph_query] >= 0)[0]
        psel = np.nonzero(pos[self.posting_query] >= 0)[0]
        g = _tables([(int(pos[r[0]]),) + tuple(r[1:]) for r in (self.graph_rows[i] for i in gsel)])
        p = _tables([(int(pos[r[0]]),) + tuple(r[1:]) for r in (self.posting_rows[i] for i in psel)])
        return g, gsel, p, psel


def _tables(rows: list, n_str_bytes=None):
    """gofann_routes arrays for route descriptions (query, start, labels,
    ints, strings): one DNF clause per route."""
    n = len(rows)
    clauses = np.zeros(max(n, 1), A.CLAUSE_DTYPE)
    ext = np.zeros(max(n, 1), A.CLAUSE_EXT_DTYPE)
    handles, ints, strs, sbytes, peqs = [], [], [], bytearray(), []
    for r, (_, _, labels, iatoms, satoms) in enumerate(rows):
        clauses[r]["label_begin"] = len(handles)
        handles += labels
        clauses[r]["label_end"] = len(handles)
        ext[r]["int_begin"] = len(ints)
        ints += iatoms
        ext[r]["int_end"] = len(ints)
        ext[r]["string_begin"] = len(strs)
        for kind, b in satoms:
            strs.append((kind, 2 if kind == A.STRING_FUZZY else 0, len(sbytes), len(b)))
            sbytes += b
            peqs.append(_string_peq(b) if kind == A.STRING_FUZZY else np.zeros(128, np.uint32))
        ext[r]["string_end"] = len(strs)
    ia = np.zeros(max(1, len(ints)), A.INT_ATOM_DTYPE)
    for i, x in enumerate(ints):
        ia[i] = x
    sa = np.zeros(max(1, len(strs)), A.STRING_ATOM_DTYPE)
    for i, x in enumerate(strs):
        sa[i] = x
    return {"query_row": np.asarray([x[0] for x in rows], np.uint32),
            "group_id": np.zeros(n, np.uint32), "start_local": np.asarray([x[1] for x in rows], np.uint32),
            "pred_offsets": np.arange(n + 1, dtype=np.uint32), "clauses": clauses[:max(n, 1)],
            "pred_handles": np.asarray(handles if handles else [0], np.uint32),
            "pred_enabled": np.ones(max(n, 1), np.uint8)[:n] if n else np.zeros(0, np.uint8),
            "pred_ext": ext, "pred_ints": ia, "pred_strings": sa,
            "pred_string_bytes": np.frombuffer(bytes(sbytes) if sbytes else b"\0", np.uint8).copy(),
            "pred_string_peq": np.stack(peqs) if peqs else np.zeros((1, 128), np.uint32)}


def plan_queries(idx: WR.RqIndex, data: dict, q: HyQueries, scan_rows=150_000, selective_rows=5_000,
                 max_scan_rows=1_000_000) -> HyPlan:
    t0 = time.perf_counter()
    fuzzy = [b if k == 3 else b"" for b, k in zip(q.string, q.kind)]
    matches = fuzzy_rewrite(data, fuzzy)
    rewrite_ms = (time.perf_counter() - t0) * 1e3
    dl, db = data["dict_len"], data["dict_bytes"]
    lookup = {db[j, :dl[j]].tobytes(): j for j in range(dl.shape[0])}
    for i in range(q.kind.shape[0]):
        if q.kind[i] == 2:
            j = lookup.get(q.string[i])
            matches[i] = np.asarray([] if j is None else [j], np.int64)
    st = idx.stats
    isorted = st["int_sorted"]
    card, tbeg = idx.posting_count.astype(np.int64), idx.posting_begin.astype(np.int64)
    g_rows, g_q, p_rows, p_q, p_b, p_c = [], [], [], [], [], []
    for i in range(q.kind.shape[0]):
        k = int(q.kind[i])
        tag_atom = [int(q.tag[i])]
        int_atom = [(0, 3, int(q.lower[i]), int(q.upper[i]))]
        lo = int(np.searchsorted(isorted, q.lower[i], "left"))
        hi = int(np.searchsorted(isorted, q.upper[i], "left"))
        if k == 0:
            if card[q.tag[i]] <= scan_rows:
                p_rows.append((i, 0, [], [], [])); p_q.append(i); p_b.append(tbeg[q.tag[i]]); p_c.append(card[q.tag[i]])
            else:
                g_rows.append((i, idx.seed, tag_atom, [], [])); g_q.append(i)
        elif k == 1:
            if hi - lo <= scan_rows:
                p_rows.append((i, 0, [], [], [])); p_q.append(i); p_b.append(st["int_order_base"] + lo); p_c.append(hi - lo)
            else:
                g_rows.append((i, idx.seed, [], int_atom, [])); g_q.append(i)
        elif k == 4:
            tc, rc = card[q.tag[i]], hi - lo
            # a conjunction expected to match few rows is scanned from its
            # smaller side even when that side is long (graph traversals
            # under very selective predicates wander)
            est = tc * rc / max(1, idx.n)
            if min(tc, rc) <= scan_rows or (est < selective_rows and min(tc, rc) <= max_scan_rows):
                if tc <= rc:
                    p_rows.append((i, 0, [], int_atom, [])); p_b.append(tbeg[q.tag[i]]); p_c.append(tc)
                else:
                    p_rows.append((i, 0, tag_atom, [], [])); p_b.append(st["int_order_base"] + lo); p_c.append(rc)
                p_q.append(i)
            else:
                g_rows.append((i, idx.seed, tag_atom, int_atom, [])); g_q.append(i)
        else:  # exact or fuzzy string: the rows of each matching dictionary string
            counts = st["string_count"][matches[i]] if len(matches[i]) else np.zeros(0, np.int64)
            if counts.sum() <= scan_rows:
                for sid, c in zip(matches[i], counts):  # the rows match: no residual
                    if c == 0:
                        continue
                    p_rows.append((i, 0, [], [], [])); p_q.append(i)
                    p_b.append(st["string_order_base"] + int(st["string_begin"][sid])); p_c.append(int(c))
            else:  # a popular string: the graph with the string atom
                atom = [(A.STRING_EXACT if k == 2 else A.STRING_FUZZY, q.string[i])]
                g_rows.append((i, idx.seed, [], [], atom)); g_q.append(i)
    graph = _tables(g_rows)
    post = _tables(p_rows)
    return HyPlan(graph, np.asarray(g_q, np.uint32), post, np.asarray(p_q, np.uint32),
                  np.asarray(p_b, np.uint64), np.asarray(p_c, np.uint32), int(q.kind.shape[0]), matches, rewrite_ms,
                  g_rows, p_rows)


def ground_truth(idx: WR.RqIndex, data: dict, q: HyQueries, plan: HyPlan, sample: np.ndarray, k=10,
                 chunk=1 << 20, with_dists=False):
    """Exact filtered top-k (FP32 distances of the FP16 rows, ties by id):
    the rows passing each query's predicate, found from the attribute
    arrays (tags from the CSR, int64 values, string ids; a fuzzy term's
    strings are those within edit distance 2, plan.matches), then a full
    distance computation over them."""
    dev = idx.base.device
    base = idx.base
    n = base.shape[0]
    sid = data["sid"]
    ival = data["ival"][:, 0]
    tag_post = idx.posting_ids
    out = np.full((len(sample), k), A.U32MAX, np.uint32)
    out_d = np.full((len(sample), k), np.inf, np.float32)
    for r, i in enumerate(sample):
        kd = int(q.kind[i])
        if kd in (0, 4):
            b0, c0 = int(idx.posting_begin[q.tag[i]]), int(idx.posting_count[q.tag[i]])
            cand = tag_post[b0:b0 + c0].to(torch.int64)
            if kd == 4:
                v = ival[cand]
                cand = cand[(v >= int(q.lower[i])) & (v < int(q.upper[i]))]
        elif kd == 1:
            cand = torch.nonzero((ival >= int(q.lower[i])) & (ival < int(q.upper[i]))).squeeze(1)
        else:  # the query's dictionary strings: the exact one, or those within the edit distance
            ids = torch.from_numpy(np.asarray(plan.matches[i], np.int64)).to(dev)
            cand = torch.nonzero(torch.isin(sid, ids)).squeeze(1)
        if cand.numel() == 0:
            continue
        x = q.vectors[i]
        best_d, best_i = None, None
        for s in range(0, cand.numel(), chunk):
            c = cand[s:s + chunk]
            d = (base[c].float() - x).square().sum(1)
            kk = min(k, c.numel())
            tk = d.topk(kk, largest=False)
            cd, ci = tk.values, c[tk.indices]
            if best_d is not None:
                cd, ci = torch.cat([best_d, cd]), torch.cat([best_i, ci])
            o = cd.topk(min(k, cd.numel()), largest=False)
            best_d, best_i = o.values, ci[o.indices]
        ids_h, dd = best_i.cpu().numpy(), best_d.cpu().numpy()
        o = np.lexsort((ids_h, dd))
        out[r, :len(o)] = ids_h[o]
        out_d[r, :len(o)] = dd[o]
    return (out, out_d) if with_dists else out
