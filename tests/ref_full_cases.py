"""Seeded cases shaped for the reference's own Full-GPU kernels.

The reference's exact-distance traversal (full_gpu_highfreq_kernel,
src/search/full_gpu/backend_full_gpu.cu:2044-2122) is instantiated for the
queue capacities 16, 32, 48, 64, 96, 128, 192, 256, 384 and 512 and top-k up
to 10, for uint8, float and half vectors (:188-214, 2980-3050).  These cases
stay inside that envelope and are built with numpy alone on the graphs and
labels of tests/ref_kernel_cases.py, so the same seed gives the same inputs
on any machine: the reference kernels' outputs recorded on a B200
(tests/golden/make_ref_full_gpu_golden.py) are replayed against the CPU
oracle here, and the GPU test rebuilds identical inputs on the box.

Per case: the u8 mixture base of ref_kernel_cases (as is, coarsened to a few
levels so that exact distances tie often, or converted to float / half),
one graph per label, queries routed to their rarer label with the other
label as a residual filter; the filtered case adds per-route filter bits
against per-row masks and float range modes.
"""
from __future__ import annotations

import functools
import hashlib

import numpy as np

from ref_kernel_cases import _data

U32MAX = 0xFFFFFFFF
DT_U8, DT_F32, DT_F16 = 0, 1, 2

# (name, dtype, coarse levels (0 = none), queue, early_stop_mode, finish, max_steps, topk, filters)
CASES = [
    ("u8_q64_adaptive", DT_U8, 0, 64, 2, 100, 0, 10, False),
    ("u8_ties_q48_adaptive", DT_U8, 8, 48, 2, 100, 0, 10, False),
    ("u8_q128_fixed_filters", DT_U8, 0, 128, 0, 30, 0, 10, True),
    ("u8_ties_q512_adaptive", DT_U8, 4, 512, 2, 100, 0, 10, False),
    ("f32_q96_off", DT_F32, 0, 96, 1, 100, 150, 7, False),
    ("f32_q16_fixed_top1", DT_F32, 0, 16, 0, 12, 0, 1, False),
    ("f16_q64_adaptive", DT_F16, 0, 64, 2, 100, 0, 10, False),
    ("f16_ties_q256_fixed_filters", DT_F16, 6, 256, 0, 60, 0, 10, True),
]
CASE_NAMES = [c[0] for c in CASES]
LOW_CASES = [("low_u8", DT_U8, 0), ("low_u8_ties", DT_U8, 8), ("low_f32", DT_F32, 0), ("low_f16", DT_F16, 0)]
LOW_NAMES = [c[0] for c in LOW_CASES]


def _vectors(base: np.ndarray, dtype: int, levels: int, rng) -> np.ndarray:
    if levels:
        base = (base.astype(np.int32) * levels // 256).astype(np.uint8)
    if dtype == DT_U8:
        return np.ascontiguousarray(base)
    x = base.astype(np.float32) / 64.0
    if not levels:
        x = x + rng.normal(0, 0.01, size=x.shape).astype(np.float32)
    if dtype == DT_F32:
        return x.astype(np.float32)
    return x.astype(np.float16).view(np.uint16)


def _routes(rng, card, seeds, n_routes, n_labels):
    qlabels = []
    for _ in range(n_routes):
        a = int(rng.integers(0, n_labels))
        if rng.random() < 0.5:
            qlabels.append(np.unique(np.array([a, int(rng.integers(0, n_labels))], np.uint32)))
        else:
            qlabels.append(np.array([a], np.uint32))
    primary = np.array([int(l[np.argmin(card[l])]) for l in qlabels], np.uint32)
    qptr = np.zeros(n_routes + 1, np.uint64)
    qptr[1:] = np.cumsum([len(l) for l in qlabels])
    routes = {
        "query_row": np.arange(n_routes, dtype=np.uint32),
        "group_id": primary.copy(),
        "start_local": seeds[primary].astype(np.uint32),
        "qlabel_indptr": qptr,
        "qlabel_indices": np.concatenate(qlabels).astype(np.uint32),
        "primary_label": primary,
    }
    return routes


@functools.lru_cache(maxsize=None)
def build_case(name: str, seed: int = 11, n: int = 2400, n_labels: int = 5, n_routes: int = 64, degree: int = 32,
               n_random: int = 8):
    """Graph-route case: numpy arrays in the gofann_* descriptor layouts."""
    c = next(x for x in CASES if x[0] == name)
    _, dtype, levels, qs, mode, finish, max_steps, topk, filters = c
    base, centres, graph, attrs, card, seeds = _data(seed, 128, n, n_labels, degree, n_random)
    rng = np.random.default_rng([seed, 100 + CASE_NAMES.index(name)])
    vec = _vectors(base, dtype, levels, rng)
    qc = rng.integers(0, centres.shape[0], size=n_routes)
    q8 = np.clip(np.rint(128 + 30 * (centres[qc] + 0.6 * rng.normal(0, 1, size=(n_routes, 128)))), 0,
                 255).astype(np.uint8)
    queries = _vectors(q8, dtype, levels, rng)
    routes = _routes(rng, card, seeds, n_routes, n_labels)
    graph = dict(graph)
    attrs = dict(attrs)
    if filters:
        rows = graph["adjacency"].shape[0]
        mask = np.zeros(rows, np.uint64)
        for _ in range(6):
            mask |= np.uint64(1) << rng.integers(0, 64, size=rows).astype(np.uint64)
        graph["row_filter_mask"] = mask
        fb = np.zeros(n_routes, np.uint64)
        for _ in range(8):
            fb |= np.uint64(1) << rng.integers(0, 64, size=n_routes).astype(np.uint64)
        fb[::9] = np.uint64(0xFFFFFFFFFFFFFFFF)
        routes["filter_bits"] = fb
        attrs["range_values"] = rng.uniform(0, 100, size=(n, 2)).astype(np.float32)
        routes["range_modes"] = rng.integers(0, 4, size=(n_routes, 2)).astype(np.uint8)
        lo = rng.uniform(0, 40, size=(n_routes, 2)).astype(np.float32)
        routes["range_lower"] = lo
        routes["range_upper"] = (lo + rng.uniform(30, 90, size=(n_routes, 2))).astype(np.float32)
    params = dict(queue_size=qs, early_stop_mode=mode, finish_limit=finish, max_steps=max_steps, result_width=topk)
    return dict(params=params, graph=graph, attrs=attrs, base=vec, queries=queries, routes=routes, dtype=dtype)


@functools.lru_cache(maxsize=None)
def build_low_case(name: str, seed: int = 11, n: int = 2400, n_labels: int = 5, n_routes: int = 48, topk: int = 10):
    """Posting-route case: each route scans its rarer label's members with the
    other label as a residual filter (one DNF clause)."""
    c = next(x for x in LOW_CASES if x[0] == name)
    _, dtype, levels = c
    base, centres, graph, attrs, card, seeds = _data(seed, 128, n, n_labels, 32, 8)
    rng = np.random.default_rng([seed, 200 + LOW_NAMES.index(name)])
    vec = _vectors(base, dtype, levels, rng)
    qc = rng.integers(0, centres.shape[0], size=n_routes)
    q8 = np.clip(np.rint(128 + 30 * (centres[qc] + 0.6 * rng.normal(0, 1, size=(n_routes, 128)))), 0,
                 255).astype(np.uint8)
    queries = _vectors(q8, dtype, levels, rng)
    routes = _routes(rng, card, seeds, n_routes, n_labels)
    posting_ids = graph["row_to_sample"]  # the label graphs' rows are each label's members, grouped by label
    off = graph["label_offset"].astype(np.uint64)
    begin = off[routes["primary_label"]]
    count = card[routes["primary_label"]].astype(np.uint32)
    ip, ind, prim = routes["qlabel_indptr"], routes["qlabel_indices"], routes["primary_label"]
    residual = [np.array([x for x in ind[ip[r]:ip[r + 1]] if x != prim[r]], np.uint32) for r in range(n_routes)]
    hptr = np.zeros(n_routes + 1, np.uint32)
    hptr[1:] = np.cumsum([len(x) for x in residual])
    clauses = np.zeros((n_routes, 4), np.uint32)
    clauses[:, 0], clauses[:, 1] = hptr[:-1], hptr[1:]
    routes.update(pred_offsets=np.arange(n_routes + 1, dtype=np.uint32), clauses=clauses,
                  pred_handles=np.concatenate(residual + [np.zeros(1, np.uint32)]).astype(np.uint32),
                  pred_enabled=np.array([len(x) > 0 for x in residual], np.uint8))
    return dict(attrs=attrs, base=vec, queries=queries, routes=routes, dtype=dtype, posting_ids=posting_ids,
                begin=begin, count=count, topk=topk)


def case_digest(c: dict) -> str:
    """SHA-256 over every input array of a case (detects generator drift)."""
    h = hashlib.sha256()
    for grp in ("graph", "attrs", "routes"):
        for k in sorted(c.get(grp, {})):
            h.update(k.encode())
            h.update(np.ascontiguousarray(c[grp][k]).tobytes())
    for k in ("base", "queries", "posting_ids", "begin", "count"):
        if k in c:
            h.update(np.ascontiguousarray(c[k]).tobytes())
    return h.hexdigest()
