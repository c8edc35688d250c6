"""Generates tests/golden/reference_structures.npz from the REFERENCE's own
headers (include/smmh2.h, include/bin_heap.h, native_visited_hash.cuh,
posting_shortlist_heap.cuh, gpu_predicate_index.cuh, rabitq_lowfreq_merge.h,
fp16_l2.h), compiled in place by oracle/Makefile into
oracle/_ref/libgofann_ref.so and driven by oracle/ref_harness.cpp.

Run where the reference tree exists (the build container):
    make -C oracle ref && python tests/golden/make_golden.py
The fixture is committed; tests/test_oracle_golden.py replays every case
through the CPU oracle and requires bit-identical results.
"""
from __future__ import annotations

import ctypes as C
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import oracle as O  # noqa: E402

OUT = Path(__file__).resolve().parent / "reference_structures.npz"
FLT_MAX = np.float32(np.finfo(np.float32).max)
U32MAX = np.uint32(0xFFFFFFFF)


def main():
    R = O.rlib()
    if R is None:
        raise SystemExit("oracle/_ref/libgofann_ref.so missing: run `make -C oracle ref` with the reference tree")
    rng = np.random.default_rng(20261201)
    g = {}

    # 1. symmetric min-max heap: insert / pop_max / pop_min sequences with ties
    for case in range(12):
        n = int(rng.integers(20, 400))
        op = rng.choice([0, 0, 0, 1, 2], size=n).astype(np.int32)
        distinct = [4, 16, 1000][case % 3]
        key = rng.integers(0, distinct, size=n).astype(np.float32) * np.float32(0.5)
        payload = rng.permutation(n).astype(np.uint32)
        f, s, popped = O.seq_smmh(op, key, payload, use_ref=True)
        g[f"smmh{case}_op"], g[f"smmh{case}_key"], g[f"smmh{case}_payload"] = op, key, payload
        g[f"smmh{case}_first"], g[f"smmh{case}_second"], g[f"smmh{case}_popped"] = f, s, popped

    # 2. bounded result heap (push_heap/pop_heap) with ties
    for case in range(8):
        n = int(rng.integers(10, 600))
        cap = int(rng.choice([1, 5, 10, 100, 512]))
        key = rng.integers(0, [3, 50, 100000][case % 3], size=n).astype(np.float32)
        payload = rng.permutation(n).astype(np.uint32)
        f, s = O.seq_result_heap(key, payload, cap, use_ref=True)
        g[f"rheap{case}_key"], g[f"rheap{case}_payload"], g[f"rheap{case}_cap"] = key, payload, np.int32(cap)
        g[f"rheap{case}_first"], g[f"rheap{case}_second"] = f, s

    # 3. visited hash: collisions, repeats and a full table
    vals = [rng.integers(0, 1 << 31, size=3000, dtype=np.uint32),
            np.concatenate([np.arange(5000, dtype=np.uint32), np.arange(100, dtype=np.uint32)]),
            (rng.integers(0, 64, size=2000).astype(np.uint32) << np.uint32(16))]
    for case, v in enumerate(vals):
        v = v.astype(np.uint32)
        table = np.zeros(4096, np.uint32)
        found = np.zeros(v.shape[0], np.int32)
        R.ref_seq_hash(O.P(v), v.shape[0], O.P(table), O.P(found))
        g[f"hash{case}_values"], g[f"hash{case}_table"], g[f"hash{case}_found_before"] = v, table, found

    # 4. (dist, id) shortlist heap with ties, FLT_MAX, inf and sentinel ids
    for case in range(8):
        n = int(rng.integers(5, 800))
        k = int(rng.choice([1, 10, 32, 100, 400]))
        d = rng.integers(0, [4, 100, 10000][case % 3], size=n).astype(np.float32)
        d[rng.random(n) < 0.05] = FLT_MAX
        d[rng.random(n) < 0.02] = np.inf
        ids = rng.permutation(n + 50)[:n].astype(np.uint32)
        ids[rng.random(n) < 0.03] = U32MAX
        for srt in (0, 1):
            od, oi = O.shortlist(d, ids, k, sort=bool(srt), use_ref=True)
            g[f"sl{case}_{srt}_d"], g[f"sl{case}_{srt}_i"] = od, oi
        g[f"sl{case}_in_d"], g[f"sl{case}_in_i"], g[f"sl{case}_k"] = d, ids, np.int32(k)

    # 5. DNF predicate over a sample-major CSR with ranges
    n_samples, n_labels, n_routes = 300, 40, 60
    rows = [np.unique(rng.integers(0, n_labels, size=rng.integers(0, 8))).astype(np.uint32) for _ in range(n_samples)]
    csr_off = np.zeros(n_samples + 1, np.uint32)
    csr_off[1:] = np.cumsum([len(r) for r in rows])
    csr_lab = np.concatenate(rows).astype(np.uint32)
    base_ranges = rng.uniform(0, 100, size=(n_samples, 2)).astype(np.float32)
    route_off, clauses, handles, ranges = [0], [], [], []
    for r in range(n_routes):
        for _ in range(int(rng.integers(0, 4))):
            lb = len(handles)
            handles.extend(rng.integers(0, n_labels, size=rng.integers(0, 3)).tolist())
            rb = len(ranges)
            for _ in range(int(rng.integers(0, 3))):
                lo, hi = np.sort(rng.uniform(0, 100, size=2)).astype(np.float32)
                dim = int(rng.integers(0, 3))  # 2 == out of stride
                ranges.append([dim, int(rng.integers(0, 5)), lo.view(np.uint32), hi.view(np.uint32)])
            clauses.append([lb, len(handles), rb, len(ranges)])
        route_off.append(len(clauses))
    route_off = np.asarray(route_off, np.uint32)
    clauses = np.asarray(clauses, np.uint32).reshape(-1, 4)
    handles = np.asarray(handles, np.uint32)
    ranges = np.asarray(ranges, np.uint32).reshape(-1, 4)
    qr = rng.integers(0, n_routes, size=4000).astype(np.uint32)
    qs = rng.integers(0, n_samples + 3, size=4000).astype(np.uint32)
    out = np.zeros(4000, np.uint8)
    R.ref_pred_matches(O.P(route_off), n_routes, O.P(clauses), O.P(handles), O.P(ranges), O.P(base_ranges), 2,
                       O.P(csr_off), O.P(csr_lab), n_samples, O.P(qr), O.P(qs), 4000, O.P(out))
    g.update(pred_route_off=route_off, pred_clauses=clauses, pred_handles=handles, pred_ranges=ranges,
             pred_base_ranges=base_ranges, pred_csr_off=csr_off, pred_csr_lab=csr_lab, pred_qr=qr, pred_qs=qs,
             pred_out=out, pred_n_samples=np.int32(n_samples))

    # 6. predicate priority (penalty) incl. sentinels
    base = np.array([0, 1, -1, 3.3e38, FLT_MAX, np.inf, -np.inf, np.nan, 1e-30, 123.25], np.float32)
    passv = np.array([0, 0, 0, 0, 0, 0, 0, 0, 0, 1], np.uint8)
    for case, pen in enumerate([0.0, 0.15, 1e38]):
        o = np.zeros_like(base)
        R.ref_priority(O.P(base), O.P(passv), base.shape[0], C.c_float(pen), O.P(o))
        g[f"prio{case}_out"], g[f"prio{case}_pen"] = o, np.float32(pen)
    g["prio_base"], g["prio_pass"] = base, passv

    # 7. route -> original merge (duplicates across routes, sentinels)
    # cases 0-3 unsorted rows (hash dedup + sort), 4-5 sorted unique rows
    # (sorted-route heap), 6 one sorted route per query (single-route copy)
    for case in range(7):
        n_routes, n_q, width, topk = int(rng.integers(5, 60)), int(rng.integers(1, 20)), int(rng.choice([5, 10, 30])), 10
        if case == 6:
            n_q = n_routes
        r2q = rng.integers(0, n_q, size=n_routes).astype(np.uint32) if case < 6 else rng.permutation(n_q).astype(np.uint32)
        ids = rng.integers(0, 80, size=(n_routes, width)).astype(np.uint32)
        ids[rng.random(ids.shape) < 0.1] = U32MAX
        d = rng.integers(0, 40, size=(n_routes, width)).astype(np.float32)
        if case >= 4:
            for r in range(n_routes):
                uid = rng.permutation(200)[:width].astype(np.uint32)
                dd = rng.integers(0, 40, size=width).astype(np.float32)
                nvalid = int(rng.integers(0, width + 1))
                order = np.lexsort((uid, dd))
                ids[r] = U32MAX
                d[r] = FLT_MAX
                ids[r, :nvalid] = uid[order][:nvalid]
                d[r, :nvalid] = dd[order][:nvalid]
        oi = np.zeros((n_q, topk), np.uint32)
        od = np.zeros((n_q, topk), np.float32)
        strat = R.ref_route_merge(O.P(r2q), n_routes, n_q, O.P(ids), O.P(d), width, topk, O.P(oi), O.P(od))
        g.update({f"rm{case}_r2q": r2q, f"rm{case}_ids": ids, f"rm{case}_d": d, f"rm{case}_oi": oi,
                  f"rm{case}_od": od, f"rm{case}_strategy": np.int32(strat)})

    # 8. fp16 decode and scalar L2
    h = np.concatenate([rng.integers(0, 1 << 16, size=4000), [0, 0x8000, 0x0001, 0x03FF, 0x7C00, 0xFC00, 0x7BFF]])
    h = h.astype(np.uint16)
    dec = np.array([R.ref_fp16_decode(int(x)) for x in h], np.float32)
    rows16 = rng.standard_normal((64, 96)).astype(np.float16).view(np.uint16)
    q = rng.standard_normal(96).astype(np.float32)
    l2 = np.zeros(64, np.float32)
    R.ref_fp16_l2(O.P(rows16), O.P(q), 64, 96, O.P(l2))
    g.update(f16_bits=h, f16_decoded=dec, f16_rows=rows16, f16_query=q, f16_l2=l2)

    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(g)} arrays)")


if __name__ == "__main__":
    main()
