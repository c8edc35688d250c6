"""Seeded inputs for the reference's own 1-bit RaBitQ estimator.

score_rabitq_code_device<kUseInt8Score = true> (src/search/rabitq/
backend_rabitq.cu:3100-3200) reads a point's 1-bit code, its factors and
anchor id, and the query's int8 vector, scale, k1xsumq and centroid
distances.  These cases fill all of them with seeded random values (numpy
PCG64 only, so the same seed gives the same inputs on any machine) at padded
dims 128, 512 and 4096: random bits, int8 queries over the full range, and
float factors whose products and sums round differently in the last bit
under different fma contractions -- what the recorded outputs of the
reference kernel (tests/golden/make_ref_rabitq_golden.py) pin.
"""
from __future__ import annotations

import hashlib

import numpy as np

PADDED_DIMS = (128, 512, 4096)


def build_case(pd: int, seed: int = 5, n_points=3000, n_rows=40, n_anchors=37, n_pairs=6000) -> dict:
    rng = np.random.default_rng([seed, pd])
    codes = rng.integers(0, 256, size=(n_points, pd // 8), dtype=np.uint8)
    factors = np.stack([rng.normal(1.0, 0.3, n_points), rng.normal(-2.0, 0.5, n_points),
                        rng.random(n_points)], 1).astype(np.float32)
    anchor_ids = rng.integers(0, n_anchors, size=n_points).astype(np.uint32)
    q8 = rng.integers(-127, 128, size=(n_rows, pd)).astype(np.int8)
    scale = (rng.random(n_rows) * 0.02 + 1e-4).astype(np.float32)
    k1 = rng.normal(0.0, 3.0, n_rows).astype(np.float32)
    gdist = (rng.random((n_rows, n_anchors)) * 4.0).astype(np.float32)
    pair_row = rng.integers(0, n_rows, size=n_pairs).astype(np.uint32)
    pair_point = rng.integers(0, n_points, size=n_pairs).astype(np.uint32)
    return dict(codes=codes, factors=factors, anchor_ids=anchor_ids, num_anchors=n_anchors, q8=q8, scale=scale,
                k1=k1, gdist=gdist, pair_row=pair_row, pair_point=pair_point, padded_dim=pd)


def case_digest(c: dict) -> str:
    h = hashlib.sha256()
    for k in ("codes", "factors", "anchor_ids", "q8", "scale", "k1", "gdist", "pair_row", "pair_point"):
        h.update(k.encode())
        h.update(np.ascontiguousarray(c[k]).tobytes())
    return h.hexdigest()


def codes_dict(c: dict) -> dict:
    return {"rq_codes": c["codes"], "rq_factors": c["factors"], "rq_anchor_ids": c["anchor_ids"],
            "num_anchors": c["num_anchors"]}


def prep_dict(c: dict) -> dict:
    return {"rq_q8": c["q8"], "rq_scale": c["scale"], "rq_k1xsumq": c["k1"], "rq_centroid_dist": c["gdist"]}
