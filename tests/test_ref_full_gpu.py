"""The Full-GPU exact mode pinned to the reference's own kernels.

Three-way agreement on the seeded cases of tests/ref_full_cases.py: the
reference's full_gpu_highfreq_kernel / full_gpu_lowfreq_kernel
(src/search/full_gpu/backend_full_gpu.cu, compiled in place by
oracle/Makefile and run on a B200 -- live where oracle/_ref was built, and
as the recorded tests/golden/reference_full_gpu.npz), the CPU oracle, and
gofann_exact_search / gofann_exact_posting_scan.  Ids, distance bits and step
counts must all be equal.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import ref_full_cases as R
from fixtures import fbits
from gofann import _abi as A
from oracle import oracle as O, ref_kernels as RK
from test_exact_gpu import run_exact

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_full_gpu.npz"


@pytest.fixture(scope="module")
def L():
    assert torch.cuda.is_available()
    return A.lib()


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN) if GOLDEN.exists() else None


def _ours(L, c):
    return run_exact(L, c["graph"], c["attrs"], c["base"], c["dtype"], c["queries"], c["routes"], **c["params"])


@pytest.mark.parametrize("name", R.CASE_NAMES)
def test_exact_search_equals_reference_kernel(L, golden, name):
    c = R.build_case(name)
    ids, d, steps = _ours(L, c)
    wi, wd, ws = O.exact_search(c["graph"], c["attrs"], c["base"], c["dtype"], c["queries"], c["routes"],
                                threads=8, **c["params"])
    assert np.array_equal(ids, wi) and np.array_equal(fbits(d), fbits(wd)) and np.array_equal(steps, ws)
    refs = []
    if golden is not None and f"{name}/ids" in golden:
        assert bytes(golden[f"{name}/digest"]).hex() == R.case_digest(c), "case inputs drifted from the golden file"
        refs.append((golden[f"{name}/ids"], golden[f"{name}/dist_bits"], golden[f"{name}/steps"]))
    if RK.full_available():
        r = RK.run_reference_full(c)
        refs.append((r["ids"], fbits(r["dists"]), r["steps"]))
    assert refs, "neither the golden file nor the reference harness is available"
    for ri, rd, rs in refs:
        assert np.array_equal(ids, ri), f"ids differ in {np.count_nonzero(np.any(ids != ri, axis=1))} routes"
        assert np.array_equal(fbits(d), rd)
        assert np.array_equal(steps, rs)


@pytest.mark.parametrize("name", R.LOW_NAMES)
def test_exact_posting_scan_equals_reference_kernel(L, golden, name):
    import ctypes as C
    from fixtures import dev, dev_dict, host
    c = R.build_low_case(name)
    k = c["topk"]
    rs, at = A.fill_routes(dev_dict(c["routes"])), A.fill_attrs(dev_dict(c["attrs"]))
    keep = dev_dict(c["routes"]), dev_dict(c["attrs"])
    rs, at = A.fill_routes(keep[0]), A.fill_attrs(keep[1])
    n = rs.n_routes
    ids = torch.empty((n, k), dtype=torch.int32, device="cuda")
    d = torch.empty((n, k), dtype=torch.float32, device="cuda")
    db, dq = dev(c["base"]), dev(c["queries"])
    pid, pb, pc = dev(c["posting_ids"]), dev(c["begin"]), dev(c["count"])
    A.check(L.gofann_exact_posting_scan(A.ptr(db), c["dtype"], c["base"].shape[0], c["base"].shape[1], A.ptr(dq),
                                        C.byref(at), C.byref(rs), A.ptr(pid), A.ptr(pb), A.ptr(pc), k, A.ptr(ids),
                                        A.ptr(d), torch.cuda.current_stream().cuda_stream), "exact_posting_scan")
    torch.cuda.synchronize()
    gi, gd = host(ids, np.uint32), fbits(d.cpu().numpy())
    wi, wd = O.exact_posting_scan(c["base"], c["dtype"], c["queries"], c["attrs"], c["routes"], c["posting_ids"],
                                  c["begin"], c["count"], k)
    assert np.array_equal(gi, wi) and np.array_equal(gd, fbits(wd))
    refs = []
    if golden is not None and f"{name}/ids" in golden:
        assert bytes(golden[f"{name}/digest"]).hex() == R.case_digest(c)
        refs.append((golden[f"{name}/ids"], golden[f"{name}/dist_bits"]))
    if RK.full_available():
        r = RK.run_reference_full_low(c)
        refs.append((r["ids"], fbits(r["dists"])))
    assert refs
    for ri, rd in refs:
        assert np.array_equal(gi, ri) and np.array_equal(gd, rd)


def test_block_pickup_equals_reference(golden):
    """The pickup rule on tie-heavy frontiers: the oracle's choice equals the
    reference block pickup's (recorded, and live where the harness is built)."""
    import sys
    sys.path.insert(0, str(GOLDEN.parent))
    from make_ref_full_gpu_golden import pickup_probe
    keys, used, sizes = pickup_probe()
    refs = []
    if golden is not None and "pickup/picked" in golden:
        refs.append(golden["pickup/picked"])
    if RK.full_available():
        refs.append(RK.block_pickup_cases(keys, used, sizes))
    assert refs
    stride = keys.shape[1]
    vals = np.arange(stride, dtype=np.uint32)[None, :] | (used.astype(np.uint32) << 31)
    mine = np.array([O.full_pickup_index(keys[c], vals[c], int(sizes[c])) for c in range(keys.shape[0])])
    for r in refs:
        assert np.array_equal(mine, r), f"{np.count_nonzero(mine != r)} of {len(r)} frontiers differ"
