"""The 1-bit RaBitQ estimator pinned to the reference's own device code.

score_rabitq_code_device<true> (src/search/rabitq/backend_rabitq.cu:
3100-3200), compiled in place by oracle/Makefile and run on a B200 (live
where oracle/_ref was built, and as the recorded
tests/golden/reference_rabitq_score.npz), gofann_rabitq_score and the CPU
oracle must give the same estimate bits on every pair of the seeded cases
of tests/ref_rabitq_cases.py (padded dims 128, 512, 4096)."""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest
import torch

import ref_rabitq_cases as R
from fixtures import dev, dev_dict, fbits
from gofann import _abi as A
from oracle import oracle as O, ref_kernels as RK

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_rabitq_score.npz"


@pytest.mark.parametrize("pd", R.PADDED_DIMS)
def test_rabitq_score_equals_reference_estimator(pd):
    L = A.lib()
    c = R.build_case(pd)
    cs, pp = A.fill_codes(dev_dict(R.codes_dict(c))), None
    dc, dp = dev_dict(R.codes_dict(c)), dev_dict(R.prep_dict(c))
    cs, pp = A.fill_codes(dc), A.fill_prepared(dp)
    n = c["pair_row"].shape[0]
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    ip = torch.empty(n, dtype=torch.int32, device="cuda")
    pr, pt = dev(c["pair_row"]), dev(c["pair_point"])
    A.check(L.gofann_rabitq_score(C.byref(cs), C.byref(pp), A.ptr(pr), A.ptr(pt), n, A.ptr(out), A.ptr(ip),
                                  torch.cuda.current_stream().cuda_stream), "rabitq_score")
    torch.cuda.synchronize()
    ours = fbits(out.cpu().numpy())
    oracle, _ = O.rabitq_score(R.codes_dict(c), R.prep_dict(c), c["pair_row"], c["pair_point"])
    assert np.array_equal(ours, fbits(oracle))
    refs = []
    if GOLDEN.exists():
        g = np.load(GOLDEN)
        assert bytes(g[f"pd{pd}/digest"]).hex() == R.case_digest(c)
        refs.append(g[f"pd{pd}/est_bits"])
    if RK.rq_available():
        refs.append(fbits(RK.run_reference_rq_score(c)))
    assert refs, "neither the golden file nor the reference harness is available"
    for r in refs:
        assert np.array_equal(ours, r), f"{np.count_nonzero(ours != r)} of {n} estimates differ"
