"""Records the reference's own 1-bit RaBitQ estimator
(score_rabitq_code_device<true>, src/search/rabitq/backend_rabitq.cu:
3100-3200, compiled in place by `make -C oracle refkernels`) on the seeded
cases of tests/ref_rabitq_cases.py into tests/golden/reference_rabitq_score.npz:
per padded dim the SHA-256 of the inputs and the estimate bits of every
pair.  Needs a CUDA device.

    python tests/golden/make_ref_rabitq_golden.py [out.npz]
"""
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
for p in (str(ROOT), str(ROOT / "go-fann_b200"), str(ROOT / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402

import ref_rabitq_cases as R  # noqa: E402
from oracle import ref_kernels as RK  # noqa: E402


def main(out: str) -> None:
    arrays = {}
    for pd in R.PADDED_DIMS:
        c = R.build_case(pd)
        est = RK.run_reference_rq_score(c)
        arrays[f"pd{pd}/digest"] = np.frombuffer(bytes.fromhex(R.case_digest(c)), np.uint8)
        arrays[f"pd{pd}/est_bits"] = np.ascontiguousarray(est, np.float32).view(np.uint32)
        print(f"padded dim {pd}: {est.shape[0]} pairs", flush=True)
    np.savez_compressed(out, **arrays)
    print(f"wrote {out}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(HERE / "reference_rabitq_score.npz"))
