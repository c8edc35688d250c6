"""Records the reference's own Full-GPU kernels on the seeded cases of
tests/ref_full_cases.py into tests/golden/reference_full_gpu.npz.

Runs on a machine with a CUDA device and oracle/_ref/libgofann_ref_full_gpu.so
(the reference's src/search/full_gpu/backend_full_gpu.cu compiled in place by
`make -C oracle refkernels`).  Per case it stores the SHA-256 of the inputs
(so a replay can prove it rebuilt the same inputs) and the reference
kernel's ids, distance bits and step counts; it also stores the block
pickup's choice on crafted tie-heavy frontiers.  tests/test_oracle_golden.py
replays the CPU oracle against this file without a GPU.

    python tests/golden/make_ref_full_gpu_golden.py [out.npz]
"""
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
for p in (str(ROOT), str(ROOT / "go-fann_b200"), str(ROOT / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402

import ref_full_cases as R  # noqa: E402
from oracle import ref_kernels as RK  # noqa: E402


def pickup_probe():
    rng = np.random.default_rng(2025)
    n_cases, stride = 600, 520
    keys = rng.integers(0, 6, size=(n_cases, stride)).astype(np.float32)
    used = rng.random((n_cases, stride)) < 0.3
    sizes = rng.integers(2, stride + 1, size=n_cases).astype(np.int32)
    return keys, used, sizes


def main(out: str) -> None:
    arrays = {}
    for name in R.CASE_NAMES:
        case = R.build_case(name)
        ref = RK.run_reference_full(case)
        arrays[f"{name}/digest"] = np.frombuffer(bytes.fromhex(R.case_digest(case)), np.uint8)
        arrays[f"{name}/ids"] = ref["ids"]
        arrays[f"{name}/dist_bits"] = np.ascontiguousarray(ref["dists"], np.float32).view(np.uint32)
        arrays[f"{name}/steps"] = ref["steps"]
        print(f"{name}: {ref['ids'].shape[0]} routes, mean steps {ref['steps'].mean():.1f}", flush=True)
    for name in R.LOW_NAMES:
        case = R.build_low_case(name)
        ref = RK.run_reference_full_low(case)
        arrays[f"{name}/digest"] = np.frombuffer(bytes.fromhex(R.case_digest(case)), np.uint8)
        arrays[f"{name}/ids"] = ref["ids"]
        arrays[f"{name}/dist_bits"] = np.ascontiguousarray(ref["dists"], np.float32).view(np.uint32)
        print(f"{name}: {ref['ids'].shape[0]} posting routes", flush=True)
    keys, used, sizes = pickup_probe()
    arrays["pickup/keys"], arrays["pickup/used"], arrays["pickup/sizes"] = keys, used, sizes
    arrays["pickup/picked"] = RK.block_pickup_cases(keys, used, sizes)
    np.savez_compressed(out, **arrays)
    print(f"wrote {out}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(HERE / "reference_full_gpu.npz"))
