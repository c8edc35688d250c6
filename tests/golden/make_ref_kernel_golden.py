"""Records the reference's own device traversal on the seeded cases of
tests/ref_kernel_cases.py into tests/golden/reference_pq_kernel.npz.

Runs on a machine with a CUDA device and oracle/_ref/libgofann_ref_kernels.so
(the reference's src/search/pq/backend_pq.cu compiled in place by
`make -C oracle refkernels`).  Per case it stores the SHA-256 of the inputs
(so a replay can prove it rebuilt the same inputs), the reference kernel's
shortlist ids, distance bits, step counts and expansion traces, and the
SHA-256 of the PQ table bits its kernel built.  tests/test_oracle_golden.py
replays the CPU oracle against this file without a GPU.

    python tests/golden/make_ref_kernel_golden.py [out.npz]
"""
import hashlib
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
for p in (str(ROOT), str(ROOT / "go-fann_b200"), str(ROOT / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402

import ref_kernel_cases as R  # noqa: E402
from oracle import ref_kernels as RK  # noqa: E402


def main(out: str) -> None:
    arrays = {}
    for name in R.CASE_NAMES:
        case = R.build_case(name)
        ref = RK.run_reference_pq(case, trace_width=64)
        arrays[f"{name}/digest"] = np.frombuffer(bytes.fromhex(R.case_digest(case)), np.uint8)
        arrays[f"{name}/ids"] = ref["ids"]
        arrays[f"{name}/dist_bits"] = np.ascontiguousarray(ref["dists"], np.float32).view(np.uint32)
        arrays[f"{name}/steps"] = ref["steps"]
        arrays[f"{name}/trace"] = ref["trace"]
        arrays[f"{name}/table_sha256"] = np.frombuffer(
            hashlib.sha256(np.ascontiguousarray(ref["pq_table"], np.float32).tobytes()).digest(), np.uint8)
        print(f"{name}: {ref['ids'].shape[0]} routes, mean steps {ref['steps'].mean():.1f}", flush=True)
    # the reference's tie-deciding primitives on crafted inputs with many
    # equal keys: cooperative pickup, and the binary result heap with its
    # final emptying order
    rng = np.random.default_rng(2024)
    n_cases, stride = 600, 520
    keys = rng.integers(0, 6, size=(n_cases, stride)).astype(np.float32)
    used = rng.random((n_cases, stride)) < 0.3
    sizes = rng.integers(2, stride + 1, size=n_cases).astype(np.int32)
    arrays["pickup/keys"], arrays["pickup/used"], arrays["pickup/sizes"] = keys, used, sizes
    arrays["pickup/picked"] = RK.pickup_cases(keys, used, sizes)
    for cap in (1, 10, 33, 100, 200):
        hk = rng.integers(0, 12, size=(200, 400)).astype(np.float32)
        hp = np.tile(np.arange(400, dtype=np.uint32), (200, 1))
        f, p = RK.result_heap_cases(hk, hp, cap)
        arrays[f"rheap{cap}/keys"], arrays[f"rheap{cap}/first"], arrays[f"rheap{cap}/payload"] = hk, f, p
    print("pickup and result-heap probes recorded", flush=True)
    np.savez_compressed(out, **arrays)
    print(f"wrote {out}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(HERE / "reference_pq_kernel.npz"))
