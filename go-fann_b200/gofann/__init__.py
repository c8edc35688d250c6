"""gofann — B200 filtered-ANN search path (host side of the C ABI).

The compute lives in libgofann_b200.so (hand-written sm_100a CUDA behind
include/gofann.h); this package loads it through ctypes, builds index
artefacts and route plans in the reference's layout, and drives the batch
pipeline on torch-managed device memory.
"""
from . import _abi  # noqa: F401

__all__ = ["_abi"]
