"""RaBitQ query preparation on the tensor cores against FP64.

gofann_rabitq_rotate (q' = q . R) and gofann_rabitq_centroid_dist_tc
(max(0, -2 q.c + |q|^2 + |c|^2)) run a hand-written tcgen05 GEMM.  They are
checked the way the reference checks its pedantic-FP32 cuBLAS versions
(tests/native/rabitq_query_rotation_test.cu:10-60): the same shapes (1x1x1
up to 3x4096x4096, rectangular and padded), queries uniform in [-1, 1],
rotation entries uniform in [-1, 1] / sqrt(d), all-zero queries, a rejected
shape, and centroid distances with the query rows as anchors (zeros on the
diagonal exercise the clamp).  Tolerances are the reference's:
|err| <= 2e-5 + 2e-5 |x| for the rotation and 1e-3 + 2e-5 x for distances,
in the FP32-accurate 3xTF32 mode; larger shapes cover many tiles.  The
one-pass TF32 mode (used at index time) is held to TF32 accuracy.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from gofann import _abi as A

pytestmark = pytest.mark.gpu

SHAPES = [(1, 1, 1), (7, 17, 32), (33, 65, 96), (13, 512, 512), (3, 4096, 4096), (300, 500, 512),
          (1000, 4096, 4096), (129, 130, 257)]


@pytest.fixture(scope="module")
def L():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return A.lib()


def stream():
    return torch.cuda.current_stream().cuda_stream


def rotate(L, q, r, precision=A.GEMM_TF32X3, expect=0):
    n, d = q.shape
    p = r.shape[1]
    dq, dr = torch.from_numpy(q).cuda(), torch.from_numpy(r).cuda()
    out = torch.full((n, p), float("nan"), dtype=torch.float32, device="cuda")
    nbytes = L.gofann_rabitq_gemm_scratch_bytes(n, d, p, precision)
    scratch = torch.empty(max(nbytes, 256), dtype=torch.uint8, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = L.gofann_rabitq_rotate(A.ptr(dq), n, d, A.ptr(dr), p, precision, A.ptr(out), A.ptr(scratch), nbytes,
                                A.ptr(status), stream())
    torch.cuda.synchronize()
    assert st == expect, L.gofann_last_error()
    assert int(status.item()) == 0
    return out.cpu().numpy()


def centroid_dist(L, q, anchors, precision=A.GEMM_TF32X3):
    n, p = q.shape
    a = anchors.shape[0]
    dq, da = torch.from_numpy(q).cuda(), torch.from_numpy(anchors).cuda()
    out = torch.full((n, a), float("nan"), dtype=torch.float32, device="cuda")
    nbytes = L.gofann_rabitq_gemm_scratch_bytes(n, p, a, precision)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    A.check(L.gofann_rabitq_centroid_dist_tc(A.ptr(dq), n, A.ptr(da), a, p, precision, A.ptr(out), A.ptr(scratch),
                                             nbytes, A.ptr(status), stream()), "centroid_dist_tc")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return out.cpu().numpy()


def inputs(n, d, p, zero=False, seed=20260927):
    rng = np.random.default_rng(seed + n * 7 + d * 13 + p)
    q = np.zeros((n, d), np.float32) if zero else rng.uniform(-1, 1, size=(n, d)).astype(np.float32)
    r = (rng.uniform(-1, 1, size=(d, p)) / np.sqrt(d)).astype(np.float32)
    return q, r


@pytest.mark.parametrize("n,d,p", SHAPES)
def test_rotation_fp64(L, n, d, p):
    q, r = inputs(n, d, p)
    got = rotate(L, q, r)
    want = q.astype(np.float64) @ r.astype(np.float64)
    assert np.all(np.isfinite(got))
    err = np.abs(got - want)
    assert np.all(err <= 2e-5 + 2e-5 * np.abs(want)), f"max err {err.max():.3g}"


def test_rotation_zero_queries(L):
    q, r = inputs(7, 17, 32, zero=True)
    assert np.array_equal(rotate(L, q, r), np.zeros((7, 32), np.float32))


def test_rotation_rejects_dim_above_padded(L):
    q, r = inputs(7, 33, 32)
    rotate(L, q, r[:, :32], expect=A.ERR_INVALID)  # dim 33 > padded_dim 32


@pytest.mark.parametrize("n,d,p", [(7, 17, 32), (300, 500, 512), (1000, 4096, 4096)])
def test_rotation_tf32_one_pass(L, n, d, p):
    q, r = inputs(n, d, p)
    got = rotate(L, q, r, precision=A.GEMM_TF32)
    want = q.astype(np.float64) @ r.astype(np.float64)
    # the tensor core reads 10 mantissa bits of each operand: a product is off
    # by at most 2^-9 of |q||r|
    bound = 2.0 ** -9 * (np.abs(q).astype(np.float64) @ np.abs(r).astype(np.float64)) + 1e-6
    assert np.all(np.abs(got - want) <= bound)


@pytest.mark.parametrize("n,d", [(1, 1), (7, 17), (33, 65), (13, 512), (3, 4096), (300, 500)])
def test_centroid_distances_fp64(L, n, d):
    q, _ = inputs(n, d, d)
    got = centroid_dist(L, q, q)  # the query rows as anchors, as the reference's test does
    qd = q.astype(np.float64)
    want = ((qd[:, None, :] - qd[None, :, :]) ** 2).sum(-1)
    assert np.all(np.isfinite(got)) and np.all(got >= 0)
    assert np.all(np.abs(got - want) <= 1e-3 + 2e-5 * want)


def test_centroid_distances_many_anchors(L):
    rng = np.random.default_rng(3)
    q = rng.standard_normal((517, 512)).astype(np.float32)
    c = rng.standard_normal((1100, 512)).astype(np.float32)
    got = centroid_dist(L, q, c)
    want = ((q.astype(np.float64) ** 2).sum(1)[:, None] + (c.astype(np.float64) ** 2).sum(1)[None, :] -
            2 * q.astype(np.float64) @ c.astype(np.float64).T)
    want = np.maximum(want, 0)
    assert np.all(np.abs(got - want) <= 1e-3 + 2e-5 * want)
