"""Ray -> pose solver (src/ray_pose.cpp:11-252, src/linalg.cpp:8-203) on the CPU: the
oracle's restatement against DA3cpplib's own known answers and its own sources.

* tests/test_linalg.cpp's known answers (torch.linalg.qr and the torch-derived QL of its
  fixed matrix at 1e-8, the Jacobi smallest eigenpair residual at 1e-9, the 12-point
  homography recovery at 1e-6), from tests/golden/linalg_ref.json;
* the reference's ray_pose.cpp + linalg.cpp compiled unmodified into oracle/_ref: the
  oracle's solver equals it bit for bit (extrinsics, intrinsics and every double
  diagnostic) on seeded synthetic ray fields (tests/rayfield.py) with 0-50 % outliers,
  and on the committed outputs in tests/golden/raypose_ref.npz;
* edge cases: an all-zero confidence (degenerate: both refuse), directions with z
  under the 1e-4 threshold, fields with at most 8000 inliers and with more (the seeded
  subsample), a 1-row field.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O

import rayfield

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def gold():
    with open(os.path.join(GOLD, "linalg_ref.json")) as f:
        return json.load(f)


def test_linalg_known_answers(gold):
    A = np.array(gold["A"]).reshape(3, 3)
    q, r = O.qr(A)
    np.testing.assert_allclose(q.ravel(), gold["QR_Q"], atol=1e-8, rtol=0)
    np.testing.assert_allclose(r.ravel(), gold["QR_R"], atol=1e-8, rtol=0)
    q, l = O.ql3(A)
    np.testing.assert_allclose(q.ravel(), gold["QL_Q"], atol=1e-8, rtol=0)
    np.testing.assert_allclose(l.ravel(), gold["QL_L"], atol=1e-8, rtol=0)
    np.testing.assert_allclose(q @ l, A, atol=1e-12, rtol=0)
    M = np.array(gold["M4"]).reshape(4, 4)
    v = O.smallest_eigvec(M)
    lam = v @ M @ v / (v @ v)
    np.testing.assert_allclose(M @ v, lam * v, atol=1e-9, rtol=0)
    assert lam == pytest.approx(np.linalg.eigvalsh(M).min(), abs=1e-9)
    H = np.array(gold["Htrue"]).reshape(3, 3)
    pts = np.array(gold["pts"]).reshape(12, 2)
    P = np.c_[pts, np.ones(12)] @ H.T
    dst = P[:, :2] / P[:, 2:]
    Hr = O.homography(pts.ravel(), dst.ravel(), np.ones(12))
    np.testing.assert_allclose(Hr, H, atol=1e-6, rtol=0)


def test_linalg_bit_exact_vs_reference(gold):
    if O.ref_lib() is None:
        pytest.skip("oracle/_ref is not built")
    rng = np.random.default_rng(5)
    mats = [np.array(gold["A"]).reshape(3, 3)] + [rng.standard_normal((3, 3)) for _ in range(20)]
    for A in mats:
        for a, b in zip(O.qr(A), O.qr(A, impl="ref")):
            assert np.array_equal(a, b)
        for a, b in zip(O.ql3(A), O.ql3(A, impl="ref")):
            assert np.array_equal(a, b)
    for _ in range(10):
        X = rng.standard_normal((9, 9))
        S = X @ X.T
        assert np.array_equal(O.smallest_eigvec(S), O.smallest_eigvec(S, impl="ref"))
        src, dst, w = rng.uniform(-1, 1, 30), rng.uniform(-1, 1, 30), rng.uniform(0, 2, 15)
        assert np.array_equal(O.homography(src, dst, w), O.homography(src, dst, w, impl="ref"))


CASES = [(1, 48, 64, 0.2), (2, 64, 64, 0.5), (3, 40, 56, 0.0), (4, 96, 72, 0.3), (5, 288, 288, 0.2), (6, 1, 96, 0.1)]


@pytest.mark.parametrize("case", CASES, ids=[f"s{c[0]}_{c[1]}x{c[2]}" for c in CASES])
def test_solver_bit_exact_vs_reference(case):
    if O.ref_lib() is None:
        pytest.skip("oracle/_ref is not built")
    seed, hy, wx, outl = case
    ray, conf, truth = rayfield.field(seed, hy, wx, outliers=outl)
    img_h, img_w = hy * 14 // 8, wx * 14 // 8
    a = O.ray_pose(ray, conf, img_h, img_w)
    b = O.ray_pose(ray, conf, img_h, img_w, impl="ref")
    assert (a is None) == (b is None)
    if a is None:
        return
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    for k in a[2]:
        assert np.array_equal(a[2][k], b[2][k]), k
    if hy > 1 and outl <= 0.3:  # a well-posed field: the focal lengths come back
        np.testing.assert_allclose(a[2]["focal"], truth["f"], rtol=3e-2)


def test_solver_committed_outputs():
    z = np.load(os.path.join(GOLD, "raypose_ref.npz"))
    from golden.make_golden import RAY_CASES  # noqa: E402  (same seeds as the fixture)

    for seed, hy, wx, outl in RAY_CASES:
        ray, conf, _ = rayfield.field(seed, hy, wx, outliers=outl)
        ext, intr, d = O.ray_pose(ray, conf, hy * 14 // 8, wx * 14 // 8)
        assert np.array_equal(ext, z[f"s{seed}_ext"]) and np.array_equal(intr, z[f"s{seed}_intr"])
        diag = np.concatenate([d["R"].ravel(), d["T"], d["focal"], d["pp"], d["A"].ravel(), [d["n_inlier_best"]]])
        assert np.array_equal(diag, z[f"s{seed}_diag"])


def test_solver_edge_cases():
    ray, conf, _ = rayfield.field(7, 32, 32)
    zero = np.zeros_like(conf)
    assert O.ray_pose(ray, zero, 56, 56) is None
    if O.ref_lib() is not None:
        assert O.ray_pose(ray, zero, 56, 56, impl="ref") is None
        flat = ray.copy()
        flat[::3, :, 2] = 1e-5  # directions under the z threshold lose their weight
        a, b = O.ray_pose(flat, conf, 56, 56), O.ray_pose(flat, conf, 56, 56, impl="ref")
        assert (a is None) == (b is None)
        if a is not None:
            assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
