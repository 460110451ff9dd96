"""Ray -> pose solver on the GPU (da3b_ray_pose) against the CPU oracle, bit for bit.

The solver's GPU kernels compute in double with no multiply-add contraction, in the
reference's operation order, and the seeded draws / shuffle run on the host with the
same standard-library calls, so extrinsics, intrinsics and every double diagnostic
(R, T, focal, pp, the refit homography, the best inlier count) must equal the oracle's
(itself bit-exact with the reference's compiled ray_pose.cpp, tests/test_ray_pose.py):
* synthetic ray fields (tests/rayfield.py) from 48x64 to 288x288 points (the aux
  resolution of a 504x504 image), 0-50 % outliers, fields above the 8000-point refit
  cap, one view of a multi-view buffer, a degenerate (zero-confidence) field;
* the ray field a DA3 model's aux head produces on the GPU (da3b_infer_device), solved
  on the device and by the oracle from its host copy.
"""
import ctypes

import numpy as np
import pytest

import rayfield

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from da3cpplib_b200 import Model, synth

    m = Model(synth.ensure_gguf("da3-t", stress=True), 0)
    yield torch, m
    m.close()


def _planar(ray, conf):
    """interleaved [Hy][Wx][6] + [Hy][Wx] -> planar [7][Hy][Wx] (the aux head layout)."""
    return np.concatenate([ray.transpose(2, 0, 1), conf[None]], 0).astype(np.float32)


def _gpu_solve(torch, m, planes, n_views, view, hy, wx, img_h, img_w):
    d = torch.from_numpy(np.ascontiguousarray(planes)).cuda()
    torch.cuda.synchronize()
    ext = np.zeros(12, np.float32)
    intr = np.zeros(9, np.float32)
    diag = np.zeros(26, np.float64)
    rc = m.lib.da3b_ray_pose(m.ctx, ctypes.c_void_p(d.data_ptr()), n_views, view, hy, wx, img_h, img_w,
                             ext.ctypes.data, intr.ctypes.data, diag.ctypes.data, None)
    return rc, ext, intr, diag


def _oracle(ray, conf, img_h, img_w):
    from oracle import oracle as O

    r = O.ray_pose(ray, conf, img_h, img_w)
    if r is None:
        return None
    ext, intr, d = r
    diag = np.concatenate([d["R"].ravel(), d["T"], d["focal"], d["pp"], d["A"].ravel(), [d["n_inlier_best"]]])
    return ext.ravel(), intr.ravel(), diag


CASES = [(1, 48, 64, 0.2), (2, 64, 64, 0.5), (3, 40, 56, 0.0), (5, 288, 288, 0.2), (8, 200, 160, 0.05)]


@pytest.mark.parametrize("case", CASES, ids=[f"s{c[0]}_{c[1]}x{c[2]}" for c in CASES])
def test_ray_pose_bit_exact(env, case):
    torch, m = env
    seed, hy, wx, outl = case
    ray, conf, _ = rayfield.field(seed, hy, wx, outliers=outl)
    img_h, img_w = hy * 14 // 8, wx * 14 // 8
    ref = _oracle(ray, conf, img_h, img_w)
    rc, ext, intr, diag = _gpu_solve(torch, m, _planar(ray, conf)[:, None], 1, 0, hy, wx, img_h, img_w)
    assert ref is not None and rc == 0, m.last_error
    assert np.array_equal(ext, ref[0]) and np.array_equal(intr, ref[1])
    assert np.array_equal(diag, ref[2]), np.nonzero(diag != ref[2])
    if hy * wx > 20000:
        assert diag[25] > 8000  # the seeded refit subsample was exercised


def test_ray_pose_view_of_batch_and_degenerate(env):
    torch, m = env
    fields = [rayfield.field(30 + v, 56, 48) for v in range(3)]
    planes = np.stack([_planar(r, c) for r, c, _ in fields], 1)  # [7][3][56][48]
    ref = _oracle(fields[2][0], fields[2][1], 98, 84)
    rc, ext, intr, diag = _gpu_solve(torch, m, planes, 3, 2, 56, 48, 98, 84)
    assert rc == 0 and np.array_equal(ext, ref[0]) and np.array_equal(diag, ref[2])
    zero = _planar(fields[0][0], np.zeros_like(fields[0][1]))[:, None]
    rc, *_ = _gpu_solve(torch, m, zero, 1, 0, 56, 48, 98, 84)
    assert rc == 1 and _oracle(fields[0][0], np.zeros_like(fields[0][1]), 98, 84) is None


def test_ray_pose_on_model_rays(env):
    """The aux ray head's output of a DA3 model, solved on the device == the oracle's
    solver on the host copy of the same field."""
    torch, m = env
    from da3cpplib_b200 import synth

    for k in range(3):
        img = synth.image(synth.IMAGE_SEED, 60 + k, 112, 112)
        out = m.infer(img, rays=True)
        rays = out["rays"]  # [7][1][64][64], confidence after exp+1
        ray = np.ascontiguousarray(rays[:6, 0].transpose(1, 2, 0))
        conf = np.ascontiguousarray(rays[6, 0])
        ref = _oracle(ray, conf, 112, 112)
        rc, ext, intr, diag = _gpu_solve(torch, m, rays, 1, 0, 64, 64, 112, 112)
        assert (ref is None) == (rc == 1)
        if ref is not None:
            assert np.array_equal(ext, ref[0]) and np.array_equal(intr, ref[1]) and np.array_equal(diag, ref[2])
