"""Camera pose of DA3 (the camera-token MLP of CamPose::pose, src/cam_pose.cpp:8-83)
through the C ABI against the CPU oracle.

Bounds: pose encodings |gpu - ref| / max(1, |ref|) <= max(2e-2, 2 * floor), floor being
the same error between the oracle with and without ggml's activation quantisation; the
extrinsic rotations orthonormal to 1e-4; intrinsics' focal lengths within the same
relative bound and the principal point at the image centre exactly."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _err(a, b):
    return float(np.max(np.abs(a - b) / np.maximum(1.0, np.abs(b))))


def _check(pe, ext, intr, ref_q, ref_f, H, W):
    rq = ref_q.reshape(-1, 30)
    rf = ref_f.reshape(-1, 30)
    floor = _err(rf[:, :9], rq[:, :9])
    bound = max(2e-2, 2 * floor)
    assert _err(pe, rq[:, :9]) <= bound, (_err(pe, rq[:, :9]), floor)
    R = ext[:, :, :3]
    assert np.abs(R @ R.transpose(0, 2, 1) - np.eye(3)).max() <= 1e-4
    assert _err(ext.reshape(-1, 12), rq[:, 9:21]) <= 4 * bound
    assert np.all(intr[:, 0, 2] == W / 2) and np.all(intr[:, 1, 2] == H / 2) and np.all(intr[:, 2, 2] == 1)
    assert np.max(np.abs(intr[:, 0, 0] / rq[:, 21] - 1)) <= 4 * bound
    assert np.max(np.abs(intr[:, 1, 1] / rq[:, 25] - 1)) <= 4 * bound


def test_pose_single_view(cuda):
    from da3cpplib_b200 import Model, synth
    from oracle.oracle import Oracle

    path = synth.ensure_gguf("da3-t", stress=True)
    img = synth.image(synth.IMAGE_SEED, 3, 112, 112)
    m = Model(path, 0)
    m.infer(img)
    pe, ext, intr = m.pose(1)
    rq = Oracle(path, act_quant=True).infer(img)["pose"]
    rf = Oracle(path, act_quant=False).infer(img)["pose"]
    _check(pe, ext, intr, rq, rf, 112, 112)


def test_pose_multi_view_original_order(cuda):
    from da3cpplib_b200 import Model, synth
    from oracle.oracle import Oracle

    path = synth.ensure_gguf("da3-t", stress=True)
    imgs = [synth.image(synth.IMAGE_SEED, 10 + i, 112, 112) for i in range(4)]
    m = Model(path, 0)
    m.infer(np.stack(imgs), views_per_scene=4)
    pe, ext, intr = m.pose(4)
    rq = Oracle(path, act_quant=True).infer_mv(imgs)
    rf = Oracle(path, act_quant=False).infer_mv(imgs)
    assert m.ref_views(1) == [rq["b_idx"]]
    _check(pe, ext, intr, rq["pose"], rf["pose"], 112, 112)


def test_capi_pose_entry_points(lib, cuda, tmp_path):
    from da3cpplib_b200 import synth

    da3 = synth.ensure_gguf("da3-t", stress=True)
    da2 = synth.ensure_gguf("da2-t", stress=True)
    paths = []
    for i in range(3):
        img = synth.image(synth.IMAGE_SEED, 20 + i, 112, 112)
        f = tmp_path / f"v{i}.ppm"
        f.write_bytes(b"P6\n112 112\n255\n" + img.tobytes())
        paths.append(str(f).encode())
    ctx = lib.da_capi_load(da3.encode(), 1)
    assert ctx
    try:
        n, h, w = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        ext = np.zeros((3, 12), np.float32)
        intr = np.zeros((3, 9), np.float32)
        arr = (ctypes.c_char_p * 3)(*paths)
        p = lib.da_capi_depth_pose_multi(ctx, arr, 3, ctypes.byref(h), ctypes.byref(w), ctypes.byref(n),
                                         ext.ctypes.data, intr.ctypes.data)
        assert p, lib.da_capi_last_error(ctx)
        lib.da_capi_free_floats(p)
        pe2, ext2, intr2 = np.zeros((3, 9), np.float32), np.zeros((3, 12), np.float32), np.zeros((3, 9), np.float32)
        assert lib.da3b_last_pose(ctx, 3, pe2.ctypes.data, ext2.ctypes.data, intr2.ctypes.data) == 0
        assert np.array_equal(ext, ext2) and np.array_equal(intr, intr2)
        R = ext.reshape(3, 3, 4)[:, :, :3]
        assert np.abs(R @ R.transpose(0, 2, 1) - np.eye(3)).max() <= 1e-4
        e1 = np.zeros(12, np.float32)
        k1 = np.zeros(9, np.float32)
        assert lib.da_capi_pose_path(ctx, paths[0], e1.ctypes.data, k1.ctypes.data) == 0
        assert k1[2] == 56 and k1[5] == 56
    finally:
        lib.da_capi_free(ctx)
    ctx = lib.da_capi_load(da2.encode(), 1)
    assert ctx
    try:
        e1 = np.zeros(12, np.float32)
        assert lib.da_capi_pose_path(ctx, paths[0], e1.ctypes.data, None) == -1
    finally:
        lib.da_capi_free(ctx)
