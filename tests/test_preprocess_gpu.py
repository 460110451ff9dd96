"""GPU preprocessing through the C ABI.

* da3b_resize_u8 against the CPU oracle's uint8 resizers (which are bit-exact with
  DA3cpplib's own src/preprocess.cpp): bit-exact, cubic and area, one or two images,
  odd sizes, and area's bilinear fallback when both axes grow.
* The preprocess_real chain (bound resize, then patch rounding) composed from it,
  normalised: bit-exact against the oracle's preprocess.
* da3b_patchify against numpy's f32 normalisation rounded to f16: bit-exact, including
  widths whose rows start unaligned and strips with fewer than 16 patches.
* da3b_infer_prepared (normalised planar f32 input, the reference's infer_preprocessed
  path) gives depth and confidence bit-identical to the RGB8 path on the same images.
* A model-level run on an image that needs resizing (da_capi_depth_path on a PPM file):
  the GPU resizes it, and the depth matches the oracle's: median relative error over
  pixels with |ref| > 1e-6 <= max(1e-2, 1.5 * floor), floor being the same error between
  the oracle with and without ggml's activation quantisation on this input (DA2's ReLU
  leaves few non-zero pixels on a random model), and the zero pattern agrees on >= 99%.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

V = ctypes.c_void_p
MEAN = (0.485, 0.456, 0.406)
STD = (0.229, 0.224, 0.225)


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _stream():
    return V(torch.cuda.current_stream().cuda_stream)


def _gpu_resize(lib, imgs, dw, dh, mode):
    src = torch.from_numpy(np.ascontiguousarray(imgs)).cuda()
    B, sh, sw, _ = imgs.shape
    dst = torch.empty((B, dh, dw, 3), dtype=torch.uint8, device="cuda")
    assert lib.da3b_resize_u8(V(src.data_ptr()), B, sw, sh, V(dst.data_ptr()), dw, dh, mode, _stream()) == 0
    torch.cuda.synchronize()
    assert lib.da3b_device_status() == 0
    return dst.cpu().numpy()


@pytest.mark.parametrize("B,sh,sw,dh,dw,mode", [
    (1, 37, 53, 112, 160, 0), (2, 90, 61, 56, 38, 1), (1, 23, 31, 40, 57, 0), (1, 400, 300, 126, 98, 1),
    (2, 7, 11, 30, 19, 0), (1, 40, 40, 13, 17, 1), (1, 20, 30, 26, 44, 1), (1, 518, 700, 518, 518, 1),
    (1, 97, 150, 112, 173, 0)])
def test_resize_u8_bit_exact(lib, cuda, B, sh, sw, dh, dw, mode):
    from oracle import oracle as orc

    rng = np.random.default_rng(sh * 1000 + sw + mode)
    imgs = rng.integers(0, 256, size=(B, sh, sw, 3), dtype=np.uint8)
    got = _gpu_resize(lib, imgs, dw, dh, mode)
    for b in range(B):
        ref = orc.resize_u8(imgs[b], dw, dh, "cubic" if mode == 0 else "area")
        assert np.array_equal(got[b], ref), f"image {b}: {np.count_nonzero(got[b] != ref)} bytes differ"


def _policy(w, h, patch, target, upper):
    """Step sizes of preprocess_real (src/preprocess.cpp:166-190)."""
    steps = []
    bound = max(w, h) if upper else min(w, h)
    if bound != target:
        scale = target / bound
        nw, nh = max(1, int(round(w * scale))), max(1, int(round(h * scale)))
        steps.append((nw, nh, 0 if scale > 1.0 else 1))
        w, h = nw, nh

    def nearest(x):
        down = (x // patch) * patch
        up = down + patch
        return up if abs(up - x) <= abs(x - down) else down

    nw, nh = max(1, nearest(w)), max(1, nearest(h))
    if (nw, nh) != (w, h):
        steps.append((nw, nh, 0 if (nw > w or nh > h) else 1))
    return steps


@pytest.mark.parametrize("h,w,target,upper", [(37, 53, 56, True), (90, 61, 56, True), (37, 53, 42, False),
                                              (29, 45, 28, True), (15, 100, 84, True), (300, 457, 518, False),
                                              (640, 480, 504, True)])
def test_preprocess_real_chain_bit_exact(lib, cuda, h, w, target, upper):
    from oracle import oracle as orc

    rng = np.random.default_rng(h * 7 + w)
    img = rng.integers(0, 256, size=(1, h, w, 3), dtype=np.uint8)
    cur = img
    for nw, nh, mode in _policy(w, h, 14, target, upper):
        cur = _gpu_resize(lib, cur, nw, nh, mode)
    chw = (cur[0].astype(np.float32) / np.float32(255.0) - np.array(MEAN, np.float32)) / np.array(STD, np.float32)
    ref = orc.preprocess_cfg(img[0], 14, target, upper)
    assert np.array_equal(chw.transpose(2, 0, 1), ref)


@pytest.mark.parametrize("B,H,W", [(2, 518, 518), (1, 56, 70), (3, 42, 238), (1, 504, 504), (2, 14, 14)])
def test_patchify_bit_exact(lib, cuda, B, H, W):
    P, ldk = 14, 640
    rng = np.random.default_rng(H + W)
    img = rng.integers(0, 256, size=(B, H, W, 3), dtype=np.uint8)
    src = torch.from_numpy(img).cuda()
    gh, gw = H // P, W // P
    out = torch.full((B * gh * gw, ldk), 7.0, dtype=torch.float16, device="cuda")
    mean = (ctypes.c_float * 3)(*MEAN)
    std = (ctypes.c_float * 3)(*STD)
    assert lib.da3b_patchify(V(src.data_ptr()), B, H, W, P, mean, std, V(out.data_ptr()), ldk, _stream()) == 0
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    x = (img.astype(np.float32) / np.float32(255.0) - np.array(MEAN, np.float32)) / np.array(STD, np.float32)
    ref = x.reshape(B, gh, P, gw, P, 3).transpose(0, 1, 3, 5, 2, 4).reshape(B * gh * gw, 3 * P * P).astype(np.float16)
    assert np.array_equal(got[:, :3 * P * P].view(np.uint16), ref.view(np.uint16))
    assert np.all(got[:, 3 * P * P:] == 0)


def test_capi_depth_path_resizes_on_gpu(lib, cuda, tmp_path):
    from da3cpplib_b200 import synth
    from oracle.oracle import Oracle

    path = synth.ensure_gguf("da2-t", stress=True)     # lower_bound, target 112
    rng = np.random.default_rng(5)
    img = rng.integers(0, 256, size=(97, 150, 3), dtype=np.uint8)
    ppm = tmp_path / "in.ppm"
    with open(ppm, "wb") as f:
        f.write(b"P6\n150 97\n255\n" + img.tobytes())
    ctx = lib.da_capi_load(path.encode(), 1)
    assert ctx
    try:
        h, w = ctypes.c_int(), ctypes.c_int()
        p = lib.da_capi_depth_path(ctx, str(ppm).encode(), ctypes.byref(h), ctypes.byref(w))
        assert p, lib.da_capi_last_error(ctx)
        got = np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(ctypes.c_float)), shape=(h.value * w.value,)).copy()
        lib.da_capi_free_floats(p)
    finally:
        lib.da_capi_free(ctx)
    ref = Oracle(path, act_quant=True).infer(img)
    reff = Oracle(path, act_quant=False).infer(img)
    assert (h.value, w.value) == (ref["H"], ref["W"]) == (112, 168)

    def median_rel(a, b):
        a, b = a.reshape(-1), b.reshape(-1)
        m = np.abs(b) > 1e-6
        return float(np.median(np.abs(a[m] - b[m]) / np.abs(b[m])))

    floor = median_rel(reff["depth"], ref["depth"])
    err = median_rel(got, ref["depth"])
    assert err <= max(1e-2, 1.5 * floor), (err, floor)
    r = ref["depth"].reshape(-1)
    assert np.mean((np.abs(got) > 1e-6) == (np.abs(r) > 1e-6)) >= 0.99


@pytest.mark.parametrize("name,n", [("da3-t", 2), ("da2-t", 1)])
def test_infer_prepared_matches_rgb_path(cuda, name, n):
    from da3cpplib_b200 import Model, synth

    path = synth.ensure_gguf(name, stress=True)
    m = Model(path, 0)
    imgs = np.stack([synth.image(synth.IMAGE_SEED, i, 112, 112) for i in range(n)])
    ref = m.infer(imgs)
    chw = (imgs.astype(np.float32) / np.float32(255.0) - np.array(MEAN, np.float32)) / np.array(STD, np.float32)
    got = m.infer_prepared(chw.transpose(0, 3, 1, 2))
    got2 = m.infer_prepared(chw.transpose(0, 3, 1, 2))      # second call: the captured graph
    for k in ref:
        assert np.array_equal(got[k], ref[k]), k
        assert np.array_equal(got2[k], ref[k]), k


@pytest.mark.parametrize("B,h,w", [(2, 120, 125), (1, 37, 53), (3, 14, 29), (1, 518, 700)])
def test_legacy_preprocess_bit_exact(lib, cuda, B, h, w):
    """da3b_preprocess_legacy (float bilinear to the floor-to-patch size + normalisation)
    against the oracle's legacy preprocess: bit-exact."""
    from oracle import oracle as orc

    rng = np.random.default_rng(h * 31 + w)
    imgs = rng.integers(0, 256, size=(B, h, w, 3), dtype=np.uint8)
    src = torch.from_numpy(imgs).cuda()
    oh, ow = ctypes.c_int(), ctypes.c_int()
    mean = (ctypes.c_float * 3)(*MEAN)
    std = (ctypes.c_float * 3)(*STD)
    assert lib.da3b_preprocess_legacy(V(src.data_ptr()), B, w, h, 14, mean, std, None, ctypes.byref(oh),
                                      ctypes.byref(ow), _stream()) == 0
    out = torch.empty((B, 3, oh.value, ow.value), dtype=torch.float32, device="cuda")
    assert lib.da3b_preprocess_legacy(V(src.data_ptr()), B, w, h, 14, mean, std, V(out.data_ptr()), ctypes.byref(oh),
                                      ctypes.byref(ow), _stream()) == 0
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for b in range(B):
        ref = orc.preprocess_cfg(imgs[b], 14, 504, True, legacy=True)
        assert got[b].shape == ref.shape and np.array_equal(got[b], ref), b


def test_capi_multiview_legacy_resize(lib, cuda, tmp_path):
    """da_capi_depth_pose_multi on three 125x120 views (legacy resize to 112x112 on the
    GPU): depth and camera poses against the oracle's multi-view run."""
    from da3cpplib_b200 import synth
    from oracle.oracle import Oracle

    path = synth.ensure_gguf("da3-t", stress=True)
    rng = np.random.default_rng(9)
    imgs = [rng.integers(0, 256, size=(120, 125, 3), dtype=np.uint8) for _ in range(3)]
    paths = []
    for i, img in enumerate(imgs):
        f = tmp_path / f"v{i}.ppm"
        f.write_bytes(b"P6\n125 120\n255\n" + img.tobytes())
        paths.append(str(f).encode())
    ctx = lib.da_capi_load(path.encode(), 1)
    assert ctx
    try:
        n, h, w = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        ext = np.zeros((3, 12), np.float32)
        intr = np.zeros((3, 9), np.float32)
        arr = (ctypes.c_char_p * 3)(*paths)
        p = lib.da_capi_depth_pose_multi(ctx, arr, 3, ctypes.byref(h), ctypes.byref(w), ctypes.byref(n),
                                         ext.ctypes.data, intr.ctypes.data)
        assert p, lib.da_capi_last_error(ctx)
        got = np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(ctypes.c_float)), shape=(3 * 112 * 112,)).copy()
        lib.da_capi_free_floats(p)
    finally:
        lib.da_capi_free(ctx)
    assert (h.value, w.value, n.value) == (112, 112, 3)
    rq = Oracle(path, act_quant=True).infer_mv(imgs)
    rf = Oracle(path, act_quant=False).infer_mv(imgs)

    def median_rel(a, b):
        a, b = a.reshape(-1), b.reshape(-1)
        m = np.abs(b) > 1e-6
        return float(np.median(np.abs(a[m] - b[m]) / np.abs(b[m])))

    floor = median_rel(rf["depth"], rq["depth"])
    assert median_rel(got, rq["depth"]) <= max(1e-2, 1.5 * floor)
    pe_floor = float(np.max(np.abs(rf["pose"][:, 9:21] - rq["pose"][:, 9:21]) / np.maximum(1, np.abs(rq["pose"][:, 9:21]))))
    err = float(np.max(np.abs(ext - rq["pose"][:, 9:21]) / np.maximum(1, np.abs(rq["pose"][:, 9:21]))))
    assert err <= max(8e-2, 8 * pe_floor), (err, pe_floor)
