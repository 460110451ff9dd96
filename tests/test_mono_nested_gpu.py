"""DA3 mono (depth + sky, Engine::depth_mono at src/engine.cpp:105-115) and the nested
metric path (Engine::depth_metric at src/engine.cpp:416-451) on the GPU, through the
C ABI, against the CPU oracle.

Bounds (as in test_e2e_gpu): median relative error over pixels with |ref| > 1e-6 <=
max(1e-2, 1.5 * floor) for depth, floor being the same metric between the oracle with
and without ggml's activation quantisation. The sky plane is relu(logits): its values
are compared where the oracle's sky exceeds 0.05 (same bound) and its sky / non-sky
split at 0.3 must agree on >= 99% of the pixels whose oracle sky is more than 0.05 away
from 0.3.

The nested path is checked twice: bit-exactly as the composition of its parts (the
anyview and metric branches run as stand-alone models on the same prepared input,
then da3b_nested_align), and end to end against the oracle's two branches plus the
reference's own alignment, with the scale factor within max(2e-2, 2 * floor) and the
aligned depth within that bound on pixels both sides classify the same way.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def median_rel(a, b, eps=1e-6):
    m = np.abs(b) > eps
    if not m.any():
        return 0.0
    return float(np.median(np.abs(a[m] - b[m]) / np.abs(b[m])))


def _sky_checks(sky, ref_sky, floor):
    m = ref_sky > 0.05
    assert m.sum() > 100
    err = float(np.median(np.abs(sky[m] - ref_sky[m]) / ref_sky[m]))
    assert err <= max(1e-2, 1.5 * floor), (err, floor)
    far = np.abs(ref_sky - 0.3) > 0.05
    agree = float(((sky < 0.3) == (ref_sky < 0.3))[far].mean())
    assert agree >= 0.99, agree


def _ppm(tmp_path, name, img):
    h, w = img.shape[:2]
    f = tmp_path / name
    f.write_bytes(f"P6\n{w} {h}\n255\n".encode() + img.tobytes())
    return str(f).encode()


@pytest.mark.parametrize("size", [(112, 112), (150, 131)])
def test_mono_depth_and_sky(cuda, size):
    """Model.infer at the processed size and da_capi_depth_dense (preprocess_real on the
    GPU for the unaligned size) against the oracle."""
    from da3cpplib_b200 import Model, synth
    from oracle.oracle import Oracle

    path = synth.ensure_gguf("da3m-t", stress=True)
    h, w = size
    img = synth.image(synth.IMAGE_SEED, 40, h, w)
    oq, of = Oracle(path, act_quant=True), Oracle(path, act_quant=False)
    rq, rf = oq.infer(img), of.infer(img)
    H, W = rq["H"], rq["W"]
    assert "conf" not in rq and rq["sky"].shape == (H, W)
    floor_d = median_rel(rf["depth"], rq["depth"])
    m = rf["sky"] > 0.05
    floor_s = float(np.median(np.abs(rf["sky"][m] - rq["sky"][m]) / np.maximum(rq["sky"][m], 1e-6)))
    m_gpu = Model(path, 0)
    assert m_gpu.has_sky and m_gpu.output_dim == 1 and not m_gpu.has_camera
    if (h, w) == (H, W):
        out = m_gpu.infer(img)
        assert "conf" not in out
        assert median_rel(out["depth"][0], rq["depth"]) <= max(1e-2, 1.5 * floor_d)
        _sky_checks(out["sky"][0], rq["sky"], floor_s)
    m_gpu.close()
    from da3cpplib_b200 import _lib

    lib = _lib.load()
    ctx = lib.da_capi_load(path.encode(), 1)
    assert ctx
    try:
        import tempfile, pathlib

        with tempfile.TemporaryDirectory() as d:
            f = _ppm(pathlib.Path(d), "m.ppm", img)
            oh, ow, met = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
            pd, pc, ps = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
            ext = np.ones(12, np.float32)
            intr = np.ones(9, np.float32)
            rc = lib.da_capi_depth_dense(ctx, f, ctypes.byref(oh), ctypes.byref(ow), ctypes.byref(pd),
                                         ctypes.byref(pc), ctypes.byref(ps), ext.ctypes.data, intr.ctypes.data,
                                         ctypes.byref(met))
            assert rc == 0, lib.da_capi_last_error(ctx)
            assert (oh.value, ow.value) == (H, W)
            assert not pc.value and pd.value and ps.value
            assert met.value == 1  # "mono" checkpoint name (src/da_capi.cpp:41-52)
            assert not ext.any() and not intr.any()
            d = np.ctypeslib.as_array(ctypes.cast(pd, ctypes.POINTER(ctypes.c_float)), (H * W,)).copy()
            s = np.ctypeslib.as_array(ctypes.cast(ps, ctypes.POINTER(ctypes.c_float)), (H * W,)).copy()
            lib.da_capi_free_floats(pd)
            lib.da_capi_free_floats(ps)
            assert median_rel(d.reshape(H, W), rq["depth"]) <= max(1e-2, 1.5 * floor_d)
            _sky_checks(s.reshape(H, W), rq["sky"], floor_s)
    finally:
        lib.da_capi_free(ctx)


def test_metric_branch_layout_is_the_same_model(cuda):
    """A metric-branch GGUF (m_vit.* / m_head.* keys and tensors) loads as the same model
    as the plain layout with the same weights: identical outputs."""
    from da3cpplib_b200 import Model, synth

    img = synth.image(synth.IMAGE_SEED, 41, 112, 112)
    a = Model(synth.ensure_gguf("da3m-t", stress=True), 0).infer(img)
    b = Model(synth.ensure_gguf("da3m-t", stress=True, metric_branch=True), 0).infer(img)
    assert np.array_equal(a["depth"], b["depth"]) and np.array_equal(a["sky"], b["sky"])


def _nested_dense(lib, ctx, f):
    oh, ow, met = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    pd, pc, ps = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
    ext = np.zeros(12, np.float32)
    intr = np.zeros(9, np.float32)
    rc = lib.da_capi_depth_dense(ctx, f, ctypes.byref(oh), ctypes.byref(ow), ctypes.byref(pd), ctypes.byref(pc),
                                 ctypes.byref(ps), ext.ctypes.data, intr.ctypes.data, ctypes.byref(met))
    assert rc == 0, lib.da_capi_last_error(ctx)
    assert not pc.value and not ps.value and met.value == 1
    H, W = oh.value, ow.value
    d = np.ctypeslib.as_array(ctypes.cast(pd, ctypes.POINTER(ctypes.c_float)), (H * W,)).copy().reshape(H, W)
    lib.da_capi_free_floats(pd)
    return d, ext, intr


def test_nested_metric(cuda, tmp_path):
    from da3cpplib_b200 import Model, _lib, synth
    from oracle import oracle as O

    lib = _lib.load()
    anyv = synth.ensure_gguf("da3-t", stress=True)
    metric = synth.ensure_gguf("da3m-t", stress=True, metric_branch=True)
    img = synth.image(synth.IMAGE_SEED, 42, 130, 121)  # legacy floor-to-patch resize to 126 x 112
    f = _ppm(tmp_path, "n.ppm", img)
    # a metric model without a sky head is refused
    assert not lib.da_capi_load_nested(anyv.encode(), anyv.encode(), 1)
    ctx = lib.da_capi_load_nested(anyv.encode(), metric.encode(), 1)
    assert ctx
    try:
        depth, ext, intr = _nested_dense(lib, ctx, f)
        depth2, _, _ = _nested_dense(lib, ctx, f)  # second call replays the captured graphs
        assert np.array_equal(depth, depth2)
        H, W = depth.shape
        assert (H, W) == (126, 112)
        # depth_path and pose_path of a nested context are the same computation
        oh, ow = ctypes.c_int(), ctypes.c_int()
        p = lib.da_capi_depth_path(ctx, f, ctypes.byref(oh), ctypes.byref(ow))
        assert p
        dp = np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(ctypes.c_float)), (H * W,)).copy()
        lib.da_capi_free_floats(p)
        assert np.array_equal(dp.reshape(H, W), depth)
        e2, k2 = np.zeros(12, np.float32), np.zeros(9, np.float32)
        assert lib.da_capi_pose_path(ctx, f, e2.ctypes.data, k2.ctypes.data) == 0
        assert np.array_equal(e2, ext) and np.array_equal(k2, intr)
    finally:
        lib.da_capi_free(ctx)

    # composition, bit-exact: both branches stand-alone on the same prepared input
    chw = O.preprocess_cfg(img, patch=14, target=112, upper=True, legacy=True)
    ma = Model(anyv, 0)
    oa = ma.infer_prepared(chw)
    _, ext_a, intr_a = ma.pose(1)
    mm = Model(metric, 0)
    om = mm.infer_prepared(chw)
    comp, comp_ext, scale = O.nested_align(oa["depth"][0], oa["conf"][0], ext_a.reshape(12), intr_a.reshape(9),
                                           om["depth"][0], om["sky"][0], impl="oracle")
    ours = np.zeros(H * W, np.float32)
    oext = np.zeros(12, np.float32)
    md = np.ascontiguousarray(om["depth"][0]).copy()
    s2 = lib.da3b_nested_align(oa["depth"][0].ctypes.data, oa["conf"][0].ctypes.data,
                               np.ascontiguousarray(ext_a.reshape(12)).ctypes.data,
                               np.ascontiguousarray(intr_a.reshape(9)).ctypes.data, md.ctypes.data,
                               np.ascontiguousarray(om["sky"][0]).ctypes.data, H * W, ours.ctypes.data,
                               oext.ctypes.data)
    assert s2 == scale and np.array_equal(ours, comp)
    assert np.array_equal(comp.reshape(H, W), depth) and np.array_equal(comp_ext, ext)
    assert np.array_equal(intr_a.reshape(9), intr)

    # end to end against the oracle branches + the alignment
    def oracle_nested(aq):
        ra = O.Oracle(anyv, act_quant=aq).infer_chw(chw)
        rm = O.Oracle(metric, act_quant=aq).infer_chw(chw)
        pose = ra["pose"]
        d, e, s = O.nested_align(ra["depth"], ra["conf"], pose[9:21], pose[21:30], rm["depth"], rm["sky"])
        return d.reshape(H, W), e, s, rm["sky"]

    dq, eq, sq, skyq = oracle_nested(True)
    df, ef, sf, _ = oracle_nested(False)
    floor_s = abs(sf / sq - 1)
    assert abs(scale / sq - 1) <= max(2e-2, 2 * floor_s), (scale, sq, sf)
    same = (om["sky"][0] < 0.3) == (skyq < 0.3)
    nonsky = same & (skyq < 0.25)
    floor_d = median_rel(df[nonsky], dq[nonsky])
    assert median_rel(depth[nonsky], dq[nonsky]) <= max(2e-2, 2 * floor_d)
    assert np.abs(ext[[3, 7, 11]] - eq[[3, 7, 11]]).max() <= max(2e-2, 2 * floor_s) * max(1.0, np.abs(eq).max()) * 4
