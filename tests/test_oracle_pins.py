"""Pins of the CPU oracle (CPU only).

* Preprocessing and the UV embedding against DA3cpplib's own src/preprocess.cpp and
  src/uv_posembed.cpp: bit-exact against the committed fixtures generated from
  oracle/_ref (tests/golden/make_golden.py), and against oracle/_ref live on seeded
  random cases when that library is present.
* The Q8_0 quantiser against gguf-py's (bit-exact with ggml's C reference quantiser).
* The whole DA2 path (patch embed, offset pos-embed interpolation, ViT blocks, attention,
  out-layer LayerNorm, DPT head, ReLU) against transformers' DepthAnythingForDepthEstimation
  with the same f32 weights: |diff| <= 1e-4 * max|ref| (f32 summation-order noise).
"""
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")


@pytest.fixture(scope="module")
def orc():
    from oracle import oracle

    return oracle


@pytest.fixture(scope="module")
def pre():
    return np.load(os.path.join(GOLD, "preprocess_ref.npz"))


def _cases(z, prefix):
    return sorted({k.split("_")[0] for k in z.files if k.startswith(prefix)})


def test_preprocess_matches_reference_fixture(orc, pre):
    cases = _cases(pre, "pre")
    assert len(cases) >= 8
    for c in cases:
        patch, target, upper, legacy = (int(v) for v in pre[c + "_cfg"])
        got = orc.preprocess_cfg(pre[c + "_in"], patch, target, bool(upper), bool(legacy))
        ref = pre[c + "_out"]
        assert got.shape == ref.shape, c
        np.testing.assert_array_equal(got, ref, err_msg=c)


def test_resize_matches_reference_fixture(orc, pre):
    for c in _cases(pre, "rs"):
        dw, dh, mode = (int(v) for v in pre[c + "_cfg"])
        got = orc.resize_u8(pre[c + "_in"], dw, dh, "cubic" if mode == 0 else "area")
        np.testing.assert_array_equal(got, pre[c + "_out"], err_msg=c)


def test_uv_pos_embed_matches_reference_fixture(orc, pre):
    for c in _cases(pre, "uv"):
        pw, ph, C, aspect = pre[c + "_cfg"]
        got = orc.uv_pos_embed(int(pw), int(ph), int(C), float(aspect))
        np.testing.assert_allclose(got, pre[c + "_out"], rtol=0, atol=1e-7, err_msg=c)


def test_preprocess_matches_reference_live(orc):
    """Seeded random sizes and policies, oracle vs. the reference's compiled
    preprocess.cpp (oracle/_ref), bit-exact."""
    if orc.ref_lib() is None:
        pytest.skip("oracle/_ref not available (no DA3cpplib checkout and no prebuilt library)")
    rng = np.random.default_rng(7)
    for i in range(40):
        h, w = (int(v) for v in rng.integers(1, 160, size=2))
        target = int(rng.choice([14, 28, 56, 98, 140, 518]))
        upper, legacy = bool(rng.integers(0, 2)), bool(i % 7 == 0)
        img = rng.integers(0, 256, size=(h, w, 3), dtype=np.uint8)
        a = orc.preprocess_cfg(img, 14, target, upper, legacy)
        b = orc.preprocess_cfg(img, 14, target, upper, legacy, impl="ref")
        np.testing.assert_array_equal(a, b, err_msg=f"{h}x{w} target {target} upper {upper} legacy {legacy}")
    for i in range(20):
        h, w, dh, dw = (int(v) for v in rng.integers(1, 90, size=4))
        img = rng.integers(0, 256, size=(h, w, 3), dtype=np.uint8)
        for mode in ("cubic", "area"):
            np.testing.assert_array_equal(orc.resize_u8(img, dw, dh, mode), orc.resize_u8(img, dw, dh, mode, "ref"))


def test_q8_0_matches_ggufpy(orc):
    z = np.load(os.path.join(GOLD, "q8_0_ggufpy.npz"))
    got = orc.quantize_q8_0(z["x"])
    np.testing.assert_array_equal(got, z["q"])


def test_q8_0_matches_ggufpy_live(orc):
    gguf = pytest.importorskip("gguf")
    from gguf import quants

    rng = np.random.default_rng(11)
    x = (rng.standard_normal((16, 512)) * rng.uniform(1e-3, 50, size=(16, 1))).astype(np.float32)
    ref = np.ascontiguousarray(quants.quantize(x, gguf.GGMLQuantizationType.Q8_0)).reshape(-1)
    np.testing.assert_array_equal(orc.quantize_q8_0(x), ref)


@pytest.mark.parametrize("tag", ["sq", "rect"])
def test_da2_matches_transformers(orc, tag):
    z = np.load(os.path.join(GOLD, "da2_hf_tiny.npz"))
    o = orc.Oracle(os.path.join(GOLD, "da2_hf_tiny.gguf"), act_quant=False, n_threads=4)
    r = o.infer(z[tag + "_img"], legacy=True)
    for i in range(4):
        ref = z[f"{tag}_feat{i}"]
        got = o.get(f"feat{i}").reshape(ref.shape)
        assert np.abs(got - ref).max() <= 1e-4 * np.abs(ref).max(), f"feature {i}"
    ref = z[tag + "_logits"]
    assert r["logits"].shape == (1,) + ref.shape
    assert np.abs(r["logits"][0] - ref).max() <= 1e-4 * np.abs(ref).max()
    ref = z[tag + "_depth"]
    assert np.abs(r["depth"] - ref).max() <= 1e-4 * np.abs(ref).max()
    assert (ref > 0).mean() > 0.3  # a live (not all-ReLU-zero) output


def test_sky_head_is_the_out2_stack(orc):
    """The sky head (src/dpt_head.cpp:205-222) is conv3x3 -> relu -> conv1x1 on the same
    feature map as output_conv2, followed by relu (src/dpt_head.cpp:334-338): with the
    sky and out2 weights swapped, the oracle's sky equals relu(main logits) of the swap,
    tying the sky head to the output_conv2 code that the transformers pin covers."""
    from da3cpplib_b200 import synth

    path = synth.ensure_gguf("da3m-t", stress=True)
    img = synth.image(synth.IMAGE_SEED, 43, 126, 112)
    a = orc.Oracle(path, act_quant=False).infer(img)
    swap = {f"head.scratch.out2{x}.{k}": f"head.scratch.sky_out2{x}.{k}" for x in "ab" for k in ("weight", "bias")}
    b = orc.Oracle(path, act_quant=False, swap=swap).infer(img)
    np.testing.assert_array_equal(a["sky"], np.maximum(b["logits"][0], 0))
    np.testing.assert_array_equal(b["sky"], np.maximum(a["logits"][0], 0))
    assert 0.2 < (a["sky"] < 0.3).mean() < 0.9  # both sides of the sky threshold occur


def test_metric_branch_layout_oracle(orc):
    """m_vit.* / m_head.* files read like the plain layout (src/model_loader.cpp:84-154)."""
    from da3cpplib_b200 import synth

    img = synth.image(synth.IMAGE_SEED, 44, 112, 112)
    a = orc.Oracle(synth.ensure_gguf("da3m-t", stress=True)).infer(img)
    b = orc.Oracle(synth.ensure_gguf("da3m-t", stress=True, metric_branch=True)).infer(img)
    np.testing.assert_array_equal(a["depth"], b["depth"])
    np.testing.assert_array_equal(a["sky"], b["sky"])
    assert "conf" not in a


# ---------------------------------------------------------------- DA3 backbone host code
def _da3_host():
    import sys

    if GOLD not in sys.path:
        sys.path.insert(0, GOLD)
    import make_golden

    return make_golden


def test_da3_host_code_matches_reference_fixture(orc):
    """The oracle's RoPE tables, offset bicubic pos-embed interpolation and saddle
    reference-view choice against DA3cpplib's own src/rope2d.cpp and
    src/dino_backbone.cpp (compiled unmodified into oracle/_ref; committed outputs):
    bit-exact, including the full-size C3/C4 tables (by SHA-256 of their bytes)."""
    mg = _da3_host()
    z = np.load(os.path.join(GOLD, "da3_host_ref.npz"))
    rope, interp, saddle = mg.da3_host_cases()
    for name, pos, hd, freq, full in rope:
        c, s = orc.rope_tables(pos, hd, freq)
        if full:
            np.testing.assert_array_equal(c, z[name + "_cos"], err_msg=name)
            np.testing.assert_array_equal(s, z[name + "_sin"], err_msg=name)
        else:
            assert [mg.sha(c), mg.sha(s)] == list(z[name + "_sha"]), name
    for name, pe, grid, gh, gw, off, full in interp:
        r = orc.interp_pos_embed(pe, grid, gh, gw, off)
        if full:
            np.testing.assert_array_equal(r, z[name + "_out"], err_msg=name)
        else:
            assert mg.sha(r) == z[name + "_sha"][0], name
    for name, cls in saddle:
        assert orc.select_saddle(cls) == int(z[name + "_idx"]), name


def test_da3_host_code_matches_reference_live(orc):
    """The same three functions against oracle/_ref on fresh seeded cases (skipped where
    the reference library is not available)."""
    if orc.ref_lib() is None:
        pytest.skip("oracle/_ref not available")
    rng = np.random.default_rng(77)
    for _ in range(20):
        T = int(rng.integers(1, 300))
        pos = rng.uniform(0, 80, size=(T, 2)).astype(np.float32)
        a, b = orc.rope_tables(pos), orc.rope_tables(pos, impl="ref")
        np.testing.assert_array_equal(a[0], b[0])
        np.testing.assert_array_equal(a[1], b[1])
        grid = int(rng.integers(2, 40))
        gh, gw = int(rng.integers(1, 45)), int(rng.integers(1, 45))
        pe = rng.standard_normal((1 + grid * grid, 8)).astype(np.float32)
        off = float(rng.choice([0.0, 0.1]))
        np.testing.assert_array_equal(orc.interp_pos_embed(pe, grid, gh, gw, off),
                                      orc.interp_pos_embed(pe, grid, gh, gw, off, impl="ref"))
        S = int(rng.integers(2, 9))
        cls = rng.standard_normal((S, 64)).astype(np.float32) * rng.uniform(0.1, 3.0, size=(S, 1)).astype(np.float32)
        assert orc.select_saddle(cls) == orc.select_saddle(cls, impl="ref")
