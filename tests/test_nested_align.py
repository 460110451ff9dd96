"""Nested metric alignment (NestedAligner, src/nested.cpp:7-96) on the host.

Three implementations on the same inputs, all bit-exact:
  * the reference's own src/nested.cpp, compiled unmodified into oracle/_ref;
  * the oracle's restatement (full-sort torch.quantile);
  * libda3b's da3b_nested_align (selection-based quantile), the function the nested
    depth path runs after its two GPU branches.
The reference's own test (tests/test_nested_align.cpp) reads a model dump that is not
part of the checkout, so the compiled reference is the pin. Cases cover the edge cases
the alignment has: at most 10 sky / non-sky pixels (the sky fill is skipped), ties at
the median confidence, depths under both validity thresholds, an empty least-squares
mask (den clamped), the 200 m cap on the sky fill, and n = 1.
"""
import numpy as np
import pytest

from oracle import oracle as O


def _case(seed, n, sky_frac=0.3, scale=1.0, conf_levels=None, low_depth=0.0):
    rng = np.random.default_rng(seed)
    ad = rng.uniform(0.0, 5.0, n).astype(np.float32) * np.float32(scale)
    if low_depth:
        ad[rng.random(n) < low_depth] = np.float32(5e-4)
    ac = rng.uniform(1.0, 3.0, n).astype(np.float32)
    if conf_levels:
        ac = rng.choice(np.array(conf_levels, np.float32), n)
    ext = rng.standard_normal(12).astype(np.float32)
    intr = np.array([rng.uniform(100, 400), 0, 56, 0, rng.uniform(100, 400), 56, 0, 0, 1], np.float32)
    md = rng.uniform(0.0, 10.0, n).astype(np.float32) * np.float32(scale)
    sky = np.where(rng.random(n) < sky_frac, rng.uniform(0.3, 1.0, n), rng.uniform(0.0, 0.3, n)).astype(np.float32)
    return ad, ac, ext, intr, md, sky


CASES = {
    "plain": dict(seed=1, n=4096),
    "hd": dict(seed=2, n=504 * 378),
    "few_sky": dict(seed=3, n=2000, sky_frac=0.004),
    "all_sky": dict(seed=4, n=500, sky_frac=1.0),
    "no_sky": dict(seed=5, n=500, sky_frac=0.0),
    "conf_ties": dict(seed=6, n=3000, conf_levels=[1.0, 2.0, 2.0, 3.0]),
    "low_depth": dict(seed=7, n=3000, low_depth=0.5),
    "cap200": dict(seed=8, n=3000, scale=300.0),
    "single": dict(seed=9, n=1),
    "tiny": dict(seed=10, n=23, sky_frac=0.5),
}


def _ours(ad, ac, ext, intr, md, sky):
    from da3cpplib_b200 import _lib

    L = _lib.load()
    a = [np.ascontiguousarray(x, dtype=np.float32) for x in (ad, ac, ext, intr, md.copy(), sky)]
    out = np.zeros(ad.size, np.float32)
    e = np.zeros(12, np.float32)
    s = L.da3b_nested_align(*[x.ctypes.data for x in a], ad.size, out.ctypes.data, e.ctypes.data)
    return out, e, float(s)


@pytest.mark.parametrize("name", sorted(CASES))
def test_nested_align_bit_exact(name):
    if O.ref_lib() is None:
        pytest.skip("oracle/_ref (the reference's nested.cpp) is not built")
    args = _case(**CASES[name])
    ref = O.nested_align(*args, impl="ref")
    ora = O.nested_align(*args, impl="oracle")
    ours = _ours(*args)
    for got in (ora, ours):
        assert got[2] == ref[2]
        assert np.array_equal(got[0], ref[0])
        assert np.array_equal(got[1], ref[1])


def test_nested_align_empty_mask():
    """All pixels invalid for the least-squares fit: den is clamped, scale 0, every
    depth and the translation go to 0 and sky pixels to the (zero) fill value."""
    args = list(_case(seed=11, n=1000, sky_frac=0.2))
    args[0] = np.full(1000, 1e-4, np.float32)  # anyview depth under 1e-3 everywhere
    ours = _ours(*args)
    assert ours[2] == 0.0
    assert not ours[0].any()
    if O.ref_lib() is not None:
        ref = O.nested_align(*args, impl="ref")
        assert ref[2] == ours[2] and np.array_equal(ref[0], ours[0])


def test_nested_align_committed_outputs():
    """The reference's outputs committed in tests/golden/nested_ref.npz (made from
    oracle/_ref by tests/golden/make_golden.py) hold without the reference checkout."""
    import os

    from golden.make_golden import NESTED_CASES, nested_inputs

    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "nested_ref.npz"))
    for seed, n, frac in NESTED_CASES:
        args = nested_inputs(seed, n, frac)
        for got in (O.nested_align(*args, impl="oracle"), _ours(*args)):
            assert np.array_equal(got[0], z[f"s{seed}_depth"])
            assert np.array_equal(got[1], z[f"s{seed}_ext"])
            assert np.float32(got[2]) == z[f"s{seed}_scale"]
