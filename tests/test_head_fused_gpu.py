"""The fused output stage (up_out2: align-corners upsample + UV pos-embed + output_conv2's
3x3 conv + relu + 1x1 conv + activation in one kernel, no full-resolution feature map)
against the unfused path (upsample_ac into a f16 map, then conv_nhwc with the same
fused out2b epilogue), selected with $DA3B_UNFUSED_UP=1 when a plan is created.

Both paths build the same f16 upsampled values; the fused kernel sums the three
horizontal taps of the 3x3 conv in its epilogue (f32) instead of in the tensor-core
accumulator, so the two differ only by f32 summation order: bound max|a - b| <=
1e-4 * max(1, max|b|) on depth, confidence, the mono sky plane and the raw logits, for
widths that are and are not multiples of the 126-pixel strip and for batches of
images. The parity of either path with the CPU oracle is covered by test_e2e_gpu.py /
test_mono_nested_gpu.py.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _run(path, imgs, unfused, raw=False):
    from da3cpplib_b200 import Model

    old = os.environ.get("DA3B_UNFUSED_UP")
    if unfused:
        os.environ["DA3B_UNFUSED_UP"] = "1"
    else:
        os.environ.pop("DA3B_UNFUSED_UP", None)
    try:
        m = Model(path, 0)
        m.set_raw_logits(raw)
        out = m.infer(np.stack(imgs))
        n = m.launches(len(imgs), imgs[0].shape[0], imgs[0].shape[1])
        m.close()
    finally:
        if old is None:
            os.environ.pop("DA3B_UNFUSED_UP", None)
        else:
            os.environ["DA3B_UNFUSED_UP"] = old
    return out, n


CASES = [("da2-t", 112, 112, 2), ("da3-t", 126, 112, 3), ("da3-t", 140, 266, 1), ("da3m-t", 112, 154, 2),
         ("da2-s", 196, 518, 1)]


@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}_{c[1]}x{c[2]}_b{c[3]}" for c in CASES])
def test_fused_matches_unfused(cuda, case):
    from da3cpplib_b200 import synth

    name, h, w, n = case
    path = synth.ensure_gguf(name, stress=True)
    imgs = [synth.image(synth.IMAGE_SEED, 70 + i, h, w) for i in range(n)]
    for raw in (False, True):
        a, la = _run(path, imgs, unfused=False, raw=raw)
        b, lb = _run(path, imgs, unfused=True, raw=raw)
        assert a.keys() == b.keys()
        for k in a:
            err = float(np.abs(a[k] - b[k]).max())
            assert err <= 1e-4 * max(1.0, float(np.abs(b[k]).max())), (k, raw, err)
        assert la == lb - 1  # one launch instead of upsample + conv
