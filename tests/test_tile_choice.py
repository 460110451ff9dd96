"""The automatic tile choice of the tcgen05 GEMM (host code, no GPU work): the linears
of one ViT-B image (M = 1370) on the one-CTA kernel with the widths and K splits the
B200 measurements favoured, one image's stride-2 DPT conv as a GEMM on a 4-CTA K split,
and the batched C3 shapes on CTA pairs."""
import ctypes

import pytest

from da3cpplib_b200 import _lib


@pytest.fixture(scope="module")
def lib():
    try:
        return _lib.load()
    except OSError as e:  # the library is built by __graft_entry__.build()
        pytest.skip(str(e))


def _tiles(lib, M, N, K):
    bn, ks = ctypes.c_int(0), ctypes.c_int(0)
    rc = lib.da3b_linear_tiles(M, N, K, ctypes.byref(bn), ctypes.byref(ks))
    return rc, bn.value, ks.value


@pytest.mark.parametrize("M,N,K,want", [
    (1370, 2304, 768, (1, 256, 1)),   # ViT-B QKV, one image: 99 tiles in one wave
    (1370, 3072, 768, (1, 256, 1)),   # ViT-B fc1
    (1370, 768, 768, (1, 64, 1)),     # ViT-B attn proj
    (1370, 768, 3072, (1, 128, 2)),   # ViT-B fc2: 66 tiles, K split over 2-CTA clusters
    (1370, 1024, 4096, (1, 128, 1)),  # ViT-L fc2, one image
    (361, 768, 6912, (1, 64, 4)),     # one image's stride-2 DPT conv (im2col GEMM)
    (87680, 4096, 1024, (0, 256, 1)),  # C3 fc1: CTA pairs
    (87680, 1024, 4096, (0, 256, 1)),  # C3 fc2
])
def test_linear_tiles(lib, M, N, K, want):
    assert _tiles(lib, M, N, K) == want


def test_linear_tiles_rejects_bad_arguments(lib):
    assert _tiles(lib, 0, 64, 64)[0] < 0
    assert lib.da3b_linear_tiles(16, 64, 64, None, None) < 0
