"""da3b_attention_noalloc (fixed static V^T scratch, caller-owned status word) against
da3b_attention on the same inputs: bit-identical outputs on two calls in a row with
different shapes, a call at the scratch's capacity, and a rejected oversize call that
launches nothing. Collected last (file name) so that it also runs after every other
GPU test in the same process; it passes alone as well."""
import ctypes

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

V = ctypes.c_void_p
VT_BYTES = 32 << 20          # DA3B_NOALLOC_VT_BYTES
ERR_TOO_LARGE = -103         # DA3B_ERR_NOALLOC_TOO_LARGE


def ptr(t):
    return V(t.data_ptr())


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _qkv(nseq, seqlen, heads, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(nseq * seqlen, 3 * heads * 64, device="cuda", generator=g) * 1.5).half()


def _both(lib, qkv, nseq, seqlen, heads, status):
    s = V(torch.cuda.current_stream().cuda_stream)
    D = heads * 64
    ref = torch.empty(nseq * seqlen, D, dtype=torch.float16, device="cuda")
    got = torch.full_like(ref, float("nan"))
    assert lib.da3b_attention(ptr(qkv), nseq, seqlen, heads, ptr(ref), s) == 0
    assert lib.da3b_attention_noalloc(ptr(qkv), nseq, seqlen, heads, ptr(got), ptr(status), s) == 0
    return ref, got


def test_noalloc_matches_two_calls_in_a_row(lib, cuda):
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    # first call, then a second one with other inputs and a shape whose V^T rows are
    # laid out differently in the same scratch
    for nseq, seqlen, heads, seed in ((3, 1370, 6, 1), (2, 200, 16, 2)):
        qkv = _qkv(nseq, seqlen, heads, seed)
        ref, got = _both(lib, qkv, nseq, seqlen, heads, status)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), f"noalloc differs at nseq={nseq} seqlen={seqlen} heads={heads}"
    assert int(status.item()) == 0
    assert lib.da3b_device_status() == 0


def test_noalloc_at_capacity_and_oversize_rejected(lib, cuda):
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    heads, seqlen = 16, 1370
    per_seq = heads * 64 * ((seqlen + 7) // 8 * 8) * 2
    nmax = VT_BYTES // per_seq
    assert nmax == 11
    qkv = _qkv(nmax, seqlen, heads, 3)
    ref, got = _both(lib, qkv, nmax, seqlen, heads, status)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    # one sequence more needs more than the fixed scratch: rejected, nothing launched
    big = _qkv(nmax + 1, seqlen, heads, 4)
    out = torch.full((big.shape[0], heads * 64), 7.0, dtype=torch.float16, device="cuda")
    s = V(torch.cuda.current_stream().cuda_stream)
    assert lib.da3b_attention_noalloc(ptr(big), nmax + 1, seqlen, heads, ptr(out), ptr(status), s) == ERR_TOO_LARGE
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())
    assert int(status.item()) == 0


def test_noalloc_argument_checks(lib, cuda):
    s = V(torch.cuda.current_stream().cuda_stream)
    qkv = _qkv(1, 16, 1, 5)
    out = torch.empty(16, 64, dtype=torch.float16, device="cuda")
    assert lib.da3b_attention_noalloc(ptr(qkv), 1, 16, 1, ptr(out), None, s) == -100   # no status word
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert lib.da3b_attention_noalloc(ptr(qkv), 0, 16, 1, ptr(out), ptr(status), s) == 0  # empty: no-op


def test_noalloc_allocates_nothing(lib, cuda):
    """After one warm-up call (which loads the kernels and resolves the scratch's
    address), a larger call that the allocating entry point has never run leaves the
    device's free memory unchanged: the no-alloc path takes no device memory."""
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = V(torch.cuda.current_stream().cuda_stream)
    small = _qkv(1, 300, 4, 6)
    out_small = torch.empty(300, 4 * 64, dtype=torch.float16, device="cuda")
    big_seq, big_heads = 2900, 16       # 2 * 1024 * 2904 * 2 B of V^T: within the scratch
    big = _qkv(2, big_seq, big_heads, 7)
    out_big = torch.empty(2 * big_seq, big_heads * 64, dtype=torch.float16, device="cuda")
    assert lib.da3b_attention_noalloc(ptr(small), 1, 300, 4, ptr(out_small), ptr(status), s) == 0
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    assert lib.da3b_attention_noalloc(ptr(big), 2, big_seq, big_heads, ptr(out_big), ptr(status), s) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"free device memory changed by {free0 - free1} bytes"
    assert int(status.item()) == 0
    # and the result is the allocating entry point's
    ref = torch.empty_like(out_big)
    assert lib.da3b_attention(ptr(big), 2, big_seq, big_heads, ptr(ref), s) == 0
    torch.cuda.synchronize()
    assert torch.equal(out_big, ref)
