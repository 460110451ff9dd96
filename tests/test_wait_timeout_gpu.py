"""The failure path of the bounded waits, on the GPU without any fault: a probe kernel
waits through the same bounded mbarrier wait every pipelined kernel uses, on a barrier
nothing arrives on, with a 1 ms limit. The wait must run out, record the timed-out-wait
status (1), free the tensor memory the probe allocated, and return; the library's
status word must be read and cleared by da3b_device_status; and the next normal
launches must run and give correct results."""
import ctypes

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

V = ctypes.c_void_p
TIMEOUT_FULL = 1  # kStatusTimeoutFull


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _attention_ok(lib):
    """A small normal attention launch against torch fp32 (the context is usable)."""
    g = torch.Generator(device="cuda").manual_seed(11)
    nseq, seqlen, heads = 2, 200, 4
    qkv = (torch.randn(nseq * seqlen, 3 * heads * 64, device="cuda", generator=g)).half()
    out = torch.empty(nseq * seqlen, heads * 64, dtype=torch.float16, device="cuda")
    s = V(torch.cuda.current_stream().cuda_stream)
    assert lib.da3b_attention(V(qkv.data_ptr()), nseq, seqlen, heads, V(out.data_ptr()), s) == 0
    torch.cuda.synchronize()
    q, k, v = qkv.float().view(nseq, seqlen, 3, heads, 64).unbind(2)
    ref = torch.softmax(torch.einsum("sqhd,skhd->shqk", q, k) / 8.0, -1)
    ref = torch.einsum("shqk,skhd->sqhd", ref, v).reshape(nseq * seqlen, heads * 64)
    assert (out.float() - ref).abs().max().item() < 2e-2


@pytest.mark.parametrize("use_tmem", [0, 1])
def test_wait_runs_out_and_kernel_returns(lib, cuda, use_tmem):
    s = V(torch.cuda.current_stream().cuda_stream)
    for _ in range(3):
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        elapsed = torch.zeros(1, dtype=torch.int64, device="cuda")
        assert lib.da3b_debug_wait_timeout(1_000_000, use_tmem, V(status.data_ptr()), V(elapsed.data_ptr()), s) == 0
        torch.cuda.synchronize()
        assert int(status.item()) == TIMEOUT_FULL
        ns = int(elapsed.item())
        assert 1_000_000 <= ns < 500_000_000, ns
    _attention_ok(lib)
    assert lib.da3b_device_status() == 0


def test_library_status_word_read_and_cleared(lib, cuda):
    s = V(torch.cuda.current_stream().cuda_stream)
    assert lib.da3b_device_status() == 0
    assert lib.da3b_debug_wait_timeout(1_000_000, 1, None, None, s) == 0
    assert lib.da3b_device_status() == TIMEOUT_FULL   # synchronises, reads, clears
    assert lib.da3b_device_status() == 0
    _attention_ok(lib)
    assert lib.da3b_device_status() == 0


def test_probe_argument_checks(lib, cuda):
    s = V(torch.cuda.current_stream().cuda_stream)
    assert lib.da3b_debug_wait_timeout(0, 0, None, None, s) == -100
    assert lib.da3b_debug_wait_timeout(2_000_000_000, 0, None, None, s) == -100
