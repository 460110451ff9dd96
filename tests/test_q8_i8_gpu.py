"""The int8 route of the Q8_0 linear (tcgen05.mma kind::i8) against the oracle's
restatement of ggml's CPU Q8_0 x Q8_0 dot product, through the C ABI:
  * activation quantiser: int8 values and f16 block scales bit-exact with ggml's
    reference quantiser (the oracle's, itself pinned to gguf-py's);
  * weight repack of GGUF Q8_0 bytes: exact;
  * the linear: every output bit-exact (the int32 block dots are exact and the f32
    rescale-accumulate runs in block order with explicitly rounded operations), on
    ragged M, several K and N, with and without bias."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

V = ctypes.c_void_p


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _p(t):
    return V(t.data_ptr())


def _stream():
    return V(torch.cuda.current_stream().cuda_stream)


def _gpu_quantize(lib, x):
    M, K = x.shape
    xd = torch.from_numpy(x).cuda()
    q = torch.empty((M, K), dtype=torch.int8, device="cuda")
    d = torch.empty((M, K // 32), dtype=torch.float32, device="cuda")
    assert lib.da3b_quantize_q8_0(_p(xd), M, K, _p(q), _p(d), _stream()) == 0
    return q, d


def _gpu_repack(lib, wq8, N, K):
    raw = torch.from_numpy(np.ascontiguousarray(wq8)).cuda()
    qw = torch.empty((N, K), dtype=torch.int8, device="cuda")
    dwt = torch.empty((K // 32, N), dtype=torch.float32, device="cuda")
    assert lib.da3b_repack_q8_0(_p(raw), N, K, _p(qw), _p(dwt), _stream()) == 0
    return qw, dwt


def test_quantizer_bit_exact(lib, cuda):
    from oracle import oracle as orc

    rng = np.random.default_rng(5)
    x = (rng.standard_normal((300, 1024)) * rng.uniform(0.01, 10, size=(300, 1))).astype(np.float32)
    x[7, 64:96] = 0.0                                    # an all-zero block: d = 0, q = 0
    x[9, :32] = np.arange(32, dtype=np.float32) - 15.5   # halves: ties round away from zero
    q, d = _gpu_quantize(lib, x)
    torch.cuda.synchronize()
    ref = orc.quantize_q8_0(x).reshape(300, 32, 34)
    ref_d = ref[:, :, :2].copy().view(np.float16).reshape(300, 32).astype(np.float32)
    ref_q = ref[:, :, 2:].copy().view(np.int8).reshape(300, 1024)
    assert np.array_equal(q.cpu().numpy(), ref_q)
    assert np.array_equal(d.cpu().numpy(), ref_d)


def test_repack_exact(lib, cuda):
    from oracle import oracle as orc

    rng = np.random.default_rng(6)
    N, K = 256, 384
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    wq8 = orc.quantize_q8_0(w)
    qw, dwt = _gpu_repack(lib, wq8, N, K)
    torch.cuda.synchronize()
    blk = wq8.reshape(N, K // 32, 34)
    assert np.array_equal(qw.cpu().numpy(), blk[:, :, 2:].copy().view(np.int8).reshape(N, K))
    ref_d = blk[:, :, :2].copy().view(np.float16).reshape(N, K // 32).T.astype(np.float32)
    assert np.array_equal(dwt.cpu().numpy(), ref_d)


@pytest.mark.parametrize("M,K,N,with_bias", [(300, 1024, 1152, True), (128, 384, 128, False),
                                             (1370, 4096, 1024, True), (77, 1536, 256, True)])
def test_linear_i8_bit_exact(lib, cuda, M, K, N, with_bias):
    from oracle import oracle as orc

    rng = np.random.default_rng(M + K + N)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32) if with_bias else None
    wq8 = orc.quantize_q8_0(w)
    q, d = _gpu_quantize(lib, x)
    qw, dwt = _gpu_repack(lib, wq8, N, K)
    b = torch.from_numpy(bias).cuda() if with_bias else None
    y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    rc = lib.da3b_linear_q8q8_i8(_p(q), _p(d), M, K, _p(qw), _p(dwt), N, _p(b) if with_bias else None, _p(y), N,
                                 _stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert lib.da3b_device_status() == 0
    ref = orc.linear_q8(x, wq8, N, bias, act_quant=True)
    got = y.cpu().numpy()
    assert np.array_equal(got, ref), f"max |d| {np.abs(got - ref).max()}"


def test_linear_i8_argument_checks(lib, cuda):
    t = torch.zeros(1024, dtype=torch.int8, device="cuda")
    f = torch.zeros(1024, dtype=torch.float32, device="cuda")
    s = _stream()
    assert lib.da3b_linear_q8q8_i8(_p(t), _p(f), 4, 100, _p(t), _p(f), 128, None, _p(f), 128, s) < 0   # K % 128
    assert lib.da3b_linear_q8q8_i8(_p(t), _p(f), 4, 128, _p(t), _p(f), 100, None, _p(f), 100, s) < 0   # N % 128
    assert lib.da3b_quantize_q8_0(_p(f), 4, 33, _p(t), _p(f), s) < 0                                   # K % 32
