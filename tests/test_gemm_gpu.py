"""tcgen05 GEMM / implicit-GEMM conv engine vs. a plain PyTorch fp32 reference.

Tolerance: |out - ref| <= 2e-3 * max|ref| + 2e-3 (f16 operands are exact in both
paths; the difference is f32 summation order plus the f16 rounding of the output).
"""
import ctypes
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

V = ctypes.c_void_p


def ptr(t):
    return V(t.data_ptr()) if t is not None else None


def stream():
    return V(torch.cuda.current_stream().cuda_stream)


def close(out, ref, rel=2e-3, abs_=2e-3):
    out = out.float()
    ref = ref.float()
    err = (out - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= rel * scale + abs_, f"max err {err} vs scale {scale}"


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield
    torch.cuda.synchronize()


def test_dequant_q8_0_exact(lib):
    rng = np.random.default_rng(1)
    rows, K, ldw = 96, 384, 448
    q = rng.integers(-127, 128, size=(rows, K // 32, 32), dtype=np.int8)
    d = rng.uniform(1e-3, 1e-2, size=(rows, K // 32)).astype(np.float16)
    raw = np.zeros((rows, K // 32, 34), dtype=np.uint8)
    raw[:, :, :2] = d.view(np.uint8).reshape(rows, K // 32, 2)
    raw[:, :, 2:] = q.view(np.uint8)
    q8 = torch.from_numpy(raw.reshape(-1)).cuda()
    w = torch.full((rows, ldw), 7.0, dtype=torch.float16, device="cuda")
    assert lib.da3b_dequant_q8_0(ptr(q8), rows, K, ptr(w), ldw, stream()) == 0
    torch.cuda.synchronize()
    ref = (d.astype(np.float32)[:, :, None] * q.astype(np.float32)).reshape(rows, K).astype(np.float16)
    got = w.cpu().numpy()
    assert np.array_equal(got[:, :K].view(np.uint16), ref.view(np.uint16))
    assert np.all(got[:, K:] == 0)
    assert lib.da3b_device_status() == 0


def _q8_0_raw(rng, N, K, tiny=False):
    """GGUF Q8_0 bytes of an N x K matrix (q in [-128, 127], f16 scales), and the
    reference f16(d * q) as numpy f16. tiny: a third of the scales near the bottom of the
    f16 range, so some products are subnormal."""
    q = rng.integers(-128, 128, size=(N, K // 32, 32), dtype=np.int8)
    d = rng.uniform(1e-3, 1e-2, size=(N, K // 32)).astype(np.float16)
    if tiny:
        d[:, ::3] = rng.uniform(2.0 ** -23, 2.0 ** -14, size=d[:, ::3].shape).astype(np.float16)
    raw = np.zeros((N, K // 32, 34), dtype=np.uint8)
    raw[:, :, :2] = d.view(np.uint8).reshape(N, K // 32, 2)
    raw[:, :, 2:] = q.view(np.uint8)
    ref = (d.astype(np.float32)[:, :, None] * q.astype(np.float32)).reshape(N, K).astype(np.float16)
    return raw.reshape(-1), ref


@pytest.mark.parametrize("N,K", [(96, 384), (64, 96), (2304, 768)])
def test_q8_planar_dequant_exact(lib, N, K):
    """Planar Q8_0 (int8 plane + transposed f16 scale plane, the GGUF bytes): the repack,
    then the staging dequantisation's f16(d * q) (exact int8 -> f16, one f16 multiply)
    against numpy's rounding of the f32 product, subnormal products included, and
    against da3b_dequant_q8_0 on the raw rows."""
    rng = np.random.default_rng(N + K)
    raw, ref = _q8_0_raw(rng, N, K, tiny=True)
    q8 = torch.from_numpy(raw).cuda()
    planar = torch.empty(N * K + (K // 32) * N * 2, dtype=torch.uint8, device="cuda")
    assert lib.da3b_repack_q8_0_planar(ptr(q8), N, K, ptr(planar), stream()) == 0
    w = torch.empty(N, K, dtype=torch.float16, device="cuda")
    assert lib.da3b_dequant_q8p(ptr(planar), N, K, ptr(w), stream()) == 0
    w0 = torch.empty(N, K, dtype=torch.float16, device="cuda")
    assert lib.da3b_dequant_q8_0(ptr(q8), N, K, ptr(w0), K, stream()) == 0
    torch.cuda.synchronize()
    assert lib.da3b_device_status() == 0
    got = w.cpu().numpy()
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))
    assert torch.equal(w, w0)


@pytest.mark.parametrize("M,K,N,kind", [(1370, 768, 2304, "f16"), (1370, 768, 3072, "gelu"), (1370, 768, 768, "resid"),
                                        (1370, 3072, 768, "resid"), (100, 384, 1152, "f16"), (257, 96, 64, "gelu"),
                                        (300, 160, 200, "f16"), (20000, 256, 1024, "f16")])
def test_linear_q8_planar_tiles(lib, M, K, N, kind):
    """The GEMM that dequantises planar Q8_0 weight tiles in shared memory (four converter
    warps write each stage's f16 B tile in the 128B-swizzled layout) against the f16 GEMM
    on the staging dequantisation's weights: bit-identical outputs (same f16 weights, same
    MMA order, same epilogue), with tile widths 64 and 128, a ragged last K block (K = 96,
    160) and ragged N. Declined (returns 1, nothing launched): the CTA-pair regime (M =
    20000), the wide linears the f16 route runs on 256-wide tiles (N >= 2048 at one
    image) and a long reduction it splits over a CTA cluster (fc2: K = 3072), so the two
    routes never sum in different orders."""
    rng = np.random.default_rng(M + K + N)
    raw, _ = _q8_0_raw(rng, N, K)
    q8 = torch.from_numpy(raw).cuda()
    planar = torch.empty(N * K + (K // 32) * N * 2, dtype=torch.uint8, device="cuda")
    assert lib.da3b_repack_q8_0_planar(ptr(q8), N, K, ptr(planar), stream()) == 0
    w = torch.empty(N, K, dtype=torch.float16, device="cuda")
    assert lib.da3b_dequant_q8p(ptr(planar), N, K, ptr(w), stream()) == 0
    g = torch.Generator(device="cuda").manual_seed(M + N)
    x = torch.randn(M, K, device="cuda", generator=g).half()
    b = torch.randn(N, device="cuda", generator=g).float()
    if kind == "resid":
        sc = torch.randn(N, device="cuda", generator=g).float()
        r0 = torch.randn(M, N, device="cuda", generator=g).float()
        ra, rb = r0.clone(), r0.clone()
        rc = lib.da3b_linear_q8p_resid_f32(ptr(x), M, K, K, ptr(planar), N, ptr(b), ptr(sc), ptr(ra), N, stream())
        if K >= 2048:
            assert rc == 1
            return
        assert rc == 0
        assert lib.da3b_linear_resid_f32(ptr(x), M, K, K, ptr(w), N, K, ptr(b), ptr(sc), ptr(rb), N, stream()) == 0
        torch.cuda.synchronize()
        assert lib.da3b_device_status() == 0
        assert torch.equal(ra, rb)
        return
    act = 2 if kind == "gelu" else 0
    oa = torch.full((M, N), 7.0, dtype=torch.float16, device="cuda")
    ob = torch.empty(M, N, dtype=torch.float16, device="cuda")
    rc = lib.da3b_linear_q8p_f16(ptr(x), M, K, K, ptr(planar), N, ptr(b), act, ptr(oa), N, stream())
    if M >= 20000 or N >= 2048:
        assert rc == 1  # CTA pairs; 256-wide tiles on the f16 route
        return
    assert rc == 0
    assert lib.da3b_linear_f16(ptr(x), M, K, K, ptr(w), N, K, ptr(b), act, ptr(ob), N, stream()) == 0
    torch.cuda.synchronize()
    assert lib.da3b_device_status() == 0
    assert torch.equal(oa, ob)
    ref = x.float() @ w.float().t() + b
    if act:
        ref = torch.nn.functional.gelu(ref)
    close(oa, ref)


@pytest.mark.parametrize("M,K,N", [(1, 64, 32), (127, 384, 1152), (128, 128, 64), (300, 200, 48),
                                   (1370, 768, 2304), (2740, 1024, 4096), (1370, 4096, 1024), (257, 640, 96),
                                   (20000, 256, 1000)])
@pytest.mark.parametrize("act", [0, 2, 3])
def test_linear_f16(lib, M, K, N, act):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + K + N)
    lda = (K + 7) // 8 * 8
    x = torch.randn(M, lda, device="cuda", generator=g).half()
    w = (torch.randn(N, lda, device="cuda", generator=g) * 0.05).half()
    b = torch.randn(N, device="cuda", generator=g).float()
    out = torch.empty(M, N, dtype=torch.float16, device="cuda")
    rc = lib.da3b_linear_f16(ptr(x), M, K, lda, ptr(w), N, lda, ptr(b), act, ptr(out), N, stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert lib.da3b_device_status() == 0
    ref = x[:, :K].float() @ w[:, :K].float().t() + b
    if act in (2, 3):
        ref = torch.nn.functional.gelu(ref)  # exact (erf) GELU; 3 uses another erf approximation
    close(out, ref)


@pytest.mark.parametrize("M,K,N", [(1370, 1024, 1024), (100, 384, 384), (4111, 4096, 1024)])
def test_linear_resid(lib, M, K, N):
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(M, K, device="cuda", generator=g).half()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).half()
    b = torch.randn(N, device="cuda", generator=g).float()
    s = torch.randn(N, device="cuda", generator=g).float()
    r0 = torch.randn(M, N, device="cuda", generator=g).float()
    r = r0.clone()
    rc = lib.da3b_linear_resid_f32(ptr(x), M, K, K, ptr(w), N, K, ptr(b), ptr(s), ptr(r), N, stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert lib.da3b_device_status() == 0
    ref = r0 + s * (x.float() @ w.float().t() + b)
    err = (r - ref).abs().max().item()
    assert err <= 1e-3 * ref.abs().max().item() + 1e-4


@pytest.mark.parametrize("B,H,W,IC,OC,ks", [(2, 5, 5, 32, 32, 3), (1, 37, 37, 64, 64, 3), (2, 19, 19, 256, 256, 3),
                                             (1, 74, 74, 48, 64, 3), (1, 37, 37, 128, 256, 1),
                                             (1, 148, 148, 256, 256, 3), (3, 9, 30, 96, 128, 3)])
def test_conv_nhwc(lib, B, H, W, IC, OC, ks):
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + H + IC + OC)
    x = torch.randn(B, H, W, IC, device="cuda", generator=g).half()
    w = torch.randn(OC, IC, ks, ks, device="cuda", generator=g).float() * 0.05
    b = torch.randn(OC, device="cuda", generator=g).float()
    r1 = torch.randn(B, H, W, OC, device="cuda", generator=g).half()
    r2 = torch.randn(B, H, W, OC, device="cuda", generator=g).half()
    icp = (IC + 63) // 64 * 64
    wp = torch.empty(OC, ks * ks, icp, dtype=torch.float16, device="cuda")
    assert lib.da3b_pack_conv_weight(ptr(w), OC, IC, ks, ptr(wp), stream()) == 0
    out = torch.empty(B, H, W, OC, dtype=torch.float16, device="cuda")
    outr = torch.empty_like(out)
    rc = lib.da3b_conv_nhwc(ptr(x), B, H, W, IC, ptr(wp), OC, ks, ptr(b), ptr(r1), ptr(r2), 0, ptr(out), ptr(outr),
                            stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert lib.da3b_device_status() == 0
    ref = torch.nn.functional.conv2d(x.permute(0, 3, 1, 2).float(), w.half().float(), b, padding=ks // 2)
    ref = ref.permute(0, 2, 3, 1) + r1.float() + r2.float()
    close(out, ref)
    close(outr, ref.clamp_min(0))


@pytest.mark.parametrize("case", ["linear", "gelu", "resid", "conv19", "conv37"])
def test_gemm_ksplit(lib, case, monkeypatch):
    """The 1-SM GEMM's K split: with few tiles and a long reduction a cluster of up to 4
    CTAs takes each tile, and the first adds the others' partial accumulators (read over
    distributed shared memory) into its own in rank order before the epilogue. Shapes of
    one image's DPT head: the stride-2 conv as a GEMM (M = 361, K = 6912, N = 768: 36
    tiles, 4 shares), and 3x3 convs through the implicit GEMM ($DA3B_CONV_HALO=0) at 19 x
    19 from 768 channels and 37 x 37 from 384. Against torch fp32, and two runs are
    bit-identical."""
    g = torch.Generator(device="cuda").manual_seed(len(case))
    outs = []
    if case in ("linear", "gelu", "resid"):
        M, K, N = 361, 6912, 768
        x = torch.randn(M, K, device="cuda", generator=g).half()
        w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
        b = torch.randn(N, device="cuda", generator=g).float()
        ref = x.float() @ w.float().t() + b
        if case == "resid":
            sc = torch.randn(N, device="cuda", generator=g).float()
            r0 = torch.randn(M, N, device="cuda", generator=g).float()
            for _ in range(2):
                r = r0.clone()
                assert lib.da3b_linear_resid_f32(ptr(x), M, K, K, ptr(w), N, K, ptr(b), ptr(sc), ptr(r), N, stream()) == 0
                outs.append(r)
            ref = r0 + sc * ref
            torch.cuda.synchronize()
            assert lib.da3b_device_status() == 0
            err = (outs[0] - ref).abs().max().item()
            assert err <= 1e-3 * ref.abs().max().item() + 1e-4
        else:
            act = 2 if case == "gelu" else 0
            for _ in range(2):
                out = torch.empty(M, N, dtype=torch.float16, device="cuda")
                assert lib.da3b_linear_f16(ptr(x), M, K, K, ptr(w), N, K, ptr(b), act, ptr(out), N, stream()) == 0
                outs.append(out)
            if act:
                ref = torch.nn.functional.gelu(ref)
            torch.cuda.synchronize()
            assert lib.da3b_device_status() == 0
            close(outs[0], ref)
    else:
        monkeypatch.setenv("DA3B_CONV_HALO", "0")
        H, IC = (19, 768) if case == "conv19" else (37, 384)
        OC = 128
        x = torch.randn(1, H, H, IC, device="cuda", generator=g).half()
        w = torch.randn(OC, IC, 3, 3, device="cuda", generator=g).float() * 0.02
        b = torch.randn(OC, device="cuda", generator=g).float()
        r1 = torch.randn(1, H, H, OC, device="cuda", generator=g).half()
        wp = torch.empty(OC, 9, IC, dtype=torch.float16, device="cuda")
        assert lib.da3b_pack_conv_weight(ptr(w), OC, IC, 3, ptr(wp), stream()) == 0
        for _ in range(2):
            out, outr = (torch.empty(1, H, H, OC, dtype=torch.float16, device="cuda") for _ in range(2))
            _conv3(lib, x, wp, OC, b, r1, None, out, outr)
            outs.append(out)
        ref = torch.nn.functional.conv2d(x.permute(0, 3, 1, 2).float(), w.half().float(), b, padding=1)
        ref = ref.permute(0, 2, 3, 1) + r1.float()
        close(outs[0], ref)
        close(outr, ref.clamp_min(0))
    assert torch.equal(outs[0], outs[1])


def _conv3(lib, x, wp, OC, b, r1, r2, out, outr, act=0):
    B, H, W, IC = x.shape
    rc = lib.da3b_conv_nhwc(ptr(x), B, H, W, IC, ptr(wp), OC, 3, ptr(b), ptr(r1), ptr(r2), act, ptr(out), ptr(outr),
                            stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert lib.da3b_device_status() == 0


@pytest.mark.parametrize("B,H,W,IC,OC", [(2, 37, 37, 256, 128), (1, 5, 9, 64, 128), (3, 17, 33, 128, 128),
                                         (1, 16, 16, 64, 128), (2, 74, 74, 256, 128), (1, 37, 37, 256, 256),
                                         (2, 19, 21, 512, 256), (1, 148, 148, 64, 128), (1, 296, 296, 128, 64),
                                         (2, 150, 150, 64, 64), (1, 37, 37, 128, 64)])
@pytest.mark.parametrize("pair", ["1", "0", ""], ids=["cta_pair", "one_cta", "auto"])
def test_conv3_halo(lib, B, H, W, IC, OC, pair, monkeypatch):
    """3x3 convs through the halo-box kernel ($DA3B_CONV_HALO=1; by default it serves 128
    output channels): one input box per 64-channel chunk, the nine taps as shifted
    no-swizzle descriptors, output channels in groups of 128. Checked against the
    torch fp32 reference and the implicit-GEMM path ($DA3B_CONV_HALO=0) on the same
    inputs, with bias, both residual addends, the relu copy, ragged tile edges, 1-8
    chunks and one or two output groups; in the CTA-pair form with two 8-wide halves
    per CTA for 128 outputs, one for 256 ($DA3B_CONV_HALO_PAIR=1; an odd number of pixel
    tiles leaves the last pair's second tile empty), the one-CTA form (=0), and the
    automatic choice, which runs 128-output maps of between half and one 16 x 16 tile
    per SM as CTA pairs of one half each (148 x 148) and leaves smaller ones to the
    implicit GEMM. 64 outputs: CTA pairs with two halves of N = 64 per CTA on maps of
    more tiles than SMs (one image's out1 at 296 x 296) or when forced, the implicit
    GEMM otherwise."""
    if pair:
        monkeypatch.setenv("DA3B_CONV_HALO_PAIR", pair)
    else:
        monkeypatch.delenv("DA3B_CONV_HALO_PAIR", raising=False)
    g = torch.Generator(device="cuda").manual_seed(B * 7 + H + W + IC)
    x = torch.randn(B, H, W, IC, device="cuda", generator=g).half()
    w = torch.randn(OC, IC, 3, 3, device="cuda", generator=g).float() * 0.05
    b = torch.randn(OC, device="cuda", generator=g).float()
    r1 = torch.randn(B, H, W, OC, device="cuda", generator=g).half()
    r2 = torch.randn(B, H, W, OC, device="cuda", generator=g).half()
    wp = torch.empty(OC, 9, IC, dtype=torch.float16, device="cuda")
    assert lib.da3b_pack_conv_weight(ptr(w), OC, IC, 3, ptr(wp), stream()) == 0
    out, outr = (torch.full((B, H, W, OC), 7.0, dtype=torch.float16, device="cuda") for _ in range(2))
    monkeypatch.setenv("DA3B_CONV_HALO", "1")  # also for 256 outputs, which default to the GEMM
    _conv3(lib, x, wp, OC, b, r1, r2, out, outr)
    ref = torch.nn.functional.conv2d(x.permute(0, 3, 1, 2).float(), w.half().float(), b, padding=1)
    ref = ref.permute(0, 2, 3, 1) + r1.float() + r2.float()
    close(out, ref)
    close(outr, ref.clamp_min(0))
    monkeypatch.setenv("DA3B_CONV_HALO", "0")
    gout, goutr = torch.empty_like(out), torch.empty_like(out)
    _conv3(lib, x, wp, OC, b, r1, r2, gout, goutr)
    close(out, gout.float(), rel=1e-3, abs_=1e-3)
    # plain form (bias only, relu activation) as output_conv1 / layer convs use it
    monkeypatch.setenv("DA3B_CONV_HALO", "1")
    out2 = torch.empty_like(out)
    _conv3(lib, x, wp, OC, b, None, None, out2, None, act=1)
    ref2 = torch.nn.functional.conv2d(x.permute(0, 3, 1, 2).float(), w.half().float(), b, padding=1)
    close(out2, ref2.permute(0, 2, 3, 1).clamp_min(0))


@pytest.mark.parametrize("nseq,seqlen,heads", [(1, 1, 1), (2, 37, 2), (3, 1370, 6), (1, 1297 * 3, 4), (2, 200, 16),
                                               (2, 128, 2), (1, 129, 3), (3, 255, 1), (1, 256, 2), (2, 257, 2),
                                               (1, 1297 * 8, 2), (1, 1370, 12), (1, 1370, 6)])
def test_attention(lib, nseq, seqlen, heads):
    """da3b_attention against torch fp32 softmax attention: sequence lengths on both sides
    of the 128-query and 128-key tile edges (one or two query tiles per CTA, ragged last
    key tile), several sequences and heads, and an 8-view global sequence, with the
    automatic key-range split: (1, 1370, 12) (one ViT-B image) runs 2 shares a query
    tile, (1, 1370, 6) 3, (1, 1297 * 3, 4) 4, the others one."""
    g = torch.Generator(device="cuda").manual_seed(seqlen + heads)
    D = heads * 64
    qkv = (torch.randn(nseq * seqlen, 3 * D, device="cuda", generator=g) * 1.5).half()
    out = torch.empty(nseq * seqlen, D, dtype=torch.float16, device="cuda")
    assert lib.da3b_attention(ptr(qkv), nseq, seqlen, heads, ptr(out), stream()) == 0
    torch.cuda.synchronize()
    assert lib.da3b_device_status() == 0
    q, k, v = qkv.float().view(nseq, seqlen, 3, heads, 64).permute(2, 0, 3, 1, 4)
    ref = torch.softmax(q @ k.transpose(-1, -2) / 8.0, dim=-1) @ v          # [nseq, heads, seqlen, 64]
    ref = ref.permute(0, 2, 1, 3).reshape(nseq * seqlen, D)
    close(out, ref, rel=5e-3, abs_=5e-3)


@pytest.mark.parametrize("shares", [2, 3, 4])
@pytest.mark.parametrize("nseq,seqlen,heads", [(1, 1370, 12), (2, 257, 2), (1, 129, 3), (3, 300, 1)])
def test_attention_split_shares(lib, nseq, seqlen, heads, shares):
    """Each query tile's keys shared out over a cluster of 2-4 CTAs (forced with
    da3b_set_attention_split; by default only when the grid leaves SMs idle and every
    share keeps 6 key tiles), merged through distributed shared memory in rank order:
    against torch fp32 attention, ragged last key tiles and uneven shares included, and
    against the unsplit kernel; two runs are bit-identical."""
    g = torch.Generator(device="cuda").manual_seed(seqlen * 3 + heads + shares)
    D = heads * 64
    qkv = (torch.randn(nseq * seqlen, 3 * D, device="cuda", generator=g) * 1.5).half()
    outs = []
    try:
        for n in (shares, shares, 1):
            assert lib.da3b_set_attention_split(n) == 0
            out = torch.empty(nseq * seqlen, D, dtype=torch.float16, device="cuda")
            assert lib.da3b_attention(ptr(qkv), nseq, seqlen, heads, ptr(out), stream()) == 0
            torch.cuda.synchronize()
            assert lib.da3b_device_status() == 0
            outs.append(out)
    finally:
        lib.da3b_set_attention_split(-1)
    q, k, v = qkv.float().view(nseq, seqlen, 3, heads, 64).permute(2, 0, 3, 1, 4)
    ref = torch.softmax(q @ k.transpose(-1, -2) / 8.0, dim=-1) @ v
    ref = ref.permute(0, 2, 1, 3).reshape(nseq * seqlen, D)
    close(outs[0], ref, rel=5e-3, abs_=5e-3)
    assert torch.equal(outs[0], outs[1])
    close(outs[0], outs[2].float(), rel=5e-3, abs_=5e-3)


@pytest.mark.parametrize("B,hs,ws,C,H,W", [(2, 296, 296, 128, 518, 518), (1, 37, 37, 256, 74, 74), (3, 19, 19, 64, 37, 37),
                                        (1, 5, 9, 40, 23, 17), (2, 8, 8, 32, 8, 8)])
def test_upsample_align_corners(lib, B, hs, ws, C, H, W):
    """da3b_upsample_nhwc vs torch bilinear interpolate with align_corners=True (the
    ggml ALIGN_CORNERS formula): within f16 output rounding."""
    g = torch.Generator(device="cuda").manual_seed(hs * 100 + C)
    x = torch.randn(B, hs, ws, C, device="cuda", generator=g).half()
    out = torch.empty(B, H, W, C, dtype=torch.float16, device="cuda")
    assert lib.da3b_upsample_nhwc(ptr(x), B, hs, ws, C, ptr(out), H, W, stream()) == 0
    torch.cuda.synchronize()
    ref = torch.nn.functional.interpolate(x.permute(0, 3, 1, 2).float(), size=(H, W), mode="bilinear",
                                          align_corners=True).permute(0, 2, 3, 1)
    close(out, ref, rel=2e-3, abs_=2e-3)


@pytest.mark.parametrize("nseq,seqlen,heads", [(2, 1370, 4), (1, 300, 2), (3, 129, 2), (2, 100, 2), (1, 257, 2),
                                                (1, 2 * 1297, 3)])
def test_attention_pp_kernel(nseq, seqlen, heads):
    """The warp-specialised attention kernel (two query tiles per CTA, one-pass softmax
    over 128-key tiles), selectable with DA3B_ATTN_PP=1 (read once per process, so it
    runs in a fresh subprocess), against torch fp32. The sizes cover CTAs with one and
    with two query tiles and ragged last key tiles."""
    import subprocess
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    code = ("import sys; sys.path.insert(0, %r); sys.path.insert(0, %r)\n"
            "from da3cpplib_b200 import _lib\n"
            "import test_gemm_gpu as t\n"
            "t.test_attention(_lib.load(), %d, %d, %d)\n"
            "print('ok')\n" % (os.path.dirname(here), here, nseq, seqlen, heads))
    env = dict(os.environ, DA3B_ATTN_PP="1")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]
