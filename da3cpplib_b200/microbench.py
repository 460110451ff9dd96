"""Isolated hot-path kernel sweep (the reference's microbench workload) on one GPU.

Part A: Q8_0 x f16 linears. Weights are GGUF Q8_0 rows (int8 uniform in [-127, 127],
f16 scales uniform in [1e-3, 1e-2]) repacked once by da3b_dequant_q8_0 (load time,
timed separately); the timed op is da3b_linear_f16 on f16 N(0, 1) activations,
M in {1370, 8*1370, 64*1370} x (K, N) in {(384, 1152), (768, 3072), (1024, 4096),
(4096, 1024), (1536, 6144)}.
Part B: DPT-head 3x3 stride-1 pad-1 convs, NHWC f16, C_in = C_out in {64, 128, 256},
spatial 37..296, batch 8 (da3b_conv_nhwc).
attn: da3b_attention at the C3 shape (64 x 1370 tokens, 16 heads) and the DA3
multi-view global layer (8 views x 1297 tokens per scene), each with the V^T
transpose and as the flash-attention kernel alone (da3b_attention_vt), next to cuDNN's
fused attention through torch on the same tensors as a yardstick.
mma: the tensor-pipe cost of one M=128, K=16 f16 tcgen05.mma for N = 64..256, A from
shared or tensor memory (da3b_debug_mma_cycles, one CTA per SM, one accumulator).
out2: da3b_output_conv2 (upsample 296 -> 518 + 3x3 conv 128 -> 32 + 1x1 -> depth) at the
C3 head shape, fused and through a materialised upsampled map.
ray: da3b_ray_pose (the ray->pose solver, both host round trips included; wall time)
on a synthetic 288 x 288 ray field, the aux resolution of a 504 x 504 image.
c4: the C4 workload end to end on one GPU: a DA3-L random-init Q8_0 GGUF, --scenes
scenes (default 16) x 8 views of 504 x 504 RGB8 already on the device, depth and
confidence out (da3b_infer_device, views_per_scene = 8: local/global alternation,
reference-view selection, camera token, UV pos-embed). One step = all scenes; the L2
is flushed (256 MB write) before each timed step. Model work per scene is the
algorithmic count of the scope table: linears 6.27 TF + attention 4.41 + pass A 2.21
+ depth head 2.26 = 15.15 TFLOP.

Each line: {"part", "case", "ms", "tflops", "frac", "peak"}; frac is against the
measured dense bf16 burst peak of this GPU pool (MEASURED_PEAKS.json, else the pool's
fallback figure). Times are CUDA events around `reps` back-to-back launches on the
launching stream after 3 warm-up launches. Usage:
    python -m da3cpplib_b200.microbench [--part A|B|attn|mma|all] [--m 87680] [--reps 20]
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

M_SET = (1370, 8 * 1370, 64 * 1370)
KN_SET = ((384, 1152), (768, 3072), (1024, 4096), (4096, 1024), (1536, 6144))
CONV_C = (64, 128, 256)
CONV_HW = (37, 74, 148, 296)


def peak_tflops():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


def peak_hbm():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def q8_0_weights(torch, N, K, gen):
    """GGUF Q8_0 bytes [N][K/32][34] on the device: f16 d then 32 int8."""
    nb = K // 32
    q = torch.randint(-127, 128, (N, nb, 32), generator=gen, device="cuda", dtype=torch.int8)
    d = (torch.rand((N, nb), generator=gen, device="cuda") * 9e-3 + 1e-3).half()
    raw = torch.empty((N, nb, 34), dtype=torch.uint8, device="cuda")
    raw[:, :, :2] = d.view(torch.uint8).view(N, nb, 2)
    raw[:, :, 2:] = q.view(torch.uint8)
    return raw


def main(argv=None):
    import torch

    from . import _lib

    ap = argparse.ArgumentParser()
    ap.add_argument("--part", default="all", choices=["A", "A8", "B", "attn", "up", "pre", "ray", "out2", "c4", "mma", "all"])
    ap.add_argument("--scenes", type=int, default=16, help="c4: scenes of 8 views")
    ap.add_argument("--m", type=int, default=0, help="Part A: only this M")
    ap.add_argument("--kn", default="", help="Part A: only this K,N (e.g. 1024,4096)")
    ap.add_argument("--act", type=int, default=0, help="Part A activation: 0 none, 2 erf-GELU")
    ap.add_argument("--c", type=int, default=0, help="Part B: only this channel count")
    ap.add_argument("--hw", type=int, default=0, help="Part B: only this spatial size")
    ap.add_argument("--cout", type=int, default=0, help="Part B: output channels (default = input channels)")
    ap.add_argument("--batch", type=int, default=8, help="Part B / up: images")
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--attn-nseq", type=int, default=0, help="attn: only the C3 shape with this many sequences")
    ap.add_argument("--attn-heads", type=int, default=16, help="attn with --attn-nseq: heads (12: the C2 shape)")
    args = ap.parse_args(argv)

    L = _lib.load()
    V = ctypes.c_void_p
    P = lambda t: V(t.data_ptr())
    s = torch.cuda.current_stream()
    S = V(s.cuda_stream)
    peak, src = peak_tflops()
    gen = torch.Generator(device="cuda").manual_seed(20260101)

    def timeit(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(s)
        for _ in range(args.reps):
            fn()
        b.record(s)
        torch.cuda.synchronize()
        if L.da3b_device_status() != 0:
            raise RuntimeError("device status set")
        return a.elapsed_time(b) / args.reps

    def emit(part, case, ms, flops, extra=None):
        tf = flops / (ms / 1e3) / 1e12
        line = {"part": part, "case": case, "ms": round(ms, 4), "tflops": round(tf, 1),
                "frac": round(tf / peak, 4), "peak": f"{peak} TFLOP/s ({src})"}
        if extra:
            line.update(extra)
        print(json.dumps(line), flush=True)

    if args.part in ("A", "all"):
        kns = KN_SET if not args.kn else (tuple(int(v) for v in args.kn.split(",")),)
        ms_set = M_SET if not args.m else (args.m,)
        for K, N in kns:
            raw = q8_0_weights(torch, N, K, gen)
            W = torch.empty((N, K), dtype=torch.float16, device="cuda")
            dq_ms = timeit(lambda: L.da3b_dequant_q8_0(P(raw), N, K, P(W), K, S))
            bias = torch.randn(N, generator=gen, device="cuda")
            for M in ms_set:
                x = torch.randn((M, K), generator=gen, device="cuda").half()
                y = torch.empty((M, N), dtype=torch.float16, device="cuda")

                def run():
                    rc = L.da3b_linear_f16(P(x), M, K, K, P(W), N, K, P(bias), args.act, P(y), N, S)
                    if rc:
                        raise RuntimeError(f"da3b_linear_f16 rc={rc}")

                ms = timeit(run)
                emit("A", f"M={M} K={K} N={N} act={args.act}", ms, 2.0 * M * K * N,
                     {"dequant_ms_load_time": round(dq_ms, 4),
                      "l2": "inputs exceed L2" if (M * K + M * N) * 2 > 126e6 else "inputs fit in L2"})
                del x, y
            del raw, W

    if args.part in ("A8", "all"):
        # the int8 route (tcgen05.mma kind::i8, ggml-exact per-block rescale) against the
        # f16 GEMM on the same shapes; TFLOP/s counts 2 M N K operations for both
        kns = ((1024, 4096), (4096, 1024)) if not args.kn else (tuple(int(v) for v in args.kn.split(",")),)
        ms_set = (10960, 87680) if not args.m else (args.m,)
        for K, N in kns:
            raw = q8_0_weights(torch, N, K, gen)
            qw = torch.empty((N, K), dtype=torch.int8, device="cuda")
            dwt = torch.empty((K // 32, N), dtype=torch.float32, device="cuda")
            if L.da3b_repack_q8_0(P(raw), N, K, P(qw), P(dwt), S):
                raise RuntimeError("repack failed")
            for M in ms_set:
                x = torch.randn((M, K), generator=gen, device="cuda")
                q = torch.empty((M, K), dtype=torch.int8, device="cuda")
                d = torch.empty((M, K // 32), dtype=torch.float32, device="cuda")
                y = torch.empty((M, N), dtype=torch.float32, device="cuda")

                def quant():
                    if L.da3b_quantize_q8_0(P(x), M, K, P(q), P(d), S):
                        raise RuntimeError("quantize failed")

                def run():
                    rc = L.da3b_linear_q8q8_i8(P(q), P(d), M, K, P(qw), P(dwt), N, None, P(y), N, S)
                    if rc:
                        raise RuntimeError(f"da3b_linear_q8q8_i8 rc={rc}")

                qms = timeit(quant)
                ms = timeit(run)
                emit("A8", f"M={M} K={K} N={N} int8 kind::i8", ms, 2.0 * M * K * N,
                     {"quantize_ms": round(qms, 4)})
                del x, q, d, y
            del raw, qw, dwt

    if args.part in ("B", "all"):
        for C in (CONV_C if not args.c else (args.c,)):
            OC = args.cout or C
            w = torch.randn((OC, C, 3, 3), generator=gen, device="cuda") * 0.02
            icp = (C + 63) // 64 * 64
            wp = torch.empty((OC, 9, icp), dtype=torch.float16, device="cuda")
            assert L.da3b_pack_conv_weight(P(w), OC, C, 3, P(wp), S) == 0
            b = torch.randn(OC, generator=gen, device="cuda")
            for hw in (CONV_HW if not args.hw else (args.hw,)):
                B = args.batch
                x = torch.randn((B, hw, hw, C), generator=gen, device="cuda").half()
                o = torch.empty((B, hw, hw, OC), dtype=torch.float16, device="cuda")

                def run():
                    rc = L.da3b_conv_nhwc(P(x), B, hw, hw, C, P(wp), OC, 3, P(b), None, None, 0, P(o), None, S)
                    if rc:
                        raise RuntimeError(f"da3b_conv_nhwc rc={rc}")

                ms = timeit(run)
                emit("B", f"B={B} {hw}x{hw} Cin={C} Cout={OC}", ms, 2.0 * B * hw * hw * C * OC * 9)
                del x, o

    if args.part in ("up", "all"):
        # align-corners bilinear upsamples: the fusion pyramid's last step (148 -> 296,
        # 256 channels) and the DPT tail without the fused output stage (296 -> 518, 128)
        for hs, hd, C in ((148, 296, 256), (296, 518, 128)):
            B = args.batch
            x = torch.randn((B, hs, hs, C), generator=gen, device="cuda").half()
            o = torch.empty((B, hd, hd, C), dtype=torch.float16, device="cuda")

            def run():
                rc = L.da3b_upsample_nhwc(P(x), B, hs, hs, C, P(o), hd, hd, S)
                if rc:
                    raise RuntimeError(f"da3b_upsample_nhwc rc={rc}")

            ms = timeit(run)
            gbs = (x.numel() + o.numel()) * 2 / (ms / 1e3) / 1e9
            hbm = peak_hbm()
            print(json.dumps({"part": "up", "case": f"B={B} {hs}->{hd} C={C}", "ms": round(ms, 4),
                              "GB/s": round(gbs, 1), "frac": round(gbs / hbm[0], 4),
                              "peak": f"{hbm[0]} GB/s ({hbm[1]})"}), flush=True)
            del x, o

    if args.part in ("pre", "all"):
        # normalise + patchify of the C3 batch: 64 RGB8 images 518x518 -> f16 operand [64*1369][640]
        B, H, W, ldk = 64, 518, 518, 640
        img = torch.randint(0, 256, (B, H, W, 3), generator=gen, device="cuda", dtype=torch.uint8)
        o = torch.empty((B * (H // 14) * (W // 14), ldk), dtype=torch.float16, device="cuda")
        mean = (ctypes.c_float * 3)(0.485, 0.456, 0.406)
        std = (ctypes.c_float * 3)(0.229, 0.224, 0.225)

        def run():
            rc = L.da3b_patchify(P(img), B, H, W, 14, mean, std, P(o), ldk, S)
            if rc:
                raise RuntimeError(f"da3b_patchify rc={rc}")

        ms = timeit(run)
        gbs = (img.numel() + o.numel() * 2) / (ms / 1e3) / 1e9
        hbm = peak_hbm()
        print(json.dumps({"part": "pre", "case": f"patchify B={B} {H}x{W}", "ms": round(ms, 4), "GB/s": round(gbs, 1),
                          "frac": round(gbs / hbm[0], 4), "peak": f"{hbm[0]} GB/s ({hbm[1]})"}), flush=True)
        del img, o

    if args.part in ("attn", "all"):
        cases = ((64, 1370, 16, "C3 per-image"), (2, 8 * 1297, 16, "C4 global, 2 scenes"))
        if args.attn_nseq:
            cases = ((args.attn_nseq, 1370, args.attn_heads, "1370 tokens"),)
        for nseq, seqlen, heads, tag in cases:
            D = heads * 64
            qkv = torch.randn((nseq * seqlen, 3 * D), generator=gen, device="cuda").half()
            out = torch.empty((nseq * seqlen, D), dtype=torch.float16, device="cuda")

            def run():
                rc = L.da3b_attention(P(qkv), nseq, seqlen, heads, P(out), S)
                if rc:
                    raise RuntimeError(f"da3b_attention rc={rc}")

            ms = timeit(run)
            emit("attn", f"{tag}: nseq={nseq} seqlen={seqlen} heads={heads}", ms, 4.0 * nseq * seqlen * seqlen * D)
            # the flash-attention kernel alone, V^T prepared once (as the QKV GEMM epilogue
            # provides it inside the engine)
            ld = (seqlen + 7) // 8 * 8
            vt = torch.empty(nseq * heads * 64 * ld, dtype=torch.float16, device="cuda")
            assert L.da3b_transpose_v(P(qkv), nseq, seqlen, heads, P(vt), ld, S) == 0

            def run_vt():
                rc = L.da3b_attention_vt(P(qkv), P(vt), ld, nseq, seqlen, heads, P(out), S)
                if rc:
                    raise RuntimeError(f"da3b_attention_vt rc={rc}")

            ms = timeit(run_vt)
            emit("attn", f"{tag}, kernel only: nseq={nseq} seqlen={seqlen} heads={heads}", ms,
                 4.0 * nseq * seqlen * seqlen * D)
            del vt
            # yardstick, not part of this library: cuDNN's fused attention through torch on
            # the same q, k, v (f16, no mask, scale 1/8)
            try:
                from torch.nn.attention import SDPBackend, sdpa_kernel
                q, k, v = (qkv.view(nseq, seqlen, 3, heads, 64)[:, :, i].transpose(1, 2).contiguous() for i in range(3))
                with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
                    ms = timeit(lambda: torch.nn.functional.scaled_dot_product_attention(q, k, v))
                emit("attn", f"{tag}, cuDNN SDPA via torch (reference): nseq={nseq} seqlen={seqlen} heads={heads}", ms,
                     4.0 * nseq * seqlen * seqlen * D)
            except Exception as e:  # noqa: BLE001 - a missing backend only drops the yardstick line
                print(json.dumps({"part": "attn", "case": f"{tag}, cuDNN SDPA", "unavailable": str(e)[:200]}))
            del qkv, out

    if args.part == "mma":
        # tensor-pipe cost per M=128, K=16 f16 tcgen05.mma, one CTA per SM, one accumulator
        nsm = torch.cuda.get_device_properties(0).multi_processor_count
        cyc = torch.zeros(nsm, dtype=torch.int64, device="cuda")
        iters = 2000
        for a_tmem in (0, 1):
            for n in (64, 80, 128, 256):
                cyc.zero_()
                rc = L.da3b_debug_mma_cycles(n, a_tmem, iters, nsm, P(cyc), S)
                torch.cuda.synchronize()
                if rc or L.da3b_device_status() != 0:
                    raise RuntimeError(f"da3b_debug_mma_cycles rc={rc}")
                c = cyc.float()
                per = c[c > 0].median().item() / (iters * 4)
                full = 128 * n * 16 / 4096  # cycles at 4096 f16 MAC per clock per SM
                print(json.dumps({"part": "mma", "A": "tmem" if a_tmem else "smem", "M": 128, "N": n, "K": 16,
                                  "cycles": round(per, 1), "full_rate_cycles": full,
                                  "frac": round(full / per, 3)}), flush=True)

    if args.part in ("out2", "all"):
        B, hs, C, H = args.batch if args.batch != 8 else 64, 296, 128, 518
        feat = (torch.randn((B, hs, hs, C), generator=gen, device="cuda") * 0.5).half()
        raw = torch.randn((32, C, 3, 3), generator=gen, device="cuda") / (9 * C) ** 0.5
        wp = torch.zeros((32, 9, C), dtype=torch.float16, device="cuda")
        if L.da3b_pack_conv_weight(P(raw), 32, C, 3, P(wp), S):
            raise RuntimeError("pack failed")
        b1 = torch.randn(32, generator=gen, device="cuda") * 0.1
        w2 = torch.randn((1, 32), generator=gen, device="cuda") * 0.2
        b2 = torch.zeros(1, device="cuda")
        out = torch.empty((B, H, H), device="cuda")
        act = (ctypes.c_int * 1)(3)
        outs = (ctypes.c_void_p * 1)(out.data_ptr())
        flops = 2.0 * B * H * H * C * 32 * 9
        for fused in (1, 0):
            def run():
                rc = L.da3b_output_conv2(P(feat), B, hs, hs, C, None, H, H, P(wp), P(b1), P(w2), P(b2), 1, act,
                                         ctypes.c_float(0.0), outs, fused, S)
                if rc:
                    raise RuntimeError(f"da3b_output_conv2 rc={rc}")

            ms = timeit(run)
            emit("out2", f"{'fused' if fused else 'unfused'} B={B} {hs}->{H} C={C}", ms, flops)
        del feat, out

    if args.part == "c4":
        from . import Model, synth

        n_sc, V, HW = args.scenes, 8, 504
        m = Model(synth.ensure_gguf("da3-l", stress=True), 0)
        rgb = torch.randint(0, 256, (n_sc * V, HW, HW, 3), generator=gen, device="cuda", dtype=torch.uint8)
        depth = torch.empty((n_sc * V, HW, HW), device="cuda")
        conf = torch.empty_like(depth)
        flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda")

        def step():
            m.infer_device(rgb.data_ptr(), n_sc * V, HW, HW, depth.data_ptr(), conf.data_ptr(),
                           views_per_scene=V, stream=s.cuda_stream)

        for _ in range(3):
            step()
        torch.cuda.synchronize()
        times = []
        for _ in range(args.reps):
            flush.fill_(1.0)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(s)
            step()
            b.record(s)
            torch.cuda.synchronize()
            times.append(a.elapsed_time(b))
        if L.da3b_device_status() != 0:
            raise RuntimeError("device status set")
        ms = sum(times) / len(times)
        tf = 15.15e12 * n_sc / (ms / 1e3) / 1e12
        print(json.dumps({"part": "c4", "case": f"DA3-L {n_sc} scenes x {V} views {HW}x{HW}", "ms": round(ms, 3),
                          "scenes/s": round(n_sc / (ms / 1e3), 2), "views/s": round(n_sc * V / (ms / 1e3), 1),
                          "model_tflops": round(tf, 1), "frac": round(tf / peak, 4),
                          "peak": f"{peak} TFLOP/s ({src})", "launches": m.launches(n_sc * V, HW, HW, V),
                          "l2": "flushed (256 MB write) before each step"}), flush=True)
        m.close()
        del rgb, depth, conf, flush

    if args.part in ("ray", "all"):
        import time

        from . import synth

        ctx = L.da3b_load(synth.ensure_gguf("da3-t", stress=True).encode(), 0)
        g = 288
        rng = np.random.default_rng(7)
        t = (np.arange(g) + 0.5) / g * 2 - 1
        X, Y = np.meshgrid(t, t)
        dirs = np.stack([X / 0.9, Y / 1.1, np.ones_like(X)], 0) + rng.standard_normal((3, g, g)) * 1e-3
        bad = rng.random((g, g)) < 0.2
        dirs[:, bad] = rng.standard_normal((3, int(bad.sum())))
        planes = np.concatenate([dirs, np.ones((3, g, g)) * 0.5, rng.uniform(1, 3, (1, g, g))], 0).astype(np.float32)
        d = torch.from_numpy(planes).cuda()
        ext = np.zeros(12, np.float32)
        intr = np.zeros(9, np.float32)
        torch.cuda.synchronize()

        def solve():
            rc = L.da3b_ray_pose(ctx, P(d), 1, 0, g, g, 504, 504, ext.ctypes.data, intr.ctypes.data, None, S)
            if rc:
                raise RuntimeError(f"da3b_ray_pose rc={rc}")

        for _ in range(3):
            solve()
        t0 = time.perf_counter()
        for _ in range(args.reps):
            solve()
        ms = (time.perf_counter() - t0) * 1e3 / args.reps
        print(json.dumps({"part": "ray", "case": f"ray->pose {g}x{g} points (504x504 image)", "ms": round(ms, 3),
                          "timing": "wall clock per call, host round trips included"}), flush=True)
        L.da_capi_free(ctx)


if __name__ == "__main__":
    main()
