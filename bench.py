#!/usr/bin/env python3
"""Benchmark of the DA3cpplib depth hot path on B200 (libda3b).

Workload (the north-star metric): Depth Anything V2 Large
(ViT-L/14, 24 layers, Q8_0 linears, DPT head with 256 features), a batch of 64
seeded uniform RGB8 518x518 images sharded 64/N per GPU (strong scaling: the job is
fixed at 64 images). Random-init GGUF weights in the reference layout (the parity
tests' stress init, whose depth map is non-degenerate; see da3cpplib_b200/synth.py).

One step = one forward of the rank's shard: RGB8 -> normalise/patchify -> 24 ViT
blocks -> DPT head -> depth maps. `value` times steps with inputs resident in HBM;
`e2e` times the same call with pinned host buffers (H2D of the images and D2H of
the depth maps inside the timed region). The L2 (126 MB) is flushed between timed
steps by writing a 256 MB buffer outside the timed events.

--impl reference times the CPU restatement of the reference (oracle/) on the host
cores instead (rank 0 only).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

MODEL = "da2-l"
IMAGES_TOTAL = 64
H = W = 518
METRIC = "images/s ViT-L Q8_0 518² at 1/2/4/8 B200; GEMM/conv % of tensor-core peak"
UNIT = "images/s"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.dev}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        loaded = [v for v in sm if v > 0.5 * (mx or max(sm))] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def images_for(rank, world):
    from da3cpplib_b200 import shard, synth

    first, end = shard.shard_range(IMAGES_TOTAL, world, rank)
    return np.stack([synth.image(synth.IMAGE_SEED, i, H, W) for i in range(first, end)]), end - first


def model_path(rank, world):
    from da3cpplib_b200 import synth

    path = None
    if rank == 0:
        path = synth.ensure_gguf(MODEL, stress=True)
    if world > 1:
        import torch.distributed as dist

        obj = [path]
        dist.broadcast_object_list(obj, src=0)
        path = obj[0]
    return path


# ---------------------------------------------------------------------- reference arm
def cpu_reference_step_seconds(n_images=1, warmup=0, steps=1, path=None):
    """Oracle (CPU restatement of the reference) on `n_images` images per step."""
    from da3cpplib_b200 import synth
    from oracle.oracle import Oracle

    if path is None:
        path = synth.ensure_gguf(MODEL, stress=True)
    orc = Oracle(path, act_quant=True, n_threads=os.cpu_count() or 1)
    img = synth.image(synth.IMAGE_SEED, 0, H, W)
    for _ in range(warmup):
        for _ in range(n_images):
            orc.infer(img)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        for _ in range(n_images):
            orc.infer(img)
        times.append(time.perf_counter() - t0)
    return times


def run_reference(args):
    world, rank, local = dist_setup(args)
    if rank != 0:
        return 0
    cores = os.cpu_count() or 1
    times = cpu_reference_step_seconds(1, args.warmup, args.steps)
    per_step = statistics.mean(times)
    value = 1.0 / per_step
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8xint8->f32 (Q8_0), f32", "data": "synthetic",
        "config": {"workload": "DA2-L (ViT-L/14) Q8_0, 518x518 RGB8, 1 image per step (bounded sample of the 64)",
                   "model": "da2-large-random", "global_batch": 1, "seq_len": 1370, "parallelism": "cpu"},
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": "1 image of DA2-L 518x518 per step (CPU restatement of the reference; "
                                   "the ggml reference cannot be built: its submodule is absent)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------- GPU arm
def run_gpu(args):
    import ctypes

    import torch

    world, rank, local = dist_setup(args)
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    from da3cpplib_b200 import Model

    path = model_path(rank, world)
    model = Model(path, local)
    imgs, per = images_for(rank, world)
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream
    rgb_dev = torch.from_numpy(imgs).cuda()
    depth_dev = torch.empty((per, H, W), dtype=torch.float32, device="cuda")
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")

    def step(rgb_ptr, depth_ptr):
        model.infer_device(rgb_ptr, per, H, W, depth_ptr, stream=sptr)
        if args.gather and dist and depth_ptr == depth_dev.data_ptr():
            # optional NCCL gather of the depth maps to rank 0 (equal-sized slabs)
            from da3cpplib_b200 import shard

            shard.gather_to_rank0(depth_dev, IMAGES_TOTAL)

    # warm-up (plan creation, graph capture)
    for _ in range(max(args.warmup, 3)):
        step(rgb_dev.data_ptr(), depth_dev.data_ptr())
    torch.cuda.synchronize()
    launches = model.launches(per, H, W)

    def timed(rgb_ptr, depth_ptr):
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        for i in range(args.steps):
            flush.fill_(float(i))
            starts[i].record(stream)
            step(rgb_ptr, depth_ptr)
            ends[i].record(stream)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
        t = torch.tensor([sum(ms)], dtype=torch.float64, device="cuda")
        if dist:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item() / args.steps

    with ClockSampler(local) as clk:
        ms_step = timed(rgb_dev.data_ptr(), depth_dev.data_ptr())
    clocks = clk.summary()
    st = model.lib.da3b_device_status()
    if st != 0:
        raise RuntimeError(f"device status {st} after the timed region")
    value = IMAGES_TOTAL / (ms_step / 1e3)

    # e2e: pinned host in / out through the same public call
    rgb_host = torch.from_numpy(imgs).pin_memory()
    depth_host = torch.empty((per, H, W), dtype=torch.float32).pin_memory()
    step(rgb_host.data_ptr(), depth_host.data_ptr())
    torch.cuda.synchronize()
    ms_e2e = timed(rgb_host.data_ptr(), depth_host.data_ptr())
    # whole-job bytes per step (every rank copies its own shard in and out)
    e2e = {"value": IMAGES_TOTAL / (ms_e2e / 1e3), "unit": UNIT, "h2d_bytes_per_step": int(IMAGES_TOTAL * H * W * 3),
           "d2h_bytes_per_step": int(IMAGES_TOTAL * H * W * 4)}
    # sanity: the host result equals the device-resident result
    if not torch.equal(depth_host, depth_dev.cpu()):
        raise RuntimeError("e2e and device-resident outputs differ")

    # live roofline of the dominant kernel: the fc1 GEMM of this workload timed alone
    hbm, tflops, src = peaks()
    M, K, N = per * (1 + (H // 14) * (W // 14)), 1024, 4096
    A = torch.randn(M, K, device="cuda").half()
    Wt = (torch.randn(N, K, device="cuda") * 0.02).half()
    bias = torch.zeros(N, device="cuda")
    out = torch.empty(M, N, dtype=torch.float16, device="cuda")
    V = ctypes.c_void_p

    def gemm():
        rc = model.lib.da3b_linear_f16(V(A.data_ptr()), M, K, K, V(Wt.data_ptr()), N, K, V(bias.data_ptr()), 2,
                                       V(out.data_ptr()), N, V(sptr))
        assert rc == 0

    for _ in range(3):
        gemm()
    torch.cuda.synchronize()
    reps = 20
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        gemm()
    e1.record(stream)
    torch.cuda.synchronize()
    gemm_ms = e0.elapsed_time(e1) / reps
    flops = 2.0 * M * K * N
    achieved = flops / (gemm_ms / 1e3) / 1e12
    # DRAM read+write of one fc1 launch from an ncu capture of the same kernel at
    # M = 21920 (profiles/gemm_fc1_m21920_k1024_n4096_gelu.txt: 53.57 MB read +
    # 123.73 MB written), scaled by M to this launch (traffic grows with M; the 8.4 MB
    # weight is the only fixed part)
    traffic = int(round((53.567488e6 + 123.73248e6) * M / 21920))
    roofline = {"bound": "tensor", "achieved": round(achieved, 1), "peak": tflops, "unit": "TFLOP/s",
                "frac": round(achieved / tflops, 4), "traffic": traffic,
                "traffic_note": "bytes per launch, ncu dram__bytes_read+write at M=21920 scaled by M",
                "algorithmic_bytes": int(2 * (M * K + K * N + M * N)),
                "kernel": f"k_tc_gemm<256> fc1 M={M} K={K} N={N} (+bias, erf-GELU), {src} bf16 dense peak",
                "ms_per_launch": round(gemm_ms, 4)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        times = cpu_reference_step_seconds(1, 0, 1, path)
        cpu = {"value": 1.0 / times[0], "unit": UNIT, "cores": os.cpu_count() or 1, "kind": "port",
               "sample": "1 image of DA2-L 518x518 through the CPU restatement of the reference (oracle/), "
                         "all host threads"}

    if rank == 0:
        flops_img = 1304e9
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16 (Q8_0 weights dequantised to f16, f32 accumulate)",
            "data": "synthetic (seeded uniform RGB8, random-init Q8_0 GGUF)",
            "config": {"workload": "C3: DA2-L ViT-L/14 Q8_0 + DPT head, 64 images 518x518 sharded 64/N",
                       "model": "da2-large-random", "global_batch": IMAGES_TOTAL, "per_gpu_batch": per,
                       "seq_len": 1370, "parallelism": f"dp{world}",
                       "gather": "depth maps to rank 0 over NCCL each step" if (args.gather and world > 1) else "none",
                       "l2": "flushed (256 MB write) between timed steps"},
            "e2e": {k: (round(v, 2) if isinstance(v, float) else v) for k, v in e2e.items()},
            "roofline": roofline,
            "model_tflops": round(flops_img * IMAGES_TOTAL / (ms_step / 1e3) / 1e12, 1),
            "gpu_launches": launches * args.steps,
            "clocks": clocks,
        }
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--gather", action="store_true",
                    help="N>1: gather every step's depth maps to rank 0 over NCCL inside the timed region")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
