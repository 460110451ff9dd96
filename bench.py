#!/usr/bin/env python3
"""Benchmark of the DA3cpplib depth hot path on B200 (libda3b).

Workloads (--workload, default c3):
  c3  the north-star metric's config: Depth Anything V2 Large (ViT-L/14, 24 layers, Q8_0
      linears, DPT head with 256 features), 64 seeded uniform RGB8 518x518 images sharded
      64/N per GPU (strong scaling: the job is fixed at 64 images).
  c4  Depth Anything 3 Large multi-view: 16 scenes x 8 views of 504x504, sharded by
      scene (16/N scenes per GPU; a scene's views share global attention), depth and
      confidence out.
  c2  Depth Anything V2 Base latency path: one 518x518 image per step on each GPU
      (replicas only at N > 1).
Random-init GGUF weights in the reference layout (the parity tests' stress init, whose
depth map is non-degenerate; see da3cpplib_b200/synth.py).

One step = one forward of the rank's shard: RGB8 -> normalise/patchify -> ViT blocks ->
DPT head -> depth maps. `value` times steps with inputs resident in HBM; `e2e` times the
same call with pinned host buffers (H2D of the images and D2H of the depth maps inside
the timed region). The L2 (126 MB) is flushed between timed steps by writing a 256 MB
buffer outside the timed events.

--impl reference times the CPU restatement of the reference (oracle/) on the host
cores instead (rank 0 only).
"""
from __future__ import annotations

import argparse
import json
import os
import platform
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "images/s ViT-L Q8_0 518² at 1/2/4/8 B200; GEMM/conv % of tensor-core peak"
UNIT = "images/s"

# name -> (model, units, views per unit, H = W, stress GGUF, model FLOP per unit, description)
WORKLOADS = {
    "c3": ("da2-l", 64, 1, 518, True, 1304e9,
           "C3: DA2-L ViT-L/14 Q8_0 + DPT head, 64 images 518x518 sharded 64/N"),
    "c4": ("da3-l", 16, 8, 504, True, 15.15e12,
           "C4: DA3-L multi-view, 16 scenes x 8 views 504x504 sharded by scene, depth + confidence"),
    "c2": ("da2-b", 1, 1, 518, True, 381e9, "C2: DA2-B ViT-B/14 Q8_0 + DPT head, batch 1 518x518 per GPU"),
}


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def profiled_traffic(name):
    """DRAM bytes per launch (read + write) recorded in profiles/<name>: the line
    'dram_bytes_per_launch: <int>' of an ncu summary; None when absent."""
    try:
        with open(os.path.join(ROOT, "profiles", name)) as f:
            for ln in f:
                if ln.startswith("dram_bytes_per_launch:"):
                    return int(ln.split(":", 1)[1].split()[0])
    except (OSError, ValueError):
        pass
    return None


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


def workload(args):
    return WORKLOADS[args.workload]


def units_for(args, rank, world):
    """This rank's slice of the workload: (images [V][H][W][3], units, views per unit)."""
    from da3cpplib_b200 import shard, synth

    model, total, vps, hw, _, _, _ = workload(args)
    if args.workload == "c2":
        first, end = rank, rank + 1  # one image per GPU (replicas)
    else:
        first, end = shard.shard_range(total, world, rank)
    imgs = np.stack([synth.image(synth.IMAGE_SEED, i, hw, hw) for i in range(first * vps, end * vps)])
    return imgs, end - first, vps


def model_path(args, rank, world):
    from da3cpplib_b200 import synth

    model, _, _, _, stress, _, _ = workload(args)
    path = None
    if rank == 0:
        path = synth.ensure_gguf(model, stress=stress)
    if world > 1:
        import torch.distributed as dist

        obj = [path]
        dist.broadcast_object_list(obj, src=0)
        path = obj[0]
    return path


# ---------------------------------------------------------------------- reference arm
ORACLE_NOTE = ("CPU restatement of the reference's ggml CPU path (oracle/: Q8_0 activation quantisation with "
               "int8 block dots, f32 flash attention, direct f32 convs; AVX2, OpenMP over all host threads), not "
               "ggml itself: the reference's ggml submodule is absent from its checkout")


def cpu_time_images(model, hw, n_images, runs, stress=True, views=1, warm=True):
    """Median seconds per image (or per scene when views > 1) of the oracle over `runs`
    runs of n_images images (scenes) each, after one warm-up unit when `warm`; returns
    (median s/unit, all run times)."""
    from da3cpplib_b200 import synth
    from oracle.oracle import Oracle

    path = synth.ensure_gguf(model, stress=stress)
    orc = Oracle(path, act_quant=True, n_threads=os.cpu_count() or 1)

    def one(i):
        if views > 1:
            orc.infer_mv([synth.image(synth.IMAGE_SEED, i * views + v, hw, hw) for v in range(views)], legacy=True)
        else:
            orc.infer(synth.image(synth.IMAGE_SEED, i, hw, hw))

    if warm:
        one(0)
    times = []
    for r in range(runs):
        t0 = time.perf_counter()
        for i in range(n_images):
            one(r * n_images + i)
        times.append((time.perf_counter() - t0) / n_images)
    return statistics.median(times), times


def run_reference(args):
    world, rank, local = dist_setup(args)
    if rank != 0:
        return 0
    cores = os.cpu_count() or 1
    model, total, vps, hw, stress, flops, desc = workload(args)
    steps = max(args.steps, 3)
    per_unit, times = cpu_time_images(model, hw, 1, steps, stress, views=vps, warm=vps == 1)
    value = 1.0 / per_unit
    unit_name = "scene" if vps > 1 else "image"
    line = {
        "metric": METRIC, "value": value, "unit": UNIT if vps == 1 else "scenes/s", "n_gpus": args.gpus,
        "steps": steps, "warmup": 1, "ms_per_step": per_unit * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8xint8->f32 (Q8_0), f32", "data": "synthetic",
        "config": {"workload": f"{desc}; CPU: 1 {unit_name} per step, median of {steps} steps",
                   "model": model, "global_batch": 1, "parallelism": "cpu"},
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": UNIT if vps == 1 else "scenes/s", "cores": cores, "kind": "port",
                         "cpu": cpu_model(), "gflops": round(flops / per_unit / 1e9, 1),
                         "sample": f"1 {unit_name} per step, median of {steps} steps ({ORACLE_NOTE})"},
        "e2e": {"value": value, "unit": UNIT if vps == 1 else "scenes/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
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

    model_name, total, vps, hw, stress, flops_unit, desc = workload(args)
    H = W = hw
    path = model_path(args, rank, world)
    model = Model(path, local)
    imgs, per, _ = units_for(args, rank, world)
    V = per * vps                      # views (images) this rank runs per step
    units_total = world if args.workload == "c2" else total
    want_conf = model.output_dim >= 2
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream
    rgb_dev = torch.from_numpy(imgs).cuda()
    depth_dev = torch.empty((V, H, W), dtype=torch.float32, device="cuda")
    conf_dev = torch.empty((V, H, W), dtype=torch.float32, device="cuda") if want_conf else None
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")

    def step(rgb_ptr, depth_ptr, conf_ptr):
        model.infer_device(rgb_ptr, V, H, W, depth_ptr, conf_ptr=conf_ptr, views_per_scene=vps, stream=sptr)
        if args.gather and dist and depth_ptr == depth_dev.data_ptr():
            # optional NCCL gather of the depth maps to rank 0 (equal-sized slabs)
            from da3cpplib_b200 import shard

            shard.gather_to_rank0(depth_dev.view(per, vps, H, W), units_total)

    dev_ptrs = (rgb_dev.data_ptr(), depth_dev.data_ptr(), conf_dev.data_ptr() if want_conf else None)
    # warm-up (plan creation, graph capture)
    for _ in range(max(args.warmup, 3)):
        step(*dev_ptrs)
    torch.cuda.synchronize()
    launches = model.launches(V, H, W, views_per_scene=vps)

    def timed(ptrs):
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        for i in range(args.steps):
            flush.fill_(float(i))
            starts[i].record(stream)
            step(*ptrs)
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
        ms_step = timed(dev_ptrs)
    clocks = clk.summary()
    st = model.lib.da3b_device_status()
    if st != 0:
        raise RuntimeError(f"device status {st} after the timed region")
    value = units_total / (ms_step / 1e3)

    # e2e: pinned host in / out through the same public call
    rgb_host = torch.from_numpy(imgs).pin_memory()
    depth_host = torch.empty((V, H, W), dtype=torch.float32).pin_memory()
    conf_host = torch.empty((V, H, W), dtype=torch.float32).pin_memory() if want_conf else None
    host_ptrs = (rgb_host.data_ptr(), depth_host.data_ptr(), conf_host.data_ptr() if want_conf else None)
    step(*host_ptrs)
    torch.cuda.synchronize()
    ms_e2e = timed(host_ptrs)
    views_total = units_total * vps
    e2e = {"value": units_total / (ms_e2e / 1e3), "unit": UNIT if vps == 1 else "scenes/s",
           "h2d_bytes_per_step": int(views_total * H * W * 3),
           "d2h_bytes_per_step": int(views_total * H * W * 4 * (2 if want_conf else 1))}
    # sanity: the host result equals the device-resident result
    if not torch.equal(depth_host, depth_dev.cpu()):
        raise RuntimeError("e2e and device-resident outputs differ")

    hbm, tflops, src = peaks()
    Vp = ctypes.c_void_p
    tokens = 1 + (H // 14) * (W // 14)

    def event_ms(fn, reps=20):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    # live roofline of the dominant kernel: the fc1 GEMM of this workload timed alone
    M, K, N = V * tokens, model.embed_dim, 4 * model.embed_dim
    A = torch.randn(M, K, device="cuda").half()
    Wt = (torch.randn(N, K, device="cuda") * 0.02).half()
    bias = torch.zeros(N, device="cuda")
    out = torch.empty(M, N, dtype=torch.float16, device="cuda")

    def gemm():
        rc = model.lib.da3b_linear_f16(Vp(A.data_ptr()), M, K, K, Vp(Wt.data_ptr()), N, K, Vp(bias.data_ptr()), 2,
                                       Vp(out.data_ptr()), N, Vp(sptr))
        assert rc == 0

    gemm_ms = event_ms(gemm)
    achieved = 2.0 * M * K * N / (gemm_ms / 1e3) / 1e12
    algo_bytes = int(2 * (M * K + K * N + M * N))
    traffic = profiled_traffic(f"gemm_fc1_m{M}_k{K}_n{N}_traffic.txt")
    roofline = {"bound": "tensor", "achieved": round(achieved, 1), "peak": tflops, "unit": "TFLOP/s",
                "frac": round(achieved / tflops, 4), "traffic": traffic,
                "traffic_note": (f"ncu dram__bytes_read.sum + dram__bytes_write.sum of this launch shape "
                                 f"(profiles/gemm_fc1_m{M}_k{K}_n{N}_traffic.txt)") if traffic else
                                "no ncu capture of this launch shape in profiles/",
                "algorithmic_bytes": algo_bytes,
                "kernel": f"k_tc_gemm2 fc1 M={M} K={K} N={N} (+bias, erf-GELU), {src} bf16 dense peak (burst)",
                "ms_per_launch": round(gemm_ms, 4)}
    del A, Wt, out

    # second entry: the flash-attention kernel alone at this workload's local-attention shape
    heads = model.num_heads
    qkv = (torch.randn(V * tokens, 3 * heads * 64, device="cuda") * 1.5).half()
    ld = (tokens + 7) // 8 * 8
    vt = torch.empty(V * heads * 64 * ld, dtype=torch.float16, device="cuda")
    ao = torch.empty(V * tokens, heads * 64, dtype=torch.float16, device="cuda")
    assert model.lib.da3b_transpose_v(Vp(qkv.data_ptr()), V, tokens, heads, Vp(vt.data_ptr()), ld, Vp(sptr)) == 0

    def attn():
        rc = model.lib.da3b_attention_vt(Vp(qkv.data_ptr()), Vp(vt.data_ptr()), ld, V, tokens, heads,
                                         Vp(ao.data_ptr()), Vp(sptr))
        assert rc == 0

    attn_ms = event_ms(attn)
    attn_flops = 4.0 * V * tokens * tokens * heads * 64
    attn_ach = attn_flops / (attn_ms / 1e3) / 1e12
    attn_traffic = profiled_traffic(f"attn_v{V}_t{tokens}_h{heads}_traffic.txt")
    roofline_attn = {"bound": "tensor", "achieved": round(attn_ach, 1), "peak": tflops, "unit": "TFLOP/s",
                     "frac": round(attn_ach / tflops, 4), "traffic": attn_traffic,
                     "algorithmic_bytes": int(V * tokens * heads * 64 * 2 * 4),
                     "kernel": f"k_attn_tc {V} x {tokens} tokens, {heads} heads (QK^T and PV), {src} bf16 dense peak",
                     "ms_per_launch": round(attn_ms, 4)}
    del qkv, vt, ao
    if model.lib.da3b_device_status() != 0:
        raise RuntimeError("device status set by the roofline kernels")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # an 8-view scene is about 10 images of CPU work: one run, no warm-up, keeps the
        # sample bounded
        runs, warm = (1, False) if vps > 1 else (3, True)
        per_unit, times = cpu_time_images(model_name, hw, 1, runs, stress, views=vps, warm=warm)
        cpu = {"value": round(1.0 / per_unit, 4), "unit": UNIT if vps == 1 else "scenes/s",
               "cores": os.cpu_count() or 1, "kind": "port", "cpu": cpu_model(),
               "gflops": round(flops_unit / per_unit / 1e9, 1),
               "sample": (f"median of {runs} run(s) of 1 {'scene' if vps > 1 else 'image'} of this workload"
                          f"{' after one warm-up' if warm else ''} ({ORACLE_NOTE})"),
               "run_s": [round(t, 2) for t in times]}
        if args.workload == "c3":
            c1, c1t = cpu_time_images("da2-s", 518, 1, 3, True)
            cpu["c1_images_per_s"] = round(1.0 / c1, 3)
            cpu["c1_note"] = "C1 (DA2-S 518x518, the designated CPU config): median of 3 single-image runs"

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT if vps == 1 else "scenes/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3), "higher_is_better": True,
            "scaling": "weak" if args.workload == "c2" else "strong",
            "vs_baseline": None, "dtype": "f16 (Q8_0 weights dequantised to f16, f32 accumulate)",
            "data": "synthetic (seeded uniform RGB8, random-init Q8_0 GGUF)",
            "config": {"workload": desc, "model": model_name, "global_batch": units_total * vps,
                       "per_gpu_batch": V, "views_per_scene": vps, "seq_len": tokens, "parallelism": f"dp{world}",
                       "gather": "depth maps to rank 0 over NCCL each step" if (args.gather and world > 1) else "none",
                       "l2": "flushed (256 MB write) between timed steps"},
            "e2e": {k: (round(v, 2) if isinstance(v, float) else v) for k, v in e2e.items()},
            "roofline": roofline,
            "roofline_attention": roofline_attn,
            "model_tflops": round(flops_unit * units_total / (ms_step / 1e3) / 1e12, 1),
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
    ap.add_argument("--workload", default="c3", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--gather", action="store_true",
                    help="N>1: gather every step's depth maps to rank 0 over NCCL inside the timed region")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
