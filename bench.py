#!/usr/bin/env python3
"""Throughput benchmark of the B200 RF-DETR engine.

Headline workload: RF-DETR Base, Q8_0 weights, batch 64 per GPU (the metric's
batch), 560 x 560 uniform-uint8 images (seeded), random-init weights written by
the repository's GGUF writer (same bytes as the reference converter).  One
step = one forward pass of the whole batch: GPU preprocess -> windowed DINOv2
backbone -> projector -> two-stage + top-K -> deformable decoder -> heads.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs one process per GPU (torchrun); each rank processes its own batch
(weak scaling, no collective on the data path); timing is the max over ranks.

The same JSON line carries a `strong_scaling` object: RF-DETR Large, F16
weights, 704 x 704, one global batch of 256 images split contiguously over the
N ranks (256 / N per GPU), timed the same way (device-resident and end to
end), with each rank's host -> device upload time of its share.

Reported (one JSON line on rank 0):
  value       images/s, inputs already resident in HBM (device pointer API)
  e2e         images/s through rfdetr_b200_submit_rgb / rfdetr_b200_wait with pinned host
              inputs and outputs (H2D + forward + D2H inside the timed region)
  p50_batch1_ms  median rfdetr_detect latency, one image, end to end
  roofline    backbone GEMM launches (the dominant kernel) vs measured peak
  cpu_baseline  the CPU oracle (a restatement of the reference forward) on
              this host's cores, on a bounded sample
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "rf-detr.cpp_b200"))

METRIC = "images/sec per GPU and whole box (1/2/4/8 B200) at batch 64; p50 batch-1 ms"
WORKLOAD = {"variant": "base", "dtype": "q8_0", "batch": 64, "image": 560}
STRONG = {"variant": "large", "dtype": "f16", "global_batch": 256}
L2_NOTE = "256 MB buffer written between timed steps (L2 is 126 MB)"
# The reference's own published CPU latency for the headline model (ggml, batch 1, 8 threads).
PUBLISHED_CPU = {"model": "base/q8_0", "median_ms": 145.7, "images_per_s": round(1000.0 / 145.7, 3),
                 "cpu": "AMD Ryzen 9 9950X3D", "threads": 8,
                 "source": "benchmarks/results/per_cell_latency.json"}


def parse(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--variant", default=WORKLOAD["variant"])
    p.add_argument("--dtype", default=WORKLOAD["dtype"])
    p.add_argument("--batch", type=int, default=WORKLOAD["batch"])
    p.add_argument("--global-batch", type=int, default=0,
                   help="split this many images over the ranks (strong scaling) instead of --batch per rank")
    p.add_argument("--strong-batch", type=int, default=STRONG["global_batch"],
                   help="global batch of the strong-scaling leg (0 = skip the leg)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args(argv)


def model_file(variant, dtype, pg):
    from rfdetr_b200 import replicas, synth
    d = os.environ.get("RFDETR_BENCH_DIR", os.path.join(tempfile.gettempdir(), "rfdetr_bench"))
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, f"{variant}-{dtype}-seed0.gguf")
    return replicas.create_once(path, lambda tmp: synth.write_model(tmp, variant, dtype, 0), pg)


def headline_config(args, world):
    """The `config` object of the line; the reference arm prints the same one."""
    from rfdetr_b200 import synth
    S = synth.get_variant(args.variant)["image_size"]
    if args.global_batch > 0:
        total = args.global_batch
        per = f"global batch {total} split over {world} GPU(s)"
    else:
        total = args.batch * world
        per = f"batch {args.batch} per GPU"
    return {"workload": f"RF-DETR {args.variant} {args.dtype}, {per}, {S}x{S} uint8 images",
            "global_batch": total, "per_gpu_batch": args.batch if args.global_batch <= 0 else None,
            "image": S, "parallelism": f"dp{world} (independent replicas)", "l2": L2_NOTE}


def smi_device(local):
    """nvidia-smi's name for this rank's GPU: its entry of CUDA_VISIBLE_DEVICES (an index or a UUID,
    both accepted by `nvidia-smi -i`) when that is set, else the local rank."""
    vis = [x.strip() for x in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if x.strip()]
    return vis[local] if local < len(vis) else str(local)


class Clocks:
    """nvidia-smi sampling around the timed region.  The sampler is started
    before the warm-up and waited for (bounded) until its first sample, so a
    short timed region on a busy host still gets samples."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def start(self, wait_first_s=5.0):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
            return
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < wait_first_s and self.p.poll() is None:
            if os.path.getsize(self.f.name) > 0:
                break
            time.sleep(0.02)

    def stop(self):
        if self.p:
            self.p.terminate()
            try:
                self.p.wait(5)
            except subprocess.TimeoutExpired:
                self.p.kill()
        self.f.flush()
        rows = []
        with open(self.f.name) as fh:
            for line in fh:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1])]
        smmax = num(rows[0][2])
        loaded = [s for s in sm if smmax and s > 0.3 * smmax] or sm
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": smmax,
                "reasons": sorted(reasons), "samples": len(rows)}


def backbone_gemm_flops(cfg, batch):
    """Algorithmic FLOPs of the backbone linear launches of one forward."""
    S, p, nw = cfg["image_size"], cfg["patch_size"], cfg["backbone"]["num_windows"]
    G = S // p
    ws = G // nw
    ntok = nw * nw * (ws * ws + 1)
    D, F = cfg["backbone"]["dim"], cfg["backbone"]["ffn_dim"]
    M = batch * ntok
    return {"qkv": 2 * M * D * 3 * D, "proj": 2 * M * D * D, "fc1": 2 * M * D * F, "fc2": 2 * M * F * D}


def backbone_gemm_bytes(cfg, batch):
    """Algorithmic HBM bytes of the same launches: each f16 operand read once, each output
    written once; the residual linears (proj, fc2) read and write the f32 residual stream."""
    S, p, nw = cfg["image_size"], cfg["patch_size"], cfg["backbone"]["num_windows"]
    G = S // p
    ws = G // nw
    ntok = nw * nw * (ws * ws + 1)
    D, F = cfg["backbone"]["dim"], cfg["backbone"]["ffn_dim"]
    M = batch * ntok
    return {"qkv": 2 * (M * D + 3 * D * D + M * 3 * D),
            "proj": 2 * (M * D + D * D) + 8 * M * D,
            "fc1": 2 * (M * D + F * D + M * F),
            "fc2": 2 * (M * F + D * F) + 8 * M * D}


def gemm_parts(fl, by, g_ms, g_n, hbm_gbs, tf_peak):
    """Per-linear figures of one profiled forward: time, TFLOP/s and GB/s against the
    tensor and HBM peaks, and which of the two bounds the launch (the larger of
    FLOPs / tensor peak and bytes / HBM peak).  `own_bound_frac` is the sum over launches
    of that bound's time divided by their measured time."""
    parts, t_bound, t_meas = {}, 0.0, 0.0
    for k in fl:
        n, ms = g_n.get(k, 0), g_ms.get(k, 0.0)
        if n == 0 or ms <= 0:
            continue
        t_t = fl[k] * n / (tf_peak * 1e12) * 1e3
        t_h = by[k] * n / (hbm_gbs * 1e9) * 1e3
        parts[k] = {"launches": n, "ms": round(ms, 4),
                    "tflops": round(fl[k] * n / (ms / 1e3) / 1e12, 1),
                    "frac_tensor": round(t_t / ms, 4),
                    "gbs": round(by[k] * n / (ms / 1e3) / 1e9, 1),
                    "frac_hbm": round(t_h / ms, 4),
                    "bound": "tensor" if t_t >= t_h else "hbm"}
        t_bound += max(t_t, t_h)
        t_meas += ms
    return parts, (round(t_bound / t_meas, 4) if t_meas > 0 else None)


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        return m["hbm_gbs"], m["bf16_tflops"], m.get("bf16_tflops_sustained", m["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, 1400.0, "fallback"


def traffic_from_profiles():
    """Per-launch DRAM bytes of the profiled backbone GEMM (ncu capture summary)."""
    try:
        with open(os.path.join(REPO, "profiles", "gemm_traffic.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return None


def host_threads():
    """Cores this process may run on (torchrun pins OMP_NUM_THREADS to 1 per
    rank, so the CPU legs set their thread count explicitly)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def cpu_oracle_run(path, n_images, seed, time_budget_s=None, threads=None):
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import numpy as np
    import oracle as O
    ora = O.Oracle(path)
    S = ora.image_size
    rng = np.random.default_rng(seed)
    nt = threads or host_threads()
    done = 0
    t0 = time.perf_counter()
    while done < n_images:
        img = rng.integers(0, 256, (S, S, 3), dtype=np.uint8)
        ora.forward(ora.preprocess(img), n_threads=nt)
        done += 1
        if time_budget_s and time.perf_counter() - t0 > time_budget_s:
            break
    return done, time.perf_counter() - t0


def run_reference(args):
    """CPU arm: the reference cannot be built here (its ggml submodule is not
    vendored), so its restated algorithm (the oracle) runs on the host cores,
    one image of the headline batch per step (a bounded sample)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    if rank != 0:
        return 0
    from rfdetr_b200 import replicas
    path = model_file(args.variant, args.dtype, replicas.ProcessGroup(replicas.RankInfo()))
    cores = host_threads()
    cpu_oracle_run(path, max(args.warmup, 0), 7, threads=cores)
    n, dt = cpu_oracle_run(path, max(args.steps, 1), 11, threads=cores)
    v = n / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "images/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / n * 1000, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded uint8 images, seeded random-init weights)",
        "config": headline_config(args, world),
        "cpu_baseline": {"value": round(v, 4), "unit": "images/s", "cores": cores, "kind": "port",
                         "cpu_model": cpu_model(), "nproc": os.cpu_count(),
                         "sample": f"{n} images (one per step) of the workload's batch, restated reference "
                                   f"forward (f32 activations x dequantized weights), OpenMP over {cores} threads"},
        "published": PUBLISHED_CPU,
        "e2e": {"value": round(v, 4), "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


class Leg:
    """One engine context with its images: the device-resident and the end-to-end
    timings of one workload on this rank."""

    def __init__(self, path, local, lo, B, S):
        import numpy as np
        import torch
        from rfdetr_b200 import lib
        self.B, self.S, self.local = B, S, local
        self.eng = lib.Engine(path, device=local, max_batch=B)
        self.stream = torch.cuda.ExternalStream(self.eng.stream(), device=torch.device("cuda", local))
        # image i of the (global) batch is drawn from seed 1000 + i, whatever rank owns it
        self.imgs = np.stack([np.random.default_rng(1000 + lo + i).integers(0, 256, (S, S, 3), dtype=np.uint8)
                              for i in range(B)])
        self.d_imgs = torch.from_numpy(self.imgs).cuda(local)

    def device(self, steps, warmup, flush, pg, clocks=None):
        """Summed device ms of `steps` forwards from device-resident images, max over ranks."""
        import torch
        eng, B, S = self.eng, self.B, self.S
        with torch.cuda.stream(self.stream):
            if clocks:
                clocks.start()
            for _ in range(warmup):
                eng.enqueue_device(self.d_imgs.data_ptr(), B, S, S)
            eng.sync()
            starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
            ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
            pg.barrier()
            torch.cuda.synchronize()
            for i in range(steps):
                flush.zero_()  # L2 flush (256 MB > 126 MB L2), outside the timed interval
                starts[i].record(self.stream)
                eng.enqueue_device(self.d_imgs.data_ptr(), B, S, S)
                ends[i].record(self.stream)
            eng.sync()
            torch.cuda.synchronize()
            clk = clocks.stop() if clocks else None
            pg.barrier()
        ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
        return pg.max_over_ranks(ms), clk

    def e2e(self, steps, warmup, pg):
        """ms of `steps` pipelined submissions from pinned host images into pinned host
        outputs (rfdetr_b200_submit_rgb / rfdetr_b200_wait), max over ranks; bytes per step."""
        import torch
        from rfdetr_b200 import lib
        eng, B, S = self.eng, self.B, self.S
        # every step uploads its images from host memory and downloads its logits and boxes into
        # host memory; the upload of step i+1 and the download of step i-1 overlap the forward of
        # step i.  The outputs are not read here, so two alternating host buffers suffice (a caller
        # reading them gives each submission of a group its own buffers and reads after the wait).
        h_imgs = torch.empty((B, S, S, 3), dtype=torch.uint8, pin_memory=True)
        h_imgs.numpy()[:] = self.imgs
        h_np = h_imgs.numpy()
        nq, nc = eng.nq, eng.nc
        h_lg = [torch.empty((B, nq, nc), dtype=torch.float32, pin_memory=True).numpy() for _ in range(2)]
        h_bx = [torch.empty((B, nq, 4), dtype=torch.float32, pin_memory=True).numpy() for _ in range(2)]
        L = lib.lib()

        def call(i):
            lib.check(L.rfdetr_b200_submit_rgb(eng.ctx, C.c_void_p(h_np.ctypes.data), B, S, S,
                                               C.c_void_p(h_lg[i & 1].ctypes.data),
                                               C.c_void_p(h_bx[i & 1].ctypes.data), None), "submit_rgb")

        for i in range(warmup):
            call(i)
        lib.check(L.rfdetr_b200_wait(eng.ctx), "wait")
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        pg.barrier()
        torch.cuda.synchronize()
        e0.record(self.stream)
        for i in range(steps):
            call(i)
        # the downloads run on the context's own transfer stream: the end event goes on the engine
        # stream after rfdetr_b200_wait, so the last step's download is inside the timed region
        lib.check(L.rfdetr_b200_wait(eng.ctx), "wait")
        e1.record(self.stream)
        torch.cuda.synchronize()
        pg.barrier()
        ms = pg.max_over_ranks(e0.elapsed_time(e1))
        return ms, B * S * S * 3, B * nq * (nc + 4) * 4, h_imgs

    def upload(self, h_imgs, steps, pg):
        """Mean ms of one host -> device copy of this rank's images from pinned memory
        (all ranks copying at the same time), gathered on rank 0."""
        import torch
        dst = torch.empty_like(self.d_imgs)
        s = torch.cuda.Stream(device=self.local)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        pg.barrier()
        torch.cuda.synchronize()
        with torch.cuda.stream(s):
            dst.copy_(h_imgs, non_blocking=True)  # warm-up
            ev[0].record(s)
            for _ in range(steps):
                dst.copy_(h_imgs, non_blocking=True)
            ev[1].record(s)
        torch.cuda.synchronize()
        pg.barrier()
        return pg.gather_to_rank0(ev[0].elapsed_time(ev[1]) / steps)

    def close(self):
        self.eng.close()


def strong_leg(args, rank, world, local, pg, flush):
    """RF-DETR Large F16, one global batch split contiguously over the ranks."""
    from rfdetr_b200 import replicas, synth
    total = args.strong_batch
    lo, hi = replicas.shard(total, rank, world)
    B = hi - lo
    S = synth.get_variant(STRONG["variant"])["image_size"]
    path = model_file(STRONG["variant"], STRONG["dtype"], pg)
    leg = Leg(path, local, lo, max(B, 1), S)
    warm = max(args.warmup, 3)
    dev_ms, _ = leg.device(args.steps, warm, flush, pg)
    e2e_ms, h2d, d2h, h_imgs = leg.e2e(args.steps, warm, pg)
    up = leg.upload(h_imgs, args.steps, pg)
    leg.close()
    shares = pg.gather_to_rank0(float(B))
    return {
        "workload": f"RF-DETR {STRONG['variant']} {STRONG['dtype']}, global batch {total} of {S}x{S} uint8 images "
                    f"split contiguously over {world} GPU(s)",
        "global_batch": total, "per_gpu_batch": [int(x) for x in shares] if shares else None,
        "steps": args.steps, "warmup": warm,
        "value": round(total * args.steps / (dev_ms / 1000.0), 2), "unit": "images/s",
        "ms_per_step": round(dev_ms / args.steps, 4),
        "e2e": {"value": round(total * args.steps / (e2e_ms / 1000.0), 2), "unit": "images/s",
                "ms_per_step": round(e2e_ms / args.steps, 4), "h2d_bytes_per_step_per_gpu": h2d,
                "d2h_bytes_per_step_per_gpu": d2h},
        "upload_ms_per_step": {"per_rank": [round(x, 4) for x in up] if up else None,
                               "max": round(max(up), 4) if up else None,
                               "what": "one pinned host -> device copy of the rank's images, all ranks at once"},
        "timing": "device: CUDA events around each forward, summed, max over ranks; e2e: events around the "
                  "pipelined submissions, max over ranks",
    }


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)

    import numpy as np
    import torch
    from rfdetr_b200 import lib, replicas, synth

    info = replicas.RankInfo.from_env()
    rank, world, local = info.rank, info.world, info.local_rank
    torch.cuda.set_device(local)
    pg = replicas.ProcessGroup(info, "nccl", timeout_s=300.0, device=torch.device("cuda", local))

    cfg = synth.get_variant(args.variant)
    S = cfg["image_size"]
    if args.global_batch > 0:
        lo, hi = replicas.shard(args.global_batch, rank, world)
        B, scaling, total = hi - lo, "strong", args.global_batch
        if B == 0:
            raise SystemExit("--global-batch smaller than the number of ranks")
    else:
        lo, B, scaling, total = rank * args.batch, args.batch, "weak", args.batch * world
    warm = max(args.warmup, 3)
    path = model_file(args.variant, args.dtype, pg)
    leg = Leg(path, local, lo, B, S)
    eng = leg.eng
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=f"cuda:{local}")
    torch.cuda.synchronize()

    # ---- device-resident throughput --------------------------------------
    ms_max, clk = leg.device(args.steps, warm, flush, pg, clocks=Clocks(smi_device(local)))
    value = total * args.steps / (ms_max / 1000.0)
    launches = eng.kernels_per_forward() * args.steps

    # ---- end to end through the C API (pinned host buffers) -------------
    e2e_ms, h2d, d2h, _ = leg.e2e(args.steps, warm, pg)
    e2e_value = total * args.steps / (e2e_ms / 1000.0)

    # ---- per-launch profile of one forward -> backbone GEMM roofline -----
    eng.profile_enable(True)
    with torch.cuda.stream(leg.stream):
        flush.zero_()
        eng.enqueue_device(leg.d_imgs.data_ptr(), B, S, S)
        eng.sync()
    prof = eng.profile_read()
    eng.profile_enable(False)
    fl = backbone_gemm_flops(cfg, B)
    g_ms = {k: 0.0 for k in fl}
    g_n = {k: 0 for k in fl}
    for name, t_ms in prof:
        if name in g_ms:
            g_ms[name] += t_ms
            g_n[name] += 1
    gemm_flops = sum(fl[k] * g_n[k] for k in fl)  # per launch actually made
    gemm_ms = sum(g_ms.values())
    total_ms = sum(t for _, t in prof)
    hbm, tf_burst, tf_sus, src = peaks()
    achieved = gemm_flops / (gemm_ms / 1000.0) / 1e12 if gemm_ms > 0 else None
    parts, own_frac = gemm_parts(fl, backbone_gemm_bytes(cfg, B), g_ms, g_n, hbm, tf_sus)
    tr = traffic_from_profiles()
    share = {}
    for name, t_ms in prof:
        share[name] = share.get(name, 0.0) + t_ms
    top = sorted(share.items(), key=lambda kv: -kv[1])[:8]

    # ---- p50 batch-1 latency through rfdetr_detect ----------------------
    p50 = None
    if rank == 0:
        L = lib.lib()
        st = C.c_int(0)
        one = np.ascontiguousarray(leg.imgs[0])
        img = L.rfdetr_image_from_rgb_buffer(C.c_void_p(one.ctypes.data), S, S, C.byref(st))
        dp = lib.DetectParams(0.5, 300, None, 0)
        outp = C.POINTER(lib.Detection)()
        n = C.c_size_t(0)
        lat = []
        for i in range(warm + args.steps):
            t0 = time.perf_counter()
            lib.check(L.rfdetr_detect(eng.ctx, img, C.byref(dp), C.byref(outp), C.byref(n)), "rfdetr_detect")
            t1 = time.perf_counter()
            L.rfdetr_detections_free(outp, n.value)
            if i >= warm:
                lat.append((t1 - t0) * 1000.0)
        L.rfdetr_image_free(img)
        p50 = statistics.median(lat)
    pg.barrier()
    leg.close()

    # ---- strong scaling: Large F16, global batch split over the ranks ---
    strong = strong_leg(args, rank, world, local, pg, flush) if args.strong_batch > 0 else None

    # ---- CPU baseline (rank 0, N = 1) ------------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cores = host_threads()
        n_img, dt = cpu_oracle_run(path, 8, 5, time_budget_s=20.0, threads=cores)
        cpu = {"value": round(n_img / dt, 4), "unit": "images/s", "cores": cores, "kind": "port",
               "cpu_model": cpu_model(), "nproc": os.cpu_count(),
               "sample": f"{n_img} images of the workload, restated reference forward (f32), "
                         f"OpenMP over {cores} threads",
               "published": PUBLISHED_CPU}

    if rank == 0:
        config = headline_config(args, world)
        config["per_gpu_batch"] = B
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "images/s", "n_gpus": world,
            "steps": args.steps, "warmup": warm, "ms_per_step": round(ms_max / args.steps, 4),
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded uint8 images, seeded random-init weights)",
            "config": config,
            "e2e": {"value": round(e2e_value, 2), "unit": "images/s", "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h * world},
            "p50_batch1_ms": round(p50, 3) if p50 is not None else None,
            "gpu_launches": launches,
            "roofline": {"kernel": "backbone linears: k_gemm qkv / proj / fc1 (+GELU) / fc2 launches",
                         "bound": "tensor",
                         "achieved": round(achieved, 1) if achieved else None,
                         "peak": tf_sus, "unit": "TFLOP/s",
                         "frac": round(achieved / tf_sus, 4) if achieved else None,
                         "peak_source": f"{src} bf16 sustained (kernel timed inside the forward)",
                         "traffic": tr.get("bytes_per_launch") if tr else None,
                         "timing": "per-launch CUDA events of one forward launched kernel by kernel outside "
                                   "the CUDA graph the timed steps replay (conservative)",
                         "gemm_ms": round(gemm_ms, 4), "forward_ms": round(total_ms, 4),
                         "gemm_share": round(gemm_ms / total_ms, 4) if total_ms else None,
                         "parts": parts,
                         "own_bound_frac": own_frac},
            "top_launches_ms": [[k, round(v, 4)] for k, v in top],
            "clocks": clk,
        }
        if strong:
            line["strong_scaling"] = strong
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    pg.barrier()  # rank 0's latency / CPU legs are done before any rank tears down
    pg.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
