"""Benchmark: YOLOv3-416 FP32 inference images/s on N B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

One step = one forward of the whole network over a batch of B images per GPU (default 8:
"batch 64 sharded over 8 GPUs").  Images are batch-partitioned across ranks with no data-path
collective (weak scaling).  Timing: W untimed steps, then K steps between a barrier +
synchronize on both sides, CUDA events on the launching stream, max over ranks.

  value       images/s over all ranks, inputs resident in HBM (graph replay of the forward)
  e2e         the same metric through StreamPredictor (TNNet.predict for a stream of batches):
              pinned-host input -> H2D, forward,
              D2H of the three yolo heads, every step
  roofline    the FP32 CUDA-core conv kernels: conv FLOPs of a forward / their summed device
              time (per-layer CUDA events), against the FFMA rate measured on this GPU
  cpu_baseline  the CPU oracle (restatement of the reference's CPU path) on this host's cores,
              on a bounded sample of images (rank 0, N = 1 only)

--impl reference times the reference's CPU algorithm (the oracle port; the FreePascal
reference cannot be built here) on the host cores with the same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

INPUT = (3, 416, 416)
HEADS = (82, 94, 106)
METRIC = "YOLOv3-416 images/sec (FP32 path)"
METRIC_TF32 = "YOLOv3-416 images/sec (TF32 tensor-core path)"
METRIC_BF16 = "YOLOv3-416 images/sec (BF16-split tensor-core path)"
MATH_MODES = {"fp32": 0, "tf32": 1, "fp32_tiled": 2, "bf16split": 3}
PROFILE_SUMMARY = ROOT / "profiles" / "conv_fp32_yolov3_b8.json"
PROFILE_SUMMARY_TF32 = ROOT / "profiles" / "k_conv_nhwc_yolov3_b8.json"


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [t.strip() for t in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(max(smax)), "samples": len(sm),
                "reasons": sorted(reasons)}


def host_threads():
    """Every host core this process may run on, whatever OMP_NUM_THREADS says (torchrun sets it
    to 1 for each rank)."""
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_baseline(specs, seconds=12.0, max_images=16):
    """The CPU oracle on this host's cores, one image at a time, for about `seconds`."""
    from oracle import oracle as O
    O.set_threads(host_threads())
    x = None
    n, t0 = 0, time.perf_counter()
    while n < max_images and (n == 0 or time.perf_counter() - t0 < seconds):
        from tensorium_b200 import synth
        x = synth.input_images(3, "yolov3", n + 1, INPUT)[n:n + 1]
        if n == 0:
            t0 = time.perf_counter()
        O.run_network(specs, x, keep=list(HEADS))
        n += 1
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "images/s", "cores": O.num_threads(), "kind": "port",
            "host_cores": os.cpu_count(), "cpu": cpu_model(),
            "sample": f"{n} YOLOv3-416 images at batch 1 (per-image oracle: im2col + k-ascending FMA "
                      f"SGEMM over rows, OpenMP, AVX2), {dt:.1f} s"}


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    from tensorium_b200 import synth
    from oracle import oracle as O
    O.set_threads(host_threads())
    specs = synth.yolov3_specs()
    xs = synth.input_images(3, "yolov3", 4, INPUT)
    for w in range(args.warmup):
        O.run_network(specs, xs[w % 4:w % 4 + 1], keep=list(HEADS))
    t0 = time.perf_counter()
    for k in range(args.steps):
        O.run_network(specs, xs[k % 4:k % 4 + 1], keep=list(HEADS))
    dt = time.perf_counter() - t0
    v = args.steps / dt
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "images/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * dt / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded uniform images, random He-init weights; no dataset or .weights in the container)",
            "config": {"workload": "YOLOv3-416 forward", "model": "yolov3-416", "input": "3x416x416",
                       "sample_per_step": "1 image (CPU)"},
            "e2e": {"value": v, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "cpu_baseline": {"value": v, "unit": "images/s", "cores": O.num_threads(), "kind": "port",
                             "host_cores": os.cpu_count(), "cpu": cpu_model(),
                             "sample": "1 YOLOv3-416 image per step through the CPU restatement of the "
                                       "reference path (the FreePascal reference cannot be built here)"}}
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch
    import torch.distributed as dist

    from tensorium_b200 import Context, synth
    from tensorium_b200.net import TNNet

    from tensorium_b200 import dist as tbd
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        tbd.init("nccl", timeout_s=300.0, device_id=torch.device("cuda", local))
    B = args.batch
    specs = synth.yolov3_specs()
    ctx = Context(local)
    net = TNNet(ctx, specs, B, INPUT, math_mode=MATH_MODES[args.math])
    # this rank's images: global images [rank*B, (rank+1)*B) of the seeded stream
    x_host = synth.input_images(3, "yolov3", (rank + 1) * B, INPUT)[rank * B:]
    x = torch.from_numpy(x_host).to(ctx.torch_device)
    stream = torch.cuda.current_stream(local)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        return tbd.max_over_ranks(v, device=ctx.torch_device)

    # ---- device-resident throughput (graph replay) ----
    for _ in range(max(args.warmup, 1)):
        net.forward(x)
    launches_per_step = net.launch_count
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with ClockSampler(local) as clk:
        if args.profile_window:
            torch.cuda.profiler.start()  # ncu --profile-from-start off captures only this region
        e0.record(stream)
        for _ in range(args.steps):
            net.forward(x, use_graph=not args.profile_window)
        e1.record(stream)
        barrier()
        if args.profile_window:
            torch.cuda.profiler.stop()
    ms = max_over_ranks(e0.elapsed_time(e1))
    clocks = clk.summary()
    value = world * B * args.steps / (ms / 1e3)

    # ---- end to end through the public API, every step: pinned host images -> H2D (upload stream,
    #      the next step's copy overlapping this step's forward) -> TNNet.forward (graph) -> GPU
    #      detection extraction -> NCCL gather of every rank's detections to rank 0 through the C
    #      ABI (tb_group_gather) -> D2H of the gathered detections on rank 0 ----
    h_in = torch.from_numpy(x_host).pin_memory()
    gat = tbd.DetectionGather(net, world, rank, capacity=4096, thresh=0.45, overlap=True)
    upload = torch.cuda.Stream(local)
    x_fixed = torch.empty_like(x)  # the forward's one input buffer (one CUDA graph)
    d_in = [torch.empty_like(x), torch.empty_like(x)]
    ev_h2d = [torch.cuda.Event(), torch.cuda.Event()]
    ev_free = [torch.cuda.Event(), torch.cuda.Event()]

    def upload_into(k, wait_free):
        with torch.cuda.stream(upload):
            if wait_free:
                upload.wait_event(ev_free[k])
            d_in[k].copy_(h_in, non_blocking=True)
            ev_h2d[k].record(upload)

    def e2e_steps(n):
        upload_into(0, False)
        for k in range(n):
            cur = k % 2
            stream.wait_event(ev_h2d[cur])
            x_fixed.copy_(d_in[cur])
            ev_free[cur].record(stream)
            if k + 1 < n:  # the next step's upload overlaps this step's forward
                upload_into(1 - cur, k >= 1)
            net.forward(x_fixed)
            gat.step(download=True)  # head snapshot here; extraction, gather, D2H on a side stream
        gat.join()  # the last step's detections are inside the timed region

    e2e_steps(max(args.warmup, 1))
    gat.wait()
    barrier()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gather_ms = []
    e0.record(stream)
    e2e_steps(args.steps)
    e1.record(stream)
    gat.wait()
    barrier()
    ms_e2e = max_over_ranks(e0.elapsed_time(e1))
    # the gather alone (device time of detection extraction + NCCL gather + D2H), max over ranks
    for _ in range(5):
        barrier()
        g0.record(stream)
        gat.step(download=True)
        gat.join()
        g1.record(stream)
        gat.wait()
        barrier()
        gather_ms.append(g0.elapsed_time(g1))
    gathered = gat.unpack()
    e2e = {"value": world * B * args.steps / (ms_e2e / 1e3), "unit": "images/s",
           "h2d_bytes_per_step": int(h_in.numel() * 4),
           "d2h_bytes_per_step": int(gat.d2h_bytes),
           "detect_and_gather_ms": max_over_ranks(float(np.median(gather_ms))),
           "gathered_on_rank0": {"images": len(gathered) if gathered is not None else None,
                                 "boxes": int(sum(len(r) for r in gathered)) if gathered is not None else None,
                                 "bytes": int(gat.d2h_bytes), "capacity_per_image": gat.capacity,
                                 "thresh": gat.thresh},
           "path": ("pinned host -> H2D (upload stream, overlapping the previous forward) -> TNNet.forward "
                    "(graph) -> device copy of the yolo outputs -> on a side stream, overlapping the next "
                    "forward: tb_yolo_detect_device -> tb_group_gather_async (NCCL, C ABI) of every rank's "
                    "records + counts to rank 0 -> D2H on rank 0; every step, the last step's tail inside "
                    "the timed region")}
    gat.close()

    # ---- roofline of the conv kernels (per-layer CUDA events, eager forward) ----
    prof = np.zeros(len(specs))
    for _ in range(3):
        prof += net.profile(x)
    prof /= 3
    conv_layers = [i for i, s in enumerate(specs) if s["type"] == "conv"]
    conv_ms = float(sum(prof[i] + (prof[i + 1] if i + 1 < len(specs) and specs[i + 1]["type"] in ("shortcut", "yolo") else 0.0)
                        for i in conv_layers))
    total_ms = float(prof.sum())
    conv_flops = synth.conv_flops(specs, INPUT, B)
    achieved = conv_flops / (conv_ms / 1e3) / 1e12
    traffic = None
    if PROFILE_SUMMARY.exists() and args.math == "fp32":
        traffic = json.loads(PROFILE_SUMMARY.read_text()).get("dram_bytes_per_forward")
    if args.math in ("fp32", "fp32_tiled"):
        fma = __import__("ctypes").c_double()
        from tensorium_b200._lib import check, lib
        check(lib.tb_diag_fp32_fma_tflops(ctx.handle, __import__("ctypes").byref(fma)))
        peak, bound, kernel = fma.value, "fp32", ("order-exact FP32 convs, bit-identical to the reference CPU path: "
                                                  "k_conv_slide (3x3 stride-1, input staged once) and k_conv_exact "
                                                  "(implicit GEMM) as the set-up autotuner picks them per geometry, "
                                                  "k_first_direct for the first layer")
        peak_source = ("FFMA rate measured in this run (tb_diag_fp32_fma_tflops); MEASURED_PEAKS.json holds HBM "
                       "and bf16 tensor peaks only")
    else:
        import ctypes as _C
        from tensorium_b200._lib import check, lib
        tc_rate, cyc = _C.c_double(), _C.c_double()
        check(lib.tb_diag_tc_mma_rate(ctx.handle, 1, _C.byref(tc_rate), _C.byref(cyc)))
        peak, bound = tc_rate.value, "tensor"
        kernel = ("k_conv_nhwc (tcgen05, A by TMA im2col, NHWC activations) for 74 convs "
                  "+ k_first_direct for the first layer (NHWC output)")
        peak_source = ("TF32 tcgen05 MMA rate measured in this run with operands resident (tb_diag_tc_mma_rate, "
                       "M=128 N=256 K=8, at the current SM clock); the BF16-split path issues twice the MMAs per "
                       "FLOP" if args.math == "bf16split" else
                       "TF32 tcgen05 MMA rate measured in this run with operands resident (tb_diag_tc_mma_rate, "
                       "M=128 N=256 K=8, at the current SM clock)")
    roofline = {"bound": bound, "kernel": kernel,
                "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "peak_source": peak_source,
                "traffic": traffic, "traffic_unit": "bytes per forward (ncu, summed over conv launches)",
                "algorithmic_flops_per_forward": conv_flops, "conv_ms_per_forward": conv_ms,
                "all_layers_ms_per_forward": total_ms,
                # the same FLOPs over the graph-replayed step (every layer, branch stream included)
                "frac_over_step": conv_flops / (ms / args.steps / 1e3) / 1e12 / peak}

    line = {"metric": {"fp32": METRIC, "tf32": METRIC_TF32, "bf16split": METRIC_BF16}.get(args.math, METRIC + " [" + args.math + "]"), "value": value, "unit": "images/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": {"fp32": "f32", "fp32_tiled": "f32", "tf32": "tf32 (fp32 accumulate)",
                      "bf16split": "bf16 (hi, lo) pairs (fp32 accumulate)"}[args.math],
            "data": "synthetic (seeded uniform images, random He-init weights, BN stats as config 0; "
                    "no dataset or .weights in the container)",
            "config": {"workload": "YOLOv3-416 forward (BASELINE config 3), batch 8 per GPU",
                       "model": "yolov3-416", "global_batch": world * B, "per_gpu_batch": B, "seq_len": None,
                       "input": "3x416x416", "parallelism": f"dp{world}",
                       "l2": "inputs larger than L2: each step streams ~1.3 GB of activations per GPU"},
            "e2e": e2e, "roofline": roofline, "clocks": clocks,
            "gpu_launches": int(launches_per_step * args.steps)}
    if args.math == "fp32" and not args.no_tf32_block:
        line["tf32_path"] = tf32_block(args, ctx, specs, x, net, world, barrier, max_over_ranks, stream)
        line["bf16split_path"] = tf32_block(args, ctx, specs, x, net, world, barrier, max_over_ranks, stream,
                                            mode="bf16split")
    if args.math == "fp32" and not args.no_configs:
        line["other_configs"] = configs_block(args, ctx, world, rank, barrier, max_over_ranks, stream, peak,
                                              cpu=(world == 1 and not args.no_cpu_baseline))
    if world == 1 and not args.no_kernel_suite:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
        mem, xnor = kernel_suite(ctx, peaks.get("hbm_gbs", 6650.0))
        line["memory_bound_kernels"] = mem
        line["xnor_conv"] = xnor
    if world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline(specs)
        cb["cpu"] = cpu_model()
        line["cpu_baseline"] = cb
    if rank == 0:
        print(json.dumps(line), flush=True)
    net.close()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def configs_block(args, ctx, world, rank, barrier, max_over_ranks, stream, fma_peak, cpu):
    """BASELINE configs 0, 1, 2, YOLOv3 at batch 1 and the XNOR sweep (config 4), each on the FP32
    path (bit-exact with the reference CPU path), timed like the headline (warm-up, CUDA events,
    max over ranks), with the conv FLOP roofline against the measured FFMA rate and, on rank 0 at
    N = 1, the CPU oracle on a bounded sample of the same workload."""
    import torch
    from tensorium_b200 import synth
    from tensorium_b200.layers import TConvolutionalLayer, TNNetState
    from tensorium_b200.net import TNNet
    from oracle import oracle as O
    if cpu:
        O.set_threads(host_threads())
    out = []

    def timed(fn, steps):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        barrier()
        return max_over_ranks(e0.elapsed_time(e1)) / steps

    def cpu_time(fn, min_s=2.0, max_reps=20):
        fn()
        t0, n = time.perf_counter(), 0
        while n < max_reps and (n == 0 or time.perf_counter() - t0 < min_s):
            fn()
            n += 1
        return (time.perf_counter() - t0) / n

    def entry(name, workload, items, unit, ms, flops, cpu_s=None, cpu_items=None, sample=None, extra=None):
        d = {"config": name, "workload": workload, "value": world * items / (ms / 1e3), "unit": unit,
             "ms_per_step": ms, "n_gpus": world,
             "roofline": {"bound": "fp32", "achieved": flops / (ms / 1e3) / 1e12, "peak": fma_peak,
                          "unit": "TFLOP/s", "frac": flops / (ms / 1e3) / 1e12 / fma_peak,
                          "note": "whole step time (every layer) against the measured FFMA rate"}}
        if cpu_s is not None:
            d["cpu_baseline"] = {"value": cpu_items / cpu_s, "unit": unit, "cores": O.num_threads(), "kind": "port",
                                 "sample": sample}
        if extra:
            d.update(extra)
        out.append(d)

    # config 0: one conv 3->32 3x3 + batchnorm (unfused, as TConvolutionalLayer.forward runs it) + leaky, 416x416
    s0 = synth.config0_spec()[0]
    L = TConvolutionalLayer(1, 416, 416, 3, 32, 1, 3, 1, 1, 1, 1, 9, True).bind(ctx)
    L.weights, L.biases = s0["weights"], s0["biases"]
    L.scales, L.rolling_mean, L.rolling_variance = s0["scales"], s0["mean"], s0["var"]
    x0h = synth.input_images(0, "cfg0", 1, (3, 416, 416))
    st0 = TNNetState(torch.from_numpy(x0h).to(ctx.torch_device))
    ms = timed(lambda: L.forward(st0), 200)
    cs = cpu_time(lambda: O.conv2d(x0h, s0["weights"], s0["biases"], 32, 3, 1, 1, 9,
                                   bn=(s0["scales"], s0["mean"], s0["var"]))) if cpu else None
    byts = (3 + 32) * 416 * 416 * 4
    entry("config0", "conv 3->32 3x3 s1 p1 + batchnorm + leaky on 1x3x416x416", 1, "layers/s", ms, 0.2990e9, cs, 1,
          "1 conv layer", {"hbm": {"bytes": byts, "achieved_gbs": byts / (ms / 1e3) / 1e9}})

    # config 1: MNIST-shaped CNN, batch 256 per GPU
    sp1 = synth.mnist_specs()
    net1 = TNNet(ctx, sp1, 256, (1, 28, 28))
    x1h = synth.input_images(1, "mnist", 256, (1, 28, 28))
    x1 = torch.from_numpy(x1h).to(ctx.torch_device)
    ms = timed(lambda: net1.forward(x1), 100)
    cs = cpu_time(lambda: O.run_network(sp1, x1h[:64], keep=[6])) if cpu else None
    f1 = synth.conv_flops(sp1, (1, 28, 28), 256) + 2 * 256 * (3136 * 1024 + 1024 * 10)
    entry("config1", "MNIST-shaped CNN (conv5x5x32, maxpool, conv5x5x64, maxpool, fc 3136-1024, fc 1024-10, softmax), "
          "batch 256 per GPU", 256, "images/s", ms, f1, cs, 64, "64 images through the oracle")
    net1.close()

    # config 2: CIFAR-shaped darknet CNN, batch 1024 sharded over the ranks
    per = 1024 // world
    sp2 = synth.cifar_specs()
    net2 = TNNet(ctx, sp2, per, (3, 32, 32))
    x2h = synth.input_images(2, "cifar", 1024, (3, 32, 32))[rank * per:(rank + 1) * per]
    x2 = torch.from_numpy(np.ascontiguousarray(x2h)).to(ctx.torch_device)
    ms = timed(lambda: net2.forward(x2), 20)
    cs = cpu_time(lambda: O.run_network(sp2, x2h[:8], keep=[11])) if cpu else None
    entry("config2", f"CIFAR-shaped darknet CNN, batch 1024 sharded over {world} GPU(s) ({per} per GPU)", per,
          "images/s", ms, synth.conv_flops(sp2, (3, 32, 32), per), cs, 8, "8 images through the oracle")
    net2.close()

    # config 3 at batch 1: YOLOv3-416 latency
    sp3 = synth.yolov3_specs()
    net3 = TNNet(ctx, sp3, 1, INPUT)
    x3 = torch.from_numpy(synth.input_images(3, "yolov3", 1, INPUT)).to(ctx.torch_device)
    ms = timed(lambda: net3.forward(x3), 50)
    entry("config3_batch1", "YOLOv3-416 forward, batch 1 per GPU (latency)", 1, "images/s", ms,
          synth.conv_flops(sp3, INPUT, 1), None, None, None,
          {"latency_ms": ms, "cpu_baseline_note": "the headline line's cpu_baseline is YOLOv3 at batch 1"})
    net3.close()
    return out


def tf32_block(args, ctx, specs, x, net32, world, barrier, max_over_ranks, stream, mode="tf32"):
    """The same forward on a tensor-core path (BASELINE config 3's optional path: TF32, or the
    BF16-split operands), timed the same way, with its head error against the FP32 path (which is
    bit-identical to the reference CPU path) on the same images."""
    import torch
    from tensorium_b200 import synth
    from tensorium_b200.net import TNNet
    B = args.batch
    net = TNNet(ctx, specs, B, INPUT, math_mode=MATH_MODES[mode])
    for _ in range(max(args.warmup, 1)):
        net.forward(x)
    launches = net.launch_count
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for _ in range(args.steps):
        net.forward(x)
    e1.record(stream)
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1))
    prof = np.zeros(len(specs))
    for _ in range(3):
        prof += net.profile(x)
    prof /= 3
    conv_ms = float(sum(prof[i] + (prof[i + 1] if i + 1 < len(specs) and specs[i + 1]["type"] in ("shortcut", "yolo") else 0.0)
                        for i, s in enumerate(specs) if s["type"] == "conv"))
    flops = synth.conv_flops(specs, INPUT, B)
    import ctypes as C
    from tensorium_b200._lib import check, lib
    tc_rate, cyc = C.c_double(), C.c_double()
    check(lib.tb_diag_tc_mma_rate(ctx.handle, 1, C.byref(tc_rate), C.byref(cyc)))
    achieved = flops / (conv_ms / 1e3) / 1e12
    # head error of the TF32 path against the FP32 path (relative L2 over the batch)
    net.forward(x)
    net32.forward(x)
    errs = []
    for h in HEADS:  # yolo outputs (the head convs are fused into them)
        a, b = net.output(h).double(), net32.output(h).double()
        errs.append(float(torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b)))
    is_bf = mode == "bf16split"
    out = {"metric": METRIC_BF16 if is_bf else METRIC_TF32, "value": world * B * args.steps / (ms / 1e3),
           "unit": "images/s", "ms_per_step": ms / args.steps,
           "dtype": ("bf16 (hi, lo) operand pairs, all four partial products, fp32 accumulate" if is_bf
                     else "tf32 operands rounded to nearest, fp32 accumulate"),
           "gpu_launches": int(launches * args.steps),
           "roofline": {"bound": "tensor", "kernel": ("k_conv_nhwc<PAIR> (tcgen05 kind::f16, 8 MMAs per 32 channels) "
                                                      if is_bf else "k_conv_nhwc (tcgen05 TF32, ") +
                                                     "A by TMA im2col, NHWC activations) + k_first_direct (first layer, "
                                                     "NHWC output) and NHWC upsample",
                        "achieved": achieved, "peak": tc_rate.value, "unit": "TFLOP/s",
                        "frac": achieved / tc_rate.value,
                        "peak_source": ("TF32 tcgen05 MMA rate measured in this run with operands resident "
                                        "(tb_diag_tc_mma_rate, M=128 N=256 K=8, at the current SM clock); the "
                                        "BF16-split path issues twice the MMAs of TF32 per FLOP, so its MMA-time "
                                        "fraction is twice this" if is_bf else
                                        "TF32 tcgen05 MMA rate measured in this run with operands resident "
                                        "(tb_diag_tc_mma_rate, M=128 N=256 K=8, at the current SM clock)"),
                        "conv_ms_per_forward": conv_ms,
                        "frac_over_step": flops / (ms / args.steps / 1e3) / 1e12 / tc_rate.value,
                        "traffic": (json.loads(PROFILE_SUMMARY_TF32.read_text()).get("dram_bytes_per_forward")
                                    if PROFILE_SUMMARY_TF32.exists() else None),
                        "traffic_unit": "bytes per forward (ncu, summed over every launch of one forward)"},
           "head_rel_l2_vs_fp32_path": errs, "heads": list(HEADS)}
    net.close()
    return out


def kernel_suite(ctx, hbm_gbs):
    """Each memory-bound layer kernel on its own, at a BASELINE shape scaled past the 126 MB L2
    (so every launch streams from HBM), and the XNOR conv over BASELINE config 4.  Bytes are the
    compulsory reads + writes of the kernel's logical inputs and outputs."""
    import ctypes as C
    import torch
    from tensorium_b200._lib import XNOR_PAD_BIT0, check, lib
    from tensorium_b200.context import ptr
    from tensorium_b200.layers import TXNORConvolutionLayer, TNNetState
    dev = ctx.torch_device
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timeit(fn, reps=20, warm=3):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    out = []

    def add(name, shape, nbytes, fn, ref):
        ms = timeit(fn)
        gbs = nbytes / (ms / 1e3) / 1e9
        out.append({"kernel": name, "replaces": ref, "shape": shape, "bytes": int(nbytes), "ms": ms,
                    "gb_s": gbs, "frac_of_measured_hbm": gbs / hbm_gbs})

    g = torch.Generator(device=dev)
    g.manual_seed(5)
    # maxpool 2x2/2, config 2 stage-1 shape [1024,128,32,32]
    x = torch.rand((1024, 128, 32, 32), device=dev, generator=g)
    y = torch.empty((1024, 128, 16, 16), device=dev)
    idx = torch.empty((1024, 128, 16, 16), dtype=torch.int64, device=dev)
    add("k_maxpool2x2", "1024x128x32x32 -> 16x16", x.numel() * 4 + y.numel() * 4,
        lambda: check(lib.tb_maxpool_fwd(ctx.handle, 1024, 128, 32, 32, 2, 2, 2, 0, ptr(x), ptr(y), None)),
        "TMaxPoolLayer.forwardMaxPool (source/nMaxPoolLayer.pas:363-463)")
    add("k_maxpool2x2 +argmax", "1024x128x32x32 -> 16x16, int64 indexes", x.numel() * 4 + y.numel() * 12,
        lambda: check(lib.tb_maxpool_fwd(ctx.handle, 1024, 128, 32, 32, 2, 2, 2, 0, ptr(x), ptr(y), ptr(idx))),
        "same, with indexes")
    del x, y, idx
    # upsample x2, YOLOv3 route-97 input [B,128,26,26] at B = 256
    x = torch.rand((256, 128, 26, 26), device=dev, generator=g)
    y = torch.empty((256, 128, 52, 52), device=dev)
    add("k_upsample2", "256x128x26x26 -> 52x52", x.numel() * 4 + y.numel() * 4,
        lambda: check(lib.tb_upsample_fwd(ctx.handle, 256, 128, 26, 26, 2, 1.0, ptr(x), ptr(y), 0)),
        "upsample (source/nupsamplelayer.pas:83-113)")
    del x, y
    # shortcut (unfused), 52x52x256 at B = 64
    a = torch.rand((64, 256, 52, 52), device=dev, generator=g)
    b = torch.rand_like(a)
    y = torch.empty_like(a)
    add("k_shortcut4", "64x256x52x52", a.numel() * 12,
        lambda: check(lib.tb_shortcut_fwd(ctx.handle, a.numel(), ptr(a), ptr(b), ptr(y), 9)),
        "TAddLayer.forward addvv + activate (source/naddlayer.pas:667-725)")
    # route (per-image concat, when not zero-copy): [64,256,26,26] + [64,512,26,26]
    r1 = a.view(-1)[: 64 * 256 * 676].view(64, 256 * 676)
    r2 = b.view(-1)[: 64 * 512 * 676].view(64, 512 * 676)
    yr = torch.empty((64, 768 * 676), device=dev)
    arr = (C.c_void_p * 2)(r1.data_ptr(), r2.data_ptr())
    sizes = (C.c_int64 * 2)(256 * 676, 512 * 676)
    add("k_copy_rows4 (route)", "64x(256+512)x26x26", yr.numel() * 8,
        lambda: check(lib.tb_route_fwd(ctx.handle, 64, 2, arr, sizes, ptr(yr), 1)),
        "TConcatLayer.forward / TTensor.concat (source/ntensors.pas:12045-12061)")
    # leaky activation in place
    add("k_activate (leaky)", "64x256x52x52", a.numel() * 8,
        lambda: check(lib.tb_activate(ctx.handle, a.numel(), ptr(a), 0, 9)),
        "activate_array (source/nactivation.pas:508-621)")
    del a, b, y, yr
    # yolo forward (unfused), [64, 3*85, 52, 52]
    x = torch.rand((64, 255, 52, 52), device=dev, generator=g)
    y = torch.empty_like(x)
    add("k_yolo", "64x255x52x52", x.numel() * 8,
        lambda: check(lib.tb_yolo_fwd(ctx.handle, 64, 3, 80, 52, 52, ptr(x), ptr(y), 1.0)),
        "TYoloLayer.forward (source/nyololayer.pas:786-825)")
    del x, y
    # input pipeline: 64 decoded full-HD RGB frames letterboxed into a 416x416 batch
    from tensorium_b200._lib import PIXEL_FPC, Image
    n_img, ih, iw = 64, 1080, 1920
    frames = torch.randint(0, 256, (n_img, ih, iw, 3), dtype=torch.uint8, device=dev, generator=g)
    xin = torch.empty((n_img, 3, 416, 416), device=dev)
    descs = (Image * n_img)(*[Image(frames[i].data_ptr(), iw, ih, iw * 3, 3, 0) for i in range(n_img)])
    nh = ih * 416 // iw
    hs = np.float32((ih - 1) / (nh - 1))
    iy = (np.arange(nh, dtype=np.float32) * hs).astype(np.int64)
    rows = set(iy.tolist()) | set((iy[:-1] + 1).tolist())  # the last row reads one source row
    add("k_images_to_tensor", f"{n_img}x{ih}x{iw}x3 u8 -> letterbox {n_img}x3x416x416",
        n_img * len(rows) * iw * 3 + xin.numel() * 4,
        lambda: check(lib.tb_images_to_tensor(ctx.handle, n_img, descs, 416, 416, 1, PIXEL_FPC, ptr(xin),
                                              0, None, None)),
        "TImageData.loadFromFile + letterBoxEx + toTensor (source/ntypes.pas:651-694,837-943), "
        "CPU-only in the reference; bytes = source rows the row pass reads + fp32 output")
    del frames, xin
    torch.cuda.empty_cache()

    # XNOR conv: C_in = C_out in {128..1024}, 3x3 s1 p1, batch 64; its
    # roofline is the measured xor+popcount+add rate of this GPU
    popc = C.c_double()
    check(lib.tb_diag_popc_tbitmac(ctx.handle, C.byref(popc)))
    xnor = [{"popc_peak_tbitmac_s": popc.value,
             "peak_source": "tb_diag_popc_tbitmac: register-resident xor+popcount+add on every SM, this run"}]
    rng = np.random.default_rng(4)
    for S in (52, 26, 13):
        for Cn in (128, 256, 512, 1024):
            L = TXNORConvolutionLayer(64, S, S, Cn, Cn, 3, 1, 1, "linear", XNOR_PAD_BIT0)
            L.upload(ctx, rng.standard_normal((Cn, Cn * 9)).astype(np.float32))
            xx = torch.randn((64, Cn, S, S), device=dev, generator=g)
            st = TNNetState(xx)
            ms = timeit(lambda: L.forward(st), reps=5, warm=2)
            bitmacs = Cn * (64 * S * S) * (Cn * 9)
            out_bytes = 64 * Cn * S * S * 4 * 2  # fp32 input read + output written
            xnor.append({"shape": f"{Cn}->{Cn} 3x3 at {S}x{S}, batch 64", "ms": ms,
                         "tbitmac_s": bitmacs / (ms / 1e3) / 1e12,
                         "frac_of_measured_popc_rate": bitmacs / (ms / 1e3) / 1e12 / popc.value,
                         "io_gb_s": out_bytes / (ms / 1e3) / 1e9})
            del L, xx, st
            torch.cuda.empty_cache()
    return out, xnor


def run_kernel_suite(args):
    from tensorium_b200 import Context
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    ctx = Context(0)
    mem, xnor = kernel_suite(ctx, peaks.get("hbm_gbs", 6650.0))
    print(json.dumps({"memory_bound_kernels": mem, "xnor_conv": xnor,
                      "hbm_peak_gb_s": peaks.get("hbm_gbs", 6650.0),
                      "peak_source": "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in peaks else "fallback 6650 GB/s"}))
    ctx.close()


def run_layer_mode(args):
    """Time one YOLOv3 conv layer (index args.layer) at batch args.batch through tb_conv2d_fwd:
    the small, self-contained case used for ncu captures and per-layer tuning."""
    import torch
    from tensorium_b200 import Context, synth
    from tensorium_b200.layers import TConvolutionalLayer, TNNetState
    specs = synth.yolov3_specs()
    shapes = synth.layer_shapes(specs, INPUT)
    i = args.layer
    s = specs[i]
    assert s["type"] == "conv", f"layer {i} is a {s['type']}"
    c, h, w = shapes[i - 1] if i > 0 else INPUT
    if args.shape:  # an arbitrary conv geometry C,H,F,k,stride (He-init weights)
        c, h, f, k, st = (int(v) for v in args.shape.split(","))
        w = h
        s = synth.conv_spec(5, "shape", c, f, k, st, k // 2, 9, False)
        specs = list(specs)
        specs[i] = s
        shapes = list(shapes)
        shapes[i] = (f, (h + 2 * (k // 2) - k) // st + 1, (w + 2 * (k // 2) - k) // st + 1)
    ctx = Context(0)
    L = TConvolutionalLayer(args.batch, h, w, c, s["filters"], 1, s["size"], s["stride"], s["stride"], 1,
                            s["pad"], s["activation"], False).bind(ctx)
    L.weights = s["weights"]
    x = torch.rand((args.batch, c, h, w), device=ctx.torch_device)
    st = TNNetState(x)
    mm = MATH_MODES[args.math]
    if args.nhwc:  # the NHWC tensor-core kernel (TF32) the TF32 network runs, through its C ABI
        import ctypes as C
        from tensorium_b200._lib import ConvDesc, check, lib
        from tensorium_b200.context import ptr
        oc, oh, ow = shapes[i]
        d = ConvDesc(args.batch, c, h, w, s["filters"], s["size"], s["size"], s["stride"], s["stride"], s["pad"],
                     s["pad"], 1, 1, s["activation"], 0, 0, 0)
        cnt = C.c_int64()
        check(lib.tb_conv_nhwc_packed_count(C.byref(d), C.byref(cnt)))
        wd = torch.from_numpy(np.ascontiguousarray(s["weights"])).to(ctx.torch_device)
        wp = torch.empty(cnt.value, device=ctx.torch_device)
        check(lib.tb_conv_pack_weights_nhwc(ctx.handle, C.byref(d), ptr(wd), ptr(wp)))
        xn = torch.rand((args.batch, h, w, c), device=ctx.torch_device)
        yn = torch.empty((args.batch, oh, ow, oc), device=ctx.torch_device)

        class _Nhwc:
            @staticmethod
            def forward(_st, math_mode=None):
                check(lib.tb_conv2d_fwd_nhwc(ctx.handle, C.byref(d), ptr(xn), c, ptr(wp), None, None, 0, ptr(yn), oc))
        L = _Nhwc
    for _ in range(args.warmup):
        L.forward(st, math_mode=mm)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if args.profile_window:
        torch.cuda.profiler.start()
    e0.record()
    for _ in range(args.steps):
        L.forward(st, math_mode=mm)
    e1.record()
    torch.cuda.synchronize()
    if args.profile_window:
        torch.cuda.profiler.stop()
    ms = e0.elapsed_time(e1) / args.steps
    oc, oh, ow = shapes[i]
    flops = 2.0 * oc * oh * ow * c * s["size"] ** 2 * args.batch
    print(json.dumps({"layer": i, "math": args.math + (" nhwc" if args.nhwc else ""), "shape": f"{c}x{h}x{w} -> {oc}x{oh}x{ow} k{s['size']} s{s['stride']}",
                      "batch": args.batch, "ms": ms, "tflops": flops / ms / 1e9}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batch", type=int, default=8, help="images per GPU per step")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-tf32-block", action="store_true", help="skip the TF32-path measurement of the default run")
    ap.add_argument("--no-kernel-suite", action="store_true", help="skip the memory-bound / XNOR kernel suite")
    ap.add_argument("--no-configs", action="store_true", help="skip BASELINE configs 0, 1, 2 and YOLOv3 batch 1")
    ap.add_argument("--suite", choices=["kernels"], default=None, help="run only the kernel suite")
    ap.add_argument("--layer", type=int, default=None, help="time one YOLOv3 conv layer only")
    ap.add_argument("--shape", default=None, help="with --layer: replace its geometry by C,H,F,k,stride")
    ap.add_argument("--math", choices=["fp32", "tf32", "fp32_tiled", "bf16split"], default="fp32",
                    help="conv mainloop: fp32 CUDA cores (reference-faithful) or tf32 tcgen05 tensor cores")
    ap.add_argument("--nhwc", action="store_true", help="with --layer and --math tf32: the NHWC tensor-core kernel")
    ap.add_argument("--profile-window", action="store_true",
                    help="eager forwards inside cudaProfilerStart/Stop (for ncu --profile-from-start off); "
                         "the printed numbers are then not bench values")
    args = ap.parse_args()
    if args.suite == "kernels":
        run_kernel_suite(args)
    elif args.layer is not None:
        run_layer_mode(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
