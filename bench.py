#!/usr/bin/env python
"""Benchmark of the N-D convolution hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2|c3|c4|c1]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...
    python bench.py --impl reference ...      # the reference's own CPU implementation

A step is one forward + dgrad + wgrad (+ bias gradient) of the configuration's
convolution over one batch of synthetic input that is already resident in HBM; with
N > 1 GPUs every rank convolves its own batch (weak scaling: per-GPU work fixed) and the
weight/bias gradients are all-reduced with NCCL, as data-parallel training does.
`value` is whole-job TFLOP/s (all ranks' algorithmic FLOPs / max-over-ranks time).
`e2e` is the same metric through the public module API with the step's inputs copied
from pinned host memory and the parameter gradients read back, inside the timed region.
`roofline` reports the dominant tcgen05 pass; `cpu_baseline` times the reference's
native CPU implementation (compiled from its sources into oracle/_ref) on a bounded
sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _path in (ROOT / "torch-convnd_b200", ROOT):
    if str(_path) not in sys.path:
        sys.path.insert(0, str(_path))

METRIC = "Conv4d/5d/6d fwd+bwd TFLOP/s per GPU and % of B200 tensor peak at 1/2/4/8 GPUs"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse_args(argv=None):
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[1])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("b200", "reference"), default="b200")
    parser.add_argument("--config", default="c2", choices=("c1", "c2", "c3", "c4"))
    parser.add_argument("--fp32-precision", default="3xtf32", choices=("3xtf32", "tf32", "ieee"))
    parser.add_argument("--no-e2e", action="store_true")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--cpu-sample-images", type=int, default=1)
    parser.add_argument("--cpu-baseline-worker", action="store_true", help=argparse.SUPPRESS)
    return parser.parse_args(argv)


def load_configs():
    """torch_convnd/configs.py loaded by path, so that the reference arm and the CPU
    baseline never import the B200 package (both register the same operators)."""
    import importlib.util

    if "b200_configs" in sys.modules:
        return sys.modules["b200_configs"]
    spec = importlib.util.spec_from_file_location(
        "b200_configs", ROOT / "torch-convnd_b200" / "torch_convnd" / "configs.py")
    module = importlib.util.module_from_spec(spec)
    sys.modules["b200_configs"] = module
    spec.loader.exec_module(module)
    return module


def config_for(name):
    configs = load_configs()
    return {"c1": configs.C1, "c2": configs.C2, "c3": configs.C3, "c4": configs.C4}[name]


def dtype_name(dtype) -> str:
    import torch

    return {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32",
            torch.float64: "fp64"}[dtype]


def workload_text(cfg) -> str:
    kind = f"Conv{cfg.rank}d"
    shape = "x".join(str(s) for s in cfg.spatial)
    kernel = "x".join(str(k) for k in cfg.kernel)
    return (f"{cfg.name}: {kind} {dtype_name(cfg.dtype)} fwd+dgrad+wgrad+dbias, "
            f"x[{cfg.batch},{cfg.in_channels},{shape}] w[{cfg.out_channels},"
            f"{cfg.in_channels // cfg.groups},{kernel}] stride {cfg.stride[0]} pad "
            f"{cfg.padding[0]}, batch {cfg.batch} per GPU")


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return data, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_id: str):
        self.device_id = device_id
        self.process = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.process = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", self.device_id, "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.process = None
            return
        self.thread = threading.Thread(target=self._drain, daemon=True)
        self.thread.start()

    def _drain(self):
        for line in self.process.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.process is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.process.terminate()
        try:
            self.process.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.process.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)
        sm, sm_max, power = [], [], []
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                sm_max.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(sm_max) if sm_max else None,
            "power_w_max": max(power) if power else None,
            "samples": len(sm),
            "reasons": sorted(reasons),
        }


def geometry_args(cfg, workspace=64 * 1024 * 1024):
    return (list(cfg.stride), list(cfg.padding), list(cfg.dilation), cfg.groups, workspace)


# ------------------------------------------------------------------------------------
# CPU baseline: the reference's own native CPU operators (oracle/_ref), or the oracle.
# ------------------------------------------------------------------------------------

def cpu_baseline_worker(args):
    """Subprocess entry: print one JSON object with the CPU timing of a bounded sample."""
    import torch

    configs = load_configs()
    cfg = config_for(args.config)
    sample = cfg.with_batch(args.cpu_sample_images)
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    inputs = configs.make_inputs(sample)
    geo = geometry_args(sample)
    ref_so = ROOT / "oracle" / "_ref" / "libtorch_convnd_ref_cpu.so"
    if ref_so.exists():
        from oracle import build_ref

        keep = build_ref.load(ref_so)  # noqa: F841  (the schema library must stay alive)
        kind = "reference"

        def step():
            y = torch.ops.torch_convnd.conv_nd(inputs.x, inputs.weight, inputs.bias, *geo)
            grads = torch.ops.torch_convnd.conv_nd_backward(
                inputs.grad, inputs.x, inputs.weight, *geo, [True, True, True])
            return y, grads
    else:
        from oracle import convnd_oracle as oracle

        kind = "port"
        cores = torch.get_num_threads()

        def step():
            y = oracle.forward(inputs.x, inputs.weight, inputs.bias, sample.stride,
                               sample.padding, sample.dilation, sample.groups)
            grads = oracle.backward(inputs.grad, inputs.x, inputs.weight, sample.stride,
                                    sample.padding, sample.dilation, sample.groups)
            return y, grads
    steps = max(1, args.steps)
    warmup = max(0, args.warmup)
    for _ in range(warmup):
        step()
    start = time.perf_counter()
    for _ in range(steps):
        step()
    seconds = (time.perf_counter() - start) / steps
    value = sample.step_flops / seconds / 1e12
    print(json.dumps({
        "value": value, "unit": "TFLOP/s", "cores": cores, "kind": kind,
        "seconds_per_step": seconds,
        "sample": f"{args.cpu_sample_images} of {cfg.batch} images of {cfg.name} per step "
                  f"(fwd+dgrad+wgrad+dbias, {dtype_name(cfg.dtype)} inputs), "
                  f"torch.set_num_threads({cores})",
    }))


def cpu_baseline(args, steps=1, warmup=0):
    command = [sys.executable, str(Path(__file__).resolve()), "--cpu-baseline-worker",
               "--config", args.config, "--cpu-sample-images", str(args.cpu_sample_images),
               "--steps", str(steps), "--warmup", str(warmup)]
    result = subprocess.run(command, capture_output=True, text=True, timeout=900)
    if result.returncode != 0:
        return {"value": None, "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "reference",
                "sample": "failed: " + result.stderr.strip().splitlines()[-1][:200]}
    return json.loads(result.stdout.strip().splitlines()[-1])


# ------------------------------------------------------------------------------------
# Reference arm
# ------------------------------------------------------------------------------------

def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    # The reference's CPU path on the host cores, one bounded sample per step.
    steps = max(1, args.steps)
    warmup = max(0, min(args.warmup, 3))
    worker_args = argparse.Namespace(config=args.config,
                                     cpu_sample_images=args.cpu_sample_images, steps=steps,
                                     warmup=warmup)
    result = cpu_baseline(worker_args, steps=steps, warmup=warmup)
    import torch  # noqa: F401

    cfg = config_for(args.config)
    value = result.get("value")
    line = {
        "metric": METRIC,
        "impl": "reference",
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": args.gpus,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": None if value is None else result["seconds_per_step"] * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": dtype_name(cfg.dtype),
        "data": "synthetic (seeded N(0,1) activations and gradients, kaiming-uniform weights)",
        "config": {"workload": workload_text(cfg) + "; reference CPU path on a bounded sample",
                   "per_gpu_batch": cfg.batch, "parallelism": "host cores"},
        "cpu_baseline": {k: result.get(k) for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


# ------------------------------------------------------------------------------------
# B200 arm
# ------------------------------------------------------------------------------------

def run_b200(args):
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=device)

    import torch_convnd

    configs = load_configs()
    torch_convnd.set_fp32_precision(args.fp32_precision)
    cfg = config_for(args.config)
    inputs = configs.make_inputs(cfg, device=device, generator_seed=cfg.seed + 1000 * rank)
    x, w, b, dy = inputs.x, inputs.weight, inputs.bias, inputs.grad
    geo = geometry_args(cfg)
    op = torch.ops.torch_convnd
    bucket_numel = w.numel() + (b.numel() if b is not None else 0)

    def allreduce(dw, db):
        if world == 1:
            return
        bucket = torch.cat([dw.reshape(-1).float(), db.reshape(-1).float()])
        dist.all_reduce(bucket)
        bucket.div_(world)
        dw.copy_(bucket[: dw.numel()].view_as(dw))
        db.copy_(bucket[dw.numel():].view_as(db))

    def step():
        y = op.conv_nd.default(x, w, b, *geo)
        dx, dw, db = op.conv_nd_backward.default(dy, x, w, *geo, [True, True, True])
        allreduce(dw, db)
        return y, dx, dw, db

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    torch_convnd.device_status()
    barrier()
    props = torch.cuda.get_device_properties(device)
    uuid = getattr(props, "uuid", None)
    sampler = ClockSampler(f"GPU-{uuid}" if uuid is not None else str(local))
    sampler.start()
    time.sleep(0.3)
    torch_convnd.launch_count(reset=True)
    stream = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(args.steps):
        step()
    end.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    launches = torch_convnd.launch_count()
    ms = start.elapsed_time(end) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = world * cfg.step_flops / (ms / 1e3) / 1e12
    torch_convnd.device_status()

    # Per-pass durations with CUDA events on the launching stream (separate loop).
    torch_convnd._native.set_kernel_timing(True)
    timing_steps = min(args.steps, 5)
    for _ in range(timing_steps):
        step()
    torch.cuda.synchronize()
    timings = torch_convnd._native.collect_kernel_timings()
    torch_convnd._native.set_kernel_timing(False)
    per_kind = {}
    for kind, t in timings:
        per_kind.setdefault(kind, []).append(t)
    kernels = {}
    for kind, values in per_kind.items():
        kernels[kind] = {"launches": len(values), "avg_ms": sum(values) / len(values),
                         "share_of_step": sum(values) / timing_steps / ms}
    peaks, source = measured_peaks()
    tensor_passes = {k: v for k, v in kernels.items() if k in ("forward", "dgrad", "wgrad")}
    roofline = None
    if tensor_passes:
        dominant = max(tensor_passes, key=lambda k: tensor_passes[k]["avg_ms"] *
                       tensor_passes[k]["launches"])
        achieved = cfg.forward_flops / (tensor_passes[dominant]["avg_ms"] / 1e3) / 1e12
        peak = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
        peak_note = f"{source} cuBLAS bf16 sustained"
        if cfg.dtype == torch.float32:
            peak = peak / 2
            peak_note = f"{source} cuBLAS bf16 sustained / 2 (dense TF32 rate)"
        traffic = traffic_from_profiles(cfg.name, dominant)
        roofline = {"kernel": f"{dominant} pass (tcgen05)", "bound": "tensor",
                    "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                    "frac": achieved / peak, "peak_source": peak_note, "traffic": traffic}
        for kind, info in tensor_passes.items():
            info["tflops"] = cfg.forward_flops / (info["avg_ms"] / 1e3) / 1e12

    # End-to-end through the public API with host buffers.
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, cfg, inputs, device, world, dist, rank)

    baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        baseline = cpu_baseline(args, steps=1, warmup=0)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": max(args.warmup, 3),
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": dtype_name(cfg.dtype),
            "data": "synthetic (seeded N(0,1) activations and gradients, kaiming-uniform "
                    "weights, uniform bias; the reference config's shapes)",
            "config": {
                "workload": workload_text(cfg),
                "per_gpu_batch": cfg.batch,
                "global_batch": cfg.batch * world,
                "parallelism": f"dp{world}",
                "step_gflop_per_gpu": cfg.step_flops / 1e9,
                "fp32_precision": args.fp32_precision if cfg.dtype == torch.float32 else None,
                "l2": "inputs larger than L2 (x, dy, y and dx together exceed 126 MB)",
            },
            "value_per_gpu": value / world,
            "roofline": roofline,
            "kernels": kernels,
            "cpu_baseline": baseline,
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clocks,
        }
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def traffic_from_profiles(config_name, kind):
    """DRAM bytes per launch of a pass, from the committed ncu summary (if any)."""
    path = ROOT / "profiles" / "traffic.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        parts = line.split()
        if len(parts) == 3 and not line.startswith("#") and parts[:2] == [config_name, kind]:
            return int(parts[2])
    return None


def run_e2e(args, cfg, inputs, device, world, dist, rank):
    import torch

    import torch_convnd

    layer = torch_convnd.ConvNd(cfg.in_channels, cfg.out_channels, cfg.kernel, cfg.stride,
                                cfg.padding, cfg.dilation, cfg.groups, bias=cfg.bias,
                                device=device, dtype=cfg.dtype, dimensions=cfg.rank)
    with torch.no_grad():
        layer.weight.copy_(inputs.weight)
        if cfg.bias:
            layer.bias.copy_(inputs.bias)
    x_host = inputs.x.cpu().pin_memory()
    dy_host = inputs.grad.cpu().pin_memory()
    grad_host = [torch.empty(p.shape, dtype=p.dtype, pin_memory=True) for p in layer.parameters()]

    def step():
        x = x_host.to(device, non_blocking=True).requires_grad_()
        dy = dy_host.to(device, non_blocking=True)
        layer(x).backward(dy)
        params = list(layer.parameters())
        if world > 1:
            bucket = torch.cat([p.grad.reshape(-1).float() for p in params])
            dist.all_reduce(bucket)
            bucket.div_(world)
            offset = 0
            for p in params:
                p.grad.copy_(bucket[offset: offset + p.numel()].view_as(p))
                offset += p.numel()
        for host, p in zip(grad_host, params):
            host.copy_(p.grad, non_blocking=True)
            p.grad = None
        return x

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        step()
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    h2d = x_host.numel() * x_host.element_size() + dy_host.numel() * dy_host.element_size()
    d2h = sum(g.numel() * g.element_size() for g in grad_host)
    return {"value": world * cfg.step_flops / (ms / 1e3) / 1e12, "unit": "TFLOP/s",
            "ms_per_step": ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "api": "torch_convnd.ConvNd forward + autograd backward"}


def main(argv=None):
    args = parse_args(argv)
    if args.cpu_baseline_worker:
        cpu_baseline_worker(args)
        return
    if args.impl == "reference":
        run_reference_arm(args)
        return
    run_b200(args)


if __name__ == "__main__":
    main()
