#!/usr/bin/env python
"""Benchmark of the N-D convolution hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c1|c2|c3|c4|c5]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...
    python bench.py --impl reference ...      # the reference's own CPU implementation

For c1-c4 a step is one forward + dgrad + wgrad (+ bias gradient) of the configuration's
convolution over one batch of synthetic input already resident in HBM; with N > 1 GPUs
every rank convolves its own batch (weak scaling: per-GPU work fixed) and the weight/bias
gradients are all-reduced with NCCL, as data-parallel training does. For c5 a step is
the three-layer training step over a global batch of 64 split across the ranks (strong
scaling), with bucketed gradient all-reduce and an SGD update.
`value` is whole-job TFLOP/s (all ranks' algorithmic FLOPs / max-over-ranks time).
`e2e` is the same metric through the public module API with the step's inputs copied
from pinned host memory and the step's result read back, inside the timed region (the
copy of the next step's inputs runs on a side stream during the current step).
Clock samples (nvidia-smi, 50 ms) are kept only when stamped inside the timed region.
`roofline` reports the pass (layer x forward/dgrad/wgrad) with the largest share of the
step against the bound its arithmetic intensity sets: the measured burst bf16 tensor peak
(halved for float32, the dense TF32 rate; the passes run in millisecond windows at full
clock) or the measured HBM copy bandwidth; `step_roofline` compares the whole step with
the sum over its passes of those bounds. `configs` holds the same measurement block for
the other BASELINE configurations (c3, c4 and c5 by default), run in the same process
after the headline. `cpu_baseline` times the reference's native CPU implementation
(compiled from its sources into oracle/_ref) on a bounded sample of the same workload.
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
    parser.add_argument("--steps", type=int, default=300)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("b200", "reference"), default="b200")
    parser.add_argument("--config", default="c2", choices=("c1", "c2", "c3", "c4", "c5"))
    parser.add_argument("--fp32-precision", default="3xtf32", choices=("3xtf32", "tf32", "ieee"))
    parser.add_argument("--extra-configs", default="c3,c4,c5",
                        help="other configurations measured in the same run ('' for none)")
    parser.add_argument("--c5-layout", default="channels-last",
                        choices=("channels-last", "channels-first"),
                        help="activation layout of the c5 training step")
    parser.add_argument("--c5-gelu", default="fused", choices=("fused", "separate"),
                        help="GELU of the c5 step inside the convolutions or as its own pass")
    parser.add_argument("--c5-graph", default="on", choices=("on", "off"),
                        help="replay the warmed-up c5 training step as one CUDA graph")
    parser.add_argument("--no-e2e", action="store_true")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--cpu-sample-images", type=int, default=1)
    parser.add_argument("--cpu-baseline-worker", action="store_true", help=argparse.SUPPRESS)
    parser.add_argument("--time-budget", type=float, default=None, help=argparse.SUPPRESS)
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
    """Samples nvidia-smi clocks and throttle reasons every 50 ms; `window()` marks the
    timed region and only samples stamped inside it are summarised."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_id: str):
        self.device_id = device_id
        self.process = None
        self.lines: list[str] = []
        self.thread = None
        self.begin = None
        self.end = None

    def window(self, begin: float, end: float):
        self.begin, self.end = begin, end

    def start(self):
        try:
            self.process = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", self.device_id, "-lms", "50"],
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
        from datetime import datetime

        sm, sm_max, power = [], [], []
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        outside = 0
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                stamp = datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                clock, clock_max, watts = float(parts[2]), float(parts[3]), float(parts[4])
            except ValueError:
                continue
            if self.begin is not None and not self.begin - 0.06 <= stamp <= self.end + 0.06:
                outside += 1
                continue
            sm.append(clock)
            sm_max.append(clock_max)
            power.append(watts)
            for name, flag in zip(names, parts[6:10]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(sm_max) if sm_max else None,
            "power_w_max": max(power) if power else None,
            "samples": len(sm),
            "samples_outside_timed_region": outside,
            "reasons": sorted(reasons),
        }


def geometry_args(cfg, workspace=64 * 1024 * 1024):
    return (list(cfg.stride), list(cfg.padding), list(cfg.dilation), cfg.groups, workspace)


# ------------------------------------------------------------------------------------
# CPU baseline: the reference's own native CPU operators (oracle/_ref), or the oracle.
# ------------------------------------------------------------------------------------

def _cpu_conv_function(kind):
    """A torch.autograd.Function running one convolution layer on the CPU through the
    reference's compiled operators (kind 'reference') or the oracle port ('port')."""
    import torch

    if kind == "reference":
        op = torch.ops.torch_convnd

        def forward(x, w, b, geo):
            return op.conv_nd(x, w, b, *geo)

        def backward(dy, x, w, geo, mask):
            return op.conv_nd_backward(dy, x, w, *geo, mask)
    else:
        from oracle import convnd_oracle as oracle

        def forward(x, w, b, geo):
            return oracle.forward(x, w, b, *geo[:4]).to(x.dtype)

        def backward(dy, x, w, geo, mask):
            grads = oracle.backward(dy, x, w, *geo[:4], mask=mask)
            return tuple(None if g is None else g.to(x.dtype) for g in grads)

    class Conv(torch.autograd.Function):
        @staticmethod
        def forward(ctx, x, w, b, geo):
            ctx.save_for_backward(x, w)
            ctx.geo = geo
            return forward(x, w, b, geo)

        @staticmethod
        def backward(ctx, dy):
            x, w = ctx.saved_tensors
            mask = [ctx.needs_input_grad[0], True, True]
            dx, dw, db = backward(dy.contiguous(), x, w, ctx.geo, mask)
            return dx, dw, db, None

    return Conv


def cpu_baseline_worker(args):
    """Subprocess entry: print one JSON object with the CPU timing of a bounded sample."""
    import torch

    configs = load_configs()
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    ref_so = ROOT / "oracle" / "_ref" / "libtorch_convnd_ref_cpu.so"
    keep = None
    if ref_so.exists():
        from oracle import build_ref

        keep = build_ref.load(ref_so)  # noqa: F841  (the schema library must stay alive)
        kind = "reference"
    else:
        kind = "port"
    conv = _cpu_conv_function(kind)
    images = args.cpu_sample_images
    if args.config == "c5":
        full_batch = configs.C5_BATCH
        data = configs.make_c5_inputs()
        x = data.x[:images].contiguous()
        target = data.target[:images].contiguous()
        params = [(w.clone().requires_grad_(), b.clone().requires_grad_())
                  for w, b in data.parameters]
        layers = configs.C5_LAYERS
        flops = configs.C5_STEP_FLOPS * images / full_batch
        name = "c5 three-layer training step (conv, GELU, conv, GELU, conv, MSE)"

        def step():
            h = x
            for index, (layer, (w, b)) in enumerate(zip(layers, params)):
                h = conv.apply(h, w, b, geometry_args(layer))
                if index + 1 < len(layers):
                    h = torch.nn.functional.gelu(h)
            loss = torch.nn.functional.mse_loss(h, target)
            loss.backward()
            for w, b in params:
                w.grad = b.grad = None
            return loss
    else:
        cfg = config_for(args.config)
        full_batch = cfg.batch
        sample = cfg.with_batch(images)
        inputs = configs.make_inputs(sample)
        x = inputs.x.clone().requires_grad_(cfg.input_grad)
        w = inputs.weight.clone().requires_grad_()
        b = inputs.bias.clone().requires_grad_() if inputs.bias is not None else None
        geo = geometry_args(sample)
        flops = sample.step_flops
        name = f"{cfg.name} (fwd+dgrad+wgrad+dbias)"

        def step():
            y = conv.apply(x, w, b, geo)
            y.backward(inputs.grad)
            x.grad = w.grad = None
            if b is not None:
                b.grad = None
            return y
    steps = max(1, args.steps)
    warmup = max(0, args.warmup)
    budget = getattr(args, "time_budget", None) or 90.0
    for _ in range(warmup):
        step()
    # Timed steps: all K of them, or as many as fit the wall-time budget (at least one),
    # so the reference arm ends within minutes at any --steps.
    timed = 0
    start = time.perf_counter()
    while timed < steps:
        step()
        timed += 1
        if time.perf_counter() - start > budget:
            break
    seconds = (time.perf_counter() - start) / timed
    print(json.dumps({
        "value": flops / seconds / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": kind,
        "seconds_per_step": seconds,
        "steps_timed": timed,
        "sample": f"{images} of {full_batch} images of {name} per step, "
                  f"{args.config} dtype inputs, torch.set_num_threads({cores})",
    }))
    del keep


def cpu_baseline(args, steps=1, warmup=0, time_budget=20.0):
    command = [sys.executable, str(Path(__file__).resolve()), "--cpu-baseline-worker",
               "--config", args.config, "--cpu-sample-images", str(args.cpu_sample_images),
               "--steps", str(steps), "--warmup", str(warmup),
               "--time-budget", str(time_budget)]
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
    result = cpu_baseline(worker_args, steps=steps, warmup=warmup, time_budget=90.0)
    import torch  # noqa: F401

    value = result.get("value")
    if args.config == "c5":
        dtype, workload, batch = "bf16", C5_WORKLOAD, load_configs().C5_BATCH
    else:
        cfg = config_for(args.config)
        dtype, workload, batch = dtype_name(cfg.dtype), workload_text(cfg), cfg.batch
    line = {
        "metric": METRIC,
        "impl": "reference",
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": args.gpus,
        "steps": result.get("steps_timed", steps),
        "steps_requested": steps,
        "warmup": warmup,
        "ms_per_step": None if value is None else result["seconds_per_step"] * 1e3,
        "higher_is_better": True,
        "scaling": "strong" if args.config == "c5" else "weak",
        "vs_baseline": None,
        "dtype": dtype,
        "data": "synthetic (seeded N(0,1) activations and gradients, kaiming-uniform weights)",
        "config": {"workload": workload + "; reference CPU path on a bounded sample",
                   "batch": batch, "parallelism": "host cores"},
        "cpu_baseline": {k: result.get(k) for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


# ------------------------------------------------------------------------------------
# B200 arm: workloads
# ------------------------------------------------------------------------------------

C5_WORKLOAD = ("c5: 3-layer Conv4d bf16 training step, x[64,16,32,32,16,16] -> L1 16->32 "
               "k3 s2 p1 -> GELU -> L2 32->32 k(3,3,1,1) p(2,2,0,0) d(2,2,1,1) g4 -> GELU -> "
               "L3 32->8 k1 -> MSE; fwd + bwd (no dgrad of L1) + gradient all-reduce + SGD")


class Prefetcher:
    """Double-buffered host-to-device input copies on a side stream: while step k runs on
    the current stream, step k+1's pinned host inputs are copied into the other buffer.
    Events order the copy after the last use of that buffer and the step after its copy,
    so every step still copies its own inputs; only the overlap is new."""

    def __init__(self, host_tensors, device):
        import torch

        self.host = host_tensors
        self.bufs = [[torch.empty_like(t, device=device) for t in host_tensors] for _ in range(2)]
        self.ready = [torch.cuda.Event() for _ in range(2)]
        self.free = [torch.cuda.Event() for _ in range(2)]
        self.copy_stream = torch.cuda.Stream(device=device)
        self.index = 0
        self.pending = False

    def _issue(self, slot):
        import torch

        self.copy_stream.wait_event(self.free[slot])
        with torch.cuda.stream(self.copy_stream):
            for dst, src in zip(self.bufs[slot], self.host):
                dst.copy_(src, non_blocking=True)
            self.ready[slot].record(self.copy_stream)

    def next(self):
        """Device copies of this step's inputs (waited on by the current stream); starts
        the copy of the following step's inputs."""
        import torch

        slot = self.index % 2
        if not self.pending:
            self._issue(slot)
        torch.cuda.current_stream().wait_event(self.ready[slot])
        self._issue(1 - slot)
        self.pending = True
        self.index += 1
        return slot, self.bufs[slot]

    def release(self, slot):
        import torch

        self.free[slot].record(torch.cuda.current_stream())


class SingleOp:
    """c1-c4: one convolution's forward + dgrad + wgrad + dbias per step. Every rank
    convolves its own batch of the config's size (weak scaling); the weight and bias
    gradients are all-reduced in one fp32 bucket."""

    scaling = "weak"

    def __init__(self, args, device, rank, world, dist):
        import torch

        configs = load_configs()
        self.cfg = cfg = config_for(args.config)
        self.world, self.dist, self.device = world, dist, device
        self.inputs = configs.make_inputs(cfg, device=device, generator_seed=cfg.seed + 1000 * rank)
        self.geo = geometry_args(cfg)
        self.layers = [cfg]
        self.job_flops = world * cfg.step_flops
        self.dtype = dtype_name(cfg.dtype)
        self.op = torch.ops.torch_convnd

    def _allreduce_start(self, grads):
        """Starts the mean all-reduce of `grads` in one fp32 bucket (NCCL runs it on its
        own stream, after the work queued so far on the current stream)."""
        import torch

        bucket = torch.cat([g.reshape(-1).float() for g in grads])
        bucket.div_(self.world)
        return bucket, self.dist.all_reduce(bucket, async_op=True)

    def _allreduce_finish(self, grads, bucket, work):
        work.wait()
        offset = 0
        for g in grads:
            g.copy_(bucket[offset: offset + g.numel()].view_as(g))
            offset += g.numel()

    def _allreduce(self, grads):
        if self.world == 1:
            return
        self._allreduce_finish(grads, *self._allreduce_start(grads))

    def step(self):
        i = self.inputs
        y = self.op.conv_nd.default(i.x, i.weight, i.bias, *self.geo)
        has_bias = i.bias is not None
        if self.world == 1:
            self.op.conv_nd_backward.default(i.grad, i.x, i.weight, *self.geo,
                                             [True, True, has_bias])
            return y
        # One backward call (dy is packed once for both gradients), then the all-reduce
        # of the weight and bias gradients. Splitting the call to run the all-reduce under
        # the input gradient cost a second dy pack, and NCCL's kernel finds no free SM
        # beside the persistent convolution kernel, so it did not overlap.
        _, dw, db = self.op.conv_nd_backward.default(i.grad, i.x, i.weight, *self.geo,
                                                     [True, True, has_bias])
        self._allreduce([g for g in (dw, db) if g is not None])
        return y

    def config(self):
        cfg = self.cfg
        return {"workload": workload_text(cfg), "per_gpu_batch": cfg.batch,
                "global_batch": cfg.batch * self.world, "parallelism": f"dp{self.world}",
                "step_gflop_per_gpu": cfg.step_flops / 1e9,
                "l2": "inputs larger than L2 (x, dy, y and dx together exceed 126 MB)"}

    def e2e_step_factory(self):
        """Through the public module API: pinned host x and dy copied in, parameter
        gradients read back, every step."""
        import torch

        import torch_convnd

        cfg, inputs, device = self.cfg, self.inputs, self.device
        layer = torch_convnd.ConvNd(cfg.in_channels, cfg.out_channels, cfg.kernel, cfg.stride,
                                    cfg.padding, cfg.dilation, cfg.groups, bias=cfg.bias,
                                    device=device, dtype=cfg.dtype, dimensions=cfg.rank)
        with torch.no_grad():
            layer.weight.copy_(inputs.weight)
            if cfg.bias:
                layer.bias.copy_(inputs.bias)
        x_host = inputs.x.cpu().pin_memory()
        dy_host = inputs.grad.cpu().pin_memory()
        params = list(layer.parameters())
        grad_host = [torch.empty(p.shape, dtype=p.dtype, pin_memory=True) for p in params]
        prefetch = Prefetcher([x_host, dy_host], device)

        def step():
            slot, (x_dev, dy) = prefetch.next()
            x = x_dev.detach().requires_grad_()
            layer(x).backward(dy)
            prefetch.release(slot)
            self._allreduce([p.grad for p in params])
            for host, p in zip(grad_host, params):
                host.copy_(p.grad, non_blocking=True)
                p.grad = None

        h2d = sum(t.numel() * t.element_size() for t in (x_host, dy_host))
        d2h = sum(g.numel() * g.element_size() for g in grad_host)
        return step, h2d, d2h, ("torch_convnd.ConvNd forward + autograd backward; inputs "
                                "copied from pinned host memory each step, the next step's "
                                "copy overlapping this step's kernels")


class C5Step:
    """c5: the three-layer training step over a global batch of 64 split across the
    ranks (strong scaling): forward, MSE loss, backward (L1's input needs no gradient),
    bucketed gradient all-reduce started from gradient hooks, SGD update."""

    scaling = "strong"

    def __init__(self, args, device, rank, world, dist):
        import torch

        import torch_convnd
        from torch_convnd.data_parallel import GradientBucketer, layer_groups, shard_fraction

        configs = load_configs()
        self.world, self.device, self.rank = world, device, rank
        self.data = configs.make_c5_inputs(device=device, rank=rank, world=world)
        # Activations channels-last end to end: the batch (and its target) arrive in that
        # layout, as from a channels-last data loader; every layer then reads its input
        # in place and writes its output channels-last (no layout pass between layers).
        self.layout = args.c5_layout
        if self.layout == "channels-last":
            self.data.x = torch_convnd.channels_last(self.data.x)
            self.data.target = torch_convnd.channels_last(self.data.target)
        shard = self.data.x.shape[0]
        self.layers = [layer.with_batch(shard) for layer in configs.C5_LAYERS]
        self.job_flops = configs.C5_STEP_FLOPS
        self.dtype = "bf16"
        # GELU fused into L1's and L2's epilogues (and its backward into their dy packs)
        self.gelu = args.c5_gelu
        self.net = configs.c5_network(torch_convnd.ConvNd, self.data.parameters, device,
                                      fused_gelu=self.gelu == "fused")
        # one bucket per layer, so L3's and L2's all-reduces run under L1's weight gradient
        self.bucketer = GradientBucketer(layer_groups(self.net),
                                         batch_fraction=shard_fraction(configs.C5_BATCH, rank,
                                                                       world))
        self.optimizer = torch.optim.SGD(self.net.parameters(), lr=1e-4)
        self.mse = torch.nn.functional.mse_loss
        self.dist = dist
        # With --c5-graph on, the warmed-up step (forward, MSE, backward with its
        # hook-started all-reduces, SGD) is captured once and replayed: at small per-GPU
        # batches the eager step is bound by host work (autograd, hooks, launches).
        self.use_graph = args.c5_graph == "on"
        self.graph = None
        self.graph_loss = None
        self.graph_launches = 0
        self.replayed_launches = 0
        self.graph_note = "off"

    def _train(self, x, target):
        loss = self.mse(self.net(x), target)
        loss.backward()
        self.bucketer.finish()
        self.optimizer.step()
        self.optimizer.zero_grad(set_to_none=True)
        return loss

    def prepare(self):
        """Captures one training step as a CUDA graph (after the eager warm-up steps).
        Every rank captures the same step; the ranks agree on success before any replay
        (one eager all-reduce), so a capture failure anywhere leaves all of them eager."""
        import torch

        import torch_convnd

        if not self.use_graph or self.graph is not None:
            return
        ok = 1
        graph = None
        try:
            torch.cuda.synchronize()
            self.optimizer.zero_grad(set_to_none=True)
            graph = torch.cuda.CUDAGraph()
            before = torch_convnd.launch_count()
            with torch.cuda.graph(graph, capture_error_mode="thread_local"):
                loss = self.mse(self.net(self.data.x), self.data.target)
                loss.backward()
                self.bucketer.finish()
                self.optimizer.step()
            self.graph_launches = torch_convnd.launch_count() - before
            self.graph_loss = loss.detach()
        except RuntimeError as error:  # capture refused: keep the eager step
            ok = 0
            self.graph_note = f"capture failed: {str(error).splitlines()[0][:120]}"
        if self.world > 1:
            flag = torch.tensor([ok], device=self.device, dtype=torch.int32)
            self.dist.all_reduce(flag, op=self.dist.ReduceOp.MIN)
            ok = int(flag.item())
        self.optimizer.zero_grad(set_to_none=True)
        if ok:
            self.graph = graph
            self.graph_note = "on"
        else:
            if graph is not None:
                graph.reset()
            if self.graph_note == "on" or self.graph_note == "off":
                self.graph_note = "capture failed on another rank"
            self.use_graph = False

    def step(self):
        if self.graph is None:
            return self._train(self.data.x, self.data.target)
        self.graph.replay()
        self.replayed_launches += self.graph_launches
        return self.graph_loss

    def eager_step(self):
        return self._train(self.data.x, self.data.target)

    def close(self):
        if self.graph is not None:
            self.graph.reset()
            self.graph = None

    def config(self):
        configs = load_configs()
        return {"workload": C5_WORKLOAD, "global_batch": configs.C5_BATCH,
                "per_gpu_batch": self.layers[0].batch, "parallelism": f"dp{self.world}",
                "activation_layout": self.layout,
                "gelu": self.gelu,
                "cuda_graph": self.graph_note,
                "launches_per_step": self.graph_launches or None,
                "step_gflop_per_gpu": sum(l.step_flops for l in self.layers) / 1e9,
                "gradient_buckets": len(self.bucketer.buckets),
                "l2": "inputs larger than L2 (x alone is 537 MB at batch 64)"}

    def e2e_step_factory(self):
        import torch

        device = self.device
        x_host = self.data.x.cpu().pin_memory()
        target_host = self.data.target.cpu().pin_memory()
        if self.layout == "channels-last":
            import torch_convnd

            x_host = torch_convnd.channels_last(self.data.x.cpu()).pin_memory()
            target_host = torch_convnd.channels_last(self.data.target.cpu()).pin_memory()
        loss_host = torch.empty((), dtype=torch.bfloat16, pin_memory=True)
        prefetch = Prefetcher([x_host, target_host], device)

        def step():
            slot, (x, target) = prefetch.next()
            loss = self._train(x, target).detach()
            prefetch.release(slot)
            loss_host.copy_(loss, non_blocking=True)

        h2d = sum(t.numel() * t.element_size() for t in (x_host, target_host))
        return step, h2d, 2, ("torch_convnd.ConvNd x3 + GELU + MSE, autograd backward, SGD; "
                              "inputs copied from pinned host memory each step, the next "
                              "step's copy overlapping this step's kernels")


# ------------------------------------------------------------------------------------
# B200 arm: timing and attribution
# ------------------------------------------------------------------------------------

def timed_ms(step, steps, world, dist, device):
    """Mean device time of `steps` steps (CUDA events on the current stream, barrier and
    synchronize on both sides), max over ranks."""
    import torch

    stream = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(steps):
        step()
    end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end) / steps
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def pass_bytes(layer) -> int:
    """Minimum HBM bytes of one pass: read x (or dy) and the weights, write y (or dx / dw):
    x, y and w once each in the layer dtype."""
    import torch

    size = torch.empty((), dtype=layer.dtype).element_size()
    x = layer.batch * layer.in_channels * math.prod(layer.spatial)
    y = layer.batch * layer.out_channels * math.prod(layer.output)
    w = layer.out_channels * (layer.in_channels // layer.groups) * math.prod(layer.kernel)
    return size * (x + y + w)


def attribute_passes(timings, layers, steps):
    """Splits the launch-ordered pass timings of `steps` steps by layer: forward passes run
    in layer order, dgrad and wgrad in reverse layer order (dgrad only where the layer's
    input needs a gradient)."""
    orders = {
        "forward": [l.name for l in layers],
        "dgrad": [l.name for l in reversed(layers) if l.input_grad],
        "wgrad": [l.name for l in reversed(layers)],
    }
    seen = {k: 0 for k in orders}
    per_layer = {}
    for kind, ms in timings:
        if kind not in orders or not orders[kind]:
            continue
        name = orders[kind][seen[kind] % len(orders[kind])]
        seen[kind] += 1
        per_layer.setdefault((kind, name), []).append(ms)
    return per_layer


def roofline_terms(layer, peaks):
    """(flop-bound seconds, byte-bound seconds, tensor peak TF/s) of one pass of `layer`:
    the conv's algorithmic FLOPs against the measured burst tensor peak (halved for float32:
    the dense TF32 rate) and its minimum HBM bytes against the measured copy bandwidth."""
    import torch

    peak_t = peaks["tensor"] / (2 if layer.dtype == torch.float32 else 1)
    return (layer.forward_flops / (peak_t * 1e12), pass_bytes(layer) / (peaks["hbm"] * 1e9),
            peak_t)


def measure(workload, args, world, dist, device, peaks):
    """Times `workload.step` (warm-up, then args.steps steps between barriers and
    synchronizes, max over ranks), then times each library pass with CUDA events on its
    launching stream over a few more steps. Returns the measurement block."""
    import torch

    import torch_convnd

    warmup = max(args.warmup, 3)
    for _ in range(warmup):
        workload.step()
    torch.cuda.synchronize()
    torch_convnd.device_status()
    # A workload may turn its warmed-up step into a CUDA graph here (c5); its replays
    # launch the library's kernels without the host seeing them, so it counts them.
    if hasattr(workload, "prepare"):
        workload.prepare()
        torch.cuda.synchronize()
    props = torch.cuda.get_device_properties(device)
    uuid = getattr(props, "uuid", None)
    sampler = ClockSampler(f"GPU-{uuid}" if uuid is not None else str(device.index))
    sampler.start()
    time.sleep(0.3)
    torch_convnd.launch_count(reset=True)
    if hasattr(workload, "replayed_launches"):
        workload.replayed_launches = 0
    begin = time.time()
    ms = timed_ms(workload.step, args.steps, world, dist, device)
    sampler.window(begin, time.time())
    clocks = sampler.stop()
    launches = torch_convnd.launch_count() + getattr(workload, "replayed_launches", 0)
    value = workload.job_flops / (ms / 1e3) / 1e12
    torch_convnd.device_status()

    # Per-pass durations with CUDA events on the launching stream (a separate loop).
    torch_convnd._native.set_kernel_timing(True)
    timing_steps = min(args.steps, 5)
    eager_step = getattr(workload, "eager_step", workload.step)  # events need eager launches
    for _ in range(timing_steps):
        eager_step()
    torch.cuda.synchronize()
    timings = torch_convnd._native.collect_kernel_timings()
    torch_convnd._native.set_kernel_timing(False)
    kernels = {}
    for kind, t in timings:
        entry = kernels.setdefault(kind, {"launches": 0, "total_ms": 0.0})
        entry["launches"] += 1
        entry["total_ms"] += t
    for entry in kernels.values():
        entry["avg_ms"] = entry["total_ms"] / entry["launches"]
        entry["share_of_step"] = entry.pop("total_ms") / timing_steps / ms

    passes = {}
    by_name = {l.name: l for l in workload.layers}
    target_ms = 0.0
    for (kind, name), values in attribute_passes(timings, workload.layers, timing_steps).items():
        layer = by_name[name]
        avg = sum(values) / len(values)
        t_flop, t_byte, _ = roofline_terms(layer, peaks)
        target_ms += max(t_flop, t_byte) * 1e3 * len(values) / timing_steps
        passes[f"{name} {kind}"] = {
            "layer": name, "kind": kind, "launches": len(values), "avg_ms": avg,
            "tflops": layer.forward_flops / (avg / 1e3) / 1e12,
            "gbs": pass_bytes(layer) / (avg / 1e3) / 1e9,
            "bound": "tensor" if t_flop >= t_byte else "hbm",
            "roofline_ms": max(t_flop, t_byte) * 1e3,
            "share_of_step": sum(values) / timing_steps / ms,
        }
    roofline = None
    if passes:
        key = max(passes, key=lambda k: passes[k]["share_of_step"])
        info = passes[key]
        layer = by_name[info["layer"]]
        traffic = traffic_from_profiles(layer.name, info["kind"])
        _, _, peak_t = roofline_terms(layer, peaks)
        if info["bound"] == "tensor":
            fp32 = layer.dtype == torch.float32
            note = (f"{peaks['source']} cuBLAS bf16 burst (the passes run in short windows at "
                    "full clock)" + (" / 2: the dense TF32 rate" if fp32 else ""))
            peak, achieved, unit = peak_t, info["tflops"], "TFLOP/s"
            algorithmic = f"{layer.forward_flops / 1e9:.1f} GFLOP per launch"
        else:
            peak, note = peaks["hbm"], f"{peaks['source']} HBM copy bandwidth"
            achieved, unit = info["gbs"], "GB/s"
            algorithmic = f"{pass_bytes(layer) / 1e6:.1f} MB per launch"
        roofline = {"kernel": f"{key} pass (tcgen05)", "bound": info["bound"],
                    "achieved": achieved, "peak": peak, "unit": unit,
                    "frac": achieved / peak, "peak_source": note,
                    "algorithmic": algorithmic, "traffic": traffic}
        if info["bound"] == "tensor":
            sustained = peaks["tensor_sustained"] / (2 if layer.dtype == torch.float32 else 1)
            roofline["frac_of_sustained"] = achieved / sustained
    # The whole step against the sum over its passes of max(FLOPs / peak, bytes / HBM).
    step_roofline = {"target_ms": target_ms, "frac": target_ms / ms if ms else None,
                     "note": "sum over the step's passes of max(FLOPs / tensor peak, "
                             "minimum bytes / HBM bandwidth); frac = target / measured"}
    return {"ms_per_step": ms, "value": value, "value_per_gpu": value / world,
            "passes": passes, "kernels": kernels, "roofline": roofline,
            "step_roofline": step_roofline, "gpu_launches": launches, "clocks": clocks,
            "warmup": warmup}


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

    torch_convnd.set_fp32_precision(args.fp32_precision)
    data, source = measured_peaks()
    peaks = {"source": source,
             "hbm": float(data.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])),
             "tensor": float(data.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])),
             "tensor_sustained": float(data.get("bf16_tflops_sustained",
                                                FALLBACK_PEAKS["bf16_tflops_sustained"]))}
    workload = (C5Step if args.config == "c5" else SingleOp)(args, device, rank, world, dist)
    block = measure(workload, args, world, dist, device, peaks)
    ms, value = block["ms_per_step"], block["value"]

    e2e = None
    if not args.no_e2e:
        step, h2d, d2h, api = workload.e2e_step_factory()
        for _ in range(3):
            step()
        torch.cuda.synchronize()
        e2e_ms = timed_ms(step, args.steps, world, dist, device)
        e2e = {"value": workload.job_flops / (e2e_ms / 1e3) / 1e12, "unit": "TFLOP/s",
               "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "api": api}
    config = workload.config()
    if workload.dtype == "fp32":
        config["fp32_precision"] = args.fp32_precision
    headline_dtype, headline_scaling = workload.dtype, workload.scaling
    if hasattr(workload, "close"):
        workload.close()  # a graph holding NCCL calls goes before the process group
    del workload
    torch.cuda.empty_cache()

    # The other BASELINE configurations, measured the same way in the same run (every
    # rank runs each in the same order, so their collectives line up).
    extra = {}
    names = [] if args.extra_configs in ("", "none") else args.extra_configs.split(",")
    for name in names:
        if name == args.config:
            continue
        sub = argparse.Namespace(**vars(args))
        sub.config = name
        other = (C5Step if name == "c5" else SingleOp)(sub, device, rank, world, dist)
        result = measure(other, sub, world, dist, device, peaks)
        result.update({"metric_unit": "TFLOP/s", "dtype": other.dtype,
                       "scaling": other.scaling, "config": other.config()})
        if other.dtype == "fp32":
            result["config"]["fp32_precision"] = args.fp32_precision
        extra[name] = result
        if hasattr(other, "close"):
            other.close()
        del other
        torch.cuda.empty_cache()

    baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        baseline = cpu_baseline(args, steps=2, warmup=1)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": block["warmup"],
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": headline_scaling,
            "vs_baseline": None,
            "dtype": headline_dtype,
            "data": "synthetic (seeded N(0,1) activations and gradients, kaiming-uniform "
                    "weights, uniform bias; the reference config's shapes)",
            "config": config,
            "value_per_gpu": block["value_per_gpu"],
            "roofline": block["roofline"],
            "step_roofline": block["step_roofline"],
            "passes": block["passes"],
            "kernels": block["kernels"],
            "cpu_baseline": baseline,
            "e2e": e2e,
            "gpu_launches": block["gpu_launches"],
            "clocks": block["clocks"],
            "configs": extra,
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
