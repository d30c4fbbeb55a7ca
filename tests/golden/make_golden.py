"""Generate the golden fixtures from the reference implementation itself.

Run in a checkout where the reference's source tree is available, as

    PYTHONPATH=<reference root>/src python tests/golden/make_golden.py

It imports the reference package (torch-convnd 0.5.0), runs its portable backend
(``backend='torch'``) in float64 on the seeded inputs of each case — the oracle BASELINE
names ("an fp64 run of the reference path") — and stores inputs (in the case dtype) and
the float64 output and gradients. The fixtures travel with the repository; nothing at
test time reads the reference.
"""

from __future__ import annotations

import importlib.util
import sys
from dataclasses import replace
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
CONFIGS_PATH = HERE.parent.parent / "torch-convnd_b200" / "torch_convnd" / "configs.py"


def _load_configs():
    # Loaded by path: this process's `torch_convnd` is the reference package.
    spec = importlib.util.spec_from_file_location("b200_configs", CONFIGS_PATH)
    module = importlib.util.module_from_spec(spec)
    sys.modules["b200_configs"] = module
    spec.loader.exec_module(module)
    return module


def golden_cases(cfg):
    """Case name -> ConvConfig. c1 at full size, reduced clones of c2-c5 (same channels,
    kernels, geometry and dtype; smaller batch/extents), and the reference tests' edge
    geometries."""
    c = {}
    c["c1"] = cfg.C1
    c["c2r"] = replace(cfg.C2, batch=1, spatial=(5, 5, 5, 5))
    c["c3r"] = replace(cfg.C3, batch=1, spatial=(4, 4, 4, 4, 4))
    c["c4r"] = replace(cfg.C4, batch=1, spatial=(4, 4, 4, 4, 4, 4))
    l1, l2, l3 = cfg.C5_LAYERS
    c["c5l1r"] = replace(l1, batch=2, spatial=(8, 8, 4, 4), input_grad=True)
    c["c5l2r"] = replace(l2, batch=2, spatial=(4, 4, 2, 2))
    c["c5l3r"] = replace(l3, batch=2, spatial=(4, 4, 2, 2))
    # tests/test_convnd.py:119-141 (dilated, strided, grouped, asymmetric geometry)
    c["tiled4d"] = cfg.ConvConfig("tiled4d", 2, 4, 6, (3, 3, 3, 4), (2, 2, 1, 2), (1, 2, 1, 1),
                                  (1, 1, 1, 0), (2, 1, 1, 1), 2, torch.float64, 11)
    # tests/test_convnd.py:98-116 (stride 2 on the first axis, groups 2), ranks 5 and 6
    for rank in (5, 6):
        c[f"full{rank}d"] = cfg.ConvConfig(
            f"full{rank}d", 1, 4, 4, (3,) * rank, (2,) * rank, (2,) + (1,) * (rank - 1),
            (0, 1) + (0,) * (rank - 2), (1,) * rank, 2, torch.float64, 44 + rank)
    # bf16 stride-2 / dilation-2 Conv4d that exercises the tensor-core strided paths
    c["strided_bf16"] = cfg.ConvConfig("strided_bf16", 2, 16, 32, (9, 8, 7, 10), (3, 2, 3, 3),
                                       (2, 1, 2, 2), (1, 0, 2, 1), (1, 2, 1, 1), 1,
                                       torch.bfloat16, 21)
    return c


def run_reference(case, cfg):
    from torch_convnd import conv_nd  # the reference package

    inputs = cfg.make_inputs(case)
    x = inputs.x.detach().to(torch.float64).requires_grad_()
    w = inputs.weight.detach().to(torch.float64).requires_grad_()
    b = inputs.bias.detach().to(torch.float64).requires_grad_() if inputs.bias is not None else None
    y = conv_nd(x, w, b, case.stride, case.padding, case.dilation, case.groups, backend="torch")
    grad = inputs.grad.detach().to(torch.float64)
    if case.name == "c1_conv4d_fp32":
        # c1's loss is y.square().mean(); its cotangent is 2 y / numel in the case dtype.
        grad = (2 * y.detach() / y.numel()).to(case.dtype).to(torch.float64)
        inputs.grad = grad.to(case.dtype)
    tensors = [t for t in (x, w, b) if t is not None]
    grads = torch.autograd.grad(y, tensors, grad)
    record = {
        "config": {
            "batch": case.batch, "in_channels": case.in_channels,
            "out_channels": case.out_channels, "spatial": case.spatial, "kernel": case.kernel,
            "stride": case.stride, "padding": case.padding, "dilation": case.dilation,
            "groups": case.groups, "dtype": str(case.dtype), "seed": case.seed,
        },
        "x": inputs.x, "weight": inputs.weight, "bias": inputs.bias, "grad": inputs.grad,
        "y": y.detach(), "dx": grads[0], "dw": grads[1],
        "db": grads[2] if b is not None else None,
    }
    return record


def main():
    import torch_convnd

    version = getattr(torch_convnd, "__version__", "?")
    cfg = _load_configs()
    torch.set_num_threads(8)
    for name, case in golden_cases(cfg).items():
        record = run_reference(case, cfg)
        record["reference_version"] = version
        torch.save(record, HERE / f"{name}.pt")
        print(name, tuple(record["y"].shape), "saved")


if __name__ == "__main__":
    main()
