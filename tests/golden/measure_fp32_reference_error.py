"""Measure the reference's own float32 error at c4's full size (a record, not a test).

Runs the reference's native CPU operators (compiled from its sources into oracle/_ref by
oracle/build_ref.py) on c4's seeded inputs in float32 and compares y, dx and dW with the
float64 tap oracle. Writes c4_fp32_reference_error.json beside this file: per tensor the
largest |expected|, the largest absolute error, the count of elements outside BASELINE's
literal float32 bar (rtol 1e-3, atol 1e-4) and the worst error as a multiple of that bar.
It shows that the reference path itself misses the literal bar on a few weight-gradient
entries (sums over a million positions), which is why the float32 checks add each
element's fp32 summation bound (tests/tolerances.py). Takes a few minutes on 8 cores.

    python tests/golden/measure_fp32_reference_error.py
"""

from __future__ import annotations

import importlib.util
import json
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))


def main():
    spec = importlib.util.spec_from_file_location(
        "b200_configs", ROOT / "torch-convnd_b200" / "torch_convnd" / "configs.py")
    configs = importlib.util.module_from_spec(spec)
    sys.modules["b200_configs"] = configs
    spec.loader.exec_module(configs)
    from oracle import build_ref
    from oracle import convnd_oracle as oracle

    keep = build_ref.load()  # noqa: F841 (the schema library must stay alive)
    cfg = configs.C4
    inputs = configs.make_inputs(cfg)
    geometry = (list(cfg.stride), list(cfg.padding), list(cfg.dilation), cfg.groups)
    workspace = 1 << 30
    op = torch.ops.torch_convnd
    y = op.conv_nd(inputs.x, inputs.weight, inputs.bias, *geometry, workspace)
    dx, dw, _ = op.conv_nd_backward(inputs.grad, inputs.x, inputs.weight, *geometry, workspace,
                                    [True, True, False])
    expected = {
        "y": oracle.tap_reference(inputs.x, inputs.weight, inputs.bias, *geometry),
        "dx": oracle.tap_dgrad(inputs.grad, inputs.weight, cfg.spatial, *geometry),
        "dw": oracle.tap_wgrad(inputs.grad, inputs.x, cfg.kernel, *geometry),
    }
    record = {"config": cfg.name, "workspace_bytes": workspace, "tensors": {}}
    for name, got in (("y", y), ("dx", dx), ("dw", dw)):
        e = expected[name]
        error = (got.double() - e).abs()
        ratio = error / (1e-4 + 1e-3 * e.abs())
        record["tensors"][name] = {
            "max_abs_expected": float(e.abs().max()), "max_abs_error": float(error.max()),
            "literal_bar_violations": int((ratio > 1).sum()), "elements": e.numel(),
            "worst_multiple_of_literal_bar": float(ratio.max()),
            "relative_l2": float((got.double() - e).norm() / e.norm())}
    (HERE / "c4_fp32_reference_error.json").write_text(json.dumps(record, indent=1) + "\n")
    print(json.dumps(record, indent=1))


if __name__ == "__main__":
    main()
