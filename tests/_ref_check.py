"""Subprocess helper: run the reference's compiled CPU operators (oracle/_ref) on golden
inputs and print the worst deviation from the golden float64 outputs. Run in a process
that has not imported torch_convnd (the B200 package), because both register CPU kernels
for the same operators."""

import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
from oracle import build_ref  # noqa: E402

_LIBRARY = build_ref.load()  # keep the schema library alive
worst = 0.0
for name in sys.argv[1:]:
    record = torch.load(ROOT / "tests" / "golden" / f"{name}.pt", weights_only=False)
    c = record["config"]
    x, w, b, g = (None if t is None else t.double() for t in
                  (record["x"], record["weight"], record["bias"], record["grad"]))
    args = (list(c["stride"]), list(c["padding"]), list(c["dilation"]), c["groups"], 1 << 26)
    y = torch.ops.torch_convnd.conv_nd(x, w, b, *args)
    dx, dw, db = torch.ops.torch_convnd.conv_nd_backward(g, x, w, *args, [True, True, b is not None])
    for got, ref in ((y, record["y"]), (dx, record["dx"]), (dw, record["dw"]), (db, record["db"])):
        if ref is not None:
            worst = max(worst, float((got - ref).abs().max() / ref.abs().max().clamp_min(1e-30)))
print(f"worst_relative_deviation={worst:.3e}")
