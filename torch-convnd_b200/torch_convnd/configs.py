"""The reference benchmark's five configurations and their seeded synthetic inputs.

Configurations c1-c5 are the ones the B200 build is measured and checked on (one Conv4d
fp32 case the reference's CPU path runs, Conv4d/5d bf16, Conv6d fp32 on TF32 tensor
cores, and a three-layer Conv4d training step). Inputs are drawn on the CPU in a fixed
order — x ~ N(0,1), weight kaiming-uniform(a=sqrt(5)), bias U(+-1/sqrt(fan_in)) (the
module initialisation, reference modules.py:97-102), then the upstream gradient ~ N(0,1)
— and only then moved to the device, so every implementation sees identical values.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field, replace

import torch


@dataclass(frozen=True)
class ConvConfig:
    """One convolution layer: shapes, geometry, dtype and seed."""

    name: str
    batch: int
    in_channels: int
    out_channels: int
    spatial: tuple[int, ...]
    kernel: tuple[int, ...]
    stride: tuple[int, ...]
    padding: tuple[int, ...]
    dilation: tuple[int, ...]
    groups: int
    dtype: torch.dtype
    seed: int
    bias: bool = True
    input_grad: bool = True

    @property
    def rank(self) -> int:
        return len(self.spatial)

    @property
    def output(self) -> tuple[int, ...]:
        return tuple(
            (size + 2 * p - d * (k - 1) - 1) // s + 1
            for size, k, s, p, d in zip(
                self.spatial, self.kernel, self.stride, self.padding, self.dilation, strict=True
            )
        )

    @property
    def forward_flops(self) -> int:
        """2 * N * Cout * (Cin/g) * prod(kernel) * prod(output): padded taps counted."""
        return (
            2
            * self.batch
            * self.out_channels
            * (self.in_channels // self.groups)
            * math.prod(self.kernel)
            * math.prod(self.output)
        )

    @property
    def step_flops(self) -> int:
        """Forward + wgrad (+ dgrad when the input needs a gradient)."""
        return self.forward_flops * (3 if self.input_grad else 2)

    def with_batch(self, batch: int) -> ConvConfig:
        return replace(self, batch=batch)


def _uniform(n):
    return (n,) * 4


C1 = ConvConfig("c1_conv4d_fp32", 2, 2, 8, _uniform(8), _uniform(3), _uniform(1), _uniform(1),
                _uniform(1), 1, torch.float32, 0)
C2 = ConvConfig("c2_conv4d_bf16", 16, 32, 64, _uniform(16), _uniform(3), _uniform(1),
                _uniform(1), _uniform(1), 1, torch.bfloat16, 1)
C3 = ConvConfig("c3_conv5d_bf16", 8, 16, 32, (12,) * 5, (3,) * 5, (1,) * 5, (1,) * 5, (1,) * 5,
                1, torch.bfloat16, 2)
C4 = ConvConfig("c4_conv6d_tf32", 4, 8, 16, (8,) * 6, (3,) * 6, (1,) * 6, (1,) * 6, (1,) * 6, 1,
                torch.float32, 3)

# c5: three Conv4d layers with GELU between them; the first layer's input is data.
C5_BATCH = 64
C5_LAYERS = (
    ConvConfig("c5_l1", C5_BATCH, 16, 32, (32, 32, 16, 16), _uniform(3), _uniform(2),
               _uniform(1), _uniform(1), 1, torch.bfloat16, 4, input_grad=False),
    ConvConfig("c5_l2", C5_BATCH, 32, 32, (16, 16, 8, 8), (3, 3, 1, 1), _uniform(1),
               (2, 2, 0, 0), (2, 2, 1, 1), 4, torch.bfloat16, 4),
    ConvConfig("c5_l3", C5_BATCH, 32, 8, (16, 16, 8, 8), _uniform(1), _uniform(1), _uniform(0),
               _uniform(1), 1, torch.bfloat16, 4),
)

CONFIGS = {c.name: c for c in (C1, C2, C3, C4)}


@dataclass
class ConvInputs:
    x: torch.Tensor
    weight: torch.Tensor
    bias: torch.Tensor | None
    grad: torch.Tensor
    extra: dict = field(default_factory=dict)


def make_inputs(config: ConvConfig, device="cpu", generator_seed: int | None = None) -> ConvInputs:
    """Seeded inputs of `config`, drawn on the CPU in the fixed order, then moved."""
    seed = config.seed if generator_seed is None else generator_seed
    generator = torch.Generator().manual_seed(seed)
    x = torch.randn((config.batch, config.in_channels, *config.spatial), generator=generator)
    fan_in = config.in_channels // config.groups * math.prod(config.kernel)
    bound = 1.0 / math.sqrt(fan_in)  # kaiming_uniform(a=sqrt(5)) bound = 1/sqrt(fan_in)
    weight = torch.empty(
        (config.out_channels, config.in_channels // config.groups, *config.kernel)
    ).uniform_(-bound, bound, generator=generator)
    bias = None
    if config.bias:
        bias = torch.empty(config.out_channels).uniform_(-bound, bound, generator=generator)
    grad = torch.randn((config.batch, config.out_channels, *config.output), generator=generator)

    def cast(t):
        return None if t is None else t.to(dtype=config.dtype).to(device)

    return ConvInputs(cast(x), cast(weight), cast(bias), cast(grad))


# ------------------------------------------------------------------------------------
# c5: the three-layer training step
# ------------------------------------------------------------------------------------

C5_STEP_FLOPS = sum(layer.step_flops for layer in C5_LAYERS)  # 190.0 GFLOP per global batch


@dataclass
class C5Inputs:
    x: torch.Tensor
    target: torch.Tensor
    parameters: list  # [(weight, bias)] per layer, in layer order


def make_c5_inputs(device="cpu", rank: int = 0, world: int = 1) -> C5Inputs:
    """Seeded c5 inputs: x, then each layer's weight and bias, then the MSE target, all
    drawn on the CPU for the whole global batch; rank `rank` of `world` keeps its
    contiguous batch shard (the first ``64 % world`` ranks one extra row)."""
    generator = torch.Generator().manual_seed(C5_LAYERS[0].seed)
    first = C5_LAYERS[0]
    x = torch.randn((C5_BATCH, first.in_channels, *first.spatial), generator=generator)
    parameters = []
    for layer in C5_LAYERS:
        fan_in = layer.in_channels // layer.groups * math.prod(layer.kernel)
        bound = 1.0 / math.sqrt(fan_in)
        weight = torch.empty(
            (layer.out_channels, layer.in_channels // layer.groups, *layer.kernel)
        ).uniform_(-bound, bound, generator=generator)
        bias = torch.empty(layer.out_channels).uniform_(-bound, bound, generator=generator)
        parameters.append((weight.to(first.dtype).to(device), bias.to(first.dtype).to(device)))
    last = C5_LAYERS[-1]
    target = torch.randn((C5_BATCH, last.out_channels, *last.output), generator=generator)
    base, extra = divmod(C5_BATCH, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return C5Inputs(x[start:stop].to(first.dtype).to(device),
                    target[start:stop].to(first.dtype).to(device), parameters)


def c5_network(conv_class, parameters, device=None, fused_gelu=False):
    """conv L1 -> GELU -> conv L2 -> GELU -> conv L3, built from `conv_class` (a ConvNd
    with the reference's constructor) and loaded with `parameters`. With `fused_gelu` the
    GELUs run inside L1's and L2's convolutions (ConvNd(..., activation='gelu'))."""
    layers = []
    for index, (layer, (weight, bias)) in enumerate(zip(C5_LAYERS, parameters, strict=True)):
        last = index + 1 == len(C5_LAYERS)
        extra = {"activation": "gelu"} if fused_gelu and not last else {}
        conv = conv_class(layer.in_channels, layer.out_channels, layer.kernel, layer.stride,
                          layer.padding, layer.dilation, layer.groups, bias=True,
                          device=device, dtype=layer.dtype, dimensions=layer.rank, **extra)
        with torch.no_grad():
            conv.weight.copy_(weight)
            conv.bias.copy_(bias)
        layers.append(conv)
        if not last and not fused_gelu:
            layers.append(torch.nn.GELU())
    return torch.nn.Sequential(*layers)
