"""Data-parallel training: batch shards plus averaged gradients equal one process.

Mirrors the reference's ``tests/test_distributed.py:54-82`` (two Gloo processes under
DDP match one process on the whole batch). On the CPU the three-layer network of the c5
configuration (conv, GELU, grouped dilated conv, GELU, 1x1 conv) is built from the fp64
oracle convolution, so the test checks the host side of data parallelism — batch
sharding, parameter broadcast, bucketed fp32 all-reduce started from gradient hooks,
averaging — exactly (1e-12). The GPU test runs the same step on two B200s over NCCL with
the native bf16 operators and compares with a one-GPU run on the whole batch.
"""

from __future__ import annotations

import datetime
import math

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from torch import nn

from oracle import convnd_oracle as oracle
from torch_convnd import data_parallel

WORLD = 2

# Reduced c5 geometry: same kernels, strides, paddings, dilations, groups and channel
# ratios as the reference config's three layers, smaller batch, channels and extents.
LAYERS = (
    dict(cin=4, cout=8, kernel=(3, 3, 3, 3), stride=(2, 2, 2, 2), padding=(1, 1, 1, 1),
         dilation=(1, 1, 1, 1), groups=1),
    dict(cin=8, cout=8, kernel=(3, 3, 1, 1), stride=(1, 1, 1, 1), padding=(2, 2, 0, 0),
         dilation=(2, 2, 1, 1), groups=4),
    dict(cin=8, cout=2, kernel=(1, 1, 1, 1), stride=(1, 1, 1, 1), padding=(0, 0, 0, 0),
         dilation=(1, 1, 1, 1), groups=1),
)
BATCH = 4
SPATIAL = (6, 6, 4, 4)


def gloo_available():
    if not dist.is_available() or not dist.is_gloo_available():
        return False
    try:
        dist.ProcessGroupGloo.create_default_device()
    except RuntimeError:
        return False
    return True


class _OracleConv(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, geometry):
        ctx.save_for_backward(x, w)
        ctx.geometry = geometry
        return oracle.forward(x, w, b, *geometry)

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dx, dw, db = oracle.backward(dy, x, w, *ctx.geometry)
        return dx, dw, db, None


class OracleConv(nn.Module):
    def __init__(self, cin, cout, kernel, stride, padding, dilation, groups):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(cout, cin // groups, *kernel, dtype=torch.float64))
        self.bias = nn.Parameter(torch.empty(cout, dtype=torch.float64))
        self.geometry = (stride, padding, dilation, groups)
        bound = 1 / math.sqrt(cin // groups * math.prod(kernel))
        nn.init.uniform_(self.weight, -bound, bound)
        nn.init.uniform_(self.bias, -bound, bound)

    def forward(self, x):
        return _OracleConv.apply(x, self.weight, self.bias, self.geometry)


def oracle_network(seed):
    torch.manual_seed(seed)
    return nn.Sequential(OracleConv(**LAYERS[0]), nn.GELU(), OracleConv(**LAYERS[1]),
                         nn.GELU(), OracleConv(**LAYERS[2]))


def batch(dtype=torch.float64, rows=BATCH, seed=7):
    generator = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, LAYERS[0]["cin"], *SPATIAL, generator=generator)
    out = oracle.output_shape(SPATIAL, LAYERS[0]["kernel"], LAYERS[0]["stride"],
                              LAYERS[0]["padding"], LAYERS[0]["dilation"])
    target = torch.randn(rows, LAYERS[2]["cout"], *out, generator=generator)
    return x.to(dtype), target.to(dtype)


def full_batch_gradients(network, rows=BATCH, micro_batches=(7,)):
    """Gradients of the mean loss over the whole batch, summed over micro-batches."""
    network.zero_grad(set_to_none=True)
    for seed in micro_batches:
        x, target = batch(rows=rows, seed=seed)
        nn.functional.mse_loss(network(x), target).backward()
    return {name: p.grad.clone() for name, p in network.named_parameters()}


# ------------------------------------------------------------------------------------
# host logic
# ------------------------------------------------------------------------------------

def test_shard_bounds_cover_the_batch_contiguously():
    for batch_size in (2, 5, 64, 67):
        for world in (1, 2, 3, 4, 8):
            if batch_size < world:
                continue
            bounds = [data_parallel.shard_bounds(batch_size, r, world) for r in range(world)]
            assert bounds[0][0] == 0 and bounds[-1][1] == batch_size
            assert all(a[1] == b[0] for a, b in zip(bounds, bounds[1:]))
            sizes = [b - a for a, b in bounds]
            assert max(sizes) - min(sizes) <= 1
    assert data_parallel.shard_bounds(64, 3, 8) == (24, 32)


def test_shard_rejects_worlds_larger_than_the_batch():
    with pytest.raises(ValueError, match="cannot be split"):
        data_parallel.shard_bounds(2, 0, 4)
    with pytest.raises(ValueError, match="outside a world"):
        data_parallel.shard_bounds(8, 2, 2)


def test_bucketer_single_process_leaves_gradients_unchanged():
    network = oracle_network(0)
    expected = full_batch_gradients(network)
    network.zero_grad(set_to_none=False)
    bucketer = data_parallel.GradientBucketer(network.parameters(), bucket_bytes=512)
    assert len(bucketer.bucket_sizes) > 1
    x, target = batch()
    nn.functional.mse_loss(network(x), target).backward()
    bucketer.finish()
    for name, p in network.named_parameters():
        torch.testing.assert_close(p.grad, expected[name], rtol=0, atol=0)


def _train_cpu(rank, store, path):
    dist.init_process_group("gloo", init_method=store, rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=120))
    try:
        results = {}
        for overlap, bucket_bytes in ((True, 512), (False, 4 << 20)):
            network = oracle_network(seed=rank)  # different on purpose: broadcast fixes it
            data_parallel.broadcast_parameters(network)
            bucketer = data_parallel.GradientBucketer(network.parameters(),
                                                      bucket_bytes=bucket_bytes,
                                                      overlap=overlap)
            x, target = batch()
            x = data_parallel.shard(x, rank, WORLD)
            target = data_parallel.shard(target, rank, WORLD)
            for _ in range(2):  # a second step re-arms the hooks
                network.zero_grad(set_to_none=True)
                nn.functional.mse_loss(network(x), target).backward()
                bucketer.finish()
            bucketer.remove_hooks()
            results[(overlap, bucket_bytes)] = (
                {n: p.detach().clone() for n, p in network.named_parameters()},
                {n: p.grad.clone() for n, p in network.named_parameters()})
        if rank == 0:
            torch.save(results, path)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not gloo_available(), reason="torch.distributed has no usable Gloo device")
def test_two_gloo_ranks_match_one_process_on_the_whole_batch(tmp_path):
    path = tmp_path / "grads.pt"
    mp.spawn(_train_cpu, args=((tmp_path / "store").as_uri(), str(path)), nprocs=WORLD,
             join=True)
    results = torch.load(path)
    reference = oracle_network(seed=0)
    expected = full_batch_gradients(reference)
    for (overlap, bucket_bytes), (params, grads) in results.items():
        for name, p in reference.named_parameters():
            torch.testing.assert_close(params[name], p.detach(), rtol=0, atol=0)
            torch.testing.assert_close(grads[name], expected[name], rtol=1e-12, atol=1e-12,
                                       msg=f"{name} overlap={overlap} bucket={bucket_bytes}")


def test_layer_groups_make_one_bucket_per_layer():
    network = oracle_network(0)
    bucketer = data_parallel.GradientBucketer(data_parallel.layer_groups(network))
    # reverse layer order, weight and bias of a layer together
    assert bucketer.bucket_sizes == [16 + 2, 144 + 8, 2592 + 8]


def test_second_backward_without_no_sync_is_an_error():
    """A second backward before finish() would drop a micro-batch; it raises instead."""
    network = oracle_network(0)
    bucketer = data_parallel.GradientBucketer(data_parallel.layer_groups(network))
    bucketer.overlap = True  # single process: exercise the hook bookkeeping directly
    for group in data_parallel.layer_groups(network):
        for p in group:
            bucketer._handles.append(p.register_post_accumulate_grad_hook(bucketer._ready))
    bucketer._launch = lambda bucket: None
    x, target = batch()
    nn.functional.mse_loss(network(x), target).backward()
    with pytest.raises(RuntimeError, match="no_sync"):
        nn.functional.mse_loss(network(x), target).backward()
    network.zero_grad(set_to_none=True)
    bucketer.finish()
    with bucketer.no_sync():
        nn.functional.mse_loss(network(x), target).backward()
    nn.functional.mse_loss(network(x), target).backward()  # the step's last micro-batch
    bucketer.remove_hooks()


def _train_uneven(rank, world, rows, store, path):
    dist.init_process_group("gloo", init_method=store, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        network = oracle_network(seed=0)
        fraction = data_parallel.shard_fraction(rows, rank, world)
        bucketer = data_parallel.GradientBucketer(data_parallel.layer_groups(network),
                                                  batch_fraction=fraction)
        network.zero_grad(set_to_none=True)
        # two micro-batches: the first accumulates only, the second starts the reduction
        for index, seed in enumerate((7, 8)):
            x, target = batch(rows=rows, seed=seed)
            x = data_parallel.shard(x, rank, world)
            target = data_parallel.shard(target, rank, world)
            loss = nn.functional.mse_loss(network(x), target)
            if index == 0:
                with bucketer.no_sync():
                    loss.backward()
            else:
                loss.backward()
        bucketer.finish()
        bucketer.remove_hooks()
        if rank == 0:
            torch.save({n: p.grad.clone() for n, p in network.named_parameters()}, path)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not gloo_available(), reason="torch.distributed has no usable Gloo device")
def test_three_gloo_ranks_uneven_shards_and_accumulation(tmp_path):
    """Batch 5 over 3 ranks (shards 2, 2, 1) with two accumulated micro-batches equals
    one process's gradient of the two whole-batch mean losses."""
    rows, world = 5, 3
    path = tmp_path / "grads.pt"
    mp.spawn(_train_uneven, args=(world, rows, (tmp_path / "store").as_uri(), str(path)),
             nprocs=world, join=True)
    grads = torch.load(path)
    expected = full_batch_gradients(oracle_network(seed=0), rows=rows, micro_batches=(7, 8))
    for name, value in expected.items():
        torch.testing.assert_close(grads[name], value, rtol=1e-12, atol=1e-12, msg=name)


# ------------------------------------------------------------------------------------
# two B200s over NCCL
# ------------------------------------------------------------------------------------

def _native_network(device):
    import torch_convnd

    torch.manual_seed(0)
    layers = []
    for index, spec in enumerate(LAYERS):
        layers.append(torch_convnd.ConvNd(spec["cin"], spec["cout"], spec["kernel"],
                                          spec["stride"], spec["padding"], spec["dilation"],
                                          spec["groups"], device=device, dtype=torch.bfloat16,
                                          dimensions=4))
        if index + 1 < len(LAYERS):
            layers.append(nn.GELU())
    return nn.Sequential(*layers)


def _train_gpu(rank, store, path):
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=store, rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=120), device_id=device)
    try:
        network = _native_network(device)
        data_parallel.broadcast_parameters(network)
        bucketer = data_parallel.GradientBucketer(network.parameters(), bucket_bytes=1024)
        x, target = (t.to(device) for t in batch(torch.bfloat16))
        x = data_parallel.shard(x, rank, WORLD)
        target = data_parallel.shard(target, rank, WORLD)
        nn.functional.mse_loss(network(x), target).backward()
        bucketer.finish()
        torch.cuda.synchronize()
        grads = {n: p.grad.detach().cpu() for n, p in network.named_parameters()}
        dist.barrier()
        if rank == 0:
            torch.save(grads, path)
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs two GPUs")
def test_two_nccl_ranks_match_one_gpu_on_the_whole_batch(tmp_path):
    from tolerances import assert_matches

    path = tmp_path / "grads.pt"
    mp.spawn(_train_gpu, args=((tmp_path / "store").as_uri(), str(path)), nprocs=WORLD,
             join=True)
    distributed = torch.load(path)
    network = _native_network(torch.device("cuda", 0))
    x, target = (t.cuda() for t in batch(torch.bfloat16))
    nn.functional.mse_loss(network(x), target).backward()
    for name, p in network.named_parameters():
        assert_matches(distributed[name], p.grad.double().cpu(), torch.bfloat16,
                       f"data-parallel {name}")
