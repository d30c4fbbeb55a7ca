"""Batch-sharded data parallelism for training steps built on the N-D convolution.

One process per GPU. Every rank convolves a contiguous shard of the global batch with
its own copy of the parameters; after backward the parameter gradients are summed over
the ranks and divided by the world size, so every rank ends the step with the gradient
of the global-batch mean loss. The reference checks exactly this property with
``torch.nn.parallel.DistributedDataParallel`` on two Gloo processes
(``tests/test_distributed.py:54-82``); here the exchange is written out:

* gradients are reduced in flat buckets of at least fp32 precision (bf16/fp16
  gradients in fp32, fp64 ones in fp64), so the sum over ranks adds no bf16 rounding
  beyond the one cast of each rank's own gradient;
* a bucket's all-reduce is started from a post-accumulate-grad hook as soon as every
  parameter in it has its gradient, so the collective of a late layer (the first to
  finish backward) overlaps the backward kernels of the layers before it;
* ``finish()`` waits for the collectives and writes the averaged values back into
  ``param.grad``. Each rank's gradient is weighted by its share of the global batch
  (``batch_fraction``; 1/world for even shards) before the sum, so uneven shards, where
  the first ``batch % world`` ranks hold one extra row, still give the gradient of the
  global-batch mean loss;
* gradient accumulation over several backward passes per step uses ``no_sync()`` for
  all but the last micro-batch; a second backward outside it before ``finish()`` is an
  error rather than a silently dropped micro-batch.

With NCCL the all-reduce runs on NCCL's own stream, ordered after the work queued on
the current stream when it is issued; with Gloo (CPU tests) it runs synchronously.
"""

from __future__ import annotations

import contextlib
from collections.abc import Sequence

import torch
import torch.distributed as dist


def shard_bounds(batch: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, stop) rows of a batch for `rank`; the first ``batch % world``
    ranks take one extra row. Raises when a rank would get no rows."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} is outside a world of {world}")
    if batch < world:
        raise ValueError(
            f"a batch of {batch} cannot be split across {world} ranks (each needs a row)")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard(tensor: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's contiguous shard of `tensor` along the batch dimension (a view)."""
    start, stop = shard_bounds(tensor.shape[0], rank, world)
    return tensor[start:stop]


def shard_fraction(batch: int, rank: int, world: int) -> float:
    """`rank`'s share of a batch split by ``shard_bounds``: the weight of its mean-loss
    gradient in the gradient of the global-batch mean loss."""
    start, stop = shard_bounds(batch, rank, world)
    return (stop - start) / batch


def layer_groups(module: torch.nn.Module) -> list[list[torch.nn.Parameter]]:
    """Parameters grouped by the submodule that owns them directly, in registration order:
    one group per layer, whose gradients one backward call produces together."""
    groups = []
    for sub in module.modules():
        params = [p for p in sub.parameters(recurse=False) if p.requires_grad]
        if params:
            groups.append(params)
    return groups


def _reduce_dtype(dtype: torch.dtype) -> torch.dtype:
    return torch.promote_types(dtype, torch.float32)


class _Bucket:
    def __init__(self, params: list[torch.nn.Parameter]):
        self.params = params
        self.numel = sum(p.numel() for p in params)
        self.flat = torch.zeros(self.numel, dtype=_reduce_dtype(params[0].dtype),
                                device=params[0].device)
        self.pending = len(params)
        self.work = None


class GradientBucketer:
    """Averages parameter gradients across the ranks of a process group.

    `parameters` is an iterable of parameters, or of parameter groups (lists, e.g. from
    ``layer_groups(module)``; a group is never split across buckets). Groups are taken in
    reverse order, the order in which backward produces their gradients for a sequential
    network, and consecutive groups are merged while a bucket stays within `bucket_bytes`
    (counted in the reduction dtype; one dtype and device per bucket). The default of 0
    gives one bucket per group: per layer for ``layer_groups``, so the all-reduce of a
    late layer starts as soon as its weight and bias gradients exist. With
    ``overlap=True`` each bucket's all-reduce starts from the gradient hook of its last
    parameter; otherwise all buckets are reduced in ``finish()``.

    `batch_fraction` is this rank's share of the global batch (``shard_fraction``); each
    rank's gradients are scaled by it and summed. None means 1/world (even shards).
    Call ``finish()`` once per step after the last ``backward()``.
    """

    def __init__(self, parameters, group=None, bucket_bytes: int = 0, overlap: bool = True,
                 batch_fraction: float | None = None):
        groups = []
        for item in parameters:
            members = list(item) if isinstance(item, (list, tuple)) else [item]
            members = [p for p in members if p.requires_grad]
            if members:
                groups.append(members)
        if not groups:
            raise ValueError("no parameters require a gradient")
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.overlap = overlap and self.world > 1
        self.scale = 1.0 / self.world if batch_fraction is None else float(batch_fraction)
        self._sync = True
        self.buckets: list[_Bucket] = []
        current: list[torch.nn.Parameter] = []
        size = 0
        for members in reversed(groups):
            members = list(reversed(members))
            nbytes = sum(p.numel() * _reduce_dtype(p.dtype).itemsize for p in members)
            kind = (members[0].dtype, members[0].device)
            if any((p.dtype, p.device) != kind for p in members):
                raise ValueError("a parameter group mixes dtypes or devices")
            if current and (size + nbytes > bucket_bytes
                            or kind != (current[0].dtype, current[0].device)):
                self.buckets.append(_Bucket(current))
                current, size = [], 0
            current.extend(members)
            size += nbytes
        self.buckets.append(_Bucket(current))
        self._owner = {}
        self._handles = []
        for bucket in self.buckets:
            for p in bucket.params:
                self._owner[id(p)] = bucket
                if self.overlap:
                    self._handles.append(p.register_post_accumulate_grad_hook(self._ready))

    # -- hooks -------------------------------------------------------------------------
    def _ready(self, param: torch.nn.Parameter) -> None:
        if not self._sync:
            return
        bucket = self._owner[id(param)]
        if bucket.pending <= 0:
            raise RuntimeError(
                "GradientBucketer: backward() ran again before finish(); run the "
                "micro-batches that only accumulate gradients under no_sync()")
        bucket.pending -= 1
        if bucket.pending == 0:
            self._launch(bucket)

    def _launch(self, bucket: _Bucket) -> None:
        offset = 0
        for p in bucket.params:
            n = p.numel()
            if p.grad is None:
                bucket.flat[offset:offset + n].zero_()
            else:
                bucket.flat[offset:offset + n].copy_(p.grad.reshape(-1))
            offset += n
        if self.world > 1:
            bucket.flat.mul_(self.scale)
            bucket.work = dist.all_reduce(bucket.flat, group=self.group, async_op=True)

    # -- per step ----------------------------------------------------------------------
    @contextlib.contextmanager
    def no_sync(self):
        """Backward passes inside only accumulate into ``param.grad``; the reduction
        starts with the first backward after the block (the step's last micro-batch)."""
        previous = self._sync
        self._sync = False
        try:
            yield
        finally:
            self._sync = previous

    def finish(self) -> None:
        """Completes every bucket's reduction and writes the averaged gradients back."""
        if self.world == 1:
            for bucket in self.buckets:
                bucket.pending = len(bucket.params)
            return
        for bucket in self.buckets:
            if bucket.work is None and (not self.overlap or bucket.pending > 0):
                self._launch(bucket)
            if bucket.work is not None:
                bucket.work.wait()
                bucket.work = None
            offset = 0
            for p in bucket.params:
                n = p.numel()
                view = bucket.flat[offset:offset + n].view_as(p)
                if p.grad is None:
                    p.grad = view.to(p.dtype).clone()
                else:
                    p.grad.copy_(view)
                offset += n
            bucket.pending = len(bucket.params)

    def remove_hooks(self) -> None:
        for handle in self._handles:
            handle.remove()
        self._handles.clear()

    @property
    def bucket_sizes(self) -> Sequence[int]:
        return [b.numel for b in self.buckets]


def broadcast_parameters(module: torch.nn.Module, src: int = 0, group=None) -> None:
    """Makes every rank's parameters equal to rank `src`'s (the initial sync of DP)."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    with torch.no_grad():
        for p in module.parameters():
            dist.broadcast(p.data, src=src, group=group)
