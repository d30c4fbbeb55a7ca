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
* ``finish()`` waits for the collectives, divides by the world size and writes the
  averaged values back into ``param.grad``.

With NCCL the all-reduce runs on NCCL's own stream, ordered after the work queued on
the current stream when it is issued; with Gloo (CPU tests) it runs synchronously.
"""

from __future__ import annotations

from collections.abc import Iterable, Sequence

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

    Parameters are grouped into buckets of at most `bucket_bytes` (counted in the
    reduction dtype; one dtype and device per bucket) in reverse registration order, the
    order in which backward produces their gradients for a sequential network. With
    ``overlap=True`` each bucket's all-reduce starts from the gradient hook of its last
    parameter; otherwise all buckets are reduced in ``finish()``. Call ``finish()`` once
    per step after ``backward()``.
    """

    def __init__(self, parameters: Iterable[torch.nn.Parameter], group=None,
                 bucket_bytes: int = 4 << 20, overlap: bool = True):
        params = [p for p in parameters if p.requires_grad]
        if not params:
            raise ValueError("no parameters require a gradient")
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.overlap = overlap and self.world > 1
        self.buckets: list[_Bucket] = []
        current: list[torch.nn.Parameter] = []
        size = 0
        for p in reversed(params):
            nbytes = p.numel() * _reduce_dtype(p.dtype).itemsize
            if current and (size + nbytes > bucket_bytes or p.dtype != current[0].dtype
                            or p.device != current[0].device):
                self.buckets.append(_Bucket(current))
                current, size = [], 0
            current.append(p)
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
        bucket = self._owner[id(param)]
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
            bucket.work = dist.all_reduce(bucket.flat, group=self.group, async_op=True)

    # -- per step ----------------------------------------------------------------------
    def finish(self) -> None:
        """Completes every bucket's reduction and writes the averaged gradients back."""
        if self.world == 1:
            return
        for bucket in self.buckets:
            if bucket.work is None and (not self.overlap or bucket.pending > 0):
                self._launch(bucket)
            if bucket.work is not None:
                bucket.work.wait()
                bucket.work = None
            bucket.flat.div_(self.world)
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
