"""Data-parallel sharding of the causal_conv1d hot path (one process per GPU).

Every (batch, channel) row of the operator is independent, so:

* forward and update shard over batch or channels with no collective;
* backward sharded over batch leaves each rank with a partial dweight/dbias; one
  ``all_reduce(SUM)`` of a flat fp32 buffer ``[dim * width + dim]`` (dweight | dbias)
  over NCCL completes them.  The kernels reduce their own shard in a fixed order, so the
  result is reproducible for a fixed world size and NCCL algorithm.

The reference has no multi-device code; this module is the B200 addition.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from causal_conv1d import _abi
from causal_conv1d.cpp_functions import _like_layout


def shard_range(n: int, world: int, rank: int, multiple: int = 1) -> tuple[int, int]:
    """Contiguous [start, stop) of ``n`` items for ``rank`` of ``world``.

    Shards are balanced to within ``multiple`` items and start on multiples of
    ``multiple`` (use 8 for channel shards so 16-byte packets stay aligned).
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    units = (n + multiple - 1) // multiple
    base, extra = divmod(units, world)
    start_u = rank * base + min(rank, extra)
    stop_u = start_u + base + (1 if rank < extra else 0)
    return min(n, start_u * multiple), min(n, stop_u * multiple)


class GradBucket:
    """One fp32 allocation holding dweight (dim, width) and dbias (dim,) views, so the
    parameter gradients cross NVLink in a single collective."""

    def __init__(self, dim: int, width: int, has_bias: bool, device):
        self.dim, self.width, self.has_bias = dim, width, has_bias
        self.flat = torch.empty(dim * width + (dim if has_bias else 0), dtype=torch.float32, device=device)
        self.dweight = self.flat[: dim * width].view(dim, width)
        self.dbias = self.flat[dim * width:] if has_bias else None


def allreduce_param_grads(bucket: GradBucket, group=None, deterministic: bool = False) -> None:
    """Sum the bucket over the process group (no-op without an initialised group).

    ``deterministic=True`` gathers every rank's partial sums and adds them locally in
    rank order, so the result is bit-identical on every rank and from run to run
    whatever algorithm the collective library picks; the default is one all-reduce.
    """
    if not (dist.is_available() and dist.is_initialized()):
        return
    world = dist.get_world_size(group)
    if world <= 1:
        return
    if not deterministic:
        dist.all_reduce(bucket.flat, op=dist.ReduceOp.SUM, group=group)
        return
    n = bucket.flat.numel()
    parts = torch.empty(world * n, dtype=bucket.flat.dtype, device=bucket.flat.device)
    dist.all_gather_into_tensor(parts, bucket.flat, group=group)
    parts = parts.view(world, n)
    total = parts[0].clone()
    for r in range(1, world):
        total += parts[r]
    bucket.flat.copy_(total)


def causal_conv1d_bwd_batch_sharded(x, weight, bias, dout, seq_idx=None, initial_states=None,
                                    dfinal_states=None, silu_activation=False, return_dinitial_states=False,
                                    bucket: GradBucket | None = None, group=None, allreduce=True,
                                    deterministic: bool = False):
    """Backward of this rank's batch shard, then the dweight/dbias all-reduce.

    Returns ``(dx, dweight, dbias, dinitial_states)`` like
    ``cpp_functions.causal_conv1d_bwd_function``; dweight/dbias are the sums over all
    ranks, in the parameter dtypes.
    """
    dim, width = weight.shape
    if bucket is None:
        bucket = GradBucket(dim, width, bias is not None, x.device)
    dout = _like_layout(dout, x)
    dx = torch.empty_like(x)
    dinitial = None
    if initial_states is not None and return_dinitial_states:
        dinitial = torch.empty_like(initial_states)
    _abi.bwd(x, weight, bias, dout, seq_idx, initial_states, dfinal_states, dx, dinitial,
             bucket.dweight, bucket.dbias, silu_activation)
    if allreduce:
        allreduce_param_grads(bucket, group, deterministic)
    dw = bucket.dweight if weight.dtype == torch.float32 else bucket.dweight.to(weight.dtype)
    db = None
    if bias is not None:
        db = bucket.dbias if bias.dtype == torch.float32 else bucket.dbias.to(bias.dtype)
    return dx, dw, db, dinitial
