"""Context-parallel causal_conv1d: the sequence dimension split across ranks.

Rank r of the group holds the r-th contiguous slice of the sequence, x_r of shape
(batch, dim, L_r) with L_r >= width - 1.  The convolution looks W-1 positions back, so:

* forward: every rank sends the last W-1 positions of its slice to rank r+1, which
  uses them as ``initial_states`` (rank 0 has none, or the caller's initial states);
* backward: the kernel returns ``dinitial_states``, the gradient with respect to those
  W-1 positions of rank r-1's slice; it goes back to rank r-1 and is added to the tail of
  that rank's dx.  dweight/dbias of each slice are partial sums and are summed over the
  group (one all-reduce of a flat fp32 buffer, or the rank-ordered reduction).

Both halo exchanges are one point-to-point message of batch * dim * (W-1) elements per
neighbour pair (NCCL send/recv over NVLink on GPUs).  This is the long-context scaling
path named in the reference's states API (initial_states / dinitial_states,
``causal_conv1d/causal_conv1d_interface.py:37-52`` and ``cpp_functions.py:115-166``); the
reference itself has no multi-device code.

The dx tail of rank r-1 receives rank r's contribution as a separate addition in x's
dtype: those W-1 positions per row carry one extra rounding compared with a
single-device run.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from causal_conv1d.cpp_functions import causal_conv1d_bwd_function, causal_conv1d_fwd_function
from causal_conv1d.distributed import GradBucket, allreduce_param_grads

# The launches the autograd function makes; host-logic tests on CPU substitute them.
_fwd_impl = causal_conv1d_fwd_function
_bwd_impl = causal_conv1d_bwd_function


def _peer(group, rank):
    return rank if group is None else dist.get_global_rank(group, rank)


def _exchange(t_send: torch.Tensor | None, shape, like: torch.Tensor, group, to_next: bool):
    """Send ``t_send`` to the next (``to_next``) or previous rank and receive the tensor
    of ``shape`` that the rank on the other side sends; returns it (None at the group's
    edge)."""
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    dst = rank + 1 if to_next else rank - 1
    src = rank - 1 if to_next else rank + 1
    ops, recv = [], None
    if 0 <= src < world:
        recv = torch.empty(shape, dtype=like.dtype, device=like.device)
        ops.append(dist.P2POp(dist.irecv, recv, _peer(group, src), group))
    if 0 <= dst < world and t_send is not None:
        ops.append(dist.P2POp(dist.isend, t_send.contiguous(), _peer(group, dst), group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    return recv


def halo_from_previous(x: torch.Tensor, width: int, group=None) -> torch.Tensor | None:
    """The W-1 positions before this rank's slice, (batch, dim, W-1), from rank r-1
    (None on rank 0)."""
    b, d, _ = x.shape
    tail = x[:, :, x.shape[2] - (width - 1):]
    return _exchange(tail, (b, d, width - 1), x, group, to_next=True)


def dinitial_to_previous(dinitial: torch.Tensor | None, like: torch.Tensor, width: int, group=None):
    """Send this rank's dinitial_states to rank r-1 and receive rank r+1's (None on the
    last rank)."""
    b, d, _ = like.shape
    return _exchange(dinitial, (b, d, width - 1), like, group, to_next=False)


class CausalConv1dContextParallelFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, initial_states, activation, group, deterministic):
        width = weight.shape[1]
        if x.shape[2] < width - 1:
            raise ValueError("every rank's sequence slice needs at least width - 1 positions")
        silu = activation in ("silu", "swish")
        halo = halo_from_previous(x, width, group)
        init = halo if halo is not None else initial_states
        out = _fwd_impl(x, weight, bias, None, init, None, silu)
        ctx.save_for_backward(x, weight, bias, init)
        ctx.silu, ctx.group, ctx.deterministic = silu, group, deterministic
        ctx.halo = halo is not None
        ctx.user_init_grad = halo is None and initial_states is not None and initial_states.requires_grad
        return out

    @staticmethod
    def backward(ctx, dout):
        x, weight, bias, init = ctx.saved_tensors
        width = weight.shape[1]
        want_dinit = init is not None and (ctx.halo or ctx.user_init_grad)
        dx, dw, db, dinit = _bwd_impl(x, weight, bias, dout, None, init, None, None, want_dinit, ctx.silu)
        # rank r+1's gradient for the tail of this slice; this rank's goes to rank r-1
        from_next = dinitial_to_previous(dinit if ctx.halo else None, x, width, ctx.group)
        if from_next is not None:
            dx[:, :, dx.shape[2] - (width - 1):] += from_next.to(dx.dtype)
        bucket = GradBucket(weight.shape[0], width, bias is not None, x.device)
        bucket.dweight.copy_(dw)
        if bias is not None:
            bucket.dbias.copy_(db)
        allreduce_param_grads(bucket, ctx.group, ctx.deterministic)
        dw = bucket.dweight.to(weight.dtype)
        db = bucket.dbias.to(bias.dtype) if bias is not None else None
        dinit_user = dinit if ctx.user_init_grad else None
        return dx, dw, db, dinit_user, None, None, None


def causal_conv1d_fn_context_parallel(x, weight, bias=None, initial_states=None, activation=None, group=None,
                                      deterministic: bool = False):
    """causal_conv1d_fn over a sequence split across the ranks of ``group``.

    x: this rank's slice (batch, dim, L_r), slices in rank order, L_r >= width - 1;
    initial_states: used by rank 0 only.  Returns this rank's slice of the output.
    ``deterministic`` selects the rank-ordered reduction of dweight/dbias.
    """
    if activation not in (None, "silu", "swish"):
        raise NotImplementedError("activation must be None, silu, or swish")
    return CausalConv1dContextParallelFn.apply(x, weight, bias, initial_states, activation, group, deterministic)
