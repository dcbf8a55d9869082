"""Varlen state gather (reference ``causal_conv1d/causal_conv1d_varlen.py``)."""

from __future__ import annotations

import torch
from torch import Tensor

from causal_conv1d import _abi


def causal_conv1d_varlen_states(x: Tensor, cu_seqlens: Tensor, state_len: int) -> Tensor:
    """Gather the last ``state_len`` tokens of each packed sequence.

    x: (total_tokens, dim) with contiguous channels; cu_seqlens: (batch + 1,) int32 or
    int64.  Returns (batch, dim, state_len) whose memory is (batch, state_len, dim):
    ``states[b, :, s] = x[cu[b+1] - state_len + s]`` when that token belongs to
    sequence b, else 0.  Bit-exact copy.
    """
    if x.ndim != 2 or x.stride(1) != 1:
        raise ValueError("x must have contiguous channels and shape (total_tokens, dim)")
    if cu_seqlens.dtype not in (torch.int32, torch.int64):
        raise TypeError("cu_seqlens must be int32 or int64")
    cu_seqlens = cu_seqlens.contiguous()
    batch = cu_seqlens.numel() - 1
    states = torch.empty(batch, state_len, x.shape[1], device=x.device, dtype=x.dtype).transpose(1, 2)
    _abi.varlen_states(x, cu_seqlens, states)
    return states


def causal_conv1d_fn_varlen_states(x: Tensor, weight: Tensor, cu_seqlens: Tensor, state_len: int,
                                   bias: Tensor | None = None, seq_idx: Tensor | None = None,
                                   activation: str | None = None) -> tuple[Tensor, Tensor]:
    """Prefill forward of packed sequences that also returns their decode states.

    For offsets that satisfy the precondition below, same results as the two calls
    ``out = causal_conv1d_fn(x, weight, bias, seq_idx=seq_idx, activation=activation)`` and
    ``states = causal_conv1d_varlen_states(x[0].transpose(0, 1), cu_seqlens, state_len)``
    (``causal_conv1d/causal_conv1d_interface.py:99-129`` and
    ``causal_conv1d/causal_conv1d_varlen.py:7-11`` in the reference), which a prefill
    makes before handing the states to ``causal_conv1d_update``.  With ``seq_idx`` and
    channel-last x, the forward kernel stores each sequence's last ``state_len`` rows
    while it streams x, so x is read once and there is no second launch; other inputs
    take the two launches.

    x: (1, dim, total_tokens), sequences packed along the last dimension;
    cu_seqlens: (nseq + 1,) int32 or int64 offsets into total_tokens, non-decreasing with
    the last entry <= total_tokens (precondition: for other offsets the states of the
    sequences concerned are unspecified, though nothing outside the given tensors is read
    or written); seq_idx: (1, total_tokens) int32 sequence ids.
    Returns ``(out, states)``: out like x, states (nseq, dim, state_len) whose memory is
    (nseq, state_len, dim).  An inference call: neither result has autograd history.
    """
    if activation not in (None, "silu", "swish"):
        raise NotImplementedError("activation must be None, silu, or swish")
    if x.dim() != 3 or x.shape[0] != 1:
        raise ValueError("x must have shape (1, dim, total_tokens): sequences packed along the last dimension")
    if weight.dim() != 2 or weight.shape[0] != x.shape[1] or weight.shape[1] not in (2, 3, 4):
        raise ValueError("weight must have shape (dim, width), with width in {2, 3, 4}")
    if bias is not None and bias.shape != (x.shape[1],):
        raise ValueError("bias must have shape (dim,)")
    if cu_seqlens.dim() != 1 or cu_seqlens.dtype not in (torch.int32, torch.int64):
        raise TypeError("cu_seqlens must be a 1-D int32 or int64 tensor")
    if state_len < 0:
        raise ValueError("state_len must be >= 0")
    if x.stride(2) != 1 and x.stride(1) != 1:
        x = x.contiguous()
    if bias is not None:
        bias = bias.contiguous()
    if seq_idx is not None:
        seq_idx = seq_idx.contiguous()
    cu_seqlens = cu_seqlens.contiguous()
    nseq = cu_seqlens.numel() - 1
    out = torch.empty_like(x)
    states = torch.empty(nseq, state_len, x.shape[1], device=x.device, dtype=x.dtype).transpose(1, 2)
    _abi.fwd_varlen_states(x, weight, bias, seq_idx, cu_seqlens, states, out, activation is not None)
    return out, states


def causal_conv1d_varlen_states_ref(x: Tensor, cu_seqlens: Tensor, state_len: int) -> Tensor:
    """PyTorch statement of :func:`causal_conv1d_varlen_states` (for users' tests)."""
    _, dim = x.shape
    batch = cu_seqlens.shape[0] - 1
    states = torch.zeros(batch, state_len, dim, dtype=x.dtype, device=x.device)
    cu = cu_seqlens.tolist()
    for b in range(batch):
        end = int(cu[b + 1])
        start = max(int(cu[b]), end - state_len)
        if end > start:
            states[b, state_len - (end - start):] = x[start:end]
    return states.transpose(1, 2)
