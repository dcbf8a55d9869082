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
