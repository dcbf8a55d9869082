"""Host dispatch onto the B200 kernels (same names and signatures as the reference's
``causal_conv1d/cpp_functions.py:64-238``).

Every layout and feature combination runs on CUDA kernels through the C ABI
(``include/causal_conv1d_b200.h``): channel-last and (batch, dim, seqlen) inputs,
``seq_idx``, ``initial_states``, ``final_states_out``, ``dfinal_states`` and
``dinitial_states``, circular / gathered / padded state updates.  There is no
PyTorch-op fallback; the functions raise if the CUDA library is unavailable.
"""

from __future__ import annotations

import os

import torch

from causal_conv1d import _abi


def _use_deterministic_mode() -> bool:
    """The reference's reduction-mode selector (``cutedsl_kernels.py:1466-1474``).

    ``CAUSAL_CONV1D_DETERMINISTIC`` starting with "1"/"0" wins, otherwise
    ``torch.are_deterministic_algorithms_enabled()``.  Kept for API compatibility: the
    B200 backward reduces dweight/dbias in a fixed order in both modes, so it is
    always deterministic.
    """
    value = os.environ.get("CAUSAL_CONV1D_DETERMINISTIC")
    if value:
        if value[0] == "1":
            return True
        if value[0] == "0":
            return False
    return torch.are_deterministic_algorithms_enabled()


def _like_layout(t: torch.Tensor, ref: torch.Tensor) -> torch.Tensor:
    """Return ``t`` with ``ref``'s fast layout (channel-last or contiguous rows)."""
    if ref.stride(1) == 1 and t.stride(1) != 1:
        return t.transpose(1, 2).contiguous().transpose(1, 2)
    if ref.stride(1) != 1 and ref.stride(2) == 1 and t.stride(2) != 1:
        return t.contiguous()
    return t


def causal_conv1d_fwd_function(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None,
    seq_idx: torch.Tensor | None,
    initial_states: torch.Tensor | None,
    final_states_out: torch.Tensor | None,
    silu_activation: bool,
) -> torch.Tensor:
    """Forward; writes ``final_states_out`` in place when given.  Returns ``out``
    (allocated like ``x``, strides preserved)."""
    if x.dim() != 3 or weight.dim() != 2 or weight.shape[0] != x.shape[1]:
        raise ValueError("x and weight must have shapes (batch, dim, seqlen) and (dim, width)")
    if weight.shape[1] not in (2, 3, 4):
        raise ValueError("weight must have shape (dim, width), with width in {2, 3, 4}")
    if bias is not None and bias.shape != (x.shape[1],):
        raise ValueError("bias must have shape (dim,)")
    out = torch.empty_like(x)
    _abi.fwd(x, weight, bias, seq_idx, initial_states, final_states_out, out, silu_activation)
    return out


def causal_conv1d_bwd_function(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None,
    dout: torch.Tensor,
    seq_idx: torch.Tensor | None,
    initial_states: torch.Tensor | None,
    dfinal_states: torch.Tensor | None,
    dx: torch.Tensor | None,
    return_dinitial_states: bool,
    silu_activation: bool,
):
    """Backward.  Returns ``(dx, dweight, dbias, dinitial_states)``: dx in x's dtype
    (``dx`` is filled in place when given), dweight/dbias in the parameter dtypes,
    dinitial_states in the initial-states dtype when requested."""
    if weight.shape[1] not in (2, 3, 4):
        raise ValueError("weight must have shape (dim, width), with width in {2, 3, 4}")
    dout = _like_layout(dout, x)
    if dx is None:
        dx = torch.empty_like(x)
    dim, width = weight.shape
    dweight = torch.empty(dim, width, device=x.device, dtype=torch.float32)
    dbias = torch.empty(dim, device=x.device, dtype=torch.float32) if bias is not None else None
    dinitial = None
    if initial_states is not None and return_dinitial_states:
        dinitial = torch.empty_like(initial_states)
    _abi.bwd(x, weight, bias, dout, seq_idx, initial_states, dfinal_states, dx, dinitial,
             dweight, dbias, silu_activation)
    return (
        dx,
        dweight if weight.dtype == torch.float32 else dweight.to(weight.dtype),
        None if dbias is None else (dbias if bias.dtype == torch.float32 else dbias.to(bias.dtype)),
        dinitial,
    )


def causal_conv1d_update_function(
    x: torch.Tensor,
    conv_state: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None,
    silu_activation: bool,
    cache_seqlens: torch.Tensor | None,
    conv_state_indices: torch.Tensor | None,
) -> torch.Tensor:
    """State update for x of shape (batch, dim, seqlen); mutates ``conv_state``."""
    if weight.shape[1] not in (2, 3, 4):
        raise ValueError("width must be 2, 3, or 4")
    if conv_state.shape[2] < weight.shape[1] - 1:
        raise ValueError("conv_state is shorter than the convolution history")
    if cache_seqlens is not None and cache_seqlens.dtype != torch.int32:
        cache_seqlens = cache_seqlens.to(torch.int32)
    if conv_state_indices is not None and conv_state_indices.dtype != torch.int32:
        conv_state_indices = conv_state_indices.to(torch.int32)
    out = torch.empty_like(x)
    _abi.update(x, conv_state, weight, bias, cache_seqlens, conv_state_indices, out, silu_activation)
    return out
