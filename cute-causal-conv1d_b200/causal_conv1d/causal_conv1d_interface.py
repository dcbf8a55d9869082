"""Public API (reference ``causal_conv1d/causal_conv1d_interface.py``).

``causal_conv1d_fn`` / ``CausalConv1dFn`` and ``causal_conv1d_update`` keep the
reference's signatures, argument checks (``NotImplementedError`` for an unknown
activation, ``AssertionError`` for seq_idx with states and for non-channel-last final
states), output ownership and autograd contract.  ``causal_conv1d_ref`` and
``causal_conv1d_update_ref`` are PyTorch statements of the same operator, kept
importable for users' tests; the kernels never call them.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from causal_conv1d.cpp_functions import (
    causal_conv1d_bwd_function,
    causal_conv1d_fwd_function,
    causal_conv1d_update_function,
)

_ACTIVATIONS = (None, "silu", "swish")


def _check_activation(activation):
    if activation not in _ACTIVATIONS:
        raise NotImplementedError("activation must be None, silu, or swish")


class CausalConv1dFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias=None, seq_idx=None, initial_states=None,
                return_final_states=False, final_states_out=None, activation=None):
        _check_activation(activation)
        if x.stride(1) != 1 and x.stride(2) != 1:
            x = x.contiguous()
        if bias is not None:
            bias = bias.contiguous()
        if seq_idx is not None:
            assert initial_states is None, "initial_states must be None if seq_idx is not None"
            assert not return_final_states, "If seq_idx is not None, we don't return final_states_out"
            seq_idx = seq_idx.contiguous()
        if initial_states is not None and initial_states.stride(1) != 1 and initial_states.stride(2) != 1:
            initial_states = initial_states.contiguous()
        if return_final_states:
            assert x.stride(1) == 1, "Only channel-last layout support returning final_states_out"
            if final_states_out is not None:
                assert final_states_out.stride(1) == 1 or final_states_out.stride(2) == 1
            else:
                batch, dim, _ = x.shape
                final_states_out = torch.empty(
                    batch, weight.shape[1] - 1, dim, device=x.device, dtype=x.dtype
                ).transpose(1, 2)
        else:
            final_states_out = None
        silu = activation in ("silu", "swish")
        out = causal_conv1d_fwd_function(x, weight, bias, seq_idx, initial_states, final_states_out, silu)
        ctx.activation = silu
        ctx.return_final_states = return_final_states
        ctx.return_dinitial_states = initial_states is not None and initial_states.requires_grad
        ctx.save_for_backward(x, weight, bias, seq_idx, initial_states)
        return (out, final_states_out) if return_final_states else out

    @staticmethod
    def backward(ctx, dout, *args):
        x, weight, bias, seq_idx, initial_states = ctx.saved_tensors
        dfinal_states = args[0] if ctx.return_final_states else None
        if dout.stride(1) != 1 and dout.stride(2) != 1:
            dout = dout.contiguous()
        dx, dweight, dbias, dinitial = causal_conv1d_bwd_function(
            x, weight, bias, dout, seq_idx, initial_states, dfinal_states, None,
            ctx.return_dinitial_states, ctx.activation,
        )
        return (
            dx,
            dweight,
            dbias if bias is not None else None,
            None,
            dinitial if initial_states is not None else None,
            None,
            None,
            None,
        )


def causal_conv1d_fn(x, weight, bias=None, seq_idx=None, initial_states=None,
                     return_final_states=False, final_states_out=None, activation=None):
    """Depthwise causal conv1d with optional bias and SiLU.

    x: (batch, dim, seqlen); weight: (dim, width), width in {2, 3, 4}; bias: (dim,);
    seq_idx: (batch, seqlen) int32 packed-sequence ids; initial_states:
    (batch, dim, width - 1); final_states_out: (batch, dim, width - 1), written in place;
    activation: None, "silu" or "swish".  Returns out (batch, dim, seqlen), or
    (out, final_states) when return_final_states.
    """
    return CausalConv1dFn.apply(x, weight, bias, seq_idx, initial_states, return_final_states,
                                final_states_out, activation)


def causal_conv1d_ref(x, weight, bias=None, initial_states=None, return_final_states=False,
                      final_states_out=None, activation=None):
    """PyTorch statement of :func:`causal_conv1d_fn` (computes in weight's dtype)."""
    _check_activation(activation)
    in_dtype = x.dtype
    width = weight.shape[1]
    seqlen = x.shape[-1]
    h = x.to(weight.dtype)
    if initial_states is not None:
        h = torch.cat([initial_states.to(weight.dtype), h], dim=-1)
        pre = F.conv1d(h, weight.unsqueeze(1), bias, groups=weight.shape[0])
    else:
        pre = F.conv1d(h, weight.unsqueeze(1), bias, padding=width - 1, groups=weight.shape[0])
    pre = pre[..., :seqlen]
    out = (F.silu(pre) if activation is not None else pre).to(in_dtype)
    if not return_final_states:
        return out
    hist = F.pad(h, (width - 1 - h.shape[-1], 0)).to(in_dtype)
    if final_states_out is not None:
        final_states_out.copy_(hist)
    else:
        final_states_out = hist
    return out, final_states_out


def causal_conv1d_update(x, conv_state, weight, bias=None, activation=None, cache_seqlens=None,
                         conv_state_indices=None):
    """One decode step (or a few speculative tokens) against a rolling conv state.

    x: (batch, dim) or (batch, dim, seqlen); conv_state: (batch or state_batch, dim,
    state_len >= width - 1), updated in place; cache_seqlens: (batch,) int32, makes the
    state a circular buffer written at cache_seqlens % state_len; conv_state_indices:
    (batch,) int32 state rows (continuous batching), negative = padded row (zero output,
    no state write).  Returns out with x's shape.
    """
    _check_activation(activation)
    squeeze = x.dim() == 2
    if squeeze:
        x = x.unsqueeze(-1)
    out = causal_conv1d_update_function(x, conv_state, weight, bias, activation in ("silu", "swish"),
                                        cache_seqlens, conv_state_indices)
    return out.squeeze(-1) if squeeze else out


def causal_conv1d_update_ref(x, conv_state, weight, bias=None, activation=None, cache_seqlens=None):
    """PyTorch statement of :func:`causal_conv1d_update` (no index gather)."""
    _check_activation(activation)
    in_dtype = x.dtype
    squeeze = x.dim() == 2
    if squeeze:
        x = x.unsqueeze(-1)
    batch, dim, seqlen = x.shape
    width = weight.shape[1]
    state_len = conv_state.shape[-1]
    assert conv_state.shape == (batch, dim, state_len)
    assert weight.shape == (dim, width)
    if cache_seqlens is None:
        window = torch.cat([conv_state, x], dim=-1).to(weight.dtype)
        conv_state.copy_(window[:, :, -state_len:])
    else:
        base = cache_seqlens.to(torch.long).unsqueeze(1)
        hist_idx = torch.remainder(torch.arange(-(width - 1), 0, device=x.device).unsqueeze(0) + base, state_len)
        hist = conv_state.gather(2, hist_idx.unsqueeze(1).expand(-1, dim, -1))
        window = torch.cat([hist, x], dim=-1).to(weight.dtype)
        put_idx = torch.remainder(torch.arange(seqlen, device=x.device).unsqueeze(0) + base, state_len)
        conv_state.scatter_(2, put_idx.unsqueeze(1).expand(-1, dim, -1), x)
    out = F.conv1d(window, weight.unsqueeze(1), bias, groups=dim)[:, :, -seqlen:]
    if squeeze:
        out = out.squeeze(-1)
    return (F.silu(out) if activation is not None else out).to(in_dtype)
