"""PyTorch operator registrations:
``torch.ops.causal_conv1d.{fwd,bwd,update,varlen_states,fwd_varlen_states}``.

The same launches as :mod:`causal_conv1d.cpp_functions`, registered as custom operators
with their mutated arguments declared (``final_states_out`` of ``fwd``, ``conv_state`` of
``update``) and shape-only fake implementations.  ``torch.compile``, FakeTensor tracing
and ``torch.library.opcheck`` can therefore see through the kernels without running
them.

* ``fwd(x, weight, bias, seq_idx, initial_states, final_states_out, silu) -> out``
* ``bwd(x, weight, bias, dout, seq_idx, initial_states, dfinal_states,
  return_dinitial_states, silu) -> (dx, dweight, dbias, dinitial_states)``.  A custom
  operator cannot return None, so ``dbias`` and ``dinitial_states`` are empty tensors
  when there is no bias or no initial-state gradient.
* ``update(x, conv_state, weight, bias, silu, cache_seqlens, conv_state_indices) -> out``
* ``varlen_states(x, cu_seqlens, state_len) -> states``
* ``fwd_varlen_states(x, weight, bias, seq_idx, cu_seqlens, state_len, silu) -> (out, states)``

The reference compiles its kernels with the CuTe DSL and registers no torch operators;
these registrations are this package's equivalent of the C++ extension's op table.
"""

from __future__ import annotations

import torch
from torch import Tensor

from causal_conv1d import cpp_functions as _cf
from causal_conv1d.causal_conv1d_varlen import causal_conv1d_fn_varlen_states as _fwd_varlen_states
from causal_conv1d.causal_conv1d_varlen import causal_conv1d_varlen_states as _varlen_states

_EMPTY = (0,)


@torch.library.custom_op("causal_conv1d::fwd", mutates_args=("final_states_out",))
def fwd(x: Tensor, weight: Tensor, bias: Tensor | None, seq_idx: Tensor | None,
        initial_states: Tensor | None, final_states_out: Tensor | None, silu: bool) -> Tensor:
    return _cf.causal_conv1d_fwd_function(x, weight, bias, seq_idx, initial_states, final_states_out, silu)


@fwd.register_fake
def _(x, weight, bias, seq_idx, initial_states, final_states_out, silu):
    return torch.empty_like(x)


@torch.library.custom_op("causal_conv1d::bwd", mutates_args=())
def bwd(x: Tensor, weight: Tensor, bias: Tensor | None, dout: Tensor, seq_idx: Tensor | None,
        initial_states: Tensor | None, dfinal_states: Tensor | None, return_dinitial_states: bool,
        silu: bool) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    dx, dw, db, di = _cf.causal_conv1d_bwd_function(x, weight, bias, dout, seq_idx, initial_states,
                                                    dfinal_states, None, return_dinitial_states, silu)
    if db is None:
        db = x.new_empty(_EMPTY, dtype=weight.dtype)
    if di is None:
        di = x.new_empty(_EMPTY)
    return dx, dw, db, di


@bwd.register_fake
def _(x, weight, bias, dout, seq_idx, initial_states, dfinal_states, return_dinitial_states, silu):
    dx = torch.empty_like(x)
    dw = torch.empty_like(weight, memory_format=torch.contiguous_format)
    db = torch.empty_like(bias) if bias is not None else x.new_empty(_EMPTY, dtype=weight.dtype)
    if initial_states is not None and return_dinitial_states:
        di = torch.empty_like(initial_states)
    else:
        di = x.new_empty(_EMPTY)
    return dx, dw, db, di


@torch.library.custom_op("causal_conv1d::update", mutates_args=("conv_state",))
def update(x: Tensor, conv_state: Tensor, weight: Tensor, bias: Tensor | None, silu: bool,
           cache_seqlens: Tensor | None, conv_state_indices: Tensor | None) -> Tensor:
    return _cf.causal_conv1d_update_function(x, conv_state, weight, bias, silu, cache_seqlens,
                                             conv_state_indices)


@update.register_fake
def _(x, conv_state, weight, bias, silu, cache_seqlens, conv_state_indices):
    return torch.empty_like(x)


@torch.library.custom_op("causal_conv1d::varlen_states", mutates_args=())
def varlen_states(x: Tensor, cu_seqlens: Tensor, state_len: int) -> Tensor:
    return _varlen_states(x, cu_seqlens, state_len)


@varlen_states.register_fake
def _(x, cu_seqlens, state_len):
    batch = cu_seqlens.shape[0] - 1
    return x.new_empty(batch, state_len, x.shape[1]).transpose(1, 2)


@torch.library.custom_op("causal_conv1d::fwd_varlen_states", mutates_args=())
def fwd_varlen_states(x: Tensor, weight: Tensor, bias: Tensor | None, seq_idx: Tensor | None,
                      cu_seqlens: Tensor, state_len: int, silu: bool) -> tuple[Tensor, Tensor]:
    return _fwd_varlen_states(x, weight, cu_seqlens, state_len, bias, seq_idx, "silu" if silu else None)


@fwd_varlen_states.register_fake
def _(x, weight, bias, seq_idx, cu_seqlens, state_len, silu):
    nseq = cu_seqlens.shape[0] - 1
    out = torch.empty_like(x) if (x.stride(2) == 1 or x.stride(1) == 1) else torch.empty_like(x.contiguous())
    return out, x.new_empty(nseq, state_len, x.shape[1]).transpose(1, 2)
