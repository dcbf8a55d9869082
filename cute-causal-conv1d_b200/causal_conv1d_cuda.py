"""``causal_conv1d_cuda``: the function table of the reference's legacy C++ extension.

Same names, argument order and output-argument convention as the pybind module the
reference builds from ``csrc/causal_conv1d.cpp:150-157,261-272,466-474,559-563``, so that
code which imports the extension directly keeps working.  The calls run the B200
kernels through the C ABI:

* ``causal_conv1d_fwd(x, weight, bias, seq_idx, initial_states, out, final_states_out,
  silu_activation)`` writes ``out`` (and ``final_states_out``);
* ``causal_conv1d_bwd(x, weight, bias, dout, seq_idx, initial_states, dfinal_states, dx,
  dweight, dbias, dinitial_states, silu_activation)`` writes ``dx`` and
  ``dinitial_states`` and **adds** into the fp32 ``dweight`` / ``dbias`` (the legacy
  kernels accumulate there with atomics; callers pass zeroed buffers);
* ``causal_conv1d_update(x, conv_state, weight, bias, out, silu_activation,
  cache_seqlens, conv_state_indices)`` writes ``out`` and updates ``conv_state``.

Argument errors raise RuntimeError, as the extension's TORCH_CHECKs do.
"""

from __future__ import annotations

import functools

import torch

from causal_conv1d import _abi
from causal_conv1d.cpp_functions import _like_layout


def _as_runtime_error(fn):
    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        try:
            return fn(*args, **kwargs)
        except (ValueError, TypeError, NotImplementedError) as e:
            raise RuntimeError(str(e)) from e

    return wrapper


@_as_runtime_error
def causal_conv1d_fwd(x, weight, bias, seq_idx, initial_states, out, final_states_out, silu_activation):
    _abi.fwd(x, weight, bias, seq_idx, initial_states, final_states_out, out, bool(silu_activation))


@_as_runtime_error
def causal_conv1d_bwd(x, weight, bias, dout, seq_idx, initial_states, dfinal_states, dx, dweight, dbias,
                      dinitial_states, silu_activation):
    if (bias is None) != (dbias is None):
        raise ValueError("bias and dbias must both be given or both be None")
    if dweight.dtype != torch.float32 or (dbias is not None and dbias.dtype != torch.float32):
        raise TypeError("dweight and dbias must be float32")
    dout = _like_layout(dout, x)
    dim, width = weight.shape
    dw = torch.empty(dim, width, device=x.device, dtype=torch.float32)
    db = torch.empty(dim, device=x.device, dtype=torch.float32) if bias is not None else None
    _abi.bwd(x, weight, bias, dout, seq_idx, initial_states, dfinal_states, dx, dinitial_states, dw, db,
             bool(silu_activation))
    dweight.add_(dw)
    if dbias is not None:
        dbias.add_(db)


@_as_runtime_error
def causal_conv1d_update(x, conv_state, weight, bias, out, silu_activation, cache_seqlens, conv_state_indices):
    squeeze = x.dim() == 2
    if squeeze:
        x, out = x.unsqueeze(-1), out.unsqueeze(-1)
    if cache_seqlens is not None and cache_seqlens.dtype != torch.int32:
        cache_seqlens = cache_seqlens.to(torch.int32)
    if conv_state_indices is not None and conv_state_indices.dtype != torch.int32:
        conv_state_indices = conv_state_indices.to(torch.int32)
    _abi.update(x, conv_state, weight, bias, cache_seqlens, conv_state_indices, out, bool(silu_activation))
