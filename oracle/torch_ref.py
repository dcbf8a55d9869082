"""PyTorch restatement of the reference's CPU path for timing (test infrastructure only).

``bench.py`` times the reference's own ``causal_conv1d_ref``
(``causal_conv1d/causal_conv1d_interface.py:132-171``) with an autograd backward as the
CPU baseline.  That function is imported from the installed reference when it is
present; this module is the stand-in when it is not: the same PyTorch operations in the
same order (upcast to the weight dtype, depthwise ``F.conv1d`` with ``groups=dim`` and
``padding=width-1``, the last ``seqlen`` outputs, SiLU, cast back to x's dtype), so the
timed CPU work is the same.  Only ``tests/`` and ``bench.py``'s CPU legs use it.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def causal_conv1d_ref(x, weight, bias=None, initial_states=None, return_final_states=False,
                      final_states_out=None, activation=None):
    """Forward of ``causal_conv1d_interface.py:132-171`` (the reference oracle)."""
    if activation not in (None, "silu", "swish"):
        raise NotImplementedError("activation must be None, silu, or swish")
    in_dtype = x.dtype
    h = x.to(weight.dtype)
    seqlen = h.shape[-1]
    dim, width = weight.shape
    if initial_states is None:
        pre = F.conv1d(h, weight.unsqueeze(1), bias, padding=width - 1, groups=dim)
    else:
        h = torch.cat([initial_states.to(weight.dtype), h], dim=-1)
        pre = F.conv1d(h, weight.unsqueeze(1), bias, padding=0, groups=dim)
    pre = pre[..., :seqlen]
    final = None
    if return_final_states:
        # a negative left pad crops: the last width-1 entries of [initial | x], zero-padded
        final = F.pad(h, (width - 1 - h.shape[-1], 0)).to(in_dtype)
        if final_states_out is not None:
            final_states_out.copy_(final)
            final = final_states_out
    out = (pre if activation is None else F.silu(pre)).to(in_dtype)
    return out if not return_final_states else (out, final)
