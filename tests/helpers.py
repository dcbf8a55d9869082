"""Helpers shared by the GPU parity tests: numpy storage <-> torch, memory layouts."""

from __future__ import annotations

import numpy as np
import torch

from oracle import numpy_oracle as O

TORCH_DT = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}
NAME_OF = {v: k for k, v in TORCH_DT.items()}


def to_torch(arr, dtype: str | None = None, device="cuda"):
    """Storage-form numpy array -> torch tensor (bf16 from uint16 bits)."""
    if arr is None:
        return None
    a = np.ascontiguousarray(arr)
    if dtype == "bfloat16" or a.dtype == np.uint16:
        t = torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
    else:
        t = torch.from_numpy(a.copy())
    return t.to(device)


def to_storage(t: torch.Tensor | None):
    """torch tensor -> storage-form numpy array (logical shape, contiguous)."""
    if t is None:
        return None
    t = t.detach().to("cpu").contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def f32(t: torch.Tensor | np.ndarray, dtype: str | None = None) -> np.ndarray:
    if isinstance(t, torch.Tensor):
        dtype = NAME_OF[t.dtype]
        t = to_storage(t)
    return O.to_f32(t, dtype)


def with_layout(t: torch.Tensor, layout: str) -> torch.Tensor:
    """Same logical (batch, dim, seqlen) values in a given memory layout.

    contiguous     (batch, dim, seqlen) dense
    channel_last   (batch, seqlen, dim) dense, viewed as (batch, dim, seqlen)
    cl_slice       channel-last slice [..., 64:64+dim] of a wider (batch, seqlen, dim+96)
                   buffer (the reference tests' strided inputs)
    rows_slice     rows slice [:, 64:64+dim, :] of a (batch, dim+96, seqlen) buffer
    """
    b, d, l = t.shape
    if layout == "contiguous":
        return t.contiguous()
    if layout == "channel_last":
        return t.transpose(1, 2).contiguous().transpose(1, 2)
    if layout == "cl_slice":
        wide = torch.zeros(b, l, d + 96, dtype=t.dtype, device=t.device)
        wide[:, :, 64:64 + d] = t.transpose(1, 2)
        return wide[:, :, 64:64 + d].transpose(1, 2)
    if layout == "rows_slice":
        wide = torch.zeros(b, d + 96, l, dtype=t.dtype, device=t.device)
        wide[:, 64:64 + d, :] = t
        return wide[:, 64:64 + d, :]
    raise ValueError(layout)


def assert_close(actual, expected_storage, dtype: str, tol, what=""):
    rtol, atol = tol
    a = f32(actual)
    e = O.to_f32(expected_storage, dtype)
    np.testing.assert_allclose(a, e, rtol=rtol, atol=atol, err_msg=what)
