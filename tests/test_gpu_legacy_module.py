"""causal_conv1d_cuda (the legacy extension's function table): same results as the
host functions; dweight/dbias accumulate; argument errors are RuntimeError."""

import pytest
import torch

import causal_conv1d_cuda as legacy
from causal_conv1d.cpp_functions import (
    causal_conv1d_bwd_function,
    causal_conv1d_fwd_function,
    causal_conv1d_update_function,
)

pytestmark = pytest.mark.gpu


def test_fwd_bwd_update_match():
    g = torch.Generator(device="cuda").manual_seed(9)
    B, D, L, W = 2, 256, 300, 4
    x = torch.randn(B, L, D, generator=g, device="cuda").to(torch.bfloat16).transpose(1, 2)
    dout = torch.randn(B, L, D, generator=g, device="cuda").to(torch.bfloat16).transpose(1, 2)
    w = torch.rand(D, W, generator=g, device="cuda") - 0.5
    b = torch.randn(D, generator=g, device="cuda") * 0.1
    out = torch.empty_like(x)
    legacy.causal_conv1d_fwd(x, w, b, None, None, out, None, True)
    assert torch.equal(out, causal_conv1d_fwd_function(x, w, b, None, None, None, True))

    dx = torch.empty_like(x)
    dw = torch.ones(D, W, device="cuda")
    db = torch.ones(D, device="cuda")
    legacy.causal_conv1d_bwd(x, w, b, dout, None, None, None, dx, dw, db, None, True)
    rdx, rdw, rdb, _ = causal_conv1d_bwd_function(x, w, b, dout, None, None, None, None, False, True)
    assert torch.equal(dx, rdx)
    assert torch.equal(dw, rdw + 1.0) and torch.equal(db, rdb + 1.0)  # accumulated

    xu = torch.randn(B, D, generator=g, device="cuda").to(torch.bfloat16)
    s1 = torch.randn(B, D, 3, generator=g, device="cuda").to(torch.bfloat16)
    s2 = s1.clone()
    ou = torch.empty_like(xu)
    legacy.causal_conv1d_update(xu, s1, w, b, ou, True, None, None)
    ref = causal_conv1d_update_function(xu.unsqueeze(-1), s2, w, b, True, None, None).squeeze(-1)
    assert torch.equal(ou, ref) and torch.equal(s1, s2)


def test_errors_are_runtime_errors():
    x = torch.randn(1, 8, 16, device="cuda")
    with pytest.raises(RuntimeError):
        legacy.causal_conv1d_fwd(x, torch.randn(8, 5, device="cuda"), None, None, None, torch.empty_like(x), None, False)
