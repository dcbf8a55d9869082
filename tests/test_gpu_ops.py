"""torch.ops.causal_conv1d.* registrations: same results as the host functions, and
torch.library.opcheck (schema, fake tensor and AOT dispatch) on small inputs."""

import pytest
import torch

import causal_conv1d  # noqa: F401  (registers the operators)
from causal_conv1d.causal_conv1d_varlen import causal_conv1d_varlen_states
from causal_conv1d.cpp_functions import (
    causal_conv1d_bwd_function,
    causal_conv1d_fwd_function,
    causal_conv1d_update_function,
)

pytestmark = pytest.mark.gpu

ops = torch.ops.causal_conv1d


def _conv_inputs(layout, dtype=torch.bfloat16, B=2, D=128, L=64, W=4):
    g = torch.Generator(device="cuda").manual_seed(3)
    if layout == "channel_last":
        x = torch.randn(B, L, D, generator=g, device="cuda").to(dtype).transpose(1, 2)
        dout = torch.randn(B, L, D, generator=g, device="cuda").to(dtype).transpose(1, 2)
    else:
        x = torch.randn(B, D, L, generator=g, device="cuda").to(dtype)
        dout = torch.randn(B, D, L, generator=g, device="cuda").to(dtype)
    w = torch.rand(D, W, generator=g, device="cuda") - 0.5
    b = torch.randn(D, generator=g, device="cuda") * 0.1
    init = torch.randn(B, D, W - 1, generator=g, device="cuda").to(dtype)
    return x, dout, w, b, init


@pytest.mark.parametrize("layout", ["channel_last", "contiguous"])
def test_fwd_bwd_ops_match_functions(layout):
    x, dout, w, b, init = _conv_inputs(layout)
    states = init if layout == "channel_last" else None
    assert torch.equal(ops.fwd(x, w, b, None, states, None, True),
                       causal_conv1d_fwd_function(x, w, b, None, states, None, True))
    got = ops.bwd(x, w, b, dout, None, states, None, states is not None, True)
    ref = causal_conv1d_bwd_function(x, w, b, dout, None, states, None, None, states is not None, True)
    for g_, r_ in zip(got, ref):
        if r_ is None:
            assert g_.numel() == 0
        else:
            assert torch.equal(g_, r_)


def test_update_and_varlen_ops_match_functions():
    g = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randn(4, 256, 1, generator=g, device="cuda").to(torch.bfloat16)
    state = torch.randn(4, 16, 256, generator=g, device="cuda").to(torch.bfloat16).transpose(1, 2)
    w = torch.rand(256, 4, generator=g, device="cuda") - 0.5
    cache = torch.randint(0, 100, (4,), generator=g, device="cuda", dtype=torch.int32)
    s1, s2 = state.clone(), state.clone()
    assert torch.equal(ops.update(x, s1, w, None, True, cache, None),
                       causal_conv1d_update_function(x, s2, w, None, True, cache, None))
    assert torch.equal(s1, s2)
    xs = torch.randn(300, 256, generator=g, device="cuda").to(torch.float16)
    cu = torch.tensor([0, 1, 120, 300], dtype=torch.int32, device="cuda")
    assert torch.equal(ops.varlen_states(xs, cu, 3), causal_conv1d_varlen_states(xs, cu, 3))


def test_opcheck():
    x, dout, w, b, init = _conv_inputs("channel_last", B=1, D=64, L=16)
    fin = torch.empty(1, 3, 64, device="cuda", dtype=torch.bfloat16).transpose(1, 2)
    torch.library.opcheck(ops.fwd, (x, w, b, None, init, fin, True))
    torch.library.opcheck(ops.bwd, (x, w, b, dout, None, init, None, True, True))
    state = torch.randn(1, 64, 3, device="cuda").to(torch.bfloat16)
    torch.library.opcheck(ops.update, (x[:, :, :1].contiguous(), state, w, b, True, None, None))
    xs = torch.randn(40, 64, device="cuda").to(torch.bfloat16)
    cu = torch.tensor([0, 10, 40], dtype=torch.int32, device="cuda")
    torch.library.opcheck(ops.varlen_states, (xs, cu, 3))
