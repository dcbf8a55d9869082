"""Context-parallel wrapper on one GPU (a one-rank group): same results as
causal_conv1d_fn, through the real kernels.  The multi-rank exchange logic is tested on
CPU (tests/test_context_parallel_gloo.py)."""

import datetime
import socket

import pytest
import torch
import torch.distributed as dist

from causal_conv1d import causal_conv1d_fn
from causal_conv1d.context_parallel import causal_conv1d_fn_context_parallel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def one_rank_group():
    if dist.is_initialized():
        yield
        return
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                            timeout=datetime.timedelta(seconds=30))
    yield
    dist.destroy_process_group()


def test_single_rank_matches_causal_conv1d_fn(one_rank_group):
    g = torch.Generator(device="cuda").manual_seed(8)
    x = torch.randn(2, 512, 256, generator=g, device="cuda").to(torch.bfloat16).transpose(1, 2)
    w = (torch.rand(256, 4, generator=g, device="cuda") - 0.5)
    b = torch.randn(256, generator=g, device="cuda") * 0.1
    init = torch.randn(2, 256, 3, generator=g, device="cuda").to(torch.bfloat16)
    dout = torch.randn(2, 512, 256, generator=g, device="cuda").to(torch.bfloat16).transpose(1, 2)
    grads = []
    for fn in (causal_conv1d_fn, causal_conv1d_fn_context_parallel):
        xr, wr, br, ir = (t.detach().clone().requires_grad_() for t in (x, w, b, init))
        out = fn(xr, wr, br, initial_states=ir, activation="silu")
        out.backward(dout)
        grads.append((out, xr.grad, wr.grad, br.grad, ir.grad))
    for a, c in zip(*grads):
        assert torch.equal(a, c)
