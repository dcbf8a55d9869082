"""causal_conv1d_cuda (the legacy extension's function table) against the CPU oracle.

The legacy extension's contract (reference ``csrc/causal_conv1d.cpp:150-157`` forward,
``:261-463`` backward, ``:466-557`` update): outputs are written into caller tensors;
the backward writes ``dx`` and ``dinitial_states`` and **adds** into the caller's fp32
``dweight`` / ``dbias`` (``dweight.add_(...)`` at ``:451-461``); the update rewrites
``conv_state`` in place; argument errors are RuntimeError (TORCH_CHECK).
"""

import numpy as np
import pytest
import torch

import causal_conv1d_cuda as legacy
from helpers import TORCH_DT, assert_close, to_storage, with_layout
from oracle import numpy_oracle as O
from tolerances import GRAD_PARAM, PARITY

pytestmark = pytest.mark.gpu


def _inputs(gen, B, D, L, W, dt, layout, states):
    tdt = TORCH_DT[dt]
    x = torch.randn(B, D, L, generator=gen).to(tdt)
    dout = torch.randn(B, D, L, generator=gen).to(tdt)
    w = torch.rand(D, W, generator=gen) - 0.5
    b = torch.randn(D, generator=gen) * 0.1
    init = torch.randn(B, D, W - 1, generator=gen).to(tdt) if states else None
    dfinal = torch.randn(B, D, W - 1, generator=gen).to(tdt) if states else None
    dev = dict(x=with_layout(x.cuda(), layout), dout=with_layout(dout.cuda(), layout), w=w.cuda(), b=b.cuda(),
               init=None if init is None else init.cuda().transpose(1, 2).contiguous().transpose(1, 2),
               dfinal=None if dfinal is None else dfinal.cuda())
    return x, dout, w, b, init, dfinal, dev


@pytest.mark.parametrize("dt", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("layout,states", [("channel_last", True), ("channel_last", False), ("contiguous", False)])
@pytest.mark.parametrize("width", [2, 4])
def test_legacy_fwd_bwd_vs_oracle(dt, layout, states, width):
    gen = torch.Generator().manual_seed(17 + width + len(layout) + states)
    B, D, L, W = 2, 264, 300, width
    x, dout, w, b, init, dfinal, g = _inputs(gen, B, D, L, W, dt, layout, states)
    eo, ef = O.fwd(to_storage(x), dt, w.numpy(), "float32", b.numpy(), initial_states=to_storage(init),
                   silu=True, return_final_states=states)
    out = torch.empty_like(g["x"])
    final = torch.empty(B, W - 1, D, device="cuda", dtype=TORCH_DT[dt]).transpose(1, 2) if states else None
    legacy.causal_conv1d_fwd(g["x"], g["w"], g["b"], None, g["init"], out, final, True)
    assert_close(out, eo, dt, PARITY[dt], "out")
    if states:
        assert np.array_equal(to_storage(final), ef), "final states are an exact copy"

    edx, edw, edb, edi = O.bwd(to_storage(x), dt, w.numpy(), "float32", to_storage(dout), b.numpy(),
                               initial_states=to_storage(init), dfinal_states=to_storage(dfinal), silu=True)
    dx = torch.empty_like(g["x"])
    # the caller's fp32 gradient buffers already hold values: the call adds into them
    dw0 = torch.rand(D, W, generator=gen) - 0.5
    db0 = torch.rand(D, generator=gen) - 0.5
    dw, db = dw0.cuda(), db0.cuda()
    dinit = torch.empty_like(g["init"]) if states else None
    legacy.causal_conv1d_bwd(g["x"], g["w"], g["b"], g["dout"], None, g["init"], g["dfinal"], dx, dw, db, dinit,
                             True)
    assert_close(dx, edx, dt, PARITY[dt], "dx")
    np.testing.assert_allclose(dw.cpu().numpy(), dw0.numpy() + edw, *GRAD_PARAM["float32"], err_msg="dweight")
    np.testing.assert_allclose(db.cpu().numpy(), db0.numpy() + edb, *GRAD_PARAM["float32"], err_msg="dbias")
    if states:
        assert_close(dinit, edi, dt, PARITY[dt], "dinitial_states")


def test_legacy_bwd_without_bias_and_twice_accumulates():
    """dbias None with bias None; two calls add twice into dweight."""
    gen = torch.Generator().manual_seed(5)
    B, D, L, W = 2, 128, 77, 3
    x, dout, w, _, _, _, g = _inputs(gen, B, D, L, W, "bfloat16", "channel_last", False)
    _, edw, _, _ = O.bwd(to_storage(x), "bfloat16", w.numpy(), "float32", to_storage(dout), None, silu=False)
    dx = torch.empty_like(g["x"])
    dw = torch.zeros(D, W, device="cuda")
    for _ in range(2):
        legacy.causal_conv1d_bwd(g["x"], g["w"], None, g["dout"], None, None, None, dx, dw, None, None, False)
    np.testing.assert_allclose(dw.cpu().numpy(), 2 * edw, *GRAD_PARAM["float32"])


@pytest.mark.parametrize("channel_last", [True, False])
@pytest.mark.parametrize("circular", [False, True])
def test_legacy_update_vs_oracle(channel_last, circular):
    gen = torch.Generator().manual_seed(23 + circular)
    B, D, W, S, rows = 6, 256, 4, 8, 9
    x = torch.randn(B, D, generator=gen).to(torch.bfloat16)
    state = torch.randn(rows, D, S, generator=gen).to(torch.bfloat16)
    w = torch.rand(D, W, generator=gen) - 0.5
    b = torch.randn(D, generator=gen) * 0.1
    cache = torch.randint(-3, 50, (B,), generator=gen, dtype=torch.int32) if circular else None
    idx = torch.tensor([4, -1, 0, 8, 2, 7], dtype=torch.int32)
    eo, es = O.update(to_storage(x)[:, :, None], "bfloat16", to_storage(state), w.numpy(), "float32", b.numpy(),
                      silu=True, cache_seqlens=None if cache is None else cache.numpy(), conv_state_indices=idx.numpy())
    sg = state.cuda()
    if channel_last:
        sg = sg.transpose(1, 2).contiguous().transpose(1, 2)
    out = torch.empty(B, D, device="cuda", dtype=torch.bfloat16)
    legacy.causal_conv1d_update(x.cuda(), sg, w.cuda(), b.cuda(), out, True,
                                None if cache is None else cache.cuda(), idx.cuda())
    assert_close(out[:, :, None], eo, "bfloat16", PARITY["bfloat16"], "out")
    assert torch.all(out[1] == 0)
    assert np.array_equal(to_storage(sg), es)


def test_errors_are_runtime_errors():
    x = torch.randn(1, 8, 16, device="cuda")
    with pytest.raises(RuntimeError):
        legacy.causal_conv1d_fwd(x, torch.randn(8, 5, device="cuda"), None, None, None, torch.empty_like(x), None, False)
    with pytest.raises(RuntimeError):  # dweight must be fp32 (the legacy accumulation buffers)
        legacy.causal_conv1d_bwd(x, torch.randn(8, 4, device="cuda"), None, torch.randn_like(x), None, None, None,
                                 torch.empty_like(x), torch.zeros(8, 4, device="cuda", dtype=torch.float16), None,
                                 None, False)
    with pytest.raises(RuntimeError):  # bias and dbias go together
        legacy.causal_conv1d_bwd(x, torch.randn(8, 4, device="cuda"), torch.randn(8, device="cuda"),
                                 torch.randn_like(x), None, None, None, torch.empty_like(x),
                                 torch.zeros(8, 4, device="cuda"), None, None, False)
