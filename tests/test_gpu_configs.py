"""GPU parity at the full benchmark sizes.

config 1  fp32 (2, 64, 512) contiguous, W=4, silu              -> whole tensor vs oracle
config 2  bf16 (4, 4096, 2048) channel-last, W=4, silu, states  -> whole tensor vs C oracle
config 3  update bf16 B=128 D=8192 (state_len 3 linear; 16 circular + gather), both
          state layouts                                         -> out vs oracle, state bit exact
config 4  fp16 (1, 5120, 65536) channel-last with seq_idx (32 packed sequences) and
          varlen states on (65536, 5120)                        -> channel slice / bit exact
config 5  (8, 16384, 8192) fp16/bf16, W=2..4, both layouts      -> channel slice vs oracle

Channels are independent (out, dx, dweight[d], dbias[d] of channel d read only channel
d), so for the largest configs the kernel runs on the whole tensor and a channel slice is
compared exactly against the oracle run on that slice.
"""

import numpy as np
import pytest
import torch

from causal_conv1d import causal_conv1d_fn, causal_conv1d_update
from causal_conv1d.causal_conv1d_varlen import causal_conv1d_varlen_states
from causal_conv1d.cpp_functions import causal_conv1d_bwd_function, causal_conv1d_fwd_function
from helpers import TORCH_DT, assert_close, to_storage, with_layout
from oracle import c_oracle as C
from oracle import numpy_oracle as O
from tolerances import GRAD_PARAM, PARITY

pytestmark = pytest.mark.gpu


def _gen(seed):
    return torch.Generator(device="cuda").manual_seed(seed)


def test_config1_fp32_contiguous():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(2, 64, 512, generator=g)
    w = torch.rand(64, 4, generator=g) - 0.5
    b = torch.randn(64, generator=g) * 0.1
    dout = torch.randn(2, 64, 512, generator=g)
    xg = x.cuda().requires_grad_()
    wg = w.cuda().requires_grad_()
    bg = b.cuda().requires_grad_()
    out = causal_conv1d_fn(xg, wg, bg, activation="silu")
    out.backward(dout.cuda())
    eo, _ = O.fwd(x.numpy(), "float32", w.numpy(), "float32", b.numpy(), silu=True)
    edx, edw, edb, _ = O.bwd(x.numpy(), "float32", w.numpy(), "float32", dout.numpy(), b.numpy(), silu=True)
    assert_close(out, eo, "float32", PARITY["float32"])
    assert_close(xg.grad, edx, "float32", PARITY["float32"])
    assert_close(wg.grad, edw, "float32", GRAD_PARAM["float32"])
    assert_close(bg.grad, edb, "float32", GRAD_PARAM["float32"])


@pytest.mark.parametrize("init_layout", ["contiguous", "channel_last"])
def test_config2_full(init_layout):
    gen = _gen(2)
    B, D, L, W = 4, 4096, 2048, 4
    x = torch.randn(B, L, D, generator=gen, device="cuda").to(torch.bfloat16).transpose(1, 2)
    w = torch.rand(D, W, generator=gen, device="cuda") - 0.5
    b = torch.randn(D, generator=gen, device="cuda") * 0.1
    init = torch.randn(B, D, W - 1, generator=gen, device="cuda").to(torch.bfloat16)
    if init_layout == "channel_last":
        init = init.transpose(1, 2).contiguous().transpose(1, 2)
    dout = torch.randn(B, L, D, generator=gen, device="cuda").to(torch.bfloat16).transpose(1, 2)
    dfinal = torch.randn(B, D, W - 1, generator=gen, device="cuda").to(torch.bfloat16)
    fin = torch.empty(B, W - 1, D, device="cuda", dtype=torch.bfloat16).transpose(1, 2)
    out = causal_conv1d_fwd_function(x, w, b, None, init, fin, True)
    dx, dw, db, di = causal_conv1d_bwd_function(x, w, b, dout, None, init, dfinal, None, True, True)
    xs, ws, bs, inits = to_storage(x), w.cpu().numpy(), b.cpu().numpy(), to_storage(init)
    eo, ef = C.fwd(xs, "bfloat16", ws, bs, initial_states=inits, silu=True, return_final_states=True)
    edx, edw, edb, edi = C.bwd(xs, "bfloat16", ws, to_storage(dout), bs, initial_states=inits,
                               dfinal_states=to_storage(dfinal), silu=True)
    assert_close(out, eo, "bfloat16", PARITY["bfloat16"], "out")
    assert np.array_equal(to_storage(fin), ef)
    assert_close(dx, edx, "bfloat16", PARITY["bfloat16"], "dx")
    assert_close(dw, edw, "float32", GRAD_PARAM["float32"], "dweight")
    assert_close(db, edb, "float32", GRAD_PARAM["float32"], "dbias")
    assert_close(di, edi, "bfloat16", PARITY["bfloat16"], "dinitial")


@pytest.mark.parametrize("variant", ["3a", "3b"])
@pytest.mark.parametrize("channel_last", [True, False])
def test_config3_update(variant, channel_last):
    gen = _gen(3)
    B, D, W = 128, 8192, 4
    S = 3 if variant == "3a" else 16
    x = torch.randn(B, D, generator=gen, device="cuda").to(torch.bfloat16)
    if channel_last:
        state = torch.randn(B, S, D, generator=gen, device="cuda").to(torch.bfloat16).transpose(1, 2)
    else:
        state = torch.randn(B, D, S, generator=gen, device="cuda").to(torch.bfloat16)
    w = torch.rand(D, W, generator=gen, device="cuda") - 0.5
    b = torch.randn(D, generator=gen, device="cuda") * 0.1
    cache = idx = None
    if variant == "3b":
        cache = torch.randint(0, 1000, (B,), generator=gen, device="cuda", dtype=torch.int32)
        idx = torch.randperm(B, generator=gen, device="cuda").to(torch.int32)
    eo, es = O.update(to_storage(x)[:, :, None], "bfloat16", to_storage(state), w.cpu().numpy(), "float32",
                      b.cpu().numpy(), silu=True, cache_seqlens=None if cache is None else cache.cpu().numpy(),
                      conv_state_indices=None if idx is None else idx.cpu().numpy())
    out = causal_conv1d_update(x, state, w, b, activation="silu", cache_seqlens=cache, conv_state_indices=idx)
    assert out.shape == (B, D)
    assert_close(out[:, :, None], eo, "bfloat16", PARITY["bfloat16"])
    assert np.array_equal(to_storage(state), es)


def _config4_split(T=65536, nseq=32):
    g = torch.Generator().manual_seed(0)
    lens = 1 + torch.bincount(torch.multinomial(torch.full((nseq,), 1.0 / nseq), T - nseq, replacement=True,
                                                generator=g), minlength=nseq)
    assert int(lens.sum()) == T and int(lens.min()) >= 1
    return lens


def test_config4_varlen_states_full():
    lens = _config4_split()
    cu = torch.nn.functional.pad(lens.cumsum(0), (1, 0)).to(torch.int32)
    x = torch.randn(65536, 5120, generator=_gen(4), device="cuda").to(torch.float16)
    out = causal_conv1d_varlen_states(x, cu.cuda(), 3)
    expected = O.varlen_states(to_storage(x), cu.numpy(), 3)
    assert np.array_equal(to_storage(out), expected)


def test_config4_packed_fwd_bwd():
    lens = _config4_split()
    T, D, W = 65536, 5120, 4
    seq = torch.repeat_interleave(torch.arange(32, dtype=torch.int32), lens).view(1, T)
    gen = _gen(44)
    x = torch.randn(1, T, D, generator=gen, device="cuda").to(torch.float16).transpose(1, 2)
    dout = torch.randn(1, T, D, generator=gen, device="cuda").to(torch.float16).transpose(1, 2)
    w = torch.rand(D, W, generator=gen, device="cuda") - 0.5
    b = torch.randn(D, generator=gen, device="cuda") * 0.1
    out = causal_conv1d_fwd_function(x, w, b, seq.cuda(), None, None, True)
    dx, dw, db, _ = causal_conv1d_bwd_function(x, w, b, dout, seq.cuda(), None, None, None, False, True)
    sl = slice(0, 128)
    xs = to_storage(x[:, sl, :])
    eo, _ = O.fwd(xs, "float16", w[sl].cpu().numpy(), "float32", b[sl].cpu().numpy(), seq_idx=seq.numpy(), silu=True)
    edx, edw, edb, _ = O.bwd(xs, "float16", w[sl].cpu().numpy(), "float32", to_storage(dout[:, sl, :]),
                             b[sl].cpu().numpy(), seq_idx=seq.numpy(), silu=True)
    assert_close(out[:, sl, :], eo, "float16", PARITY["float16"], "out")
    assert_close(dx[:, sl, :], edx, "float16", PARITY["float16"], "dx")
    assert_close(dw[sl], edw, "float32", GRAD_PARAM["float32"], "dweight")
    assert_close(db[sl], edb, "float32", GRAD_PARAM["float32"], "dbias")


@pytest.mark.parametrize("dt,width,layout", [
    ("bfloat16", 4, "channel_last"), ("bfloat16", 4, "contiguous"),
    ("float16", 4, "channel_last"), ("float16", 3, "contiguous"),
    ("bfloat16", 2, "channel_last"), ("float16", 2, "contiguous"),
])
def test_config5_slice(dt, width, layout):
    gen = _gen(5 + width)
    B, D, L = 8, 16384, 8192
    tdt = TORCH_DT[dt]
    if layout == "channel_last":
        x = torch.randn(B, L, D, generator=gen, device="cuda", dtype=tdt).transpose(1, 2)
        dout = torch.randn(B, L, D, generator=gen, device="cuda", dtype=tdt).transpose(1, 2)
    else:
        x = torch.randn(B, D, L, generator=gen, device="cuda", dtype=tdt)
        dout = torch.randn(B, D, L, generator=gen, device="cuda", dtype=tdt)
    w = torch.rand(D, width, generator=gen, device="cuda") - 0.5
    b = torch.randn(D, generator=gen, device="cuda") * 0.1
    silu = width != 2
    out = causal_conv1d_fwd_function(x, w, b, None, None, None, silu)
    dx, dw, db, _ = causal_conv1d_bwd_function(x, w, b, dout, None, None, None, None, False, silu)
    for sl in (slice(0, 32), slice(D - 32, D)):
        xs = to_storage(x[:, sl, :])
        eo, _ = O.fwd(xs, dt, w[sl].cpu().numpy(), "float32", b[sl].cpu().numpy(), silu=silu)
        edx, edw, edb, _ = O.bwd(xs, dt, w[sl].cpu().numpy(), "float32", to_storage(dout[:, sl, :]),
                                 b[sl].cpu().numpy(), silu=silu)
        assert_close(out[:, sl, :], eo, dt, PARITY[dt], "out")
        assert_close(dx[:, sl, :], edx, dt, PARITY[dt], "dx")
        assert_close(dw[sl], edw, "float32", GRAD_PARAM["float32"], "dweight")
        assert_close(db[sl], edb, "float32", GRAD_PARAM["float32"], "dbias")
    del x, dout, out, dx
    torch.cuda.empty_cache()


@pytest.mark.parametrize("shape,width,dt,states,silu", [
    ((1, 2048, 2048), 3, "float16", False, True),    # reference README forward shape 1
    ((1, 4096, 2048), 4, "bfloat16", False, True),   # reference README forward shape 2
    ((2, 4096, 2048), 4, "bfloat16", True, True),
    ((3, 1000, 777), 2, "float32", True, False),
    ((2, 2048, 4099), 4, "float16", True, True),
    ((8, 1024, 8192), 4, "bfloat16", False, True),
])
def test_forward_sizes_across_kernel_choices(shape, width, dt, states, silu):
    """Channel-last forwards from one small layer to a large batch (the streamed kernel's
    planner cuts them into very different warp units): whole output and final states
    against the oracle."""
    B, D, L = shape
    g = torch.Generator().manual_seed(B * D + L + width)
    x = torch.randn(B, L, D, generator=g).to(TORCH_DT[dt]).transpose(1, 2)
    w = torch.rand(D, width, generator=g) - 0.5
    b = torch.randn(D, generator=g) * 0.1
    init = torch.randn(B, D, width - 1, generator=g).to(TORCH_DT[dt]) if states else None
    eo, ef = O.fwd(to_storage(x), dt, w.numpy(), "float32", b.numpy(), initial_states=to_storage(init), silu=silu,
                   return_final_states=states)
    xg = x.transpose(1, 2).contiguous().cuda().transpose(1, 2)
    final = torch.empty(B, width - 1, D, device="cuda", dtype=TORCH_DT[dt]).transpose(1, 2) if states else None
    out = causal_conv1d_fwd_function(xg, w.cuda(), b.cuda(), None, None if init is None else init.cuda(), final, silu)
    assert_close(out, eo, dt, PARITY[dt], "out")
    if states:
        assert np.array_equal(to_storage(final), ef)
