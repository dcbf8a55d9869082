"""GPU parity of the state-update and varlen-state kernels (public API -> C ABI).

conv_state and varlen states must match bit for bit (reference
tests/test_causal_conv1d.py:140-339 and tests/test_cpp_functions.py:10-54); outputs
within the parity tolerance.
"""

import numpy as np
import pytest
import torch

from causal_conv1d import causal_conv1d_update
from causal_conv1d.causal_conv1d_varlen import causal_conv1d_varlen_states
from golden_io import case_id, load_cases
from helpers import TORCH_DT, assert_close, to_storage, to_torch
from oracle import numpy_oracle as O
from tolerances import PARITY

pytestmark = pytest.mark.gpu

UPD = load_cases("update")
VAR = load_cases("varlen")


def state_layout(t: torch.Tensor, channel_last: bool) -> torch.Tensor:
    return t.transpose(1, 2).contiguous().transpose(1, 2) if channel_last else t.contiguous()


@pytest.mark.parametrize("case", UPD, ids=[case_id(m) for m, _ in UPD])
@pytest.mark.parametrize("channel_last", [True, False])
def test_golden_update(case, channel_last):
    meta, a = case
    dt = meta["x_dtype"]
    x = state_layout(to_torch(a["x"], dt), channel_last)
    state = state_layout(to_torch(a["state"], dt), channel_last)
    cache = to_torch(a.get("cache_seqlens"))
    idx = to_torch(a.get("indices"))
    out = causal_conv1d_update(x, state, to_torch(a["weight"]), to_torch(a["bias"]),
                               activation="silu" if meta["silu"] else None,
                               cache_seqlens=cache, conv_state_indices=idx)
    assert_close(out, a["out"], dt, PARITY[dt], "out")
    if idx is not None:
        pad = (idx < 0).cpu()
        assert torch.all(out.cpu()[pad] == 0)
    assert np.array_equal(to_storage(state), a["new_state"]), "conv_state must match bit for bit"


def run_update_vs_oracle(gen, batch, dim, seqlen, width, state_len, dt, circular, mode, channel_last,
                         silu=True, squeeze=False, cache_low=0):
    tdt = TORCH_DT[dt]
    total = batch if mode == "plain" else 3 * batch
    x = torch.randn(batch, dim, seqlen, generator=gen).to(tdt)
    state = torch.randn(total, dim, state_len, generator=gen).to(tdt)
    w = torch.rand(dim, width, generator=gen) - 0.5
    b = torch.randn(dim, generator=gen) * 0.1
    cache = torch.randint(cache_low, 1000, (batch,), generator=gen, dtype=torch.int32) if circular else None
    idx = None
    if mode != "plain":
        idx = torch.randperm(total, generator=gen)[:batch].to(torch.int32)
        if mode == "padding":
            idx[torch.randperm(batch, generator=gen)[: batch // 2]] = -1
            idx[batch // 2] = total  # out of range: also a padding row
    # the oracle takes negative indices as padding rows; out-of-range ones are padding too
    idx_oracle = None if idx is None else np.where(idx.numpy() >= total, -1, idx.numpy())
    eo, es = O.update(to_storage(x), dt, to_storage(state), w.numpy(), "float32", b.numpy(), silu=silu,
                      cache_seqlens=None if cache is None else cache.numpy(), conv_state_indices=idx_oracle)
    xg = state_layout(x.cuda(), channel_last)
    sg = state_layout(state.cuda(), channel_last)
    if squeeze:
        xg = xg[:, :, 0]
    out = causal_conv1d_update(xg, sg, w.cuda(), b.cuda(), activation="silu" if silu else None,
                               cache_seqlens=None if cache is None else cache.cuda(),
                               conv_state_indices=None if idx is None else idx.cuda())
    if squeeze:
        assert out.shape == (batch, dim)
        out = out.unsqueeze(-1)
    assert_close(out, eo, dt, PARITY[dt], "out")
    assert np.array_equal(to_storage(sg), es)


@pytest.mark.parametrize("dim", [2048, 2048 + 16, 4096])
@pytest.mark.parametrize("width", [2, 3, 4])
@pytest.mark.parametrize("seqlen", [1, 4, 5])
@pytest.mark.parametrize("dt", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("circular", [False, True])
@pytest.mark.parametrize("mode", ["plain", "gather", "padding"])
def test_update_grid(dim, width, seqlen, dt, circular, mode):
    """The reference update grid (batch 64, random state_len in [W-1, W+10))."""
    gen = torch.Generator().manual_seed(dim + 10 * width + seqlen)
    state_len = int(torch.randint(width - 1, width + 10, (1,), generator=gen))
    channel_last = (dim + seqlen + width) % 2 == 0
    run_update_vs_oracle(gen, 64, dim, seqlen, width, state_len, dt, circular, mode, channel_last)


@pytest.mark.parametrize("dt", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("width", [2, 3, 4])
@pytest.mark.parametrize("state_len", ["w-1", 6, 8, 16])
@pytest.mark.parametrize("circular", [False, True])
@pytest.mark.parametrize("mode", ["plain", "gather", "padding"])
@pytest.mark.parametrize("channel_last", [True, False])
def test_update_single_token(dt, width, state_len, circular, mode, channel_last):
    """seqlen == 1 (the decode step) in every state layout the single-token kernels take:
    channel-last shift and circular, (B, D, W-1) blocks, (B, D, S) circular rings with
    S % 4 == 0 (16-bit), and the layouts that fall back to the general kernel (S = 6
    contiguous, fp32 rings, linear with S > W-1).  Batch 37 leaves a partial row tile;
    cache_seqlens include negative values (non-negative modulo, as the oracle)."""
    S = width - 1 if state_len == "w-1" else state_len
    gen = torch.Generator().manual_seed(100 * width + 7 * S + 3 * circular + len(mode) + channel_last)
    run_update_vs_oracle(gen, 37, 1040, 1, width, S, dt, circular, mode, channel_last, cache_low=-40)


def test_update_single_token_unaligned_views():
    """x, out and state views whose channel packets are not 16-byte aligned take the
    general kernel; results are the same."""
    gen = torch.Generator().manual_seed(31)
    for channel_last in (True, False):
        B, D, W, S = 9, 520, 4, 16
        x = torch.randn(B, D + 1, 1, generator=gen).to(torch.bfloat16)[:, 1:]
        state = torch.randn(B, D, S, generator=gen).to(torch.bfloat16)
        w = torch.rand(D, W, generator=gen) - 0.5
        cache = torch.randint(-5, 100, (B,), generator=gen, dtype=torch.int32)
        eo, es = O.update(to_storage(x.contiguous()), "bfloat16", to_storage(state), w.numpy(), "float32", None,
                          silu=True, cache_seqlens=cache.numpy())
        sg = state_layout(state.cuda(), channel_last)
        out = causal_conv1d_update(x.cuda(), sg, w.cuda(), None, activation="silu", cache_seqlens=cache.cuda())
        assert_close(out, eo, "bfloat16", PARITY["bfloat16"], "out")
        assert np.array_equal(to_storage(sg), es)


@pytest.mark.parametrize("dim", [2048, 2052, 2050])
@pytest.mark.parametrize("width", [2, 3, 4])
@pytest.mark.parametrize("seqlen", [1, 2, 5])
@pytest.mark.parametrize("dt", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("mode", ["plain", "gather", "padding"])
def test_update_shift_contiguous_state(dim, width, seqlen, dt, mode):
    """(batch, dim, W-1) state with contiguous entries and no circular buffer (config 3a's
    benchmark layout): whole channel blocks of the history per thread, bit-exact
    state.  dim 2050 is not a whole number of 8-byte channel blocks for 16-bit types and
    takes the per-channel kernel."""
    gen = torch.Generator().manual_seed(dim + 7 * width + seqlen)
    run_update_vs_oracle(gen, 64, dim, seqlen, width, width - 1, dt, False, mode, False)


def test_update_shift_contiguous_state_strided_weight():
    """The same kernel with weights that are not one contiguous fp32 (dim, W) block."""
    gen = torch.Generator().manual_seed(9)
    x = torch.randn(16, 512, 1, generator=gen).to(torch.bfloat16)
    state = torch.randn(16, 512, 3, generator=gen).to(torch.bfloat16)
    w = torch.rand(4, 512, generator=gen) - 0.5
    eo, es = O.update(to_storage(x), "bfloat16", to_storage(state), w.t().contiguous().numpy(), "float32", None,
                      silu=True)
    sg = state.cuda()
    out = causal_conv1d_update(x.cuda(), sg, w.cuda().t(), None, activation="silu")
    assert_close(out, eo, "bfloat16", PARITY["bfloat16"], "out")
    assert np.array_equal(to_storage(sg), es)


@pytest.mark.parametrize("state_len", [3, 6])
@pytest.mark.parametrize("circular", [False, True])
@pytest.mark.parametrize("channel_last", [True, False])
def test_update_out_of_range_index_is_a_padding_row(state_len, circular, channel_last):
    """A conv_state_indices entry >= the number of state rows (undefined in the
    reference) writes nothing and gives a zero output row, like a negative index."""
    gen = torch.Generator().manual_seed(21)
    B, D, W, rows = 4, 256, 4, 5
    x = torch.randn(B, D, 1, generator=gen).to(torch.bfloat16)
    state = torch.randn(rows, D, state_len, generator=gen).to(torch.bfloat16)
    w = torch.rand(D, W, generator=gen) - 0.5
    idx = torch.tensor([0, 7, 3, rows], dtype=torch.int32)
    cache = torch.tensor([5, 9, 0, 2], dtype=torch.int32) if circular else None
    as_padding = torch.where(idx >= rows, torch.full_like(idx, -1), idx)
    eo, es = O.update(to_storage(x), "bfloat16", to_storage(state), w.numpy(), "float32", None, silu=True,
                      cache_seqlens=None if cache is None else cache.numpy(), conv_state_indices=as_padding.numpy())
    sg = state_layout(state.cuda(), channel_last)
    out = causal_conv1d_update(state_layout(x.cuda(), channel_last), sg, w.cuda(), None, activation="silu",
                               cache_seqlens=None if cache is None else cache.cuda(), conv_state_indices=idx.cuda())
    assert_close(out, eo, "bfloat16", PARITY["bfloat16"], "out")
    assert torch.all(out[1] == 0) and torch.all(out[3] == 0)
    assert np.array_equal(to_storage(sg), es)


def test_varlen_states_rows_past_the_end_are_zero():
    """cu_seqlens pointing past the last row of x (undefined in the reference) gathers
    zeros for those rows instead of reading outside x."""
    gen = torch.Generator().manual_seed(22)
    x = torch.randn(20, 64, generator=gen).to(torch.float16)
    cu = torch.tensor([0, 5, 18, 30], dtype=torch.int32)
    padded = torch.cat([x, torch.zeros(10, 64, dtype=x.dtype)])
    expected = O.varlen_states(to_storage(padded), cu.numpy(), 4)
    out = causal_conv1d_varlen_states(x.cuda(), cu.cuda(), 4)
    assert np.array_equal(to_storage(out), expected)


@pytest.mark.parametrize("channel_last", [True, False])
def test_update_squeezed_2d_input(channel_last):
    gen = torch.Generator().manual_seed(3)
    run_update_vs_oracle(gen, 8, 256, 1, 4, 5, "bfloat16", True, "gather", channel_last, squeeze=True)


def test_update_seqlen_longer_than_state():
    """Linear mode with seqlen > state_len keeps the last state_len inputs; circular mode
    writes in order so the last duplicate wins (reference cutedsl_kernels.py:474-490)."""
    gen = torch.Generator().manual_seed(4)
    for circular in (False, True):
        run_update_vs_oracle(gen, 4, 64, 9, 4, 3, "float32", circular, "plain", True)
        run_update_vs_oracle(gen, 4, 64, 9, 2, 1, "float16", circular, "plain", False)


@pytest.mark.parametrize("has_cache", [False, True])
def test_update_channel_first_masks_negative_indices(has_cache):
    """reference tests/test_cpp_functions.py:10-54, exact."""
    gen = torch.Generator().manual_seed(11)
    x = torch.randn(4, 8, 2, generator=gen)
    state = torch.randn(6, 8, 4, generator=gen)
    idx = torch.tensor([1, -1, 4, -1], dtype=torch.int32)
    cache = torch.tensor([3, 7, 5, 9], dtype=torch.int32) if has_cache else None
    w = torch.randn(8, 3, generator=gen)
    b = torch.randn(8, generator=gen)
    eo, es = O.update(x.numpy(), "float32", state.numpy(), w.numpy(), "float32", b.numpy(), silu=True,
                      cache_seqlens=None if cache is None else cache.numpy(), conv_state_indices=idx.numpy())
    sg = state.cuda()
    out = causal_conv1d_update(x.cuda(), sg, w.cuda(), b.cuda(), activation="silu",
                               cache_seqlens=None if cache is None else cache.cuda(),
                               conv_state_indices=idx.cuda())
    assert_close(out, eo, "float32", PARITY["float32"])
    assert torch.all(out[1] == 0) and torch.all(out[3] == 0)
    assert np.array_equal(sg.cpu().numpy(), es)


@pytest.mark.parametrize("case", VAR, ids=[case_id(m) for m, _ in VAR])
def test_golden_varlen_states(case):
    meta, a = case
    x = to_torch(a["x"], meta["x_dtype"])
    cu = to_torch(a["cu_seqlens"])
    out = causal_conv1d_varlen_states(x, cu, meta["state_len"])
    assert out.shape == a["out"].shape
    assert out.stride(1) == 1
    assert np.array_equal(to_storage(out), a["out"])


@pytest.mark.parametrize("dt", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("dim", [2048, 2048 + 16, 4096, 36])
@pytest.mark.parametrize("cu_dtype", [torch.int32, torch.int64])
def test_varlen_states_grid(dt, dim, cu_dtype):
    """reference tests/test_causal_conv1d.py:324-339 plus odd dims, int32/int64 offsets."""
    gen = torch.Generator().manual_seed(dim)
    seqlens = torch.randint(1, 32, (100,), generator=gen)
    seqlens[5] = 0  # an empty sequence gives an all-zero state row
    cu = torch.nn.functional.pad(seqlens.cumsum(0), (1, 0)).to(cu_dtype)
    x = torch.randn(int(seqlens.sum()), dim, generator=gen).to(TORCH_DT[dt])
    expected = O.varlen_states(to_storage(x), cu.numpy(), 20)
    out = causal_conv1d_varlen_states(x.cuda(), cu.cuda(), 20)
    assert np.array_equal(to_storage(out), expected)


def test_varlen_states_strided_rows():
    gen = torch.Generator().manual_seed(8)
    wide = torch.randn(300, 200, generator=gen).to(torch.bfloat16)
    x = wide[:, 8:8 + 128]  # row stride 200, channels contiguous
    cu = torch.tensor([0, 10, 11, 150, 300], dtype=torch.int32)
    expected = O.varlen_states(to_storage(x), cu.numpy(), 4)
    out = causal_conv1d_varlen_states(wide.cuda()[:, 8:8 + 128], cu.cuda(), 4)
    assert np.array_equal(to_storage(out), expected)
