"""Forward that also writes the varlen decode states (``causal_conv1d_fn_varlen_states``).

Its two results must equal, bit for bit, the two calls it fuses:
``causal_conv1d_fn(x, w, b, seq_idx=seq_idx)`` and
``causal_conv1d_varlen_states(x[0].T, cu_seqlens, state_len)``, and the states must
equal the numpy oracle's gather.  The cases put sequence ends inside and across the warp
segments of the streamed kernel (length-1 sequences, empty ones first, in the middle and
last, sequences shorter than state_len, state_len above the width), use int32 and int64
offsets, and cover the inputs that take two launches (no seq_idx, contiguous x).
"""

import numpy as np
import pytest
import torch

from causal_conv1d import _abi, causal_conv1d_fn
from causal_conv1d.causal_conv1d_varlen import causal_conv1d_fn_varlen_states, causal_conv1d_varlen_states
from helpers import TORCH_DT, to_storage
from oracle import numpy_oracle as O

pytestmark = pytest.mark.gpu


def packed_problem(gen, dim, lengths, tail, dt, width, cu_dtype=torch.int32, channel_last=True):
    lengths = torch.as_tensor(lengths, dtype=torch.int64)
    cu = torch.nn.functional.pad(lengths.cumsum(0), (1, 0))
    total = int(cu[-1]) + tail  # `tail` rows after the last sequence belong to none (seq_idx -1)
    seq = torch.full((1, total), -1, dtype=torch.int32)
    for k in range(len(lengths)):
        seq[0, int(cu[k]):int(cu[k + 1])] = k
    if channel_last:
        x = torch.randn(1, total, dim, generator=gen).to(TORCH_DT[dt]).transpose(1, 2)
    else:
        x = torch.randn(1, dim, total, generator=gen).to(TORCH_DT[dt])
    w = torch.rand(dim, width, generator=gen) - 0.5
    b = torch.randn(dim, generator=gen) * 0.1
    return x.cuda(), w.cuda(), b.cuda(), seq.cuda(), cu.to(cu_dtype).cuda()


def check(x, w, b, seq, cu, state_len, silu=True, launches=None):
    act = "silu" if silu else None
    before = _abi.launch_count()
    out, states = causal_conv1d_fn_varlen_states(x, w, cu, state_len, bias=b, seq_idx=seq, activation=act)
    made = _abi.launch_count() - before
    if launches is not None:
        assert made == launches
    ref_out = causal_conv1d_fn(x, w, b, seq_idx=seq, activation=act)
    # the public gather wants contiguous channels; the fused call takes any strides
    ref_states = causal_conv1d_varlen_states(x[0].transpose(0, 1).contiguous(), cu, state_len)
    assert out.shape == x.shape and out.stride() == x.stride()
    assert torch.equal(out, ref_out), "out must equal causal_conv1d_fn's"
    assert states.shape == (cu.numel() - 1, x.shape[1], state_len) and states.stride(1) == 1
    assert np.array_equal(to_storage(states), to_storage(ref_states)), "states must equal the separate gather"
    expected = O.varlen_states(to_storage(x[0].transpose(0, 1)), cu.cpu().numpy(), state_len)
    assert np.array_equal(to_storage(states), expected), "states must equal the oracle's"


def lengths_with_edges(gen, n, hi):
    lengths = torch.randint(1, hi, (n,), generator=gen)
    lengths[0] = 0  # empty first sequence: written by the unit holding row 0
    lengths[n // 3] = 0  # two empty sequences in a row in the middle
    lengths[n // 3 + 1] = 0
    lengths[n // 2] = 1
    lengths[-1] = 0  # empty last sequence
    return lengths


@pytest.mark.parametrize("dt", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("width", [2, 3, 4])
@pytest.mark.parametrize("state_len", [1, 3, 8, 40])
def test_fused_matches_two_calls(dt, width, state_len):
    gen = torch.Generator().manual_seed(width * 100 + state_len)
    lengths = lengths_with_edges(gen, 60, 90)
    x, w, b, seq, cu = packed_problem(gen, 256, lengths, 0, dt, width)
    check(x, w, b, seq, cu, state_len, launches=1)


@pytest.mark.parametrize("dim", [64, 264, 5120])
@pytest.mark.parametrize("cu_dtype", [torch.int32, torch.int64])
def test_fused_dims_offsets_and_tail(dim, cu_dtype):
    gen = torch.Generator().manual_seed(dim)
    lengths = lengths_with_edges(gen, 40, 300)
    x, w, b, seq, cu = packed_problem(gen, dim, lengths, 37, "bfloat16", 4, cu_dtype)
    check(x, w, b, seq, cu, 5, launches=1)
    check(x, w, None, seq, cu, 3, silu=False, launches=1)


def test_fused_degenerate_offsets():
    gen = torch.Generator().manual_seed(7)
    # every sequence empty, a single sequence, and cu starting past row 0
    x, w, b, seq, cu = packed_problem(gen, 128, [0, 0, 0], 50, "float16", 4)
    check(x, w, b, seq, cu, 4, launches=1)
    x, w, b, seq, cu = packed_problem(gen, 128, [777], 0, "float16", 4)
    check(x, w, b, seq, cu, 4, launches=1)
    lengths = torch.tensor([5, 0, 2, 300, 1])
    x, w, b, seq, cu = packed_problem(gen, 128, lengths, 9, "float16", 3)
    cu_shift = cu.clone()
    cu_shift[0] = 3  # rows 0-2 belong to no sequence
    seq[0, :3] = -1
    check(x, w, b, seq, cu_shift, 6, launches=1)


def test_two_launch_paths():
    gen = torch.Generator().manual_seed(11)
    lengths = lengths_with_edges(gen, 20, 64)
    # no seq_idx: plain forward plus the gather
    x, w, b, seq, cu = packed_problem(gen, 256, lengths, 0, "bfloat16", 4)
    before = _abi.launch_count()
    out, states = causal_conv1d_fn_varlen_states(x, w, cu, 3, bias=b, activation="silu")
    assert _abi.launch_count() - before == 2
    assert torch.equal(out, causal_conv1d_fn(x, w, b, activation="silu"))
    assert torch.equal(states, causal_conv1d_varlen_states(x[0].transpose(0, 1), cu, 3))
    # contiguous x with seq_idx: the general kernels plus the gather
    x, w, b, seq, cu = packed_problem(gen, 256, lengths, 0, "bfloat16", 4, channel_last=False)
    check(x, w, b, seq, cu, 3, launches=2)


def test_config4_prefill_states():
    """Config 4's packed prefill: fp16 x (1, 5120, 65536) channel-last, 32 sequences
    (lengths 1 + multinomial counts, seed 0), width 4, SiLU, state_len 3."""
    gen = torch.Generator().manual_seed(0)
    counts = torch.multinomial(torch.full((32,), 1 / 32), 65536 - 32, replacement=True, generator=gen)
    lengths = 1 + torch.bincount(counts, minlength=32)
    x, w, b, seq, cu = packed_problem(gen, 5120, lengths, 0, "float16", 4)
    check(x, w, b, seq, cu, 3, launches=1)


def test_argument_errors():
    gen = torch.Generator().manual_seed(1)
    x, w, b, seq, cu = packed_problem(gen, 64, [10, 20], 0, "bfloat16", 4)
    with pytest.raises(ValueError):
        causal_conv1d_fn_varlen_states(torch.cat([x, x]), w, cu, 3, seq_idx=torch.cat([seq, seq]))
    with pytest.raises(TypeError):
        causal_conv1d_fn_varlen_states(x, w, cu.float(), 3, seq_idx=seq)
    with pytest.raises(NotImplementedError):
        causal_conv1d_fn_varlen_states(x, w, cu, 3, seq_idx=seq, activation="relu")
