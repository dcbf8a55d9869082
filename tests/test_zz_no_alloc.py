"""cc1d_bwd_launch_static: the backward entry point that takes its scratch from a static
array in the library instead of a caller workspace.

Called through the C ABI (ctypes) and compared with cc1d_bwd_launch on the same inputs,
twice in a row, so that the second call runs on scratch the first one left behind.  The
cases reach every backward kernel family: the streamed channel-last kernel, the
row-stream kernel for (batch, dim, seqlen) contiguous tensors, and the strided fallback
whose arrival counters must be cleared before each call.  The file is named to be
collected last; it needs nothing from the other test files.
"""

import ctypes

import pytest
import torch

from causal_conv1d import _abi
from helpers import assert_close, with_layout
from tolerances import GRAD_PARAM, PARITY

pytestmark = pytest.mark.gpu

NAME = {torch.float32: "float32", torch.float16: "float16", torch.bfloat16: "bfloat16"}


def _params(x, w, b, dout, seq, init, dfinal, dx, dinit, dw, db, silu):
    return _abi.BwdParams(
        x.shape[0], x.shape[1], x.shape[2], w.shape[1],
        _abi._ct(x), _abi._ct(w), _abi._ct(b), _abi._ct(seq), _abi._ct(init), _abi._ct(dout),
        _abi._ct(dfinal), _abi._ct(dx), _abi._ct(dinit),
        dw.data_ptr(), db.data_ptr() if db is not None else None, None, 0, int(silu), 0,
    )


def _outputs(x, w, b, init):
    dx = torch.full_like(x, float("nan"))
    dw = torch.full(w.shape, float("nan"), device="cuda")
    db = torch.full(b.shape, float("nan"), device="cuda") if b is not None else None
    dinit = torch.full_like(init, float("nan")) if init is not None else None
    return dx, dw, db, dinit


def _run(static, x, w, b, dout, seq, init, dfinal, silu):
    lib = _abi.load_library()
    dx, dw, db, dinit = _outputs(x, w, b, init)
    p = _params(x, w, b, dout, seq, init, dfinal, dx, dinit, dw, db, silu)
    stream = torch.cuda.current_stream().cuda_stream
    if static:
        status = lib.cc1d_bwd_launch_static(ctypes.byref(p), stream)
    else:
        need = lib.cc1d_bwd_workspace_bytes(ctypes.byref(p))
        assert need >= 0, lib.cc1d_last_error().decode()
        ws = torch.empty(max(need, 1), dtype=torch.uint8, device="cuda")
        p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
        status = lib.cc1d_bwd_launch(ctypes.byref(p), stream)
    assert status == 0, lib.cc1d_last_error().decode()
    torch.cuda.synchronize()
    return dx, dw, db, dinit


CASES = [
    # (dtype, batch, dim, seqlen, width, layout, seq_idx, states, silu)
    (torch.bfloat16, 2, 1024, 1000, 4, "channel_last", False, True, True),
    (torch.float16, 3, 512, 777, 3, "contiguous", False, False, True),
    (torch.float32, 2, 99, 300, 4, "cl_slice", True, False, False),
    (torch.bfloat16, 4, 4096, 2048, 4, "channel_last", False, True, True),
]


@pytest.mark.parametrize("dt,B,D,L,W,layout,use_seq,states,silu", CASES)
def test_static_matches_workspace_entry(dt, B, D, L, W, layout, use_seq, states, silu):
    g = torch.Generator(device="cuda").manual_seed(1234 + D + L)
    x = with_layout(torch.randn(B, D, L, generator=g, device="cuda").to(dt), layout)
    dout = with_layout(torch.randn(B, D, L, generator=g, device="cuda").to(dt), layout)
    w = (torch.rand(D, W, generator=g, device="cuda") - 0.5).to(dt)
    b = (torch.randn(D, generator=g, device="cuda") * 0.1).to(dt)
    seq = init = dfinal = None
    if use_seq:
        cuts = torch.sort(torch.randint(1, L, (3,), generator=g, device="cuda")).values
        seq = torch.searchsorted(cuts, torch.arange(L, device="cuda"), right=True).to(torch.int32)
        seq = seq.expand(B, L).contiguous()
    if states:
        init = torch.randn(B, D, W - 1, generator=g, device="cuda").to(dt)
        dfinal = torch.randn(B, D, W - 1, generator=g, device="cuda").to(dt)
    args = (x, w, b, dout, seq, init, dfinal, silu)
    ref = _run(False, *args)
    first = _run(True, *args)
    second = _run(True, *args)
    name = NAME[dt]
    for got in (first, second):
        for r, o, label in zip(ref, got, ("dx", "dweight", "dbias", "dinitial_states")):
            if r is None:
                assert o is None
                continue
            tol = PARITY[name] if label in ("dx", "dinitial_states") else GRAD_PARAM["float32"]
            assert_close(o, r.float().cpu().numpy(), "float32", tol, label)
    # the reduction order does not depend on the scratch: both calls agree bit for bit
    for a, c in zip(first, second):
        if a is not None:
            assert torch.equal(a, c)


def test_static_rejects_problems_beyond_the_array():
    lib = _abi.load_library()
    limit = _abi.STATIC_SCRATCH_BYTES
    # strided (non-packet) channel-last tensors use the fallback kernel, whose scratch
    # holds (width + 1) fp32 partial sums per (batch row, channel) for short sequences
    D, L, W = 4096, 2, 4
    B = limit // (D * (W + 1) * 4) + 8
    wide = torch.zeros(B, L, D + 1, dtype=torch.float32, device="cuda")
    x = wide[:, :, 1:].transpose(1, 2)
    dout = torch.zeros_like(wide)[:, :, 1:].transpose(1, 2)
    w = torch.zeros(D, W, device="cuda")
    b = torch.zeros(D, device="cuda")
    dx, dw, db, _ = _outputs(x, w, b, None)
    p = _params(x, w, b, dout, None, None, None, dx, None, dw, db, False)
    need = lib.cc1d_bwd_workspace_bytes(ctypes.byref(p))
    assert need > limit, (need, limit)
    before = lib.cc1d_launch_count()
    status = lib.cc1d_bwd_launch_static(ctypes.byref(p), torch.cuda.current_stream().cuda_stream)
    assert status == 1  # CC1D_ERR_VALUE
    msg = lib.cc1d_last_error().decode()
    assert "static array" in msg and str(need) in msg and str(limit) in msg
    assert lib.cc1d_launch_count() == before  # nothing was launched
    assert torch.isnan(dx).all()


def test_static_entry_allocates_nothing():
    """The property the entry point exists for: after its first call on the device (which
    may load the library's device code, the static array included), further calls leave
    the device's free memory and the PyTorch allocator unchanged."""
    g = torch.Generator(device="cuda").manual_seed(77)
    B, D, L, W = 2, 512, 600, 4
    x = with_layout(torch.randn(B, D, L, generator=g, device="cuda").to(torch.bfloat16), "channel_last")
    dout = with_layout(torch.randn(B, D, L, generator=g, device="cuda").to(torch.bfloat16), "channel_last")
    w = torch.rand(D, W, generator=g, device="cuda") - 0.5
    b = torch.randn(D, generator=g, device="cuda") * 0.1
    lib = _abi.load_library()
    dx, dw, db, _ = _outputs(x, w, b, None)
    p = _params(x, w, b, dout, None, None, None, dx, None, dw, db, True)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.cc1d_bwd_launch_static(ctypes.byref(p), stream) == 0, lib.cc1d_last_error().decode()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    torch0 = torch.cuda.memory_reserved()
    for _ in range(3):
        assert lib.cc1d_bwd_launch_static(ctypes.byref(p), stream) == 0, lib.cc1d_last_error().decode()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
    assert torch.cuda.memory_reserved() == torch0
