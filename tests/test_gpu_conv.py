"""GPU parity of the forward/backward kernels (through the public API -> C ABI).

Reference behaviour pinned two ways: the committed golden vectors made by the
reference's own oracles, and the numpy oracle (itself pinned to those vectors) on
seeded inputs over the reference test grid (tests/test_causal_conv1d.py:50-137,401-557
in the reference).  Tolerances: tests/tolerances.py.
"""

import itertools

import numpy as np
import pytest
import torch

from causal_conv1d import causal_conv1d_fn
from causal_conv1d.cpp_functions import causal_conv1d_bwd_function, causal_conv1d_fwd_function
from golden_io import case_id, load_cases
from helpers import TORCH_DT, assert_close, f32, to_storage, to_torch, with_layout
from oracle import numpy_oracle as O
from tolerances import GRAD_PARAM, PARITY

pytestmark = pytest.mark.gpu

GOLD = load_cases("fwd_bwd") + load_cases("seq_idx")


def run_fn(x, w, b, seq_idx, init, final, silu, dout, dfinal):
    """Forward + autograd backward through causal_conv1d_fn."""
    x = x.detach().requires_grad_()
    w = w.detach().requires_grad_()
    b = b.detach().requires_grad_() if b is not None else None
    init = init.detach().requires_grad_() if init is not None else None
    res = causal_conv1d_fn(x, w, b, seq_idx=seq_idx, initial_states=init, return_final_states=final,
                           activation="silu" if silu else None)
    out, fin = res if final else (res, None)
    outs, grads = [out], [dout]
    if final:
        outs.append(fin)
        grads.append(dfinal)
    torch.autograd.backward(outs, grads)
    return (out, fin, x.grad, w.grad, b.grad if b is not None else None,
            init.grad if init is not None else None)


def layouts_for(meta):
    if meta.get("final"):
        return ["channel_last", "cl_slice"]  # final states need channel-last x
    return ["channel_last", "contiguous", "cl_slice", "rows_slice"]


GOLD_PARAMS = [(c, lay) for c in GOLD for lay in layouts_for(c[0])]


@pytest.mark.parametrize("case,layout", GOLD_PARAMS,
                         ids=[f"{case_id(c[0])}-{lay}" for c, lay in GOLD_PARAMS])
def test_golden_fwd_bwd(case, layout):
    meta, a = case
    xdt, wdt = meta["x_dtype"], meta["w_dtype"]
    x = with_layout(to_torch(a["x"], xdt), layout)
    w = to_torch(a["weight"], wdt)
    b = to_torch(a.get("bias"), wdt)
    init = to_torch(a.get("init"), xdt)
    if init is not None:  # the reference tests pass (batch, width-1, dim).T
        init = init.transpose(1, 2).contiguous().transpose(1, 2)
    seq = to_torch(a.get("seq_idx")) if "seq_idx" in a else None
    dout = with_layout(to_torch(a["dout"], xdt), layout)
    dfinal = to_torch(a.get("dfinal"), xdt)
    out, fin, dx, dw, db, dinit = run_fn(x, w, b, seq, init, meta["final"], meta["silu"], dout, dfinal)
    assert out.stride() == x.stride() or layout.endswith("slice")
    assert_close(out, a["out"], xdt, PARITY[xdt], "out")
    if meta["final"]:
        assert np.array_equal(to_storage(fin), a["final"]), "final states must be bit exact"
    assert_close(dx, a["dx"], xdt, PARITY[xdt], "dx")
    assert_close(dw, a["dweight"], wdt, GRAD_PARAM[wdt], "dweight")
    if b is not None:
        assert_close(db, a["dbias"], wdt, GRAD_PARAM[wdt], "dbias")
    if init is not None:
        assert_close(dinit, a["dinit"], xdt, PARITY[xdt], "dinitial_states")


# ------------------------------------------------------------ oracle sweep
SEQLENS = [1, 2, 8, 16, 32, 64, 128, 129, 130, 151, 256, 372, 512, 784, 1024, 1134, 2048, 4096]
DTYPES = ["float32", "float16", "bfloat16"]
LAYOUTS = ["channel_last", "contiguous", "cl_slice", "rows_slice"]


def sweep_cases():
    cases = []
    k = 0
    for seqlen, width, dt in itertools.product(SEQLENS, (2, 3, 4), DTYPES):
        k += 1
        dim = 4128 if (k % 3 == 0 and seqlen <= 1134) else 64 + 8 * (k % 5)
        layout = LAYOUTS[k % 4]
        cl = layout in ("channel_last", "cl_slice")
        init = cl and k % 2 == 0
        final = cl and k % 5 != 0
        cases.append((dim, seqlen, width, dt, layout, bool(k % 7), bool(k % 3), init, final))
    return cases


def make_inputs(gen, batch, dim, seqlen, width, dt, has_bias, has_init, final, w_scale=1.0):
    x = torch.randn(batch, dim, seqlen, generator=gen).to(TORCH_DT[dt])
    w = torch.randn(dim, width, generator=gen) * w_scale
    b = torch.randn(dim, generator=gen) if has_bias else None
    init = torch.randn(batch, dim, width - 1, generator=gen).to(TORCH_DT[dt]) if has_init else None
    dout = torch.randn(batch, dim, seqlen, generator=gen).to(TORCH_DT[dt])
    dfinal = torch.randn(batch, dim, width - 1, generator=gen).to(TORCH_DT[dt]) if final else None
    return x, w, b, init, dout, dfinal


def check_against_oracle(x, w, b, seq, init, final, silu, dout, dfinal, layout, init_layout="cl"):
    dt = {v: k for k, v in TORCH_DT.items()}[x.dtype]
    xs, ws, bs = to_storage(x), to_storage(w), to_storage(b)
    inits, douts, dfs = to_storage(init), to_storage(dout), to_storage(dfinal)
    seqs = None if seq is None else seq.numpy()
    eo, ef = O.fwd(xs, dt, ws, "float32", bs, "float32", seq_idx=seqs, initial_states=inits,
                   silu=silu, return_final_states=final)
    edx, edw, edb, edi = O.bwd(xs, dt, ws, "float32", douts, bs, "float32", seq_idx=seqs,
                               initial_states=inits, dfinal_states=dfs, silu=silu)
    xg = with_layout(x.cuda(), layout)
    ig = None
    if init is not None:
        ig = init.cuda()
        if init_layout == "cl":
            ig = ig.transpose(1, 2).contiguous().transpose(1, 2)
    out, fin, dx, dw, db, di = run_fn(xg, w.cuda(), None if b is None else b.cuda(),
                                      None if seq is None else seq.cuda(), ig, final, silu,
                                      with_layout(dout.cuda(), layout),
                                      None if dfinal is None else dfinal.cuda())
    assert_close(out, eo, dt, PARITY[dt], "out")
    if final:
        assert np.array_equal(to_storage(fin), ef)
    assert_close(dx, edx, dt, PARITY[dt], "dx")
    assert_close(dw, edw, "float32", GRAD_PARAM["float32"], "dweight")
    if b is not None:
        assert_close(db, edb, "float32", GRAD_PARAM["float32"], "dbias")
    if init is not None:
        assert_close(di, edi, dt, PARITY[dt], "dinitial")


@pytest.mark.parametrize("dim,seqlen,width,dt,layout,has_bias,silu,has_init,final", sweep_cases())
def test_sweep_vs_oracle(dim, seqlen, width, dt, layout, has_bias, silu, has_init, final):
    gen = torch.Generator().manual_seed(dim * 7919 + seqlen * 31 + width)
    x, w, b, init, dout, dfinal = make_inputs(gen, 2, dim, seqlen, width, dt, has_bias, has_init, final)
    check_against_oracle(x, w, b, None, init, final, silu, dout, dfinal, layout)


@pytest.mark.parametrize("seqlen", [1, 2, 3, 65])
@pytest.mark.parametrize("width", [2, 3, 4])
@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("feat", range(16))
def test_feature_matrix(seqlen, width, dt, feat):
    has_bias, silu, has_init, final = bool(feat & 1), bool(feat & 2), bool(feat & 4), bool(feat & 8)
    gen = torch.Generator().manual_seed(feat * 1000 + seqlen * 10 + width)
    x, w, b, init, dout, dfinal = make_inputs(gen, 2, 72, seqlen, width, dt, has_bias, has_init, final)
    layout = "channel_last" if (final or feat % 2) else "contiguous"
    check_against_oracle(x, w, b, None, init, final, silu, dout, dfinal, layout,
                         init_layout="cl" if feat % 3 else "contiguous")


def make_seq_idx(gen, batch, seqlen, pad):
    seq = torch.empty(batch, seqlen, dtype=torch.int32)
    for bi in range(batch):
        true_len = seqlen - (int(torch.randint(1, max(2, seqlen // 3), (1,), generator=gen)) if pad else 0)
        nsplit = int(torch.randint(1, 5, (1,), generator=gen))
        cuts = sorted(set(int(c) for c in torch.randint(1, max(2, true_len), (nsplit,), generator=gen)))
        bounds = [0] + [c for c in cuts if c < true_len] + [true_len]
        for si in range(len(bounds) - 1):
            seq[bi, bounds[si]:bounds[si + 1]] = si
        seq[bi, true_len:] = -1
    return seq


@pytest.mark.parametrize("seqlen", [8, 64, 151, 1134])
@pytest.mark.parametrize("width", [2, 3, 4])
@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("pad", [False, True])
def test_seq_idx_vs_oracle(seqlen, width, dt, pad):
    gen = torch.Generator().manual_seed(seqlen * 13 + width + 100 * pad)
    dim = 4128 if seqlen == 151 else 64
    x, w, b, _, dout, _ = make_inputs(gen, 3, dim, seqlen, width, dt, True, False, False)
    seq = make_seq_idx(gen, 3, seqlen, pad)
    for layout in ("channel_last", "contiguous"):
        check_against_oracle(x, w, b, seq, None, False, True, dout, None, layout)


# ------------------------------------------------------------- silu accuracy
@pytest.mark.parametrize("dt", DTYPES)
def test_silu_range(dt):
    """Pre-activations across [-40, 40] (identity weight, no bias) vs the oracle."""
    vals = torch.linspace(-40, 40, 8 * 4096)
    x = vals.reshape(8, 1, 4096).expand(8, 64, 4096).contiguous().to(TORCH_DT[dt])
    w = torch.zeros(64, 4)
    w[:, -1] = 1.0
    dout = torch.ones_like(x)
    check_against_oracle(x, w, None, None, None, False, True, dout, None, "channel_last")


# ----------------------------------------------------------- determinism
def test_backward_is_bit_reproducible():
    """The reference's race detector (tests/test_causal_conv1d.py:342-398), fewer rounds."""
    gen = torch.Generator().manual_seed(0)
    dim, seqlen = 4096 + 32, 2048
    wide = torch.randn(2, seqlen, 4096 + dim + 64, generator=gen).to(torch.bfloat16).cuda()
    x = wide[:, :, 4096:4096 + dim].transpose(1, 2).requires_grad_()
    w = torch.randn(dim, 4, generator=gen).cuda().requires_grad_()
    b = torch.randn(dim, generator=gen).cuda().requires_grad_()
    out0 = causal_conv1d_fn(x, w, b, activation="silu")
    g = torch.randn(out0.shape, generator=gen).to(torch.bfloat16).cuda()
    dx0, dw0, db0 = torch.autograd.grad(out0, (x, w, b), g)
    for _ in range(200):
        out = causal_conv1d_fn(x, w, b, activation="silu")
        dx, dw, db = torch.autograd.grad(out, (x, w, b), g)
        assert torch.equal(out, out0)
        assert torch.equal(dx, dx0)
        assert torch.equal(dw, dw0)
        assert torch.equal(db, db0)


@pytest.mark.parametrize("channel_last", [False, True])
def test_deterministic_env_modes_agree(channel_last, monkeypatch):
    gen = torch.Generator().manual_seed(123)
    x = torch.randn(4, 1024, 2048, generator=gen).to(torch.bfloat16).cuda()
    if channel_last:
        x = with_layout(x, "channel_last")
    w = torch.randn(1024, 4, generator=gen).cuda()
    b = torch.randn(1024, generator=gen).cuda()
    g = torch.randn(x.shape, generator=gen).to(torch.bfloat16).cuda()
    res = []
    for mode in ("1", "0"):
        monkeypatch.setenv("CAUSAL_CONV1D_DETERMINISTIC", mode)
        res.append(causal_conv1d_bwd_function(x, w, b, g, None, None, None, None, False, True))
    for u, v in zip(res[0][:3], res[1][:3]):
        assert torch.equal(u, v)


def test_runs_on_the_current_stream():
    """Launches follow torch.cuda.current_stream() (reference
    tests/test_cutedsl_backward.py:418-452)."""
    gen = torch.Generator().manual_seed(1165)
    xs = torch.randn(2, 65, 72, generator=gen).to(torch.bfloat16)
    ws = torch.randn(72, 4, generator=gen)
    bs = torch.randn(72, generator=gen)
    gs = torch.randn(2, 65, 72, generator=gen).to(torch.bfloat16)
    stream = torch.cuda.Stream()
    done = torch.cuda.Event()
    with torch.cuda.stream(stream):
        x = xs.cuda().transpose(1, 2)
        w, b, g = ws.cuda(), bs.cuda(), gs.cuda().transpose(1, 2)
        torch.cuda._sleep(20_000_000)  # keep the side stream busy so ordering matters
        dx, dw, db, _ = causal_conv1d_bwd_function(x, w, b, g, None, None, None, None, False, True)
        done.record(stream)
    torch.cuda.current_stream().wait_event(done)
    edx, edw, edb, _ = O.bwd(to_storage(xs.transpose(1, 2)), "bfloat16", ws.numpy(), "float32",
                             to_storage(gs.transpose(1, 2)), bs.numpy(), "float32", silu=True)
    assert_close(dx, edx, "bfloat16", PARITY["bfloat16"])
    assert_close(dw, edw, "float32", GRAD_PARAM["float32"])
    assert_close(db, edb, "float32", GRAD_PARAM["float32"])


def test_caller_dx_buffer_is_filled():
    """bwd_function writes a caller-provided dx in place (reference interface.py:75-77)."""
    gen = torch.Generator().manual_seed(5)
    x = torch.randn(2, 128, 300, generator=gen).to(torch.float16).cuda()
    w = torch.randn(128, 3, generator=gen).cuda()
    g = torch.randn(x.shape, generator=gen).to(torch.float16).cuda()
    dx = torch.full_like(x, 7.0)
    ret = causal_conv1d_bwd_function(x, w, None, g, None, None, None, dx, False, False)
    assert ret[0] is dx
    edx, _, _, _ = O.bwd(to_storage(x), "float16", to_storage(w), "float32", to_storage(g))
    assert_close(dx, edx, "float16", PARITY["float16"])


def test_mixed_layout_dout():
    """dout in a different layout than x still runs on the kernels."""
    gen = torch.Generator().manual_seed(9)
    x = torch.randn(2, 64, 100, generator=gen).to(torch.bfloat16)
    w = torch.randn(64, 4, generator=gen)
    g = torch.randn(x.shape, generator=gen).to(torch.bfloat16)
    xg = with_layout(x.cuda(), "channel_last")
    gg = g.cuda().contiguous()
    dx, dw, _, _ = causal_conv1d_bwd_function(xg, w.cuda(), None, gg, None, None, None, None, False, True)
    edx, edw, _, _ = O.bwd(to_storage(x), "bfloat16", w.numpy(), "float32", to_storage(g), silu=True)
    assert_close(dx, edx, "bfloat16", PARITY["bfloat16"])
    assert_close(dw, edw, "float32", GRAD_PARAM["float32"])


def test_fwd_function_final_states_contiguous_buffer():
    """final_states_out may be (batch, dim, width-1) contiguous (the benchmark's layout)."""
    gen = torch.Generator().manual_seed(4)
    x = torch.randn(4, 256, 37, generator=gen).to(torch.bfloat16)
    w = torch.randn(256, 4, generator=gen) - 0.5
    init = torch.randn(4, 256, 3, generator=gen).to(torch.bfloat16)
    fin = torch.empty(4, 256, 3, dtype=torch.bfloat16, device="cuda")
    out = causal_conv1d_fwd_function(with_layout(x.cuda(), "channel_last"), w.cuda(), None, None,
                                     init.cuda(), fin, True)
    eo, ef = O.fwd(to_storage(x), "bfloat16", w.numpy(), "float32", initial_states=to_storage(init),
                   silu=True, return_final_states=True)
    assert_close(out, eo, "bfloat16", PARITY["bfloat16"])
    assert np.array_equal(to_storage(fin), ef)


@pytest.mark.parametrize("dt", ["float32", "bfloat16"])
@pytest.mark.parametrize("seqlen", [8, 96, 256, 1000])
@pytest.mark.parametrize("width", [2, 4])
def test_contiguous_states_through_functions(dt, seqlen, width):
    """(batch, dim, seqlen)-contiguous x with initial/final states and dinitial/dfinal.
    The public interface only returns final states for channel-last x, so this drives
    the row-walk state handling through the host functions directly."""
    from causal_conv1d.cpp_functions import causal_conv1d_bwd_function, causal_conv1d_fwd_function

    gen = torch.Generator().manual_seed(seqlen * 17 + width)
    x, w, b, init, dout, dfinal = make_inputs(gen, 3, 40, seqlen, width, dt, True, True, True)
    fin = torch.empty(3, 40, width - 1, dtype=TORCH_DT[dt], device="cuda")
    out = causal_conv1d_fwd_function(x.cuda(), w.cuda(), b.cuda(), None, init.cuda(), fin, True)
    dx, dw, db, di = causal_conv1d_bwd_function(x.cuda(), w.cuda(), b.cuda(), dout.cuda(), None, init.cuda(),
                                                dfinal.cuda(), None, True, True)
    xs, ws, bs, inits = to_storage(x), to_storage(w), to_storage(b), to_storage(init)
    eo, ef = O.fwd(xs, dt, ws, "float32", bs, "float32", initial_states=inits, silu=True, return_final_states=True)
    edx, edw, edb, edi = O.bwd(xs, dt, ws, "float32", to_storage(dout), bs, "float32", initial_states=inits,
                               dfinal_states=to_storage(dfinal), silu=True)
    assert_close(out, eo, dt, PARITY[dt], "out")
    assert np.array_equal(to_storage(fin), ef)
    assert_close(dx, edx, dt, PARITY[dt], "dx")
    assert_close(dw, edw, "float32", GRAD_PARAM["float32"], "dweight")
    assert_close(db, edb, "float32", GRAD_PARAM["float32"], "dbias")
    assert_close(di, edi, dt, PARITY[dt], "dinitial")


@pytest.mark.parametrize("dt", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("width", [2, 3, 4])
@pytest.mark.parametrize("states", [False, True])
def test_dx_into_slice_of_wider_gradient_buffer(dt, width, states):
    """Producer/consumer fusion: x is the channel slice [..., 64:64+D] of a wider
    (B, L, D+96) projection (reference tests/test_causal_conv1d.py:84-88) and the backward
    writes dx straight into the same slice of a (B, L, D+96) gradient buffer
    (reference causal_conv1d_interface.py:72-74).  dx matches the oracle and the columns
    outside the slice are left untouched."""
    gen = torch.Generator().manual_seed(31 * width + states + len(dt))
    B, D, L, W = 2, 136, 515, width
    tdt = TORCH_DT[dt]
    x, w, b, init, dout, dfinal = make_inputs(gen, B, D, L, W, dt, True, states, states)
    wide_x = torch.randn(B, L, D + 96, generator=gen).to(tdt).cuda()
    wide_x[:, :, 64:64 + D] = x.transpose(1, 2).cuda()
    xg = wide_x[:, :, 64:64 + D].transpose(1, 2)
    grad_buf = torch.full((B, L, D + 96), 3.0, dtype=tdt, device="cuda")
    dxg = grad_buf[:, :, 64:64 + D].transpose(1, 2)
    init_g = None if init is None else init.cuda()
    dfinal_g = None if dfinal is None else dfinal.cuda()
    ret = causal_conv1d_bwd_function(xg, w.cuda(), b.cuda(), with_layout(dout.cuda(), "channel_last"), None, init_g,
                                     dfinal_g, dxg, states, True)
    assert ret[0] is dxg
    edx, edw, edb, edi = O.bwd(to_storage(x), dt, to_storage(w), "float32", to_storage(dout), to_storage(b),
                               "float32", initial_states=to_storage(init), dfinal_states=to_storage(dfinal),
                               silu=True)
    assert_close(dxg, edx, dt, PARITY[dt], "dx in the slice")
    assert_close(ret[1], edw, "float32", GRAD_PARAM["float32"], "dweight")
    assert_close(ret[2], edb, "float32", GRAD_PARAM["float32"], "dbias")
    if states:
        assert_close(ret[3], edi, dt, PARITY[dt], "dinitial")
    outside = torch.cat([grad_buf[:, :, :64], grad_buf[:, :, 64 + D:]], dim=2)
    assert torch.all(outside == 3.0), "columns outside the slice must not be written"
