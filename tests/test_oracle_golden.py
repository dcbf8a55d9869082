"""Pin the CPU oracle against golden vectors made by the reference's own oracles.

CPU only.  Each case in ``tests/golden/*.npz`` was produced by the reference's Python
oracles (see ``tests/golden/make_golden.py``); the numpy restatement in
``oracle/numpy_oracle.py`` must reproduce every one of them.
"""

import numpy as np
import pytest

from golden_io import case_id, load_cases
from oracle import numpy_oracle as O
from tolerances import PIN

FWD = load_cases("fwd_bwd")
SEQ = load_cases("seq_idx")
UPD = load_cases("update")
VAR = load_cases("varlen")


def close(actual, expected, dtype, tol=None, what=""):
    rtol, atol = tol or PIN[dtype]
    a = O.to_f32(actual, dtype)
    e = O.to_f32(expected, dtype)
    assert a.shape == e.shape, (what, a.shape, e.shape)
    np.testing.assert_allclose(a, e, rtol=rtol, atol=atol, err_msg=what)


def grad_tol(dtype, scale):
    rtol, atol = PIN[dtype]
    return rtol, max(atol, 1e-5 * scale)


@pytest.mark.parametrize("case", FWD + SEQ, ids=[case_id(m) for m, _ in FWD + SEQ])
def test_fwd_bwd_matches_reference_oracle(case):
    meta, a = case
    xdt, wdt = meta["x_dtype"], meta["w_dtype"]
    out, final = O.fwd(a["x"], xdt, a["weight"], wdt, a.get("bias"), wdt,
                       seq_idx=a.get("seq_idx"), initial_states=a.get("init"), i_dtype=xdt,
                       silu=meta["silu"], return_final_states=meta["final"])
    close(out, a["out"], xdt, what="out")
    if meta["final"]:
        # final states are a copy: bit exact
        assert np.array_equal(final, a["final"])
    dx, dw, db, dinit = O.bwd(a["x"], xdt, a["weight"], wdt, a["dout"], a.get("bias"), wdt,
                              seq_idx=a.get("seq_idx"), initial_states=a.get("init"), i_dtype=xdt,
                              dfinal_states=a.get("dfinal"), silu=meta["silu"])
    close(dx, a["dx"], xdt, what="dx")
    scale = float(np.abs(O.to_f32(a["dweight"], wdt)).max()) + 1.0
    close(dw, a["dweight"], wdt, grad_tol(wdt, scale), what="dweight")
    if meta["has_bias"]:
        close(db, a["dbias"], wdt, grad_tol(wdt, scale), what="dbias")
    if meta["has_init"]:
        close(dinit, a["dinit"], xdt, what="dinit")


@pytest.mark.parametrize("case", UPD, ids=[case_id(m) for m, _ in UPD])
def test_update_matches_reference_oracle(case):
    meta, a = case
    xdt = meta["x_dtype"]
    out, state = O.update(a["x"], xdt, a["state"], a["weight"], meta["w_dtype"], a["bias"],
                          silu=meta["silu"], cache_seqlens=a.get("cache_seqlens"),
                          conv_state_indices=a.get("indices"))
    close(out, a["out"], xdt, what="out")
    if meta["mode"] == "padding":
        pad = a["indices"] < 0
        assert np.all(O.to_f32(out, xdt)[pad] == 0.0)
    # conv_state is updated bit exactly
    assert np.array_equal(state, a["new_state"])


@pytest.mark.parametrize("case", VAR, ids=[case_id(m) for m, _ in VAR])
def test_varlen_states_matches_reference_oracle(case):
    meta, a = case
    out = O.varlen_states(a["x"], a["cu_seqlens"], meta["state_len"])
    assert np.array_equal(out, a["out"])


def test_bf16_rounding_is_nearest_even():
    vals = np.array([1.0, 1.00390625, 1.005859375, -2.5e-8, 3.0e38, np.inf, -np.inf], np.float32)
    bits = O.f32_to_bf16_bits(vals)
    back = O.bf16_bits_to_f32(bits)
    assert back[0] == 1.0
    assert back[1] == 1.0  # exact tie rounds to even
    assert back[2] == np.float32(1.0078125)
    assert np.isinf(back[5]) and np.isinf(back[6])
    assert np.isnan(O.bf16_bits_to_f32(O.f32_to_bf16_bits(np.array([np.nan], np.float32))))[0]
