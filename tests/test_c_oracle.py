"""The C restatement (timed CPU baseline) agrees with the numpy oracle and the golden
vectors.  CPU only."""

import numpy as np
import pytest

from golden_io import case_id, load_cases
from oracle import c_oracle as C
from oracle import numpy_oracle as O
from tolerances import PIN

CASES = [c for c in load_cases("fwd_bwd") + load_cases("seq_idx") if c[0]["w_dtype"] == "float32"]


@pytest.mark.parametrize("case", CASES, ids=[case_id(m) for m, _ in CASES])
def test_c_oracle_matches_golden(case):
    meta, a = case
    dt = meta["x_dtype"]
    out, fin = C.fwd(a["x"], dt, a["weight"], a.get("bias"), seq_idx=a.get("seq_idx"),
                     initial_states=a.get("init"), silu=meta["silu"], return_final_states=meta["final"])
    rtol, atol = PIN[dt]
    np.testing.assert_allclose(O.to_f32(out, dt), O.to_f32(a["out"], dt), rtol=rtol, atol=atol)
    if meta["final"]:
        assert np.array_equal(fin, a["final"])
    dx, dw, db, di = C.bwd(a["x"], dt, a["weight"], a["dout"], a.get("bias"), seq_idx=a.get("seq_idx"),
                           initial_states=a.get("init"), dfinal_states=a.get("dfinal"), silu=meta["silu"])
    np.testing.assert_allclose(O.to_f32(dx, dt), O.to_f32(a["dx"], dt), rtol=rtol, atol=atol)
    scale = float(np.abs(a["dweight"]).max()) + 1.0
    np.testing.assert_allclose(dw, a["dweight"], rtol=2e-5, atol=2e-5 * scale)
    if meta["has_bias"]:
        np.testing.assert_allclose(db, a["dbias"], rtol=2e-5, atol=2e-5 * scale)
    if meta["has_init"]:
        np.testing.assert_allclose(O.to_f32(di, dt), O.to_f32(a["dinit"], dt), rtol=rtol, atol=atol)


def test_c_oracle_channel_last_strides():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((2, 37, 96), dtype=np.float32)  # (b, l, d)
    xv = x.transpose(0, 2, 1)  # logical (b, d, l), channel-last memory
    w = rng.uniform(-0.5, 0.5, (96, 4)).astype(np.float32)
    out, _ = C.fwd(xv, "float32", w, silu=True)
    ref, _ = O.fwd(np.ascontiguousarray(xv), "float32", w, "float32", silu=True)
    np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-5)
