"""C-ABI checks that need no GPU: the library loads, exports every symbol declared in
include/causal_conv1d_b200.h, and its structs match the ctypes mirror byte for byte."""

import ctypes
import os
import re
import subprocess

import pytest

from causal_conv1d import _abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "causal_conv1d_b200.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*[\w\s\*]+?\b(cc1d_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_bound_functions():
    assert declared_functions() == sorted(_abi.SIGNATURES)


def test_static_scratch_size_matches_header():
    m = re.search(r"#define CC1D_STATIC_SCRATCH_BYTES \((\d+) \* 1024 \* 1024\)", open(HEADER).read())
    assert m and int(m.group(1)) * 1024 * 1024 == _abi.STATIC_SCRATCH_BYTES


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_abi.LIB_PATH)
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_library_metadata_calls():
    lib = _abi.load_library()
    assert lib.cc1d_abi_version() == 1
    assert lib.cc1d_status_string(2) == b"CC1D_ERR_TYPE"
    assert lib.cc1d_last_error() == b""


def test_validation_errors_need_no_gpu():
    # bad width is rejected on the host before any CUDA call
    lib = _abi.load_library()
    p = _abi.FwdParams()
    p.batch, p.dim, p.seqlen, p.width = 1, 8, 4, 5
    assert lib.cc1d_fwd_launch(ctypes.byref(p), None) == 1
    assert b"width" in lib.cc1d_last_error()
    p.width = 4
    p.x.dtype = 3  # int32 x
    assert lib.cc1d_fwd_launch(ctypes.byref(p), None) == 2
    u = _abi.UpdateParams()
    u.batch, u.dim, u.seqlen, u.width, u.state_batch, u.state_len = 1, 8, 1, 4, 1, 2
    assert lib.cc1d_update_launch(ctypes.byref(u), None) == 1  # state_len < width - 1
    assert b"shorter" in lib.cc1d_last_error()
    v = _abi.VarlenParams()
    v.batch, v.dim, v.state_len = 1, 8, 2
    v.cu_seqlens.dtype = 0  # float cu_seqlens
    assert lib.cc1d_varlen_states_launch(ctypes.byref(v), None) == 2
    f = _abi.FwdVarlenStatesParams()
    f.fwd.batch, f.fwd.dim, f.fwd.seqlen, f.fwd.width = 2, 8, 4, 4  # packed sequences need batch 1
    assert lib.cc1d_fwd_varlen_states_launch(ctypes.byref(f), None) == 1
    assert b"batch == 1" in lib.cc1d_last_error()
    f.fwd.batch, f.nseq, f.state_len = 1, 2, 3
    f.cu_seqlens.dtype = 2  # bf16 cu_seqlens
    assert lib.cc1d_fwd_varlen_states_launch(ctypes.byref(f), None) == 2


def test_shape_errors_before_any_launch():
    """The launchers check every tensor's shape against the call's (batch, dim, seqlen,
    width) before touching the device: the C ABI sees only pointers and strides, so a
    tensor that is too small would otherwise be read or written out of bounds."""
    import torch

    from causal_conv1d import causal_conv1d_fn

    x = torch.empty(2, 8, 16)
    w = torch.empty(8, 4)
    out = torch.empty_like(x)
    with pytest.raises(ValueError, match="seq_idx"):
        _abi.fwd(x, w, None, torch.empty(2, 15, dtype=torch.int32), None, None, out, True)
    with pytest.raises(ValueError, match="seq_idx"):
        causal_conv1d_fn(x, w, seq_idx=torch.zeros(1, 16, dtype=torch.int32))
    with pytest.raises(ValueError, match="initial_states"):
        _abi.fwd(x, w, None, None, torch.empty(2, 8, 2), None, out, True)
    with pytest.raises(ValueError, match="final_states"):
        _abi.fwd(x, w, None, None, None, torch.empty(2, 3, 8), out, True)
    with pytest.raises(ValueError, match="bias"):
        _abi.fwd(x, w, torch.empty(7), None, None, None, out, True)
    with pytest.raises(ValueError, match="dout"):
        _abi.bwd(x, w, None, torch.empty(2, 8, 15), None, None, None, out, None, torch.empty(8, 4), None, True)
    with pytest.raises(ValueError, match="dfinal_states"):
        _abi.bwd(x, w, None, out, None, None, torch.empty(2, 8, 4), out, None, torch.empty(8, 4), None, True)
    x1 = torch.empty(2, 8, 1)
    with pytest.raises(ValueError, match="conv_state_indices"):
        _abi.update(x1, torch.empty(2, 8, 3), w, None, None, torch.empty(3, dtype=torch.int32), x1, True)
    with pytest.raises(ValueError, match="cache_seqlens"):
        _abi.update(x1, torch.empty(2, 8, 3), w, None, torch.empty(1, dtype=torch.int32), None, x1, True)
    with pytest.raises(ValueError, match="conv_state"):
        _abi.update(x1, torch.empty(2, 7, 3), w, None, None, None, x1, True)
    with pytest.raises(ValueError, match="states"):
        _abi.varlen_states(torch.empty(20, 8), torch.zeros(4, dtype=torch.int32), torch.empty(2, 8, 3))
    with pytest.raises(ValueError, match="seq_idx"):
        _abi.fwd_varlen_states(torch.empty(1, 8, 16), w, None, torch.empty(1, 12, dtype=torch.int32),
                               torch.zeros(3, dtype=torch.int32), torch.empty(2, 8, 3), torch.empty(1, 8, 16), True)


def test_empty_problem_is_a_no_op():
    lib = _abi.load_library()
    p = _abi.FwdParams()
    p.batch, p.dim, p.seqlen, p.width = 0, 8, 4, 4
    assert lib.cc1d_fwd_launch(ctypes.byref(p), None) == 0
    b = _abi.BwdParams()
    b.batch, b.dim, b.seqlen, b.width = 2, 8, 0, 3
    assert lib.cc1d_bwd_workspace_bytes(ctypes.byref(b)) == 0


C_LAYOUT_PROBE = r"""
#include <stddef.h>
#include <stdio.h>
#include "causal_conv1d_b200.h"
#define P(T, F) printf(#T "." #F " %zu\n", offsetof(T, F))
int main(void) {
  printf("cc1d_tensor %zu\ncc1d_fwd_params %zu\ncc1d_bwd_params %zu\n", sizeof(cc1d_tensor),
         sizeof(cc1d_fwd_params), sizeof(cc1d_bwd_params));
  printf("cc1d_update_params %zu\ncc1d_varlen_states_params %zu\n", sizeof(cc1d_update_params),
         sizeof(cc1d_varlen_states_params));
  P(cc1d_fwd_params, out); P(cc1d_fwd_params, silu);
  P(cc1d_bwd_params, dweight); P(cc1d_bwd_params, workspace_bytes); P(cc1d_bwd_params, silu);
  P(cc1d_update_params, out); P(cc1d_update_params, silu);
  P(cc1d_varlen_states_params, states);
  printf("cc1d_fwd_varlen_states_params %zu\n", sizeof(cc1d_fwd_varlen_states_params));
  P(cc1d_fwd_varlen_states_params, nseq); P(cc1d_fwd_varlen_states_params, states);
  return 0;
}
"""


def test_struct_layout_matches_ctypes(tmp_path):
    src = tmp_path / "probe.c"
    exe = tmp_path / "probe"
    src.write_text(C_LAYOUT_PROBE)
    try:
        subprocess.run(["gcc", "-I", os.path.dirname(HEADER), str(src), "-o", str(exe)], check=True)
    except (OSError, subprocess.CalledProcessError):
        pytest.skip("gcc unavailable")
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    got = dict(line.split() for line in out.strip().splitlines())
    py = {
        "cc1d_tensor": ctypes.sizeof(_abi.CTensor),
        "cc1d_fwd_params": ctypes.sizeof(_abi.FwdParams),
        "cc1d_bwd_params": ctypes.sizeof(_abi.BwdParams),
        "cc1d_update_params": ctypes.sizeof(_abi.UpdateParams),
        "cc1d_varlen_states_params": ctypes.sizeof(_abi.VarlenParams),
        "cc1d_fwd_params.out": _abi.FwdParams.out.offset,
        "cc1d_fwd_params.silu": _abi.FwdParams.silu.offset,
        "cc1d_bwd_params.dweight": _abi.BwdParams.dweight.offset,
        "cc1d_bwd_params.workspace_bytes": _abi.BwdParams.workspace_bytes.offset,
        "cc1d_bwd_params.silu": _abi.BwdParams.silu.offset,
        "cc1d_update_params.out": _abi.UpdateParams.out.offset,
        "cc1d_update_params.silu": _abi.UpdateParams.silu.offset,
        "cc1d_varlen_states_params.states": _abi.VarlenParams.states.offset,
        "cc1d_fwd_varlen_states_params": ctypes.sizeof(_abi.FwdVarlenStatesParams),
        "cc1d_fwd_varlen_states_params.nseq": _abi.FwdVarlenStatesParams.nseq.offset,
        "cc1d_fwd_varlen_states_params.states": _abi.FwdVarlenStatesParams.states.offset,
    }
    assert {k: int(v) for k, v in got.items()} == py


def test_torch_ops_registered_with_fake_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode

    import causal_conv1d  # noqa: F401  (registers the operators)
    import torch

    for name in ("fwd", "bwd", "update", "varlen_states", "fwd_varlen_states"):
        assert hasattr(torch.ops.causal_conv1d, name), name
    with FakeTensorMode():
        x = torch.empty(2, 512, 64).transpose(1, 2)  # (batch, dim, seqlen), channel-last
        w = torch.empty(64, 4)
        b = torch.empty(64)
        out = torch.ops.causal_conv1d.fwd(x, w, b, None, None, None, True)
        assert out.shape == x.shape and out.stride() == x.stride()
        dx, dw, db, di = torch.ops.causal_conv1d.bwd(x, w, b, x, None, None, None, False, True)
        assert dx.shape == x.shape and dw.shape == (64, 4) and db.shape == (64,) and di.numel() == 0
        st = torch.empty(2, 64, 3)
        assert torch.ops.causal_conv1d.update(x[:, :, :1], st, w, b, True, None, None).shape == (2, 64, 1)
        xs = torch.empty(100, 64)
        cu = torch.empty(4, dtype=torch.int32)
        assert torch.ops.causal_conv1d.varlen_states(xs, cu, 3).shape == (3, 64, 3)
        xp = torch.empty(1, 100, 64).transpose(1, 2)  # packed sequences, channel-last
        sq = torch.empty(1, 100, dtype=torch.int32)
        out, states = torch.ops.causal_conv1d.fwd_varlen_states(xp, w, b, sq, cu, 5, True)
        assert out.shape == xp.shape and out.stride() == xp.stride()
        assert states.shape == (3, 64, 5) and states.stride() == (320, 1, 64)


def test_legacy_module_function_table():
    import causal_conv1d_cuda

    for name in ("causal_conv1d_fwd", "causal_conv1d_bwd", "causal_conv1d_update"):
        assert callable(getattr(causal_conv1d_cuda, name))
