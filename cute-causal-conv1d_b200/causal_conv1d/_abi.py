"""ctypes binding of ``libcc1d_b200.so`` (the C ABI in ``include/causal_conv1d_b200.h``).

Every call launches on the current PyTorch stream of the tensors' device, under a device
guard, and returns without synchronising.  There is no CPU fallback: if the library is
missing or a tensor is not on a CUDA device, the call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

LIB_NAME = "libcc1d_b200.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

_DTYPES = {
    torch.float32: 0,
    torch.float16: 1,
    torch.bfloat16: 2,
    torch.int32: 3,
    torch.int64: 4,
}

c_i32, c_i64, c_void_p = ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p


class CTensor(ctypes.Structure):
    _fields_ = [("data", c_void_p), ("dtype", c_i32), ("reserved", c_i32), ("stride", c_i64 * 3)]


class FwdParams(ctypes.Structure):
    _fields_ = [
        ("batch", c_i64), ("dim", c_i64), ("seqlen", c_i64), ("width", c_i64),
        ("x", CTensor), ("weight", CTensor), ("bias", CTensor), ("seq_idx", CTensor),
        ("initial_states", CTensor), ("final_states", CTensor), ("out", CTensor),
        ("silu", c_i32), ("reserved", c_i32),
    ]


class BwdParams(ctypes.Structure):
    _fields_ = [
        ("batch", c_i64), ("dim", c_i64), ("seqlen", c_i64), ("width", c_i64),
        ("x", CTensor), ("weight", CTensor), ("bias", CTensor), ("seq_idx", CTensor),
        ("initial_states", CTensor), ("dout", CTensor), ("dfinal_states", CTensor),
        ("dx", CTensor), ("dinitial_states", CTensor),
        ("dweight", c_void_p), ("dbias", c_void_p), ("workspace", c_void_p),
        ("workspace_bytes", c_i64), ("silu", c_i32), ("reserved", c_i32),
    ]


class UpdateParams(ctypes.Structure):
    _fields_ = [
        ("batch", c_i64), ("dim", c_i64), ("seqlen", c_i64), ("width", c_i64),
        ("state_batch", c_i64), ("state_len", c_i64),
        ("x", CTensor), ("conv_state", CTensor), ("weight", CTensor), ("bias", CTensor),
        ("cache_seqlens", CTensor), ("conv_state_indices", CTensor), ("out", CTensor),
        ("silu", c_i32), ("reserved", c_i32),
    ]


class VarlenParams(ctypes.Structure):
    _fields_ = [
        ("batch", c_i64), ("dim", c_i64), ("state_len", c_i64), ("total_tokens", c_i64),
        ("x", CTensor), ("cu_seqlens", CTensor), ("states", CTensor),
    ]


class FwdVarlenStatesParams(ctypes.Structure):
    _fields_ = [
        ("fwd", FwdParams), ("nseq", c_i64), ("state_len", c_i64),
        ("cu_seqlens", CTensor), ("states", CTensor),
    ]


# Bytes of the library's static backward scratch array (CC1D_STATIC_SCRATCH_BYTES).
STATIC_SCRATCH_BYTES = 32 * 1024 * 1024

# symbol -> (restype, argtypes); the same list is checked by the CPU test suite
SIGNATURES = {
    "cc1d_fwd_launch": (c_i32, [ctypes.POINTER(FwdParams), c_void_p]),
    "cc1d_bwd_workspace_bytes": (c_i64, [ctypes.POINTER(BwdParams)]),
    "cc1d_bwd_launch": (c_i32, [ctypes.POINTER(BwdParams), c_void_p]),
    "cc1d_bwd_launch_static": (c_i32, [ctypes.POINTER(BwdParams), c_void_p]),
    "cc1d_update_launch": (c_i32, [ctypes.POINTER(UpdateParams), c_void_p]),
    "cc1d_varlen_states_launch": (c_i32, [ctypes.POINTER(VarlenParams), c_void_p]),
    "cc1d_fwd_varlen_states_launch": (c_i32, [ctypes.POINTER(FwdVarlenStatesParams), c_void_p]),
    "cc1d_last_error": (ctypes.c_char_p, []),
    "cc1d_status_string": (ctypes.c_char_p, [c_i32]),
    "cc1d_abi_version": (c_i32, []),
    "cc1d_launch_count": (c_i64, []),
}

_ERRORS = {1: ValueError, 2: TypeError, 3: NotImplementedError, 4: RuntimeError}

_lib = None
_lock = threading.Lock()


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load (once) and return the C-ABI library; raise ImportError if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(path):
                raise ImportError(
                    f"{path} is missing: build it with `python cute-causal-conv1d_b200/cc1d_build.py` "
                    "(nvcc, sm_100a). causal_conv1d has no CPU fallback."
                )
            lib = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def _ct(t: torch.Tensor | None) -> CTensor:
    if t is None:
        return CTensor()
    try:
        code = _DTYPES[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}") from None
    s = list(t.stride()) + [0] * (3 - t.dim())
    return CTensor(t.data_ptr(), code, 0, (c_i64 * 3)(*s[:3]))


def _check(status: int) -> None:
    if status != 0:
        msg = load_library().cc1d_last_error().decode()
        raise _ERRORS.get(status, RuntimeError)(msg or f"causal_conv1d error {status}")


def _expect(name: str, t: torch.Tensor | None, shape: tuple) -> None:
    """Reject a tensor whose shape is not the one the kernels will index.  The C ABI
    receives pointers and strides only, so a tensor that is too small would otherwise be
    read or written out of bounds."""
    if t is not None and tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {tuple(shape)}, got {tuple(t.shape)}")


def _expect_dims(name: str, t: torch.Tensor, ndim: int) -> None:
    if t.dim() != ndim:
        raise ValueError(f"{name} must have {ndim} dimensions, got shape {tuple(t.shape)}")


def _conv_shapes(x, weight, bias, seq_idx, initial_states):
    """(batch, dim, seqlen, width) of a conv call after checking its input shapes."""
    _expect_dims("x", x, 3)
    _expect_dims("weight", weight, 2)
    B, D, L = x.shape
    W = weight.shape[1]
    _expect("weight", weight, (D, W))
    _expect("bias", bias, (D,))
    _expect("seq_idx", seq_idx, (B, L))
    _expect("initial_states", initial_states, (B, D, W - 1))
    return B, D, L, W


def _device_of(*tensors: torch.Tensor | None) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("causal_conv1d needs CUDA tensors (there is no CPU implementation)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"all tensors must be on one device ({dev} vs {t.device})")
    return dev


class _Guard:
    """Make ``device`` current for the launch (cheap when it already is)."""

    __slots__ = ("dev", "prev")

    def __init__(self, dev: torch.device):
        self.dev = dev.index if dev.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.dev:
            self.prev = cur
            torch.cuda.set_device(self.dev)
        return torch.cuda.current_stream(self.dev).cuda_stream

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False


def fwd(x, weight, bias, seq_idx, initial_states, final_states, out, silu: bool) -> None:
    B, D, L, W = _conv_shapes(x, weight, bias, seq_idx, initial_states)
    _expect("final_states", final_states, (B, D, W - 1))
    _expect("out", out, (B, D, L))
    lib = load_library()
    dev = _device_of(x, weight, bias, seq_idx, initial_states, final_states, out)
    p = FwdParams(
        x.shape[0], x.shape[1], x.shape[2], weight.shape[1],
        _ct(x), _ct(weight), _ct(bias), _ct(seq_idx), _ct(initial_states),
        _ct(final_states), _ct(out), int(bool(silu)), 0,
    )
    with _Guard(dev) as stream:
        _check(lib.cc1d_fwd_launch(ctypes.byref(p), stream))


def _bwd_params(x, weight, bias, dout, seq_idx, initial_states, dfinal_states, dx, dinitial_states,
                dweight_f32, dbias_f32, silu: bool):
    B, D, L, W = _conv_shapes(x, weight, bias, seq_idx, initial_states)
    for name, t in (("dout", dout), ("dx", dx)):
        _expect(name, t, (B, D, L))
    for name, t in (("dfinal_states", dfinal_states), ("dinitial_states", dinitial_states)):
        _expect(name, t, (B, D, W - 1))
    _expect("dweight", dweight_f32, (D, W))
    _expect("dbias", dbias_f32, (D,))
    dev = _device_of(x, weight, bias, dout, seq_idx, initial_states, dfinal_states, dx,
                     dinitial_states, dweight_f32, dbias_f32)
    p = BwdParams(
        x.shape[0], x.shape[1], x.shape[2], weight.shape[1],
        _ct(x), _ct(weight), _ct(bias), _ct(seq_idx), _ct(initial_states), _ct(dout),
        _ct(dfinal_states), _ct(dx), _ct(dinitial_states),
        dweight_f32.data_ptr(), dbias_f32.data_ptr() if dbias_f32 is not None else None,
        None, 0, int(bool(silu)), 0,
    )
    return p, dev


def bwd_workspace_bytes(x, weight, bias, dout, seq_idx, initial_states, dfinal_states, dx,
                        dinitial_states, dweight_f32, dbias_f32, silu: bool) -> int:
    """Device scratch bytes ``bwd`` needs for these arguments (``cc1d_bwd_workspace_bytes``),
    so that a caller can allocate it once and pass it to every call."""
    p, _ = _bwd_params(x, weight, bias, dout, seq_idx, initial_states, dfinal_states, dx,
                       dinitial_states, dweight_f32, dbias_f32, silu)
    lib = load_library()
    need = lib.cc1d_bwd_workspace_bytes(ctypes.byref(p))
    if need < 0:
        _check(lib.cc1d_bwd_launch(ctypes.byref(p), None))  # raises with the message
    return int(need)


def bwd(x, weight, bias, dout, seq_idx, initial_states, dfinal_states, dx, dinitial_states,
        dweight_f32, dbias_f32, silu: bool, workspace: torch.Tensor | None = None) -> None:
    p, dev = _bwd_params(x, weight, bias, dout, seq_idx, initial_states, dfinal_states, dx,
                         dinitial_states, dweight_f32, dbias_f32, silu)
    lib = load_library()
    need = lib.cc1d_bwd_workspace_bytes(ctypes.byref(p))
    if need < 0:
        _check(lib.cc1d_bwd_launch(ctypes.byref(p), None))  # raises with the message
    if need > 0:
        if workspace is None or workspace.numel() < need:
            workspace = torch.empty(need, dtype=torch.uint8, device=dev)
        p.workspace = workspace.data_ptr()
        p.workspace_bytes = workspace.numel()
    with _Guard(dev) as stream:
        _check(lib.cc1d_bwd_launch(ctypes.byref(p), stream))


def update(x, conv_state, weight, bias, cache_seqlens, conv_state_indices, out, silu: bool) -> None:
    B, D, T, W = _conv_shapes(x, weight, bias, None, None)
    _expect_dims("conv_state", conv_state, 3)
    if conv_state.shape[1] != D:
        raise ValueError(f"conv_state must have dim {D} in its second dimension, got shape {tuple(conv_state.shape)}")
    _expect("cache_seqlens", cache_seqlens, (B,))
    _expect("conv_state_indices", conv_state_indices, (B,))
    _expect("out", out, (B, D, T))
    lib = load_library()
    dev = _device_of(x, conv_state, weight, bias, cache_seqlens, conv_state_indices, out)
    p = UpdateParams(
        x.shape[0], x.shape[1], x.shape[2], weight.shape[1], conv_state.shape[0], conv_state.shape[2],
        _ct(x), _ct(conv_state), _ct(weight), _ct(bias), _ct(cache_seqlens),
        _ct(conv_state_indices), _ct(out), int(bool(silu)), 0,
    )
    with _Guard(dev) as stream:
        _check(lib.cc1d_update_launch(ctypes.byref(p), stream))


def varlen_states(x, cu_seqlens, states) -> None:
    _expect_dims("x", x, 2)
    _expect_dims("cu_seqlens", cu_seqlens, 1)
    _expect_dims("states", states, 3)
    _expect("states", states, (cu_seqlens.shape[0] - 1, x.shape[1], states.shape[2]))
    lib = load_library()
    dev = _device_of(x, cu_seqlens, states)
    p = VarlenParams(states.shape[0], x.shape[1], states.shape[2], x.shape[0],
                     _ct(x), _ct(cu_seqlens), _ct(states))
    with _Guard(dev) as stream:
        _check(lib.cc1d_varlen_states_launch(ctypes.byref(p), stream))


def fwd_varlen_states(x, weight, bias, seq_idx, cu_seqlens, states, out, silu: bool) -> None:
    B, D, L, W = _conv_shapes(x, weight, bias, seq_idx, None)
    _expect("out", out, (B, D, L))
    _expect_dims("cu_seqlens", cu_seqlens, 1)
    _expect_dims("states", states, 3)
    _expect("states", states, (cu_seqlens.shape[0] - 1, D, states.shape[2]))
    lib = load_library()
    dev = _device_of(x, weight, bias, seq_idx, cu_seqlens, states, out)
    f = FwdParams(
        x.shape[0], x.shape[1], x.shape[2], weight.shape[1],
        _ct(x), _ct(weight), _ct(bias), _ct(seq_idx), _ct(None), _ct(None), _ct(out), int(bool(silu)), 0,
    )
    p = FwdVarlenStatesParams(f, states.shape[0], states.shape[2], _ct(cu_seqlens), _ct(states))
    with _Guard(dev) as stream:
        _check(lib.cc1d_fwd_varlen_states_launch(ctypes.byref(p), stream))


def launch_count() -> int:
    """Kernel launches made through the library by this process."""
    return int(load_library().cc1d_launch_count())
