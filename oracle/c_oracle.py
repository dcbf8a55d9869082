"""ctypes wrapper of the C restatement (``oracle/cc1d_oracle.c``), test infrastructure only.

``build()`` compiles ``oracle/_build/libcc1d_oracle.so`` with gcc -O3 -fopenmp.  The
wrappers take numpy arrays in storage form (bf16 as uint16 bits) with any strides and
mirror :mod:`oracle.numpy_oracle`'s ``fwd``/``bwd``.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "cc1d_oracle.c")
LIB = os.path.join(HERE, "_build", "libcc1d_oracle.so")
DT = {"float32": 0, "float16": 1, "bfloat16": 2}

_lib = None


def build(force: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    cmd = ["gcc", "-O3", "-march=x86-64-v2", "-fopenmp", "-fPIC", "-shared", SRC, "-o", LIB + ".tmp", "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


def load():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(LIB)
        _lib.cc1d_oracle_max_threads.restype = ctypes.c_int
    return _lib


def max_threads() -> int:
    return int(load().cc1d_oracle_max_threads())


def use_all_cores() -> int:
    """Run the OpenMP loops on every core this process may use; returns that count."""
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    load().cc1d_oracle_set_threads(ctypes.c_int(n))
    return max_threads()


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _strides(a, ndim=3):
    if a is None:
        return None
    s = [st // a.itemsize for st in a.strides] + [0] * (ndim - a.ndim)
    return (ctypes.c_int64 * 3)(*s[:3])


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def _store_dtype(dtype):
    return {"float32": np.float32, "float16": np.float16, "bfloat16": np.uint16}[dtype]


def fwd(x, x_dtype, weight_f32, bias_f32=None, seq_idx=None, initial_states=None, i_dtype=None,
        silu=False, return_final_states=False, out=None):
    """Forward on storage arrays; weights/bias as float32.  Returns (out, final)."""
    lib = load()
    b, d, l = x.shape
    w = _f32(weight_f32)
    width = w.shape[1]
    bias = _f32(bias_f32)
    seq = None if seq_idx is None else np.ascontiguousarray(seq_idx, dtype=np.int32)
    if out is None:
        out = np.empty((b, d, l), _store_dtype(x_dtype))
    fin = np.empty((b, d, width - 1), _store_dtype(x_dtype)) if return_final_states else None
    lib.cc1d_oracle_fwd(
        ctypes.c_int64(b), ctypes.c_int64(d), ctypes.c_int64(l), ctypes.c_int(width),
        ctypes.c_int(DT[x_dtype]), _ptr(x), _strides(x), _ptr(w), _ptr(bias), _ptr(seq),
        ctypes.c_int(DT[i_dtype or x_dtype]), _ptr(initial_states), _strides(initial_states),
        ctypes.c_int(int(silu)), _ptr(out), _strides(out), ctypes.c_int(DT[x_dtype]), _ptr(fin), _strides(fin))
    return out, fin


def bwd(x, x_dtype, weight_f32, dout, bias_f32=None, seq_idx=None, initial_states=None, i_dtype=None,
        dfinal_states=None, silu=False, return_dinitial=True, dx=None):
    """Backward on storage arrays; returns (dx, dweight_f32, dbias_f32, dinitial)."""
    lib = load()
    b, d, l = x.shape
    w = _f32(weight_f32)
    width = w.shape[1]
    bias = _f32(bias_f32)
    seq = None if seq_idx is None else np.ascontiguousarray(seq_idx, dtype=np.int32)
    if dx is None:
        dx = np.empty((b, d, l), _store_dtype(x_dtype))
    dinit = None
    if initial_states is not None and return_dinitial:
        dinit = np.empty((b, d, width - 1), _store_dtype(i_dtype or x_dtype))
    dweight = np.empty((d, width), np.float32)
    dbias = np.empty((d,), np.float32) if bias is not None else None
    rc = lib.cc1d_oracle_bwd(
        ctypes.c_int64(b), ctypes.c_int64(d), ctypes.c_int64(l), ctypes.c_int(width),
        ctypes.c_int(DT[x_dtype]), _ptr(x), _strides(x), _ptr(w), _ptr(bias), _ptr(seq),
        ctypes.c_int(DT[i_dtype or x_dtype]), _ptr(initial_states), _strides(initial_states),
        _ptr(dout), _strides(dout), ctypes.c_int(DT[x_dtype]), _ptr(dfinal_states), _strides(dfinal_states),
        ctypes.c_int(int(silu)), _ptr(dx), _strides(dx), _ptr(dinit), _strides(dinit),
        _ptr(dweight), _ptr(dbias))
    if rc != 0:
        raise MemoryError("cc1d_oracle_bwd: allocation failed")
    return dx, dweight, dbias, dinit
