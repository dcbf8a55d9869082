"""Build libcc1d_b200.so (the C-ABI library of the causal_conv1d B200 kernels).

    python cute-causal-conv1d_b200/cc1d_build.py [--force] [--verbose]

Compiles every kernel file for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``)
with nvcc, in parallel; the per-element-type kernel files are compiled once per type.
The library is written next to the Python package (``causal_conv1d/libcc1d_b200.so``),
in the source tree, and is rebuilt only when a source or header is newer.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "causal_conv1d", "libcc1d_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2",
    "-I" + INCLUDE, "-I" + CSRC,
]

# (source, extra defines, object name)
UNITS = [
    ("cc1d_abi.cu", [], "cc1d_abi.o"),
    ("cc1d_update.cu", [], "cc1d_update.o"),
    ("cc1d_decode.cu", [], "cc1d_decode.o"),
    ("cc1d_static.cu", [], "cc1d_static.o"),
] + [
    (src, [f"-DCC1D_DT={dt}"], f"{src[:-3]}_{name}.o")
    for src in ("cc1d_fwd.cu", "cc1d_bwd.cu", "cc1d_rows.cu", "cc1d_rowwalk.cu")
    for dt, name in ((0, "f32"), (1, "f16"), (2, "bf16"))
]


def nvcc() -> str:
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(exe):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libcc1d_b200.so")
    return exe


def _inputs():
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    files += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    files.append(os.path.abspath(__file__))
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    lib_mtime = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= lib_mtime for f in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    exe = nvcc()

    def compile_unit(unit):
        src, defs, obj = unit
        cmd = [exe] + NVCC_FLAGS + defs + ["-c", os.path.join(CSRC, src), "-o", os.path.join(BUILD, obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src} {defs}:\n{res.stdout}\n{res.stderr}")
        return res.stderr

    workers = max(1, min(len(UNITS), os.cpu_count() or 4))
    with ThreadPoolExecutor(workers) as pool:
        logs = list(pool.map(compile_unit, UNITS))
    if verbose:
        for log in logs:
            sys.stderr.write(log)
    objs = [os.path.join(BUILD, u[2]) for u in UNITS]
    tmp = LIB + ".tmp"
    cmd = [exe] + ARCH + ["-shared", "-o", tmp] + objs
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
