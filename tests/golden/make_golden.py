"""Generate golden vectors from the reference's own Python oracles.

Run in a container where the reference project is importable (it is a Python package;
its oracles run on the CPU).  The output ``*.npz`` files are committed; tests load them
on machines without the reference.  Nothing else in the repository imports the
reference.

    REFERENCE_ROOT=<path to the reference checkout> python tests/golden/make_golden.py

Reference functions used (paths relative to the reference project root):

* ``causal_conv1d/causal_conv1d_interface.py:135-174`` ``causal_conv1d_ref`` and autograd
  through it -> forward / backward / final-states vectors;
* ``causal_conv1d/cpp_functions.py:21-54`` ``_causal_conv1d_torch`` and autograd through
  it (``cpp_functions.py:115-166``) -> seq_idx (packed / padded) vectors;
* ``tests/test_cutedsl_backward.py:155-173`` fp32-accumulated formulation -> mixed-dtype
  vectors (bf16/fp16 weights), which is what the reference's fused kernels compute;
* ``causal_conv1d/causal_conv1d_interface.py:208-245`` ``causal_conv1d_update_ref`` and
  ``causal_conv1d/cpp_functions.py:190-238`` (batch gather, -1 padding) -> update vectors;
* ``causal_conv1d/causal_conv1d_varlen.py:14-26`` -> varlen state vectors.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
REF_ROOT = os.environ.get("REFERENCE_ROOT")
if not REF_ROOT:
    sys.exit("set REFERENCE_ROOT to the reference checkout (the directory holding causal_conv1d/)")
sys.path.insert(0, REF_ROOT)

from causal_conv1d.causal_conv1d_interface import (  # noqa: E402
    causal_conv1d_ref,
    causal_conv1d_update_ref,
)
from causal_conv1d.causal_conv1d_varlen import causal_conv1d_varlen_states_ref  # noqa: E402
from causal_conv1d.cpp_functions import (  # noqa: E402
    _causal_conv1d_torch,
    causal_conv1d_update_function,
)

TORCH_DT = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def store(t: torch.Tensor | None):
    """Tensor -> numpy storage form (bf16 as uint16 bits), logical shape kept."""
    if t is None:
        return None
    t = t.detach().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


class Writer:
    def __init__(self, name):
        self.name = name
        self.arrays = {}
        self.metas = []

    def add(self, meta: dict, **arrays):
        i = len(self.metas)
        meta = dict(meta, id=i)
        self.metas.append(meta)
        for k, v in arrays.items():
            if v is not None:
                self.arrays[f"c{i}_{k}"] = v

    def save(self):
        path = HERE / f"{self.name}.npz"
        np.savez_compressed(path, meta=np.array(json.dumps(self.metas)), **self.arrays)
        print(f"{path.name}: {len(self.metas)} cases, {path.stat().st_size} bytes")


def gen_fwd_bwd(w: Writer):
    """causal_conv1d_ref forward + autograd backward (stateless and stateful)."""
    shapes = [
        # (batch, dim, seqlen, bias, silu, initial, final)
        (2, 16, 1, True, True, False, True),
        (2, 16, 2, False, True, True, True),
        (1, 8, 3, True, True, True, True),
        (2, 24, 17, True, False, False, False),
        (1, 32, 65, True, True, True, True),
        (2, 8, 129, True, True, False, True),
        (2, 40, 64, False, False, True, False),
    ]
    gen = torch.Generator().manual_seed(1234)
    for itype in ("float32", "float16", "bfloat16"):
        for width in (2, 3, 4):
            for (b, d, l, has_bias, silu, has_init, final) in shapes:
                dt = TORCH_DT[itype]
                x = torch.randn(b, d, l, generator=gen).to(dt)
                weight = torch.randn(d, width, generator=gen)
                bias = torch.randn(d, generator=gen) if has_bias else None
                init = torch.randn(b, d, width - 1, generator=gen).to(dt) if has_init else None
                xr = x.clone().requires_grad_()
                wr = weight.clone().requires_grad_()
                br = bias.clone().requires_grad_() if bias is not None else None
                ir = init.clone().requires_grad_() if init is not None else None
                act = "silu" if silu else None
                res = causal_conv1d_ref(xr, wr, br, initial_states=ir,
                                        return_final_states=final, activation=act)
                out, fin = (res if final else (res, None))
                dout = torch.randn(out.shape, generator=gen).to(dt)
                outs, gouts = [out], [dout]
                dfin = None
                if final:
                    dfin = torch.randn(fin.shape, generator=gen).to(dt)
                    outs.append(fin)
                    gouts.append(dfin)
                inputs = [xr, wr] + ([br] if br is not None else []) + ([ir] if ir is not None else [])
                grads = torch.autograd.grad(outs, inputs, gouts, allow_unused=True)
                gi = iter(grads)
                dx = next(gi)
                dwt = next(gi)
                dbs = next(gi) if br is not None else None
                din = next(gi) if ir is not None else None
                if din is None and ir is not None:
                    din = torch.zeros_like(init)
                meta = dict(kind="fwd_bwd", x_dtype=itype, w_dtype="float32", width=width,
                            silu=silu, has_bias=has_bias, has_init=has_init, final=final,
                            source="causal_conv1d_interface.py:135-174 + autograd")
                w.add(meta, x=store(x), weight=store(weight), bias=store(bias), init=store(init),
                      out=store(out), final=store(fin), dout=store(dout), dfinal=store(dfin),
                      dx=store(dx), dweight=store(dwt), dbias=store(dbs), dinit=store(din))


def gen_mixed(w: Writer):
    """Mixed dtypes, fp32 accumulation (tests/test_cutedsl_backward.py:155-173)."""
    gen = torch.Generator().manual_seed(99)
    combos = [("float32", "float16"), ("bfloat16", "bfloat16"), ("float16", "bfloat16"),
              ("bfloat16", "float16"), ("float32", "bfloat16")]
    for itype, wtype in combos:
        for width in (2, 4):
            b, d, l = 2, 24, 33
            x = torch.randn(b, d, l, generator=gen).to(TORCH_DT[itype])
            weight = torch.randn(d, width, generator=gen).to(TORCH_DT[wtype])
            bias = torch.randn(d, generator=gen).to(TORCH_DT[wtype])
            xr = x.clone().requires_grad_()
            wr = weight.clone().requires_grad_()
            br = bias.clone().requires_grad_()
            pre = F.conv1d(xr.float(), wr.float().unsqueeze(1), br.float(),
                           padding=width - 1, groups=d)[..., :l]
            out = F.silu(pre).to(x.dtype)
            dout = torch.randn(out.shape, generator=gen).to(x.dtype)
            dx, dwt, dbs = torch.autograd.grad(out, (xr, wr, br), dout)
            meta = dict(kind="mixed", x_dtype=itype, w_dtype=wtype, width=width, silu=True,
                        has_bias=True, has_init=False, final=False,
                        source="tests/test_cutedsl_backward.py:155-173")
            w.add(meta, x=store(x), weight=store(weight), bias=store(bias), out=store(out),
                  dout=store(dout), dx=store(dx), dweight=store(dwt), dbias=store(dbs))


def gen_seq_idx(w: Writer):
    """Packed sequences (seq_idx), with and without -1 padding (cpp_functions.py:21-54)."""
    gen = torch.Generator().manual_seed(4321)
    for itype in ("float32", "float16", "bfloat16"):
        for width in (2, 3, 4):
            for (b, d, l, pad) in ((2, 16, 40, False), (3, 8, 67, True), (1, 24, 9, False)):
                dt = TORCH_DT[itype]
                seq = torch.empty(b, l, dtype=torch.int32)
                for bi in range(b):
                    true_len = l - (int(torch.randint(1, max(2, l // 4), (1,), generator=gen)) if pad else 0)
                    nsplit = int(torch.randint(1, 5, (1,), generator=gen))
                    cuts = torch.randperm(max(true_len - 1, 1), generator=gen)[:nsplit].sort().values + 1
                    bounds = [0] + [int(c) for c in cuts if int(c) < true_len] + [true_len]
                    for si in range(len(bounds) - 1):
                        seq[bi, bounds[si]:bounds[si + 1]] = si + 10 * bi
                    seq[bi, true_len:] = -1
                x = torch.randn(b, d, l, generator=gen).to(dt)
                weight = torch.randn(d, width, generator=gen)
                bias = torch.randn(d, generator=gen)
                xr = x.clone().requires_grad_()
                wr = weight.clone().requires_grad_()
                br = bias.clone().requires_grad_()
                for silu in (False, True):
                    out = _causal_conv1d_torch(xr, wr, br, seq, None, silu)
                    dout = torch.randn(out.shape, generator=gen).to(dt)
                    dx, dwt, dbs = torch.autograd.grad(out, (xr, wr, br), dout)
                    meta = dict(kind="seq_idx", x_dtype=itype, w_dtype="float32", width=width,
                                silu=silu, has_bias=True, has_init=False, final=False, padded=pad,
                                source="cpp_functions.py:21-54 + autograd (cpp_functions.py:115-166)")
                    w.add(meta, x=store(x), weight=store(weight), bias=store(bias),
                          seq_idx=seq.numpy().copy(), out=store(out), dout=store(dout),
                          dx=store(dx), dweight=store(dwt), dbias=store(dbs))


def _channel_first(t: torch.Tensor) -> torch.Tensor:
    """A view with stride(1) != 1 so cpp_functions takes its PyTorch update path."""
    wide = torch.zeros(*t.shape[:-1], t.shape[-1] + 1, dtype=t.dtype)
    wide[..., : t.shape[-1]] = t
    return wide[..., : t.shape[-1]]


def gen_update(w: Writer):
    """causal_conv1d_update_ref and the gather/padding path of cpp_functions."""
    gen = torch.Generator().manual_seed(777)
    for itype in ("float32", "float16", "bfloat16"):
        dt = TORCH_DT[itype]
        for width in (2, 3, 4):
            for seqlen in (1, 4, 5):
                for circular in (False, True):
                    for mode in ("plain", "gather", "padding"):
                        b, d = 6, 8
                        state_len = int(torch.randint(width - 1, width + 10, (1,), generator=gen))
                        if seqlen == 5 and mode == "plain":
                            state_len = width - 1  # seqlen > state_len: wrap / duplicate writes
                        x = torch.randn(b, d, seqlen, generator=gen).to(dt)
                        weight = torch.randn(d, width, generator=gen)
                        bias = torch.randn(d, generator=gen)
                        silu = bool(torch.randint(0, 2, (1,), generator=gen))
                        act = "silu" if silu else None
                        cache = (torch.randint(0, 1024, (b,), generator=gen, dtype=torch.int32)
                                 if circular else None)
                        if mode == "plain":
                            state = torch.randn(b, d, state_len, generator=gen).to(dt)
                            indices = None
                            st = state.clone()
                            out = causal_conv1d_update_ref(x, st, weight, bias, activation=act,
                                                           cache_seqlens=cache)
                            src = "causal_conv1d_interface.py:208-245"
                        else:
                            total = 3 * b
                            state = torch.randn(total, d, state_len, generator=gen).to(dt)
                            indices = torch.randperm(total, generator=gen)[:b].to(torch.int32)
                            if mode == "padding":
                                indices[torch.randperm(b, generator=gen)[: b // 2]] = -1
                            st = _channel_first(state.clone())
                            out = causal_conv1d_update_function(
                                _channel_first(x), st, weight, bias, silu, cache, indices)
                            src = "cpp_functions.py:190-238"
                        meta = dict(kind="update", x_dtype=itype, w_dtype="float32",
                                    width=width, silu=silu, circular=circular, mode=mode,
                                    source=src)
                        w.add(meta, x=store(x), state=store(state), weight=store(weight),
                              bias=store(bias), cache_seqlens=None if cache is None else cache.numpy(),
                              indices=None if indices is None else indices.numpy(),
                              out=store(out), new_state=store(st))


def gen_varlen(w: Writer):
    """causal_conv1d_varlen_states_ref (causal_conv1d_varlen.py:14-26)."""
    gen = torch.Generator().manual_seed(31)
    for itype in ("float32", "float16", "bfloat16"):
        for (nseq, maxlen, dim, state_len, idx_dtype) in (
            (100, 32, 16, 20, torch.int64),
            (7, 5, 24, 3, torch.int32),
            (12, 40, 8, 4, torch.int32),
        ):
            seqlens = torch.randint(1, maxlen, (nseq,), generator=gen)
            cu = F.pad(seqlens.cumsum(0), (1, 0)).to(idx_dtype)
            x = torch.randn(int(seqlens.sum()), dim, generator=gen).to(TORCH_DT[itype])
            out = causal_conv1d_varlen_states_ref(x, cu, state_len)
            meta = dict(kind="varlen", x_dtype=itype, state_len=state_len,
                        cu_dtype=str(idx_dtype).replace("torch.", ""),
                        source="causal_conv1d_varlen.py:14-26")
            w.add(meta, x=store(x), cu_seqlens=cu.numpy(), out=store(out))


def gen_config1(w: Writer):
    """Benchmark config 1: fp32 (2, 64, 512) contiguous, W=4, silu, seed 0."""
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(2, 64, 512, generator=gen)
    weight = torch.rand(64, 4, generator=gen) - 0.5
    bias = torch.randn(64, generator=gen) * 0.1
    xr = x.clone().requires_grad_()
    wr = weight.clone().requires_grad_()
    br = bias.clone().requires_grad_()
    out = causal_conv1d_ref(xr, wr, br, activation="silu")
    dout = torch.randn(out.shape, generator=gen)
    dx, dwt, dbs = torch.autograd.grad(out, (xr, wr, br), dout)
    meta = dict(kind="fwd_bwd", x_dtype="float32", w_dtype="float32", width=4, silu=True,
                has_bias=True, has_init=False, final=False, config="config1",
                source="causal_conv1d_interface.py:135-174 + autograd")
    w.add(meta, x=store(x), weight=store(weight), bias=store(bias), out=store(out),
          dout=store(dout), dx=store(dx), dweight=store(dwt), dbias=store(dbs))


def main():
    torch.set_num_threads(4)
    w = Writer("fwd_bwd")
    gen_fwd_bwd(w)
    gen_mixed(w)
    gen_config1(w)
    w.save()
    w = Writer("seq_idx")
    gen_seq_idx(w)
    w.save()
    w = Writer("update")
    gen_update(w)
    w.save()
    w = Writer("varlen")
    gen_varlen(w)
    w.save()


if __name__ == "__main__":
    main()
