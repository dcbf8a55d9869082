"""Context-parallel host logic on CPU (gloo, world size 3).

The sequence of one problem is split over 3 ranks.  The kernel launches of
causal_conv1d.context_parallel are stood in for by the CPU oracle (fp32), so these tests
check the halo exchanges, the dinitial_states return path and the dweight/dbias
reduction: the concatenated outputs and input gradients, and every rank's parameter
gradients, must equal the oracle on the whole sequence.  The kernels' own parity is
covered by the -m gpu suite.
"""

import datetime
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import numpy_oracle as O

B, D, L, W = 2, 6, 30, 4
SPLITS = (0, 7, 19, 30)  # uneven slices, each >= W - 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((B, D, L), dtype=np.float32)
    w = rng.uniform(-0.5, 0.5, (D, W)).astype(np.float32)
    b = (0.1 * rng.standard_normal(D)).astype(np.float32)
    dout = rng.standard_normal((B, D, L), dtype=np.float32)
    init = rng.standard_normal((B, D, W - 1), dtype=np.float32)
    return x, w, b, dout, init


def _oracle_fwd(x, w, b, seq_idx, init, final, silu):
    out, _ = O.fwd(x.numpy(), "float32", w.numpy(), "float32", None if b is None else b.numpy(),
                   initial_states=None if init is None else init.detach().numpy(), silu=silu)
    return torch.from_numpy(out)


def _oracle_bwd(x, w, b, dout, seq_idx, init, dfinal, dx, want_dinit, silu):
    dx_, dw, db, di = O.bwd(x.numpy(), "float32", w.numpy(), "float32", dout.numpy(),
                            None if b is None else b.numpy(),
                            initial_states=None if init is None else init.detach().numpy(), silu=silu)
    return (torch.from_numpy(dx_), torch.from_numpy(dw), None if db is None else torch.from_numpy(db),
            torch.from_numpy(di) if (want_dinit and di is not None) else None)


def _worker(rank, world, port, result_dir, deterministic):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        from causal_conv1d import context_parallel as cp

        cp._fwd_impl, cp._bwd_impl = _oracle_fwd, _oracle_bwd
        x, w, b, dout, init = _problem()
        lo, hi = SPLITS[rank], SPLITS[rank + 1]
        xr = torch.from_numpy(x[:, :, lo:hi].copy()).requires_grad_()
        wt = torch.from_numpy(w).requires_grad_()
        bt = torch.from_numpy(b).requires_grad_()
        it = torch.from_numpy(init).requires_grad_()
        out = cp.causal_conv1d_fn_context_parallel(xr, wt, bt, initial_states=it, activation="silu",
                                                   deterministic=deterministic)
        out.backward(torch.from_numpy(dout[:, :, lo:hi].copy()))
        np.savez(os.path.join(result_dir, f"rank{rank}.npz"), out=out.detach().numpy(), dx=xr.grad.numpy(),
                 dw=wt.grad.numpy(), db=bt.grad.numpy(),
                 di=it.grad.numpy() if it.grad is not None else np.zeros(0, np.float32))
    finally:
        dist.destroy_process_group()


def _run(tmp_path, deterministic):
    world = len(SPLITS) - 1
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path), deterministic), nprocs=world, join=True)
    x, w, b, dout, init = _problem()
    eo, _ = O.fwd(x, "float32", w, "float32", b, initial_states=init, silu=True)
    edx, edw, edb, edi = O.bwd(x, "float32", w, "float32", dout, b, initial_states=init, silu=True)
    res = [np.load(os.path.join(str(tmp_path), f"rank{r}.npz")) for r in range(world)]
    np.testing.assert_allclose(np.concatenate([r["out"] for r in res], axis=2), eo, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(np.concatenate([r["dx"] for r in res], axis=2), edx, rtol=1e-5, atol=1e-5)
    for r in res:  # parameter gradients are complete on every rank
        np.testing.assert_allclose(r["dw"], edw, rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(r["db"], edb, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(res[0]["di"], edi, rtol=1e-5, atol=1e-5)  # rank 0 owns initial_states
    if deterministic:
        for r in res[1:]:
            assert np.array_equal(r["dw"], res[0]["dw"]) and np.array_equal(r["db"], res[0]["db"])


def test_context_parallel_matches_whole_sequence(tmp_path):
    _run(tmp_path, deterministic=False)


def test_context_parallel_rank_ordered_reduction(tmp_path):
    _run(tmp_path, deterministic=True)
