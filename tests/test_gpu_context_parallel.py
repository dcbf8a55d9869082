"""Context-parallel causal_conv1d through the real kernels.

* one GPU, a one-rank group: bit-identical to causal_conv1d_fn;
* two GPUs (skipped with fewer), NCCL: the sequence split over two processes matches the
  oracle on the whole sequence.
The multi-rank exchange logic is also tested on CPU with 3 gloo ranks
(tests/test_context_parallel_gloo.py)."""

import datetime
import socket

import pytest
import torch
import torch.distributed as dist

from causal_conv1d import causal_conv1d_fn
from causal_conv1d.context_parallel import causal_conv1d_fn_context_parallel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def one_rank_group():
    if dist.is_initialized():
        yield
        return
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                            timeout=datetime.timedelta(seconds=30))
    yield
    dist.destroy_process_group()


def test_single_rank_matches_causal_conv1d_fn(one_rank_group):
    g = torch.Generator(device="cuda").manual_seed(8)
    x = torch.randn(2, 512, 256, generator=g, device="cuda").to(torch.bfloat16).transpose(1, 2)
    w = (torch.rand(256, 4, generator=g, device="cuda") - 0.5)
    b = torch.randn(256, generator=g, device="cuda") * 0.1
    init = torch.randn(2, 256, 3, generator=g, device="cuda").to(torch.bfloat16)
    dout = torch.randn(2, 512, 256, generator=g, device="cuda").to(torch.bfloat16).transpose(1, 2)
    grads = []
    for fn in (causal_conv1d_fn, causal_conv1d_fn_context_parallel):
        xr, wr, br, ir = (t.detach().clone().requires_grad_() for t in (x, w, b, init))
        out = fn(xr, wr, br, initial_states=ir, activation="silu")
        out.backward(dout)
        grads.append((out, xr.grad, wr.grad, br.grad, ir.grad))
    for a, c in zip(*grads):
        assert torch.equal(a, c)


# ------------------------------------------------------- two GPUs, NCCL, real kernels
CP_B, CP_D, CP_L, CP_W = 2, 264, 1000, 4
CP_SPLITS = (0, 389, 1000)  # uneven slices, one per GPU


def _cp_problem():
    gen = torch.Generator().manual_seed(44)
    x = torch.randn(CP_B, CP_D, CP_L, generator=gen).to(torch.bfloat16)
    w = torch.rand(CP_D, CP_W, generator=gen) - 0.5
    b = torch.randn(CP_D, generator=gen) * 0.1
    dout = torch.randn(CP_B, CP_D, CP_L, generator=gen).to(torch.bfloat16)
    init = torch.randn(CP_B, CP_D, CP_W - 1, generator=gen).to(torch.bfloat16)
    return x, w, b, dout, init


def _cp_worker(rank, world, port, result_dir, deterministic):
    import os

    import numpy as np

    from helpers import to_storage

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        x, w, b, dout, init = _cp_problem()
        lo, hi = CP_SPLITS[rank], CP_SPLITS[rank + 1]

        def cl(t):  # channel-last storage on this rank's GPU
            return t.transpose(1, 2).contiguous().to(dev).transpose(1, 2)

        xr = cl(x[:, :, lo:hi]).requires_grad_()
        wt = w.to(dev).requires_grad_()
        bt = b.to(dev).requires_grad_()
        it = init.to(dev).requires_grad_()
        out = causal_conv1d_fn_context_parallel(xr, wt, bt, initial_states=it, activation="silu",
                                                deterministic=deterministic)
        out.backward(cl(dout[:, :, lo:hi]))
        torch.cuda.synchronize()
        np.savez(os.path.join(result_dir, f"rank{rank}.npz"), out=to_storage(out), dx=to_storage(xr.grad),
                 dw=to_storage(wt.grad), db=to_storage(bt.grad),
                 di=to_storage(it.grad) if it.grad is not None else np.zeros(0, np.uint16))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("deterministic", [False, True])
def test_two_gpus_nccl_matches_whole_sequence_oracle(tmp_path, deterministic):
    """The sequence split over two GPUs (NCCL send/recv of the W-1 halo forward and of
    dinitial_states backward, NCCL reduction of dweight/dbias) against the oracle on the
    whole sequence: concatenated out and dx, dweight/dbias on every rank, rank 0's
    dinitial_states."""
    import numpy as np
    import torch.multiprocessing as mp

    from helpers import to_storage
    from oracle import numpy_oracle as O
    from tolerances import GRAD_PARAM, PARITY

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    world = len(CP_SPLITS) - 1
    mp.start_processes(_cp_worker, args=(world, port, str(tmp_path), deterministic), nprocs=world, join=True,
                       start_method="spawn")
    x, w, b, dout, init = _cp_problem()
    xs, gs, inits = to_storage(x), to_storage(dout), to_storage(init)
    eo, _ = O.fwd(xs, "bfloat16", w.numpy(), "float32", b.numpy(), initial_states=inits, silu=True)
    edx, edw, edb, edi = O.bwd(xs, "bfloat16", w.numpy(), "float32", gs, b.numpy(), initial_states=inits, silu=True)
    res = [np.load(str(tmp_path / f"rank{r}.npz")) for r in range(world)]
    bf = lambda a: O.to_f32(a, "bfloat16")  # noqa: E731
    rtol, atol = PARITY["bfloat16"]
    np.testing.assert_allclose(bf(np.concatenate([r["out"] for r in res], axis=2)), bf(eo), rtol=rtol, atol=atol)
    np.testing.assert_allclose(bf(np.concatenate([r["dx"] for r in res], axis=2)), bf(edx), rtol=rtol, atol=atol)
    for r in res:
        np.testing.assert_allclose(r["dw"], edw, *GRAD_PARAM["float32"])
        np.testing.assert_allclose(r["db"], edb, *GRAD_PARAM["float32"])
    np.testing.assert_allclose(bf(res[0]["di"]), bf(edi), rtol=rtol, atol=atol)
    if deterministic:
        for r in res[1:]:
            assert np.array_equal(r["dw"], res[0]["dw"]) and np.array_equal(r["db"], res[0]["db"])
