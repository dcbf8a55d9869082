"""Multi-rank host logic on CPU (gloo, world size 2).

The batch-sharded backward leaves each rank a partial dweight/dbias; one all-reduce of
the flat GradBucket completes them.  Here each rank's local kernel is stood in for by
the CPU oracle (the GPU kernel's parity is covered by the -m gpu suite), and the
all-reduced result must equal the full-batch oracle.  A rank that leaves before the
collective must make the other rank fail with an error within the group timeout, not
hang.
"""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from causal_conv1d.distributed import GradBucket, allreduce_param_grads, shard_range
from oracle import numpy_oracle as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    rng = np.random.default_rng(7)
    b, d, l, w = 5, 24, 40, 4
    x = rng.standard_normal((b, d, l), dtype=np.float32)
    weight = rng.uniform(-0.5, 0.5, (d, w)).astype(np.float32)
    bias = (0.1 * rng.standard_normal(d)).astype(np.float32)
    dout = rng.standard_normal((b, d, l), dtype=np.float32)
    return x, weight, bias, dout


def _sharded_worker(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        x, weight, bias, dout = _inputs()
        start, stop = shard_range(x.shape[0], world, rank)
        _, dw, db, _ = O.bwd(x[start:stop], "float32", weight, "float32", dout[start:stop], bias, silu=True)
        bucket = GradBucket(weight.shape[0], weight.shape[1], True, "cpu")
        bucket.dweight.copy_(torch.from_numpy(dw))
        bucket.dbias.copy_(torch.from_numpy(db))
        allreduce_param_grads(bucket)
        np.save(os.path.join(result_dir, f"rank{rank}.npy"), bucket.flat.numpy())
    finally:
        dist.destroy_process_group()


def _deterministic_worker(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        bucket = GradBucket(8, 4, True, "cpu")
        bucket.flat.copy_(torch.from_numpy(_rank_partials(world)[rank]))
        allreduce_param_grads(bucket, deterministic=True)
        np.save(os.path.join(result_dir, f"rank{rank}.npy"), bucket.flat.numpy())
    finally:
        dist.destroy_process_group()


def _rank_partials(world):
    # magnitudes far apart, so that fp32 sums depend on their order
    rng = np.random.default_rng(11)
    n = 8 * 4 + 8
    return [(rng.standard_normal(n) * 10.0 ** (3 * (r % 3))).astype(np.float32) for r in range(world)]


def test_deterministic_reduction_is_rank_ordered(tmp_path):
    world = 3
    mp.spawn(_deterministic_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    parts = _rank_partials(world)
    expected = parts[0].copy()
    for r in range(1, world):
        expected = (expected + parts[r]).astype(np.float32)
    for r in range(world):
        got = np.load(os.path.join(str(tmp_path), f"rank{r}.npy"))
        assert np.array_equal(got, expected), r


def test_batch_sharded_backward_allreduce(tmp_path):
    world = 2
    mp.spawn(_sharded_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    x, weight, bias, dout = _inputs()
    _, dw, db, _ = O.bwd(x, "float32", weight, "float32", dout, bias, silu=True)
    expected = np.concatenate([dw.reshape(-1), db])
    for r in range(world):
        got = np.load(tmp_path / f"rank{r}.npy")
        np.testing.assert_allclose(got, expected, rtol=1e-5, atol=1e-5)
    # both ranks hold the identical sum
    assert np.array_equal(np.load(tmp_path / "rank0.npy"), np.load(tmp_path / "rank1.npy"))


def _leaving_worker(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        return  # leaves between steps without joining the collective
    bucket = GradBucket(8, 4, True, "cpu")
    bucket.flat.fill_(1.0)
    outcome = "completed"
    try:
        allreduce_param_grads(bucket)
    except Exception as exc:  # noqa: BLE001 - any error is the expected outcome
        outcome = f"error: {type(exc).__name__}"
    with open(os.path.join(result_dir, "outcome.txt"), "w") as f:
        f.write(outcome)


def test_missing_rank_fails_with_timeout(tmp_path):
    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung instead of failing")
    outcome = (tmp_path / "outcome.txt").read_text()
    assert outcome.startswith("error"), outcome


@pytest.mark.parametrize("n,world,multiple", [(4, 2, 1), (5, 2, 1), (16384, 8, 8), (4100, 3, 8), (3, 4, 1)])
def test_shard_range_partitions(n, world, multiple):
    spans = [shard_range(n, world, r, multiple) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0
    for s0, s1 in spans:
        assert s0 % multiple == 0 and s0 <= s1
    sizes = [s1 - s0 for s0, s1 in spans]
    assert max(sizes) - min(sizes) <= multiple
    with pytest.raises(ValueError):
        shard_range(n, world, world)
