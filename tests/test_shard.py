"""Batch sharding (trispconv_b200.shard): range arithmetic, and the
shard -> per-rank work -> gather round trip on two gloo ranks (CPU)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from trispconv_b200.shard import batch_range, gather_sparse, shard


@pytest.mark.parametrize("batch,world", [(4, 1), (4, 2), (5, 2), (3, 4), (16, 8), (7, 3)])
def test_batch_ranges_partition_the_batch(batch, world):
    ranges = [batch_range(batch, r, world) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == batch
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0
    sizes = [b1 - b0 for b0, b1 in ranges]
    assert max(sizes) - min(sizes) <= 1 and min(sizes) >= 0


def test_batch_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        batch_range(4, 2, 2)


def _batch_major(rng, batch, per):
    rows = []
    for b in range(batch):
        n = int(per[b])
        zyx = rng.integers(0, 50, (n, 3))
        rows.append(np.concatenate([np.full((n, 1), b), zyx], 1))
    idx = np.concatenate(rows).astype(np.int32)
    feats = rng.standard_normal((len(idx), 6)).astype(np.float32)
    return torch.from_numpy(idx), torch.from_numpy(feats)


def test_shard_keeps_global_batch_ids_and_order():
    rng = np.random.default_rng(0)
    idx, f = _batch_major(rng, 5, [3, 0, 7, 2, 4])
    parts = [shard(idx, f, 5, r, 2) for r in range(2)]
    assert torch.equal(torch.cat([p[0] for p in parts]), idx)
    assert torch.equal(torch.cat([p[1] for p in parts]), f)
    assert set(parts[0][0][:, 0].tolist()) <= {0, 1, 2}
    assert set(parts[1][0][:, 0].tolist()) <= {3, 4}


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, batch, per, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(1)
        idx, f = _batch_major(rng, batch, per)
        li, lf = shard(idx, f, batch, rank, world)
        lf = lf * 2.0 + li[:, :1].float()  # per-row work on the rank's samples
        gi, gf = gather_sparse(li, lf)
        q.put((rank, gi.numpy(), gf.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("batch,per", [(4, [5, 9, 0, 3]), (3, [4, 4, 4])])
def test_shard_gather_round_trip_two_gloo_ranks(batch, per):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, batch, per, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rng = np.random.default_rng(1)
    idx, f = _batch_major(rng, batch, per)
    want_f = (f * 2.0 + idx[:, :1].float()).numpy()
    for _, gi, gf in results:
        np.testing.assert_array_equal(gi, idx.numpy())
        np.testing.assert_array_equal(gf, want_f)


def _failing_worker(rank, world, port, q):
    """Rank 1 dies between steps, before the output gather; rank 0 must get an
    error from its next collective (short process-group timeout), not hang."""
    from datetime import timedelta

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        q.put((rank, "left"))
        q.close()
        q.join_thread()  # flush the message before the hard exit
        os._exit(3)
    try:
        gather_sparse(torch.zeros((2, 4), dtype=torch.int32), torch.zeros((2, 3)))
        q.put((rank, "returned"))
    except Exception as e:  # the failure the test expects
        q.put((rank, "raised " + type(e).__name__))


def test_gather_raises_when_a_rank_has_left():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert results[1] == "left" and procs[1].exitcode == 3
    assert results[0].startswith("raised"), results[0]
    assert procs[0].exitcode == 0
