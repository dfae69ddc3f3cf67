"""N-sharding host logic: contiguous split, gloo world_size-2 gather, host-side peer failure detection."""
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp
import torch.nn.functional as F

from sparseflow_b200.Utils.shard import PeerFailure, PeerMonitor, gather_shards, shard_batch, shard_range


@pytest.mark.parametrize("n,world", [(64, 1), (64, 8), (65, 8), (3, 8), (0, 2), (1024, 3)])
def test_shard_range_partitions_contiguously(n, world):
    ranges = [shard_range(n, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (s0, e0), (s1, e1) in zip(ranges, ranges[1:]):
        assert e0 == s1
    sizes = [e - s for s, e in ranges]
    assert max(sizes) - min(sizes) <= 1 and sum(sizes) == n


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)
    with pytest.raises(ValueError):
        shard_range(8, 0, 0)


def test_shard_batch_5d_splits_n_and_keeps_t():
    x = torch.arange(4 * 10 * 2).reshape(4, 10, 2, 1, 1).float()
    parts = [shard_batch(x, 3, r) for r in range(3)]
    assert [p.shape[1] for p in parts] == [4, 3, 3]
    assert all(p.shape[0] == 4 for p in parts)
    assert torch.equal(torch.cat(parts, 1), x)
    x4 = x[0]
    assert torch.equal(torch.cat([shard_batch(x4, 4, r) for r in range(4)], 0), x4)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker_gather(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(7)
        x = (torch.rand(4, 5, 8, 9, 9, generator=g) < 0.05).float()  # T=4, N=5 (uneven over 2 ranks)
        w = torch.randn(6, 8, 3, 3, generator=g)
        local = shard_batch(x, world, rank)
        t, n = local.shape[:2]
        y = F.conv2d(local.reshape(t * n, 8, 9, 9), w, padding=1).reshape(t, n, 6, 9, 9)
        full = gather_shards(y, x.shape[1])
        ref = F.conv2d(x.reshape(20, 8, 9, 9), w, padding=1).reshape(4, 5, 6, 9, 9)
        q.put((rank, bool(torch.allclose(full, ref, atol=1e-5)), tuple(local.shape)))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_shard_and_gather():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_gather, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [r[1] for r in res] == [True, True]
    assert res[0][2] == (4, 3, 8, 9, 9) and res[1][2] == (4, 2, 8, 9, 9)


def _worker_heartbeat(rank, world, port, dead_rank, steps, q):
    store = torch.distributed.TCPStore("127.0.0.1", port, world, rank == 0, timeout=__import__("datetime").timedelta(seconds=30))
    mon = PeerMonitor(store, rank, world, timeout_s=1.0)
    done = 0
    try:
        for step in range(steps):
            if rank == dead_rank and step == 2:
                q.put((rank, "exited", step))
                return  # leaves between steps, nothing in flight
            mon.beat(step)
            mon.wait_peers(step)
            done = step + 1
        q.put((rank, "ok", done))
    except PeerFailure as e:
        q.put((rank, "peer_failure", e.ranks, e.step))
    finally:
        if rank == 0:
            time.sleep(0.5)  # keep the store server up until the peer has read its keys


def test_gloo_peer_failure_detected_between_steps():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_heartbeat, args=(r, 2, port, 1, 5, q)) for r in range(2)]
    t0 = time.monotonic()
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        item = q.get(timeout=120)
        res[item[0]] = item[1:]
    for p in procs:
        p.join(timeout=60)
    assert res[1] == ("exited", 2)
    assert res[0] == ("peer_failure", [1], 2)
    assert time.monotonic() - t0 < 60


def test_peer_monitor_all_alive():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_heartbeat, args=(r, 2, port, -1, 4, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        item = q.get(timeout=120)
        res[item[0]] = item[1:]
    for p in procs:
        p.join(timeout=60)
    assert res == {0: ("ok", 4), 1: ("ok", 4)}
