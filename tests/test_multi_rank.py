"""Multi-rank host logic under gloo, world size 2 (CPU only).

Each rank computes its kv-head shard of a decode batch with the oracle; gathering the
shards reproduces the unsharded result exactly.  Migration pairing and the request
assignment are checked the same way: each prefill rank "moves" its requests' blocks on
the host and the decode ranks' pools end up equal to a single-process move.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _decode_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    from gollek_b200.sharding import kv_head_shard, q_head_shard
    from oracle import oracle as O
    from tests.helpers import decode_case
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        qx, k, v, bt, ctx = decode_case([5, 70, 300], hq=16, hkv=4, d=32, bs=16, seed=3)
        lo, hi = kv_head_shard(4, world, rank)
        qlo, qhi = q_head_shard(16, 4, world, rank)
        part = O.a2_compute(qx[:, None, qlo:qhi], np.ascontiguousarray(k[:, lo:hi]),
                            np.ascontiguousarray(v[:, lo:hi]), bt, ctx, 0.2,
                            num_kv_heads=hi - lo, block_size=16)[:, 0]
        parts = [torch.zeros_like(torch.from_numpy(part)) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(part))
        if rank == 0:
            full = np.concatenate([p.numpy() for p in parts], axis=1)
            want = O.a2_compute(qx[:, None], k, v, bt, ctx, 0.2, num_kv_heads=4, block_size=16)[:, 0]
            q.put(bool(np.array_equal(full, want)))
    finally:
        dist.destroy_process_group()


def _migrate_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    from gollek_b200.sharding import assign_requests, migration_peer
    from oracle import oracle as O
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        L, bpb, nb = 3, 32, 24
        rng = np.random.default_rng(9)
        src_pool = rng.integers(0, 256, (nb * L * bpb,), dtype=np.uint8)
        req_blocks = [[0, 1, 2], [5, 6], [9], [12, 13, 14, 15]]
        dst_ids = [[20, 3, 7], [11, 4], [21], [8, 10, 16, 17]]
        owner = assign_requests(len(req_blocks), world)
        is_src, peer = migration_peer(world, rank)
        # prefill rank: copy its requests into a staging pool and send it to its decode peer
        if is_src:
            stage = np.zeros_like(src_pool)
            mine = [i for i in range(len(req_blocks)) if owner[i] == rank]
            for i in mine:
                O.migrate(src_pool, src_pool, stage, stage, req_blocks[i], dst_ids[i], L, bpb)
            dist.send(torch.from_numpy(stage), dst=peer)
        else:
            got = torch.zeros(src_pool.shape, dtype=torch.uint8)
            dist.recv(got, src=peer)
            want = np.zeros_like(src_pool)
            for i in range(len(req_blocks)):
                if owner[i] == peer:
                    O.migrate(src_pool, src_pool, want, want, req_blocks[i], dst_ids[i], L, bpb)
            q.put(bool(np.array_equal(got.numpy(), want)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("worker", [_decode_worker, _migrate_worker])
def test_two_rank(worker):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    mp.start_processes(worker, args=(2, port, q), nprocs=2, join=True, start_method="spawn")
    assert q.get() is True


def test_sharding_rules():
    from gollek_b200.sharding import assign_requests, kv_head_shard, migration_peer, q_head_shard
    assert [kv_head_shard(8, 4, r) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    assert q_head_shard(64, 8, 8, 3) == (24, 32)
    assert migration_peer(8, 1) == (True, 5) and migration_peer(8, 6) == (False, 2)
    assert assign_requests(5, 4) == [0, 1, 0, 1, 0]
    with pytest.raises(ValueError):
        kv_head_shard(8, 3, 0)
    with pytest.raises(ValueError):
        migration_peer(3, 0)
