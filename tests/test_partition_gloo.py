"""Multi-process host logic of the partitioner on CPU (gloo, world size 2).

Each rank computes its row block of C with the oracle (the per-rank compute
is checked on the GPU elsewhere); this test covers the shard plan and the
all-gather that replicates C, including unequal shards."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, m, n, k, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        import oracle
        from sptiles_b200.partition import gather_row_shards, matmul_row_shard, vector_add_shard

        rng = np.random.default_rng(123)
        a = rng.standard_normal((m, k)).astype(np.float32)
        b = rng.standard_normal((k, n)).astype(np.float32)
        r0, r1 = matmul_row_shard(m, world, rank)
        c_local = torch.from_numpy(oracle.matmul(a, b, rows=(r0, r1), threads=1))
        full = gather_row_shards(c_local, m)
        want = oracle.matmul(a, b, threads=1)
        ok_mm = full.numpy().tobytes() == want.tobytes()
        e0, e1 = vector_add_shard(1000, world, rank)
        sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(sizes, torch.tensor([e1 - e0]))
        ok_va = sum(int(s) for s in sizes) == 1000 and e0 % 4 == 0
        q.put((rank, ok_mm, ok_va))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("m", [256, 300])  # equal shards, and unequal shards (128 + 172 rows)
def test_row_shards_all_gather_to_full_matrix(m):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, m, 40, 24, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok_mm, ok_va in results:
        assert ok_mm, f"rank {rank}: gathered C differs from the oracle"
        assert ok_va, f"rank {rank}: vector_add shards do not cover the range"
