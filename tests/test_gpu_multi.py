"""Multi-GPU partitioner on real GPUs: one process per GPU over NCCL.

Each rank computes its M-row block of C with the tensor-core kernels and the
row blocks are all-gathered into a replicated C; vector_add shards by element
range.  Runs one rank per visible GPU (up to 8); needs two (skipped
otherwise)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

needs_two = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        import oracle
        from sptiles_b200.partition import matmul_row_shard, sharded_matmul, sharded_vector_add, vector_add_shard

        dev = torch.device("cuda", rank)
        out = {}
        # known-answer matmul, unequal shards (3000 rows -> 1536 + 1464)
        m, n, k = 3000, 1024, 2048
        a = oracle.kat_values(m * k, 17, 8, 0.25).reshape(m, k)
        b = oracle.kat_values(k * n, 13, 6, 0.5).reshape(k, n)
        r0, r1 = matmul_row_shard(m, world, rank)
        A = torch.from_numpy(a[r0:r1]).to(dev, torch.bfloat16)
        B = torch.from_numpy(b).to(dev, torch.bfloat16)
        C = sharded_matmul(A, B, m_total=m, out_dtype=torch.float32, replicate_output=True)
        out["matmul"] = C.cpu().numpy().tobytes() == oracle.matmul_kat_expected(m, n, k).tobytes()
        local = sharded_matmul(A, B, m_total=m, out_dtype=torch.float32)
        out["local_rows"] = local.shape[0] == r1 - r0
        # vector_add by element range
        total = 1_000_003
        x = np.random.default_rng(5).uniform(-1, 1, total).astype(np.float32)
        y = np.random.default_rng(6).uniform(-1, 1, total).astype(np.float32)
        e0, e1 = vector_add_shard(total, world, rank)
        Z = sharded_vector_add(torch.from_numpy(x[e0:e1]).to(dev), torch.from_numpy(y[e0:e1]).to(dev))
        out["vector_add"] = Z.cpu().numpy().tobytes() == (x[e0:e1] + y[e0:e1]).tobytes()
        # the all-gather fused into the GEMM epilogue (peer stores over NVLink)
        from sptiles_b200.partition import ReplicatedOutput

        rep = ReplicatedOutput(m, n, torch.float32)
        Cf = rep.matmul(A, B)
        out["fused_kat"] = Cf.cpu().numpy().tobytes() == oracle.matmul_kat_expected(m, n, k).tobytes()
        rep.close()
        m2 = 2048  # equal shards, bf16 out with a bias, random inputs
        g = torch.Generator(device="cpu").manual_seed(77)
        A2 = (torch.randn((m2, 1024), generator=g) * 0.1).to(torch.bfloat16)
        B2 = (torch.randn((1024, 768), generator=g) * 0.1).to(torch.bfloat16)
        bias2 = torch.randn(768, generator=g)
        s0, s1 = matmul_row_shard(m2, world, rank)
        rep2 = ReplicatedOutput(m2, 768, torch.bfloat16)
        C2 = rep2.matmul(A2[s0:s1].to(dev), B2.to(dev), bias2.to(dev))
        want = sharded_matmul(A2[s0:s1].to(dev), B2.to(dev), bias2.to(dev), m_total=m2, out_dtype=torch.bfloat16,
                              replicate_output=True)
        out["fused_vs_nccl"] = torch.equal(C2, want)
        rep2.close()
        # fp32 operands (packed 3xTF32; a few tiles per rank, so the stream-K
        # split with peer copies) and a 16-bit replicated C
        m4, n4, k4 = 1000, 520, 700
        a4 = oracle.kat_values(m4 * k4, 17, 8, 0.25).reshape(m4, k4)
        b4 = oracle.kat_values(k4 * n4, 13, 6, 0.5).reshape(k4, n4)
        u0, u1 = matmul_row_shard(m4, world, rank)
        rep4 = ReplicatedOutput(m4, n4, torch.float32)
        C4 = rep4.matmul(torch.from_numpy(a4[u0:u1]).to(dev), torch.from_numpy(b4).to(dev))
        out["fused_fp32_kat"] = C4.cpu().numpy().tobytes() == oracle.matmul_kat_expected(m4, n4, k4).tobytes()
        rep4.close()
        rep5 = ReplicatedOutput(m2, 768, torch.float16)
        C5 = rep5.matmul(A2[s0:s1].to(dev).half(), B2.to(dev).half(), bias2.to(dev))
        want5 = sharded_matmul(A2[s0:s1].to(dev).half(), B2.to(dev).half(), bias2.to(dev), m_total=m2,
                               out_dtype=torch.float16, replicate_output=True)
        out["fused_f16_out"] = torch.equal(C5, want5)
        rep5.close()
        # host operands: 1/N of B's rows per rank, all-gathered on the GPUs
        from sptiles_b200.partition import sharded_matmul_host

        hA = torch.from_numpy(a[r0:r1]).to(torch.bfloat16).pin_memory()
        hB = torch.from_numpy(b).to(torch.bfloat16).pin_memory()
        Ch = sharded_matmul_host(hA, hB, m_total=m, out_dtype=torch.float32)
        out["host_kat"] = Ch.numpy().tobytes() == oracle.matmul_kat_expected(m, n, k)[r0:r1].tobytes()
        m3, n3, k3 = 1100, 200, 1001  # B's rows split unevenly (the last slice short and zero padded)
        a3 = oracle.kat_values(m3 * k3, 17, 8, 0.25).reshape(m3, k3)
        b3 = oracle.kat_values(k3 * n3, 13, 6, 0.5).reshape(k3, n3)
        t0, t1 = matmul_row_shard(m3, world, rank)
        C3 = sharded_matmul_host(torch.from_numpy(a3[t0:t1]).half().pin_memory(), torch.from_numpy(b3).half(),
                                 m_total=m3, out_dtype=torch.float32)
        out["host_kat_odd_k"] = C3.numpy().tobytes() == oracle.matmul_kat_expected(m3, n3, k3)[t0:t1].tobytes()
        # fewer 128-row blocks than some ranks' share: empty shards (300 rows
        # over 4 or 8 ranks leave ranks without rows)
        m6, n6, k6 = 300, 256, 256
        a6 = oracle.kat_values(m6 * k6, 17, 8, 0.25).reshape(m6, k6)
        b6 = oracle.kat_values(k6 * n6, 13, 6, 0.5).reshape(k6, n6)
        v0, v1 = matmul_row_shard(m6, world, rank)
        C6 = sharded_matmul(torch.from_numpy(a6[v0:v1]).to(dev, torch.float16), torch.from_numpy(b6).to(dev,
                            torch.float16), m_total=m6, out_dtype=torch.float32, replicate_output=True)
        out["empty_shards_kat"] = C6.cpu().numpy().tobytes() == oracle.matmul_kat_expected(m6, n6, k6).tobytes()
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


@needs_two
def test_row_sharded_matmul_and_allgather_on_every_gpu():
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, out in results.items():
        assert all(out.values()), f"rank {rank}: {out}"
