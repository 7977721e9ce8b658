"""LpPool's row-sharded forms without a GPU: the slicing rule and the
gather, with two gloo ranks on CPU.

Each rank computes its row slice with the CPU oracle (the checker stands in
for the kernel here) and ``Pool.gather`` assembles y over torch.distributed;
the result must equal the serial oracle bit for bit (test_parallel.nim's
sharded == serial), including an uneven last slice and the GEMM's per-row
columns.
"""
import os
import socket

import numpy as np
import pytest

from gpu_util import F, acts, weights
from oracle import oracle as O

torch = pytest.importorskip("torch")

from nim_lowprec_b200 import parallel as P  # noqa: E402


@pytest.mark.parametrize("m,nranks", [(0, 1), (1, 1), (7, 3), (10, 3), (64, 8), (11008, 8),
                                      (14336, 7), (5, 8)])
def test_shard_rows_follow_the_reference(m, nranks):
    covered = []
    for r in range(nranks):
        b, e = P.shardRows(m, nranks, r)
        assert (b, e - b) == O.shard(m, nranks, r)
        covered.extend(range(b, e))
    assert covered == list(range(m))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, M, K, n, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pool = P.Pool()
        w = weights(5, M * K)
        x = acts(5, K * n)
        wq, wd = O.quantizeQ8_0Split(w)
        xq, xd = O.quantizeQ8_0Split(x)
        out = {}
        # GEMV: local slice by the oracle, gather by the pool
        y = torch.zeros(M)
        b, e = pool.rows(M)
        gpr = K // 32
        def local_gemv(ys):
            ys.copy_(torch.from_numpy(O.dequantGemvQ8(wq[b * K:e * K], wd[b * gpr:e * gpr], 32,
                                                      xq[:K], xd[:gpr])))
        pool.run(local_gemv, y, M)
        out["gemv"] = y.numpy().copy()
        # GEMM: n columns per row
        Y = torch.zeros(M * n)
        def local_gemm(ys):
            ys.copy_(torch.from_numpy(O.dequantGemmQ8(wq[b * K:e * K], wd[b * gpr:e * gpr], 32,
                                                      xq, xd, n)))
        pool.run(local_gemm, Y, M, per_row=n)
        out["gemm"] = Y.numpy().copy()
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,M", [(2, 37), (2, 128), (3, 100)])
def test_pool_gather_equals_serial_on_gloo(world, M):
    import torch.multiprocessing as mp
    K, n = 256, 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, M, K, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    w = weights(5, M * K)
    x = acts(5, K * n)
    wq, wd = O.quantizeQ8_0Split(w)
    xq, xd = O.quantizeQ8_0Split(x)
    want_gemv = O.dequantGemvQ8(wq, wd, 32, xq[:K], xd[:K // 32])
    want_gemm = O.dequantGemmQ8(wq, wd, 32, xq, xd, n)
    for r in range(world):
        assert np.array_equal(results[r]["gemv"].view(np.uint32), want_gemv.view(np.uint32))
        assert np.array_equal(results[r]["gemm"].view(np.uint32), want_gemm.view(np.uint32))
