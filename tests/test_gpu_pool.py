"""LpPool's row-sharded forms on several GPUs (one process per GPU, NCCL).

Skipped unless at least two GPUs are visible; runs one rank per visible GPU
(up to 8).  Every rank computes the whole result on its own GPU with the
ordinary entry points, then the pooled forms -- ``Pool`` (torch.distributed
gather) and ``NcclPool`` (the C-ABI pool: NVLink peer stores from the GEMV,
or an NCCL group) -- and the two must agree bit for bit: sharded == serial
(test_parallel.nim), with an uneven row count so the last rank takes the
remainder, and the reference test's own cases (300 / 64 / 1 rows, so some
ranks hold no rows at all) for every pooled GEMV form.
"""
import contextlib
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available() or torch.cuda.device_count() < 2:  # pragma: no cover
    pytest.skip("needs two or more GPUs", allow_module_level=True)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    bad = []
    try:
        import nim_lowprec_b200 as L
        from nim_lowprec_b200 import parallel as P
        g = torch.Generator(device="cuda").manual_seed(11)
        M, K, n = 1001, 512, 8

        def rnd(k, scale=1.0):
            return torch.randn(k, device="cuda", generator=g) * scale

        w = rnd(M * K, 0.02)
        x = rnd(K * n)
        wq = torch.empty(M * K, dtype=torch.int8, device="cuda")
        wd = torch.empty(M * K // 32, device="cuda")
        L.quantizeQ8_0Split(w, wq, wd)
        xq = torch.empty(K * n, dtype=torch.int8, device="cuda")
        xd = torch.empty(K * n // 32, device="cuda")
        L.quantizeQ8_0Split(x, xq, xd)
        blk = torch.empty(M * K // 32 * 18, dtype=torch.uint8, device="cuda")
        L.quantizeQ4_0Batch(w, blk)
        pools = [P.Pool(), P.NcclPool()]

        def same(tag, a, b):
            torch.cuda.synchronize()
            if not torch.equal(a.view(torch.int32), b.view(torch.int32)):
                bad.append(tag)

        ref = torch.empty(M, device="cuda")
        L.dequantGemvQ8(wq, wd, 32, xq[:K], xd[:K // 32], ref)
        for i, pool in enumerate(pools):
            y = torch.full((M,), float("nan"), device="cuda")
            P.parDequantGemvQ8(pool, wq, wd, 32, xq[:K], xd[:K // 32], y)
            same(f"q8/{i}", y, ref)
            # weights already sharded: only this rank's rows are passed
            y2 = torch.full((M,), float("nan"), device="cuda")
            P.parDequantGemvQ8(pool, pool.slice(wq, M).clone(), pool.slice(wd, M).clone(), 32,
                               xq[:K], xd[:K // 32], y2, sharded=True)
            same(f"q8-sharded/{i}", y2, ref)
        for mode in ("fast", "exact"):
            with L.fp32_mode(mode):
                ref = torch.empty(M, device="cuda")
                L.dequantGemvQ4_0(blk, K // 32, x[:K], ref)
                for i, pool in enumerate(pools):
                    y = torch.full((M,), float("nan"), device="cuda")
                    P.parDequantGemvQ4_0(pool, blk, K // 32, x[:K], y)
                    same(f"q4_0-{mode}/{i}", y, ref)
        ref = torch.empty(M * n, device="cuda")
        L.dequantGemmQ8(wq, wd, 32, xq, xd, n, ref)
        for i, pool in enumerate(pools):
            y = torch.full((M * n,), float("nan"), device="cuda")
            P.parDequantGemmQ8(pool, wq, wd, 32, xq, xd, n, y)
            same(f"gemm/{i}", y, ref)
        # test_parallel.nim:48-100 cases through the library pool: 300 / 64 / 1
        # rows over every rank (with 1 row all but the last rank hold none)
        import refcases as R
        xp = torch.from_numpy(R.par_x()).cuda()
        npl = pools[1]
        for Mp in R.PAR_ROWS:
            wq8, sc8 = (torch.from_numpy(a).cuda() for a in R.par_int8(Mp))
            w4, sc4 = (torch.from_numpy(a).cuda() for a in R.par_int4(Mp))
            wf4, scf = (torch.from_numpy(a).cuda() for a in R.par_f4(Mp))
            q80, bpr = R.par_q8_0(Mp)
            q40, _ = R.par_q4_0(Mp)
            q80 = torch.from_numpy(q80.reshape(-1)).cuda()
            q40 = torch.from_numpy(q40.reshape(-1)).cuda()
            cases = [
                ("int8", lambda y_: L.dequantGemv(wq8, sc8, R.PAR_GS, xp, y_),
                 lambda y_: P.parDequantGemv(npl, wq8, sc8, R.PAR_GS, xp, y_)),
                ("int4", lambda y_: L.dequantGemvI4(w4, sc4, R.PAR_GS, xp, y_),
                 lambda y_: P.parDequantGemvI4(npl, w4, sc4, R.PAR_GS, xp, y_)),
                ("f4", lambda y_: L.dequantGemvF4(wf4, scf, R.PAR_GS, xp, y_),
                 lambda y_: P.parDequantGemvF4(npl, wf4, scf, R.PAR_GS, xp, y_)),
                ("q8_0", lambda y_: L.dequantGemvQ8_0(q80, bpr, xp, y_),
                 lambda y_: P.parDequantGemvQ8_0(npl, q80, bpr, xp, y_)),
                ("q4_0", lambda y_: L.dequantGemvQ4_0(q40, bpr, xp, y_),
                 lambda y_: P.parDequantGemvQ4_0(npl, q40, bpr, xp, y_)),
            ]
            for mode in ("exact", "fast"):
                with L.fp32_mode(mode):
                    for tag, ser, par in cases:
                        ref_ = torch.full((Mp,), float("nan"), device="cuda")
                        ser(ref_)
                        y_ = torch.full((Mp,), float("nan"), device="cuda")
                        par(y_)
                        same(f"par-{tag}-{mode}-M{Mp}", y_, ref_)
            pwq, pw4, pws, pxq, pxs = (torch.from_numpy(a).cuda() for a in R.pooled_case(Mp))
            for tag, ser, par, w_ in (("q8", L.dequantGemvQ8, P.parDequantGemvQ8, pwq),
                                      ("i4q8", L.dequantGemvI4Q8, P.parDequantGemvI4Q8, pw4)):
                ref_ = torch.full((Mp,), float("nan"), device="cuda")
                ser(w_, pws, R.PAR_GS, pxq, pxs, ref_)
                y_ = torch.full((Mp,), float("nan"), device="cuda")
                par(npl, w_, pws, R.PAR_GS, pxq, pxs, y_)
                same(f"pooled-{tag}-M{Mp}", y_, ref_)
        # a gather group: two pooled GEMVs (pushing) and a wide pooled GEMM
        # (tensor-core path, which does not push) as parts of one vector,
        # received once -- the single-GPU bits, twice in a row
        npl = pools[1]
        if npl.p2p:
            ng = 24
            refq8 = torch.empty(M, device="cuda")
            L.dequantGemvQ8(wq, wd, 32, xq[:K], xd[:K // 32], refq8)
            refq4 = torch.empty(M, device="cuda")
            L.dequantGemvQ4_0(blk, K // 32, x[:K], refq4)
            xqg = torch.empty(K * ng, dtype=torch.int8, device="cuda")
            xdg = torch.empty(K * ng // 32, device="cuda")
            L.quantizeQ8_0Split(rnd(K * ng), xqg, xdg)
            refgm = torch.empty(M * ng, device="cuda")
            L.dequantGemmQ8(wq, wd, 32, xqg, xdg, ng, refgm)
            for rep_ in range(2):
                yg = torch.full((2 * M + M * ng,), float("nan"), device="cuda")
                npl.group_begin(yg)
                P.parDequantGemvQ8(npl, wq, wd, 32, xq[:K], xd[:K // 32], yg[:M])
                P.parDequantGemvQ4_0(npl, blk, K // 32, x[:K], yg[M:2 * M])
                P.parDequantGemmQ8(npl, wq, wd, 32, xqg, xdg, ng, yg[2 * M:])
                npl.group_end()
                same(f"group{rep_}-q8", yg[:M], refq8)
                same(f"group{rep_}-q4_0", yg[M:2 * M], refq4)
                same(f"group{rep_}-gemm", yg[2 * M:], refgm)
            # pooled GEMVs queued in batches inside one gather group (the
            # decode-sweep form): the batch kernels push every call's rows
            # from their folds, a format change starts a second batch launch,
            # and the group's receive runs once
            jobs = []
            for mj, kj in ((M, K), (300, 1024), (7, 64), (M, K), (1, 32)):
                wj = rnd(mj * kj, 0.02)
                sj = torch.empty(mj * kj // 32, device="cuda")
                L.calibrateSymmetric(wj, 32, 7.0, sj)
                pj = torch.empty(mj * kj // 2, dtype=torch.uint8, device="cuda")
                L.quantizeI4Packed(wj, sj, 32, pj)
                xqj = torch.empty(kj, dtype=torch.int8, device="cuda")
                xsj = torch.empty(kj // 32, device="cuda")
                L.quantizeQ8_0Split(rnd(kj), xqj, xsj)
                rj = torch.empty(mj, device="cuda")
                L.dequantGemvI4Q8(pj, sj, 32, xqj, xsj, rj)
                jobs.append((mj, pj, sj, xqj, xsj, rj))
            tot = sum(j[0] for j in jobs) + M
            for rep_ in range(2):
                yb = torch.full((tot,), float("nan"), device="cuda")
                with L.batch():
                    npl.group_begin(yb)
                    off = 0
                    for mj, pj, sj, xqj, xsj, _ in jobs:
                        P.parDequantGemvI4Q8(npl, pj, sj, 32, xqj, xsj, yb[off:off + mj])
                        off += mj
                    P.parDequantGemvQ8(npl, wq, wd, 32, xq[:K], xd[:K // 32], yb[off:])
                    npl.group_end()
                off = 0
                for i_, (mj, *_r, rj) in enumerate(jobs):
                    same(f"batch-group{rep_}-{i_}", yb[off:off + mj], rj)
                    off += mj
                same(f"batch-group{rep_}-q8", yb[off:], refq8)
            # a group of >= 2^18 floats takes the pull form of the exchange
            # (outputs published in their owner's buffer, read by the others),
            # batched and as lone calls, with a part whose kernel does not
            # publish (the tensor-core GEMM) sent by the receive kernel
            big = []
            for mj in (130_003, 120_000, 64):
                wj = rnd(mj * 64, 0.02)
                sj = torch.empty(mj * 2, device="cuda")
                L.calibrateSymmetric(wj, 32, 7.0, sj)
                pj = torch.empty(mj * 32, dtype=torch.uint8, device="cuda")
                L.quantizeI4Packed(wj, sj, 32, pj)
                rj = torch.empty(mj, device="cuda")
                L.dequantGemvI4Q8(pj, sj, 32, xq[:64], xd[:2], rj)
                big.append((mj, pj, sj, rj))
            totb = sum(b_[0] for b_ in big) + M * ng
            assert totb >= 1 << 18
            for batched in (True, False):
                yb = torch.full((totb,), float("nan"), device="cuda")
                ctx = L.batch() if batched else contextlib.nullcontext()
                with ctx:
                    npl.group_begin(yb)
                    off = 0
                    for mj, pj, sj, _ in big:
                        P.parDequantGemvI4Q8(npl, pj, sj, 32, xq[:64], xd[:2], yb[off:off + mj])
                        off += mj
                    P.parDequantGemmQ8(npl, wq, wd, 32, xqg, xdg, ng, yb[off:])
                    npl.group_end()
                off = 0
                for i_, (mj, _p, _s, rj) in enumerate(big):
                    same(f"pull-group-b{int(batched)}-{i_}", yb[off:off + mj], rj)
                    off += mj
                same(f"pull-group-b{int(batched)}-gemm", yb[off:], refgm)
            # a pull-form group whose every part is published by a queued
            # GEMV's fold: the receive rides in the last batch launch (one
            # receive warp per CTA reads the other ranks' rows while the
            # GEMVs run), the parts in two formats (two batch launches, the
            # receive in whichever comes last), three times in a row with a
            # lone pooled call (its own gather) in between
            with L.fp32_mode("exact"):
                refq4x = torch.empty(M, device="cuda")
                L.dequantGemvQ4_0(blk, K // 32, x[:K], refq4x)
                nq4 = 13
                totf = sum(b_[0] for b_ in big) + nq4 * M
                assert totf >= 1 << 18
                for rep_ in range(3):
                    yf = torch.full((totf,), float("nan"), device="cuda")
                    q4_first = rep_ == 1
                    with L.batch():
                        npl.group_begin(yf)
                        off = 0
                        spans = []
                        order = ["q4", "i4"] if q4_first else ["i4", "q4"]
                        for kind in order:
                            if kind == "i4":
                                for mj, pj, sj, rj in big:
                                    P.parDequantGemvI4Q8(npl, pj, sj, 32, xq[:64], xd[:2],
                                                         yf[off:off + mj])
                                    spans.append((off, mj, rj))
                                    off += mj
                            else:
                                for _ in range(nq4):
                                    P.parDequantGemvQ4_0(npl, blk, K // 32, x[:K], yf[off:off + M])
                                    spans.append((off, M, refq4x))
                                    off += M
                        npl.group_end()
                    for i_, (o_, mj, rj) in enumerate(spans):
                        same(f"fused-recv{rep_}-{i_}", yf[o_:o_ + mj], rj)
                    y1 = torch.full((M,), float("nan"), device="cuda")
                    P.parDequantGemvQ8(npl, wq, wd, 32, xq[:K], xd[:K // 32], y1)
                    same(f"fused-recv{rep_}-lone", y1, refq8)
        # the library pool gathers over NVLink by default (one GPU per rank);
        # both transports, back-to-back gathers (alternating exchange halves)
        # and CUDA-graph replays give the single-GPU bits
        npool = pools[1]
        if not npool.p2p:
            bad.append("p2p exchange not enabled")
        refs = []
        for j in range(n):
            r_ = torch.empty(M, device="cuda")
            L.dequantGemvQ8(wq, wd, 32, xq[j * K:(j + 1) * K], xd[j * K // 32:(j + 1) * K // 32], r_)
            refs.append(r_)
        for mode in (True, False, True):
            npool.p2p = mode
            for j in range(n):
                y = torch.full((M,), float("nan"), device="cuda")
                P.parDequantGemvQ8(npool, wq, wd, 32, xq[j * K:(j + 1) * K],
                                   xd[j * K // 32:(j + 1) * K // 32], y)
                same(f"q8-col{j}-p2p{int(mode)}", y, refs[j])
        ys = [torch.full((M,), float("nan"), device="cuda") for _ in range(n)]
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for j in range(n):
                    P.parDequantGemvQ8(npool, wq, wd, 32, xq[j * K:(j + 1) * K],
                                       xd[j * K // 32:(j + 1) * K // 32], ys[j])
        torch.cuda.current_stream().wait_stream(s)
        for rep in range(3):
            for yy in ys:
                yy.fill_(float("nan"))
            g.replay()
            for j in range(n):
                same(f"graph{rep}-col{j}", ys[j], refs[j])
        del g
        pools[1].shutdown()
        from nim_lowprec_b200 import _native as N
        if N.device_error() != 0:
            bad.append("device_error")
    except Exception as e:  # report, do not hang the other rank
        bad.append(f"exception: {e!r}")
    finally:
        dist.barrier()
        dist.destroy_process_group()
    q.put((rank, bad))


def test_pooled_forms_equal_single_gpu_bits():
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    assert all(not results[r] for r in range(world)), results
