#!/usr/bin/env python3
"""Benchmark of the fused dequant-GEMV hot path (BASELINE.json `metric`).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload (N = 1): BASELINE config 1 -- ggml Q4_0 fused dequant-GEMV
with fp32 activations, 11008 x 4096 (Llama-7B MLP up), synthetic seeded
N(0, 0.02) weights encoded on the GPU by the library's own Q4_0 encoder and
N(0, 1) activations.  A step is one GEMV call.  `value` is algorithmic HBM
bytes per step (weights + activations + output) / device time, with the
weights resident; 16+ distinct weight copies (> 3x the 126 MB L2) rotate so no
step reads another step's weights from L2.  The timed K steps run as CUDA
graph replays bracketed by CUDA events on the launching stream.

N > 1 (torchrun, one process per GPU): weak scaling of the LpPool form -- each
rank owns 11008 contiguous rows of an (N*11008) x 4096 matrix, runs the same
GEMV on them and gathers the output vector every step (the pool's NVLink
transport: peer stores from the GEMV itself), so every rank ends the step
holding the whole y.

`--impl reference` times the reference's algorithm on the host cores (the C
restatement in oracle/, pooled over every core like LpPool) on the same
workload; under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "dequant-GEMV HBM GB/s (% of B200 peak) per format; Q8_0 GEMM int8 TOPS"
FALLBACK_HBM_GBS = 6650.0
L2_BYTES = 126 * 1024 * 1024

M1, K1 = 11008, 4096   # config 1
# config 4: one Llama-7B layer is q, k, v, o (4096 x 4096) and gate, up
# (11008 x 4096) over the 4096-vector, stored as one 38400-row matrix, plus
# down (4096 x 11008) over the 11008-vector; packed int4, group 32.
CAT_ROWS, DOWN_ROWS, DOWN_K, LAYERS = 4 * 4096 + 2 * 11008, 4096, 11008, 32


def cfg1_bytes(M=M1, K=K1) -> int:
    """Algorithmic bytes of one config-1 call: Q4_0 blocks + fp32 x + fp32 y."""
    return M * (K // 32) * 18 + K * 4 + M * 4


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def load_traffic():
    """Per-launch DRAM bytes of the top kernel from a committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_id: str):
        self.device_id = device_id
        self.proc = None
        self.out = None

    def start(self):
        self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", self.device_id], stdout=self.out, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.out.flush()
        self.out.seek(0)
        rows = [r.split(",") for r in self.out.read().strip().splitlines() if r.strip()]
        os.unlink(self.out.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for nm, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(nm)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------ GPU workload
class Cfg1Workload:
    """Rotating copies of one rank's Q4_0 weight rows, x, y (device)."""

    def __init__(self, torch, L, M, K, seed, ncopies=None):
        self.torch, self.L, self.M, self.K = torch, L, M, K
        self.bpr = K // 32
        g = torch.Generator(device="cuda")
        g.manual_seed(seed)
        w = torch.randn(M * K, generator=g, device="cuda", dtype=torch.float32) * 0.02
        blocks = torch.empty(M * self.bpr * 18, dtype=torch.uint8, device="cuda")
        L.quantizeQ4_0Batch(w, blocks)
        del w
        wbytes = blocks.numel()
        self.ncopies = ncopies or max(2, -(-3 * L2_BYTES // wbytes) + 1)
        self.w = [blocks] + [blocks.clone() for _ in range(self.ncopies - 1)]
        g.manual_seed(seed + 1_000_000)
        self.x = torch.randn(K, generator=g, device="cuda", dtype=torch.float32)
        self.y = torch.empty(M, dtype=torch.float32, device="cuda")

    def step(self, i):
        self.L.dequantGemvQ4_0(self.w[i % self.ncopies], self.bpr, self.x, self.y)


def cfg4_bytes_per_layer() -> int:
    """Weight bytes (int4 codes + fp32 group scales) of one layer, all GPUs."""
    return (CAT_ROWS * (K1 // 2 + K1 // 32 * 4) + DOWN_ROWS * (DOWN_K // 2 + DOWN_K // 32 * 4))


class Cfg4Workload:
    """Config 4: 32 Llama-7B layers of packed-int4 weights, this rank's rows.

    Each rank holds rows [r * rows / P, (r + 1) * rows / P) of the concatenated
    matrix and of down (P divides both).  A step is one decode sweep: per
    layer, quantize the 4096-vector to Q8_0 on the GPU, dequantGemvI4Q8 over
    the concatenated matrix, quantize the 11008-vector, dequantGemvI4Q8 over
    down; with P > 1 the layer's outputs are then all-gathered once.  The
    layer's output buffer is rank-major -- rank r's [concatenated slice | down
    slice] -- so the gather is one call over 42496 / P floats per rank."""

    def __init__(self, torch, L, world, rank, layers=LAYERS):
        assert CAT_ROWS % world == 0 and DOWN_ROWS % world == 0
        self.torch, self.L, self.world, self.rank, self.layers = torch, L, world, rank, layers
        self.rc, self.rd = CAT_ROWS // world, DOWN_ROWS // world
        self.per = self.rc + self.rd
        g = torch.Generator(device="cuda")
        self.wc, self.sc, self.wd, self.sd = [], [], [], []
        for layer in range(layers):
            for rows, k, W, S, part in ((self.rc, K1, self.wc, self.sc, 0),
                                        (self.rd, DOWN_K, self.wd, self.sd, 1)):
                g.manual_seed(4000 + layer + 100 * part + 1000 * rank)
                w = torch.randn(rows * k, generator=g, device="cuda", dtype=torch.float32) * 0.02
                sc = torch.empty(rows * k // 32, dtype=torch.float32, device="cuda")
                L.calibrateSymmetric(w, 32, 7.0, sc)
                pk = torch.empty(rows * k // 2, dtype=torch.uint8, device="cuda")
                L.quantizeI4Packed(w, sc, 32, pk)
                del w
                W.append(pk)
                S.append(sc)
        g.manual_seed(4000 + 1_000_000)
        self.x = torch.randn(layers, K1, generator=g, device="cuda", dtype=torch.float32)
        self.xd = torch.randn(layers, DOWN_K, generator=g, device="cuda", dtype=torch.float32)
        self.xq = torch.empty(K1, dtype=torch.int8, device="cuda")
        self.xs = torch.empty(K1 // 32, dtype=torch.float32, device="cuda")
        self.dq = torch.empty(DOWN_K, dtype=torch.int8, device="cuda")
        self.ds = torch.empty(DOWN_K // 32, dtype=torch.float32, device="cuda")
        self.y = torch.empty(layers, world * self.per, dtype=torch.float32, device="cuda")
        torch.cuda.empty_cache()

    def layer(self, pool, layer, fused=True):
        """fused: each GEMV quantizes its fp32 activations to Q8_0 itself
        (quantizeDequantGemvI4Q8, two launches per layer); else the separate
        quantizeQ8_0 launches (four per layer) -- the same bits."""
        L = self.L
        yl = self.y[layer]
        off = self.rank * self.per
        if fused:
            L.quantizeDequantGemvI4Q8(self.wc[layer], self.sc[layer], 32, self.x[layer],
                                      yl[off:off + self.rc])
            L.quantizeDequantGemvI4Q8(self.wd[layer], self.sd[layer], 32, self.xd[layer],
                                      yl[off + self.rc:off + self.per])
        else:
            L.quantizeQ8_0Split(self.x[layer], self.xq, self.xs)
            L.dequantGemvI4Q8(self.wc[layer], self.sc[layer], 32, self.xq, self.xs,
                              yl[off:off + self.rc])
            L.quantizeQ8_0Split(self.xd[layer], self.dq, self.ds)
            L.dequantGemvI4Q8(self.wd[layer], self.sd[layer], 32, self.dq, self.ds,
                              yl[off + self.rc:off + self.per])
        if pool is not None:
            from nim_lowprec_b200 import parallel as P
            pool.call("lp_pool_gather_rows", yl.data_ptr(), self.world * self.per, 1, P._stream())

    def step(self, pool, i):
        for layer in range(self.layers):
            self.layer(pool, layer)


def graph_time(torch, step, K, W, barrier, chunk=500):
    """W eager warm-up steps, then exactly K steps timed as graph replays."""
    for i in range(W):
        step(i)
    torch.cuda.synchronize()
    G = min(chunk, K)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graphs = []
    with torch.cuda.stream(s):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(G):
                step(i)
        graphs.append((g, K // G))
        rem = K % G
        if rem:
            g2 = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g2, stream=s):
                for i in range(rem):
                    step(i)
            graphs.append((g2, 1))
    torch.cuda.current_stream().wait_stream(s)
    for g, _ in graphs:       # upload + one untimed pass
        g.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    start.record(stream)
    for g, reps in graphs:
        for _ in range(reps):
            g.replay()
    end.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = start.elapsed_time(end)
    return ms, graphs


def device_uuid(torch):
    try:
        u = torch.cuda.get_device_properties(torch.cuda.current_device()).uuid
        s = str(u)
        return s if s.startswith("GPU-") else "GPU-" + s
    except Exception:
        return str(torch.cuda.current_device())


# -------------------------------------------------------------- CPU side
def cpu_baseline(seconds=8.0, M=M1, K=K1, threads=0):
    """The reference's algorithm (oracle port, pooled over all host cores)
    on config 1; returns (GB/s, cores, sample description)."""
    from oracle import oracle as O
    rng = np.random.default_rng(1)
    w = (rng.standard_normal(M * K, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    x = rng.standard_normal(K, dtype=np.float32)
    blocks = O.quantizeQ4_0(w).reshape(-1)
    del w
    pool = O.Pool(threads)
    cores = pool.threadCount()
    try:
        O.dequantGemvQ4_0(blocks, K // 32, x, pool=pool)   # warm
        n = 0
        t0 = time.perf_counter()
        while True:
            O.dequantGemvQ4_0(blocks, K // 32, x, pool=pool)
            n += 1
            dt = time.perf_counter() - t0
            if dt >= seconds:
                break
    finally:
        pool.shutdown()
    gbs = n * cfg1_bytes(M, K) / dt / 1e9
    return gbs, cores, f"{n} full config-1 GEMVs ({M}x{K}) in {dt:.1f} s, LpPool-style row shards over {cores} threads"


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from oracle import oracle as O
    rng = np.random.default_rng(1)
    w = (rng.standard_normal(M1 * K1, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    x = rng.standard_normal(K1, dtype=np.float32)
    blocks = O.quantizeQ4_0(w).reshape(M1, -1)
    del w
    pool = O.Pool(0)
    cores = pool.threadCount()
    # size a step so the whole run stays within ~2 minutes
    t0 = time.perf_counter()
    O.dequantGemvQ4_0(blocks, K1 // 32, x, pool=pool)
    t_full = time.perf_counter() - t0
    budget = 90.0 / max(1, args.steps + args.warmup)
    rows = int(min(M1, max(64 * cores, M1 * budget / max(t_full, 1e-6))))
    rows = max(1, min(M1, rows))
    sub = np.ascontiguousarray(blocks[:rows]).reshape(-1)
    for _ in range(args.warmup):
        O.dequantGemvQ4_0(sub, K1 // 32, x, pool=pool)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.dequantGemvQ4_0(sub, K1 // 32, x, pool=pool)
    dt = time.perf_counter() - t0
    pool.shutdown()
    nbytes = cfg1_bytes(rows, K1)
    gbs = args.steps * nbytes / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config1: ggml Q4_0 fused dequant-GEMV, fp32 activations, 11008x4096",
                   "sample_rows": rows},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"{rows} of {M1} rows per step (C restatement of the scalar path, LpPool-style pool)"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-formats", action="store_true")
    ap.add_argument("--profile", action="store_true",
                    help="launch each hot kernel once (for ncu), no timing")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.profile:
        import torch

        import nim_lowprec_b200 as L
        for name in profile_kernels(torch, L):
            print("launched:", name, flush=True)
        return 0

    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))

    def barrier():
        if dist is not None:
            dist.barrier()

    import nim_lowprec_b200 as L

    wl = Cfg1Workload(torch, L, M1, K1, seed=1 + rank)
    # N > 1: one (M1 * N)-row matrix row-sharded over the GPUs (rank r holds
    # rows [M1 r, M1 (r + 1)) -- the pool's slicing), each step a pooled call of
    # the library's own pool: local GEMV + NCCL gather of all of y.
    pool = None
    y_all = None
    if world > 1:
        from nim_lowprec_b200 import parallel as P
        pool = P.NcclPool()
        y_all = torch.empty(world * M1, dtype=torch.float32, device="cuda")

    def step(i):
        if pool is not None:
            P.parDequantGemvQ4_0(pool, wl.w[i % wl.ncopies], wl.bpr, wl.x, y_all, sharded=True)
        else:
            wl.step(i)

    clk = ClockSampler(device_uuid(torch))
    clk.start()
    ms, graphs = graph_time(torch, step, args.steps, max(3, args.warmup), barrier)
    clocks = clk.stop()
    del graphs
    t = torch.tensor([ms], device="cuda")
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    per_step_ms = ms / args.steps
    total_bytes = world * args.steps * cfg1_bytes()
    value = total_bytes / (ms / 1e3) / 1e9

    # roofline of the dominant kernel (this rank's GEMV launches)
    peak, peak_kind = load_peaks()
    if world == 1:
        kernel_ms = per_step_ms
    else:  # time the GEMV alone for the roofline
        kms, g2 = graph_time(torch, wl.step, min(args.steps, 20000), 3, barrier)
        del g2
        kernel_ms = kms / min(args.steps, 20000)
    achieved = cfg1_bytes() / (kernel_ms / 1e3) / 1e9
    traffic = load_traffic().get("gemv_q4_0_cfg1")

    # e2e through the public API: x from pinned host memory in, y back out
    xh = torch.empty(K1, dtype=torch.float32).pin_memory()
    xh.copy_(torch.randn(K1))
    yh = torch.empty(M1, dtype=torch.float32).pin_memory()

    yh_all = torch.empty(world * M1, dtype=torch.float32).pin_memory() if world > 1 else None

    if pool is None:
        # One GPU: x comes in from page-locked memory by the library's copy-in
        # kernel (one read over the host link, overlapping the previous GEMV;
        # every CTA stages all of x, so the GEMV reading it in place would
        # cross it 148 times); the C-ABI call writes y straight into
        # page-locked host memory (its device address), each value once.
        from nim_lowprec_b200 import _native as NV
        xh_dev, yh_dev = NV.host_device_pointer(xh.data_ptr()), NV.host_device_pointer(yh.data_ptr())
        lib, nblk = NV.lib(), M1 * wl.bpr

        def e2e_step(i):
            st = torch.cuda.current_stream().cuda_stream
            NV.check(lib.lp_copy_in(wl.x.data_ptr(), xh_dev, K1 * 4, st), "e2e copy_in")
            NV.check(lib.lp_dequant_gemv_q4_0(wl.w[i % wl.ncopies].data_ptr(), nblk, wl.bpr,
                                              wl.x.data_ptr(), K1, yh_dev, M1,
                                              torch.cuda.current_stream().cuda_stream),
                     "e2e dequantGemvQ4_0")
        transfer = ("x: lp_copy_in kernel from page-locked memory; y: written by the GEMV "
                    "into page-locked host memory")
    elif not pool.p2p:
        # the pool's NCCL transport gathers device buffers only
        def e2e_step(i):
            wl.x.copy_(xh, non_blocking=True)
            step(i)
            yh_all.copy_(y_all, non_blocking=True)
        transfer = "cudaMemcpyAsync of x in and of the gathered y out, per step"
    else:
        # N GPUs: x in by the copy-in kernel; the pooled call's y is the
        # page-locked host vector itself -- the GEMV writes this rank's rows
        # and the receive kernel the other ranks' rows straight into it.
        from nim_lowprec_b200 import _native as NV
        xh_dev = NV.host_device_pointer(xh.data_ptr())
        yall_dev = NV.host_device_pointer(yh_all.data_ptr())
        lib, nblk = NV.lib(), M1 * wl.bpr

        def e2e_step(i):
            st = torch.cuda.current_stream().cuda_stream
            NV.check(lib.lp_copy_in(wl.x.data_ptr(), xh_dev, K1 * 4, st), "e2e copy_in")
            pool.call("lp_pool_dequant_gemv_q4_0", wl.w[i % wl.ncopies].data_ptr(), nblk, wl.bpr,
                      wl.x.data_ptr(), K1, yall_dev, world * M1, st)
        transfer = ("x: lp_copy_in kernel from page-locked memory; y: the pooled call writes the "
                    "whole gathered vector into page-locked host memory")

    e2e_steps = min(args.steps, 20000)
    e_ms, g3 = graph_time(torch, e2e_step, e2e_steps, 3, barrier)
    t = torch.tensor([e_ms], device="cuda")
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e_ms = float(t.item())
    e2e_value = world * e2e_steps * cfg1_bytes() / (e_ms / 1e3) / 1e9
    # the host-buffer path gives the device path's bits (every rank, same calls)
    del g3
    torch.cuda.synchronize()
    barrier()
    wl.x.copy_(xh)
    step(0)
    e2e_step(0)
    torch.cuda.synchronize()
    got, want = (yh, wl.y) if pool is None else (yh_all, y_all)
    if not torch.equal(got, want.cpu()):
        raise SystemExit("e2e: host-buffer GEMV differs from the device-buffer GEMV")
    g3 = None

    # config 4 (every rank): the 32-layer int4 decode sweep, pooled for N > 1
    cfg4 = None
    if not args.no_formats:
        wl4 = Cfg4Workload(torch, L, world, rank)
        st4 = 20
        ms4, g5 = graph_time(torch, lambda i: wl4.step(pool, i), st4, 3, barrier, chunk=st4)
        del g5
        t = torch.tensor([ms4], device="cuda")
        if dist is not None:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        sweep_ms = float(t.item()) / st4
        gbs = LAYERS * cfg4_bytes_per_layer() / (sweep_ms / 1e3) / 1e9
        cfg4 = {"GB/s": round(gbs, 1), "frac_per_gpu": round(gbs / world / peak, 3),
                "ms_per_sweep": round(sweep_ms, 4), "layers": LAYERS,
                "weight_bytes_per_sweep": LAYERS * cfg4_bytes_per_layer(),
                "launches_per_layer": 2, "gather_per_layer": world > 1}
        del wl4
        torch.cuda.empty_cache()

    formats = None
    if not args.no_formats and world == 1:
        formats = per_format(torch, L, barrier)
        # the same headline workload in the bit-exact fp32 mode
        with L.fp32_mode("exact"):
            xms, g4 = graph_time(torch, wl.step, 5000, 5, barrier)
        del g4
        v = cfg1_bytes() / (xms / 5000 / 1e3) / 1e9
        formats["config1_q4_0_exact_mode"] = {"GB/s": round(v, 1), "frac": round(v / peak, 3),
                                              "us": round(xms / 5000 * 1e3, 2)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, sample = cpu_baseline()
        cpu = {"value": round(v, 3), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample}

    if dist is not None:
        del g3
        dist.barrier()
        if pool is not None:
            pool.shutdown()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_step_ms, 6),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {
            "workload": "config1: ggml Q4_0 fused dequant-GEMV, fp32 activations, 11008x4096 per GPU",
            "rows_per_gpu": M1, "k": K1, "algorithmic_bytes_per_step_per_gpu": cfg1_bytes(),
            "l2": f"{wl.ncopies} rotating weight copies ({wl.ncopies * M1 * K1 // 32 * 18 / 1e6:.0f} MB > 3x L2)",
            "parallelism": "single GPU" if world == 1 else
                           f"{world * M1}x{K1} rows sharded over {world} GPUs (library pool), NCCL gather of y per step",
            "timing": "CUDA-graph replays, CUDA events on the launching stream, max over ranks",
            "fp32_mode": "fast: block-float activations, exact integer group dots "
                         "(tested within 1e-6 of sum|w||x| per row vs the reference order)",
        },
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "peak_kind": f"{peak_kind} hbm_gbs"},
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": K1 * 4,
                "d2h_bytes_per_step": world * M1 * 4, "steps": e2e_steps, "transfer": transfer},
        "gpu_launches": args.steps,
        "clocks": clocks,
    }
    if formats:
        line["formats"] = formats
    if cfg4:
        line["config4_llama7b_i4q8_sweep"] = cfg4
    print(json.dumps(line), flush=True)
    return 0


PROFILE_KERNELS = ("gemv_kernel|k_gemm_tc|k_quantize_q8_0|k_dequantize_q4_k|k_dequantize_q6_k"
                   "|k_dequantize_batch")


def profile_kernels(torch, L):
    """One launch of every hot kernel, for an ncu capture of exactly these
    launches (`-k regex:` PROFILE_KERNELS `-c 15`).  Inputs are prepared
    with other kernels (torch RNG, the weight encoders), and each workload is
    freed before the next, so a capture holds a few hundred MB at most."""
    g = torch.Generator(device="cuda")
    sync = torch.cuda.synchronize
    done = []

    def rnd(n, seed, scale=1.0):
        g.manual_seed(seed)
        return torch.randn(n, generator=g, device="cuda", dtype=torch.float32) * scale

    def i8(n, seed):
        g.manual_seed(seed)
        return torch.randint(-127, 128, (n,), dtype=torch.int8, device="cuda", generator=g)

    def scales(n, seed):
        g.manual_seed(seed)
        return torch.rand(n, generator=g, device="cuda", dtype=torch.float32) * 1e-3

    def run(name, fn):
        sync()
        fn()
        sync()
        done.append(name)

    M = K = 4096
    wq, wd = i8(M * K, 0), scales(M * K // 32, 0)
    xq, xs, y = i8(K, 1), scales(K // 32, 1), torch.empty(M, device="cuda")
    run("config0 dequantGemvQ8 4096x4096", lambda: L.dequantGemvQ8(wq, wd, 32, xq, xs, y))
    for B in (8, 64, 512):
        xqB, xsB = i8(K * B, 2 + B), scales(K * B // 32, 2 + B)
        yB = torch.empty(M * B, device="cuda")
        run(f"config3 dequantGemmQ8 B={B}",
            lambda: L.dequantGemmQ8(wq, wd, 32, xqB, xsB, B, yB))
        del xqB, xsB, yB
    del wq, wd, xq, xs, y
    torch.cuda.empty_cache()

    w = rnd(M1 * K1, 1, 0.02)
    blocks = torch.empty(M1 * K1 // 32 * 18, dtype=torch.uint8, device="cuda")
    L.quantizeQ4_0Batch(w, blocks)
    del w
    x, y = rnd(K1, 1_000_001), torch.empty(M1, device="cuda")
    run("config1 dequantGemvQ4_0 block-float", lambda: L.dequantGemvQ4_0(blocks, K1 // 32, x, y))
    with L.fp32_mode("exact"):
        run("config1 dequantGemvQ4_0 exact", lambda: L.dequantGemvQ4_0(blocks, K1 // 32, x, y))
    del blocks, x, y
    torch.cuda.empty_cache()

    M2 = 14336
    w = rnd(M2 * K1, 2, 0.02)
    sc = torch.empty(M2 * K1 // 32, dtype=torch.float32, device="cuda")
    L.calibrateMX(w, 32, 2, sc)
    pk = torch.empty(M2 * K1 // 2, dtype=torch.uint8, device="cuda")
    L.quantizeF4Packed(w, sc, 32, pk)
    del w
    x, y = rnd(K1, 1_000_002), torch.empty(M2, device="cuda")
    run("config2 dequantGemvF4 block-float", lambda: L.dequantGemvF4(pk, sc, 32, x, y))
    del sc, pk, x, y
    torch.cuda.empty_cache()

    n = 16_777_216
    xb = rnd(n, 5)
    qs = torch.empty(n, dtype=torch.int8, device="cuda")
    d = torch.empty(n // 32, dtype=torch.float32, device="cuda")
    run("quantizeQ8_0 K=16777216", lambda: L.quantizeQ8_0Split(xb, qs, d))
    del xb, qs, d
    torch.cuda.empty_cache()

    wl4 = Cfg4Workload(torch, L, 1, 0, layers=1)
    run("config4 layer 0: quantizeQ8_0 (4096), dequantGemvI4Q8 38400x4096, "
        "quantizeQ8_0 (11008), dequantGemvI4Q8 4096x11008", lambda: wl4.layer(None, 0, fused=False))
    del wl4
    torch.cuda.empty_cache()

    # k-quant super-block dequantization, 65536 super-blocks (16.7 M values)
    nb = 65536
    for bb, fn, name in ((144, L.dequantizeQ4_K, "Q4_K"), (210, L.dequantizeQ6_K, "Q6_K")):
        g.manual_seed(7)
        raw = torch.randint(0, 256, (nb, bb), dtype=torch.uint8, device="cuda", generator=g)
        dpos = (0, 2) if bb == 144 else (208,)
        for p_ in dpos:  # finite f16 scales
            raw[:, p_:p_ + 2] = (torch.randn(nb, device="cuda", generator=g) * 0.1).half() \
                .view(torch.uint8).view(nb, 2)
        out = torch.empty(nb * 256, device="cuda")
        run(f"dequantize{name} 65536 super-blocks", lambda: fn(raw.view(-1), out))
        del raw, out

    # dequantizeBatch, int8 per group of 128, 16,000,000 values
    q, sc = i8(16_000_000, 8), scales(125_000, 8)
    out = torch.empty(16_000_000, device="cuda")
    run("dequantizeBatch 16000000 group 128", lambda: L.dequantizeBatch(q, sc, 128, out))
    del q, sc, out
    return done


def per_format(torch, L, barrier, steps=5000):
    """Secondary numbers for the other BASELINE configs (not the headline)."""
    out = {}
    peak, _ = load_peaks()
    g = torch.Generator(device="cuda")

    def rnd(n, seed, scale=1.0):
        g.manual_seed(seed)
        return torch.randn(n, generator=g, device="cuda", dtype=torch.float32) * scale

    # config 0: dequantGemvQ8 4096^2, weights and activations Q8_0 (split form)
    M = K = 4096
    w = rnd(M * K, 0, 0.02)
    wq = torch.empty(M * K, dtype=torch.int8, device="cuda")
    wd = torch.empty(M * K // 32, dtype=torch.float32, device="cuda")
    L.quantizeQ8_0Split(w, wq, wd)
    del w
    x = rnd(K, 1_000_000)
    xq = torch.empty(K, dtype=torch.int8, device="cuda")
    xs = torch.empty(K // 32, dtype=torch.float32, device="cuda")
    L.quantizeQ8_0Split(x, xq, xs)
    y = torch.empty(M, dtype=torch.float32, device="cuda")
    nb = M * K + M * K // 32 * 4 + K + K // 32 * 4 + M * 4
    R = -(-3 * L2_BYTES // (M * K + M * K // 8)) + 1
    copies = [(wq, wd)] + [(wq.clone(), wd.clone()) for _ in range(R - 1)]
    ms, gr = graph_time(torch, lambda i: L.dequantGemvQ8(*copies[i % R], 32, xq, xs, y), steps, 5, barrier)
    del gr
    v = nb / (ms / steps / 1e3) / 1e9
    out["config0_q8xq8_4096"] = {"GB/s": round(v, 1), "frac": round(v / peak, 3), "us": round(ms / steps * 1e3, 2)}
    del copies

    # config 2: MXFP4 14336x4096
    M, K = 14336, 4096
    w = rnd(M * K, 2, 0.02)
    sc = torch.empty(M * K // 32, dtype=torch.float32, device="cuda")
    L.calibrateMX(w, 32, 2, sc)
    pk = torch.empty(M * K // 2, dtype=torch.uint8, device="cuda")
    L.quantizeF4Packed(w, sc, 32, pk)
    del w
    x = rnd(K, 1_000_002)
    y = torch.empty(M, dtype=torch.float32, device="cuda")
    nb = M * K // 2 + M * K // 32 * 4 + K * 4 + M * 4
    R = -(-3 * L2_BYTES // nb) + 1
    copies = [(pk, sc)] + [(pk.clone(), sc.clone()) for _ in range(R - 1)]
    for mode in ("fast", "exact"):
        with L.fp32_mode(mode):
            ms, gr = graph_time(torch, lambda i: L.dequantGemvF4(copies[i % R][0], copies[i % R][1], 32, x, y),
                                steps, 5, barrier)
        del gr
        v = nb / (ms / steps / 1e3) / 1e9
        key = "config2_mxfp4_14336x4096" + ("" if mode == "fast" else "_exact_mode")
        out[key] = {"GB/s": round(v, 1), "frac": round(v / peak, 3), "us": round(ms / steps * 1e3, 2)}
    del copies

    # the Q8_0 activation quantizer at the README's size (K = 16,777,216):
    # 4 bytes in, 34/32 bytes out per element
    n = 16_777_216
    xb = [rnd(n, 5 + c) for c in range(3)]  # 3 x 67 MB inputs rotate: more than L2
    qs = torch.empty(n, dtype=torch.int8, device="cuda")
    d = torch.empty(n // 32, dtype=torch.float32, device="cuda")
    ms, gr = graph_time(torch, lambda i: L.quantizeQ8_0Split(xb[i % 3], qs, d), 200, 3, barrier)
    del gr
    nb = 4 * n + n + 4 * (n // 32)
    v = nb / (ms / 200 / 1e3) / 1e9
    out["quantizeQ8_0_16M"] = {"GB/s": round(v, 1), "frac": round(v / peak, 3),
                               "us": round(ms / 200 * 1e3, 2)}
    del xb, qs, d

    # k-quant super-block dequantization (GGUF ingestion), 65536 super-blocks
    nbk = 65536
    outs = [torch.empty(nbk * 256, device="cuda") for _ in range(3)]  # 3 x 67 MB: more than L2
    for bb, fn, name in ((144, L.dequantizeQ4_K, "Q4_K"), (210, L.dequantizeQ6_K, "Q6_K")):
        g.manual_seed(7)
        raw = torch.randint(0, 256, (nbk, bb), dtype=torch.uint8, device="cuda", generator=g)
        for p_ in ((0, 2) if bb == 144 else (208,)):
            raw[:, p_:p_ + 2] = (torch.randn(nbk, device="cuda", generator=g) * 0.1).half() \
                .view(torch.uint8).view(nbk, 2)
        flat = raw.view(-1)
        ms, gr = graph_time(torch, lambda i: fn(flat, outs[i % 3]), 300, 3, barrier)
        del gr
        nbytes = nbk * bb + nbk * 256 * 4
        v = nbytes / (ms / 300 / 1e3) / 1e9
        out[f"dequantize{name}_65536"] = {"GB/s": round(v, 1), "frac": round(v / peak, 3),
                                          "us": round(ms / 300 * 1e3, 2)}
        del raw, flat
    del outs

    # dequantizeBatch, int8 per group of 128 over 16,000,000 values (the shape of
    # the reference's elementwise-dequant benchmark, bench_dequant.nim:13-14)
    n, gsz = 16_000_000, 128
    qb = [torch.randint(-128, 128, (n,), dtype=torch.int8, device="cuda", generator=g)
          for _ in range(3)]
    scb = torch.rand(n // gsz, device="cuda", generator=g) * 0.1
    dst = [torch.empty(n, device="cuda") for _ in range(3)]  # 3 x 80 MB: more than L2
    ms, gr = graph_time(torch, lambda i: L.dequantizeBatch(qb[i % 3], scb, gsz, dst[i % 3]),
                        300, 3, barrier)
    del gr
    nbytes = n + 4 * n + 4 * (n // gsz)
    v = nbytes / (ms / 300 / 1e3) / 1e9
    out["dequantizeBatch_16M_g128"] = {"GB/s": round(v, 1), "frac": round(v / peak, 3),
                                       "us": round(ms / 300 * 1e3, 2)}
    del qb, scb, dst

    # config 3: dequantGemmQ8 4096^2 x B
    M = K = 4096
    w = rnd(M * K, 3, 0.02)
    wq = torch.empty(M * K, dtype=torch.int8, device="cuda")
    wd = torch.empty(M * K // 32, dtype=torch.float32, device="cuda")
    L.quantizeQ8_0Split(w, wq, wd)
    del w
    R = -(-3 * L2_BYTES // (M * K + M * K // 8)) + 1
    copies = [(wq, wd)] + [(wq.clone(), wd.clone()) for _ in range(R - 1)]
    for B in (8, 64, 512):
        x = rnd(K * B, 1_000_003)
        xq = torch.empty(K * B, dtype=torch.int8, device="cuda")
        xs = torch.empty(K * B // 32, dtype=torch.float32, device="cuda")
        L.quantizeQ8_0Split(x, xq, xs)
        y = torch.empty(M * B, dtype=torch.float32, device="cuda")
        st = 200 if B == 512 else 1000
        ms, gr = graph_time(torch, lambda i: L.dequantGemmQ8(*copies[i % R], 32, xq, xs, B, y), st, 3,
                            barrier)
        del gr
        us = ms / st * 1e3
        tops = 2 * M * K * B / (us / 1e6) / 1e12
        out[f"config3_gemm_q8_B{B}"] = {"TOPS": round(tops, 2), "us": round(us, 2),
                                        "path": "GEMV-skeleton columns (CUDA-core dp4a)" if B <= 16
                                        else "tcgen05 kind::i8"}
    del copies
    return out


if __name__ == "__main__":
    sys.exit(main())
