"""LpPool's row-sharded forms across the GPUs of one box (parallel.nim:82-474).

One process per GPU, joined by ``torch.distributed``.  Rank r of P owns the
rows ``[per*r, per*r + per)`` of every weight matrix, ``per = m div P``, and
the last rank takes the remainder -- the slicing of ``parallel.nim:118-124``
(``shardRows``, computed by the library's ``lp_pool_rows``).  Every output row
depends only on its own weight row, so a sharded call gives the serial bits.

* ``Pool(group)`` gathers the row slices of y with ``torch.distributed``
  (NCCL for CUDA tensors; any backend works, gloo included).
* ``NcclPool(group, device)`` is the C-ABI pool of one process per GPU
  (``lp_pool_*``): the library runs the local slice and assembles y on every
  rank itself, over NVLink peer stores (or an NCCL group of broadcasts).
* ``LocalPool(threads)`` is the reference's own shape of pool -- one process,
  one worker per GPU, host arrays (``lph_pool_*`` / ``lph_par_*``): every
  worker runs its row slice on its GPU and writes its rows of the caller's
  host y.  This is the form the Nim shim binds (``initPool``, ``shutdown``,
  ``threadCount``, the pooled and per-call ``par*`` procs).

The ``par*`` procs take the reference's arguments.  For the multi-process
pools the weight arrays are either whole (the reference's call: each rank
slices its rows) or, with ``sharded=True``, already this rank's slice
(weights resident per GPU); activations and ``y`` are whole and every rank
ends with all of ``y``.  For ``LocalPool`` every array is a whole host array.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _native as N
from . import dequant as D

try:
    import torch
except Exception:  # pragma: no cover
    torch = None


def shardRows(m: int, nranks: int, rank: int):
    """(begin, end) of rank's row slice (parallel.nim:118-124)."""
    b, e = ctypes.c_int64(), ctypes.c_int64()
    N.check(N.lib().lp_pool_rows(int(m), int(nranks), int(rank), ctypes.byref(b), ctypes.byref(e)),
            "lp_pool_rows")
    return b.value, e.value


def _numel(a) -> int:
    return int(a.numel()) if (torch is not None and isinstance(a, torch.Tensor)) else int(np.asarray(a).size)


def _flat(a):
    return a.reshape(-1)


class Pool:
    """A member of a row-sharded pool over a ``torch.distributed`` group."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self._dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)

    # -- the reference's slicing -------------------------------------------
    def rows(self, m: int):
        return shardRows(m, self.size, self.rank)

    def slice(self, a, m: int):
        """This rank's rows of a row-major array holding m rows."""
        n = _numel(a)
        if m == 0 or n % m:
            raise AssertionError(f"array of {n} elements is not {m} rows")
        per = n // m
        b, e = self.rows(m)
        return _flat(a)[b * per:e * per]

    # -- gather ------------------------------------------------------------
    def gather(self, y, m: int, per_row: int = 1):
        """Every rank's row slice of y (m rows of per_row values) into y."""
        P = self.size
        if P == 1 or m == 0:
            return y
        yf = _flat(y)
        spans = [shardRows(m, P, r) for r in range(P)]
        mx = max(e - b for b, e in spans) * per_row
        b, e = spans[self.rank]
        send = torch.zeros(mx, dtype=yf.dtype, device=yf.device)
        send[:(e - b) * per_row] = yf[b * per_row:e * per_row]
        recv = [torch.empty_like(send) for _ in range(P)]
        self._dist.all_gather(recv, send, group=self.group)
        for r, (rb, re_) in enumerate(spans):
            yf[rb * per_row:re_ * per_row] = recv[r][:(re_ - rb) * per_row]
        return y

    def run(self, local, y, m: int, per_row: int = 1):
        """local(y_slice) computes this rank's rows in place; then gather."""
        b, e = self.rows(m)
        local(_flat(y)[b * per_row:e * per_row])
        return self.gather(y, m, per_row)

    def shutdown(self):  # parallel.nim:153-167; the group belongs to the caller
        pass


class NcclPool:
    """The library's own pool (``lp_pool_*``): NCCL communicator inside."""

    def __init__(self, group=None, device: int | None = None):
        import torch.distributed as dist
        rank, size = dist.get_rank(group), dist.get_world_size(group)
        ident = bytearray(128)
        if rank == 0:
            buf = (ctypes.c_uint8 * 128)()
            N.check(N.lib().lp_pool_unique_id(buf), "lp_pool_unique_id")
            ident = bytearray(bytes(buf))
        obj = [bytes(ident)]
        dist.broadcast_object_list(obj, src=dist.get_global_rank(group, 0) if group else 0,
                                   group=group)
        dev = torch.cuda.current_device() if device is None else int(device)
        self._h = ctypes.c_void_p()
        idbuf = (ctypes.c_uint8 * 128).from_buffer_copy(obj[0])
        N.check(N.lib().lp_pool_init(ctypes.byref(self._h), idbuf, size, rank, dev), "lp_pool_init")
        self.rank, self.size, self.device = rank, size, dev

    def rows(self, m: int):
        return shardRows(m, self.size, self.rank)

    def slice(self, a, m: int):
        n = _numel(a)
        if m == 0 or n % m:
            raise AssertionError(f"array of {n} elements is not {m} rows")
        per = n // m
        b, e = self.rows(m)
        return _flat(a)[b * per:e * per]

    def call(self, name: str, *args):
        N.check(getattr(N.lib(), name)(self._h, *args), name)

    def group_begin(self, y, n=None):
        """Pooled calls until group_end write parts of y and are received
        once (lp_pool_group_begin).  y: a device tensor, or a device address
        (e.g. of page-locked host memory, _native.host_device_pointer) with
        its length n in floats."""
        ptr, length = (y, n) if n is not None else (_dev(y), _numel(y))
        N.check(N.lib().lp_pool_group_begin(self._h, ptr, length), "lp_pool_group_begin")

    def group_end(self):
        N.check(N.lib().lp_pool_group_end(self._h, _stream()), "lp_pool_group_end")

    @property
    def p2p(self) -> bool:
        """True when gathers use the NVLink exchange buffers (the default when
        every rank has its own GPU), False for the NCCL group."""
        v = ctypes.c_int(0)
        N.check(N.lib().lp_pool_get_p2p(self._h, ctypes.byref(v)), "lp_pool_get_p2p")
        return bool(v.value)

    @p2p.setter
    def p2p(self, enable: bool) -> None:
        # every rank must switch before its next gather
        N.check(N.lib().lp_pool_set_p2p(self._h, 1 if enable else 0), "lp_pool_set_p2p")

    def shutdown(self):
        if self._h:
            N.check(N.lib().lp_pool_destroy(self._h), "lp_pool_destroy")
            self._h = ctypes.c_void_p()

    def __del__(self):  # pragma: no cover
        try:
            self.shutdown()
        except Exception:
            pass


class LocalPool:
    """initPool(threads) of the reference (parallel.nim:134-171) over this
    box's GPUs in one process: ``threads`` workers, one per GPU (<= 0: every
    visible GPU).  ``shutdown`` is idempotent; ``threadCount`` is 0 after it."""

    def __init__(self, threads: int = 0):
        self._h = ctypes.c_void_p()
        N.check(N.lib().lph_pool_init(ctypes.byref(self._h), int(threads)), "lph_pool_init")

    def threadCount(self) -> int:
        return int(N.lib().lph_pool_thread_count(self._h))

    def shutdown(self):
        N.check(N.lib().lph_pool_shutdown(ctypes.byref(self._h)), "lph_pool_shutdown")

    def call(self, name: str, *args):
        N.check(getattr(N.lib(), name)(self._h, *args), name)

    def __del__(self):  # pragma: no cover
        try:
            self.shutdown()
        except Exception:
            pass


def initPool(group=None, nccl: bool = False, device: int | None = None):
    """initPool (parallel.nim:134-151): this process's member of the pool."""
    return NcclPool(group, device) if nccl else Pool(group)


def _hp(a):
    a = np.ascontiguousarray(a)
    return a, (a.ctypes.data_as(ctypes.c_void_p) if a.size else None)


def _host_par(name, w, sc, gs, x, y, threads, wdt, blocks=None):
    """lph_par_* over host arrays: the per-call par* procs (parallel.nim:186-418)."""
    w, pw = _hp(w)
    x, px = _hp(x)
    if not (isinstance(y, np.ndarray) and y.flags.c_contiguous and y.dtype == np.float32):
        raise TypeError("y must be a contiguous float32 numpy array")
    py = y.ctypes.data_as(ctypes.c_void_p) if y.size else None
    if blocks is not None:
        N.check(getattr(N.lib(), name)(pw, w.size // blocks, int(gs), px, x.size, py, y.size,
                                       int(threads)), name)
        return
    sc, ps = _hp(sc)
    N.check(getattr(N.lib(), name)(pw, w.size, ps, sc.size, int(gs), px, x.size, py, y.size,
                                   int(threads)), name)


def parDequantGemvThreads(wq, scales, groupSize, x, y, threads=0):
    """parDequantGemv(..., threads) (parallel.nim:186-253) on this box's GPUs."""
    _host_par("lph_par_dequant_gemv", wq, scales, groupSize, x, y, threads, np.int8)


def parDequantGemvI4Threads(wpacked, scales, groupSize, x, y, threads=0):
    """parDequantGemvI4(..., threads) (parallel.nim:186-255)."""
    _host_par("lph_par_dequant_gemv_i4", wpacked, scales, groupSize, x, y, threads, np.uint8)


def parDequantGemvF4Threads(wpacked, scales, groupSize, x, y, threads=0):
    """parDequantGemvF4(..., threads) (parallel.nim:186-257)."""
    _host_par("lph_par_dequant_gemv_f4", wpacked, scales, groupSize, x, y, threads, np.uint8)


def parDequantGemvQ8_0Threads(w, blocksPerRow, x, y, threads=0):
    """parDequantGemvQ8_0(..., threads) (parallel.nim:260-307); w: Q8_0 block bytes."""
    _host_par("lph_par_dequant_gemv_q8_0", np.asarray(w).reshape(-1).view(np.uint8), None,
              blocksPerRow, x, y, threads, np.uint8, blocks=34)


def parDequantGemvQ4_0Threads(w, blocksPerRow, x, y, threads=0):
    """parDequantGemvQ4_0(..., threads) (parallel.nim:260-308); w: Q4_0 block bytes."""
    _host_par("lph_par_dequant_gemv_q4_0", np.asarray(w).reshape(-1).view(np.uint8), None,
              blocksPerRow, x, y, threads, np.uint8, blocks=18)


def _host_q8(name, pool, w, ws, gs, xq, xs, y, threads=None, n=None):
    w, pw = _hp(w)
    ws, pws = _hp(ws)
    xq, pxq = _hp(xq)
    xs, pxs = _hp(xs)
    if not (isinstance(y, np.ndarray) and y.flags.c_contiguous and y.dtype == np.float32):
        raise TypeError("y must be a contiguous float32 numpy array")
    py = y.ctypes.data_as(ctypes.c_void_p) if y.size else None
    args = [pw, w.size, pws, ws.size, int(gs), pxq, xq.size, pxs, xs.size]
    if n is not None:
        args.append(int(n))
    args += [py, y.size]
    if pool is not None:
        pool.call(name, *args)
    else:
        N.check(getattr(N.lib(), name)(*args, int(threads)), name)


def parDequantGemvQ8Threads(wq, wScales, groupSize, xq, xScales, y, threads=0):
    """The per-call parDequantGemvQ8 overload (parallel.nim:376-415)."""
    _host_q8("lph_par_dequant_gemv_q8", None, wq, wScales, groupSize, xq, xScales, y, threads)


def parDequantGemvI4Q8Threads(wpacked, wScales, groupSize, xq, xScales, y, threads=0):
    """The per-call parDequantGemvI4Q8 overload (parallel.nim:376-418)."""
    _host_q8("lph_par_dequant_gemv_i4q8", None, wpacked, wScales, groupSize, xq, xScales, y,
             threads)


# ------------------------------------------------------------ par* procs --

def _w(pool, a, m, sharded):
    return a if sharded else pool.slice(a, m)


def _dev(a):
    return a.data_ptr()


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _nccl_gemv(pool, name, wq, ws, gs, x, y, sharded):
    m = _numel(y)
    wq, ws = _w(pool, wq, m, sharded), _w(pool, ws, m, sharded)
    pool.call(name, _dev(wq), _numel(wq), _dev(ws), _numel(ws), int(gs), _dev(x), _numel(x),
              _dev(y), m, _stream())


def parDequantGemv(pool, wq, scales, groupSize, x, y, sharded=False):
    """parallel.nim:186-253 (defParGemv, int8 weights, fp32 activations)."""
    m = _numel(y)
    if isinstance(pool, NcclPool):
        return _nccl_gemv(pool, "lp_pool_dequant_gemv", wq, scales, groupSize, x, y, sharded)
    w, s = _w(pool, wq, m, sharded), _w(pool, scales, m, sharded)
    pool.run(lambda ys: D.dequantGemv(w, s, groupSize, x, ys), y, m)


def parDequantGemvI4(pool, wpacked, scales, groupSize, x, y, sharded=False):
    """parallel.nim:186-255 (defParGemv over dequantGemvI4)."""
    m = _numel(y)
    if isinstance(pool, NcclPool):
        return _nccl_gemv(pool, "lp_pool_dequant_gemv_i4", wpacked, scales, groupSize, x, y, sharded)
    w, s = _w(pool, wpacked, m, sharded), _w(pool, scales, m, sharded)
    pool.run(lambda ys: D.dequantGemvI4(w, s, groupSize, x, ys), y, m)


def parDequantGemvF4(pool, wpacked, scales, groupSize, x, y, sharded=False):
    """parallel.nim:186-257 (defParGemv over dequantGemvF4)."""
    m = _numel(y)
    if isinstance(pool, NcclPool):
        return _nccl_gemv(pool, "lp_pool_dequant_gemv_f4", wpacked, scales, groupSize, x, y, sharded)
    w, s = _w(pool, wpacked, m, sharded), _w(pool, scales, m, sharded)
    pool.run(lambda ys: D.dequantGemvF4(w, s, groupSize, x, ys), y, m)


def _blocks_rows(pool, w, m, sharded):
    return w if sharded else pool.slice(w, m)


def parDequantGemvQ8_0(pool, w, blocksPerRow, x, y, sharded=False):
    """parallel.nim:260-307 (defParBlockGemv, ggml Q8_0 weights, fp32 activations)."""
    m = _numel(y)
    ws = _blocks_rows(pool, w, m, sharded)
    if isinstance(pool, NcclPool):
        return pool.call("lp_pool_dequant_gemv_q8_0", _dev(ws), D._blocks(ws, 34),
                         int(blocksPerRow), _dev(x), _numel(x), _dev(y), m, _stream())
    pool.run(lambda ys: D.dequantGemvQ8_0(ws, blocksPerRow, x, ys), y, m)


def parDequantGemvQ4_0(pool, w, blocksPerRow, x, y, sharded=False):
    """parallel.nim:260-308 (defParBlockGemv over dequantGemvQ4_0)."""
    m = _numel(y)
    ws = _blocks_rows(pool, w, m, sharded)
    if isinstance(pool, NcclPool):
        return pool.call("lp_pool_dequant_gemv_q4_0", _dev(ws), D._blocks(ws, 18),
                         int(blocksPerRow), _dev(x), _numel(x), _dev(y), m, _stream())
    pool.run(lambda ys: D.dequantGemvQ4_0(ws, blocksPerRow, x, ys), y, m)


def _q8(pool, name, fn, w, wScales, groupSize, xq, xScales, y, sharded):
    if isinstance(pool, LocalPool):
        return _host_q8(name.replace("lp_pool_", "lph_pool_"), pool, w, wScales, groupSize, xq,
                        xScales, y)
    m = _numel(y)
    wl, sl = _w(pool, w, m, sharded), _w(pool, wScales, m, sharded)
    if isinstance(pool, NcclPool):
        return pool.call(name, _dev(wl), _numel(wl), _dev(sl), _numel(sl), int(groupSize), _dev(xq),
                         _numel(xq), _dev(xScales), _numel(xScales), _dev(y), m, _stream())
    pool.run(lambda ys: fn(wl, sl, groupSize, xq, xScales, ys), y, m)


def parDequantGemvQ8(pool, wq, wScales, groupSize, xq, xScales, y, sharded=False):
    """parallel.nim:310-415 (defParQ8Gemv: pooled and per-call int8 x int8)."""
    _q8(pool, "lp_pool_dequant_gemv_q8", D.dequantGemvQ8, wq, wScales, groupSize, xq, xScales, y,
        sharded)


def parDequantGemvI4Q8(pool, wpacked, wScales, groupSize, xq, xScales, y, sharded=False):
    """parallel.nim:310-418 (defParQ8Gemv over dequantGemvI4Q8)."""
    _q8(pool, "lp_pool_dequant_gemv_i4q8", D.dequantGemvI4Q8, wpacked, wScales, groupSize, xq,
        xScales, y, sharded)


def _gemm(pool, name, fn, w, wScales, groupSize, xq, xScales, n, y, sharded):
    if isinstance(pool, LocalPool):
        return _host_q8(name.replace("lp_pool_", "lph_pool_"), pool, w, wScales, groupSize, xq,
                        xScales, y, n=n)
    m = _numel(y) // n
    wl, sl = _w(pool, w, m, sharded), _w(pool, wScales, m, sharded)
    if isinstance(pool, NcclPool):
        return pool.call(name, _dev(wl), _numel(wl), _dev(sl), _numel(sl), int(groupSize), _dev(xq),
                         _numel(xq), _dev(xScales), _numel(xScales), int(n), _dev(y), _numel(y),
                         _stream())
    pool.run(lambda ys: fn(wl, sl, groupSize, xq, xScales, n, ys), y, m, per_row=n)


def parDequantGemmQ8(pool, wq, wScales, groupSize, xq, xScales, n, y, sharded=False):
    """parallel.nim:420-473 (defParGemm; y rows are row-major, n columns)."""
    _gemm(pool, "lp_pool_dequant_gemm_q8", D.dequantGemmQ8, wq, wScales, groupSize, xq, xScales, n,
          y, sharded)


def parDequantGemmI4Q8(pool, wpacked, wScales, groupSize, xq, xScales, n, y, sharded=False):
    """parallel.nim:420-474 (defParGemm over dequantGemmI4Q8)."""
    _gemm(pool, "lp_pool_dequant_gemm_i4q8", D.dequantGemmI4Q8, wpacked, wScales, groupSize, xq,
          xScales, n, y, sharded)
