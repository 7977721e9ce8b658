// host_pool.cu -- LpPool for one process driving several GPUs, with the
// reference's host-array calls (parallel.nim:82-474).
//
// The reference's LpPool is an in-process pool of worker threads: initPool
// starts them (parallel.nim:134-151), dispatch hands every worker its row
// range and blocks until all are done (:173-184), shutdown joins them and is
// idempotent (:153-167), threadCount reports the workers (:169-171).  Here a
// worker is a host thread bound to one GPU.  A pooled call slices the rows
// exactly as the reference does -- per = rows div n, worker t owns
// [per*t, per*t + per), the last one the remainder (:118-124) -- and every
// worker runs the library's own host form (lph_*) on its slice: its rows of
// the weights and scales and the whole activations are copied to its GPU, the
// kernel runs there, and the slice of y comes straight back into the
// caller's y.  The slices are disjoint, so no gather is needed: y is host
// memory and every worker writes its own rows of it.  Each output row depends
// only on its own weight row, so the result is the single-GPU bits.
//
// The per-call forms (par*(..., threads), parallel.nim:186-418) use one pool
// of every visible GPU, created on first use and kept for the process
// (threads are not created per call here: a GPU call is microseconds).  Their
// shard count follows shardCount (:45-53): min(threads, rows div 64), at
// least 1, with threads <= 0 meaning every GPU; one shard runs the serial
// host form on the calling thread's current device.  The pooled forms fall
// back to the serial form when the pool has one worker or the rows are fewer
// than 2 * 64 (:358-360), as the reference does.
#include <condition_variable>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

#include "lp_internal.h"

namespace {

constexpr int64_t kMinRowsPerThread = 64;  // parallel.nim:42

}  // namespace

struct lph_pool {
  std::vector<int> devices;
  std::vector<std::thread> threads;
  std::mutex mu;
  std::condition_variable has_work, all_done;
  std::function<int(int)> job;
  std::vector<int> status;
  int64_t generation = 0;
  int pending = 0;
  bool stopping = false;

  void worker_loop(int id) {
    int64_t seen = 0;
    for (;;) {
      std::function<int(int)> fn;
      {
        std::unique_lock<std::mutex> lk(mu);
        has_work.wait(lk, [&] { return generation != seen || stopping; });
        if (stopping) return;
        seen = generation;
        fn = job;
      }
      int st = lp::cuda_status(cudaSetDevice(devices[id]));
      if (st == LP_OK) st = fn(id);
      std::lock_guard<std::mutex> lk(mu);
      status[id] = st;
      if (--pending == 0) all_done.notify_all();
    }
  }

  // Runs fn(worker) on every worker; blocks; the first failing status.
  int dispatch(std::function<int(int)> fn) {
    std::unique_lock<std::mutex> lk(mu);
    job = std::move(fn);
    pending = static_cast<int>(threads.size());
    for (int& s : status) s = LP_OK;
    ++generation;
    has_work.notify_all();
    all_done.wait(lk, [&] { return pending == 0; });
    for (int s : status)
      if (s != LP_OK) return s;
    return LP_OK;
  }
};

namespace {

int visible_devices() {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

int make_pool(lph_pool** out, int threads) {
  *out = nullptr;
  const int ndev = visible_devices();
  if (ndev <= 0) return LP_ERR_NO_DEVICE;
  const int nw = std::max(1, std::min(threads > 0 ? threads : ndev, ndev));
  lph_pool* p = new lph_pool;
  for (int i = 0; i < nw; ++i) p->devices.push_back(i);
  p->status.assign(nw, LP_OK);
  for (int i = 0; i < nw; ++i) p->threads.emplace_back([p, i] { p->worker_loop(i); });
  *out = p;
  return LP_OK;
}

void stop_pool(lph_pool* p) {
  {
    std::lock_guard<std::mutex> lk(p->mu);
    p->stopping = true;
  }
  p->has_work.notify_all();
  for (std::thread& t : p->threads) t.join();
  delete p;
}

// The pool of every visible GPU behind the per-call forms.
lph_pool* default_pool(int* status) {
  static std::mutex mu;
  static lph_pool* pool = nullptr;
  std::lock_guard<std::mutex> lk(mu);
  *status = LP_OK;
  if (!pool) *status = make_pool(&pool, 0);
  return pool;
}

// Row range of worker t of n over m rows (parallel.nim:118-124, 230-250).
inline void slice_of(int64_t m, int n, int t, int64_t* b, int64_t* e) {
  const int64_t per = m / n;
  *b = per * t;
  *e = (t == n - 1) ? m : *b + per;
}

// shardCount (parallel.nim:45-53), capped at the GPUs a pool has.
inline int shard_count(int64_t rows, int threads, int workers) {
  const int64_t want = threads > 0 ? threads : workers;
  return static_cast<int>(std::max<int64_t>(
      1, std::min<int64_t>(std::min<int64_t>(want, workers), rows / kMinRowsPerThread)));
}

// Runs serial(b, e) -- the host form over rows [b, e) -- on `nt` workers of
// `pool`; nt <= 1 runs it on the calling thread.
int run_sharded(lph_pool* pool, int nt, int64_t rows, const std::function<int(int64_t, int64_t)>& serial) {
  if (nt <= 1 || !pool) return serial(0, rows);
  return pool->dispatch([&](int t) -> int {
    if (t >= nt) return LP_OK;
    int64_t b, e;
    slice_of(rows, nt, t, &b, &e);
    return e > b ? serial(b, e) : LP_OK;
  });
}

// Shape checks of the whole call (the serial entry point in validate-only
// mode) before anything is sliced.
#define LPP_PRECHECK(call)                 \
  do {                                     \
    lp::set_validate_only(true);           \
    const int pre_ = (call);               \
    lp::set_validate_only(false);          \
    if (pre_ != LP_OK) return pre_;        \
  } while (0)

}  // namespace

extern "C" {

int lph_pool_init(lph_pool_t* pool, int threads) {
  if (!pool) return LP_ERR_ARG;
  return make_pool(pool, threads);
}

int lph_pool_shutdown(lph_pool_t* pool) {
  if (!pool || !*pool) return LP_OK;  // idempotent (parallel.nim:153-167)
  stop_pool(*pool);
  *pool = nullptr;
  return LP_OK;
}

int lph_pool_thread_count(lph_pool_t pool) {
  return pool ? static_cast<int>(pool->threads.size()) : 0;
}

// ------------------------------------------------------- pooled forms --
// parDequantGemvQ8 / parDequantGemvI4Q8 (parallel.nim:346-374): rows = y_len,
// k = xq_len; a row holds k / wpe weight elements and k / gs scales.
#define LPH_POOL_Q8(NAME, SERIAL, DEVFN, WT, WPE)                                                        \
  int NAME(lph_pool_t pool, const WT* w, int64_t w_len, const float* ws, int64_t ws_len,         \
           int64_t gs, const int8_t* xq, int64_t xq_len, const float* xs, int64_t xs_len,        \
           float* y, int64_t y_len) {                                                            \
    if (!pool) return LP_ERR_ARG;                                                                 \
    LPP_PRECHECK(DEVFN(w, w_len, ws, ws_len, gs, xq, xq_len, xs, xs_len, y, y_len, nullptr));    \
    const int64_t rows = y_len;                                                                   \
    const int nt = (pool->threads.size() <= 1 || rows < 2 * kMinRowsPerThread)                   \
                       ? 1 : static_cast<int>(pool->threads.size());                              \
    const int64_t wr = xq_len / (WPE), sr = gs > 0 ? xq_len / gs : 0;                            \
    return run_sharded(pool, nt, rows, [&](int64_t b, int64_t e) {                               \
      return SERIAL(w + b * wr, (e - b) * wr, ws + b * sr, (e - b) * sr, gs, xq, xq_len, xs,     \
                    xs_len, y + b, e - b);                                                        \
    });                                                                                           \
  }

LPH_POOL_Q8(lph_pool_dequant_gemv_q8, lph_dequant_gemv_q8, lp_dequant_gemv_q8, int8_t, 1)
LPH_POOL_Q8(lph_pool_dequant_gemv_i4q8, lph_dequant_gemv_i4q8, lp_dequant_gemv_i4q8, uint8_t, 2)

// parDequantGemmQ8 / parDequantGemmI4Q8 (parallel.nim:420-474): rows =
// y_len / n, k = xq_len / n; y is rows x n row-major.
#define LPH_POOL_GEMM(NAME, SERIAL, DEVFN, WT, WPE)                                                      \
  int NAME(lph_pool_t pool, const WT* w, int64_t w_len, const float* ws, int64_t ws_len,         \
           int64_t gs, const int8_t* xq, int64_t xq_len, const float* xs, int64_t xs_len,        \
           int64_t n, float* y, int64_t y_len) {                                                 \
    if (!pool) return LP_ERR_ARG;                                                                 \
    LPP_PRECHECK(DEVFN(w, w_len, ws, ws_len, gs, xq, xq_len, xs, xs_len, n, y, y_len, nullptr)); \
    const int64_t rows = y_len / n, k = xq_len / n;                                              \
    const int nt = (pool->threads.size() <= 1 || rows < 2 * kMinRowsPerThread)                   \
                       ? 1 : static_cast<int>(pool->threads.size());                              \
    const int64_t wr = k / (WPE), sr = gs > 0 ? k / gs : 0;                                      \
    return run_sharded(pool, nt, rows, [&](int64_t b, int64_t e) {                               \
      return SERIAL(w + b * wr, (e - b) * wr, ws + b * sr, (e - b) * sr, gs, xq, xq_len, xs,     \
                    xs_len, n, y + b * n, (e - b) * n);                                           \
    });                                                                                           \
  }

LPH_POOL_GEMM(lph_pool_dequant_gemm_q8, lph_dequant_gemm_q8, lp_dequant_gemm_q8, int8_t, 1)
LPH_POOL_GEMM(lph_pool_dequant_gemm_i4q8, lph_dequant_gemm_i4q8, lp_dequant_gemm_i4q8, uint8_t, 2)

// ---------------------------------------------------- per-call forms --
// par*(..., threads) (parallel.nim:186-418) over the pool of every GPU.
#define LPH_PAR_GROUP_F32(NAME, SERIAL, DEVFN, WT, WPE)                                                  \
  int NAME(const WT* w, int64_t w_len, const float* sc, int64_t sc_len, int64_t gs,              \
           const float* x, int64_t x_len, float* y, int64_t y_len, int threads) {                \
    LPP_PRECHECK(DEVFN(w, w_len, sc, sc_len, gs, x, x_len, y, y_len, nullptr));                  \
    int st = LP_OK;                                                                               \
    lph_pool* pool = default_pool(&st);                                                           \
    if (st != LP_OK) return st;                                                                   \
    const int64_t rows = y_len, wr = x_len / (WPE), sr = gs > 0 ? x_len / gs : 0;                \
    const int nt = shard_count(rows, threads, static_cast<int>(pool->threads.size()));           \
    return run_sharded(pool, nt, rows, [&](int64_t b, int64_t e) {                               \
      return SERIAL(w + b * wr, (e - b) * wr, sc + b * sr, (e - b) * sr, gs, x, x_len, y + b,    \
                    e - b);                                                                       \
    });                                                                                           \
  }

LPH_PAR_GROUP_F32(lph_par_dequant_gemv, lph_dequant_gemv, lp_dequant_gemv, int8_t, 1)
LPH_PAR_GROUP_F32(lph_par_dequant_gemv_i4, lph_dequant_gemv_i4, lp_dequant_gemv_i4, uint8_t, 2)
LPH_PAR_GROUP_F32(lph_par_dequant_gemv_f4, lph_dequant_gemv_f4, lp_dequant_gemv_f4, uint8_t, 2)

#define LPH_PAR_BLOCKS_F32(NAME, SERIAL, DEVFN, BB)                                                      \
  int NAME(const void* w, int64_t w_len, int64_t bpr, const float* x, int64_t x_len, float* y,   \
           int64_t y_len, int threads) {                                                         \
    LPP_PRECHECK(DEVFN(w, w_len, bpr, x, x_len, y, y_len, nullptr));                             \
    int st = LP_OK;                                                                               \
    lph_pool* pool = default_pool(&st);                                                           \
    if (st != LP_OK) return st;                                                                   \
    const int64_t rows = y_len;                                                                   \
    const int nt = shard_count(rows, threads, static_cast<int>(pool->threads.size()));           \
    const uint8_t* wb = static_cast<const uint8_t*>(w);                                          \
    return run_sharded(pool, nt, rows, [&](int64_t b, int64_t e) {                               \
      return SERIAL(wb + b * bpr * (BB), (e - b) * bpr, bpr, x, x_len, y + b, e - b);            \
    });                                                                                           \
  }

LPH_PAR_BLOCKS_F32(lph_par_dequant_gemv_q8_0, lph_dequant_gemv_q8_0, lp_dequant_gemv_q8_0, 34)
LPH_PAR_BLOCKS_F32(lph_par_dequant_gemv_q4_0, lph_dequant_gemv_q4_0, lp_dequant_gemv_q4_0, 18)

#define LPH_PAR_Q8(NAME, SERIAL, DEVFN, WT, WPE)                                                         \
  int NAME(const WT* w, int64_t w_len, const float* ws, int64_t ws_len, int64_t gs,              \
           const int8_t* xq, int64_t xq_len, const float* xs, int64_t xs_len, float* y,          \
           int64_t y_len, int threads) {                                                         \
    LPP_PRECHECK(DEVFN(w, w_len, ws, ws_len, gs, xq, xq_len, xs, xs_len, y, y_len, nullptr));    \
    int st = LP_OK;                                                                               \
    lph_pool* pool = default_pool(&st);                                                           \
    if (st != LP_OK) return st;                                                                   \
    const int64_t rows = y_len, wr = xq_len / (WPE), sr = gs > 0 ? xq_len / gs : 0;              \
    const int nt = shard_count(rows, threads, static_cast<int>(pool->threads.size()));           \
    return run_sharded(pool, nt, rows, [&](int64_t b, int64_t e) {                               \
      return SERIAL(w + b * wr, (e - b) * wr, ws + b * sr, (e - b) * sr, gs, xq, xq_len, xs,     \
                    xs_len, y + b, e - b);                                                        \
    });                                                                                           \
  }

LPH_PAR_Q8(lph_par_dequant_gemv_q8, lph_dequant_gemv_q8, lp_dequant_gemv_q8, int8_t, 1)
LPH_PAR_Q8(lph_par_dequant_gemv_i4q8, lph_dequant_gemv_i4q8, lp_dequant_gemv_i4q8, uint8_t, 2)

}  // extern "C"
