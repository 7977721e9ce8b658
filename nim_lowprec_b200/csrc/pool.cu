// pool.cu -- LpPool's row-sharded forms (parallel.nim:82-474) across the GPUs
// of one box: one process per GPU, each holding a contiguous row slice of the
// weights, an NCCL gather of y over NVLink.
//
// The slicing rule is the reference's (parallel.nim:118-124): per = m div P,
// rank r owns rows [per*r, per*r + per) and the last rank takes the
// remainder.  Every output row depends only on its own weight row, so a
// sharded call gives exactly the serial bits (test_parallel.nim).  The local
// slice runs through the ordinary device entry points; the slices then meet
// with one NCCL group of per-rank broadcasts (an all-gather with unequal
// counts), in place in y, on the caller's stream.
//
// NCCL is loaded at pool creation (dlopen), so the library itself loads and
// runs on machines without NCCL; only the pool calls report LP_ERR_NCCL.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "lp_internal.h"

struct lp_pool {
  ncclComm_t comm;
  int nranks, rank, device;
};

namespace {

struct NcclApi {
  bool ok = false;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  ncclResult_t (*broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
#define LP_SYM(field, name) api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, name))
    LP_SYM(get_unique_id, "ncclGetUniqueId");
    LP_SYM(comm_init_rank, "ncclCommInitRank");
    LP_SYM(comm_destroy, "ncclCommDestroy");
    LP_SYM(group_start, "ncclGroupStart");
    LP_SYM(group_end, "ncclGroupEnd");
    LP_SYM(broadcast, "ncclBroadcast");
    LP_SYM(error_string, "ncclGetErrorString");
#undef LP_SYM
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.group_start &&
             api.group_end && api.broadcast && api.error_string;
  });
  return api;
}

int nccl_status(ncclResult_t r) {
  if (r == ncclSuccess) return LP_OK;
  lp::note_text(nccl().error_string ? nccl().error_string(r) : "NCCL error");
  return LP_ERR_NCCL;
}

inline cudaStream_t S(lp_stream_t s) { return static_cast<cudaStream_t>(s); }

void rows_of(int64_t m, int nranks, int rank, int64_t* b, int64_t* e) {
  const int64_t per = m / nranks;
  *b = per * rank;
  *e = (rank == nranks - 1) ? m : *b + per;
}

// y[0, m*per_row) from every rank's slice of rows.
int gather(lp_pool* p, float* y, int64_t m, int64_t per_row, cudaStream_t st) {
  const NcclApi& api = nccl();
  int r = nccl_status(api.group_start());
  if (r) return r;
  int first = LP_OK;
  for (int q = 0; q < p->nranks; ++q) {
    int64_t b, e;
    rows_of(m, p->nranks, q, &b, &e);
    if (e <= b) continue;
    float* at = y + b * per_row;
    r = nccl_status(api.broadcast(at, at, static_cast<size_t>((e - b) * per_row), ncclFloat32, q,
                                  p->comm, st));
    if (r && !first) first = r;
  }
  r = nccl_status(api.group_end());
  return first ? first : r;
}

}  // namespace

extern "C" {

int lp_pool_rows(int64_t m, int nranks, int rank, int64_t* begin, int64_t* end) {
  if (m < 0 || nranks < 1 || rank < 0 || rank >= nranks || !begin || !end) return LP_ERR_ARG;
  rows_of(m, nranks, rank, begin, end);
  return LP_OK;
}

int lp_pool_unique_id(uint8_t* id) {
  if (!id) return LP_ERR_ARG;
  const NcclApi& api = nccl();
  if (!api.ok) {
    lp::note_text("libnccl.so.2 could not be loaded");
    return LP_ERR_NCCL;
  }
  ncclUniqueId u;
  const int r = nccl_status(api.get_unique_id(&u));
  if (r) return r;
  std::memcpy(id, u.internal, NCCL_UNIQUE_ID_BYTES);
  return LP_OK;
}

int lp_pool_init(lp_pool_t* pool, const uint8_t* id, int nranks, int rank, int device) {
  if (!pool || !id || nranks < 1 || rank < 0 || rank >= nranks || device < 0) return LP_ERR_ARG;
  *pool = nullptr;
  const NcclApi& api = nccl();
  if (!api.ok) {
    lp::note_text("libnccl.so.2 could not be loaded");
    return LP_ERR_NCCL;
  }
  int r = lp::cuda_status(cudaSetDevice(device));
  if (r) return r;
  ncclUniqueId u;
  std::memcpy(u.internal, id, NCCL_UNIQUE_ID_BYTES);
  lp_pool* p = new lp_pool{nullptr, nranks, rank, device};
  r = nccl_status(api.comm_init_rank(&p->comm, nranks, u, rank));
  if (r) {
    delete p;
    return r;
  }
  *pool = p;
  return LP_OK;
}

int lp_pool_destroy(lp_pool_t pool) {
  if (!pool) return LP_OK;  // idempotent, like shutdown (parallel.nim:153-167)
  int r = LP_OK;
  if (pool->comm) r = nccl_status(nccl().comm_destroy(pool->comm));
  delete pool;
  return r;
}

int lp_pool_size(lp_pool_t pool, int* nranks, int* rank) {
  if (!pool || !nranks || !rank) return LP_ERR_ARG;
  *nranks = pool->nranks;
  *rank = pool->rank;
  return LP_OK;
}

int lp_pool_gather_rows(lp_pool_t pool, float* y, int64_t m, int64_t per_row, lp_stream_t stream) {
  if (!pool || m < 0 || per_row < 1 || (m > 0 && !y)) return LP_ERR_ARG;
  int r = lp::cuda_status(cudaSetDevice(pool->device));
  if (r) return r;
  return gather(pool, y, m, per_row, S(stream));
}

// Pooled forms: weights and weight scales are this rank's row slice, the
// activations are whole, y is whole (every rank ends with all of it).
#define LP_POOL_PRE(ylen, per_row)                                    \
  if (!pool) return LP_ERR_ARG;                                       \
  if ((ylen) < 0 || (per_row) < 1) return LP_ERR_SHAPE;               \
  {                                                                   \
    const int r0 = lp::cuda_status(cudaSetDevice(pool->device));      \
    if (r0) return r0;                                                \
  }                                                                   \
  const int64_t m_ = (ylen) / (per_row);                              \
  if (m_ * (per_row) != (ylen)) return LP_ERR_SHAPE;                  \
  int64_t b_, e_;                                                     \
  rows_of(m_, pool->nranks, pool->rank, &b_, &e_);                    \
  float* yl_ = y + b_ * (per_row);                                    \
  const int64_t yl_len_ = (e_ - b_) * (per_row);

#define LP_POOL_POST(per_row)                                         \
  if (r_) return r_;                                                  \
  return gather(pool, y, m_, per_row, S(stream));

int lp_pool_dequant_gemv(lp_pool_t pool, const int8_t* wq, int64_t wq_len, const float* scales,
                         int64_t scales_len, int64_t group_size, const float* x, int64_t x_len,
                         float* y, int64_t y_len, lp_stream_t stream) {
  LP_POOL_PRE(y_len, 1)
  const int r_ = lp_dequant_gemv(wq, wq_len, scales, scales_len, group_size, x, x_len, yl_,
                                 yl_len_, stream);
  LP_POOL_POST(1)
}
int lp_pool_dequant_gemv_i4(lp_pool_t pool, const uint8_t* wp, int64_t wp_len,
                            const float* scales, int64_t scales_len, int64_t group_size,
                            const float* x, int64_t x_len, float* y, int64_t y_len,
                            lp_stream_t stream) {
  LP_POOL_PRE(y_len, 1)
  const int r_ = lp_dequant_gemv_i4(wp, wp_len, scales, scales_len, group_size, x, x_len, yl_,
                                    yl_len_, stream);
  LP_POOL_POST(1)
}
int lp_pool_dequant_gemv_f4(lp_pool_t pool, const uint8_t* wp, int64_t wp_len,
                            const float* scales, int64_t scales_len, int64_t group_size,
                            const float* x, int64_t x_len, float* y, int64_t y_len,
                            lp_stream_t stream) {
  LP_POOL_PRE(y_len, 1)
  const int r_ = lp_dequant_gemv_f4(wp, wp_len, scales, scales_len, group_size, x, x_len, yl_,
                                    yl_len_, stream);
  LP_POOL_POST(1)
}
int lp_pool_dequant_gemv_q8_0(lp_pool_t pool, const void* w, int64_t w_len, int64_t bpr,
                              const float* x, int64_t x_len, float* y, int64_t y_len,
                              lp_stream_t stream) {
  LP_POOL_PRE(y_len, 1)
  const int r_ = lp_dequant_gemv_q8_0(w, w_len, bpr, x, x_len, yl_, yl_len_, stream);
  LP_POOL_POST(1)
}
int lp_pool_dequant_gemv_q4_0(lp_pool_t pool, const void* w, int64_t w_len, int64_t bpr,
                              const float* x, int64_t x_len, float* y, int64_t y_len,
                              lp_stream_t stream) {
  LP_POOL_PRE(y_len, 1)
  const int r_ = lp_dequant_gemv_q4_0(w, w_len, bpr, x, x_len, yl_, yl_len_, stream);
  LP_POOL_POST(1)
}
int lp_pool_dequant_gemv_q8(lp_pool_t pool, const int8_t* wq, int64_t wq_len,
                            const float* w_scales, int64_t w_scales_len, int64_t group_size,
                            const int8_t* xq, int64_t xq_len, const float* x_scales,
                            int64_t x_scales_len, float* y, int64_t y_len, lp_stream_t stream) {
  LP_POOL_PRE(y_len, 1)
  const int r_ = lp_dequant_gemv_q8(wq, wq_len, w_scales, w_scales_len, group_size, xq, xq_len,
                                    x_scales, x_scales_len, yl_, yl_len_, stream);
  LP_POOL_POST(1)
}
int lp_pool_dequant_gemv_i4q8(lp_pool_t pool, const uint8_t* wp, int64_t wp_len,
                              const float* w_scales, int64_t w_scales_len, int64_t group_size,
                              const int8_t* xq, int64_t xq_len, const float* x_scales,
                              int64_t x_scales_len, float* y, int64_t y_len, lp_stream_t stream) {
  LP_POOL_PRE(y_len, 1)
  const int r_ = lp_dequant_gemv_i4q8(wp, wp_len, w_scales, w_scales_len, group_size, xq,
                                      xq_len, x_scales, x_scales_len, yl_, yl_len_, stream);
  LP_POOL_POST(1)
}
int lp_pool_dequant_gemm_q8(lp_pool_t pool, const int8_t* wq, int64_t wq_len,
                            const float* w_scales, int64_t w_scales_len, int64_t group_size,
                            const int8_t* xq, int64_t xq_len, const float* x_scales,
                            int64_t x_scales_len, int64_t n, float* y, int64_t y_len,
                            lp_stream_t stream) {
  if (n < 1) return LP_ERR_SHAPE;
  LP_POOL_PRE(y_len, n)
  const int r_ = lp_dequant_gemm_q8(wq, wq_len, w_scales, w_scales_len, group_size, xq, xq_len,
                                    x_scales, x_scales_len, n, yl_, yl_len_, stream);
  LP_POOL_POST(n)
}
int lp_pool_dequant_gemm_i4q8(lp_pool_t pool, const uint8_t* wp, int64_t wp_len,
                              const float* w_scales, int64_t w_scales_len, int64_t group_size,
                              const int8_t* xq, int64_t xq_len, const float* x_scales,
                              int64_t x_scales_len, int64_t n, float* y, int64_t y_len,
                              lp_stream_t stream) {
  if (n < 1) return LP_ERR_SHAPE;
  LP_POOL_PRE(y_len, n)
  const int r_ = lp_dequant_gemm_i4q8(wp, wp_len, w_scales, w_scales_len, group_size, xq,
                                      xq_len, x_scales, x_scales_len, n, yl_, yl_len_, stream);
  LP_POOL_POST(n)
}

}  // extern "C"
