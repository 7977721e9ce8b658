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
// The gather has two forms.  By default every rank also maps every other
// rank's exchange buffer (CUDA IPC over NVLink; the handles travel over the
// pool's own NCCL communicator at creation): one small kernel stores this
// rank's slice into every peer's buffer, each value with the gather's number
// in the same 8-byte word, and reads the peers' slices out of its own buffer
// as their words arrive (bounded waits).  That is one launch
// of a few microseconds where an NCCL call costs ~12 us of latency.  The NCCL
// group is the fallback (lp_pool_set_p2p(pool, 0), outputs larger than the
// exchange buffer, or a box where the mapping is not possible on every rank).
//
// NCCL is loaded at pool creation (dlopen), so the library itself loads and
// runs on machines without NCCL; only the pool calls report LP_ERR_NCCL.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "lp_device.cuh"
#include "lp_internal.h"

namespace {
constexpr int kMaxP2pRanks = lp::kMaxPushRanks;
constexpr int64_t kXchgFloats = lp::kXchgWords;      // values per half
constexpr int64_t kXchgBytes = 2 * kXchgFloats * 8;  // two halves of 8-byte words
struct PeerBufs {
  uint8_t* p[kMaxP2pRanks];
};
// A gathered vector made of up to kMaxParts regions, each m rows of per_row
// floats at element offset off, its rows sliced over the ranks.
constexpr int kMaxParts = lp::kMaxGatherParts;
struct GatherParts {
  int64_t off[kMaxParts], m[kMaxParts], prow[kMaxParts];
  int send[kMaxParts];  // 1: the receive kernel also stores this rank's rows of the part
  int n;
};
using lp::RecvSegs;
}  // namespace

struct lp_pool {
  ncclComm_t comm;
  int nranks, rank, device;
  int p2p;         // 1: gathers through the exchange buffers
  int p2p_ready;   // the exchange was mapped on every rank at creation
  uint8_t* xbuf;   // this rank's exchange buffer: two halves of 8-byte words
  uint32_t* state; // [0] gathers finished, [1] CTAs finished in the current one
  PeerBufs peers;  // every rank's exchange buffer as mapped here
  lp::PushCtx* push;  // device copies of peers/state for the GEMVs' own stores:
  lp::PushCtx* pull;  // push form, and pull form (large gathers; see gather_parts)
  // gather group (lp_pool_group_begin/end): pooled calls whose outputs are
  // parts of one vector push into it and the group receives once
  bool grp;
  float* grp_y;
  int64_t grp_len;
  GatherParts grp_parts;
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
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
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
    LP_SYM(all_gather, "ncclAllGather");
    LP_SYM(error_string, "ncclGetErrorString");
#undef LP_SYM
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.group_start &&
             api.group_end && api.broadcast && api.all_gather && api.error_string;
  });
  return api;
}

int nccl_status(ncclResult_t r) {
  if (r == ncclSuccess) return LP_OK;
  lp::note_text(nccl().error_string ? nccl().error_string(r) : "NCCL error");
  return LP_ERR_NCCL;
}

// The stream of a receive or NCCL gather: the GEMVs queued in this thread's
// open batch (lp_batch_begin) launch first -- they push what is received.
inline cudaStream_t S(lp_stream_t s) {
  if (lp::batch_open()) lp::batch_flush_keep();
  return static_cast<cudaStream_t>(s);
}
inline cudaStream_t SG(lp_stream_t s) { return static_cast<cudaStream_t>(s); }

__host__ __device__ inline void rows_of(int64_t m, int nranks, int rank, int64_t* b, int64_t* e) {
  const int64_t per = m / nranks;
  *b = per * rank;
  *e = (rank == nranks - 1) ? m : *b + per;
}

// ------------------------------------------------- NVLink exchange gather
// Every value travels as one naturally aligned 8-byte word (gather number <<
// 32 | value bits), written whole; the receiver polls each word until it
// carries this gather's number.  Push form: the owner stores the word into
// every other rank's exchange buffer and each receiver reads its own buffer.
// Pull form (large gathers, see kPullFloats): the owner stores the word once,
// into its own buffer, and each receiver reads the owners' buffers over NVLink
// (every buffer is mapped into every rank).  No fences or counters: a
// system-scope fence costs microseconds here.
__device__ __forceinline__ void st_word(uint64_t* a, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_word(const uint64_t* a) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
  return v;
}

// Gather number e (1, 2, ...) uses exchange half e & 1, so a rank one gather
// ahead writes the other half while its peers still read this one (two ahead
// is impossible: finishing a gather needs every peer's words of that gather,
// and a peer sends them only after finishing the previous one, its reads
// included).  This holds for both forms and for gathers of mixed forms.  e is kept on
// the device (state[0]) so CUDA-graph replays count too; all ranks make the
// same gathers, so they agree on it.  Waits are bounded (error word on
// timeout).
// send == 0: this rank's words were already published by the GEMV that made
// its slice (the fused pooled form); only receive.  The kernel is launched
// with programmatic stream serialization and releases its dependents at
// once, so the next kernel (typically the next GEMV) can stage its weights
// while this gather runs; every kernel of this library launched that way
// waits for its grid dependency before it reads activations or writes
// outputs.  The gather itself
// waits for the kernel before it (the GEMV that made this rank's slice) to
// complete before it reads the gather count: that GEMV had waited for the
// previous gather in turn, so the count is final, and this gather completes
// only after its GEMV has.
__global__ void __launch_bounds__(256) k_gather_p2p(float* y, const __grid_constant__ GatherParts parts,
                                                   const __grid_constant__ RecvSegs segs,
                                                   int nranks, int rank, PeerBufs peers,
                                                   uint32_t* state, int pull) {
  __shared__ uint32_t s_e;
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int64_t C = gridDim.x;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (tid == 0) s_e = reinterpret_cast<volatile uint32_t*>(state)[0] + 1u;
  __syncthreads();
  const uint32_t e = s_e;
  const uint64_t tag = static_cast<uint64_t>(e) << 32;
  const int64_t half = (e & 1u) * kXchgFloats;
  for (int pi = 0; pi < parts.n; ++pi) {
    if (!parts.send[pi]) continue;
    int64_t b, en;
    rows_of(parts.m[pi], nranks, rank, &b, &en);
    const int64_t off = parts.off[pi] + b * parts.prow[pi], len = (en - b) * parts.prow[pi];
    const int64_t chunk = (len + C - 1) / C;
    const int64_t lo = min(len, blockIdx.x * chunk), hi = min(len, lo + chunk);
    for (int64_t i = lo + tid; i < hi; i += nthr) {
      const uint64_t w = tag | __float_as_uint(y[off + i]);
      if (pull) {
        st_word(reinterpret_cast<uint64_t*>(peers.p[rank]) + half + off + i, w);
      } else {
        for (int q = 0; q < nranks; ++q)
          if (q != rank) st_word(reinterpret_cast<uint64_t*>(peers.p[q]) + half + off + i, w);
      }
    }
  }
  bool ok = true;
  const uint64_t t0 = lp::global_ns();
  // The segments laid end to end, split evenly over the CTAs; each thread
  // keeps eight words in flight across segment boundaries (one wait for
  // the whole vector rather than one per part and peer).
  const int64_t total = segs.start[segs.n];
  const int64_t per = (total + C - 1) / C;
  const int64_t lo = min(total, blockIdx.x * per), hi = min(total, lo + per);
  int sg = 0;  // the segment of index lo + tid, advanced as the index grows
  {
    int a = 0, z = segs.n;  // last segment whose start <= lo + tid
    const int64_t i = lo + tid;
    while (z - a > 1) {
      const int mid = (a + z) >> 1;
      if (segs.start[mid] <= i) a = mid; else z = mid;
    }
    sg = a;
  }
  for (int64_t i0 = lo + tid; i0 < hi && ok; i0 += 8 * nthr) {
    uint64_t w[8];
    int64_t at[8];
    const uint64_t* from[8];  // the word in its owner's exchange buffer
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int64_t i = i0 + k * nthr;
      at[k] = -1;
      w[k] = 0;
      from[k] = nullptr;
      if (i < hi) {
        while (sg + 1 < segs.n && segs.start[sg + 1] <= i) ++sg;
        at[k] = segs.off[sg] + (i - segs.start[sg]);
        from[k] = reinterpret_cast<const uint64_t*>(peers.p[pull ? segs.src[sg] : rank]) + half +
                  at[k];
        w[k] = ld_word(from[k]);
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (at[k] < 0 || !ok) continue;
      for (uint32_t n = 1; (w[k] >> 32) != e; ++n) {
        if ((n & 255u) == 0 && lp::global_ns() - t0 > lp::kWaitLimitNs) {
          lp::raise_error(LP_ERR_TIMEOUT);
          ok = false;
          break;
        }
        __nanosleep(64);  // leave the issue slots to the GEMV on this SM
        w[k] = ld_word(from[k]);
      }
      if (ok) y[at[k]] = __uint_as_float(static_cast<uint32_t>(w[k]));
    }
  }
  // the last CTA to finish publishes e as the finished gather count
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(state + 1, 1u) == static_cast<uint32_t>(C) - 1) {
      state[1] = 0;
      __threadfence();
      atomicExch(state, e);
    }
  }
}

// A gather of at least kPullFloats values (a whole decode step in one group)
// takes the pull form: its GEMVs publish each output with one local store and
// the receive reads the other ranks' buffers.  Smaller ones take the push
// form.  Measured on 2 GPUs: the config-4 sweep in one group gains 6 % with
// pull (0.91 against 1.62 us of exchange per layer); a group per layer loses
// 18 % (each receive waits on remote reads).  The choice depends on the
// group's length only, so every rank makes the same one.
constexpr int64_t kPullFloats = int64_t{1} << 18;

// Every other rank's rows of every part, in part order, then rank order.
void build_segs(const lp_pool* p, const GatherParts& parts, RecvSegs& segs) {
  segs.n = 0;
  segs.start[0] = 0;
  for (int i = 0; i < parts.n; ++i)
    for (int q = 0; q < p->nranks; ++q) {
      if (q == p->rank) continue;
      int64_t b, e;
      rows_of(parts.m[i], p->nranks, q, &b, &e);
      if (e == b) continue;
      segs.off[segs.n] = parts.off[i] + b * parts.prow[i];
      segs.src[segs.n] = q;
      segs.start[segs.n + 1] = segs.start[segs.n] + (e - b) * parts.prow[i];
      ++segs.n;
    }
}

int gather_parts(lp_pool* p, float* y, const GatherParts& parts, cudaStream_t st, int pull) {
  static thread_local RecvSegs segs;
  build_segs(p, parts, segs);
  // CTAs enough for ~2048 received words each, at most two per SM (all
  // resident at once: a sending CTA waits only after its own stores)
  const int64_t recv = segs.start[segs.n];
  const int grid = static_cast<int>(
      std::max<int64_t>(1, std::min<int64_t>(2 * lp::device_info().sm_count, (recv + 2047) / 2048)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return lp::cuda_status(cudaLaunchKernelEx(&cfg, k_gather_p2p, y, parts, segs, p->nranks,
                                            p->rank, p->peers, p->state, pull));
}

int gather_p2p(lp_pool* p, float* y, int64_t m, int64_t per_row, cudaStream_t st, int send) {
  GatherParts parts{};
  parts.n = 1;
  parts.off[0] = 0;
  parts.m[0] = m;
  parts.prow[0] = per_row;
  parts.send[0] = send;
  return gather_parts(p, y, parts, st, 0);
}

// y[0, m*per_row) from every rank's slice of rows.
int gather(lp_pool* p, float* y, int64_t m, int64_t per_row, cudaStream_t st) {
  if (p->nranks == 1 || m == 0) return LP_OK;
  if (p->p2p && m * per_row <= kXchgFloats) return gather_p2p(p, y, m, per_row, st, 1);
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

// Maps every rank's exchange buffer into this process.  All ranks take part
// (two NCCL all-gathers); the exchange is used only when every rank mapped
// every peer and every rank has its own GPU.
void setup_p2p(lp_pool* p) {
  p->p2p = p->p2p_ready = 0;
  p->xbuf = nullptr;
  p->state = nullptr;
  p->push = nullptr;
  p->pull = nullptr;
  std::memset(&p->peers, 0, sizeof(p->peers));
  if (p->nranks < 2) return;
  const NcclApi& api = nccl();
  struct Card {
    cudaIpcMemHandle_t h;
    char bus[32];
    int ok;
  };
  Card mine;
  std::memset(&mine, 0, sizeof(mine));
  bool ok = p->nranks <= kMaxP2pRanks;
  ok = ok && cudaMalloc(&p->xbuf, kXchgBytes) == cudaSuccess;
  ok = ok && cudaMemset(p->xbuf, 0, kXchgBytes) == cudaSuccess;
  ok = ok && cudaMalloc(&p->state, 4 * sizeof(uint32_t)) == cudaSuccess;
  ok = ok && cudaMemset(p->state, 0, 4 * sizeof(uint32_t)) == cudaSuccess;
  ok = ok && cudaIpcGetMemHandle(&mine.h, p->xbuf) == cudaSuccess;
  ok = ok && cudaDeviceGetPCIBusId(mine.bus, sizeof(mine.bus), p->device) == cudaSuccess;
  mine.ok = ok ? 1 : 0;
  cudaGetLastError();
  // every rank reaches both all-gathers, whatever happened above
  Card* dev = nullptr;
  Card* all = new Card[p->nranks];
  cudaStream_t st = nullptr;
  bool xok = cudaMalloc(&dev, sizeof(Card) * (p->nranks + 1)) == cudaSuccess &&
             cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) == cudaSuccess &&
             cudaMemcpy(dev + p->nranks, &mine, sizeof(Card), cudaMemcpyHostToDevice) == cudaSuccess;
  xok = xok && api.all_gather(dev + p->nranks, dev, sizeof(Card), ncclChar, p->comm, st) == ncclSuccess;
  xok = xok && cudaStreamSynchronize(st) == cudaSuccess &&
        cudaMemcpy(all, dev, sizeof(Card) * p->nranks, cudaMemcpyDeviceToHost) == cudaSuccess;
  bool mapped = xok;
  for (int q = 0; q < p->nranks && mapped; ++q) {
    mapped = all[q].ok != 0;
    for (int r = 0; r < q && mapped; ++r) mapped = std::strcmp(all[q].bus, all[r].bus) != 0;
  }
  for (int q = 0; q < p->nranks && mapped; ++q) {
    if (q == p->rank) {
      p->peers.p[q] = p->xbuf;
      continue;
    }
    void* ptr = nullptr;
    mapped = cudaIpcOpenMemHandle(&ptr, all[q].h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
    p->peers.p[q] = static_cast<uint8_t*>(ptr);
  }
  cudaGetLastError();
  // agree: the exchange is on only if every rank mapped every peer
  int agree = mapped ? 1 : 0;
  int* dflag = nullptr;
  bool aok = xok && cudaMalloc(&dflag, sizeof(int) * (p->nranks + 1)) == cudaSuccess &&
             cudaMemcpy(dflag + p->nranks, &agree, sizeof(int), cudaMemcpyHostToDevice) == cudaSuccess &&
             api.all_gather(dflag + p->nranks, dflag, sizeof(int), ncclChar, p->comm, st) == ncclSuccess &&
             cudaStreamSynchronize(st) == cudaSuccess;
  int all_ok = aok ? 1 : 0;
  if (aok) {
    int* flags = new int[p->nranks];
    if (cudaMemcpy(flags, dflag, sizeof(int) * p->nranks, cudaMemcpyDeviceToHost) != cudaSuccess)
      all_ok = 0;
    for (int q = 0; q < p->nranks && all_ok; ++q) all_ok = flags[q] != 0;
    delete[] flags;
  }
  if (dflag) cudaFree(dflag);
  if (dev) cudaFree(dev);
  if (st) cudaStreamDestroy(st);
  delete[] all;
  cudaGetLastError();
  if (all_ok) {
    lp::PushCtx h;
    std::memset(&h, 0, sizeof(h));
    for (int q = 0; q < p->nranks; ++q) h.peers[q] = p->peers.p[q];
    h.state = p->state;
    h.nranks = p->nranks;
    h.rank = p->rank;
    lp::PushCtx hh[2] = {h, h};
    hh[1].pull = 1;
    if (cudaMalloc(&p->push, sizeof(hh)) != cudaSuccess ||
        cudaMemcpy(p->push, hh, sizeof(hh), cudaMemcpyHostToDevice) != cudaSuccess) {
      if (p->push) cudaFree(p->push);
      p->push = nullptr;
    }
    p->pull = p->push ? p->push + 1 : nullptr;
    cudaGetLastError();
  }
  p->p2p = all_ok;
  p->p2p_ready = all_ok;
}

void teardown_p2p(lp_pool* p) {
  cudaDeviceSynchronize();
  for (int q = 0; q < kMaxP2pRanks; ++q)
    if (p->peers.p[q] && q != p->rank) cudaIpcCloseMemHandle(p->peers.p[q]);
  if (p->xbuf) cudaFree(p->xbuf);
  if (p->state) cudaFree(p->state);
  if (p->push) cudaFree(p->push);  // both contexts (one allocation)
  p->push = nullptr;
  p->pull = nullptr;
  std::memset(&p->peers, 0, sizeof(p->peers));
  p->xbuf = nullptr;
  p->state = nullptr;
  p->p2p = p->p2p_ready = 0;
  cudaGetLastError();
}

}  // namespace

namespace lp {
// The error word of this translation unit (see lp_device.cuh).
unsigned int take_error_pool() {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return LP_ERR_CUDA;
  if (v) {
    const unsigned int z = 0;
    cudaMemcpyToSymbol(g_device_error, &z, sizeof(z));
  }
  return v;
}
}  // namespace lp

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
  lp_pool* p = new lp_pool{};
  p->nranks = nranks;
  p->rank = rank;
  p->device = device;
  r = nccl_status(api.comm_init_rank(&p->comm, nranks, u, rank));
  if (r) {
    delete p;
    return r;
  }
  setup_p2p(p);
  *pool = p;
  return LP_OK;
}

int lp_pool_destroy(lp_pool_t pool) {
  if (!pool) return LP_OK;  // idempotent, like shutdown (parallel.nim:153-167)
  int r = LP_OK;
  cudaSetDevice(pool->device);
  teardown_p2p(pool);
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

int lp_pool_set_p2p(lp_pool_t pool, int enable) {
  if (!pool) return LP_ERR_ARG;
  if (!enable) {
    pool->p2p = 0;
    return LP_OK;
  }
  if (!pool->p2p_ready) return LP_ERR_UNSUPPORTED;
  pool->p2p = 1;
  return LP_OK;
}

int lp_pool_get_p2p(lp_pool_t pool, int* enabled) {
  if (!pool || !enabled) return LP_ERR_ARG;
  *enabled = pool->p2p;
  return LP_OK;
}

int lp_pool_group_begin(lp_pool_t pool, float* y, int64_t y_len) {
  if (!pool || y_len < 0 || (y_len > 0 && !y) || pool->grp) return LP_ERR_ARG;
  if (pool->p2p && y_len > kXchgFloats) return LP_ERR_UNSUPPORTED;  // beyond the exchange buffer
  pool->grp = true;
  pool->grp_y = y;
  pool->grp_len = y_len;
  pool->grp_parts.n = 0;
  return LP_OK;
}

int lp_pool_group_end(lp_pool_t pool, lp_stream_t stream) {
  if (!pool || !pool->grp) return LP_ERR_ARG;
  pool->grp = false;
  if (pool->grp_parts.n == 0 || pool->nranks < 2) return LP_OK;
  int r = lp::cuda_status(cudaSetDevice(pool->device));
  if (r) return r;
  const int pull = pool->grp_len >= kPullFloats;
  const GatherParts& gp = pool->grp_parts;
  bool published = pool->p2p != 0;
  for (int i = 0; i < gp.n && published; ++i) published = gp.send[i] == 0;
  // A group whose rows were all published by the GEMVs' folds, with GEMVs of
  // it still queued in an open batch: the receive rides at the end of that
  // batch's launch instead of in a receive kernel after it.
  if (published && lp::batch_takes_recv(pull ? pool->pull : pool->push, SG(stream))) {
    static thread_local RecvSegs segs;
    build_segs(pool, gp, segs);
    bool taken = false;
    r = lp::batch_flush_recv(pool->grp_y, segs, &taken);
    if (r != LP_OK || taken) {
      pool->grp_parts.n = 0;
      return r;
    }
  }
  r = gather_parts(pool, pool->grp_y, gp, S(stream), pull);
  pool->grp_parts.n = 0;
  return r;
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
  const int64_t yl_len_ = (e_ - b_) * (per_row);                      \
  /* inside a gather group: this output is a part of the group's vector */ \
  const int64_t goff_ = pool->grp ? static_cast<int64_t>(y - pool->grp_y) : 0; \
  const bool ingrp_ = pool->grp && pool->p2p && pool->push && goff_ >= 0 &&   \
                      goff_ + (ylen) <= pool->grp_len && pool->grp_parts.n < kMaxParts; \
  /* an open group on the exchange takes every pooled call as a part */ \
  if (pool->grp && pool->p2p && pool->push && !ingrp_) return LP_ERR_ARG; \
  const bool fuse_ = pool->p2p && pool->push &&                        \
                     (ingrp_ ? pool->grp_len : m_ * (per_row)) <= kXchgFloats; \
  lp::g_push = !fuse_ ? nullptr                                       \
               : (ingrp_ && pool->grp_len >= kPullFloats) ? pool->pull : pool->push; \
  lp::g_push_off = goff_ * ingrp_ + b_ * (per_row);                   \
  lp::g_pushed = false;

// The local GEMV stored its outputs into the other ranks already (fused
// form): only receive.  Otherwise (a kernel without the push, or no
// exchange) the whole gather.  The choice depends on shapes only, so every
// rank makes the same one.
#define LP_POOL_POST(per_row)                                         \
  const bool pushed_ = lp::g_pushed;                                  \
  lp::g_push = nullptr;                                               \
  lp::g_pushed = false;                                               \
  if (r_) return r_;                                                  \
  if (ingrp_ && pool->nranks > 1) {                                   \
    /* received with the rest of the group at lp_pool_group_end; a   \
       kernel without the push has its rows sent there too */         \
    GatherParts& gp_ = pool->grp_parts;                               \
    gp_.off[gp_.n] = goff_;                                           \
    gp_.m[gp_.n] = m_;                                                \
    gp_.prow[gp_.n] = per_row;                                     \
    gp_.send[gp_.n] = pushed_ ? 0 : 1;                                \
    ++gp_.n;                                                          \
    return LP_OK;                                                     \
  }                                                                   \
  if (pushed_ && pool->nranks > 1)                                    \
    return gather_p2p(pool, y, m_, per_row, S(stream), 0);            \
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
int lp_pool_quantize_dequant_gemv_q8(lp_pool_t pool, const int8_t* wq, int64_t wq_len,
                                     const float* w_scales, int64_t w_scales_len,
                                     int64_t group_size, const float* x, int64_t x_len, float* y,
                                     int64_t y_len, lp_stream_t stream) {
  LP_POOL_PRE(y_len, 1)
  const int r_ = lp_quantize_dequant_gemv_q8(wq, wq_len, w_scales, w_scales_len, group_size, x,
                                             x_len, yl_, yl_len_, stream);
  LP_POOL_POST(1)
}
int lp_pool_quantize_dequant_gemv_i4q8(lp_pool_t pool, const uint8_t* wp, int64_t wp_len,
                                       const float* w_scales, int64_t w_scales_len,
                                       int64_t group_size, const float* x, int64_t x_len,
                                       float* y, int64_t y_len, lp_stream_t stream) {
  LP_POOL_PRE(y_len, 1)
  const int r_ = lp_quantize_dequant_gemv_i4q8(wp, wp_len, w_scales, w_scales_len, group_size,
                                               x, x_len, yl_, yl_len_, stream);
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
