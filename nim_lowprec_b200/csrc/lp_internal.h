// lp_internal.h -- host-side plumbing shared by the library's .cu files.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "lowprec_cuda.h"

namespace lp {

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  int ordinal = -1;
  int sm_count = 0;
  int max_smem_optin = 0;
  int smem_per_sm = 0;        // shared memory of one SM
  int smem_reserved = 0;      // shared memory the runtime reserves per block
  int cc_major = 0, cc_minor = 0;
};

// Properties of the current device (queried once per device, cached).
const DeviceInfo& device_info();

struct GemvParams;

// LpPool over NVLink: each rank's exchange buffer holds two halves of
// kXchgWords 8-byte words (value bits | gather number << 32), mapped into
// every rank.  A pooled GEMV given a PushCtx stores its outputs straight into
// every other rank's buffer from its fold (pool.cu then only receives).
constexpr int kMaxPushRanks = 8;
constexpr int64_t kXchgWords = int64_t{1} << 21;
struct PushCtx {
  uint8_t* peers[kMaxPushRanks];  // every rank's exchange buffer as mapped here
  uint32_t* state;                // this rank's finished-gather count (state[0])
  int nranks, rank;
  // 1: publish each output in this rank's own buffer, the receivers read it
  // over NVLink (large gathers); 0: store it into every other rank's buffer
  int pull;
};
// Set by the pool around its local call (this thread only): the device copy of
// the context and the slice's offset in y; launch_gemv reports in g_pushed
// whether its kernel takes the push.
extern thread_local const PushCtx* g_push;
extern thread_local int64_t g_push_off;
extern thread_local bool g_pushed;
struct FmtI8;
struct FmtI4;
struct FmtF4;
struct FmtQ8_0;
struct FmtQ4_0;
struct FmtI8F;
struct FmtI4F;
struct FmtF4F;
struct FmtQ8_0F;
struct FmtQ4_0F;
struct FmtQ4_KF;
struct FmtQ6_KF;
struct FmtQ8FromF32;
struct FmtI4Q8FromF32;
struct FmtQ8;
struct FmtI4Q8;
struct FmtQ8_0Q8;
struct FmtQ4_0Q8;
struct FmtQ8Cols;
struct FmtI4Q8Cols;

template <class Fmt>
int launch_gemv(GemvParams p, cudaStream_t st);

// Batched GEMV launches (gemv.cu): GEMVs this thread makes on the stream of
// its open batch are recorded and launched together at the next flush.
// Every other launch of the library flushes first, so stream order holds.
bool batch_open();
int batch_flush();
// What a rank receives in a gather over the exchange: every other rank's rows
// of every part, as segments of the vector laid end to end (start: prefix
// sums of their lengths; off: each segment's first element in y and in the
// exchange; src: the rank whose buffer holds it).
constexpr int kMaxGatherParts = 64;  // a 32-layer sweep's two GEMVs per layer
constexpr int kMaxRecvSegs = kMaxGatherParts * (kMaxPushRanks - 1);
struct RecvSegs {
  int64_t start[kMaxRecvSegs + 1];
  int64_t off[kMaxRecvSegs];
  int src[kMaxRecvSegs];
  int n;
};
// A gather whose rows were all published by queued GEMVs with context
// `push` can ride in the open batch's launch on `st`:
// batch_flush_recv launches the queue with a receive warp per CTA reading
// segs into y, and says in *taken whether it did (not when the queue fell
// back to lone launches; the caller then launches the receive kernel).
bool batch_takes_recv(const PushCtx* push, cudaStream_t st);
int batch_flush_recv(float* y, const RecvSegs& segs, bool* taken);
void batch_flush_keep();  // a failure is returned by batch_end
int batch_begin(cudaStream_t st);
int batch_end(cudaStream_t st);

// per-step inputs from page-locked host memory (transfer.cu)
int launch_copy_in(void* dst, const void* src, int64_t bytes, cudaStream_t st);

// encoders (quant.cu)
int launch_quantize_q8_0(const float* src, int64_t n, uint8_t* blocks, int8_t* qs, float* d,
                         cudaStream_t st);
int launch_quantize_q4_0(const float* src, int64_t n, uint8_t* blocks, cudaStream_t st);
int launch_quantize_batch(const float* x, int64_t n, const float* scales, const float* zp,
                          int64_t gs, int8_t* dst, cudaStream_t st);
int launch_dequantize_batch(const int8_t* q, int64_t n, const float* scales, const float* zp,
                            int64_t gs, float* dst, cudaStream_t st);
int launch_calibrate(const float* x, int64_t n, int64_t gs, float qmax, int mx_emax, int mx,
                     float* scales, int64_t nscales, cudaStream_t st);
int launch_quantize_packed(const float* x, int64_t n, const float* scales, int64_t gs, int f4,
                           uint8_t* packed, cudaStream_t st);
int launch_dequantize_blocks(const uint8_t* blocks, int64_t nblocks, int q4, float* dst,
                             cudaStream_t st);
int launch_dequantize_kquant(const uint8_t* blocks, int64_t nblocks, int q6, float* dst,
                             cudaStream_t st);
int launch_quantize_nvfp4(const float* x, int64_t n, uint8_t* codes, uint8_t* scales,
                          float* gds_out, cudaStream_t st);
int launch_dequantize_nvfp4(const uint8_t* codes, const uint8_t* scales, float gds, int64_t n,
                            float* dst, cudaStream_t st);

// GEMM (gemm_tc.cu: tcgen05, LP_ERR_UNSUPPORTED outside its shapes; gemm.cu: CUDA cores)
int launch_gemm_tc(const void* wq, int packed_i4, const float* ws, int64_t gs, const int8_t* xq,
                   const float* xs, int64_t n, float* y, int64_t m, int64_t k, cudaStream_t st);
int launch_gemm(const uint8_t* w, int packed_i4, const float* ws, int64_t gs, const int8_t* xq,
                const float* xs, int64_t n, float* y, int64_t m, int64_t k, cudaStream_t st);
// FP4 x FP4 block-scaled tensor-core GEMMs (gemm_fp4.cu)
int launch_gemm_mxf4(const uint8_t* w, const float* ws, const uint8_t* x, const float* xs,
                     int64_t n, float* y, int64_t m, int64_t k, cudaStream_t st);
int launch_gemm_nvf4(const uint8_t* w, const uint8_t* ws, const float* gw, const uint8_t* x,
                     const uint8_t* xs, const float* gx, int64_t n, float* y, int64_t m, int64_t k,
                     cudaStream_t st);

// error words of the translation units whose kernels wait (read + clear)
unsigned int take_error_gemv();
unsigned int take_error_gemm_tc();
unsigned int take_error_pool();
unsigned int take_error_gemm_fp4();

// While on (this thread only), the lp_* entry points run their shape and
// argument checks and return without launching anything (capi.cu).
void set_validate_only(bool on);

// Records the CUDA error text for lp_last_error_detail() and maps to a status.
void note_cuda_error(cudaError_t e);
void note_text(const char* text);
const char* t_detail_ptr();
inline int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return LP_OK;
  note_cuda_error(e);
  return LP_ERR_CUDA;
}

}  // namespace lp
