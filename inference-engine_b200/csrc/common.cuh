// Shared helpers for libie_tpq.so: error state, element conversions, bounded
// waits and the internal launch interfaces between the translation units.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include "../../include/ie_tpq.h"

namespace ie {

// ---- host error state ------------------------------------------------------
int set_error(int code, const char* fmt, ...);
const char* last_error();

#define IE_CUDA_TRY(expr)                                                       \
  do {                                                                          \
    cudaError_t _e = (expr);                                                    \
    if (_e != cudaSuccess)                                                      \
      return ::ie::set_error(IE_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,         \
                             cudaGetErrorString(_e), __FILE__, __LINE__);        \
  } while (0)

#define IE_CHECK(cond, ...)                                                     \
  do {                                                                          \
    if (!(cond)) return ::ie::set_error(IE_ERR_INVALID, __VA_ARGS__);          \
  } while (0)

inline int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error(IE_ERR_CUDA, "launch of %s failed: %s", what, cudaGetErrorString(e));
  return IE_OK;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// ---- element conversion ------------------------------------------------------
// ---------------------------------------------------------------------------
// round_to_float_format (ie/quant/formats.py:74-79)
// ---------------------------------------------------------------------------
// The reference clips to +-max, takes frexp's mantissa m in [0.5, 1), rounds
// m * 2^mb half-to-even and rescales: the value keeps mb significant bits.
// Rounding an IEEE float to its top `sig` significant bits is an integer add
// on its bit pattern: add just under half an ulp of the kept field plus the
// kept field's lowest bit (ties to even), then clear the dropped bits; a
// carry out of the mantissa correctly bumps the exponent.
struct FloatFmt {
  int mantissa_bits;
  float max_value;
  float flush_below;  // min_normal * 2^-mantissa_bits
};

__device__ __forceinline__ float round_to_format(float x, FloatFmt f) {
  x = fminf(fmaxf(x, -f.max_value), f.max_value);
  const int drop = 23 - (f.mantissa_bits - 1);
  uint32_t u = __float_as_uint(x);
  const uint32_t lsb = (u >> drop) & 1u;
  u += ((1u << (drop - 1)) - 1u) + lsb;
  u &= ~((1u << drop) - 1u);
  float out = __uint_as_float(u);
  out = fminf(fmaxf(out, -f.max_value), f.max_value);
  return fabsf(out) < f.flush_below ? 0.0f : out;
}

template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ __half from_f32<__half>(float v) {
  return __float2half_rn(v);
}

// ---- memory-model helpers for peer flags ---------------------------------------
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits until *flag >= want (flags carry monotonically increasing epochs).
// Gives up after `limit_ns` of wall time, records IE_ERR_TIMEOUT in *status and
// returns false; the caller then skips the dependent work and exits normally.
__device__ __forceinline__ bool bounded_wait_geq(const uint32_t* flag, uint32_t want,
                                                 uint64_t limit_ns, uint32_t* status) {
  if (ld_acquire_sys(flag) >= want) return true;
  const uint64_t start = globaltimer_ns();
  uint32_t polls = 0;
  while (true) {
    if (ld_acquire_sys(flag) >= want) return true;
    if (((++polls) & 63u) == 0u) {
      if (globaltimer_ns() - start > limit_ns) {
        atomicMax(status, (uint32_t)IE_ERR_TIMEOUT);
        return false;
      }
      // a peer that already timed out will never arrive: stop early too
      if (*(volatile uint32_t*)status != 0u) return false;
    }
    __nanosleep(64);
  }
}

// ---- one-shot all-reduce context passed by value into fused kernels -----------------
// The epoch that pairs pushes with waits lives in device memory: every fused
// kernel reads it at start (epoch = *epoch_dev + 1, landing parity = epoch & 1)
// and the last CTA to finish stores it back.  Host code never tracks it, so a
// captured CUDA graph that replays the same launches still advances it.
constexpr int kMaxWorld = 8;
struct ReduceCtx {
  float* landing[kMaxWorld];   // every rank's landing buffer base (parity 0)
  uint32_t* flags[kMaxWorld];  // every rank's flag table [tile][kMaxWorld]
  uint32_t* status;            // this rank's status word
  uint32_t* epoch_dev;         // this rank's epoch counter
  uint32_t* done;              // this rank's CTA completion counter
  uint64_t timeout_ns;
  int64_t parity_stride;       // floats between the two landing parities
  int64_t slot_floats;         // floats per source-rank slot in a landing buffer
  int32_t rank;
  int32_t world;
};

__device__ __forceinline__ uint32_t reduce_epoch(const ReduceCtx& rc) {
  return *(volatile uint32_t*)rc.epoch_dev + 1u;
}
__device__ __forceinline__ float* landing_slot(const ReduceCtx& rc, int dst, uint32_t epoch) {
  return rc.landing[dst] + (int64_t)(epoch & 1u) * rc.parity_stride;
}
// Called by every CTA once at the end (after its last __syncthreads): the last
// CTA publishes the new epoch and resets the completion counter.  No fence is
// needed: every CTA read the epoch at its start, before it counted itself
// here, and the next call reads it only after this kernel has completed.
__device__ __forceinline__ void reduce_finish(const ReduceCtx& rc, uint32_t epoch) {
  if (threadIdx.x == 0) {
    if (atomicAdd(rc.done, 1u) == gridDim.x - 1) {
      *(volatile uint32_t*)rc.epoch_dev = epoch;
      *(volatile uint32_t*)rc.done = 0u;
    }
  }
}

// ---- internal launchers (defined in the .cu files) ---------------------------------
int validate_qweight(const ie_qweight& w);
int launch_qlinear_gemv(const ie_qlinear_args& a, const ReduceCtx* rc, int max_ctas,
                        cudaStream_t s);
int64_t gemv_tiles(const ie_qlinear_args& a);
int gemv_resident_ctas(const ie_qlinear_args& a, int* out);
// tcgen05 tensor-core path (qgemm_sm100.cu)
bool tc_usable(const ie_qlinear_args& a);
size_t tc_workspace_bytes(const ie_qlinear_args& a);
int64_t tc_tiles(const ie_qlinear_args& a);
int launch_qlinear_tc(const ie_qlinear_args& a, const ReduceCtx* rc, cudaStream_t s);
uint32_t tc_read_status(bool clear);
// The tensor-core call with its split-K scratch in the library's static device
// array instead of a caller workspace (ie_qlinear_noalloc); allocates nothing.
int launch_qlinear_tc_static(const ie_qlinear_args& a, cudaStream_t s);
// Fills rc for a collective call of comm c after checking its limits.
int comm_context(ie_comm* c, ReduceCtx* rc, int64_t tiles, int64_t floats_per_rank);

}  // namespace ie
