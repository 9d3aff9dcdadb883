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

template <typename T> __host__ __device__ constexpr int dtype_of();
template <> __host__ __device__ constexpr int dtype_of<float>() { return IE_DT_F32; }
template <> __host__ __device__ constexpr int dtype_of<__nv_bfloat16>() { return IE_DT_BF16; }
template <> __host__ __device__ constexpr int dtype_of<__half>() { return IE_DT_F16; }

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

// ---- fused all-reduce context passed by value into the kernels ---------------------
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
  int32_t algo;                // kArOneShot or kArTwoShot (resolved on the host)
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

// ---- the two in-kernel protocols ------------------------------------------------
// One-shot (IE_AR_ONESHOT): every rank pushes each tile's f32 partial into slot
//   [rank] of every rank's landing buffer and raises flags[tile][rank] there;
//   every rank waits for all slots of every tile and sums them in rank order.
//   NVLink bytes sent per rank: (world - 1) * 4 per element.
// Two-shot (IE_AR_TWOSHOT): tile t belongs to rank t % world.  A rank pushes a
//   tile's partial to its owner only (reduce-scatter); the owner sums the slots
//   in rank order, applies bias and residual, stores its own output and pushes
//   the finished f32 values into slot [owner] of every other rank's landing
//   buffer, raising flags[t][owner] there (all-gather); the others round them
//   to the output type.  NVLink bytes sent per rank: 8 (world - 1) / world per
//   element, one more flag round trip.  The sum order is the same, so both
//   protocols give bitwise equal outputs.  Two-shot needs tiles >= world: then
//   every rank receives something from every peer in every call, which is what
//   keeps the double-buffered landing parity safe (a rank starts call e + 2
//   only after each peer has finished call e).
// A flag word (rank x, tile t, source s) carries the partial of s when x owns t
// (or in one-shot), and the finished tile when s owns t and x does not; the
// two uses never meet in one call.
constexpr int kArOneShot = 1;
constexpr int kArTwoShot = 2;

// Landing buffers that receive tile t's partial: [d0, d1).
__device__ __forceinline__ void ar_push_range(const ReduceCtx& rc, int64_t t, int& d0, int& d1) {
  if (rc.algo == kArTwoShot) {
    d0 = (int)(t % rc.world);
    d1 = d0 + 1;
  } else {
    d0 = 0;
    d1 = rc.world;
  }
}
// Raises tile t's partial flags; call after a CTA barrier that follows every
// push of the tile (st.release.sys then publishes them: the barrier orders the
// block's stores before this thread's release, and a peer's ld.acquire.sys of
// the flag sees them).
__device__ __forceinline__ void ar_publish(const ReduceCtx& rc, int64_t t, uint32_t epoch,
                                           int tid) {
  int d0, d1;
  ar_push_range(rc, t, d0, d1);
  if (tid < d1 - d0) st_release_sys(rc.flags[d0 + tid] + t * kMaxWorld + rc.rank, epoch);
}

__device__ __forceinline__ float ar_load(const void* p, int dt, int64_t i) {
  if (dt == IE_DT_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  if (dt == IE_DT_F16) return __half2float(static_cast<const __half*>(p)[i]);
  return static_cast<const float*>(p)[i];
}
__device__ __forceinline__ void ar_store(void* p, int dt, int64_t i, float v) {
  if (dt == IE_DT_BF16) static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else if (dt == IE_DT_F16) static_cast<__half*>(p)[i] = __float2half_rn(v);
  else static_cast<float*>(p)[i] = v;
}

// Where the reduced tiles go: out[m * ldo + n] = [residual[m * ldr + n] +]
// (sum + [bias[n]]) for tokens m < M and rows n < N; landing offsets are m * N + n.
struct ArOut {
  void* out;
  const void* residual;
  const float* bias;
  int64_t ldo, ldr, M, N;
  int dtype;
  bool has_bias, has_res;
};

// Finishes tile t = rows [n0, n0 + rows) x tokens [m0, m0 + cols) of a fused
// all-reduce with all kT threads of the CTA: one-shot and the two-shot owner
// wait for every rank's partial and sum them in rank order (the owner then
// pushes the finished values to the other ranks); a two-shot non-owner waits
// for the owner's values.  kPer elements per thread are loaded together, so a
// round costs one memory round trip, not one per element.  Returns false when
// a wait expired (the status word records it); every thread gets the same answer.
template <int kT, int kRows>
__device__ bool ar_finish_tile(const ReduceCtx& rc, uint32_t epoch, const ArOut& o, int64_t t,
                               int64_t n0, int64_t m0, int cols, int* s_ok) {
  static_assert((kRows & (kRows - 1)) == 0, "tile rows: a power of two");
  const int tid = threadIdx.x;
  const bool two = rc.algo == kArTwoShot;
  const int owner = two ? (int)(t % rc.world) : rc.rank;
  const bool owns = owner == rc.rank;
  if (tid == 0) *s_ok = 1;
  __syncthreads();
  if (owns) {
    if (tid < rc.world &&
        !bounded_wait_geq(rc.flags[rc.rank] + t * kMaxWorld + tid, epoch, rc.timeout_ns,
                          rc.status))
      *s_ok = 0;
  } else if (tid == 0 &&
             !bounded_wait_geq(rc.flags[rc.rank] + t * kMaxWorld + owner, epoch, rc.timeout_ns,
                               rc.status)) {
    *s_ok = 0;
  }
  __syncthreads();
  if (!*s_ok) return false;
  const float* mine = landing_slot(rc, rc.rank, epoch);
  const float* src0 = mine + (owns ? 0 : (int64_t)owner * rc.slot_floats);
  constexpr int kPer = 8;
  const int count = kRows * cols;
  // element e of the tile: row n0 + e % kRows, token m0 + e / kRows (shift and
  // mask, computed once per element); 32-bit locals keep this tail of the
  // fused kernels within their register budget
  for (int e0 = tid; e0 < count; e0 += kT * kPer) {
    int nl[kPer], ml[kPer];
    bool ok[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int e = e0 + j * kT;
      nl[j] = e & (kRows - 1);
      ml[j] = e / kRows;
      ok[j] = e < count && m0 + ml[j] < o.M && n0 + nl[j] < o.N;
    }
    auto at = [&](int j, int64_t ld) { return (m0 + ml[j]) * ld + (n0 + nl[j]); };
    float v[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) v[j] = ok[j] ? __ldcg(src0 + at(j, o.N)) : 0.0f;
    if (owns) {
      float r[kPer];
#pragma unroll
      for (int j = 0; j < kPer; ++j)
        r[j] = (o.has_res && ok[j]) ? ar_load(o.residual, o.dtype, at(j, o.ldr)) : 0.0f;
      for (int src = 1; src < rc.world; ++src) {
        const float* slot = mine + (int64_t)src * rc.slot_floats;
        float w[kPer];
#pragma unroll
        for (int j = 0; j < kPer; ++j) w[j] = ok[j] ? __ldcg(slot + at(j, o.N)) : 0.0f;
#pragma unroll
        for (int j = 0; j < kPer; ++j) v[j] += w[j];
      }
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        if (o.has_bias) v[j] += ok[j] ? o.bias[n0 + nl[j]] : 0.0f;
        if (o.has_res) v[j] = r[j] + v[j];
      }
      if (two) {
        for (int dst = 0; dst < rc.world; ++dst) {
          if (dst == rc.rank) continue;
          float* peer = landing_slot(rc, dst, epoch) + (int64_t)rc.rank * rc.slot_floats;
#pragma unroll
          for (int j = 0; j < kPer; ++j)
            if (ok[j]) peer[at(j, o.N)] = v[j];
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kPer; ++j)
      if (ok[j]) ar_store(o.out, o.dtype, at(j, o.ldo), v[j]);
  }
  __syncthreads();
  if (two && owns && tid < rc.world && tid != rc.rank)
    st_release_sys(rc.flags[tid] + t * kMaxWorld + rc.rank, epoch);
  return true;
}

// Phase 2 of a fused all-reduce over `tiles` tiles for the whole grid: a
// two-shot rank finishes the tiles it owns first (they unblock the peers),
// then copies out the rest.  tile(t, n0, m0, cols) describes tile t (kRows
// rows from n0, cols tokens from m0).
template <int kT, int kRows, typename TileFn>
__device__ void ar_finish_all(const ReduceCtx& rc, uint32_t epoch, const ArOut& o, int64_t tiles,
                              TileFn tile, int* s_ok) {
  const bool two = rc.algo == kArTwoShot;
  for (int pass = 0; pass < (two ? 2 : 1); ++pass) {
    // pass 0 of two-shot: owned tiles rank, rank + world, ...; otherwise all
    // tiles (pass 1 skips the owned ones)
    const int64_t count = (two && pass == 0) ? (tiles - rc.rank + rc.world - 1) / rc.world : tiles;
    for (int64_t i = blockIdx.x; i < count; i += gridDim.x) {
      const int64_t t = (two && pass == 0) ? rc.rank + i * rc.world : i;
      if (two && pass == 1 && t % rc.world == rc.rank) continue;
      int64_t n0, m0;
      int cols;
      tile(t, n0, m0, cols);
      if (!ar_finish_tile<kT, kRows>(rc, epoch, o, t, n0, m0, cols, s_ok)) return;
    }
  }
}

// ---- internal launchers (defined in the .cu files) ---------------------------------
int validate_qweight(const ie_qweight& w);
int launch_qlinear_gemv(const ie_qlinear_args& a, const ReduceCtx* rc, int max_ctas,
                        cudaStream_t s);
int64_t gemv_tiles(const ie_qlinear_args& a);
// the decode GEMV serves this call (at most two tokens, x' of the whole K in
// shared memory; it also folds the RMS norm); without a fused all-reduce
bool gemv_decode_ok(const ie_qlinear_args& a);
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
// Fills rc for a collective call of comm c after checking its limits, with
// the protocol for `algo` (IE_AR_*) resolved for this call's tile count and size.
int comm_context(ie_comm* c, ReduceCtx* rc, int64_t tiles, int64_t floats_per_rank,
                 int32_t algo);

}  // namespace ie
