// tcgen05 tensor-core quantized GEMM for sm_100a, with split-K and an optional
// one-shot all-reduce fused into the epilogue.
//
// The weight is the MMA's A operand (M = 128 output rows per tile) and the
// token batch is its N dimension (16..256), so decode batches of 16 and
// prefill batches use the same kernel.  Per CTA (320 threads, one per SM):
//
//   warp 0      TMA producer: packed weight tile [128 rows x 128 K], the
//               activation tile [BN tokens x 128 K] (bf16/f16, 128-byte
//               swizzle) and the stage's scale tables (group-128 scale/zero
//               rows, or the per-K scales) into a ring of shared-memory stages
//               (no multicast).
//   warp 1      MMA issuer: one elected thread issues tcgen05.mma
//               (kind::f16 with f16 operands, f32 accumulator in TMEM,
//               8 x K=16 per stage) and tcgen05.commit releases the stage.
//   warps 2..9  dequantize each weight stage in registers (int4 pairs widened
//               with one mask+or into the mantissas of an f16x2, zero
//               subtracted exactly, group scale applied once) into the
//               canonical SW128 K-major layout of the A ring; bf16 activation
//               tiles are converted to f16 in place (f16 keeps 11 significant
//               bits, so the dequantized weight carries at most 2^-12 relative
//               rounding, against 2^-9 for bf16); then, per work
//               unit, read the accumulator with tcgen05.ld and run the
//               epilogue (split-K reduction in split order, per-N / per-tensor
//               scale, bias, SiLU*up, residual, store or all-reduce push).
//
// Work units are (row tile, token tile, K split); CTAs loop over them.  A
// split writes its f32 partial to the caller's workspace and the last split
// to arrive (atomic ticket) sums all splits in split order, so results do not
// depend on scheduling.  Every mbarrier wait is bounded by wall time; on
// expiry the kernel records an error bit, drains its TMA copies and MMAs,
// frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace ie {
namespace tc {

constexpr int kDqWarps = 8;     // dequant + epilogue warps (two per SM sub-partition)
constexpr int kDqThreads = kDqWarps * 32;
constexpr int kThreads = 64 + kDqThreads;
constexpr int kTileN = 128;     // weight rows per tile = MMA M
constexpr int kBK = 128;        // K per stage (one int4 group)
constexpr int kMaxAStages = 4;  // dequantized A ring depth (4 for decode tiles, 2 for wide)
constexpr int kABytes = kTileN * kBK * 2;   // one A stage (f16)
constexpr uint64_t kWaitNs = 2000000000ull; // bounded mbarrier waits

enum Fmt { F_INT4G = 0, F_INT4SYM = 1, F_INT8 = 2, F_FP8 = 3 };

// error bits recorded by kernels of this file (read with ie_device_status)
__device__ uint32_t g_tc_status = 0;
constexpr uint32_t kErrWait = 1u;

struct TcParams {
  int64_t M, K, N;          // tokens, contraction, packed rows
  int axis, gate_up, epilogue, out_dtype;
  int x_bf16;               // activations arrive as bf16 and are converted to f16
  const float* scale;       // per-K [K] / [2][K], per-N [N], per-tensor [1] / [2]
  const __half* gscale;     // group-128 [K/128][N]
  const __half* gzero;
  const float* bias;
  const void* residual;
  int64_t ldr;
  void* out;
  int64_t ldo;
  int bn;                   // tokens per tile (MMA N)
  int n_tiles, m_tiles, splits, kstages;   // kstages = K / kBK
  int ns;                   // TMA ring depth
  int na;                   // A ring depth
  int w_stage_bytes;        // packed weight bytes per stage
  int t_kind;               // stage tables: 0 none, 1 group s/z f16 [128] each, 2 per-K f32
  int t_rows;               // per-K tables: 1, or 2 for gate/up pairs
  int t_stage_bytes;        // table bytes per stage (1024-aligned slot)
  float* ws;                // split-K partials [splits][M][N]
  uint32_t* counters;       // per (m_tile, n_tile) tickets, self-resetting
};

// ---------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait on an mbarrier phase; false (and an error bit) after kWaitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          const volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > kWaitNs) {
      atomicOr(&g_tc_status, kErrWait);
      return false;
    }
  }
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void named_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), version 1 for sm_100.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;                 // LBO (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;       // SBO
  d |= (uint64_t)1 << 46;                 // descriptor version
  d |= (uint64_t)2 << 61;                 // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::f16, f32 accumulator, A/B of type ab (0 f16,
// 1 bf16), both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t make_idesc(int ab, int n) {
  return (1u << 4) | ((uint32_t)ab << 7) | ((uint32_t)ab << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(kTileN >> 4) << 24);
}

// Offset of the 16-byte chunk holding K elements [8j, 8j+8) of row r inside a
// 64-wide SW128 K-major block (rows 128 bytes apart, chunks XOR-swizzled).
__device__ __forceinline__ uint32_t sw128_offset(int r, int j) {
  return (uint32_t)(r * 128 + ((j ^ (r & 7)) << 4));
}

// ---------------------------------------------------------------------------
// dequantization of one 16-byte input chunk into A-operand chunks
// ---------------------------------------------------------------------------
template <typename TA> struct AType;
template <> struct AType<__nv_bfloat16> {
  static constexpr uint32_t kMagic = 0x43004300u;   // bf16x2 (128, 128)
  static constexpr float kBias = 128.0f;
  __device__ static uint32_t pack(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ static uint32_t sub_mul(uint32_t v, uint32_t off, uint32_t s) {
    __nv_bfloat162 x = *reinterpret_cast<__nv_bfloat162*>(&v);
    __nv_bfloat162 o = *reinterpret_cast<__nv_bfloat162*>(&off);
    __nv_bfloat162 sc = *reinterpret_cast<__nv_bfloat162*>(&s);
    __nv_bfloat162 r = __hmul2(__hsub2(x, o), sc);
    return *reinterpret_cast<uint32_t*>(&r);
  }
  __device__ static uint32_t splat(float v) { return pack(v, v); }
};
template <> struct AType<__half> {
  static constexpr uint32_t kMagic = 0x64006400u;   // f16x2 (1024, 1024)
  static constexpr float kBias = 1024.0f;
  __device__ static uint32_t pack(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ static uint32_t sub_mul(uint32_t v, uint32_t off, uint32_t s) {
    __half2 x = *reinterpret_cast<__half2*>(&v);
    __half2 o = *reinterpret_cast<__half2*>(&off);
    __half2 sc = *reinterpret_cast<__half2*>(&s);
    __half2 r = __hmul2(__hsub2(x, o), sc);
    return *reinterpret_cast<uint32_t*>(&r);
  }
  __device__ static uint32_t splat(float v) { return pack(v, v); }
};

__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)(b & 0xFFu), __NV_E4M3);
  return __half2float(__half(h));
}

// Dequantize one work item (row r of the tile, 16-byte input chunk c) of the
// stage at K offset k0 into the A stage buffer `a` (two 64-wide SW128 blocks).
template <int FMT>
__device__ __forceinline__ void dequant_item(const TcParams& p, const uint8_t* wst, uint8_t* a,
                                             int r, int c, int64_t n_row, const float* tbl,
                                             uint32_t g_off, uint32_t g_scale) {
  using AT = AType<__half>;
  const int row_bytes = p.w_stage_bytes / kTileN;
  const uint4 in = *reinterpret_cast<const uint4*>(wst + r * row_bytes + c * 16);
  const uint32_t w4[4] = {in.x, in.y, in.z, in.w};
  if constexpr (FMT == F_INT4G) {
    // 32 codes: K = c*32 .. c*32+31; one A chunk (8 values) per 32-bit word
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t t = ((w4[j] >> (4 * q)) & 0x000F000Fu) | AT::kMagic;
        o[q] = AT::sub_mul(t, g_off, g_scale);
      }
      const int kk = c * 32 + 8 * j;
      uint8_t* dst = a + (kk >> 6) * (kTileN * 128) + sw128_offset(r, (kk & 63) >> 3);
      *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  } else {
    // 8 or 32 codes per chunk; value per code in f32, then paired
    constexpr int kPer = (FMT == F_INT4SYM) ? 32 : 16;
    const int kbase = c * kPer;
    const float* sk = nullptr;
    if (p.axis == IE_AXIS_K) sk = tbl + (p.t_rows == 2 ? (n_row & 1) * kBK : 0) + kbase;
#pragma unroll
    for (int j = 0; j < kPer / 8; ++j) {
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int idx = 8 * j + e;
        float q;
        if constexpr (FMT == F_INT4SYM) {
          const uint32_t word = w4[idx >> 3];
          const int pos = idx & 7;
          const int nib = (pos & 1) ? 4 + (pos >> 1) : (pos >> 1);
          q = (float)((word >> (4 * nib)) & 0xFu) - 8.0f;
        } else if constexpr (FMT == F_INT8) {
          q = (float)(int8_t)((w4[idx >> 2] >> (8 * (idx & 3))) & 0xFFu);
        } else {
          q = e4m3_to_f32(w4[idx >> 2] >> (8 * (idx & 3)));
        }
        v[e] = sk ? q * sk[idx] : q;
      }
      const int kk = kbase + 8 * j;
      uint8_t* dst = a + (kk >> 6) * (kTileN * 128) + sw128_offset(r, (kk & 63) >> 3);
      *reinterpret_cast<uint4*>(dst) = make_uint4(AT::pack(v[0], v[1]), AT::pack(v[2], v[3]),
                                                  AT::pack(v[4], v[5]), AT::pack(v[6], v[7]));
    }
  }
}

__device__ __forceinline__ void store_val(void* out, int dt, int64_t i, float v) {
  if (dt == IE_DT_BF16) static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
  else if (dt == IE_DT_F16) static_cast<__half*>(out)[i] = __float2half_rn(v);
  else static_cast<float*>(out)[i] = v;
}
__device__ __forceinline__ float load_val(const void* in, int dt, int64_t i) {
  if (dt == IE_DT_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(in)[i]);
  if (dt == IE_DT_F16) return __half2float(static_cast<const __half*>(in)[i]);
  return static_cast<const float*>(in)[i];
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
// bf16 -> f16 of one 16-byte chunk (8 values), in place.
__device__ __forceinline__ void bf16_to_f16_chunk(uint4* p) {
  uint4 v = *p;
  uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float lo = __uint_as_float(w[i] << 16);
    const float hi = __uint_as_float(w[i] & 0xFFFF0000u);
    w[i] = AType<__half>::pack(lo, hi);
  }
  *p = make_uint4(w[0], w[1], w[2], w[3]);
}

template <int FMT>
__global__ void __launch_bounds__(kThreads, 1)
qgemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_z,
                TcParams p, ReduceCtx rc, int reduce) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int ns = p.ns, na = p.na;
  const int x_stage_bytes = p.bn * kBK * 2;
  uint8_t* a_ring = smem;                                   // na x 32 KB
  uint8_t* x_ring = a_ring + na * kABytes;                  // ns x x_stage_bytes
  uint8_t* w_ring = x_ring + ns * x_stage_bytes;            // ns x w_stage_bytes
  uint8_t* t_ring = w_ring + ns * p.w_stage_bytes;          // ns x t_stage_bytes
  uint64_t* bars = reinterpret_cast<uint64_t*>(t_ring + ns * p.t_stage_bytes);
  uint64_t* full = bars;                 // [ns]  TMA landed (count 1 + tx)
  uint64_t* empty = full + ns;           // [ns]  MMA done + dequant done (count 2)
  uint64_t* afull = empty + ns;          // [na] dequant -> MMA (count 1)
  uint64_t* aempty = afull + na;         // [na] MMA -> dequant (count 1)
  uint64_t* accfull = aempty + na;       // MMA -> epilogue
  uint64_t* accempty = accfull + 1;      // epilogue -> MMA (count 1)
  uint64_t* mma_done = accempty + 1;     // final commit: all MMAs retired
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* s_ticket = const_cast<int*>(abort_flag) + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t tmem_cols = p.bn <= 32 ? 32 : (p.bn <= 64 ? 64 : (p.bn <= 128 ? 128 : 256));
  const uint32_t epoch = reduce ? reduce_epoch(rc) : 0u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 2);
    }
    for (int s = 0; s < na; ++s) {
      mbar_init(&afull[s], 1);
      mbar_init(&aempty[s], 1);
    }
    mbar_init(accfull, 1);
    mbar_init(accempty, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int units = p.n_tiles * p.m_tiles * p.splits;
  auto unit_range = [&](int u, int& nt, int& mt, int& ks0, int& ks1, int& sp) {
    nt = u % p.n_tiles;
    const int rest = u / p.n_tiles;
    mt = rest % p.m_tiles;
    sp = rest / p.m_tiles;
    const int per = (p.kstages + p.splits - 1) / p.splits;
    ks0 = sp * per;
    ks1 = min(p.kstages, ks0 + per);
  };

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      int it = 0;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        int nt, mt, ks0, ks1, sp;
        unit_range(u, nt, mt, ks0, ks1, sp);
        for (int ks = ks0; ks < ks1; ++ks, ++it) {
          const int s = it % ns;
          if (!mbar_wait(&empty[s], ((it / ns) & 1) ^ 1, abort_flag)) {
            *abort_flag = 1;
            break;
          }
          const uint32_t tbytes = p.t_kind == 1 ? 2 * kTileN * 2
                                  : (p.t_kind == 2 ? (uint32_t)(p.t_rows * kBK * 4) : 0u);
          mbar_expect_tx(&full[s], (uint32_t)(p.w_stage_bytes + x_stage_bytes) + tbytes);
          tma_load_2d(w_ring + s * p.w_stage_bytes, &tm_w, ks * (p.w_stage_bytes / kTileN),
                      nt * kTileN, &full[s]);
          uint8_t* ts = t_ring + s * p.t_stage_bytes;
          if (p.t_kind == 1) {
            tma_load_2d(ts, &tm_s, nt * kTileN, ks, &full[s]);
            tma_load_2d(ts + kTileN * 2, &tm_z, nt * kTileN, ks, &full[s]);
          } else if (p.t_kind == 2) {
            tma_load_2d(ts, &tm_s, ks * kBK, 0, &full[s]);
          }
          uint8_t* xs = x_ring + s * x_stage_bytes;
          tma_load_2d(xs, &tm_x, ks * kBK, mt * p.bn, &full[s]);
          tma_load_2d(xs + p.bn * 128, &tm_x, ks * kBK + 64, mt * p.bn, &full[s]);
        }
      }
      // drain: every issued stage's copy must have landed before exit
      const int first = it > ns ? it - ns : 0;
      for (int j = first; j < it; ++j) {
        const int s = j % ns;
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&full[s], (j / ns) & 1) && globaltimer_ns() - t0 < kWaitNs) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------
    if (lane == 0) {
      const uint32_t idesc = make_idesc(0, p.bn);   // f16 x f16 -> f32
      int it = 0, ait = 0, unit_i = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++unit_i) {
        int nt, mt, ks0, ks1, sp;
        unit_range(u, nt, mt, ks0, ks1, sp);
        if (!mbar_wait(accempty, (unit_i & 1) ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int ks = ks0; ks < ks1; ++ks, ++it, ++ait) {
          const int s = it % ns, a = ait % na;
          if (!mbar_wait(&full[s], (it / ns) & 1, abort_flag) ||
              !mbar_wait(&afull[a], (ait / na) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(a_ring + a * kABytes);
          const uint32_t x_base = smem_u32(x_ring + s * x_stage_bytes);
#pragma unroll
          for (int kb = 0; kb < 2; ++kb)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = sw128_desc(a_base + kb * (kTileN * 128) + kk * 32);
              const uint64_t bd = sw128_desc(x_base + kb * (p.bn * 128) + kk * 32);
              tc_mma(tmem, ad, bd, idesc, (ks > ks0 || kb > 0 || kk > 0) ? 1u : 0u);
            }
          tc_commit(&empty[s]);
          tc_commit(&aempty[a]);
        }
        if (!ok) break;
        tc_commit(accfull);
      }
      if (!ok) *abort_flag = 1;
      // every MMA this thread issued must finish before TMEM is released
      tc_commit(mma_done);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(mma_done, 0) && globaltimer_ns() - t0 < kWaitNs) {
      }
    }
  } else {
    // ---------------------- dequantize + epilogue (256 threads) ----------------------
    const int dt = threadIdx.x - 64;
    const int quarter = warp & 3;                 // TMEM lanes 32*quarter ..
    const int half = (warp - 2) >> 2;             // which half of the columns
    const int row = quarter * 32 + lane;          // accumulator row of this thread
    constexpr int kChunks = (FMT == F_INT4G || FMT == F_INT4SYM) ? 4 : 8;  // per row per stage
    constexpr int kItems = kTileN * kChunks / kDqThreads;                  // per thread
    int it = 0, ait = 0, unit_i = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++unit_i) {
      int nt, mt, ks0, ks1, sp;
      unit_range(u, nt, mt, ks0, ks1, sp);
      for (int ks = ks0; ks < ks1; ++ks, ++it, ++ait) {
        const int s = it % ns, a = ait % na;
        if (!mbar_wait(&full[s], (it / ns) & 1, abort_flag) ||
            !mbar_wait(&aempty[a], ((ait / na) & 1) ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        const uint8_t* wst = w_ring + s * p.w_stage_bytes;
        uint8_t* ast = a_ring + a * kABytes;
        const uint8_t* tst = t_ring + s * p.t_stage_bytes;
#pragma unroll
        for (int i = 0; i < kItems; ++i) {
          const int item = dt + i * kDqThreads;
          const int r = item / kChunks, c = item % kChunks;
          const int64_t n_row = (int64_t)nt * kTileN + r;
          uint32_t g_off = 0, g_scale = 0;
          if constexpr (FMT == F_INT4G) {
            // rows past N were zero-filled by the TMA, so s = 0 there
            const __half s_ = reinterpret_cast<const __half*>(tst)[r];
            const __half z_ = reinterpret_cast<const __half*>(tst + kTileN * 2)[r];
            const __half zb = __hadd(z_, __float2half_rn(AType<__half>::kBias));
            g_off = (uint32_t)__half_as_ushort(zb) * 0x10001u;
            g_scale = (uint32_t)__half_as_ushort(s_) * 0x10001u;
          }
          dequant_item<FMT>(p, wst, ast, r, c, n_row, reinterpret_cast<const float*>(tst),
                            g_off, g_scale);
        }
        if (p.x_bf16) {
          uint4* xs = reinterpret_cast<uint4*>(x_ring + s * x_stage_bytes);
          for (int i = dt; i < x_stage_bytes / 16; i += kDqThreads) bf16_to_f16_chunk(xs + i);
        }
        fence_proxy_async();
        named_sync(1, kDqThreads);
        if (dt == 0) {
          mbar_arrive(&afull[a]);
          mbar_arrive(&empty[s]);
        }
      }
      if (!ok) break;

      // ---- epilogue of this unit ----
      if (!mbar_wait(accfull, unit_i & 1, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int64_t n = (int64_t)nt * kTileN + row;
      const int64_t m0 = (int64_t)mt * p.bn;
      const bool split = p.splits > 1;
      float nscale = 1.0f;
      if (n < p.N) {
        if (p.axis == IE_AXIS_N) nscale = p.scale[n];
        else if (p.axis == IE_AXIS_TENSOR) nscale = p.scale[p.gate_up ? (n & 1) : 0];
      }
      // pass 1: TMEM -> registers -> (workspace | final); this warp owns the
      // columns [c_lo, c_hi) of its lane quarter
      const int c_lo = half * (p.bn / 2), c_hi = c_lo + p.bn / 2;
      for (int c0 = c_lo; c0 < c_hi; c0 += 8) {
        float v[8];
        tmem_ld8(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0, v);
        if (split) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int64_t m = m0 + c0 + j;
            if (m < p.M && n < p.N) p.ws[((int64_t)sp * p.M + m) * p.N + n] = v[j];
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            // finalize token m0+c0+j for row n
            const int64_t m = m0 + c0 + j;
            float val = v[j] * nscale;
            if (p.epilogue & IE_EPI_SILU_MUL) {
              if (p.epilogue & IE_EPI_BIAS) val += (n < p.N) ? p.bias[n] : 0.0f;
              const float partner = __shfl_xor_sync(0xffffffffu, val, 1);
              if ((lane & 1) == 0 && m < p.M && n + 1 < p.N) {
                float o = (val / (1.0f + __expf(-val))) * partner;
                const int64_t jcol = n >> 1;
                if (p.epilogue & IE_EPI_RESIDUAL) o += load_val(p.residual, p.out_dtype, m * p.ldr + jcol);
                store_val(p.out, p.out_dtype, m * p.ldo + jcol, o);
              }
            } else if (m < p.M && n < p.N) {
              if (reduce) {
                for (int dst = 0; dst < rc.world; ++dst)
                  landing_slot(rc, dst, epoch)[rc.rank * rc.slot_floats + m * p.N + n] = val;
              } else {
                if (p.epilogue & IE_EPI_BIAS) val += p.bias[n];
                if (p.epilogue & IE_EPI_RESIDUAL)
                  val = load_val(p.residual, p.out_dtype, m * p.ldr + n) + val;
                store_val(p.out, p.out_dtype, m * p.ldo + n, val);
              }
            }
          }
        }
      }
      tc_fence_before();
      named_sync(1, kDqThreads);
      if (dt == 0) mbar_arrive(accempty);

      const int tile_id = mt * p.n_tiles + nt;
      bool finalize_here = !split;
      if (split) {
        // ticket: the last split to arrive sums all splits in split order
        __threadfence();
        named_sync(1, kDqThreads);
        if (dt == 0) {
          const uint32_t t = atomicAdd(&p.counters[tile_id], 1u);
          *s_ticket = (t == (uint32_t)(p.splits - 1)) ? 1 : 0;
        }
        named_sync(1, kDqThreads);
        finalize_here = *s_ticket != 0;
        if (finalize_here) {
          __threadfence();
          for (int j = c_lo; j < c_hi; ++j) {
            const int64_t m = m0 + j;
            float acc = 0.0f;
            if (m < p.M && n < p.N) {
              acc = __ldcg(p.ws + m * p.N + n);
              for (int q = 1; q < p.splits; ++q)
                acc += __ldcg(p.ws + ((int64_t)q * p.M + m) * p.N + n);
            }
            float val = acc * nscale;
            if (p.epilogue & IE_EPI_SILU_MUL) {
              if (p.epilogue & IE_EPI_BIAS) val += (n < p.N) ? p.bias[n] : 0.0f;
              const float partner = __shfl_xor_sync(0xffffffffu, val, 1);
              if ((lane & 1) == 0 && m < p.M && n + 1 < p.N) {
                float o = (val / (1.0f + __expf(-val))) * partner;
                const int64_t jcol = n >> 1;
                if (p.epilogue & IE_EPI_RESIDUAL) o += load_val(p.residual, p.out_dtype, m * p.ldr + jcol);
                store_val(p.out, p.out_dtype, m * p.ldo + jcol, o);
              }
            } else if (m < p.M && n < p.N) {
              if (reduce) {
                for (int dst = 0; dst < rc.world; ++dst)
                  landing_slot(rc, dst, epoch)[rc.rank * rc.slot_floats + m * p.N + n] = val;
              } else {
                if (p.epilogue & IE_EPI_BIAS) val += p.bias[n];
                if (p.epilogue & IE_EPI_RESIDUAL)
                  val = load_val(p.residual, p.out_dtype, m * p.ldr + n) + val;
                store_val(p.out, p.out_dtype, m * p.ldo + n, val);
              }
            }
          }
          if (dt == 0) p.counters[tile_id] = 0u;
        }
      }
      if (reduce && finalize_here) {
        named_sync(1, kDqThreads);
        if (dt < rc.world) {
          __threadfence_system();
          st_release_sys(rc.flags[dt] + (int64_t)tile_id * kMaxWorld + rc.rank, epoch);
        }
      }
    }
    if (!ok) *abort_flag = 1;
  }

  // ------------------------------ teardown ------------------------------
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(tmem_cols)
                 : "memory");
  }

  if (reduce) {
    // ---- all-reduce phase 2: wait for every rank's tile, sum in rank order ----
    __shared__ int s_ok;
    const float* mine = landing_slot(rc, rc.rank, epoch);
    const int tiles = p.n_tiles * p.m_tiles;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      if (threadIdx.x == 0) s_ok = 1;
      __syncthreads();
      if (threadIdx.x < rc.world &&
          !bounded_wait_geq(rc.flags[rc.rank] + (int64_t)t * kMaxWorld + threadIdx.x, epoch,
                            rc.timeout_ns, rc.status))
        s_ok = 0;
      __syncthreads();
      if (!s_ok) break;
      const int nt = t % p.n_tiles, mt = t / p.n_tiles;
      for (int e = threadIdx.x; e < kTileN * p.bn; e += kThreads) {
        const int64_t n = (int64_t)nt * kTileN + (e % kTileN);
        const int64_t m = (int64_t)mt * p.bn + (e / kTileN);
        if (m >= p.M || n >= p.N) continue;
        const int64_t off = m * p.N + n;
        float v = mine[off];
        for (int src = 1; src < rc.world; ++src) v += mine[src * rc.slot_floats + off];
        if (p.epilogue & IE_EPI_BIAS) v += p.bias[n];
        if (p.epilogue & IE_EPI_RESIDUAL) v = load_val(p.residual, p.out_dtype, m * p.ldr + n) + v;
        store_val(p.out, p.out_dtype, m * p.ldo + n, v);
      }
      __syncthreads();
    }
    __syncthreads();
    reduce_finish(rc, epoch);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                              const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                              const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}

struct Plan {
  int fmt = 0, bn = 16, m_tiles = 1, n_tiles = 1, splits = 1, kstages = 1, ns = 2, na = 2;
  int w_stage_bytes = 0;
  int t_kind = 0, t_rows = 0, t_stage_bytes = 0;
  size_t smem = 0;
  size_t ws_bytes = 0;       // counters + partials
  size_t counters_bytes = 0;
};

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

int fmt_of(const ie_qweight& w) {
  if (w.format == IE_FMT_INT8) return F_INT8;
  if (w.format == IE_FMT_FP8_E4M3) return F_FP8;
  return w.axis == IE_AXIS_GROUP128 ? F_INT4G : F_INT4SYM;
}

// Tile/split choice: BN covers the tokens (<= 256 per tile); splits of K raise
// the unit count toward a whole number of waves over the SMs, discounted by the
// extra f32 partial traffic they cost relative to the weight bytes.
Plan make_plan(const ie_qlinear_args& a, bool allow_split) {
  Plan pl;
  pl.fmt = fmt_of(a.w);
  const int64_t M = a.m;
  pl.bn = (int)std::min<int64_t>(256, ((M + 15) / 16) * 16);
  pl.m_tiles = (int)((M + pl.bn - 1) / pl.bn);
  pl.n_tiles = (int)((a.w.n + kTileN - 1) / kTileN);
  pl.kstages = (int)(a.w.k / kBK);
  const int row_stage = (pl.fmt == F_INT4G || pl.fmt == F_INT4SYM) ? kBK / 2 : kBK;
  pl.w_stage_bytes = row_stage * kTileN;
  const int sms = sm_count();
  const double wbytes = (double)a.w.n * a.w.k * (row_stage / (double)kBK);
  double best = -1.0;
  const int tiles = pl.n_tiles * pl.m_tiles;
  for (int s = 1; s <= (allow_split ? 16 : 1); ++s) {
    if (s > 1 && pl.kstages < 2 * s) break;
    // every split must own at least one stage: (s-1) * ceil(kstages/s) < kstages
    const int per = (pl.kstages + s - 1) / s;
    if ((s - 1) * per >= pl.kstages) continue;
    const int units = tiles * s;
    const int waves = (units + sms - 1) / sms;
    const double eff = (double)units / ((double)waves * sms);
    const double extra = s > 1 ? (2.0 * s * (double)M * a.w.n * 4.0) / wbytes : 0.0;
    const double score = eff / (1.0 + extra);
    if (score > best + 1e-9) {
      best = score;
      pl.splits = s;
    }
  }
  if (a.w.axis == IE_AXIS_GROUP128) {
    pl.t_kind = 1;
    pl.t_stage_bytes = 1024;
  } else if (a.w.axis == IE_AXIS_K) {
    pl.t_kind = 2;
    pl.t_rows = a.w.gate_up ? 2 : 1;
    pl.t_stage_bytes = 1024;
  }
  const size_t x_stage = (size_t)pl.bn * kBK * 2;
  const size_t budget = 220 * 1024;
  pl.na = pl.bn <= 64 ? kMaxAStages : 2;
  const size_t fixed = (size_t)pl.na * kABytes + 1024 + 256;
  const size_t per = x_stage + pl.w_stage_bytes + pl.t_stage_bytes;
  pl.ns = (int)std::min<size_t>(8, (budget - fixed) / per);
  if (pl.ns < 2) pl.ns = 2;
  pl.smem = fixed + (size_t)pl.ns * per + 8 * (2 * pl.ns + 2 * pl.na + 3) + 16;
  if (pl.splits > 1) {
    pl.counters_bytes = (((size_t)tiles * 4) + 255) / 256 * 256;
    pl.ws_bytes = pl.counters_bytes + (size_t)pl.splits * M * a.w.n * 4;
  }
  return pl;
}

bool tc_eligible(const ie_qlinear_args& a) {
  if (a.act_dtype != IE_DT_BF16 && a.act_dtype != IE_DT_F16) return false;
  if (a.w.k % kBK) return false;
  if (((uintptr_t)a.x & 15) || ((a.ldx * 2) & 15)) return false;
  if (((uintptr_t)a.w.codes & 15)) return false;
  if (((uintptr_t)a.w.scale & 15)) return false;
  if (a.w.axis == IE_AXIS_GROUP128 && ((a.w.n % 8) || ((uintptr_t)a.w.zero & 15))) return false;
  return encode_fn() != nullptr;
}

template <int FMT>
int launch_typed(const ie_qlinear_args& a, const Plan& pl, const CUtensorMap& tw,
                 const CUtensorMap& tx, const CUtensorMap& ts, const CUtensorMap& tz,
                 const TcParams& prm, const ReduceCtx* rc, cudaStream_t s) {
  auto kern = qgemm_tc_kernel<FMT>;
  IE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)pl.smem));
  const int units = pl.n_tiles * pl.m_tiles * pl.splits;
  const int grid = std::min(units, sm_count());
  ReduceCtx none{};
  kern<<<grid, kThreads, pl.smem, s>>>(tw, tx, ts, tz, prm, rc ? *rc : none, rc ? 1 : 0);
  return launch_status("qgemm_tc_kernel");
}

}  // namespace tc

size_t tc_workspace_bytes(const ie_qlinear_args& a) {
  if (!tc::tc_eligible(a)) return 0;
  return tc::make_plan(a, true).ws_bytes;
}

bool tc_usable(const ie_qlinear_args& a) { return tc::tc_eligible(a); }

int64_t tc_tiles(const ie_qlinear_args& a) {
  const tc::Plan pl = tc::make_plan(a, a.workspace != nullptr);
  return (int64_t)pl.n_tiles * pl.m_tiles;
}

int launch_qlinear_tc(const ie_qlinear_args& a, const ReduceCtx* rc, cudaStream_t s) {
  using namespace tc;
  IE_CHECK(tc_eligible(a), "qlinear: the tensor-core path needs bf16/f16 activations, K %% 128 "
                           "== 0, 16-byte aligned rows and the driver's TMA encoder");
  Plan pl = make_plan(a, true);
  if (pl.splits > 1 && (!a.workspace || a.workspace_bytes < pl.ws_bytes)) pl = make_plan(a, false);
  EncodeFn enc = encode_fn();
  CUtensorMap tw, tx;
  {
    const cuuint64_t row_bytes = (cuuint64_t)(a.w.format == IE_FMT_INT4 ? a.w.k / 2 : a.w.k);
    const cuuint64_t dims[2] = {row_bytes, (cuuint64_t)a.w.n};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)(pl.w_stage_bytes / kTileN), (cuuint32_t)kTileN};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(a.w.codes), dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(IE_ERR_CUDA, "cuTensorMapEncodeTiled(weights): %d", (int)r);
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)a.w.k, (cuuint64_t)a.m};
    const cuuint64_t strides[1] = {(cuuint64_t)a.ldx * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)pl.bn};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = a.act_dtype == IE_DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                             : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUresult r = enc(&tx, dt, 2, const_cast<void*>(a.x), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(IE_ERR_CUDA, "cuTensorMapEncodeTiled(x): %d", (int)r);
  }
  CUtensorMap ts = tw, tz = tw;   // unused copies when the stage carries no tables
  if (pl.t_kind == 1) {
    const cuuint64_t dims[2] = {(cuuint64_t)a.w.n, (cuuint64_t)(a.w.k / 128)};
    const cuuint64_t strides[1] = {(cuuint64_t)a.w.n * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kTileN, 1};
    const cuuint32_t estr[2] = {1, 1};
    for (int i = 0; i < 2; ++i) {
      CUresult r = enc(i ? &tz : &ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                       const_cast<void*>(i ? a.w.zero : a.w.scale), dims, strides, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r != CUDA_SUCCESS) return set_error(IE_ERR_CUDA, "cuTensorMapEncodeTiled(groups): %d", (int)r);
    }
  } else if (pl.t_kind == 2) {
    const cuuint64_t dims[2] = {(cuuint64_t)a.w.k, (cuuint64_t)pl.t_rows};
    const cuuint64_t strides[1] = {(cuuint64_t)a.w.k * 4};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)pl.t_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(&ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(a.w.scale), dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(IE_ERR_CUDA, "cuTensorMapEncodeTiled(k scales): %d", (int)r);
  }
  TcParams prm{};
  prm.M = a.m;
  prm.K = a.w.k;
  prm.N = a.w.n;
  prm.axis = a.w.axis;
  prm.gate_up = a.w.gate_up;
  prm.epilogue = a.epilogue;
  prm.out_dtype = a.out_dtype;
  if (a.w.axis == IE_AXIS_GROUP128) {
    prm.gscale = static_cast<const __half*>(a.w.scale);
    prm.gzero = static_cast<const __half*>(a.w.zero);
  } else {
    prm.scale = static_cast<const float*>(a.w.scale);
  }
  prm.bias = a.bias;
  prm.residual = a.residual;
  prm.ldr = a.ldr;
  prm.out = a.out;
  prm.ldo = a.ldo;
  prm.bn = pl.bn;
  prm.n_tiles = pl.n_tiles;
  prm.m_tiles = pl.m_tiles;
  prm.splits = pl.splits;
  prm.kstages = pl.kstages;
  prm.ns = pl.ns;
  prm.na = pl.na;
  prm.w_stage_bytes = pl.w_stage_bytes;
  prm.t_kind = pl.t_kind;
  prm.t_rows = pl.t_rows;
  prm.t_stage_bytes = pl.t_stage_bytes;
  if (pl.splits > 1) {
    prm.counters = static_cast<uint32_t*>(a.workspace);
    prm.ws = reinterpret_cast<float*>(static_cast<char*>(a.workspace) + pl.counters_bytes);
  }
  prm.x_bf16 = a.act_dtype == IE_DT_BF16 ? 1 : 0;
  switch (pl.fmt) {
    case F_INT4G: return launch_typed<F_INT4G>(a, pl, tw, tx, ts, tz, prm, rc, s);
    case F_INT4SYM: return launch_typed<F_INT4SYM>(a, pl, tw, tx, ts, tz, prm, rc, s);
    case F_INT8: return launch_typed<F_INT8>(a, pl, tw, tx, ts, tz, prm, rc, s);
    default: return launch_typed<F_FP8>(a, pl, tw, tx, ts, tz, prm, rc, s);
  }
}

uint32_t tc_read_status(bool clear) {
  uint32_t v = 0;
  cudaMemcpyFromSymbol(&v, tc::g_tc_status, sizeof(v));
  if (clear && v) {
    const uint32_t z = 0;
    cudaMemcpyToSymbol(tc::g_tc_status, &z, sizeof(z));
  }
  return v;
}

}  // namespace ie
