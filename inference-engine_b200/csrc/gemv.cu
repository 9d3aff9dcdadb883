// Weight-streaming quantized GEMV/skinny GEMM for decode-sized M, with an
// optional one-shot all-reduce fused into the epilogue.
//
// y[m, n] = sum_k x[m, k] * deq(W)[k, n] for a packed K-contiguous weight
// (row n of the device array is column n of the reference's [K, N] weight).
//
// Structure (per CTA of 8 warps, a tile of 16 rows x MT tokens):
//   * x for a K chunk is staged in shared memory as f32 with any per-K scale
//     already folded in (x'[m,k] = x[m,k] * s[k]; the reference's default
//     PER_OUTPUT_CHANNEL scale sits on K, ie/quant/weights.py:10,45-48), padded
//     so that 16-byte shared loads of consecutive lanes hit distinct banks;
//   * each warp owns two rows; every lane streams 16-byte vectors of both rows
//     with non-allocating global loads (all of a chunk's vectors are issued
//     before any is consumed), dequantizes in registers and accumulates in f32;
//   * int4 codes are widened two at a time with one mask+or: the nibble pair
//     lands in the mantissas of a bf16x2 whose exponent makes it 128 + q, and
//     the 128 + zero offset is removed once per 32 codes with a per-chunk sum
//     of x' (sum (128+q) x - (128+z) sum x = sum (q-z) x);
//   * a warp-shuffle butterfly reduces the lanes; the epilogue applies per-N /
//     per-tensor / per-group scales, bias, SiLU*up pairing and the residual.
// With a ReduceCtx the CTA grid is made co-resident (persistent loop over
// tiles): every tile's f32 partial is first pushed to all ranks' landing
// buffers over NVLink and flagged, then each rank waits (bounded) for the
// tile's flags and sums the partials in rank order (the reference's
// all_reduce order, ie/parallel/sharding.py:40-44) before the epilogue.
#include <algorithm>

#include "common.cuh"

namespace ie {
namespace {

enum Variant { V_INT8 = 0, V_INT4SYM = 1, V_INT4G = 2, V_FP8 = 3 };

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRows = 4;                    // weight rows per warp
constexpr int kTileRows = kWarps * kRows;

// x' buffers the kernel may hold: two for gate/up pairs with per-K scales
template <int V> __host__ __device__ constexpr int nbuf_max() { return 2; }

template <int V> struct VecInfo {
  static constexpr int kElems = (V == V_INT4SYM || V == V_INT4G) ? 32 : 16;  // per 16 bytes
  static constexpr int kPadded = kElems + 4;   // floats per padded x run
  static constexpr bool kInt4 = (V == V_INT4SYM || V == V_INT4G);
};

struct GemvParams {
  int64_t M, K, N;
  const void* x;
  int64_t ldx;
  int act_dtype;
  const uint8_t* codes;
  int64_t row_bytes;
  const float* scale;     // per-K ([K] or [2][K]), per-N [N], per-tensor [1] or [2]
  const __half* gscale;   // group-128 [K/128][N]
  const __half* gzero;
  int axis;
  int gate_up;
  int epilogue;
  const float* bias;
  const void* residual;
  int64_t ldr;
  void* out;
  int64_t ldo;
  int out_dtype;
  int kc;                 // K elements staged per chunk
  // decode kernel only: RMS norm folded into the staging of x'
  // (x' = x * rinv_m * norm_w[k], rinv_m = 1 / sqrt(mean_k(x^2) + eps))
  const float* norm_w;
  float norm_eps;
};

__device__ __forceinline__ float load_act(const void* p, int dt, int64_t i) {
  if (dt == IE_DT_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  if (dt == IE_DT_F16) return __half2float(static_cast<const __half*>(p)[i]);
  return static_cast<const float*>(p)[i];
}
__device__ __forceinline__ void store_out(void* p, int dt, int64_t i, float v) {
  if (dt == IE_DT_BF16) static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else if (dt == IE_DT_F16) static_cast<__half*>(p)[i] = __float2half_rn(v);
  else static_cast<float*>(p)[i] = v;
}

__device__ __forceinline__ uint4 ldg_stream(const uint8_t* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + __expf(-g)); }

// Packed f32x2 FMA (sm_100): acc.{x,y} += a.{x,y} * b.{x,y}, each lane
// rounded once like fmaf.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(d)
      : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)),
        "l"(*reinterpret_cast<uint64_t*>(&c)));
  return *reinterpret_cast<float2*>(&d);
}

// Word j (32 bits) of a row's 16-byte code vector against the matching K
// values of x' (xw[m]: this word's K values of token m, as f32 pairs), added
// into part[m] as f32 pairs.
//   int4: the pair (8j+2p, 8j+2p+1) sits in nibbles (p, p+4); one mask+or
//     makes a bf16x2 of 128 + q, whose halves are exact f32 (bits << 16);
//   int8: byte i as f32 2^23 + 128 + q minus 2^23 + 128 (exact);
//   fp8: e4m3 pairs widened through f16 (exact).
template <int V, int MT>
__device__ __forceinline__ void dot_word(uint32_t w, const float2 (&xw)[MT][VecInfo<V>::kElems / 8],
                                         float2 (&part)[MT]) {
  if constexpr (VecInfo<V>::kInt4) {
#pragma unroll
    for (int pp = 0; pp < 4; ++pp) {
      const uint32_t t = ((w >> (4 * pp)) & 0x000F000Fu) | 0x43004300u;
      const float2 q = make_float2(__uint_as_float(t << 16), __uint_as_float(t & 0xFFFF0000u));
#pragma unroll
      for (int m = 0; m < MT; ++m) part[m] = ffma2(q, xw[m][pp], part[m]);
    }
  } else if constexpr (V == V_INT8) {
    const uint32_t u = w ^ 0x80808080u;   // q + 128 per byte
    // 0x4B0000bb as f32 is 2^23 + b: subtracting 2^23 + 128 recovers q exactly
    const float2 q0 = make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440)) - 8388736.0f,
                                  __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441)) - 8388736.0f);
    const float2 q1 = make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442)) - 8388736.0f,
                                  __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443)) - 8388736.0f);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      part[m] = ffma2(q0, xw[m][0], part[m]);
      part[m] = ffma2(q1, xw[m][1], part[m]);
    }
  } else {  // V_FP8
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const __nv_fp8x2_storage_t pr = (__nv_fp8x2_storage_t)((w >> (16 * h)) & 0xFFFFu);
      const float2 q = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(pr, __NV_E4M3)));
#pragma unroll
      for (int m = 0; m < MT; ++m) part[m] = ffma2(q, xw[m][h], part[m]);
    }
  }
}

template <int V, int MT>
__global__ void __launch_bounds__(kThreads)
gemv_kernel(GemvParams p, ReduceCtx rc, int reduce) {
  using VI = VecInfo<V>;
  extern __shared__ __align__(16) float smem[];
  const int kc = p.kc;
  const int runs = kc / VI::kElems;
  const int xstride = runs * VI::kPadded;                 // floats per token per buffer
  const int nbuf = (p.gate_up && p.axis == IE_AXIS_K) ? 2 : 1;
  float* xs = smem;                                       // [nbuf][MT][xstride]
  float* xsum = xs + nbuf * MT * xstride;                 // [nbuf][MT][runs] (int4 only)
  float* tile = xsum + (VI::kInt4 ? nbuf * MT * runs : 0);  // [MT][kTileRows] (reduce)

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t epoch = reduce ? reduce_epoch(rc) : 0u;
  const int64_t row_blocks = (p.N + kTileRows - 1) / kTileRows;
  const int64_t m_chunks = (p.M + MT - 1) / MT;
  const int64_t tiles = row_blocks * m_chunks;

  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int64_t rb = t % row_blocks, mc = t / row_blocks;
    const int64_t m0 = mc * MT;
    const int64_t r0 = rb * kTileRows + warp * kRows;      // this warp's rows
    bool row_ok[kRows];
#pragma unroll
    for (int r = 0; r < kRows; ++r) row_ok[r] = r0 + r < p.N;
    float acc[kRows][MT];
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int m = 0; m < MT; ++m) acc[r][m] = 0.0f;

    for (int64_t k0 = 0; k0 < p.K; k0 += kc) {
      const int kce = (int)((p.K - k0) < (int64_t)kc ? (p.K - k0) : (int64_t)kc);
      // ---- stage x' (per-K scale folded in) -------------------------------
      for (int i = threadIdx.x; i < MT * kc; i += kThreads) {
        const int m = i / kc, kk = i % kc;
        float v = 0.0f;
        if (m0 + m < p.M && kk < kce) v = load_act(p.x, p.act_dtype, (m0 + m) * p.ldx + k0 + kk);
        const int pos = (kk / VI::kElems) * VI::kPadded + kk % VI::kElems;
        if (p.axis == IE_AXIS_K) {
          const float s0 = kk < kce ? p.scale[k0 + kk] : 0.0f;
          xs[m * xstride + pos] = v * s0;
          if (nbuf == 2) {
            const float s1 = kk < kce ? p.scale[p.K + k0 + kk] : 0.0f;
            xs[(MT + m) * xstride + pos] = v * s1;
          }
        } else {
          xs[m * xstride + pos] = v;
        }
      }
      __syncthreads();
      if constexpr (VI::kInt4) {
        for (int i = threadIdx.x; i < nbuf * MT * runs; i += kThreads) {
          const float* run = xs + (i / runs) * xstride + (i % runs) * VI::kPadded;
          float s = 0.0f;
#pragma unroll 8
          for (int e = 0; e < VI::kElems; ++e) s += run[e];
          xsum[i] = s;
        }
        __syncthreads();
      }

      // ---- stream the weights of this chunk -------------------------------
      // Every lane takes one 16-byte code vector of each of the warp's rows at
      // a K position; the x' values of that position are read from shared
      // memory once per word and token (16-byte loads) and serve all rows.
      constexpr int kU = MT >= 4 ? 1 : 2;     // vectors per row in flight
      constexpr int kXw = VI::kElems / 8;     // f32 pairs of x' per 32-bit word
      const int nvec = kce / VI::kElems;
      for (int base = 0; base < nvec; base += 32 * kU) {
        uint4 wv[kU][kRows];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int c = base + u * 32 + lane;
#pragma unroll
          for (int r = 0; r < kRows; ++r) {
            if (c < nvec && row_ok[r])
              wv[u][r] = ldg_stream(p.codes + (r0 + r) * p.row_bytes +
                                    (k0 / VI::kElems + c) * 16);
            else
              wv[u][r] = make_uint4(0, 0, 0, 0);
          }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int c = base + u * 32 + lane;
          if (c >= nvec) continue;
          float2 part[kRows][MT];
#pragma unroll
          for (int r = 0; r < kRows; ++r)
#pragma unroll
            for (int m = 0; m < MT; ++m) part[r][m] = make_float2(0.0f, 0.0f);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int b = 0; b < (nbuf_max<V>()); ++b) {
              if (b >= nbuf) break;
              // this word's K values of every token of buffer b
              float2 xw[MT][kXw];
#pragma unroll
              for (int m = 0; m < MT; ++m) {
                const float4* xr = reinterpret_cast<const float4*>(
                    xs + (b * MT + m) * xstride + c * VI::kPadded + j * (2 * kXw));
#pragma unroll
                for (int h = 0; h < kXw / 2; ++h) {
                  const float4 v = xr[h];
                  xw[m][2 * h] = make_float2(v.x, v.y);
                  xw[m][2 * h + 1] = make_float2(v.z, v.w);
                }
              }
#pragma unroll
              for (int r = 0; r < kRows; ++r) {
                if (nbuf == 2 && (r & 1) != b) continue;   // gate/up rows alternate buffers
                const uint32_t w = j == 0 ? wv[u][r].x : j == 1 ? wv[u][r].y
                                 : j == 2 ? wv[u][r].z : wv[u][r].w;
                dot_word<V, MT>(w, xw, part[r]);
              }
            }
          }
#pragma unroll
          for (int r = 0; r < kRows; ++r) {
            if (!row_ok[r]) continue;
            const int buf = (nbuf == 2) ? (r & 1) : 0;
            if constexpr (V == V_INT4G) {
              const int64_t g = (k0 + (int64_t)c * VI::kElems) / 128;
              const int64_t gi = g * p.N + (r0 + r);
              const float sc = __half2float(p.gscale[gi]);
              const float off = 128.0f + __half2float(p.gzero[gi]);
#pragma unroll
              for (int m = 0; m < MT; ++m)
                acc[r][m] += sc * ((part[r][m].x + part[r][m].y) -
                                   off * xsum[(buf * MT + m) * runs + c]);
            } else if constexpr (V == V_INT4SYM) {
#pragma unroll
              for (int m = 0; m < MT; ++m)
                acc[r][m] += (part[r][m].x + part[r][m].y) -
                             136.0f * xsum[(buf * MT + m) * runs + c];
            } else {
#pragma unroll
              for (int m = 0; m < MT; ++m) acc[r][m] += part[r][m].x + part[r][m].y;
            }
          }
        }
      }
      __syncthreads();
    }

    // ---- lane reduction ---------------------------------------------------
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        float v = acc[r][m];
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        acc[r][m] = v;
      }

    // ---- scales that sit on N ------------------------------------------------
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      if (!row_ok[r]) continue;
      float s = 1.0f;
      if (p.axis == IE_AXIS_N) s = p.scale[r0 + r];
      else if (p.axis == IE_AXIS_TENSOR) s = p.scale[p.gate_up ? (r & 1) : 0];
#pragma unroll
      for (int m = 0; m < MT; ++m) acc[r][m] *= s;
    }

    if (!reduce) {
      if (lane == 0) {
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          const int64_t gm = m0 + m;
          if (gm >= p.M) continue;
          if (p.epilogue & IE_EPI_SILU_MUL) {
            // rows (r0 + 2i, r0 + 2i + 1) are a gate/up pair
#pragma unroll
            for (int i2 = 0; i2 < kRows / 2; ++i2) {
              if (!row_ok[2 * i2 + 1]) continue;
              float g = acc[2 * i2][m], u = acc[2 * i2 + 1][m];
              if (p.epilogue & IE_EPI_BIAS) {
                g += p.bias[r0 + 2 * i2];
                u += p.bias[r0 + 2 * i2 + 1];
              }
              const int64_t j = r0 / 2 + i2;
              float v = silu(g) * u;
              if (p.epilogue & IE_EPI_RESIDUAL) v += load_act(p.residual, p.out_dtype, gm * p.ldr + j);
              store_out(p.out, p.out_dtype, gm * p.ldo + j, v);
            }
          } else {
#pragma unroll
            for (int r = 0; r < kRows; ++r) {
              if (!row_ok[r]) continue;
              const int64_t n = r0 + r;
              float v = acc[r][m];
              if (p.epilogue & IE_EPI_BIAS) v += p.bias[n];
              if (p.epilogue & IE_EPI_RESIDUAL)
                v = load_act(p.residual, p.out_dtype, gm * p.ldr + n) + v;
              store_out(p.out, p.out_dtype, gm * p.ldo + n, v);
            }
          }
        }
      }
      continue;
    }

    // ---- fused all-reduce, phase 1: push this tile's partial to every rank --
    if (lane == 0) {
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int r = 0; r < kRows; ++r) tile[m * kTileRows + warp * kRows + r] = acc[r][m];
    }
    __syncthreads();
    const int64_t nbase = rb * kTileRows;
    int d0, d1;
    ar_push_range(rc, t, d0, d1);
    for (int i = threadIdx.x; i < (d1 - d0) * MT * kTileRows; i += kThreads) {
      const int dst = d0 + i / (MT * kTileRows);
      const int e = i % (MT * kTileRows);
      const int m = e / kTileRows, rr = e % kTileRows;
      const int64_t gm = m0 + m, n = nbase + rr;
      if (gm < p.M && n < p.N)
        landing_slot(rc, dst, epoch)[rc.rank * rc.slot_floats + gm * p.N + n] = tile[e];
    }
    __syncthreads();
    ar_publish(rc, t, epoch, threadIdx.x);
  }

  if (!reduce) return;

  // ---- phase 2 (one-shot: every tile; two-shot: see ar_finish_all) --------------
  __shared__ int s_ok;
  const ArOut o{p.out, p.residual, p.bias, p.ldo, p.ldr, p.M, p.N, p.out_dtype,
                (p.epilogue & IE_EPI_BIAS) != 0, (p.epilogue & IE_EPI_RESIDUAL) != 0};
  ar_finish_all<kThreads, kTileRows>(rc, epoch, o, tiles,
                          [=](int64_t t, int64_t& n0, int64_t& m0, int& cols) {
                            n0 = (t % row_blocks) * kTileRows;
                            m0 = (t / row_blocks) * MT;
                            cols = MT;
                          },
                          &s_ok);
  __syncthreads();
  reduce_finish(rc, epoch);
}

// ---------------------------------------------------------------------------
// Decode GEMV (M <= 2 tokens, no fused all-reduce).  The general kernel above
// stages x' chunk by chunk inside every 32-row tile (three CTA barriers per
// chunk), so a warp has one round of weight loads in flight between
// barriers.  Here x' for the whole K is staged once per CTA -- after the first
// row group's weight loads are issued -- and every warp then walks row groups
// of kRows rows (persistent grid) with no CTA barrier, each lane keeping
// kDecVec 16-byte code vectors of each row in flight.
// ---------------------------------------------------------------------------
constexpr int kDecVec = 4;

template <int V, int MT>
__device__ __forceinline__ void dec_epilogue(const GemvParams& p, float (&acc)[kRows][MT],
                                             int64_t r0) {
#pragma unroll
  for (int r = 0; r < kRows; ++r) {
    float s = 1.0f;
    if (r0 + r < p.N) {
      if (p.axis == IE_AXIS_N) s = p.scale[r0 + r];
      else if (p.axis == IE_AXIS_TENSOR) s = p.scale[p.gate_up ? (r & 1) : 0];
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[r][m] *= s;
  }
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    if (m >= p.M) continue;
    if (p.epilogue & IE_EPI_SILU_MUL) {
#pragma unroll
      for (int i2 = 0; i2 < kRows / 2; ++i2) {
        if (r0 + 2 * i2 + 1 >= p.N) continue;
        float g = acc[2 * i2][m], u = acc[2 * i2 + 1][m];
        if (p.epilogue & IE_EPI_BIAS) {
          g += p.bias[r0 + 2 * i2];
          u += p.bias[r0 + 2 * i2 + 1];
        }
        const int64_t j = r0 / 2 + i2;
        float v = silu(g) * u;
        if (p.epilogue & IE_EPI_RESIDUAL) v += load_act(p.residual, p.out_dtype, m * p.ldr + j);
        store_out(p.out, p.out_dtype, m * p.ldo + j, v);
      }
    } else {
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        const int64_t n = r0 + r;
        if (n >= p.N) continue;
        float v = acc[r][m];
        if (p.epilogue & IE_EPI_BIAS) v += p.bias[n];
        if (p.epilogue & IE_EPI_RESIDUAL) v = load_act(p.residual, p.out_dtype, m * p.ldr + n) + v;
        store_out(p.out, p.out_dtype, m * p.ldo + n, v);
      }
    }
  }
}

template <int V, int MT>
__global__ void __launch_bounds__(kThreads)
gemv_dec_kernel(GemvParams p) {
  using VI = VecInfo<V>;
  constexpr int kXw = VI::kElems / 8;
  extern __shared__ __align__(16) float smem[];
  const int nvec = (int)(p.K / VI::kElems);            // 16-byte code vectors per row
  const int xstride = nvec * VI::kPadded;              // floats per token per buffer
  const int nbuf = (p.gate_up && p.axis == IE_AXIS_K) ? 2 : 1;
  float* xs = smem;                                    // [nbuf][MT][xstride]
  float* xsum = xs + nbuf * MT * xstride;              // [nbuf][MT][nvec] (int4 only)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t groups = (p.N + kRows - 1) / kRows;
  const int64_t g_step = (int64_t)gridDim.x * kWarps;
  int64_t g = (int64_t)blockIdx.x * kWarps + warp;

  uint4 wv[kDecVec][kRows];
  auto load_round = [&](int64_t grp, int c0) {
    const int64_t r0 = grp * kRows;
#pragma unroll
    for (int u = 0; u < kDecVec; ++u) {
      const int c = c0 + u * 32 + lane;
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        if (grp < groups && r0 + r < p.N && c < nvec)
          wv[u][r] = ldg_stream(p.codes + (r0 + r) * p.row_bytes + (int64_t)c * 16);
        else
          wv[u][r] = make_uint4(0, 0, 0, 0);
      }
    }
  };
  // the first round's weights do not depend on x: in flight while x' is staged
  load_round(g, 0);
  __shared__ float s_red[MT][kWarps];
  __shared__ float s_rinv[MT];
  if (p.norm_w) {
    // per-token RMS factor, with the tensor-core prologue's operations
    // (sum of squares in f32, then 1 / sqrt(ss / K + eps) correctly rounded)
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      float ss = 0.0f;
      if (m < p.M)
        for (int kk = threadIdx.x; kk < (int)p.K; kk += kThreads) {
          const float v = load_act(p.x, p.act_dtype, m * p.ldx + kk);
          ss = fmaf(v, v, ss);
        }
#pragma unroll
      for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) s_red[m][warp] = ss;
    }
    __syncthreads();
    if (threadIdx.x < MT) {
      float ss = 0.0f;
      for (int w = 0; w < kWarps; ++w) ss += s_red[threadIdx.x][w];
      s_rinv[threadIdx.x] = 1.0f / __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)p.K), p.norm_eps));
    }
    __syncthreads();
  }
  for (int i = threadIdx.x; i < MT * (int)p.K; i += kThreads) {
    const int m = i / (int)p.K, kk = i % (int)p.K;
    float v = m < p.M ? load_act(p.x, p.act_dtype, m * p.ldx + kk) : 0.0f;
    if (p.norm_w) v = (v * s_rinv[m]) * p.norm_w[kk];
    const int pos = (kk / VI::kElems) * VI::kPadded + kk % VI::kElems;
    if (p.axis == IE_AXIS_K) {
      xs[m * xstride + pos] = v * p.scale[kk];
      if (nbuf == 2) xs[(MT + m) * xstride + pos] = v * p.scale[p.K + kk];
    } else {
      xs[m * xstride + pos] = v;
    }
  }
  __syncthreads();
  if constexpr (VI::kInt4) {
    for (int i = threadIdx.x; i < nbuf * MT * nvec; i += kThreads) {
      const float* run = xs + (i / nvec) * xstride + (i % nvec) * VI::kPadded;
      float sum = 0.0f;
#pragma unroll 8
      for (int e = 0; e < VI::kElems; ++e) sum += run[e];
      xsum[i] = sum;
    }
    __syncthreads();
  }

  for (; g < groups; g += g_step) {
    const int64_t r0 = g * kRows;
    float acc[kRows][MT];
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int m = 0; m < MT; ++m) acc[r][m] = 0.0f;
    for (int c0 = 0; c0 < nvec; c0 += 32 * kDecVec) {
      if (c0 > 0) load_round(g, c0);   // (a group's first round was loaded ahead)
#pragma unroll
      for (int u = 0; u < kDecVec; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c >= nvec) continue;
        float2 part[kRows][MT];
#pragma unroll
        for (int r = 0; r < kRows; ++r)
#pragma unroll
          for (int m = 0; m < MT; ++m) part[r][m] = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
          for (int b = 0; b < 2; ++b) {
            if (b >= nbuf) break;
            float2 xw[MT][kXw];
#pragma unroll
            for (int m = 0; m < MT; ++m) {
              const float4* xr = reinterpret_cast<const float4*>(
                  xs + (b * MT + m) * xstride + c * VI::kPadded + j * (2 * kXw));
#pragma unroll
              for (int h = 0; h < kXw / 2; ++h) {
                const float4 v = xr[h];
                xw[m][2 * h] = make_float2(v.x, v.y);
                xw[m][2 * h + 1] = make_float2(v.z, v.w);
              }
            }
#pragma unroll
            for (int r = 0; r < kRows; ++r) {
              if (nbuf == 2 && (r & 1) != b) continue;
              const uint32_t w = j == 0 ? wv[u][r].x : j == 1 ? wv[u][r].y
                               : j == 2 ? wv[u][r].z : wv[u][r].w;
              dot_word<V, MT>(w, xw, part[r]);
            }
          }
        }
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
          if (r0 + r >= p.N) continue;
          const int buf = (nbuf == 2) ? (r & 1) : 0;
          if constexpr (V == V_INT4G) {
            const int64_t gi = ((int64_t)c * VI::kElems / 128) * p.N + (r0 + r);
            const float sc = __half2float(p.gscale[gi]);
            const float off = 128.0f + __half2float(p.gzero[gi]);
#pragma unroll
            for (int m = 0; m < MT; ++m)
              acc[r][m] += sc * ((part[r][m].x + part[r][m].y) -
                                 off * xsum[(buf * MT + m) * nvec + c]);
          } else if constexpr (V == V_INT4SYM) {
#pragma unroll
            for (int m = 0; m < MT; ++m)
              acc[r][m] += (part[r][m].x + part[r][m].y) - 136.0f * xsum[(buf * MT + m) * nvec + c];
          } else {
#pragma unroll
            for (int m = 0; m < MT; ++m) acc[r][m] += part[r][m].x + part[r][m].y;
          }
        }
      }
    }
    // the next group's first round goes out before this group's reduction
    load_round(g + g_step, 0);
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        float v = acc[r][m];
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        acc[r][m] = v;
      }
    if (lane == 0) dec_epilogue<V, MT>(p, acc, r0);
  }
}

int variant_of(const ie_qweight& w) {
  if (w.format == IE_FMT_INT8) return V_INT8;
  if (w.format == IE_FMT_FP8_E4M3) return V_FP8;
  return w.axis == IE_AXIS_GROUP128 ? V_INT4G : V_INT4SYM;
}

int pick_mt(int64_t m) { return m >= 4 ? 4 : (m >= 2 ? 2 : 1); }
int pick_kc(int mt) { return mt >= 4 ? 1024 : 2048; }

template <int V, int MT>
size_t smem_bytes(const GemvParams& p) {
  using VI = VecInfo<V>;
  const int runs = p.kc / VI::kElems;
  const int nbuf = (p.gate_up && p.axis == IE_AXIS_K) ? 2 : 1;
  size_t f = (size_t)nbuf * MT * runs * VI::kPadded;
  if (VI::kInt4) f += (size_t)nbuf * MT * runs;
  f += (size_t)MT * kTileRows;
  return f * sizeof(float);
}

template <int V, int MT>
int launch_vm(const GemvParams& p, const ReduceCtx* rc, int max_ctas, cudaStream_t s,
              int* resident_out) {
  const size_t smem = smem_bytes<V, MT>(p);
  auto kern = gemv_kernel<V, MT>;
  if (smem > 48 * 1024)
    IE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  if (resident_out) {
    int per_sm = 0, dev = 0, sms = 0;
    IE_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem));
    IE_CUDA_TRY(cudaGetDevice(&dev));
    IE_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    *resident_out = per_sm * sms;
    return IE_OK;
  }
  const int64_t tiles = ((p.N + kTileRows - 1) / kTileRows) * ((p.M + MT - 1) / MT);
  int64_t grid = tiles;
  if (max_ctas > 0) grid = std::min<int64_t>(grid, max_ctas);
  ReduceCtx none{};
  kern<<<(unsigned)grid, kThreads, smem, s>>>(p, rc ? *rc : none, rc ? 1 : 0);
  return launch_status("gemv_kernel");
}

template <int V>
int launch_v(const GemvParams& p, int mt, const ReduceCtx* rc, int max_ctas, cudaStream_t s,
             int* resident_out) {
  switch (mt) {
    case 1: return launch_vm<V, 1>(p, rc, max_ctas, s, resident_out);
    case 2: return launch_vm<V, 2>(p, rc, max_ctas, s, resident_out);
    default: return launch_vm<V, 4>(p, rc, max_ctas, s, resident_out);
  }
}

GemvParams make_params(const ie_qlinear_args& a) {
  GemvParams p{};
  const ie_qweight& w = a.w;
  p.M = a.m;
  p.K = w.k;
  p.N = w.n;
  p.x = a.x;
  p.ldx = a.ldx;
  p.act_dtype = a.act_dtype;
  p.codes = static_cast<const uint8_t*>(w.codes);
  p.row_bytes = w.format == IE_FMT_INT4 ? w.k / 2 : w.k;
  p.axis = w.axis;
  p.gate_up = w.gate_up;
  if (w.axis == IE_AXIS_GROUP128) {
    p.gscale = static_cast<const __half*>(w.scale);
    p.gzero = static_cast<const __half*>(w.zero);
  } else {
    p.scale = static_cast<const float*>(w.scale);
  }
  p.epilogue = a.epilogue;
  p.bias = a.bias;
  p.residual = a.residual;
  p.ldr = a.ldr;
  p.out = a.out;
  p.ldo = a.ldo;
  p.out_dtype = a.out_dtype;
  p.kc = pick_kc(pick_mt(a.m));
  if (a.epilogue & IE_EPI_RMS_NORM) {
    p.norm_w = a.norm_weight;
    p.norm_eps = a.norm_eps;
  }
  return p;
}

// Shared memory of the decode kernel (x' of the whole K, padded runs, and the
// int4 run sums), or 0 when it does not apply: more than two tokens, K not a
// whole number of code vectors, or x' beyond kDecSmemMax.
constexpr size_t kDecSmemMax = 160 * 1024;
size_t dec_smem(const ie_qlinear_args& a) {
  if (a.m > 2) return 0;
  const int v = variant_of(a.w);
  const int elems = (v == V_INT4G || v == V_INT4SYM) ? 32 : 16;
  const int padded = elems + 4;
  if (a.w.k % elems) return 0;
  const int64_t nvec = a.w.k / elems;
  const int mt = pick_mt(a.m);
  const int nbuf = (a.w.gate_up && a.w.axis == IE_AXIS_K) ? 2 : 1;
  size_t f = (size_t)nbuf * mt * nvec * padded;
  if (elems == 32) f += (size_t)nbuf * mt * nvec;
  const size_t bytes = f * sizeof(float);
  return bytes <= kDecSmemMax ? bytes : 0;
}

template <int V, int MT>
int launch_dec(const GemvParams& p, size_t smem, cudaStream_t s) {
  auto kern = gemv_dec_kernel<V, MT>;
  IE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 0, dev = 0, sms = 0;
  IE_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem));
  IE_CUDA_TRY(cudaGetDevice(&dev));
  IE_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int64_t groups = (p.N + kRows - 1) / kRows;
  const int64_t need = (groups + kWarps - 1) / kWarps;
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(need, (int64_t)std::max(per_sm, 1) * sms));
  kern<<<(unsigned)grid, kThreads, smem, s>>>(p);
  return launch_status("gemv_dec_kernel");
}

int dispatch_dec(const ie_qlinear_args& a, size_t smem, cudaStream_t s) {
  const GemvParams p = make_params(a);
  const bool two = a.m > 1;
  switch (variant_of(a.w)) {
    case V_INT8: return two ? launch_dec<V_INT8, 2>(p, smem, s) : launch_dec<V_INT8, 1>(p, smem, s);
    case V_INT4SYM:
      return two ? launch_dec<V_INT4SYM, 2>(p, smem, s) : launch_dec<V_INT4SYM, 1>(p, smem, s);
    case V_INT4G: return two ? launch_dec<V_INT4G, 2>(p, smem, s) : launch_dec<V_INT4G, 1>(p, smem, s);
    default: return two ? launch_dec<V_FP8, 2>(p, smem, s) : launch_dec<V_FP8, 1>(p, smem, s);
  }
}

int dispatch(const ie_qlinear_args& a, const ReduceCtx* rc, int max_ctas, cudaStream_t s,
             int* resident_out) {
  const GemvParams p = make_params(a);
  const int mt = pick_mt(a.m);
  switch (variant_of(a.w)) {
    case V_INT8: return launch_v<V_INT8>(p, mt, rc, max_ctas, s, resident_out);
    case V_INT4SYM: return launch_v<V_INT4SYM>(p, mt, rc, max_ctas, s, resident_out);
    case V_INT4G: return launch_v<V_INT4G>(p, mt, rc, max_ctas, s, resident_out);
    default: return launch_v<V_FP8>(p, mt, rc, max_ctas, s, resident_out);
  }
}

}  // namespace

bool gemv_decode_ok(const ie_qlinear_args& a) { return dec_smem(a) > 0; }

int64_t gemv_tiles(const ie_qlinear_args& a) {
  const int mt = pick_mt(a.m);
  return ((a.w.n + kTileRows - 1) / kTileRows) * ((a.m + mt - 1) / mt);
}

int gemv_resident_ctas(const ie_qlinear_args& a, int* out) {
  return dispatch(a, nullptr, 0, nullptr, out);
}

int launch_qlinear_gemv(const ie_qlinear_args& a, const ReduceCtx* rc, int max_ctas,
                        cudaStream_t s) {
  if (!rc) {
    const size_t smem = dec_smem(a);
    if (smem) return dispatch_dec(a, smem, s);
  }
  return dispatch(a, rc, max_ctas, s, nullptr);
}

}  // namespace ie
