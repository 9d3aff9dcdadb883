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
constexpr int kTileRows = kWarps * 2;

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

// Accumulate one 16-byte vector of one row against MT token runs of x'.
// `xr` points at the padded run for token 0; runs of successive tokens are
// `xstride` floats apart.  Returns per-token dot products in part[].
template <int V, int MT>
__device__ __forceinline__ void dot_vec(const uint4& wv, const float* __restrict__ xr,
                                        int xstride, float (&part)[MT]) {
  const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
  if constexpr (VecInfo<V>::kInt4) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const uint32_t t = ((w4[j] >> (4 * p)) & 0x000F000Fu) | 0x43004300u;
        const float lo = __uint_as_float(t << 16);           // 128 + q[k0 + 2p]
        const float hi = __uint_as_float(t & 0xFFFF0000u);   // 128 + q[k0 + 2p + 1]
        const int k = 8 * j + 2 * p;
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          const float2 xv = *reinterpret_cast<const float2*>(xr + m * xstride + k);
          part[m] = fmaf(lo, xv.x, part[m]);
          part[m] = fmaf(hi, xv.y, part[m]);
        }
      }
    }
  } else if constexpr (V == V_INT8) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t u = w4[j] ^ 0x80808080u;   // q + 128 per byte
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        // 0x4B0000bb as f32 is 2^23 + b: subtracting 2^23 + 128 recovers q exactly
        const float q = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440 | i)) - 8388736.0f;
        const int k = 4 * j + i;
#pragma unroll
        for (int m = 0; m < MT; ++m) part[m] = fmaf(q, xr[m * xstride + k], part[m]);
      }
    }
  } else {  // V_FP8
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const __nv_fp8x2_storage_t pr = (__nv_fp8x2_storage_t)((w4[j] >> (16 * h)) & 0xFFFFu);
        const __half2 hv = __half2(__nv_cvt_fp8x2_to_halfraw2(pr, __NV_E4M3));
        const float2 f = __half22float2(hv);
        const int k = 4 * j + 2 * h;
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          const float2 xv = *reinterpret_cast<const float2*>(xr + m * xstride + k);
          part[m] = fmaf(f.x, xv.x, part[m]);
          part[m] = fmaf(f.y, xv.y, part[m]);
        }
      }
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
    const int64_t r0 = rb * kTileRows + warp * 2;          // this warp's two rows
    const bool row_ok[2] = {r0 < p.N, r0 + 1 < p.N};
    float acc[2][MT];
#pragma unroll
    for (int r = 0; r < 2; ++r)
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
      const int nvec = kce / VI::kElems;
      for (int base = 0; base < nvec; base += 32 * 4) {
        uint4 wv[4][2];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = base + u * 32 + lane;
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            if (c < nvec && row_ok[r])
              wv[u][r] = ldg_stream(p.codes + (r0 + r) * p.row_bytes +
                                    (k0 / VI::kElems + c) * 16);
            else
              wv[u][r] = make_uint4(0, 0, 0, 0);
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = base + u * 32 + lane;
          if (c >= nvec) continue;
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            if (!row_ok[r]) continue;
            const int buf = (nbuf == 2) ? r : 0;
            const float* xr = xs + buf * MT * xstride + c * VI::kPadded;
            float part[MT];
#pragma unroll
            for (int m = 0; m < MT; ++m) part[m] = 0.0f;
            dot_vec<V, MT>(wv[u][r], xr, xstride, part);
            if constexpr (V == V_INT4G) {
              const int64_t g = (k0 + (int64_t)c * VI::kElems) / 128;
              const int64_t gi = g * p.N + (r0 + r);
              const float s = __half2float(p.gscale[gi]);
              const float off = 128.0f + __half2float(p.gzero[gi]);
#pragma unroll
              for (int m = 0; m < MT; ++m)
                acc[r][m] += s * (part[m] - off * xsum[(buf * MT + m) * runs + c]);
            } else if constexpr (V == V_INT4SYM) {
#pragma unroll
              for (int m = 0; m < MT; ++m)
                acc[r][m] += part[m] - 136.0f * xsum[(buf * MT + m) * runs + c];
            } else {
#pragma unroll
              for (int m = 0; m < MT; ++m) acc[r][m] += part[m];
            }
          }
        }
      }
      __syncthreads();
    }

    // ---- lane reduction ---------------------------------------------------
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        float v = acc[r][m];
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        acc[r][m] = v;
      }

    // ---- scales that sit on N ------------------------------------------------
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      if (!row_ok[r]) continue;
      float s = 1.0f;
      if (p.axis == IE_AXIS_N) s = p.scale[r0 + r];
      else if (p.axis == IE_AXIS_TENSOR) s = p.scale[p.gate_up ? r : 0];
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
            if (!row_ok[1]) continue;
            float g = acc[0][m], u = acc[1][m];
            if (p.epilogue & IE_EPI_BIAS) {
              g += p.bias[r0];
              u += p.bias[r0 + 1];
            }
            const int64_t j = r0 / 2;
            float v = silu(g) * u;
            if (p.epilogue & IE_EPI_RESIDUAL) v += load_act(p.residual, p.out_dtype, gm * p.ldr + j);
            store_out(p.out, p.out_dtype, gm * p.ldo + j, v);
          } else {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
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
      for (int m = 0; m < MT; ++m) {
        tile[m * kTileRows + warp * 2] = acc[0][m];
        tile[m * kTileRows + warp * 2 + 1] = acc[1][m];
      }
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
  ar_finish_all<kThreads>(rc, epoch, o, tiles,
                          [=](int64_t t, int64_t& n0, int& rows, int64_t& m0, int& cols) {
                            n0 = (t % row_blocks) * kTileRows;
                            rows = kTileRows;
                            m0 = (t / row_blocks) * MT;
                            cols = MT;
                          },
                          &s_ok);
  __syncthreads();
  reduce_finish(rc, epoch);
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
  return p;
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

int64_t gemv_tiles(const ie_qlinear_args& a) {
  const int mt = pick_mt(a.m);
  return ((a.w.n + kTileRows - 1) / kTileRows) * ((a.m + mt - 1) / mt);
}

int gemv_resident_ctas(const ie_qlinear_args& a, int* out) {
  return dispatch(a, nullptr, 0, nullptr, out);
}

int launch_qlinear_gemv(const ie_qlinear_args& a, const ReduceCtx* rc, int max_ctas,
                        cudaStream_t s) {
  return dispatch(a, rc, max_ctas, s, nullptr);
}

}  // namespace ie
