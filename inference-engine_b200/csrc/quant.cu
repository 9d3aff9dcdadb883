// Quantizer, packer and dequantizer kernels.
//
// The quantizer reproduces the reference engine's NumPy arithmetic bit for bit
// (ie/quant/weights.py:51-81, ie/quant/formats.py:74-79): every scale, zero
// point and code is computed with the same IEEE f32 operations in the same
// order (f32 division, f32 add, round-half-to-even), and the per-axis maxima
// and minima are order-independent, so the GPU tables equal NumPy's exactly.
#include <algorithm>
#include <cfloat>
#include <cmath>

#include "common.cuh"

namespace ie {
namespace {

constexpr int kThreads = 256;

// round_to_float_format (ie/quant/formats.py:74-79): round_to_format and
// FloatFmt in common.cuh.
FloatFmt make_float_fmt(int e, int m, int reserves_inf) {
  const int bias = (1 << (e - 1)) - 1;
  double largest, mscale;
  if (reserves_inf) {
    largest = (1 << e) - 2 - bias;
    mscale = 2.0 - std::ldexp(1.0, -m);
  } else {
    largest = (1 << e) - 1 - bias;
    mscale = 2.0 - std::ldexp(1.0, 1 - m);
  }
  FloatFmt f;
  f.mantissa_bits = m;
  f.max_value = (float)(std::ldexp(1.0, (int)largest) * mscale);
  f.flush_below = (float)(std::ldexp(1.0, 1 - bias) * std::ldexp(1.0, -m));
  return f;
}

__global__ void round_kernel(const float* __restrict__ x, float* __restrict__ out, int64_t n,
                             FloatFmt f) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = round_to_format(x[i], f);
}

// ---------------------------------------------------------------------------
// Per-axis statistics.  Stats are max|w| (symmetric / float) or (min, max)
// (asymmetric); they are exact, so any reduction order gives NumPy's value.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t ordered_bits(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float from_ordered(uint32_t o) {
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o);
}

struct QuantSpec {
  int kind;       // 0 symmetric int, 1 asymmetric int, 2 float
  int qmax;       // signed_max (sym) or unsigned_max (asym)
  FloatFmt ff;    // float formats
};

// Scale and zero from the statistics, exactly as ie/quant/weights.py computes them.
__device__ __forceinline__ void finish_scale(const QuantSpec& q, float lo, float hi,
                                             float* scale, float* zero) {
  if (q.kind == 1) {
    float span = __fsub_rn(hi, lo);
    if (span == 0.0f) span = 1.0f;                          // weights.py:63
    const float s = __fdiv_rn(span, (float)q.qmax);         // weights.py:64
    *scale = s;
    *zero = rintf(__fdiv_rn(-lo, s));                       // weights.py:65
  } else {
    const float peak = hi;
    const float denom = q.kind == 0 ? (float)q.qmax : q.ff.max_value;
    *scale = peak == 0.0f ? 1.0f : __fdiv_rn(peak, denom);  // weights.py:56,76
    *zero = 0.0f;
  }
}

__device__ __forceinline__ float code_of(const QuantSpec& q, float w, float s, float z) {
  if (q.kind == 0) {                                        // weights.py:57
    const float r = rintf(__fdiv_rn(w, s));
    return fminf(fmaxf(r, -(float)q.qmax), (float)q.qmax);
  }
  if (q.kind == 1) {                                        // weights.py:66
    const float r = rintf(__fadd_rn(__fdiv_rn(w, s), z));
    return fminf(fmaxf(r, 0.0f), (float)q.qmax);
  }
  return round_to_format(__fdiv_rn(w, s), q.ff);            // weights.py:77
}

// axis 0: one block per row, reduce over columns, then write that row's codes.
__global__ void quant_rows_kernel(const float* __restrict__ w, int64_t rows, int64_t cols,
                                  QuantSpec q, void* __restrict__ codes, int codes_f32,
                                  float* __restrict__ scale, float* __restrict__ zero) {
  __shared__ float s_lo[kThreads / 32], s_hi[kThreads / 32];
  __shared__ float s_scale, s_zero;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* row = w + r * cols;
    float lo = FLT_MAX, hi = q.kind == 1 ? -FLT_MAX : 0.0f;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
      const float v = row[c];
      if (q.kind == 1) {
        lo = fminf(lo, v);
        hi = fmaxf(hi, v);
      } else {
        hi = fmaxf(hi, fabsf(v));
      }
    }
    for (int o = 16; o; o >>= 1) {
      lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
      hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    if ((threadIdx.x & 31) == 0) {
      s_lo[threadIdx.x >> 5] = lo;
      s_hi[threadIdx.x >> 5] = hi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int i = 1; i < (int)(blockDim.x >> 5); ++i) {
        lo = fminf(lo, s_lo[i]);
        hi = fmaxf(hi, s_hi[i]);
      }
      float sc, ze;
      finish_scale(q, lo, hi, &sc, &ze);
      s_scale = sc;
      s_zero = ze;
      scale[r] = sc;
      if (q.kind == 1) zero[r] = ze;
    }
    __syncthreads();
    const float sc = s_scale, ze = s_zero;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
      const float code = code_of(q, row[c], sc, ze);
      if (codes_f32)
        static_cast<float*>(codes)[r * cols + c] = code;
      else
        static_cast<int32_t*>(codes)[r * cols + c] = (int32_t)code;
    }
    __syncthreads();
  }
}

// axis 1: 32 columns per block, 8 row lanes, reduce over rows.
__global__ void quant_cols_stats_kernel(const float* __restrict__ w, int64_t rows, int64_t cols,
                                        QuantSpec q, float* __restrict__ scale,
                                        float* __restrict__ zero) {
  __shared__ float s_lo[8][33], s_hi[8][33];
  const int64_t c = blockIdx.x * 32 + threadIdx.x;
  float lo = FLT_MAX, hi = q.kind == 1 ? -FLT_MAX : 0.0f;
  if (c < cols) {
    for (int64_t r = threadIdx.y; r < rows; r += 8) {
      const float v = w[r * cols + c];
      if (q.kind == 1) {
        lo = fminf(lo, v);
        hi = fmaxf(hi, v);
      } else {
        hi = fmaxf(hi, fabsf(v));
      }
    }
  }
  s_lo[threadIdx.y][threadIdx.x] = lo;
  s_hi[threadIdx.y][threadIdx.x] = hi;
  __syncthreads();
  if (threadIdx.y == 0 && c < cols) {
    for (int i = 1; i < 8; ++i) {
      lo = fminf(lo, s_lo[i][threadIdx.x]);
      hi = fmaxf(hi, s_hi[i][threadIdx.x]);
    }
    float sc, ze;
    finish_scale(q, lo, hi, &sc, &ze);
    scale[c] = sc;
    if (q.kind == 1) zero[c] = ze;
  }
}

// axis None: ordered-integer atomics.  The statistics land in the caller's
// own one-element scale (min, asymmetric only) and zero/scale (max) words, and
// the finishing kernel overwrites them with the real scale and zero point.
__global__ void quant_tensor_init_kernel(uint32_t* lo_slot, uint32_t* hi_slot) {
  if (lo_slot) *lo_slot = 0xFFFFFFFFu;
  *hi_slot = 0u;
}

__global__ void quant_tensor_stats_kernel(const float* __restrict__ w, int64_t n, QuantSpec q,
                                          uint32_t* lo_slot, uint32_t* hi_slot) {
  float lo = FLT_MAX, hi = q.kind == 1 ? -FLT_MAX : 0.0f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = w[i];
    if (q.kind == 1) {
      lo = fminf(lo, v);
      hi = fmaxf(hi, v);
    } else {
      hi = fmaxf(hi, fabsf(v));
    }
  }
  for (int o = 16; o; o >>= 1) {
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  if ((threadIdx.x & 31) == 0) {
    if (lo_slot) atomicMin(lo_slot, ordered_bits(lo));
    atomicMax(hi_slot, ordered_bits(hi));
  }
}

__global__ void quant_tensor_finish_kernel(uint32_t* lo_slot, uint32_t* hi_slot, QuantSpec q,
                                           float* scale, float* zero) {
  const float lo = lo_slot ? from_ordered(*lo_slot) : 0.0f;
  const float hi = from_ordered(*hi_slot);
  float sc, ze;
  finish_scale(q, lo, hi, &sc, &ze);
  scale[0] = sc;
  if (q.kind == 1) zero[0] = ze;
}

__global__ void quant_codes_kernel(const float* __restrict__ w, int64_t rows, int64_t cols,
                                   int axis, QuantSpec q, void* __restrict__ codes,
                                   int codes_f32, const float* __restrict__ scale,
                                   const float* __restrict__ zero) {
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t idx = axis == 1 ? (i % cols) : 0;
    const float sc = scale[idx];
    const float ze = q.kind == 1 ? zero[idx] : 0.0f;
    const float code = code_of(q, w[i], sc, ze);
    if (codes_f32)
      static_cast<float*>(codes)[i] = code;
    else
      static_cast<int32_t*>(codes)[i] = (int32_t)code;
  }
}

int grid_for(int64_t n, int per_thread = 4) {
  int64_t g = (n + (int64_t)kThreads * per_thread - 1) / ((int64_t)kThreads * per_thread);
  if (g < 1) g = 1;
  if (g > 148 * 32) g = 148 * 32;
  return (int)g;
}

int run_quantize(const float* w, int64_t rows, int64_t cols, int axis, QuantSpec q, void* codes,
                 int codes_f32, float* scale, float* zero, cudaStream_t s) {
  IE_CHECK(w && codes && scale, "quantize: null pointer");
  IE_CHECK(rows > 0 && cols > 0, "quantize: empty weight [%lld, %lld]", (long long)rows,
           (long long)cols);
  IE_CHECK(axis == 0 || axis == 1 || axis == -1, "quantize: axis must be 0, 1 or -1 (None)");
  IE_CHECK(q.kind != 1 || zero, "quantize: asymmetric format needs a zero-point buffer");
  if (axis == 0) {
    const int grid = (int)std::min<int64_t>(rows, 148 * 16);
    quant_rows_kernel<<<grid, kThreads, 0, s>>>(w, rows, cols, q, codes, codes_f32, scale, zero);
    return launch_status("quant_rows_kernel");
  }
  if (axis == 1) {
    quant_cols_stats_kernel<<<(int)((cols + 31) / 32), dim3(32, 8), 0, s>>>(w, rows, cols, q,
                                                                              scale, zero);
    int rc = launch_status("quant_cols_stats_kernel");
    if (rc) return rc;
  } else {
    uint32_t* lo_slot = q.kind == 1 ? reinterpret_cast<uint32_t*>(scale) : nullptr;
    uint32_t* hi_slot = reinterpret_cast<uint32_t*>(q.kind == 1 ? zero : scale);
    quant_tensor_init_kernel<<<1, 1, 0, s>>>(lo_slot, hi_slot);
    int rc = launch_status("quant_tensor_init_kernel");
    if (rc) return rc;
    quant_tensor_stats_kernel<<<grid_for(rows * cols), kThreads, 0, s>>>(w, rows * cols, q,
                                                                         lo_slot, hi_slot);
    rc = launch_status("quant_tensor_stats_kernel");
    if (rc) return rc;
    quant_tensor_finish_kernel<<<1, 1, 0, s>>>(lo_slot, hi_slot, q, scale, zero);
    rc = launch_status("quant_tensor_finish_kernel");
    if (rc) return rc;
  }
  quant_codes_kernel<<<grid_for(rows * cols), kThreads, 0, s>>>(w, rows, cols, axis, q, codes,
                                                               codes_f32, scale, zero);
  return launch_status("quant_codes_kernel");
}

// ---------------------------------------------------------------------------
// Packing: reference tables -> K-contiguous device rows.
// ---------------------------------------------------------------------------
// int4 word layout: the 32-bit word covering k0..k0+7 stores the code of
// k0 + kPerm[p] in nibble p, so that (word >> 4p) & 0x000F000F yields the pair
// (k0+2p, k0+2p+1) in the two 16-bit halves.
__constant__ int kPerm[8] = {0, 2, 4, 6, 1, 3, 5, 7};

// int8 / fp8: codes_kn [k][n] -> [n][k] bytes through a 32x32 shared tile.
__global__ void pack_bytes_kernel(const void* __restrict__ codes, int is_fp8, int64_t k,
                                  int64_t n, uint8_t* __restrict__ out,
                                  int32_t* __restrict__ unrepresentable) {
  __shared__ uint8_t tile[32][33];
  const int64_t k0 = (int64_t)blockIdx.y * 32, n0 = (int64_t)blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int64_t kk = k0 + i, nn = n0 + threadIdx.x;
    uint8_t b = 0;
    if (kk < k && nn < n) {
      if (is_fp8) {
        const float v = static_cast<const float*>(codes)[kk * n + nn];
        const __nv_fp8_storage_t e = __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
        b = (uint8_t)e;
        if (unrepresentable) {
          const __half_raw h = __nv_cvt_fp8_to_halfraw(e, __NV_E4M3);
          if (__half2float(__half(h)) != v) atomicAdd(unrepresentable, 1);
        }
      } else {
        b = (uint8_t)(int8_t)static_cast<const int32_t*>(codes)[kk * n + nn];
      }
    }
    tile[i][threadIdx.x] = b;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int64_t nn = n0 + i, kk = k0 + threadIdx.x;
    if (nn < n && kk < k) out[nn * k + kk] = tile[threadIdx.x][i];
  }
}

// int4 from [k][n] codes (symmetric, stored +8): one thread per output word.
// Threads of a warp take consecutive n, so the strided reads stay coalesced.
__global__ void pack_int4_kn_kernel(const int32_t* __restrict__ codes, int64_t k, int64_t n,
                                    uint32_t* __restrict__ out) {
  const int64_t words = k / 8;
  const int64_t total = words * n;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t nn = i % n, wi = i / n;
    uint32_t word = 0;
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      const int32_t q = codes[(wi * 8 + kPerm[p]) * n + nn] + 8;
      word |= ((uint32_t)q & 0xFu) << (4 * p);
    }
    out[nn * words + wi] = word;
  }
}

// int4 group-128 from the [n][k] group view: codes in [0, 15].
__global__ void pack_int4_nk_kernel(const int32_t* __restrict__ codes, int64_t k, int64_t n,
                                    uint32_t* __restrict__ out) {
  const int64_t words = k / 8;
  const int64_t total = words * n;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t nn = i / words, wi = i % words;
    const int32_t* src = codes + nn * k + wi * 8;
    uint32_t word = 0;
#pragma unroll
    for (int p = 0; p < 8; ++p) word |= ((uint32_t)src[kPerm[p]] & 0xFu) << (4 * p);
    out[i] = word;
  }
}

// f32 group tables [n][k/128] (the reference's view order) -> f16 tables
// [k/128][n], N-contiguous so one K group of 128 consecutive rows is one
// contiguous run.  A zero point that f16 cannot hold exactly, or a scale that
// overflows / flushes in f16, is counted as unrepresentable.
__global__ void pack_group_tables_kernel(const float* __restrict__ scale,
                                         const float* __restrict__ zero, int64_t n,
                                         int64_t groups, __half* __restrict__ s16,
                                         __half* __restrict__ z16,
                                         int32_t* __restrict__ unrepresentable) {
  const int64_t count = n * groups;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t g = i / n, nn = i % n;
    const float s = scale[nn * groups + g], z = zero[nn * groups + g];
    const __half hs = __float2half_rn(s), hz = __float2half_rn(z);
    s16[i] = hs;
    z16[i] = hz;
    if (unrepresentable) {
      const float bs = __half2float(hs);
      const bool bad_s = !(isfinite(bs)) || (bs == 0.0f && s != 0.0f);
      const bool bad_z = __half2float(hz) != z;
      if (bad_s || bad_z) atomicAdd(unrepresentable, 1);
    }
  }
}

// ---------------------------------------------------------------------------
// Dequantize a packed weight (ie/quant/weights.py:22-26).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float packed_code(const ie_qweight& w, int64_t row, int64_t kk) {
  const uint8_t* base = static_cast<const uint8_t*>(w.codes);
  if (w.format == IE_FMT_INT4) {
    const int64_t words = w.k / 8;
    const uint32_t word = reinterpret_cast<const uint32_t*>(base)[row * words + kk / 8];
    const int j = (int)(kk & 7);
    const int p = (j & 1) ? 4 + (j >> 1) : (j >> 1);   // inverse of kPerm
    return (float)((word >> (4 * p)) & 0xFu);
  }
  const uint8_t b = base[row * w.k + kk];
  if (w.format == IE_FMT_INT8) return (float)(int8_t)b;
  const __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3);
  return __half2float(__half(h));
}

__device__ __forceinline__ float dequant_value(const ie_qweight& w, int64_t row, int64_t kk) {
  float q = packed_code(w, row, kk);
  const float* sc = static_cast<const float*>(w.scale);
  if (w.axis == IE_AXIS_GROUP128) {
    const int64_t gi = (kk / 128) * w.n + row;
    const float s = __half2float(static_cast<const __half*>(w.scale)[gi]);
    const float z = __half2float(static_cast<const __half*>(w.zero)[gi]);
    return __fmul_rn(__fsub_rn(q, z), s);
  }
  if (w.format == IE_FMT_INT4 && w.int4_symmetric) q -= 8.0f;
  const int half = w.gate_up ? (int)(row & 1) : 0;
  float s;
  if (w.axis == IE_AXIS_K) s = sc[half * w.k + kk];
  else if (w.axis == IE_AXIS_N) s = sc[row];
  else s = sc[half];
  return __fmul_rn(q, s);
}

template <typename T>
__global__ void dequant_kernel(ie_qweight w, int layout, T* __restrict__ out) {
  const int64_t total = w.k * w.n;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    if (layout == 0) {  // [k][n]
      const int64_t kk = i / w.n, row = i % w.n;
      out[i] = from_f32<T>(dequant_value(w, row, kk));
    } else {            // [n][k]
      const int64_t row = i / w.k, kk = i % w.k;
      out[i] = from_f32<T>(dequant_value(w, row, kk));
    }
  }
}

}  // namespace

int validate_qweight(const ie_qweight& w) {
  IE_CHECK(w.codes && w.scale, "qweight: null codes or scale");
  IE_CHECK(w.k > 0 && w.n > 0, "qweight: empty shape");
  IE_CHECK(w.format == IE_FMT_INT8 || w.format == IE_FMT_INT4 || w.format == IE_FMT_FP8_E4M3,
           "qweight: unknown format %d", w.format);
  IE_CHECK(w.axis >= IE_AXIS_K && w.axis <= IE_AXIS_GROUP128, "qweight: unknown axis %d", w.axis);
  if (w.axis == IE_AXIS_GROUP128) {
    IE_CHECK(w.format == IE_FMT_INT4 && !w.int4_symmetric,
             "qweight: group-128 tables are for asymmetric int4");
    IE_CHECK(w.zero != nullptr, "qweight: group-128 needs zero points");
    IE_CHECK(w.k % 128 == 0, "qweight: K=%lld is not a multiple of 128", (long long)w.k);
  }
  if (w.format == IE_FMT_INT4) {
    IE_CHECK(w.k % 32 == 0, "qweight: int4 needs K %% 32 == 0 (K=%lld)", (long long)w.k);
    IE_CHECK(w.axis == IE_AXIS_GROUP128 || w.int4_symmetric,
             "qweight: asymmetric int4 is supported with group-128 tables");
  } else {
    IE_CHECK(w.k % 16 == 0, "qweight: 8-bit codes need K %% 16 == 0 (K=%lld)", (long long)w.k);
  }
  if (w.gate_up) IE_CHECK(w.n % 2 == 0, "qweight: gate/up pairs need an even row count");
  IE_CHECK(((uintptr_t)w.codes & 15) == 0, "qweight: codes must be 16-byte aligned");
  return IE_OK;
}

}  // namespace ie

using namespace ie;

extern "C" int ie_round_to_float_format(const float* x, float* out, int64_t count,
                                        int32_t exponent_bits, int32_t mantissa_bits,
                                        int32_t reserves_infinity, void* stream) {
  IE_CHECK(count >= 0, "round_to_float_format: negative count");
  IE_CHECK(exponent_bits >= 2 && exponent_bits <= 8 && mantissa_bits >= 1 && mantissa_bits <= 10,
           "round_to_float_format: unsupported format e%dm%d", exponent_bits, mantissa_bits);
  if (count == 0) return IE_OK;
  IE_CHECK(x && out, "round_to_float_format: null pointer");
  round_kernel<<<grid_for(count), kThreads, 0, as_stream(stream)>>>(
      x, out, count, make_float_fmt(exponent_bits, mantissa_bits, reserves_infinity));
  return launch_status("round_kernel");
}

extern "C" int ie_quantize_integer(const float* w, int64_t rows, int64_t cols, int32_t bits,
                                   int32_t symmetric, int32_t axis, int32_t* codes,
                                   float* scale, float* zero, void* stream) {
  IE_CHECK(bits >= 2 && bits <= 16, "quantize_integer: bits must be in [2, 16], got %d", bits);
  QuantSpec q{};
  q.kind = symmetric ? 0 : 1;
  q.qmax = symmetric ? ((1 << bits) / 2 - 1) : ((1 << bits) - 1);
  return run_quantize(w, rows, cols, axis, q, codes, 0, scale, zero, as_stream(stream));
}

extern "C" int ie_quantize_float(const float* w, int64_t rows, int64_t cols,
                                 int32_t exponent_bits, int32_t mantissa_bits,
                                 int32_t reserves_infinity, int32_t axis, float* codes,
                                 float* scale, void* stream) {
  IE_CHECK(exponent_bits >= 2 && exponent_bits <= 8 && mantissa_bits >= 1 && mantissa_bits <= 10,
           "quantize_float: unsupported format e%dm%d", exponent_bits, mantissa_bits);
  QuantSpec q{};
  q.kind = 2;
  q.ff = make_float_fmt(exponent_bits, mantissa_bits, reserves_infinity);
  return run_quantize(w, rows, cols, axis, q, codes, 1, scale, nullptr, as_stream(stream));
}

extern "C" int ie_pack_weight(int32_t format, int32_t axis, int32_t int4_symmetric, int64_t k,
                              int64_t n, const void* codes, const float* scale_f32,
                              const float* zero_f32, void* out_codes, void* out_scale16,
                              void* out_zero16, int32_t* unrepresentable, void* stream) {
  cudaStream_t s = as_stream(stream);
  IE_CHECK(codes && out_codes, "pack_weight: null pointer");
  IE_CHECK(k > 0 && n > 0, "pack_weight: empty shape");
  IE_CHECK(((uintptr_t)out_codes & 15) == 0, "pack_weight: output must be 16-byte aligned");
  if (format == IE_FMT_INT8 || format == IE_FMT_FP8_E4M3) {
    IE_CHECK(axis != IE_AXIS_GROUP128, "pack_weight: group-128 tables are for int4");
    dim3 grid((unsigned)((n + 31) / 32), (unsigned)((k + 31) / 32));
    pack_bytes_kernel<<<grid, dim3(32, 8), 0, s>>>(codes, format == IE_FMT_FP8_E4M3, k, n,
                                                   static_cast<uint8_t*>(out_codes),
                                                   unrepresentable);
    return launch_status("pack_bytes_kernel");
  }
  IE_CHECK(format == IE_FMT_INT4, "pack_weight: unknown format %d", format);
  IE_CHECK(k % 32 == 0, "pack_weight: int4 needs K %% 32 == 0 (K=%lld)", (long long)k);
  const int64_t total = (k / 8) * n;
  if (axis == IE_AXIS_GROUP128) {
    IE_CHECK(k % 128 == 0, "pack_weight: K=%lld is not a multiple of 128", (long long)k);
    IE_CHECK(scale_f32 && zero_f32 && out_scale16 && out_zero16,
             "pack_weight: group-128 needs f32 scale/zero inputs and f16 outputs");
    pack_int4_nk_kernel<<<grid_for(total, 1), kThreads, 0, s>>>(
        static_cast<const int32_t*>(codes), k, n, static_cast<uint32_t*>(out_codes));
    int rc = launch_status("pack_int4_nk_kernel");
    if (rc) return rc;
    const int64_t groups = k / 128;
    pack_group_tables_kernel<<<grid_for(groups * n), kThreads, 0, s>>>(
        scale_f32, zero_f32, n, groups, static_cast<__half*>(out_scale16),
        static_cast<__half*>(out_zero16), unrepresentable);
    return launch_status("pack_group_tables_kernel");
  }
  IE_CHECK(int4_symmetric, "pack_weight: per-axis int4 must be symmetric (codes in [-7, 7])");
  pack_int4_kn_kernel<<<grid_for(total, 1), kThreads, 0, s>>>(
      static_cast<const int32_t*>(codes), k, n, static_cast<uint32_t*>(out_codes));
  return launch_status("pack_int4_kn_kernel");
}

extern "C" int ie_dequantize(const ie_qweight* w, int32_t layout, int32_t out_dtype, void* out,
                             void* stream) {
  IE_CHECK(w && out, "dequantize: null pointer");
  int rc = validate_qweight(*w);
  if (rc) return rc;
  IE_CHECK(layout == 0 || layout == 1, "dequantize: layout must be 0 ([k][n]) or 1 ([n][k])");
  cudaStream_t s = as_stream(stream);
  const int grid = grid_for(w->k * w->n);
  if (out_dtype == IE_DT_F32)
    dequant_kernel<float><<<grid, kThreads, 0, s>>>(*w, layout, static_cast<float*>(out));
  else if (out_dtype == IE_DT_BF16)
    dequant_kernel<__nv_bfloat16><<<grid, kThreads, 0, s>>>(*w, layout,
                                                            static_cast<__nv_bfloat16*>(out));
  else if (out_dtype == IE_DT_F16)
    dequant_kernel<__half><<<grid, kThreads, 0, s>>>(*w, layout, static_cast<__half*>(out));
  else
    return set_error(IE_ERR_INVALID, "dequantize: unsupported output dtype %d", out_dtype);
  return launch_status("dequant_kernel");
}
