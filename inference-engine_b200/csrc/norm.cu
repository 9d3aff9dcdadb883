// RMSNorm over the hidden dimension (ie/layers/functional.py:6-8):
//   out = x / sqrt(mean(x^2) + eps) * weight, accumulated in f32.
// One CTA per token row.  Rows whose length and strides allow it are read with
// 16-byte vector loads into registers once (both passes use them); other rows
// take a scalar loop.  The two differ only in the order of the f32 sum of
// squares (an ulp of the mean at most); the scaling is the same f32 division.
#include "common.cuh"

namespace ie {
namespace norm_detail {

constexpr int kThreads = 256;

template <typename TI, typename TO>
__global__ void __launch_bounds__(kThreads)
rms_norm_kernel(const TI* __restrict__ x, int64_t ldx, const float* __restrict__ w,
                TO* __restrict__ out, int64_t ldo, int64_t m, int64_t h, float eps) {
  __shared__ float red[kThreads / 32];
  for (int64_t row = blockIdx.x; row < m; row += gridDim.x) {
    const TI* xr = x + row * ldx;
    float ss = 0.0f;
    for (int64_t i = threadIdx.x; i < h; i += kThreads) {
      const float v = to_f32<TI>(xr[i]);
      ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int i = 0; i < kThreads / 32; ++i) tot += red[i];
    const float denom = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)h), eps));
    for (int64_t i = threadIdx.x; i < h; i += kThreads)
      out[row * ldo + i] = from_f32<TO>(__fdiv_rn(to_f32<TI>(xr[i]), denom) * w[i]);
    __syncthreads();
  }
}

// 8 elements per 16 bytes of bf16/f16 (two float4 for f32); up to kMaxChunks
// chunks of 8 per thread, so rows up to 8 * 8 * kThreads = 16384 elements.
constexpr int kMaxChunks = 8;

template <typename TI> __device__ __forceinline__ void load8(const TI* p, float (&v)[8]);
template <> __device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p,
                                                                 float (&v)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
template <> __device__ __forceinline__ void load8<__half>(const __half* p, float (&v)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <> __device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

template <typename TI, typename TO>
__global__ void __launch_bounds__(kThreads)
rms_norm_vec_kernel(const TI* __restrict__ x, int64_t ldx, const float* __restrict__ w,
                    TO* __restrict__ out, int64_t ldo, int64_t m, int64_t h, float eps) {
  __shared__ float red[kThreads / 32];
  for (int64_t row = blockIdx.x; row < m; row += gridDim.x) {
    const TI* xr = x + row * ldx;
    float v[kMaxChunks][8];
    float ss = 0.0f;
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
      const int64_t i = ((int64_t)c * kThreads + threadIdx.x) * 8;
      if (i < h) {
        load8<TI>(xr + i, v[c]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[c][j] = 0.0f;
      }
    }
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c)
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(v[c][j], v[c][j], ss);
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int i = 0; i < kThreads / 32; ++i) tot += red[i];
    const float denom = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)h), eps));
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
      const int64_t i = ((int64_t)c * kThreads + threadIdx.x) * 8;
      if (i < h) {
        const float4 w0 = __ldg(reinterpret_cast<const float4*>(w + i));
        const float4 w1 = __ldg(reinterpret_cast<const float4*>(w + i) + 1);
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j)
          out[row * ldo + i + j] = from_f32<TO>(__fdiv_rn(v[c][j], denom) * wv[j]);
      }
    }
    __syncthreads();
  }
}

template <typename TI>
int launch_to(int out_dtype, const void* x, int64_t ldx, const float* w, void* out, int64_t ldo,
              int64_t m, int64_t h, float eps, cudaStream_t s) {
  const int grid = (int)(m < 148 * 8 ? m : 148 * 8);
  const bool vec = h % 8 == 0 && ldx % 8 == 0 && h <= (int64_t)kMaxChunks * 8 * kThreads &&
                   (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(w) & 15) == 0;
  if (vec) {
    if (out_dtype == IE_DT_F32)
      rms_norm_vec_kernel<TI, float><<<grid, kThreads, 0, s>>>(
          static_cast<const TI*>(x), ldx, w, static_cast<float*>(out), ldo, m, h, eps);
    else if (out_dtype == IE_DT_BF16)
      rms_norm_vec_kernel<TI, __nv_bfloat16><<<grid, kThreads, 0, s>>>(
          static_cast<const TI*>(x), ldx, w, static_cast<__nv_bfloat16*>(out), ldo, m, h, eps);
    else if (out_dtype == IE_DT_F16)
      rms_norm_vec_kernel<TI, __half><<<grid, kThreads, 0, s>>>(
          static_cast<const TI*>(x), ldx, w, static_cast<__half*>(out), ldo, m, h, eps);
    else
      return set_error(IE_ERR_INVALID, "rms_norm: unsupported output dtype %d", out_dtype);
    return launch_status("rms_norm_vec_kernel");
  }
  if (out_dtype == IE_DT_F32)
    rms_norm_kernel<TI, float><<<grid, kThreads, 0, s>>>(static_cast<const TI*>(x), ldx, w,
                                                         static_cast<float*>(out), ldo, m, h, eps);
  else if (out_dtype == IE_DT_BF16)
    rms_norm_kernel<TI, __nv_bfloat16><<<grid, kThreads, 0, s>>>(
        static_cast<const TI*>(x), ldx, w, static_cast<__nv_bfloat16*>(out), ldo, m, h, eps);
  else if (out_dtype == IE_DT_F16)
    rms_norm_kernel<TI, __half><<<grid, kThreads, 0, s>>>(static_cast<const TI*>(x), ldx, w,
                                                          static_cast<__half*>(out), ldo, m, h,
                                                          eps);
  else
    return set_error(IE_ERR_INVALID, "rms_norm: unsupported output dtype %d", out_dtype);
  return launch_status("rms_norm_kernel");
}

}  // namespace norm_detail
}  // namespace ie

using namespace ie;
using namespace ie::norm_detail;

extern "C" int ie_rms_norm(const void* x, int64_t ldx, int32_t x_dtype, const float* weight,
                           void* out, int64_t ldo, int32_t out_dtype, int64_t m, int64_t h,
                           float eps, void* stream) {
  IE_CHECK(m >= 0 && h > 0, "rms_norm: bad shape [%lld, %lld]", (long long)m, (long long)h);
  if (m == 0) return IE_OK;
  IE_CHECK(x && weight && out, "rms_norm: null pointer");
  IE_CHECK(ldx >= h && ldo >= h, "rms_norm: row stride smaller than the hidden size");
  cudaStream_t s = as_stream(stream);
  if (x_dtype == IE_DT_F32) return launch_to<float>(out_dtype, x, ldx, weight, out, ldo, m, h, eps, s);
  if (x_dtype == IE_DT_BF16)
    return launch_to<__nv_bfloat16>(out_dtype, x, ldx, weight, out, ldo, m, h, eps, s);
  if (x_dtype == IE_DT_F16) return launch_to<__half>(out_dtype, x, ldx, weight, out, ldo, m, h, eps, s);
  return set_error(IE_ERR_INVALID, "rms_norm: unsupported input dtype %d", x_dtype);
}
