// RMSNorm over the hidden dimension (ie/layers/functional.py:6-8):
//   out = x / sqrt(mean(x^2) + eps) * weight, accumulated in f32.
// One CTA per token row; the row is read once into registers.
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

template <typename TI>
int launch_to(int out_dtype, const void* x, int64_t ldx, const float* w, void* out, int64_t ldo,
              int64_t m, int64_t h, float eps, cudaStream_t s) {
  const int grid = (int)(m < 148 * 8 ? m : 148 * 8);
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
