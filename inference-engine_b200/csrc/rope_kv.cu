// Rotary embedding of q and k plus the KV-cache write, in one kernel, for the
// output of the fused q|k|v projection.
//
// The reference applies RoPE to q and k (ie/layers/functional.py:34-61,
// ie/kernels/torch_backend.py) and then writes k and v into the paged cache
// at each token's slot (ie/kernels/torch_backend.py:13-16); on the GPU that is
// a dozen elementwise launches per layer.  Here one thread takes one (token,
// head, rotation pair): a q or k pair is rotated and stored to q_out or to the
// token's cache slot, a v pair is copied to its slot.  The arithmetic is the
// elementwise tensor arithmetic of those steps in the activation type: cos and
// sin rounded to it, every product and the sum / difference rounded to it
// (for bf16 and f16 each step computes in f32 and rounds once, as the
// elementwise kernels of a tensor library do), so the result is bitwise equal
// to the unfused steps.
#include "common.cuh"

namespace ie {
namespace rope_detail {

constexpr int kThreads = 256;

// _rn intrinsics: each product rounded on its own, never contracted into an
// FMA with the following sum (which would round once for both)
template <typename T>
__device__ __forceinline__ T rmul(T a, T b) {
  return from_f32<T>(__fmul_rn(to_f32<T>(a), to_f32<T>(b)));
}
template <typename T>
__device__ __forceinline__ T radd(T a, T b) {
  return from_f32<T>(__fadd_rn(to_f32<T>(a), to_f32<T>(b)));
}
template <typename T>
__device__ __forceinline__ T rsub(T a, T b) {
  return from_f32<T>(__fsub_rn(to_f32<T>(a), to_f32<T>(b)));
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
rope_kv_kernel(const T* __restrict__ qkv, int64_t ld, int64_t tokens, int nh, int nkv, int hd,
               const int64_t* __restrict__ positions, const float* __restrict__ cos_t,
               const float* __restrict__ sin_t, int64_t max_pos, int halved,
               const int64_t* __restrict__ slots, int64_t cache_slots, T* __restrict__ kc,
               T* __restrict__ vc, T* __restrict__ q_out) {
  const int pairs = hd / 2;
  const int64_t per_tok = (int64_t)(nh + 2 * nkv) * pairs;
  const int64_t total = tokens * per_tok;
  for (int64_t idx = (int64_t)blockIdx.x * kThreads + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * kThreads) {
    const int64_t t = idx / per_tok;
    const int r = (int)(idx - t * per_tok);
    const int head = r / pairs, i = r - head * pairs;
    const T* src = qkv + t * ld + (int64_t)head * hd;
    const int64_t slot = slots[t];
    const bool slot_ok = slot >= 0 && slot < cache_slots;
    // element pair: interleaved (2i, 2i+1) or halved (i, i + hd/2)
    const int e0 = halved ? i : 2 * i, e1 = halved ? i + pairs : 2 * i + 1;
    if (head >= nh + nkv) {   // v: copied to the cache
      if (slot_ok) {
        T* dst = vc + (slot * nkv + (head - nh - nkv)) * (int64_t)hd;
        dst[e0] = src[e0];
        dst[e1] = src[e1];
      }
      continue;
    }
    const int64_t pos = positions[t];
    if (pos < 0 || pos >= max_pos) continue;
    const T c = from_f32<T>(cos_t[pos * pairs + i]);
    const T s = from_f32<T>(sin_t[pos * pairs + i]);
    const T a = src[e0], b = src[e1];
    // interleaved: (a c - b s, a s + b c); halved: (a c - b s, b c + a s)
    const T o0 = rsub(rmul(a, c), rmul(b, s));
    const T o1 = halved ? radd(rmul(b, c), rmul(a, s)) : radd(rmul(a, s), rmul(b, c));
    T* dst;
    if (head < nh) {
      dst = q_out + (t * nh + head) * (int64_t)hd;
    } else {
      if (!slot_ok) continue;
      dst = kc + (slot * nkv + (head - nh)) * (int64_t)hd;
    }
    dst[e0] = o0;
    dst[e1] = o1;
  }
}

template <typename T>
int launch(const void* qkv, int64_t ld, int64_t tokens, int nh, int nkv, int hd,
           const int64_t* positions, const float* cos_t, const float* sin_t, int64_t max_pos,
           int halved, const int64_t* slots, int64_t cache_slots, void* kc, void* vc,
           void* q_out, cudaStream_t s) {
  const int64_t total = tokens * (int64_t)(nh + 2 * nkv) * (hd / 2);
  const int64_t want = (total + kThreads - 1) / kThreads;
  const int grid = (int)(want < 4096 ? want : 4096);
  rope_kv_kernel<T><<<grid, kThreads, 0, s>>>(
      static_cast<const T*>(qkv), ld, tokens, nh, nkv, hd, positions, cos_t, sin_t, max_pos,
      halved, slots, cache_slots, static_cast<T*>(kc), static_cast<T*>(vc),
      static_cast<T*>(q_out));
  return launch_status("rope_kv_kernel");
}

}  // namespace rope_detail
}  // namespace ie

using namespace ie;

extern "C" int ie_rope_kv(const void* qkv, int64_t ld_qkv, int32_t dtype, int64_t tokens,
                          int32_t heads, int32_t kv_heads, int32_t head_dim,
                          const int64_t* positions, const float* cos_table,
                          const float* sin_table, int64_t max_position, int32_t halved,
                          const int64_t* slots, void* k_cache, void* v_cache,
                          int64_t cache_slots, void* q_out, void* stream) {
  IE_CHECK(tokens >= 0 && heads > 0 && kv_heads > 0 && head_dim > 0 && head_dim % 2 == 0,
           "rope_kv: bad shape (tokens %lld, heads %d, kv heads %d, head dim %d)",
           (long long)tokens, heads, kv_heads, head_dim);
  IE_CHECK(ld_qkv >= (int64_t)(heads + 2 * kv_heads) * head_dim,
           "rope_kv: row stride %lld < q|k|v width", (long long)ld_qkv);
  if (tokens == 0) return IE_OK;
  IE_CHECK(qkv && positions && cos_table && sin_table && slots && k_cache && v_cache && q_out,
           "rope_kv: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  using namespace rope_detail;
  if (dtype == IE_DT_BF16)
    return launch<__nv_bfloat16>(qkv, ld_qkv, tokens, heads, kv_heads, head_dim, positions,
                                 cos_table, sin_table, max_position, halved, slots, cache_slots,
                                 k_cache, v_cache, q_out, s);
  if (dtype == IE_DT_F16)
    return launch<__half>(qkv, ld_qkv, tokens, heads, kv_heads, head_dim, positions, cos_table,
                          sin_table, max_position, halved, slots, cache_slots, k_cache, v_cache,
                          q_out, s);
  if (dtype == IE_DT_F32)
    return launch<float>(qkv, ld_qkv, tokens, heads, kv_heads, head_dim, positions, cos_table,
                         sin_table, max_position, halved, slots, cache_slots, k_cache, v_cache,
                         q_out, s);
  return set_error(IE_ERR_INVALID, "rope_kv: unsupported dtype %d", dtype);
}
