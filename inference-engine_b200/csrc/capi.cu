// extern "C" entry points of libie_tpq.so that are not tied to one kernel
// family: version, error reporting, argument validation and dispatch of the
// quantized linear layer (single-rank and fused with the all-reduce), and the
// in-process reduction of a list of partials.
#include <algorithm>
#include <cstring>

#include "common.cuh"

namespace ie {

namespace {
thread_local char g_err[512] = "";
}

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

const char* last_error() { return g_err; }

namespace {

int validate_linear(const ie_qlinear_args& a) {
  int rc = validate_qweight(a.w);
  if (rc) return rc;
  IE_CHECK(a.m >= 0, "qlinear: negative token count");
  IE_CHECK(a.act_dtype == IE_DT_BF16 || a.act_dtype == IE_DT_F16 || a.act_dtype == IE_DT_F32,
           "qlinear: unsupported activation dtype %d", a.act_dtype);
  IE_CHECK(a.out_dtype == IE_DT_BF16 || a.out_dtype == IE_DT_F16 || a.out_dtype == IE_DT_F32,
           "qlinear: unsupported output dtype %d", a.out_dtype);
  if (a.m == 0) return IE_OK;
  IE_CHECK(a.x && a.out, "qlinear: null x or out");
  IE_CHECK(a.ldx >= a.w.k, "qlinear: ldx %lld < K %lld", (long long)a.ldx, (long long)a.w.k);
  const int64_t ncols = (a.epilogue & IE_EPI_SILU_MUL) ? a.w.n / 2 : a.w.n;
  IE_CHECK(a.ldo >= ncols, "qlinear: ldo %lld < output columns %lld", (long long)a.ldo,
           (long long)ncols);
  if (a.epilogue & IE_EPI_SILU_MUL)
    IE_CHECK(a.w.gate_up, "qlinear: SILU_MUL needs a weight packed as gate/up row pairs");
  if (a.epilogue & IE_EPI_BIAS) IE_CHECK(a.bias, "qlinear: BIAS flag without a bias pointer");
  if (a.epilogue & IE_EPI_RESIDUAL) {
    IE_CHECK(a.residual, "qlinear: RESIDUAL flag without a residual pointer");
    IE_CHECK(a.ldr >= ncols, "qlinear: ldr %lld < output columns", (long long)a.ldr);
  }
  IE_CHECK((a.epilogue & ~(IE_EPI_BIAS | IE_EPI_RESIDUAL | IE_EPI_SILU_MUL | IE_EPI_RMS_NORM)) ==
               0,
           "qlinear: unknown epilogue flags 0x%x", a.epilogue);
  if (a.epilogue & IE_EPI_RMS_NORM) {
    IE_CHECK(a.norm_weight, "qlinear: RMS_NORM flag without a norm weight");
    IE_CHECK(a.norm_eps >= 0.0f, "qlinear: negative norm eps");
    IE_CHECK(a.algo != 1 || gemv_decode_ok(a),
             "qlinear: the fused RMS norm runs on the tensor-core path, or on the "
             "weight-streaming path for at most two tokens");
  }
  IE_CHECK(a.algo >= 0 && a.algo <= 2, "qlinear: unknown algo %d", a.algo);
  IE_CHECK(a.act_quant == IE_ACT_NONE || a.act_quant == IE_ACT_FP8_TOKEN,
           "qlinear: unknown act_quant %d", a.act_quant);
  if (a.act_quant == IE_ACT_FP8_TOKEN) {
    IE_CHECK(a.w.format == IE_FMT_FP8_E4M3 &&
                 (a.w.axis == IE_AXIS_N || a.w.axis == IE_AXIS_TENSOR),
             "qlinear: fp8 activations need an FP8 weight with per-N or per-tensor scales "
             "(per-K scales vary along the contraction)");
    IE_CHECK(a.act_dtype == IE_DT_BF16 || a.act_dtype == IE_DT_F16,
             "qlinear: fp8 activations are quantized from bf16/f16 x");
    IE_CHECK(a.algo != 1 && !(a.epilogue & IE_EPI_RMS_NORM),
             "qlinear: fp8 activations run on the tensor-core path, without the fused norm");
    IE_CHECK(a.w.k % 128 == 0, "qlinear: fp8 activations need K %% 128 == 0");
  }
  return IE_OK;
}

// Auto routing (algo 0): every bf16/f16 batch takes the tensor-core kernel.
// Measured on B200 over Llama-3-8B layers with distinct weights (nothing
// reused from L2), the decode GEMV is slower from a single token on (o 14.6
// against 13.3 us, gate/up 38.2 against 36.7 us); it serves algo 1 and f32
// activations.
bool use_tc(const ie_qlinear_args& a) {
  if (a.algo == 1) return false;
  if (a.algo == 2) return true;
  return tc_usable(a);
}

// The fused all-reduce runs on the tensor-core kernel whenever it can (the
// decode GEMV has no all-reduce; the general one streams far slower).
bool use_tc_reduce(const ie_qlinear_args& a) {
  if (a.algo == 1) return false;
  if (a.algo == 2) return true;
  return tc_usable(a);
}

}  // namespace
}  // namespace ie

using namespace ie;

extern "C" int ie_version(void) { return IE_TPQ_ABI_VERSION; }

extern "C" int ie_last_error(char* buf, size_t n) {
  if (!buf || n == 0) return IE_ERR_INVALID;
  std::strncpy(buf, last_error(), n - 1);
  buf[n - 1] = '\0';
  return IE_OK;
}

extern "C" size_t ie_qlinear_workspace_size(const ie_qlinear_args* a) {
  if (!a || validate_linear(*a) != IE_OK || a->m == 0 || !use_tc(*a)) return 0;
  return tc_workspace_bytes(*a);
}

extern "C" int ie_qlinear(const ie_qlinear_args* a, void* stream) {
  IE_CHECK(a, "qlinear: null args");
  int rc = validate_linear(*a);
  if (rc || a->m == 0) return rc;
  if (use_tc(*a)) return launch_qlinear_tc(*a, nullptr, as_stream(stream));
  if ((a->epilogue & IE_EPI_RMS_NORM) && !gemv_decode_ok(*a))
    return set_error(IE_ERR_UNSUPPORTED, "qlinear: the fused RMS norm needs bf16/f16 "
                                         "activations, K %% 128 == 0 and aligned rows, or "
                                         "at most two tokens");
  return launch_qlinear_gemv(*a, nullptr, 0, as_stream(stream));
}

extern "C" int ie_qlinear_noalloc(const ie_qlinear_args* a, void* stream) {
  IE_CHECK(a, "qlinear_noalloc: null args");
  int rc = validate_linear(*a);
  if (rc) return rc;
  return launch_qlinear_tc_static(*a, as_stream(stream));
}

extern "C" int ie_kernel_status(uint32_t* bits, int32_t clear) {
  IE_CHECK(bits, "kernel_status: null output");
  *bits = tc_read_status(clear != 0);
  return IE_OK;
}

extern "C" int ie_qlinear_allreduce(ie_comm* c, const ie_qlinear_args* a, int32_t algo,
                                    void* stream) {
  IE_CHECK(c && a, "qlinear_allreduce: null pointer");
  int rc = validate_linear(*a);
  if (rc || a->m == 0) return rc;
  IE_CHECK(!(a->epilogue & IE_EPI_SILU_MUL),
           "qlinear_allreduce: SILU_MUL belongs to the column-parallel gate/up layer");
  IE_CHECK(!a->w.gate_up, "qlinear_allreduce: gate/up pairs are column-parallel");
  if (use_tc_reduce(*a)) {
    ReduceCtx ctx;
    rc = comm_context(c, &ctx, tc_tiles(*a), a->m * a->w.n, algo);
    if (rc) return rc;
    return launch_qlinear_tc(*a, &ctx, as_stream(stream));
  }
  if (a->epilogue & IE_EPI_RMS_NORM)
    return set_error(IE_ERR_UNSUPPORTED, "qlinear_allreduce: the fused RMS norm needs bf16/f16 "
                                         "activations, K %% 128 == 0 and aligned rows");
  int resident = 0;
  rc = gemv_resident_ctas(*a, &resident);
  if (rc) return rc;
  IE_CHECK(resident > 0, "qlinear_allreduce: kernel cannot be resident on this device");
  ReduceCtx ctx;
  rc = comm_context(c, &ctx, gemv_tiles(*a), a->m * a->w.n, algo);
  if (rc) return rc;
  return launch_qlinear_gemv(*a, &ctx, resident, as_stream(stream));
}

namespace ie {
namespace reduce_detail {

constexpr int kMaxPartials = 64;
struct PartialList {
  const void* p[kMaxPartials];
};

template <typename T>
__global__ void reduce_partials_kernel(PartialList pl, int count, T* __restrict__ out,
                                       int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float v = to_f32<T>(static_cast<const T*>(pl.p[0])[i]);
    for (int r = 1; r < count; ++r) v += to_f32<T>(static_cast<const T*>(pl.p[r])[i]);
    out[i] = from_f32<T>(v);
  }
}

}  // namespace reduce_detail
}  // namespace ie

using namespace ie::reduce_detail;

extern "C" int ie_reduce_partials(const void* const* partials, int32_t count, void* out,
                                  int64_t numel, int32_t dtype, void* stream) {
  IE_CHECK(partials && out, "reduce_partials: null pointer");
  IE_CHECK(count >= 1 && count <= kMaxPartials, "reduce_partials: %d partials outside [1, %d]",
           count, kMaxPartials);
  IE_CHECK(numel >= 0, "reduce_partials: negative size");
  if (numel == 0) return IE_OK;
  PartialList pl{};
  for (int i = 0; i < count; ++i) {
    IE_CHECK(partials[i], "reduce_partials: partial %d is null", i);
    pl.p[i] = partials[i];
  }
  cudaStream_t s = as_stream(stream);
  const int threads = 256;
  const int grid = (int)std::min<int64_t>((numel + threads * 4 - 1) / (threads * 4), 148 * 16);
  if (dtype == IE_DT_F32)
    reduce_partials_kernel<float><<<grid, threads, 0, s>>>(pl, count, static_cast<float*>(out),
                                                           numel);
  else if (dtype == IE_DT_BF16)
    reduce_partials_kernel<__nv_bfloat16><<<grid, threads, 0, s>>>(
        pl, count, static_cast<__nv_bfloat16*>(out), numel);
  else if (dtype == IE_DT_F16)
    reduce_partials_kernel<__half><<<grid, threads, 0, s>>>(pl, count, static_cast<__half*>(out),
                                                            numel);
  else
    return set_error(IE_ERR_INVALID, "reduce_partials: unsupported dtype %d", dtype);
  return launch_status("reduce_partials_kernel");
}
