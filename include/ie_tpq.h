/*
 * ie_tpq.h -- C ABI of libie_tpq.so, the B200 (sm_100a) tensor-parallel
 * quantized linear path.
 *
 * This is the drop-in boundary for the reference engine's column-/row-parallel
 * Linear layers (ie/parallel/sharding.py) combined with its int8 / int4 / fp8
 * weight formats (ie/quant/).  Everything crossing it is a plain pointer, an
 * integer or a POD struct: no C++ or torch types.  Device pointers are raw
 * CUDA addresses; `stream` is a cudaStream_t passed as void*.
 *
 * Conventions
 *   - Every entry point returns IE_OK (0) or an error code; the message of the
 *     last failure on the calling thread is available from ie_last_error().
 *   - Nothing synchronises the host: work is enqueued on the caller's stream.
 *   - The caller owns inputs, outputs and workspace.  The library owns only
 *     what ie_comm_create() allocates (landing buffers, flags, status word).
 *   - Weight layout of the reference: W is [K_in, N_out] and y = x @ W
 *     (ie/model/transformer.py:48-61).  Packed device layouts are K-contiguous
 *     per output row ([N, K]) so that the weight streams row by row.
 */
#ifndef IE_TPQ_H
#define IE_TPQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define IE_TPQ_ABI_VERSION 4   /* 2: ie_qlinear_args gained norm_weight / norm_eps;
                                  3: its last field became act_quant;
                                  4: ie_qlinear_allreduce / ie_allreduce take an algo */

/* ---- status codes --------------------------------------------------- */
#define IE_OK 0
#define IE_ERR_INVALID 1     /* bad shape / format / alignment / rank: Python raises ValueError */
#define IE_ERR_CUDA 2        /* a CUDA runtime call failed: RuntimeError */
#define IE_ERR_TIMEOUT 3     /* a bounded wait on a peer ran out (device status word) */
#define IE_ERR_UNSUPPORTED 4 /* valid request this build does not implement */

/* ---- enums ------------------------------------------------------------ */
/* weight formats (ie/quant/formats.py:67-71 and the group-128 int4 scheme) */
#define IE_FMT_INT8 0        /* int8 codes in [-127, 127], symmetric (INT8) */
#define IE_FMT_INT4 1        /* 4-bit codes: asym [0,15] with zeros, or sym [-7,7] stored +8 */
#define IE_FMT_FP8_E4M3 2    /* e4m3 bytes of the reference's f32 codes (FP8_E4M3) */

/* where the scale sits.  The reference's axis argument is the KEPT dimension
 * of the [K, N] weight (ie/quant/weights.py:45-48): PER_OUTPUT_CHANNEL = 0
 * keeps K, i.e. one scale per input row. */
#define IE_AXIS_K 0          /* f32 scale[K]        (reference axis=0, its default) */
#define IE_AXIS_N 1          /* f32 scale[N]        (reference axis=1)              */
#define IE_AXIS_TENSOR 2     /* f32 scale[1]        (reference axis=None)           */
#define IE_AXIS_GROUP128 3   /* f16 scale[K/128][N] and f16 zero[K/128][N]          */

/* element types */
#define IE_DT_BF16 0
#define IE_DT_F16 1
#define IE_DT_F32 2
#define IE_DT_I32 3
#define IE_DT_U8 4

/* epilogue flags for ie_qlinear / ie_qlinear_allreduce */
#define IE_EPI_BIAS 1        /* out += bias[n] (f32), added once after any reduction */
#define IE_EPI_RESIDUAL 2    /* out = residual + (...), residual has out's dtype      */
#define IE_EPI_SILU_MUL 4    /* rows are gate/up pairs: out[:, j] = silu(row 2j) * row 2j+1 */
/* Prologue: x is RMS-normalised first, x -> x / sqrt(mean_k(x^2) + norm_eps) * norm_weight
 * (ie/layers/functional.py:6-8; ie/kernels/torch_backend.py:103-105 before the qkv and
 * gate/up projections), folded into the tensor-core kernel: bf16/f16 x only, otherwise
 * IE_ERR_UNSUPPORTED (IE_ERR_INVALID with algo = 1). */
#define IE_EPI_RMS_NORM 8

/* ---- packed weight ------------------------------------------------------ */
typedef struct ie_qweight {
  int32_t format;       /* IE_FMT_* */
  int32_t axis;         /* IE_AXIS_* */
  int64_t k;            /* contraction length (reference rows of W) */
  int64_t n;            /* packed rows (reference columns of W; 2x for gate/up pairs) */
  const void* codes;    /* INT8/FP8: [n][k] bytes.  INT4: [n][k/2] bytes; each 32-bit word
                           holds k0..k0+7 with nibble p = code of k0 + {0,2,4,6,1,3,5,7}[p] */
  const void* scale;    /* per axis above; for gate/up pairs with IE_AXIS_K: f32 [2][k]
                           (gate table then up table) */
  const void* zero;     /* f16 [k/128][n] for IE_AXIS_GROUP128, else NULL */
  int32_t int4_symmetric; /* INT4 only: 1 = codes stored as q+8 with an implicit zero of 8 */
  int32_t gate_up;        /* 1 = rows interleaved gate/up (use with IE_EPI_SILU_MUL) */
} ie_qweight;

/* ---- one linear layer --------------------------------------------------- */
typedef struct ie_qlinear_args {
  ie_qweight w;
  int64_t m;            /* tokens */
  int32_t act_dtype;    /* x dtype: IE_DT_BF16 / IE_DT_F16 / IE_DT_F32 */
  int32_t out_dtype;    /* out dtype: IE_DT_BF16 / IE_DT_F16 / IE_DT_F32 */
  const void* x;        /* [m][k] row stride ldx (elements) */
  int64_t ldx;
  void* out;            /* [m][n] (or [m][n/2] with SILU_MUL), row stride ldo */
  int64_t ldo;
  const float* bias;    /* [n] f32 or NULL */
  const void* residual; /* [m][n] of out_dtype, row stride ldr, or NULL */
  int64_t ldr;
  int32_t epilogue;     /* IE_EPI_* flags */
  int32_t algo;         /* 0 = auto; 1 = weight-streaming GEMV; 2 = tcgen05 tensor-core GEMM
                           (bf16/f16 activations, K % 128 == 0, 16-byte aligned rows) */
  void* workspace;      /* caller-owned scratch (see ie_qlinear_workspace_size), may be NULL */
  size_t workspace_bytes;
  const float* norm_weight;  /* IE_EPI_RMS_NORM: f32 [k], 16-byte aligned */
  float norm_eps;
  int32_t act_quant;    /* IE_ACT_* (0: the activations as given) */
} ie_qlinear_args;

/* Activation quantization (ie_qlinear_args.act_quant).  IE_ACT_FP8_TOKEN: each
 * token row of x is quantized to e4m3 with its own scale, the reference's
 * quantize_float(x, FP8_E4M3, axis=0) (ie/quant/weights.py:73-81, scale
 * max|x_t| / 448, codes by round_to_float_format), and the e4m3 codes of x and
 * of an FP8 weight are contracted directly by the tensor cores
 * (tcgen05.mma kind::f8f6f4, f32 accumulators); the epilogue multiplies by the
 * token's scale and the weight's per-N or per-tensor scale.  FP8 weights with
 * IE_AXIS_N or IE_AXIS_TENSOR scales, bf16/f16 x, the tensor-core path and a
 * workspace (ie_qlinear_workspace_size) only; else IE_ERR_INVALID. */
#define IE_ACT_NONE 0
#define IE_ACT_FP8_TOKEN 1

/* All-reduce protocols of ie_qlinear_allreduce / ie_allreduce (the `algo` argument).
 * Both sum the ranks' f32 partials in rank order, so they give bitwise equal
 * outputs, identical on every rank (ie/parallel/sharding.py:40-44).
 *   IE_AR_ONESHOT: every rank pushes each output tile's partial to every rank over
 *     NVLink and every rank sums all of them: one flag round trip, (world-1) * 4
 *     bytes sent per output element per rank.  Lowest latency (decode).
 *   IE_AR_TWOSHOT: tile t belongs to rank t % world; partials go to the owner only,
 *     the owner sums them, applies bias and residual and pushes the finished
 *     tile to the other ranks: two flag round trips, 8 * (world-1) / world bytes
 *     per element per rank.  Needs at least `world` output tiles (one tile is 128
 *     output columns by up to 256 tokens on the tensor-core path); with fewer it
 *     runs one-shot.
 *   IE_AR_AUTO: one-shot below world 4 (two-shot sends as many bytes at world 2)
 *     and below ~2.5 MB of NVLink bytes saved per rank; two-shot above.
 *   IE_AR_NVLS (NVLink SHARP multicast) is not built: IE_ERR_UNSUPPORTED. */
#define IE_AR_AUTO 0
#define IE_AR_ONESHOT 1
#define IE_AR_TWOSHOT 2
#define IE_AR_NVLS 3
/* The protocol IE_AR_AUTO (or `algo`) resolves to for a call of `world` ranks
 * over `tiles` output tiles and `numel` output elements: IE_AR_ONESHOT or
 * IE_AR_TWOSHOT; -1 for an unknown or unsupported algo.  Host-only, no GPU. */
int ie_allreduce_resolve(int32_t world, int64_t tiles, int64_t numel, int32_t algo);

/* ---- library ------------------------------------------------------------ */
int ie_version(void);
/* Copy the last error message of this thread into buf (NUL-terminated). */
int ie_last_error(char* buf, size_t n);

/* ---- quantizer (reference semantics, bit-exact) ----------------------------
 * Replaces ie/quant/weights.py:51-70 (quantize_integer) and :73-81
 * (quantize_float) for a 2-D f32 weight w[rows][cols] in device memory.
 * axis: 0 keeps rows (one scale per row), 1 keeps columns, -1 = per tensor.
 *   integer (fmt_bits 8 or 4): codes int32 [rows][cols]; symmetric -> zero NULL;
 *     asymmetric -> zero f32, same shape as scale.
 *   float (IE_FMT_FP8_E4M3 via ie_quantize_float): codes f32 [rows][cols].
 * scale/zero hold rows (axis 0), cols (axis 1) or 1 (axis -1) f32 values. */
int ie_quantize_integer(const float* w, int64_t rows, int64_t cols, int32_t bits,
                        int32_t symmetric, int32_t axis, int32_t* codes, float* scale,
                        float* zero, void* stream);
/* exponent/mantissa bits and reserves_infinity as in ie/quant/formats.py:34-64 */
int ie_quantize_float(const float* w, int64_t rows, int64_t cols, int32_t exponent_bits,
                      int32_t mantissa_bits, int32_t reserves_infinity, int32_t axis,
                      float* codes, float* scale, void* stream);
/* Replaces ie/quant/formats.py:74-79 (round_to_float_format), elementwise. */
int ie_round_to_float_format(const float* x, float* out, int64_t count, int32_t exponent_bits,
                             int32_t mantissa_bits, int32_t reserves_infinity, void* stream);

/* ---- packing: reference tables -> device layout ------------------------------
 * Replaces nothing in the reference (it keeps f32 fake-quant weights,
 * ie/quant/model.py:48-52); this is the step that makes the weights real.
 * codes_kn: the reference's codes, [k][n] (int32 for INT8/INT4, f32 for FP8).
 * For IE_AXIS_GROUP128 pass codes_nk [n][k] int32 (the group view of
 * ie/quant/weights.py:51-70 on W.T), scale_f32/zero_f32 [n][k/128].
 * Outputs: packed codes in out_codes, f16 tables [k/128][n] for GROUP128 in
 * out_scale16 / out_zero16 (zero points must be exact in f16, else counted).  *unrepresentable (device int32, may be NULL) counts FP8 codes
 * that e4m3 cannot hold and were rounded to the nearest e4m3 value. */
int ie_pack_weight(int32_t format, int32_t axis, int32_t int4_symmetric, int64_t k, int64_t n,
                   const void* codes, const float* scale_f32, const float* zero_f32,
                   void* out_codes, void* out_scale16, void* out_zero16,
                   int32_t* unrepresentable, void* stream);
/* Packed -> dense reference-equivalent weight.  layout 0: f32 [k][n]
 * (ie/quant/weights.py:22-26); layout 1: out_dtype [n][k] (for cuBLAS). */
int ie_dequantize(const ie_qweight* w, int32_t layout, int32_t out_dtype, void* out,
                  void* stream);

/* ---- single-rank quantized linear --------------------------------------------
 * Replaces ColumnParallelLinear.forward / RowParallelLinear.forward
 * (ie/parallel/sharding.py:51-66) and the projections of TorchBlock.forward
 * (ie/model/torch_transformer.py:36-38,60) and torch_backend.swiglu
 * (ie/kernels/torch_backend.py:125-127) on a packed shard. */
/* Bytes of caller-owned workspace the call would use with the tensor-core
 * kernel: 256 bytes of grid-barrier and launch-generation words (offset 0),
 * the split-K tile tickets, the activations converted once per launch (bf16 ->
 * f16, RMS norm folded in) and the split-K partials.  The workspace must be
 * zero-filled before its first use; afterwards those words stay consistent by
 * themselves (also after a launch that gave up on an expired wait), and every
 * ticket carries the tag of the launch that counted it, so leftovers of an
 * earlier launch are ignored and nothing is cleared between calls.  A
 * smaller workspace (or none) runs the best plan that fits: split-K without
 * the activation pre-pass, the pre-pass without split-K, or neither. */
size_t ie_qlinear_workspace_size(const ie_qlinear_args* a);
int ie_qlinear(const ie_qlinear_args* a, void* stream);

/* ---- quantized linear that allocates nothing ----------------------------------
 * No counterpart in the reference (whose linear layers are CPU numpy): an
 * addition for callers that cannot allocate device memory at call time -- an
 * engine whose allocator has already claimed all the HBM it may use, or a
 * latency-bound decode loop that must never enter the CUDA allocator -- yet
 * want the split-K tensor-core kernel.
 * Same arguments and result as ie_qlinear on the tensor-core path; workspace
 * and workspace_bytes are ignored.  The split-K partials, tile tickets and the
 * converted activations of the pre-pass live in a static device array of
 * IE_QLINEAR_NOALLOC_SCRATCH_BYTES inside the library; a call whose preferred
 * plan needs more runs the best plan that fits (without split-K, then also
 * without the pre-pass, which needs no scratch at all).  A call the
 * tensor-core kernel cannot serve (f32 activations, K % 128 != 0, unaligned
 * rows, algo 1) returns IE_ERR_UNSUPPORTED.  The first call on a device looks
 * up that device's copy of the array (cudaGetSymbolAddress, which may load the
 * module): make it before any stream capture.  The array is shared by all calls
 * on a device, so calls that overlap on the GPU (concurrent streams) race. */
#define IE_QLINEAR_NOALLOC_SCRATCH_BYTES (8u << 20)
int ie_qlinear_noalloc(const ie_qlinear_args* a, void* stream);
/* Error bits recorded by kernels (1 = a bounded pipeline wait expired);
 * synchronous read of device state, optionally cleared. */
int ie_kernel_status(uint32_t* bits, int32_t clear);

/* ---- RMSNorm ------------------------------------------------------------------
 * Replaces ie/layers/functional.py:6-8 (rms_norm) and
 * ie/kernels/torch_backend.py:103-105: out = x / sqrt(mean(x^2) + eps) * weight
 * per row of x [m][h], f32 arithmetic; weight is f32 [h]. */
int ie_rms_norm(const void* x, int64_t ldx, int32_t x_dtype, const float* weight, void* out,
                int64_t ldo, int32_t out_dtype, int64_t m, int64_t h, float eps, void* stream);

/* ---- rotary embedding + KV-cache write ------------------------------------------
 * Replaces, for the output of the fused q|k|v projection, the RoPE of q and k
 * (ie/layers/functional.py:34-61, interleaved or halved) and write_kv
 * (ie/kernels/torch_backend.py:13-16) with one launch.  qkv [tokens][ld_qkv]
 * holds q (heads*head_dim), k and v (kv_heads*head_dim each) per row; cos /
 * sin are f32 [max_position][head_dim/2]; q_out [tokens][heads][head_dim];
 * the caches [cache_slots][kv_heads][head_dim] receive token t's rotated k and
 * its v at slots[t].  All activations one dtype (bf16, f16 or f32); each
 * product and sum is rounded to it, as the unfused elementwise steps do.
 * Tokens whose slot is outside [0, cache_slots) write no cache row, and
 * tokens whose position is outside the tables write no rotated q / k. */
int ie_rope_kv(const void* qkv, int64_t ld_qkv, int32_t dtype, int64_t tokens, int32_t heads,
               int32_t kv_heads, int32_t head_dim, const int64_t* positions,
               const float* cos_table, const float* sin_table, int64_t max_position,
               int32_t halved, const int64_t* slots, void* k_cache, void* v_cache,
               int64_t cache_slots, void* q_out, void* stream);

/* ---- all_reduce over a list of partials in one process -----------------------
 * Replaces ie/parallel/sharding.py:40-44: out = p[0] + p[1] + ... in rank order
 * (f32 arithmetic, the reference's order).  dtype applies to inputs and out. */
int ie_reduce_partials(const void* const* partials, int32_t count, void* out, int64_t numel,
                       int32_t dtype, void* stream);

/* ---- tensor-parallel communicator (one process per GPU) ------------------------
 * The reference's all_reduce runs ranks as list entries in one process
 * (ie/parallel/tensor_parallel.py:68-73); here each rank is a process on its
 * own GPU and peers reach each other's landing buffers over NVLink through
 * CUDA IPC.  Sequence: ie_comm_create -> ie_comm_export (bytes to all-gather
 * between ranks) -> ie_comm_open -> any number of collectives -> ie_comm_destroy. */
typedef struct ie_comm ie_comm;
#define IE_COMM_HANDLE_BYTES 64
int ie_comm_create(int32_t rank, int32_t world, int32_t device, size_t max_bytes,
                   ie_comm** out);
/* writes IE_COMM_HANDLE_BYTES bytes describing this rank's landing buffer */
int ie_comm_export(ie_comm* c, void* handle_out);
/* handles: world * IE_COMM_HANDLE_BYTES bytes, rank order */
int ie_comm_open(ie_comm* c, const void* handles);
int ie_comm_destroy(ie_comm* c);
/* bounded-wait limit in nanoseconds for every peer wait (default 2e9) */
int ie_comm_set_timeout(ie_comm* c, uint64_t ns);
/* IE_OK, or IE_ERR_TIMEOUT if a kernel of this comm gave up waiting; the
 * status word is read with a synchronous copy and then cleared. */
int ie_comm_check(ie_comm* c);

/* Fused row-parallel linear + all-reduce for this rank: every rank calls it with
 * its own K-shard (ie/parallel/sharding.py:60-66) and gets the reduced
 * out = [residual +] sum_r x_r @ W_r [+ bias] (ie/parallel/tensor_parallel.py:70,73).
 * Partials cross NVLink as f32 with P2P stores from the GEMM epilogue and are
 * summed in rank order, so every rank's output is bitwise identical.  algo:
 * IE_AR_* (above); every rank must pass the same algo and shapes. */
int ie_qlinear_allreduce(ie_comm* c, const ie_qlinear_args* a, int32_t algo, void* stream);
/* Standalone all-reduce of a device tensor (same protocols; a tile is 2048 elements). */
int ie_allreduce(ie_comm* c, const void* in, void* out, int64_t numel, int32_t dtype,
                 int32_t algo, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* IE_TPQ_H */
