// tcgen05 tensor-core quantized GEMM for sm_100a, with split-K and an optional
// one-shot all-reduce fused into the epilogue.
//
// The weight is the MMA's A operand (M = 128 output rows per tile) and the
// token batch is its N dimension (16..256), so decode batches and prefill
// batches use the same kernel.  Per CTA (608 threads = 19 warps, one CTA per SM):
//
//   warp 0      TMA producer: the packed weight tile [128 rows x 128 K]
//               (64- or 128-byte swizzle), the activation tile [BN tokens x
//               128 K] (128-byte swizzle, the MMA's B operand) and the stage's
//               scale tables (group-128 scale/zero rows, or per-K scales) into
//               a ring of shared-memory stages.  No multicast.
//   warps 1-2   MMA issuers: one thread each issues tcgen05.mma kind::f16 with A
//               read from tensor memory and B from shared memory, f32
//               accumulators in TMEM, 8 x K=16 per 128-K sub-stage;
//               tcgen05.commit releases the stages.  With two issuers they take
//               alternate sub-stages into separate accumulators.  For narrow
//               token tiles the 8 MMAs of a sub-stage rotate over two
//               accumulators, so consecutive MMAs do not wait on each other's
//               results; the epilogue adds everything up.
//   warps 3-18 dequantizers, then the epilogue.  They form four groups of four
//               warps (one warp per TMEM lane quarter); the groups take every
//               fourth 128-K sub-stage, so four sub-stages are dequantized at
//               once.  Each thread owns one weight row of its sub-stage: it reads the codes from
//               shared memory, widens int4 pairs with one mask+or into the
//               mantissas of an f16x2 (1024 + q), subtracts 1024 + zero exactly,
//               applies the group scale (one f16 rounding, 2^-12 relative) and
//               writes the f16 pairs straight into the TMEM A ring with
//               tcgen05.st -- the dequantized operand never touches shared
//               memory.  bf16 activation tiles are converted to f16 in place.
//               Per work unit they then read the accumulator (tcgen05.ld) and
//               run the epilogue: split-K reduction in split order, per-N /
//               per-tensor scale, bias, SiLU*up, residual, store or all-reduce.
//
// Work units are (row tile, token tile, K split); CTAs loop over them, or, in
// the stream-K order, each CTA takes an equal contiguous range of the
// (tile, K stage) order and a tile shared by several ranges is split between
// them.  A split writes its f32 partial to the caller's workspace and the last
// split to arrive (tagged atomic ticket) sums all splits in split order, so
// results do not depend on scheduling.  Every mbarrier wait is bounded (SM clock cycles); on
// expiry the kernel records an error bit, drains its TMA copies and MMAs, frees
// TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"


namespace ie {
namespace tc {

// Dequant warps: groups of four (one per TMEM lane quarter).  kPairs sub-stages
// are in flight at once, each split between kHalves groups by K.  Four groups
// each taking whole sub-stages (two 64-K halves per task) issue ~3 % fewer
// instructions than two pairs of groups splitting every sub-stage by K: the
// per-task loop, wait and hand-off cost is paid once per 128 K.
constexpr int kPairs = 4;
constexpr int kHalves = 1;
constexpr int kGroups = kPairs * kHalves;
constexpr int kDqWarps = 4 * kGroups;
constexpr int kDqThreads = kDqWarps * 32;
constexpr int kMmaWarps = 2;    // MMA issuing warps (the plan may use one)
constexpr int kDqWarp0 = 1 + kMmaWarps;
constexpr int kThreads = 32 * (kDqWarp0 + kDqWarps);
constexpr int kTileN = 128;     // weight rows per tile = MMA M
constexpr int kBK = 128;        // K per stage (one int4 group)
constexpr int kACols = kBK / 2; // TMEM columns of one A stage (two f16 per column)
constexpr int kMaxAStages = 6;
constexpr long long kWaitCycles = 4000000000ll;   // ~2 s at 2 GHz
constexpr int kMinSmem = 120 * 1024;              // keeps one CTA per SM
constexpr size_t kTicketBytes = 128 * 1024;       // workspace ticket region: 32768 tiles

// F_FP8N: fp8 weights contracted natively with per-token fp8 activations
// (IE_ACT_FP8_TOKEN): no dequantization, A read by the MMA from shared memory.
enum Fmt { F_INT4G = 0, F_INT4SYM = 1, F_INT8 = 2, F_FP8 = 3, F_FP8N = 4 };
constexpr int kFmts = 5;

// error bits recorded by kernels of this file (read with ie_kernel_status)
__device__ uint32_t g_tc_status = 0;
constexpr uint32_t kErrWait = 1u;

struct TcParams {
  int64_t M, K, N;          // tokens, contraction, packed rows
  int axis, gate_up, epilogue, out_dtype;
  int x_bf16;               // activations arrive as bf16 and are converted to f16
  const float* scale;       // per-N [N], per-tensor [1] / [2] (epilogue scales)
  const float* bias;
  const void* residual;
  int64_t ldr;
  void* out;
  int64_t ldo;
  int bn;                   // tokens per tile (MMA N)
  int n_tiles, m_tiles, splits, kstages;   // kstages = K / kBK
  int ns;                   // TMA ring depth
  int na;                   // TMEM A ring depth
  int acc_cols;             // TMEM columns of one accumulator chain
  int chains;               // independent accumulator chains per issuer (1 or 2)
  int issuers;              // MMA issuing threads (2 for tiles up to 128 tokens)
  int tmem_cols;            // TMEM columns allocated
  int w_stage_bytes;        // packed weight bytes per stage
  int t_kind;               // stage tables: 0 none, 1 group s/z f16 [128] each, 2 per-K f32
  int t_rows;               // per-K tables: 1, or 2 for gate/up pairs
  int t_stage_bytes;        // table bytes per stage (1024-aligned slot)
  int t_joint;              // group scale and zero tables are one [2][G][N] array
  int sub;                  // 128-K sub-stages per TMA stage
  int csplit;               // the splits of a tile form one cluster (rank = split)
  int nclusters;            // clusters in the grid (csplit)
  int recv_bytes;           // csplit: leader's receive buffer [splits-1][bn][128] f32
  float* ws;                // split-K partials [splits][M][N]
  uint32_t* counters;       // per (m_tile, n_tile) tickets, tagged with the launch (below)
  int streamk;              // stream-K order: CTA b takes TMA stages [b T / G, (b+1) T / G)
                            // of the tile-major (tile, stage) order, T = tiles * stages
  // RMS-norm prologue: x rows (plain loads for the per-token sum of squares)
  // and the f32 weight over K; the x tiles are scaled while they are converted
  const void* x;
  int64_t ldx;
  const float* norm_w;      // null: no prologue
  float norm_eps;
  int nw_off;               // byte offset of a stage's norm weights [sub][128] in its table slot
  // Activation pre-pass (the XPRE kernels): the CTAs first write the MMA's f16 operand
  // xh[M][K] (bf16 -> f16, RMS norm applied) into the workspace, each a slice,
  // then meet at a grid barrier; the x tiles are then TMA-loaded from xh as
  // they are.  Barrier words: xbar[0] counts this launch's arrivals (the last
  // arriver sets it back to zero), xbar[1] is a generation the last arriver
  // advances; waiters wait for it to leave the value read at kernel start.
  // Every CTA arrives exactly once (at teardown if it gave up before), so
  // the words are consistent for the next launch without being cleared.
  // xbar[2] is the launch generation of the split-K tickets and xbar[3] counts
  // the CTAs that finished: the last one advances xbar[2] and clears xbar[3].
  // A ticket word holds (tag << 8) | arrivals, tag = generation % (2^24 - 1) + 1:
  // a word left by another launch (one that gave up part-way included) carries
  // another tag and counts as zero, so tickets need no clearing between launches.
  __half* xh;               // F_FP8N: the e4m3 codes of x, [M][K] bytes
  uint32_t* xbar;
  float* xs;                // F_FP8N: per-token activation scales [M]
  // Launched as a programmatic dependent of the previous kernel on the stream:
  // the prologue and the first weight stages overlap that kernel's tail, and
  // nothing it writes (x, the residual, RMS-norm rows, the all-reduce epoch,
  // the workspace) is read or written before griddepcontrol.wait.
  int pdl;
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
// Bounded wait on an mbarrier phase: false (and an error bit) once the SM
// clock has advanced kWaitCycles, or at once if another role aborted.  (A
// try_wait with a suspend-time hint was slower: a suspended warp noticed the
// completed phase late.)
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          const volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) {
      atomicOr(&g_tc_status, kErrWait);
      return false;
    }
  }
}
// Bounded wait with cluster-scope acquire (for arrivals from other CTAs).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity,
                                                  const volatile int* abort_flag);
// Unconditional bounded drain wait used at teardown.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity) && clock64() - t0 < kWaitCycles) {
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
// Plain (untiled) bulk copy of `bytes` (a multiple of 16, both addresses
// 16-byte aligned) into this CTA's shared memory.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
// ---- thread-block cluster helpers (cluster split-K) ----
// The K splits of a tile run as one cluster: the non-leader CTAs store their
// f32 partial tiles into the leader's shared memory (distributed shared memory)
// and arrive on the leader's mbarrier; no global memory is involved.
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of `local` (a shared::cta address) in CTA `rank`
__device__ __forceinline__ uint32_t dsmem_map(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
__device__ __forceinline__ void dsmem_st(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
// arrive on an mbarrier of another CTA of the cluster, releasing this thread's
// prior writes at cluster scope
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ void fence_acq_rel_cluster() {
  asm volatile("fence.acq_rel.cluster;" ::: "memory");
}
// try_wait with acquire at cluster scope (pairs with remote releases)
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Hardware barrier across the cluster's threads: used once after barrier
// initialisation and once at teardown, points every CTA reaches on every path.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity,
                                                  const volatile int* abort_flag) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) {
      atomicOr(&g_tc_status, kErrWait);
      return false;
    }
  }
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}

// Ticket of a split-K tile: acquire-release at GPU scope, so the arriving CTA's
// partials (ordered before this by a CTA barrier) are published with it and
// the last CTA sees every earlier CTA's partials.
__device__ __forceinline__ uint32_t ticket_add(uint32_t* p) {
  uint32_t old;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(p) : "memory");
  return old;
}
// Tagged ticket (see TcParams::xbar): the arrivals of launch `tag` before this
// one.  An arrival that finds another launch's tag installs (tag << 8) with
// one compare-and-swap against the value it read, which fails harmlessly when
// another arrival got there first (a word never returns to a stale value
// within a launch); the count itself is an atomic add, acquire-release at GPU
// scope like ticket_add, so arrivals never retry.
__device__ __forceinline__ uint32_t ticket_tagged(uint32_t* p, uint32_t tag) {
  const uint32_t cur = *reinterpret_cast<volatile uint32_t*>(p);
  if ((cur >> 8) != tag) {
    uint32_t prev;
    asm volatile("atom.cas.relaxed.gpu.global.b32 %0, [%1], %2, %3;"
                 : "=r"(prev)
                 : "l"(p), "r"(cur), "r"(tag << 8)
                 : "memory");
    (void)prev;
  }
  return ticket_add(p) & 0xFFu;
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Orders this thread's generic-proxy global accesses with its async-proxy
// (TMA) accesses: after writing data another CTA's TMA will read, and after
// acquiring such data before issuing the TMA that reads it.
__device__ __forceinline__ void fence_proxy_async_all() {
  asm volatile("fence.proxy.async;" ::: "memory");
}
// Programmatic dependent launch: let the next kernel on the stream launch (its
// CTAs take SMs as this grid's CTAs exit), and wait for the previous kernel to
// complete with its memory visible (a no-op without a programmatic edge).
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
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
// D[tmem] (+)= A[tmem] * B[smem]
__device__ __forceinline__ void tc_mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[smem] * B[smem], e4m3 x e4m3 (K = 32 per instruction)
__device__ __forceinline__ void tc_mma_ss_f8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// The loaded registers are defined only once tcgen05.wait::ld returns, so the
// load and the wait form one asm statement (no use can be scheduled between).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
// Four 8-column loads (columns a, a + step, a + 2 step, a + 3 step of this
// thread's lane) behind a single wait: one TMEM round trip instead of four.
__device__ __forceinline__ void tmem_ld8x4(uint32_t a, uint32_t step, float (&v)[4][8]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%32];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%8,%9,%10,%11,%12,%13,%14,%15}, [%33];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%16,%17,%18,%19,%20,%21,%22,%23}, [%34];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%24,%25,%26,%27,%28,%29,%30,%31}, [%35];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(a), "r"(a + step), "r"(a + 2 * step), "r"(a + 3 * step)
      : "memory");
#pragma unroll
  for (int q = 0; q < 4; ++q)
#pragma unroll
    for (int i = 0; i < 8; ++i) v[q][i] = __uint_as_float(r[8 * q + i]);
}
// 32 consecutive TMEM columns of this thread's lane <- v[0..31]
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
      "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
      "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
// 16 consecutive TMEM columns of this thread's lane <- v[0..15]
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), version 1 for sm_100.
// The low word holds the start address (16-byte units, bits 0-13) and LBO
// (unused for swizzled K-major); adding a byte offset >> 4 to it moves the
// start address as long as the result stays inside shared memory.
__device__ __forceinline__ uint32_t sw128_desc_lo(uint32_t saddr) {
  return ((saddr & 0x3FFFFu) >> 4) | (1u << 16);
}
__device__ __forceinline__ uint64_t sw128_desc_from(uint32_t lo) {
  constexpr uint32_t hi = (1024u >> 4)     // SBO
                          | (1u << 14)     // descriptor version (bit 46)
                          | (2u << 29);    // SWIZZLE_128B (bits 61-63)
  return ((uint64_t)hi << 32) | lo;
}
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return sw128_desc_from(sw128_desc_lo(saddr));
}

// Instruction descriptor: f32 accumulator, A and B type 0 (f16 for kind::f16,
// e4m3 for kind::f8f6f4), both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t make_idesc(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kTileN >> 4) << 24);
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  return h2_bits(__floats2half2_rn(a, b));
}
// f32 pair -> f16x2 (a in the low half), saturating: magnitudes beyond f16's
// largest finite value (65504) become +-65504 instead of +-inf.  Activations
// reach the tensor cores as f16, so a bf16 activation outside f16's range is
// clamped to it; one instruction, the same cost as the plain conversion.
__device__ __forceinline__ uint32_t pack_h2_sat(float a, float b) {
  uint32_t r;
  asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  return r;
}

// ---------------------------------------------------------------------------
// dequantization of 32 K values of one row into 16 f16x2 words (TMEM columns)
// ---------------------------------------------------------------------------
// The sub-stage's packed row r lives at wst + r * row_bytes with its 16-byte
// chunks XOR-swizzled by the TMA (64-byte swizzle for int4 rows: chunk ^
// ((r>>1)&3); 128-byte swizzle for 8-bit rows: chunk ^ (r&7)), which keeps the 32
// lanes of a warp -- 32 consecutive rows -- on distinct shared-memory banks.
// q4 selects K values [32*q4, 32*q4 + 32) of the 128-wide sub-stage.
template <int FMT>
__device__ __forceinline__ void dequant_q4(const uint8_t* wst, int r, int q4, const uint8_t* tst,
                                           int t_rows, int axis, int64_t n_row, int j_sub,
                                           int sub, uint32_t (&o)[16]) {
  if constexpr (FMT == F_INT4G || FMT == F_INT4SYM) {
    const uint4 c = *reinterpret_cast<const uint4*>(wst + r * 64 + ((q4 ^ ((r >> 1) & 3)) << 4));
    const uint32_t w[4] = {c.x, c.y, c.z, c.w};
    if constexpr (FMT == F_INT4G) {
      // (1024 + q) - (1024 + z) is exact in f16; one rounding for * s.
      // stage tables: [scale | zero][sub][128 rows] f16
      const __half s = reinterpret_cast<const __half*>(tst)[j_sub * kTileN + r];
      const __half z = reinterpret_cast<const __half*>(tst)[(sub + j_sub) * kTileN + r];
      const __half2 off = __half2half2(__hadd(z, __float2half_rn(1024.0f)));
      const __half2 sc = __half2half2(s);
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t t = ((w[j] >> (4 * q)) & 0x000F000Fu) | 0x64006400u;
          o[4 * j + q] = h2_bits(__hmul2(__hsub2(bits_h2(t), off), sc));
        }
    } else {
      // symmetric int4 stored q + 8: (1024 + q + 8) - 1032 = q exactly
      const __half2 off = __half2half2(__float2half_rn(1032.0f));
      // per-K tables: [rows][sub][128] f32
      const float* sk = (axis == IE_AXIS_K)
                            ? reinterpret_cast<const float*>(tst) +
                                  ((t_rows == 2 ? (n_row & 1) : 0) * sub + j_sub) * kBK + 32 * q4
                            : nullptr;
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t t = ((w[j] >> (4 * q)) & 0x000F000Fu) | 0x64006400u;
          const __half2 v = __hsub2(bits_h2(t), off);
          if (sk) {
            const float2 f = __half22float2(v);
            o[4 * j + q] = pack_h2(f.x * sk[8 * j + 2 * q], f.y * sk[8 * j + 2 * q + 1]);
          } else {
            o[4 * j + q] = h2_bits(v);
          }
        }
    }
  } else {
    // 8-bit codes: 32 bytes = K values 32*q4 .. 32*q4+31
    const uint8_t* row = wst + r * 128;
    const int sw = r & 7;
    uint32_t w[8];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const uint4 v = *reinterpret_cast<const uint4*>(row + (((2 * q4 + c) ^ sw) << 4));
      w[4 * c] = v.x;
      w[4 * c + 1] = v.y;
      w[4 * c + 2] = v.z;
      w[4 * c + 3] = v.w;
    }
    const float* sk = (axis == IE_AXIS_K)
                          ? reinterpret_cast<const float*>(tst) +
                                ((t_rows == 2 ? (n_row & 1) : 0) * sub + j_sub) * kBK + 32 * q4
                          : nullptr;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const uint32_t pair = (w[j] >> (16 * q)) & 0xFFFFu;   // K = 4j+2q, 4j+2q+1
        __half2 v;
        if constexpr (FMT == F_INT8) {
          // bytes as f16 1024 + (b ^ 0x80) = 1152 + q, exact; minus 1152 is exact
          const uint32_t u = pair ^ 0x8080u;
          const uint32_t t = (u & 0xFFu) | ((u & 0xFF00u) << 8) | 0x64006400u;
          v = __hsub2(bits_h2(t), __half2half2(__float2half_rn(1152.0f)));
        } else {
          v = __half2(__nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)pair, __NV_E4M3));
        }
        if (sk) {
          const float2 f = __half22float2(v);
          const int k = 4 * j + 2 * q;
          o[2 * j + q] = pack_h2(f.x * sk[k], f.y * sk[k + 1]);
        } else {
          o[2 * j + q] = h2_bits(v);
        }
      }
    }
  }
}

// One 64-K half (`half` 0 or 1) of a 128-K row of a sub-stage -> 32 f16x2
// words in K order.  The half's code vectors are loaded before any arithmetic
// so the loads overlap.
// Group-128 int4: the pair (k0+2i, k0+2i+1) of a code word sits in nibbles
// (i, i+4); nibbles 0/4 and 1/5 are masked in place (1024 + q and 1024 + 16q
// as f16), nibbles 2/6 and 3/7 after one shift by 8.  (1024 + q) - (1024 + z)
// and (1024 + 16q) / 16 - (64 + z) are both exact, so every word equals the
// per-pair form: (q - z) exactly, then one rounding for * s.
template <int FMT>
__device__ __forceinline__ void dequant_half(const uint8_t* wst, int r, int half,
                                             const uint8_t* tst, int t_rows, int axis,
                                             int64_t n_row, int j_sub, int sub,
                                             uint32_t (&o)[32]) {
  if constexpr (FMT == F_INT4G) {
    uint32_t w[8];
#pragma unroll
    for (int c2 = 0; c2 < 2; ++c2) {
      const int q4 = 2 * half + c2;
      const uint4 c = *reinterpret_cast<const uint4*>(wst + r * 64 + ((q4 ^ ((r >> 1) & 3)) << 4));
      w[4 * c2] = c.x;
      w[4 * c2 + 1] = c.y;
      w[4 * c2 + 2] = c.z;
      w[4 * c2 + 3] = c.w;
    }
    const __half s = reinterpret_cast<const __half*>(tst)[j_sub * kTileN + r];
    const __half z = reinterpret_cast<const __half*>(tst)[(sub + j_sub) * kTileN + r];
    const __half2 off1 = __half2half2(__hadd(z, __float2half_rn(1024.0f)));
    const __half2 neg_off16 = __half2half2(__hneg(__hadd(z, __float2half_rn(64.0f))));
    const __half2 sixteenth = __float2half2_rn(0.0625f);
    const __half2 sc = __half2half2(s);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t lo = w[i], hi = w[i] >> 8;
      const __half2 t0 = bits_h2((lo & 0x000F000Fu) | 0x64006400u);
      const __half2 t1 = bits_h2((lo & 0x00F000F0u) | 0x64006400u);
      const __half2 t2 = bits_h2((hi & 0x000F000Fu) | 0x64006400u);
      const __half2 t3 = bits_h2((hi & 0x00F000F0u) | 0x64006400u);
      o[4 * i] = h2_bits(__hmul2(__hsub2(t0, off1), sc));
      o[4 * i + 1] = h2_bits(__hmul2(__hfma2(t1, sixteenth, neg_off16), sc));
      o[4 * i + 2] = h2_bits(__hmul2(__hsub2(t2, off1), sc));
      o[4 * i + 3] = h2_bits(__hmul2(__hfma2(t3, sixteenth, neg_off16), sc));
    }
  } else {
#pragma unroll
    for (int c2 = 0; c2 < 2; ++c2) {
      uint32_t (&part)[16] = *reinterpret_cast<uint32_t(*)[16]>(&o[16 * c2]);
      dequant_q4<FMT>(wst, r, 2 * half + c2, tst, t_rows, axis, n_row, j_sub, sub, part);
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

// 8 values at base + j * stride (j < valid) of an activation-typed array; the
// dtype is decided once for the 8, so the executed code is one straight run.
__device__ __forceinline__ void load8(const void* in, int dt, int64_t base, int64_t stride,
                                      int valid, float (&r)[8]) {
  if (dt == IE_DT_BF16) {
    const __nv_bfloat16* q = static_cast<const __nv_bfloat16*>(in) + base;
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = j < valid ? __bfloat162float(q[j * stride]) : 0.0f;
  } else if (dt == IE_DT_F16) {
    const __half* q = static_cast<const __half*>(in) + base;
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = j < valid ? __half2float(q[j * stride]) : 0.0f;
  } else {
    const float* q = static_cast<const float*>(in) + base;
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = j < valid ? q[j * stride] : 0.0f;
  }
}
__device__ __forceinline__ void store8(void* out, int dt, int64_t base, int64_t stride,
                                       int valid, const float (&v)[8]) {
  if (dt == IE_DT_BF16) {
    __nv_bfloat16* q = static_cast<__nv_bfloat16*>(out) + base;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j < valid) q[j * stride] = __float2bfloat16_rn(v[j]);
  } else if (dt == IE_DT_F16) {
    __half* q = static_cast<__half*>(out) + base;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j < valid) q[j * stride] = __float2half_rn(v[j]);
  } else {
    float* q = static_cast<float*>(out) + base;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j < valid) q[j * stride] = v[j];
  }
}

// bf16 -> f16 of one 16-byte chunk (8 values), in place, saturating at +-65504.
__device__ __forceinline__ void bf16_to_f16_chunk(uint4* p) {
  uint4 v = *p;
  uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i)
    w[i] = pack_h2_sat(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xFFFF0000u));
  *p = make_uint4(w[0], w[1], w[2], w[3]);
}

// Packed f32 pairs: Blackwell multiplies two f32 lanes per instruction.
__device__ __forceinline__ uint64_t f32x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint32_t f32x2_to_h2(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return pack_h2_sat(lo, hi);
}

// RMS-norm prologue, one 16-byte chunk of the x tile (8 consecutive K of one
// token): f16((x * rinv) * w), with rinv = 1 / sqrt(mean(x^2) + eps) of the
// token; each product rounded to f32 (round to nearest), two lanes per
// instruction.  The 8 weights come from the stage's copy in shared memory.
template <bool XBF16>
__device__ __forceinline__ void norm_chunk(uint4* p, const float* w8, float rinv) {
  const uint4 v = *p;
  const ulonglong2 wa = reinterpret_cast<const ulonglong2*>(w8)[0];
  const ulonglong2 wb = reinterpret_cast<const ulonglong2*>(w8)[1];
  const uint64_t wv[4] = {wa.x, wa.y, wb.x, wb.y};
  const uint64_t rr = f32x2(rinv, rinv);
  const uint32_t u[4] = {v.x, v.y, v.z, v.w};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint64_t xv;
    if constexpr (XBF16) {
      xv = f32x2(__uint_as_float(u[i] << 16), __uint_as_float(u[i] & 0xFFFF0000u));
    } else {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[i]));
      xv = f32x2(f.x, f.y);
    }
    o[i] = f32x2_to_h2(mul_f32x2(mul_f32x2(xv, rr), wv[i]));
  }
  *p = make_uint4(o[0], o[1], o[2], o[3]);
}

// Sum of squares of one K-long row of x by one warp: 16-byte loads, sixteen
// in flight per lane (a 4096-wide row in one round trip), then a butterfly;
// the same order on every call.
constexpr int kSumsqLoads = 8;
__device__ __forceinline__ float row_sumsq(const void* row, int64_t K, int x_bf16, int lane) {
  float ss = 0.0f;
  const uint4* r = static_cast<const uint4*>(row);   // 8 elements per uint4
  const int64_t chunks = K / 8;
  for (int64_t c0 = lane; c0 < chunks; c0 += 32 * kSumsqLoads) {
    uint4 v[kSumsqLoads];
#pragma unroll
    for (int j = 0; j < kSumsqLoads; ++j)
      v[j] = c0 + 32 * j < chunks ? __ldcg(r + c0 + 32 * j) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int j = 0; j < kSumsqLoads; ++j) {
      const uint32_t u[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float lo, hi;
        if (x_bf16) {
          lo = __uint_as_float(u[i] << 16);
          hi = __uint_as_float(u[i] & 0xFFFF0000u);
        } else {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[i]));
          lo = f.x;
          hi = f.y;
        }
        ss = fmaf(lo, lo, ss);
        ss = fmaf(hi, hi, ss);
      }
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  return ss;
}

// Activation pre-pass of one CTA (the dequant threads, dt = 0 .. kDqThreads-1):
// chunks [c0, c1) of xh's M*K/8 16-byte chunks, chunk i = token i / (K/8),
// K values 8 * (i % (K/8)) ...  Each chunk is what the in-loop conversion
// makes of it: bf16 -> f16 (saturating), or with the RMS norm
// f16((x * rinv) * w) with the same rinv and products, so xh is bit-identical
// to the converted x tiles.  The RMS factors of the slice's tokens are
// computed here, up to kDqWarps tokens per round (one warp each), into s_rinv.
template <class Sync>
__device__ __forceinline__ bool xpre_slice(const TcParams& p, int dt, int warp_i, int lane,
                                           float* s_rinv, int64_t c0, int64_t c1,
                                           const Sync& dq_sync) {
  const int64_t cpr = p.K / 8;   // chunks per token row
  const uint4* x = static_cast<const uint4*>(p.x);
  uint4* xh = reinterpret_cast<uint4*>(p.xh);
  const int64_t rs = p.ldx / 8;  // x row stride in chunks
  if (c1 <= c0) return true;
  const int64_t t_first = c0 / cpr, t_last = (c1 - 1) / cpr;
  for (int64_t t0 = t_first; t0 <= t_last; t0 += kDqWarps) {
    const int64_t t1 = t_last + 1 < t0 + kDqWarps ? t_last + 1 : t0 + kDqWarps;
    if (p.norm_w) {
      for (int64_t t = t0 + warp_i; t < t1; t += kDqWarps) {
        const float ss = row_sumsq(static_cast<const char*>(p.x) + t * p.ldx * 2, p.K, p.x_bf16,
                                   lane);
        if (lane == 0)
          s_rinv[t - t0] = 1.0f / __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)p.K), p.norm_eps));
      }
      if (!dq_sync()) return false;
    }
    const int64_t a = c0 > t0 * cpr ? c0 : t0 * cpr, b = c1 < t1 * cpr ? c1 : t1 * cpr;
    for (int64_t i = a + dt; i < b; i += kDqThreads) {
      const int64_t t = i / cpr, kc = i - t * cpr;
      uint4 v = __ldcg(x + t * rs + kc);
      if (p.norm_w) {
        if (p.x_bf16) norm_chunk<true>(&v, p.norm_w + kc * 8, s_rinv[t - t0]);
        else norm_chunk<false>(&v, p.norm_w + kc * 8, s_rinv[t - t0]);
      } else {
        bf16_to_f16_chunk(&v);
      }
      xh[t * cpr + kc] = v;
    }
    if (a + dt < b) fence_proxy_async_all();   // these stores, before other CTAs' TMA reads
    if (p.norm_w && !dq_sync()) return false;   // s_rinv is rewritten next round
  }
  return true;
}

// Largest |x| of one K-long row by one warp (exact in any order).
__device__ __forceinline__ float row_amax(const void* row, int64_t K, int x_bf16, int lane) {
  float mx = 0.0f;
  const uint4* r = static_cast<const uint4*>(row);
  const int64_t chunks = K / 8;
  for (int64_t c0 = lane; c0 < chunks; c0 += 32 * kSumsqLoads) {
    uint4 v[kSumsqLoads];
#pragma unroll
    for (int j = 0; j < kSumsqLoads; ++j)
      v[j] = c0 + 32 * j < chunks ? __ldcg(r + c0 + 32 * j) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int j = 0; j < kSumsqLoads; ++j) {
      const uint32_t u[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (x_bf16) {   // |bf16| as the top half of an f32 with the sign cleared
          mx = fmaxf(mx, __uint_as_float((u[i] << 16) & 0x7FFFFFFFu));
          mx = fmaxf(mx, __uint_as_float(u[i] & 0x7FFF0000u));
        } else {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[i]));
          mx = fmaxf(mx, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
      }
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  return mx;
}

// Per-token e4m3 activations (IE_ACT_FP8_TOKEN), the reference's
// quantize_float(x, FP8_E4M3, axis=0) (ie/quant/weights.py:73-81): scale
// max|x_t| / 448 (1 for an all-zero row), codes round_to_float_format(x / s)
// (ie/quant/formats.py:74-79), stored as e4m3 bytes.  Each CTA takes the same
// share of all M*K/8 chunks as the bf16 pre-pass (xpre_slice): per round of
// up to kDqWarps tokens its warps take one token's row maximum each (every
// CTA that touches a token computes the same value, the one holding the
// token's first chunk stores its scale), then all threads quantize the
// round's chunks.  The maximum is exact in any order and the divisions are
// IEEE f32, so codes and scales equal the reference's (a code below e4m3's
// normal range that keeps more fraction bits than an e4m3 subnormal becomes
// the nearest e4m3 value).
template <class Sync>
__device__ __forceinline__ bool fp8_act_slice(const TcParams& p, int dt, int warp_i, int lane,
                                              float* s_sc, int64_t c0, int64_t c1,
                                              const Sync& dq_sync) {
  const FloatFmt e4m3{3, 448.0f, 0.001953125f};   // max 448, flush below 2^-6 * 2^-3
  const int64_t cpr = p.K / 8;
  const uint4* x = static_cast<const uint4*>(p.x);
  uint8_t* xq = reinterpret_cast<uint8_t*>(p.xh);
  const int64_t rs = p.ldx / 8;
  if (c1 <= c0) return true;
  const int64_t t_first = c0 / cpr, t_last = (c1 - 1) / cpr;
  bool wrote = false;
  for (int64_t t0 = t_first; t0 <= t_last; t0 += kDqWarps) {
    const int64_t t1 = t_last + 1 < t0 + kDqWarps ? t_last + 1 : t0 + kDqWarps;
    for (int64_t t = t0 + warp_i; t < t1; t += kDqWarps) {
      const float amax = row_amax(static_cast<const char*>(p.x) + t * p.ldx * 2, p.K,
                                  p.x_bf16, lane);
      const float sc = amax == 0.0f ? 1.0f : __fdiv_rn(amax, 448.0f);
      if (lane == 0) {
        s_sc[t - t0] = sc;
        if (t * cpr >= c0) p.xs[t] = sc;
      }
    }
    if (!dq_sync()) return false;
    const int64_t a = c0 > t0 * cpr ? c0 : t0 * cpr, b = c1 < t1 * cpr ? c1 : t1 * cpr;
    for (int64_t i = a + dt; i < b; i += kDqThreads) {
      const int64_t t = i / cpr, kc = i - t * cpr;
      const uint4 v = __ldcg(x + t * rs + kc);
      const float sc = s_sc[t - t0];
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
      uint32_t bytes[2] = {0u, 0u};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float f;
        if (p.x_bf16) {
          f = __uint_as_float((e & 1) ? (u[e >> 1] & 0xFFFF0000u) : (u[e >> 1] << 16));
        } else {
          const float2 h = __half22float2(*reinterpret_cast<const __half2*>(&u[e >> 1]));
          f = (e & 1) ? h.y : h.x;
        }
        const float code = round_to_format(__fdiv_rn(f, sc), e4m3);
        const uint32_t byte = (uint32_t)__nv_cvt_float_to_fp8(code, __NV_SATFINITE, __NV_E4M3);
        bytes[e >> 2] |= byte << (8 * (e & 3));
      }
      *reinterpret_cast<uint2*>(xq + t * p.K + kc * 8) = make_uint2(bytes[0], bytes[1]);
      wrote = true;
    }
    if (!dq_sync()) return false;   // s_sc is rewritten next round
  }
  if (wrote) fence_proxy_async_all();   // these stores, before other CTAs' TMA reads
  return true;
}

// Epilogue value of token m, row n, before the residual: scale, then bias.
struct Epi {
  const TcParams& p;
  const ReduceCtx& rc;
  uint32_t epoch;
  int reduce;
  int d0, d1;   // landing buffers that receive this tile's partial (reduce)
  // Writes the finished values of the 8 tokens m0 .. m0+7 of row n; gate/up
  // pairs combine lanes (n even, n+1).  Every shuffle, then every residual
  // load, is issued before the stores, so the loads of one token do not wait
  // behind the previous token's store (out may alias nothing, but the compiler
  // cannot know).  SiLU divides with __fdividef (2 ulp), far below the
  // bf16/f16 rounding of the output.
  // Residual values of those tokens (the half-width column for gate/up pairs),
  // zero where there is none.
  __device__ __forceinline__ void load_res8(int64_t m0, int64_t n, int lane, float (&r)[8]) const {
    const bool silu = (p.epilogue & IE_EPI_SILU_MUL) != 0;
    const bool want = (p.epilogue & IE_EPI_RESIDUAL) && !(reduce && !silu) &&
                      (silu ? ((lane & 1) == 0 && n + 1 < p.N) : n < p.N);
    const int64_t col = silu ? (n >> 1) : n;
    const int valid = want ? (int)(p.M - m0 < 8 ? (int)(p.M - m0) : 8) : 0;
    load8(p.residual, p.out_dtype, m0 * p.ldr + col, p.ldr, valid, r);
  }
  __device__ __forceinline__ void emit8(int64_t m0, int64_t n, float (&v)[8], int lane,
                                        const float* pre_res = nullptr) const {
    const bool has_res = (p.epilogue & IE_EPI_RESIDUAL) != 0;
    float r[8];
    if (pre_res) {
#pragma unroll
      for (int j = 0; j < 8; ++j) r[j] = pre_res[j];
    } else {
      load_res8(m0, n, lane, r);
    }
    if (p.epilogue & IE_EPI_SILU_MUL) {
      const float b = ((p.epilogue & IE_EPI_BIAS) && n < p.N) ? p.bias[n] : 0.0f;
      float partner[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (p.epilogue & IE_EPI_BIAS) v[j] += b;
        partner[j] = __shfl_xor_sync(0xffffffffu, v[j], 1);
      }
      if ((lane & 1) == 0 && n + 1 < p.N) {
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          o[j] = __fdividef(v[j], 1.0f + __expf(-v[j])) * partner[j];
          if (has_res) o[j] += r[j];
        }
        store8(p.out, p.out_dtype, m0 * p.ldo + (n >> 1), p.ldo, (int)(p.M - m0 < 8 ? (int)(p.M - m0) : 8), o);
      }
    } else if (n < p.N) {
      if (reduce) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (m0 + j < p.M)
            for (int dst = d0; dst < d1; ++dst)
              landing_slot(rc, dst, epoch)[rc.rank * rc.slot_floats + (m0 + j) * p.N + n] = v[j];
      } else {
        const float b = (p.epilogue & IE_EPI_BIAS) ? p.bias[n] : 0.0f;
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float val = v[j];
          if (p.epilogue & IE_EPI_BIAS) val += b;
          if (has_res) val = r[j] + val;
          o[j] = val;
        }
        store8(p.out, p.out_dtype, m0 * p.ldo + n, p.ldo, (int)(p.M - m0 < 8 ? (int)(p.M - m0) : 8), o);
      }
    }
  }
};

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
// CSPLIT: the K splits of a tile reduce inside a thread-block cluster instead
// of through global partials; each instantiation carries only one of the two
// paths, so neither takes registers from the dequant loop of the other.
// XPRE: the activation pre-pass (x tiles from xh, loaded on their own
// barriers once the grid barrier opens); without it the x tiles share the
// weights' stage barrier and bf16 / RMS-norm tiles are converted in the loop.
template <int FMT, bool CSPLIT, bool XPRE>
__global__ void __launch_bounds__(kThreads, 1)
qgemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_z,
                TcParams p, ReduceCtx rc, int reduce) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base, derived from smem_raw by pointer arithmetic so that
  // the compiler still knows every derived pointer is shared memory (a round
  // trip through an integer would turn their accesses into generic ones)
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  constexpr bool NATIVE = FMT == F_FP8N;
  static_assert(!NATIVE || XPRE, "fp8 activations are made by the pre-pass");
  const int ns = p.ns, na = p.na, sub = p.sub;
  // one TMA stage = `sub` consecutive 128-K sub-stages behind one full/empty pair
  const int w_sub_bytes = p.w_stage_bytes / sub;           // [128 rows][row bytes] per sub
  // f16 x: two SW128 blocks per sub-stage; e4m3 x (NATIVE): one
  const int x_sub_bytes = p.bn * kBK * (NATIVE ? 1 : 2);
  const int x_stage_bytes = x_sub_bytes * sub;
  uint8_t* x_ring = smem;                                   // ns x x_stage_bytes
  uint8_t* w_ring = x_ring + ns * x_stage_bytes;            // ns x w_stage_bytes
  uint8_t* t_ring = w_ring + ns * p.w_stage_bytes;          // ns x t_stage_bytes
  float* recv = reinterpret_cast<float*>(t_ring + ns * p.t_stage_bytes);   // csplit
  uint64_t* bars = reinterpret_cast<uint64_t*>(t_ring + ns * p.t_stage_bytes + p.recv_bytes);
  uint64_t* full = bars;                 // [ns]  weights + tables landed (count 1 + tx)
  uint64_t* empty = full + ns;           // [ns]  MMA done + every dequant warp done
  uint64_t* xfull = empty + ns;          // [ns]  XPRE: the stage's x tile landed (count 1 + tx)
  uint64_t* afull = xfull + ns;          // [na]  a pair's 4 * kHalves warps wrote A
  uint64_t* aempty = afull + na;         // [na]  MMA read A (commit)
  uint64_t* accfull = aempty + na;       // every issuer's MMAs of a unit done -> epilogue
  uint64_t* accempty = accfull + 1;      // epilogue -> MMA (count 1)
  uint64_t* mma_done = accempty + 1;     // [kMmaWarps] final commits: all MMAs retired
  uint64_t* dqbar = mma_done + kMmaWarps;   // bounded barrier of the dequant threads
  uint64_t* rfull = dqbar + 1;   // csplit leader: every other split's partial arrived
  uint64_t* rfree = rfull + 1;   // csplit non-leader: the leader consumed the receive buffer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rfree + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* s_ticket = const_cast<int*>(abort_flag) + 1;
  // [max(bn, kDqWarps)]: RMS factors of a token tile, or of one pre-pass round
  float* s_rinv = reinterpret_cast<float*>(s_ticket + 1);
  // pre-pass barrier: [0] generation at kernel start, [1] this CTA has arrived
  volatile uint32_t* s_xb =
      reinterpret_cast<volatile uint32_t*>(s_rinv + (p.bn > kDqWarps ? p.bn : kDqWarps));
  auto xbar_arrive = [&]() {
    if (ticket_add(p.xbar) == gridDim.x - 1u) {
      *reinterpret_cast<volatile uint32_t*>(p.xbar) = 0u;   // ordered by the release below
      st_release_gpu(p.xbar + 1, s_xb[0] + 1u);
    }
    s_xb[1] = 1u;
  };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_launch_dependents();
  // The all-reduce epoch, the pre-pass barrier generation and the pre-pass's
  // reads of x all depend on the previous kernel: such launches wait at once.
  // The others overlap their prologue and first weight stages with it; their
  // split-K partials, tickets and ticket generation are touched only in an
  // epilogue, after MMAs that read x tiles the producer loads only after its
  // own wait, and by thread 0 (the producer) after that wait.
  if (reduce || XPRE) pdl_wait();
  const uint32_t epoch = reduce ? reduce_epoch(rc) : 0u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(&full[s], 1);
      // each issuer's commit + every dequant warp (NATIVE: the issuers only)
      mbar_init(&empty[s], p.issuers + (NATIVE ? 0 : kDqWarps));
      mbar_init(&xfull[s], 1);
    }
    for (int s = 0; s < na; ++s) {
      mbar_init(&afull[s], 4 * kHalves);
      mbar_init(&aempty[s], 1);
    }
    mbar_init(accfull, p.issuers);
    mbar_init(accempty, 1);
    for (int i = 0; i < kMmaWarps; ++i) mbar_init(&mma_done[i], 1);
    mbar_init(dqbar, kDqThreads);
    mbar_init(rfull, (uint32_t)((p.splits - 1) * kDqWarps));
    mbar_init(rfree, (uint32_t)kDqWarps);
    *abort_flag = 0;
    if constexpr (XPRE) {   // before any arrival of this CTA, hence before the barrier opens
      s_xb[0] = ld_acquire_gpu(p.xbar + 1);
      s_xb[1] = 0u;
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"((uint32_t)p.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // every CTA's barriers are initialised before any CTA of the cluster arrives
  // on them remotely
  if constexpr (CSPLIT) cluster_sync();
  // accumulators: issuer i, chain c at columns (i * chains + c) * acc_cols; A ring after them
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_a = tmem + (uint32_t)(p.acc_cols * p.chains * p.issuers);

  // Work unit u = (row tile, token tile, K split).  Splits own whole TMA
  // stages: sub-stages [ks0, ks1), ks0 a multiple of `sub`.
  const int units = p.n_tiles * p.m_tiles * p.splits;
  const int tstages = (p.kstages + sub - 1) / sub;
  // Unit iteration: CTAs step through units by the grid size; with cluster
  // split-K, the cluster steps through tiles and CTA rank r takes split r.
  const int tiles_all = p.n_tiles * p.m_tiles;
  const int crank = CSPLIT ? (int)cluster_rank() : 0;
  // Stream-K: CTA b takes the TMA stages [lo, hi) = [b T / G, (b+1) T / G) of
  // the tile-major order (tile * tstages + stage, T = tiles * tstages), its
  // units are the tiles that range touches, and the unit of tile t is segment
  // (b - first CTA of t) of t's nsp segments.  (Never with cluster split-K.)
  // (32-bit arithmetic: the plan keeps T * G below 2^31)
  const bool sk = !CSPLIT && p.streamk;
  const int sk_total = tiles_all * tstages;
  const int sk_g = (int)gridDim.x, sk_b = (int)blockIdx.x;
  const int sk_lo = sk ? sk_b * sk_total / sk_g : 0;
  const int sk_hi = sk ? (sk_b + 1) * sk_total / sk_g : 0;
  // the CTA whose range holds stage i
  auto sk_cta = [&](int i) { return ((i + 1) * sk_g - 1) / sk_total; };
  const int u_first = sk ? sk_lo / tstages
                      : CSPLIT ? (int)(blockIdx.x / p.splits) + tiles_all * crank
                               : (int)blockIdx.x;
  const int u_step = sk ? 1 : CSPLIT ? p.nclusters : (int)gridDim.x;
  const int u_end = sk ? (sk_hi - 1) / tstages + 1 : CSPLIT ? tiles_all * (crank + 1) : units;
  // unit u: row tile nt, token tile mt, sub-stages [ks0, ks1), segment sp of nsp
  auto unit_range = [&](int u, int& nt, int& mt, int& ks0, int& ks1, int& sp, int& nsp) {
    if constexpr (!CSPLIT) {
      if (sk) {
        nt = u % p.n_tiles;
        mt = u / p.n_tiles;
        const int t0 = u * tstages;
        ks0 = (max(sk_lo, t0) - t0) * sub;
        ks1 = min(p.kstages, (min(sk_hi, t0 + tstages) - t0) * sub);
        const int first = sk_cta(t0);
        sp = sk_b - first;
        nsp = sk_cta(t0 + tstages - 1) - first + 1;
        return;
      }
    }
    nt = u % p.n_tiles;
    const int rest = u / p.n_tiles;
    mt = rest % p.m_tiles;
    sp = rest / p.m_tiles;
    nsp = p.splits;
    const int per = (tstages + p.splits - 1) / p.splits;
    ks0 = sp * per * sub;
    ks1 = min(p.kstages, ks0 + per * sub);
  };

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    // Weights and tables of a stage land on full[s]; its x tile too, or with
    // XPRE on xfull[s].  With the pre-pass the x tiles come from xh, which is complete
    // only once every CTA has passed the grid barrier: until then the producer
    // issues weight stages only (remembering each one's x coordinates) and
    // waits for the barrier when the ring is full -- reusing a slot needs that
    // stage's MMAs, hence its x tile, anyway.  (Polling the barrier between
    // stages put an L2 round trip in front of every early weight copy.)
    if (lane == 0) {
      prefetch_tmap(&tm_w);
      prefetch_tmap(&tm_x);
      if (p.t_kind) prefetch_tmap(&tm_s);
      if (p.t_kind == 1 && !p.t_joint) prefetch_tmap(&tm_z);
      int ti = 0;
      const uint32_t tbytes = p.t_kind == 1 ? (uint32_t)(2 * kTileN * 2 * sub)
                              : (p.t_kind == 2 ? (uint32_t)(p.t_rows * kBK * 4 * sub) : 0u);
      const int row_sub = w_sub_bytes / kTileN;
      bool xready = !XPRE && !p.pdl;
      int x_next = 0;                 // first stage whose x tile is not issued yet
      uint32_t pend[12];   // x coordinates (mt << 16 | ks) of stages x_next .. ti, by slot
      bool ok = true;
      auto issue_x = [&](int tj, int mt, int ks) {
        const int sj = tj % ns;
        // every 64-wide K block of the stage's activation tile in one copy
        if constexpr (XPRE) {   // (K blocks of 64 f16, or NATIVE of 128 e4m3 bytes)
          mbar_expect_tx(&xfull[sj], (uint32_t)x_stage_bytes);
          tma_load_3d(x_ring + sj * x_stage_bytes, &tm_x, 0, mt * p.bn, NATIVE ? ks : ks * 2,
                      &xfull[sj]);
        } else {   // the stage's full barrier already expects these bytes
          tma_load_3d(x_ring + sj * x_stage_bytes, &tm_x, 0, mt * p.bn, ks * 2, &full[sj]);
        }
      };
      // x tiles of the remembered stages x_next .. limit - 1
      auto flush_x = [&](int limit) {
        for (; x_next < limit; ++x_next)
          issue_x(x_next, (int)(pend[x_next % ns] >> 16), (int)(pend[x_next % ns] & 0xFFFFu));
      };
      auto poll_x = [&](int limit) -> bool {
        if (xready) return true;
        if constexpr (!XPRE) {   // programmatic launch: x is the previous kernel's output
          pdl_wait();
          xready = true;
          flush_x(limit);
          return true;
        }
        const uint32_t gen0 = s_xb[0];
        if (ld_acquire_gpu(p.xbar + 1) == gen0) {
          const long long t0 = clock64();
          while (ld_acquire_gpu(p.xbar + 1) == gen0) {
            if (*abort_flag) return false;
            if (clock64() - t0 > kWaitCycles) {
              atomicOr(&g_tc_status, kErrWait);
              return false;
            }
            __nanosleep(64);
          }
        }
        fence_proxy_async_all();   // xh was written by other CTAs' generic stores
        xready = true;
        flush_x(limit);
        return true;
      };
      for (int u = u_first; u < u_end && ok && !*abort_flag; u += u_step) {
        int nt, mt, ks0, ks1, sp, nsp;
        unit_range(u, nt, mt, ks0, ks1, sp, nsp);
        for (int ks = ks0; ks < ks1; ks += sub, ++ti) {
          const int s = ti % ns;
          // reusing a slot needs the MMAs of stage ti - ns, hence its x tile
          if (ti >= ns && !(ok = poll_x(ti))) break;
          if (!mbar_wait(&empty[s], ((ti / ns) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t nbytes =
              (p.norm_w && !XPRE) ? (uint32_t)(min(sub, p.kstages - ks) * kBK * 4) : 0u;
          mbar_expect_tx(&full[s], (uint32_t)p.w_stage_bytes + tbytes + nbytes +
                                       (XPRE ? 0u : (uint32_t)x_stage_bytes));
          uint8_t* ws_ = w_ring + s * p.w_stage_bytes;
          for (int j = 0; j < sub; ++j)   // K past the end reads as zeros
            tma_load_2d(ws_ + j * w_sub_bytes, &tm_w, (ks + j) * row_sub, nt * kTileN, &full[s]);
          uint8_t* ts = t_ring + s * p.t_stage_bytes;
          if (p.t_kind == 1) {
            if (p.t_joint) {
              tma_load_3d(ts, &tm_s, nt * kTileN, ks, 0, &full[s]);   // [s|z][sub][128]
            } else {
              tma_load_2d(ts, &tm_s, nt * kTileN, ks, &full[s]);
              tma_load_2d(ts + sub * kTileN * 2, &tm_z, nt * kTileN, ks, &full[s]);
            }
          } else if (p.t_kind == 2) {
            tma_load_3d(ts, &tm_s, 0, ks, 0, &full[s]);               // [rows][sub][128]
          }
          if (nbytes)   // the stage's norm weights, only those inside [0, K)
            bulk_load(ts + p.nw_off, p.norm_w + (int64_t)ks * kBK, nbytes, &full[s]);
          if (xready) {
            issue_x(ti, mt, ks);
            x_next = ti + 1;
          } else {
            pend[s] = ((uint32_t)mt << 16) | (uint32_t)ks;
          }
        }
      }
      // stages whose x is still pending: the MMA issuers wait for it.  Without
      // the pre-pass their full barriers expect the x bytes, so they are
      // issued even after an abort, for the drain below to complete.
      if (ti > x_next) {
        if constexpr (XPRE) {
          if (ok) ok = poll_x(ti);
        } else {
          poll_x(ti);
        }
      }
      if (!ok) *abort_flag = 1;
      // drain: every issued stage's copies must have landed before exit
      const int first = ti > ns ? ti - ns : 0;
      for (int j = first; j < ti; ++j) {
        mbar_drain(&full[j % ns], (j / ns) & 1);
        if (XPRE && j < x_next) mbar_drain(&xfull[j % ns], (j / ns) & 1);
      }
    }
  } else if (warp <= kMmaWarps) {
    // ------------------------------ MMA issuers -------------------------------
    // issuer i takes the unit's sub-stages with local index % issuers == i
    const int issuer = warp - 1;
    if (lane == 0 && issuer < p.issuers) {
      // The issuing thread shares its scheduler with two dequant warps, so the
      // per-MMA work is kept to an add and the MMA itself: B descriptor offsets
      // (16-byte units) and accumulator columns of the 8 MMAs of a sub-stage
      // are fixed for the launch, ring slots advance by increment.
      const uint32_t idesc = make_idesc(p.bn);
      const uint32_t acc0 = tmem + (uint32_t)(issuer * p.chains * p.acc_cols);
      uint32_t boff[kBK / 16], dcol[kBK / 16];
#pragma unroll
      for (int kk = 0; kk < kBK / 16; ++kk) {
        boff[kk] = (uint32_t)(((kk >> 2) * p.bn * 128 + (kk & 3) * 32) >> 4);
        dcol[kk] = acc0 + (uint32_t)((kk & (p.chains - 1)) * p.acc_cols);
      }
      // MMAs kk < chains of a unit's first sub-stage start their chain (no accumulate)
      const uint32_t fresh_mask = 0xFFu & ~((1u << p.chains) - 1u);
      const uint32_t x_lo0 = sw128_desc_lo(smem_u32(x_ring));
      const uint32_t x_stage16 = (uint32_t)x_stage_bytes >> 4, x_sub16 = (uint32_t)x_sub_bytes >> 4;
      uint32_t s = 0, s_ph = 0;   // TMA ring slot and its phase parity
      uint32_t a = 0, a_ph = 0;   // A ring slot and its phase parity
      int unit_i = 0;
      bool ok = true;
      for (int u = u_first; u < u_end && ok; u += u_step, ++unit_i) {
        int nt, mt, ks0, ks1, sp, nsp;
        unit_range(u, nt, mt, ks0, ks1, sp, nsp);
        if (!mbar_wait(accempty, (unit_i & 1) ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t mask = fresh_mask;
        int lsub = 0;   // sub-stage index within the unit
        for (int ks = ks0; ks < ks1 && ok; ks += sub) {
          const int nsub = min(sub, ks1 - ks);
          const uint32_t x_lo = x_lo0 + s * x_stage16;
          // Every role that arrives on empty[s] first waits for this use of the
          // stage to land, so no arrival can be credited to an earlier phase;
          // the issuers wait for the stage's x tile (the B operand).
          if (!mbar_wait(XPRE ? &xfull[s] : &full[s], s_ph, abort_flag)) {
            ok = false;
            break;
          }
          if constexpr (NATIVE) {   // the stage's weight tile is the A operand as it landed
            if (!mbar_wait(&full[s], s_ph, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          // this issuer's sub-stages of the stage, j = first, first + issuers, ...;
          // sub-stage j uses A slot (a + j) mod na
          const int first = p.issuers == 1 ? 0 : (issuer ^ (lsub & 1));
          for (int j = first; j < nsub && NATIVE; j += p.issuers) {
            // e4m3 weights [128 rows][128 K] and x [bn][128 K], both one SW128
            // block: four K = 32 steps of 32 bytes
            const uint32_t w_lo =
                sw128_desc_lo(smem_u32(w_ring + s * p.w_stage_bytes + j * w_sub_bytes));
            const uint32_t xb = x_lo + (uint32_t)j * x_sub16;
#pragma unroll
            for (int kk = 0; kk < kBK / 32; ++kk)
              tc_mma_ss_f8(dcol[kk], sw128_desc_from(w_lo + (uint32_t)(kk * 2)),
                           sw128_desc_from(xb + (uint32_t)(kk * 2)), idesc, (mask >> kk) & 1u);
            mask = 0xFFu;
          }
          for (int j = first; j < nsub && !NATIVE; j += p.issuers) {
            uint32_t aj = a + (uint32_t)j, phj = a_ph;
            while (aj >= (uint32_t)na) {
              aj -= (uint32_t)na;
              phj ^= 1u;
            }
            // afull implies the stage's TMA landed: the dequant warps waited on it
            if (!mbar_wait(&afull[aj], phj, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_col = tmem_a + aj * (uint32_t)kACols;
            const uint32_t xb = x_lo + (uint32_t)j * x_sub16;
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              tc_mma_ts(dcol[kk], a_col + (uint32_t)(kk * 8), sw128_desc_from(xb + boff[kk]),
                        idesc, (mask >> kk) & 1u);
            mask = 0xFFu;
            tc_commit(&aempty[aj]);
          }
          if (!ok) break;
          lsub += nsub;
          if constexpr (!NATIVE) {   // (NATIVE has no A ring)
            a += (uint32_t)nsub;
            while (a >= (uint32_t)na) {
              a -= (uint32_t)na;
              a_ph ^= 1u;
            }
          }
          tc_commit(&empty[s]);
          if (++s == (uint32_t)ns) {
            s = 0;
            s_ph ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(accfull);
      }
      if (!ok) *abort_flag = 1;
      // every MMA this thread issued must finish before TMEM is released
      tc_commit(&mma_done[issuer]);
      mbar_drain(&mma_done[issuer], 0);
    }
  } else {
    // ---------------------- dequantize + epilogue ----------------------
    const int dt = threadIdx.x - 32 * kDqWarp0;   // 0 .. kDqThreads-1
    const int quarter = warp & 3;                 // TMEM lanes 32*quarter ..
    const int group = (warp - kDqWarp0) >> 2;     // 0 .. kGroups-1
    const int pair = group / kHalves;             // which sub-stages this warp dequantizes
    const int half = group % kHalves;             // and which 64-K half of them
    const int pt = half * 128 + (dt & 127);       // thread index within the pair
    const int row = quarter * 32 + lane;          // weight row = accumulator lane
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    uint32_t s = 0, s_ph = 0;   // TMA ring slot and its phase parity
    uint32_t a = 0, a_ph = 0;   // A ring slot and its phase parity
    int unit_i = 0;
    bool ok = true;
    // Barrier of the dequant threads with a bounded wait (bar.sync cannot give
    // up): if one warp leaves on an expired wait, the others follow it out
    // instead of blocking the CTA's teardown.
    uint32_t dq_ph = 0;
    auto dq_sync = [&]() -> bool {
      mbar_arrive(dqbar);
      const bool done = mbar_wait(dqbar, dq_ph, abort_flag);
      dq_ph ^= 1u;
      return done;
    };
    if constexpr (XPRE) {
      // Activation pre-pass: this CTA's share of xh, then the grid barrier.
      // The dequant warps do not wait for the barrier themselves (the weights
      // need no activations); the producer waits before loading x tiles.
      const int64_t total = p.M * (p.K / 8);
      const int64_t g = gridDim.x, b = blockIdx.x;
      if constexpr (NATIVE)
        ok = fp8_act_slice(p, dt, warp - kDqWarp0, lane, s_rinv, total * b / g,
                           total * (b + 1) / g, dq_sync);
      else
        ok = xpre_slice(p, dt, warp - kDqWarp0, lane, s_rinv, total * b / g,
                        total * (b + 1) / g, dq_sync);
      if (ok) ok = dq_sync();
      if (ok && dt == 0) xbar_arrive();
    }
    // NATIVE: the accumulators are sums of e4m3 code products; token t's values
    // take its activation scale after the weight's (nscale)
    auto token_scales = [&](int64_t m0c, float (&v)[8]) {
      if constexpr (NATIVE) {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] *= (m0c + j < p.M) ? p.xs[m0c + j] : 0.0f;
      }
    };
    int norm_mt = -1;   // token tile whose RMS factors s_rinv holds
    for (int u = u_first; u < u_end && ok; u += u_step, ++unit_i) {
      int nt, mt, ks0, ks1, sp, nsp;
      unit_range(u, nt, mt, ks0, ks1, sp, nsp);
      const int64_t n = (int64_t)nt * kTileN + row;
      if (p.norm_w && !XPRE && mt != norm_mt) {
        if (p.pdl) pdl_wait();   // the rows are the previous kernel's output
        // RMS factors of the tile's tokens over the full K (every split needs
        // them, so each CTA reads the rows itself, from L2): dequant warp w
        // takes tokens w, w + 16, ...  The previous unit's conversions all
        // finished before its epilogue barrier, so s_rinv is free to rewrite.
        norm_mt = mt;
        for (int t = warp - kDqWarp0; t < p.bn; t += kDqWarps) {
          const int64_t m = (int64_t)mt * p.bn + t;
          float rinv = 0.0f;
          if (m < p.M) {
            const float ss = row_sumsq(static_cast<const char*>(p.x) + m * p.ldx * 2, p.K,
                                       p.x_bf16, lane);
            rinv = 1.0f / __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)p.K), p.norm_eps));
          }
          if (lane == 0) s_rinv[t] = rinv;
        }
        if (!dq_sync()) {
          ok = false;
          break;
        }
      }
      int lsub = 0;   // sub-stage index within the unit; pair lsub % kPairs takes it
      // (NATIVE: nothing to dequantize, the MMAs read the stages themselves)
      for (int ks = ks0; ks < ks1 && ok && !NATIVE; ks += sub) {
        const int nsub = min(sub, ks1 - ks);
        // wait for this use of the stage even without a sub-stage to dequantize:
        // the arrival on empty[s] below must not run ahead of the producer
        if (!mbar_wait(&full[s], s_ph, abort_flag)) {
          ok = false;
          break;
        }
        // this pair's sub-stages of the stage: j = first, first + kPairs, ...;
        // sub-stage j uses A slot (a + j) mod na
        const int first = (pair - lsub % kPairs + kPairs) % kPairs;
        for (int j = first; j < nsub; j += kPairs) {
          uint32_t aj = a + (uint32_t)j, phj = a_ph;
          while (aj >= (uint32_t)na) {
            aj -= (uint32_t)na;
            phj ^= 1u;
          }
          if (!mbar_wait(&aempty[aj], phj ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          const uint8_t* wst = w_ring + s * p.w_stage_bytes + j * w_sub_bytes;
          const uint8_t* tst = t_ring + s * p.t_stage_bytes;
          // the task's 64-K halves (one when two groups share the sub-stage)
#pragma unroll
          for (int hh = 0; hh < 2 / kHalves; ++hh) {
            const int h = kHalves == 1 ? hh : half;
            uint32_t o[32];
            dequant_half<FMT>(wst, row, h, tst, p.t_rows, p.axis, n, j, sub, o);
            tmem_st32(tmem_a + lane_addr + aj * (uint32_t)kACols + (uint32_t)(h * 32), o);
          }
          if constexpr (XPRE) {
            // x tiles arrive from xh already converted
          } else if (p.norm_w) {
            // chunk i of the sub-stage: 128-byte line i / 8 = (64-K block,
            // token), 16-byte column (i % 8) XOR (line % 8) under the
            // 128-byte swizzle (bn is a multiple of 16, so line % 8 is the
            // token's); every chunk of a TMA stage lies inside [0, K)
            uint4* xs = reinterpret_cast<uint4*>(x_ring + s * x_stage_bytes + j * x_sub_bytes);
            const float* wk =
                reinterpret_cast<const float*>(t_ring + s * p.t_stage_bytes + p.nw_off) + j * kBK;
            for (int i = pt; i < x_sub_bytes / 16; i += 128 * kHalves) {
              const int line = i >> 3;                 // < 2 * bn
              const bool hi = line >= p.bn;            // second 64-K block
              const int t = hi ? line - p.bn : line;
              const int kof = (hi ? 64 : 0) + (((i & 7) ^ (line & 7)) << 3);
              if (p.x_bf16) norm_chunk<true>(xs + i, wk + kof, s_rinv[t]);
              else norm_chunk<false>(xs + i, wk + kof, s_rinv[t]);
            }
            fence_proxy_async();
          } else if (p.x_bf16) {
            uint4* xs = reinterpret_cast<uint4*>(x_ring + s * x_stage_bytes + j * x_sub_bytes);
            for (int i = pt; i < x_sub_bytes / 16; i += 128 * kHalves) bf16_to_f16_chunk(xs + i);
            fence_proxy_async();
          }
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&afull[aj]);
        }
        if (!ok) break;
        lsub += nsub;
        a += (uint32_t)nsub;
        while (a >= (uint32_t)na) {
          a -= (uint32_t)na;
          a_ph ^= 1u;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);   // this warp is done with the stage
        if (++s == (uint32_t)ns) {
          s = 0;
          s_ph ^= 1u;
        }
      }
      if (!ok) break;

      // ---- epilogue of this unit ----
      if (!mbar_wait(accfull, unit_i & 1, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int64_t m0 = (int64_t)mt * p.bn;
      const bool split = nsp > 1;
      float nscale = 1.0f;
      if (n < p.N) {
        if (p.axis == IE_AXIS_N) nscale = p.scale[n];
        else if (p.axis == IE_AXIS_TENSOR) nscale = p.scale[p.gate_up ? (n & 1) : 0];
      }
      const int tile_id = mt * p.n_tiles + nt;
      int d0 = 0, d1 = 0;
      if (reduce) ar_push_range(rc, tile_id, d0, d1);
      const Epi epi{p, rc, epoch, reduce, d0, d1};
      // accumulators holding this unit: issuers that took at least one sub-stage
      const int nacc = p.chains * min(p.issuers, ks1 - ks0);
      constexpr bool csplit = CSPLIT;
      // cluster split-K, non-leader: the leader must have consumed this
      // cluster's previous tile from its receive buffer
      if (csplit && crank > 0 && unit_i > 0 &&
          !mbar_wait_cluster(rfree, (uint32_t)((unit_i - 1) & 1), abort_flag)) {
        ok = false;
        break;
      }
      float own[8];   // csplit leader: this thread's chunk of its own split
      bool has_own = false;
      // this warp owns the 8-token column chunks c0 = 8 * (group + kGroups * i)
      for (int c0 = 8 * group; c0 < p.bn; c0 += 8 * kGroups) {
        // accumulators summed in chain order 0, 1, ..., nacc - 1; four loads
        // share one TMEM round trip when there are at least four
        float v[8];
        if (nacc % 4 == 0) {
          {
            float w[4][8];
            tmem_ld8x4(tmem + lane_addr + (uint32_t)c0, (uint32_t)p.acc_cols, w);
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = ((w[0][j] + w[1][j]) + w[2][j]) + w[3][j];
          }
          for (int c4 = 4; c4 < nacc; c4 += 4) {
            float w[4][8];
            tmem_ld8x4(tmem + lane_addr + (uint32_t)(c4 * p.acc_cols + c0), (uint32_t)p.acc_cols,
                       w);
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = (((v[j] + w[0][j]) + w[1][j]) + w[2][j]) + w[3][j];
          }
        } else {
          tmem_ld8(tmem + lane_addr + (uint32_t)c0, v);
          for (int c = 1; c < nacc; ++c) {
            float w[8];
            tmem_ld8(tmem + lane_addr + (uint32_t)(c * p.acc_cols + c0), w);
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] += w[j];
          }
        }
        if constexpr (csplit) {
          if (crank > 0) {
            // into the leader's receive buffer [split-1][token][row]
            const uint32_t base = dsmem_map(
                smem_u32(recv + ((crank - 1) * p.bn + c0) * kTileN + row), 0u);
#pragma unroll
            for (int j = 0; j < 8; ++j) dsmem_st(base + (uint32_t)(j * kTileN * 4), v[j]);
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) own[j] = v[j];
            has_own = true;
          }
        } else if (split) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int64_t m = m0 + c0 + j;
            if (m < p.M && n < p.N) p.ws[((int64_t)sp * p.M + m) * p.N + n] = v[j];
          }
        }
        if (!split) {
#pragma unroll
          for (int j = 0; j < 8; ++j) v[j] *= nscale;
          token_scales(m0 + c0, v);
          epi.emit8(m0 + c0, n, v, lane);
        }
      }
      if (csplit && crank > 0) {
        // publish this warp's partial stores to the leader
        fence_acq_rel_cluster();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(dsmem_map(smem_u32(rfull), 0u));
      }
      tc_fence_before();
      if (!dq_sync()) {
        ok = false;
        break;
      }
      if (dt == 0) mbar_arrive(accempty);

      bool finalize_here = !split;
      if constexpr (csplit) {
        finalize_here = crank == 0;
        if (crank == 0) {
          if (!mbar_wait_cluster(rfull, (uint32_t)(unit_i & 1), abort_flag)) {
            ok = false;
            break;
          }
          if (has_own) {
            // splits add in split order: own (split 0), then 1, 2, ...
            const int c0 = 8 * group;
            float acc[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = own[j];
            for (int q = 1; q < p.splits; ++q) {
              const float* part = recv + ((q - 1) * p.bn + c0) * kTileN + row;
#pragma unroll
              for (int j = 0; j < 8; ++j) acc[j] += part[j * kTileN];
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] *= nscale;
            token_scales(m0 + c0, acc);
            epi.emit8(m0 + c0, n, acc, lane);
          }
          // hand the receive buffer back to every other split of the cluster
          __syncwarp();
          if (lane == 0)
            for (int q = 1; q < p.splits; ++q) mbar_arrive_remote(dsmem_map(smem_u32(rfree), (uint32_t)q));
        }
      } else if (split) {   // global partials (only instantiated without CSPLIT)
        // ticket: the last split to arrive sums all splits in split order.  The
        // barrier orders every thread's partial stores before the ticket
        // thread's release; its acquire (then the barrier) orders the
        // finalizer's loads after every other split's release.
        if (!dq_sync()) {
          ok = false;
          break;
        }
        if (dt == 0) {
          // the generation changes only after every CTA of this launch is done
          const uint32_t t = ticket_tagged(&p.counters[tile_id],
                                           ld_acquire_gpu(p.xbar + 2) % 0xFFFFFFu + 1u);
          *s_ticket = (t == (uint32_t)(nsp - 1)) ? 1 : 0;
        }
        if (!dq_sync()) {
          ok = false;
          break;
        }
        finalize_here = *s_ticket != 0;
        if (finalize_here) {
          // same column ownership as above; the 8 tokens of a chunk and two
          // splits at a time (plus, first, the residual) load together, and
          // splits add in split order
          for (int c0 = 8 * group; c0 < p.bn; c0 += 8 * kGroups) {
            float acc[8], res[8];
            epi.load_res8(m0 + c0, n, lane, res);
            for (int q0 = 0; q0 < nsp; q0 += 2) {
              float v[2][8];
        #pragma unroll
              for (int qq = 0; qq < 2; ++qq) {
                const float* part = p.ws + (int64_t)(q0 + qq) * p.M * p.N;
        #pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                  const int64_t m = m0 + c0 + jj;
                  v[qq][jj] = (q0 + qq < nsp && m < p.M && n < p.N) ? __ldcg(part + m * p.N + n)
                                                                     : 0.0f;
                }
              }
        #pragma unroll
              for (int qq = 0; qq < 2; ++qq)
        #pragma unroll
                for (int jj = 0; jj < 8; ++jj)
                  if (q0 + qq < nsp) acc[jj] = (q0 + qq == 0) ? v[0][jj] : acc[jj] + v[qq][jj];
            }
        #pragma unroll
            for (int jj = 0; jj < 8; ++jj) acc[jj] *= nscale;
            token_scales(m0 + c0, acc);
            epi.emit8(m0 + c0, n, acc, lane, res);
          }
        }
      }
      if (reduce && finalize_here) {
        if (!dq_sync()) {
          ok = false;
          break;
        }
        // the barrier above orders every dequant thread's pushes before the
        // releases
        ar_publish(rc, tile_id, epoch, dt);
      }
    }
    if (!ok) *abort_flag = 1;
  }

  // ------------------------------ teardown ------------------------------
  __syncthreads();
  // the last CTA to finish advances the ticket generation for the next launch
  // (every CTA's tickets precede its arrival here)
  if (p.counters && threadIdx.x == 0 && ticket_add(p.xbar + 3) == gridDim.x - 1u) {
    *reinterpret_cast<volatile uint32_t*>(p.xbar + 3) = 0u;   // ordered by the release below
    st_release_gpu(p.xbar + 2, ld_acquire_gpu(p.xbar + 2) + 1u);
  }
  // a CTA that gave up before arriving at the pre-pass barrier arrives now, so
  // the barrier words end every launch consistent (the error bit is set)
  if constexpr (XPRE) {
    if (threadIdx.x == 0 && !s_xb[1]) xbar_arrive();
  }
  // no CTA leaves while another CTA of its cluster may still write to its
  // shared memory or arrive on its barriers
  if constexpr (CSPLIT) cluster_sync();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"((uint32_t)p.tmem_cols)
                 : "memory");
  }

  if (reduce) {
    // ---- all-reduce phase 2 (one-shot: every tile; two-shot: see ar_finish_all)
    __shared__ int s_ok;
    const ArOut o{p.out, p.residual, p.bias, p.ldo, p.ldr, p.M, p.N, p.out_dtype,
                  (p.epilogue & IE_EPI_BIAS) != 0, (p.epilogue & IE_EPI_RESIDUAL) != 0};
    const int n_tiles = p.n_tiles, bn = p.bn;
    ar_finish_all<kThreads, kTileN>(rc, epoch, o, (int64_t)p.n_tiles * p.m_tiles,
                            [=](int64_t t, int64_t& n0, int64_t& m0, int& cols) {
                              n0 = (t % n_tiles) * kTileN;
                              m0 = (t / n_tiles) * bn;
                              cols = bn;
                            },
                            &s_ok);
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
  int acc_cols = 32, chains = 1, issuers = 1, tmem_cols = 512, sub = 1;
  int w_stage_bytes = 0;
  int t_kind = 0, t_rows = 0, t_stage_bytes = 0, nw_off = 0;
  size_t smem = 0;
  size_t ws_bytes = 0;       // counters + pre-pass activations + partials
  size_t counters_off = 0;   // split-K tile tickets, cleared by every launch that uses them
  size_t counters_bytes = 0;
  size_t xh_off = 0;         // pre-pass activations xh [M][K] f16 (F_FP8N: e4m3 bytes)
  size_t xs_off = 0;         // F_FP8N: per-token activation scales [M] f32
  size_t part_off = 0;       // split-K partials [splits][M][N] f32
  bool csplit = false;       // splits of a tile as one thread-block cluster
  bool streamk = false;      // stream-K order (splits = most CTAs sharing one tile)
  int grid = 0;              // CTAs launched (clusters: the cluster count decides)
  bool xpre = false;         // activation pre-pass (bf16 or RMS-norm activations)
  int recv_bytes = 0;
};

// Per-device caches are indexed by the current device's ordinal, so a process
// that drives GPUs of different sizes plans each launch for its own device.
constexpr int kMaxDevOrdinals = 64;

int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return (dev >= 0 && dev < kMaxDevOrdinals) ? dev : 0;
}

int sm_count() {
  static int n[kMaxDevOrdinals] = {};
  const int dev = current_device();
  if (!n[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    n[dev] = v > 0 ? v : 148;
  }
  return n[dev];
}

int fmt_of(const ie_qweight& w) {
  if (w.format == IE_FMT_INT8) return F_INT8;
  if (w.format == IE_FMT_FP8_E4M3) return F_FP8;
  return w.axis == IE_AXIS_GROUP128 ? F_INT4G : F_INT4SYM;
}

// Tile/split choice: BN covers the tokens (<= 256 per tile).  The split count
// minimises the slowest CTA's time in TMA-stage units: the stages of its units,
// a fixed cost per unit (pipeline drain and epilogue) and per split-K finalize,
// plus the f32 partials' extra traffic spread over the SMs.
Plan make_plan(const ie_qlinear_args& a, bool allow_split, bool allow_xpre) {
  Plan pl;
  pl.fmt = a.act_quant == IE_ACT_FP8_TOKEN ? F_FP8N : fmt_of(a.w);
  const bool native = pl.fmt == F_FP8N;
  const int xe = native ? 1 : 2;   // bytes of one x element in the MMA's B operand
  const int64_t M = a.m;
  pl.bn = (int)std::min<int64_t>(256, ((M + 15) / 16) * 16);
  pl.m_tiles = (int)((M + pl.bn - 1) / pl.bn);
  pl.n_tiles = (int)((a.w.n + kTileN - 1) / kTileN);
  pl.kstages = (int)(a.w.k / kBK);
  // Activations that need converting (bf16, or the RMS norm applied) can be
  // converted once per launch into the workspace (xh) instead of once per work
  // unit inside every CTA, at the price of a grid barrier before the first
  // MMA.  Measured on B200 (Llama-3-8B shapes, int4-g128) it pays for folded
  // norms above 16 tokens (each unit otherwise re-reads its tokens' rows for
  // the RMS factors: qkv 32.8 -> 28.7 us, gate/up 65.9 -> 48.9 us at 64
  // tokens) and for plain bf16 launches whose repeated conversion is large
  // (gate/up at 64 tokens 51.2 -> 47.5 us); at 16 tokens and on small grids
  // the barrier costs more (o 13.2 -> 16.9 us).
  {
    const bool norm = (a.epilogue & IE_EPI_RMS_NORM) != 0;
    const double per_sm = (double)pl.n_tiles * (double)M * (double)a.w.k / sm_count();
    const bool pays = norm ? M > 16 : per_sm >= 256.0 * 1024.0;
    pl.xpre = allow_xpre && (native || ((a.act_dtype == IE_DT_BF16 || norm) && pays));
  }
  const int row_stage = (pl.fmt == F_INT4G || pl.fmt == F_INT4SYM) ? kBK / 2 : kBK;
  // a TMA stage carries 32 KB of weights (4 int4 groups or 2 8-bit ones) when the
  // token tile leaves room: large stages amortise the barrier round trips
  pl.sub = row_stage == kBK / 2 ? 4 : 2;
  while (pl.sub > 1 && (size_t)pl.sub * (row_stage * kTileN + pl.bn * kBK * xe) > 100 * 1024)
    pl.sub /= 2;
  pl.w_stage_bytes = row_stage * kTileN * pl.sub;
  const int sms = sm_count();
  constexpr double kUnitCost = 1.5, kFinalizeCost = 1.5, kSkUnitCost = 1.0;
  double best = 1e300;
  const int tiles = pl.n_tiles * pl.m_tiles;
  const int tst = (pl.kstages + pl.sub - 1) / pl.sub;   // TMA stages along K
  // Token tiles up to 32 tokens may also reduce their splits inside a cluster
  // (2, 4 or 8 CTAs: those sizes pack the GPCs evenly, so a launch's clusters
  // are all resident at once), which finalizes slightly sooner than global
  // partials; each split count is scored both ways.
  const bool cluster_ok = pl.bn <= 8 * kGroups;
  constexpr double kClusterGain = 0.25;
  bool best_cluster = false;
  // (global split-K keeps one ticket per tile in the fixed ticket region)
  const bool split_ok = allow_split && (size_t)tiles * 4 <= kTicketBytes;
  for (int s = 1; s <= (split_ok ? 16 : 1); ++s) {
    if (s > 1 && tst < 2 * s) break;
    // every split must own at least one TMA stage: (s-1) * ceil(tst/s) < tst
    const int per = (tst + s - 1) / s;
    if ((s - 1) * per >= tst) continue;
    const int units = tiles * s;
    const int waves = (units + sms - 1) / sms;
    const double partial =
        s > 1 ? 2.0 * s * (double)M * a.w.n * 4.0 / ((double)sms * pl.w_stage_bytes) : 0.0;
    const double t = waves * (per + kUnitCost + (s > 1 ? kFinalizeCost : 0.0)) + partial;
    // Token tiles that can reduce their splits inside a cluster never take
    // global partials: measured on B200, the Llama-3-8B int4 decode step at 16
    // tokens runs 3.10 ms with qkv on cluster split-K against 3.29 ms with its
    // 3-way global split (the ticket round trips sit on every tile's finalize).
    if ((s == 1 || !cluster_ok) && t < best - 1e-9) {
      best = t;
      pl.splits = s;
      best_cluster = false;
    }
    if (cluster_ok && (s == 2 || s == 4 || s == 8) && t - kClusterGain < best - 1e-9) {
      best = t - kClusterGain;
      pl.splits = s;
      best_cluster = true;
    }
  }
  // Stream-K: one CTA per SM, each taking an equal contiguous range of the
  // tile-major (tile, TMA stage) order, so no SM idles through a last partial
  // wave; a tile shared by several ranges is finished by ticket from global
  // partials.  The longest range pays a unit cost for every tile it touches.
  // Measured on B200 it pays only for the native fp8 contraction over at
  // least one full wave of tiles (Llama-3-70B gate/up at 32 tokens: 103 ->
  // 93 us): where the dequant warps also run the epilogue (int4 / int8 / fp8
  // dequantized), the extra segment epilogues and partials cost more than
  // the tail they remove (Llama-3-8B int4 gate/up at 16 tokens: 37 -> 43 us),
  // and on shorter grids the split plans already balance the SMs.
  if (split_ok && native && tiles >= sms) {
    const int64_t total = (int64_t)tiles * tst;
    const int g = (int)std::min<int64_t>(sms, total);
    // (the kernel's schedule arithmetic is 32-bit: (total + 1) * g < 2^31)
    const bool fits32 = (total + 1) * g < (int64_t)1 << 31;
    const int64_t q = total / g;   // stages of the shortest range
    const double longest = std::ceil((double)total / g);
    const int touched = (int)std::ceil(longest / tst) + 1;
    const int max_seg = (int)((tst - 1 + q - 1) / q) + 1;
    const double partial = 4.0 * (double)std::min<int64_t>(M, pl.bn) * kTileN * 4.0 /
                           pl.w_stage_bytes;
    const double t = longest + touched * kSkUnitCost + kFinalizeCost + partial;
    if (fits32 && max_seg > 1 && t < best - 1e-9) {
      best = t;
      pl.streamk = true;
      pl.splits = max_seg;
      best_cluster = false;
      pl.grid = g;
    }
  }
  if (!pl.streamk) pl.grid = std::min(tiles * pl.splits, sms);
  int tbytes = 0;   // table bytes of a stage
  if (a.w.axis == IE_AXIS_GROUP128) {
    pl.t_kind = 1;
    tbytes = 2 * kTileN * 2 * pl.sub;
  } else if (a.w.axis == IE_AXIS_K) {
    pl.t_kind = 2;
    pl.t_rows = a.w.gate_up ? 2 : 1;
    tbytes = pl.t_rows * kBK * 4 * pl.sub;
  }
  // the RMS-norm weights of a stage follow its tables in the same slot (only
  // when the x tiles are normalised in the loop, not by the pre-pass)
  pl.nw_off = (tbytes + 15) / 16 * 16;
  if ((a.epilogue & IE_EPI_RMS_NORM) && !pl.xpre) tbytes = pl.nw_off + kBK * 4 * pl.sub;
  pl.t_stage_bytes = (tbytes + 1023) / 1024 * 1024;
  // TMEM: accumulators, then the A ring (64 columns a sub-stage).  Narrow token
  // tiles rotate their MMAs over independent accumulator chains, and two issuing
  // threads take alternate sub-stages into separate accumulators whenever TMEM
  // holds both sets next to a 4-deep A ring: a single issuer leaves the tensor
  // pipe idle between its sub-stages (barrier wait, fence, commit), and shares
  // its scheduler with two dequant warps.
  pl.acc_cols = ((pl.bn + 15) / 16) * 16;
  // (Two chains for tiles up to 64 tokens: four were no faster in the mainloop
  // and cost the epilogue a second TMEM round trip for the extra accumulators.)
  pl.chains = pl.bn <= 64 ? 2 : 1;
  pl.issuers = (2 * pl.acc_cols * pl.chains + (native ? 0 : 4 * kACols) <= 512) ? 2 : 1;
  const int accs = pl.acc_cols * pl.chains * pl.issuers;
  // The A ring covers a sub-stage's dequant plus its MMAs' latency (8 MMAs take
  // ~0.45 us from issue to commit), so it is as deep as TMEM allows.  F_FP8N
  // reads A from shared memory and has none.
  pl.na = native ? 0
                 : (accs + kMaxAStages * kACols <= 512 ? kMaxAStages
                                                       : (accs + 4 * kACols <= 512 ? 4 : 2));
  pl.tmem_cols = 32;
  while (pl.tmem_cols < accs + pl.na * kACols) pl.tmem_cols *= 2;
  const size_t x_stage = (size_t)pl.bn * kBK * xe * pl.sub;
  // Small token tiles: the splits of a tile run as one cluster and reduce
  // through the leader's shared memory (receive buffer); no workspace.
  if (pl.splits > 1 && best_cluster) {
    pl.csplit = true;
    pl.recv_bytes = (pl.splits - 1) * pl.bn * kTileN * 4;
  }
  const size_t budget = 220 * 1024;
  const size_t fixed = 1024 + 256 + (size_t)pl.recv_bytes;
  const size_t per = x_stage + pl.w_stage_bytes + pl.t_stage_bytes;
  pl.ns = (int)std::min<size_t>(12, (budget - fixed) / per);
  if (pl.ns < 2) pl.ns = 2;
  // barriers, then TMEM slot, abort flag, ticket, the RMS factors and the pre-pass words
  pl.smem = fixed + (size_t)pl.ns * per + 8 * (3 * pl.ns + 2 * pl.na + 2 + kMmaWarps + 3) + 16 +
            4 * (size_t)std::max(pl.bn, kDqWarps) + 8;
  if (pl.smem < (size_t)kMinSmem) pl.smem = kMinSmem;   // one CTA per SM: TMEM and co-residency
  // workspace: [barrier and generation words, 256 B | tile tickets | xh |
  // split-K partials].  The words at offset 0 serve every plan and keep
  // themselves consistent (zero on first use); the tickets carry the launch's
  // tag, so they are never cleared.
  const bool global_split = pl.splits > 1 && !pl.csplit;   // stream-K included
  pl.counters_off = 256;
  // a fixed ticket region for every plan that has a workspace: the words are
  // only ever written as tickets (another plan's xh or partials never land
  // there), so a leftover word always carries some launch's tag
  pl.counters_bytes = kTicketBytes;
  pl.xh_off = pl.counters_off + pl.counters_bytes;
  const size_t xh_bytes = pl.xpre ? ((size_t)M * a.w.k * xe + 255) / 256 * 256 : 0;
  pl.xs_off = pl.xh_off + xh_bytes;
  const size_t xs_bytes = native ? ((size_t)M * 4 + 255) / 256 * 256 : 0;
  pl.part_off = pl.xs_off + xs_bytes;
  const size_t part_bytes = global_split ? (size_t)pl.splits * M * a.w.n * 4 : 0;
  pl.ws_bytes = (global_split || pl.xpre) ? pl.part_off + part_bytes : 0;
  return pl;
}

// The best plan whose workspace fits in `avail` bytes: split-K and the
// activation pre-pass, then split-K alone (cluster split-K needs no
// workspace), then the pre-pass alone, then neither.
Plan fitting_plan(const ie_qlinear_args& a, size_t avail) {
  Plan pl = make_plan(a, true, true);
  if (pl.ws_bytes > avail) pl = make_plan(a, true, false);
  if (pl.ws_bytes > avail) pl = make_plan(a, false, true);
  if (pl.ws_bytes > avail) pl = make_plan(a, false, false);
  return pl;
}

bool tc_eligible(const ie_qlinear_args& a) {
  if (a.act_dtype != IE_DT_BF16 && a.act_dtype != IE_DT_F16) return false;
  if (a.w.k % kBK) return false;
  if (((uintptr_t)a.x & 15) || ((a.ldx * 2) & 15)) return false;
  if (((uintptr_t)a.w.codes & 15)) return false;
  if (((uintptr_t)a.w.scale & 15)) return false;
  if (a.w.axis == IE_AXIS_GROUP128 && ((a.w.n % 8) || ((uintptr_t)a.w.zero & 15))) return false;
  if ((a.epilogue & IE_EPI_RMS_NORM) && ((uintptr_t)a.norm_weight & 15)) return false;
  return encode_fn() != nullptr;
}

template <int FMT>
int launch_typed(const ie_qlinear_args& a, const Plan& pl, const CUtensorMap& tw,
                 const CUtensorMap& tx, const CUtensorMap& ts, const CUtensorMap& tz,
                 const TcParams& prm, const ReduceCtx* rc, cudaStream_t s) {
  // (F_FP8N always has the pre-pass: it makes the e4m3 activations)
  decltype(&qgemm_tc_kernel<FMT, false, true>) kern;
  if constexpr (FMT == F_FP8N) {
    kern = pl.csplit ? qgemm_tc_kernel<FMT, true, true> : qgemm_tc_kernel<FMT, false, true>;
  } else {
    kern = pl.csplit ? (pl.xpre ? qgemm_tc_kernel<FMT, true, true>
                                : qgemm_tc_kernel<FMT, true, false>)
                     : (pl.xpre ? qgemm_tc_kernel<FMT, false, true>
                                : qgemm_tc_kernel<FMT, false, false>);
  }
  IE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)pl.smem));
  ReduceCtx none{};
  const ReduceCtx ctx = rc ? *rc : none;
  const int reduce = rc ? 1 : 0;
  // programmatic dependent launch (TcParams::pdl): the kernel may start while
  // the previous kernel on the stream finishes
  cudaLaunchAttribute pdl_attr;
  pdl_attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  pdl_attr.val.programmaticStreamSerializationAllowed = 1;
  if (!pl.csplit) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)pl.grid);
    cfg.blockDim = dim3((unsigned)kThreads);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = s;
    cfg.attrs = &pdl_attr;
    cfg.numAttrs = prm.pdl ? 1 : 0;
    IE_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, tw, tx, ts, tz, prm, ctx, reduce));
    return launch_status("qgemm_tc_kernel");
  }
  // cluster split-K: one cluster of `splits` CTAs per tile in flight, as many
  // clusters as the device holds at once (every CTA co-resident, which the
  // fused all-reduce relies on)
  const int tiles = pl.n_tiles * pl.m_tiles;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3((unsigned)kThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)pl.splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3((unsigned)(tiles * pl.splits));
  // occupancy of one (shared memory, cluster size) configuration, per device
  static std::mutex mu;
  static int cached_key[kMaxDevOrdinals][kFmts], cached_max[kMaxDevOrdinals][kFmts];
  static bool cache_init = false;
  int max_clusters = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!cache_init) {
      for (auto& row : cached_key)
        for (int& k : row) k = -1;
      cache_init = true;
    }
    const int dev = current_device();
    const int key = ((int)pl.smem * 16 + pl.splits) * 2 + (pl.xpre ? 1 : 0);
    if (cached_key[dev][FMT] == key) {
      max_clusters = cached_max[dev][FMT];
    } else {
      IE_CUDA_TRY(cudaOccupancyMaxActiveClusters(&max_clusters, (const void*)kern, &cfg));
      cached_key[dev][FMT] = key;
      cached_max[dev][FMT] = max_clusters;
    }
  }
  if (max_clusters <= 0)
    return set_error(IE_ERR_UNSUPPORTED, "qlinear: no cluster of %d CTAs with %zu bytes of shared "
                                         "memory fits on this device", pl.splits, pl.smem);
  TcParams prm2 = prm;
  prm2.nclusters = std::min(tiles, max_clusters);
  cfg.gridDim = dim3((unsigned)(prm2.nclusters * pl.splits));
  if (prm.pdl) {
    attr[1] = pdl_attr;
    cfg.numAttrs = 2;
  }
  IE_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, tw, tx, ts, tz, prm2, ctx, reduce));
  return launch_status("qgemm_tc_kernel");
}

}  // namespace tc

size_t tc_workspace_bytes(const ie_qlinear_args& a) {
  if (!tc::tc_eligible(a)) return 0;
  return tc::make_plan(a, true, true).ws_bytes;
}

bool tc_usable(const ie_qlinear_args& a) { return tc::tc_eligible(a); }

int64_t tc_tiles(const ie_qlinear_args& a) {
  const tc::Plan pl = tc::fitting_plan(a, a.workspace ? a.workspace_bytes : 0);
  return (int64_t)pl.n_tiles * pl.m_tiles;
}

int launch_qlinear_tc(const ie_qlinear_args& a, const ReduceCtx* rc, cudaStream_t s) {
  using namespace tc;
  IE_CHECK(tc_eligible(a), "qlinear: the tensor-core path needs bf16/f16 activations, K %% 128 "
                           "== 0, 16-byte aligned rows (and norm weight) and the driver's TMA "
                           "encoder");
  const Plan pl = fitting_plan(a, a.workspace ? a.workspace_bytes : 0);
  if (pl.fmt == F_FP8N && !pl.xpre)
    return set_error(IE_ERR_INVALID, "qlinear: fp8 activations need a workspace of %zu bytes "
                                     "(ie_qlinear_workspace_size); %zu given",
                     make_plan(a, false, true).ws_bytes, a.workspace ? a.workspace_bytes : 0);
  // the pre-pass producer remembers a stage's x coordinates in 16 bits each
  IE_CHECK(!pl.xpre || (pl.m_tiles < 65536 && pl.kstages < 65536),
           "qlinear: %d token tiles / %d K stages exceed the pre-pass limits", pl.m_tiles,
           pl.kstages);
  EncodeFn enc = encode_fn();
  CUtensorMap tw, tx;
  {
    const cuuint64_t row_bytes = (cuuint64_t)(a.w.format == IE_FMT_INT4 ? a.w.k / 2 : a.w.k);
    const cuuint64_t dims[2] = {row_bytes, (cuuint64_t)a.w.n};
    const cuuint64_t strides[1] = {row_bytes};
    const int row_sub = pl.w_stage_bytes / pl.sub / kTileN;   // bytes of one row per sub-stage
    const cuuint32_t box[2] = {(cuuint32_t)row_sub, (cuuint32_t)kTileN};
    const cuuint32_t estr[2] = {1, 1};
    // 64-byte int4 rows use the 64-byte swizzle, 128-byte 8-bit rows the 128-byte one,
    // so the dequant threads (one row each) read distinct banks
    const CUtensorMapSwizzle sw = row_sub == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                : CU_TENSOR_MAP_SWIZZLE_128B;
    CUresult r = enc(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(a.w.codes), dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(IE_ERR_CUDA, "cuTensorMapEncodeTiled(weights): %d", (int)r);
  }
  char* ws = static_cast<char*>(a.workspace);
  {
    // x viewed as [K/64][M][64]: one box {64, BN, 2} is a stage's two SW128 blocks;
    // with the pre-pass the tiles come from xh (f16, rows of K)
    // (F_FP8N: e4m3 codes [K/128][M][128 bytes], one block {128, BN, sub} a stage)
    const bool native = pl.fmt == F_FP8N;
    const int64_t ld = pl.xpre ? a.w.k : a.ldx;
    const cuuint64_t inner = native ? 128 : 64;
    const cuuint64_t dims[3] = {inner, (cuuint64_t)a.m, (cuuint64_t)(a.w.k / inner)};
    const cuuint64_t strides[2] = {(cuuint64_t)ld * (native ? 1 : 2), 128};
    const cuuint32_t box[3] = {(cuuint32_t)inner, (cuuint32_t)pl.bn,
                               (cuuint32_t)((native ? 1 : 2) * pl.sub)};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapDataType dt = native ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                   : (a.act_dtype == IE_DT_BF16 && !pl.xpre)
                                       ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    void* base = pl.xpre ? static_cast<void*>(ws + pl.xh_off) : const_cast<void*>(a.x);
    CUresult r = enc(&tx, dt, 3, base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(IE_ERR_CUDA, "cuTensorMapEncodeTiled(x): %d", (int)r);
  }
  CUtensorMap ts = tw, tz = tw;   // unused copies when the stage carries no tables
  const bool joint = pl.t_kind == 1 &&
                     static_cast<const char*>(a.w.zero) ==
                         static_cast<const char*>(a.w.scale) + (a.w.k / 128) * a.w.n * 2;
  if (joint) {
    const cuuint64_t dims[3] = {(cuuint64_t)a.w.n, (cuuint64_t)(a.w.k / 128), 2};
    const cuuint64_t strides[2] = {(cuuint64_t)a.w.n * 2, (cuuint64_t)(a.w.k / 128) * a.w.n * 2};
    const cuuint32_t box[3] = {(cuuint32_t)kTileN, (cuuint32_t)pl.sub, 2};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(&ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(a.w.scale), dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(IE_ERR_CUDA, "cuTensorMapEncodeTiled(tables): %d", (int)r);
  } else if (pl.t_kind == 1) {
    const cuuint64_t dims[2] = {(cuuint64_t)a.w.n, (cuuint64_t)(a.w.k / 128)};
    const cuuint64_t strides[1] = {(cuuint64_t)a.w.n * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kTileN, (cuuint32_t)pl.sub};
    const cuuint32_t estr[2] = {1, 1};
    for (int i = 0; i < 2; ++i) {
      CUresult r = enc(i ? &tz : &ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                       const_cast<void*>(i ? a.w.zero : a.w.scale), dims, strides, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r != CUDA_SUCCESS) return set_error(IE_ERR_CUDA, "cuTensorMapEncodeTiled(groups): %d", (int)r);
    }
  } else if (pl.t_kind == 2) {
    // per-K scales viewed as [rows][K/128][128]
    const cuuint64_t dims[3] = {(cuuint64_t)kBK, (cuuint64_t)(a.w.k / kBK), (cuuint64_t)pl.t_rows};
    const cuuint64_t strides[2] = {(cuuint64_t)kBK * 4, (cuuint64_t)a.w.k * 4};
    const cuuint32_t box[3] = {(cuuint32_t)kBK, (cuuint32_t)pl.sub, (cuuint32_t)pl.t_rows};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(&ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(a.w.scale), dims,
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
  if (a.w.axis != IE_AXIS_GROUP128) prm.scale = static_cast<const float*>(a.w.scale);
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
  prm.acc_cols = pl.acc_cols;
  prm.chains = pl.chains;
  prm.issuers = pl.issuers;
  prm.tmem_cols = pl.tmem_cols;
  prm.w_stage_bytes = pl.w_stage_bytes;
  prm.t_kind = pl.t_kind;
  prm.t_rows = pl.t_rows;
  prm.t_stage_bytes = pl.t_stage_bytes;
  prm.t_joint = joint ? 1 : 0;
  prm.sub = pl.sub;
  prm.csplit = pl.csplit ? 1 : 0;
  prm.recv_bytes = pl.recv_bytes;
  prm.streamk = pl.streamk ? 1 : 0;
  if (pl.splits > 1 && !pl.csplit) {
    // tickets tagged with the launch generation (TcParams::xbar): a launch that
    // gave up part-way leaves counted tickets that the next launch ignores
    prm.counters = reinterpret_cast<uint32_t*>(ws + pl.counters_off);
    prm.ws = reinterpret_cast<float*>(ws + pl.part_off);
    prm.xbar = reinterpret_cast<uint32_t*>(ws);
  }
  prm.x_bf16 = a.act_dtype == IE_DT_BF16 ? 1 : 0;
  if (a.epilogue & IE_EPI_RMS_NORM) {
    prm.norm_w = a.norm_weight;
    prm.norm_eps = a.norm_eps;
    prm.nw_off = pl.nw_off;
  }
  if ((a.epilogue & IE_EPI_RMS_NORM) || pl.xpre) {
    prm.x = a.x;
    prm.ldx = a.ldx;
  }
  // every launch may overlap the previous kernel's tail
  prm.pdl = 1;
  if (pl.xpre) {
    prm.xh = reinterpret_cast<__half*>(ws + pl.xh_off);
    prm.xbar = reinterpret_cast<uint32_t*>(ws);
    if (pl.fmt == F_FP8N) prm.xs = reinterpret_cast<float*>(ws + pl.xs_off);
  }
  switch (pl.fmt) {
    case F_INT4G: return launch_typed<F_INT4G>(a, pl, tw, tx, ts, tz, prm, rc, s);
    case F_INT4SYM: return launch_typed<F_INT4SYM>(a, pl, tw, tx, ts, tz, prm, rc, s);
    case F_INT8: return launch_typed<F_INT8>(a, pl, tw, tx, ts, tz, prm, rc, s);
    case F_FP8N: return launch_typed<F_FP8N>(a, pl, tw, tx, ts, tz, prm, rc, s);
    default: return launch_typed<F_FP8>(a, pl, tw, tx, ts, tz, prm, rc, s);
  }
}

// ---------------------------------------------------------------------------
// Static split-K scratch (ie_qlinear_noalloc).  Callers that may not allocate
// device memory at call time -- an engine whose allocator has already claimed
// every byte of HBM it may use, or a real-time decode loop that must never
// enter the CUDA allocator -- still need somewhere for the f32 split-K
// partials and tile tickets.  This
// array is part of the module image: the driver reserves it on each device
// when the module loads, so using it never allocates.  It is shared by every
// call on a device: two such calls overlapping on the GPU (different streams,
// or threads without ordering between them) race on the partials and tickets.
namespace tc {

static_assert(IE_QLINEAR_NOALLOC_SCRATCH_BYTES % 256 == 0, "scratch size");
static __device__ __align__(256) unsigned char g_static_scratch[IE_QLINEAR_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::once_flag g_scratch_once[kMaxDevices];
void* g_scratch_ptr[kMaxDevices];
cudaError_t g_scratch_err[kMaxDevices];

// Device address of this device's copy of the array, looked up once per device
// with that device current (the look-up may load the module, which is why the
// first call on a device belongs before any stream capture).
int static_scratch(void** out) {
  int dev = 0;
  IE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(IE_ERR_UNSUPPORTED, "qlinear_noalloc: device ordinal %d >= %d", dev,
                     kMaxDevices);
  std::call_once(g_scratch_once[dev], [dev] {
    void* p = nullptr;
    g_scratch_err[dev] = cudaGetSymbolAddress(&p, g_static_scratch);
    g_scratch_ptr[dev] = g_scratch_err[dev] == cudaSuccess ? p : nullptr;
  });
  if (g_scratch_err[dev] != cudaSuccess)
    return set_error(IE_ERR_CUDA, "qlinear_noalloc: cudaGetSymbolAddress(scratch) on device %d: %s",
                     dev, cudaGetErrorString(g_scratch_err[dev]));
  *out = g_scratch_ptr[dev];
  return IE_OK;
}

}  // namespace tc

int launch_qlinear_tc_static(const ie_qlinear_args& a, cudaStream_t s) {
  using namespace tc;
  void* scratch = nullptr;
  int rc = static_scratch(&scratch);
  if (rc || a.m == 0) return rc;
  if (a.algo == 1 || !tc_eligible(a))
    return set_error(IE_ERR_UNSUPPORTED,
                     "qlinear_noalloc: only the tensor-core path is served (bf16/f16 "
                     "activations, K %% 128 == 0, 16-byte aligned rows, algo 0 or 2)");
  ie_qlinear_args b = a;
  b.workspace = scratch;
  b.workspace_bytes = IE_QLINEAR_NOALLOC_SCRATCH_BYTES;
  // launch_qlinear_tc runs the best plan whose scratch fits in the array
  // (fitting_plan: split-K and the activation pre-pass, the pre-pass alone, or
  // neither); its tile tickets carry the launch's tag and the barrier and
  // generation words (zero at module load) keep themselves consistent, so a
  // call that ended early leaves nothing to clear
  return launch_qlinear_tc(b, nullptr, s);
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
