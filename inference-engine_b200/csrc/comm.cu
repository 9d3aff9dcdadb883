// Tensor-parallel communicator: one process per GPU, peers reach each other's
// landing buffers over NVLink through CUDA IPC mappings.
//
// One device allocation per rank holds, in order:
//   landing[2][world][slot_floats] f32   (double-buffered by call parity)
//   flags[kMaxTiles][kMaxWorld] u32      (epoch of the last push per tile/source)
//   status u32, epoch u32, done u32      (timeout status, call counter, CTA counter)
// A collective call e pushes f32 partials into slot [rank] of every rank's
// landing[e % 2], then stores epoch e with release semantics into that rank's
// flags[tile][rank].  Readers wait (bounded) for flags >= e and sum the slots in
// rank order.  Rank r can only run call e+2 -- which reuses parity e % 2 --
// after every peer pushed call e+1, which each peer does only after finishing
// call e, so a slot is never overwritten while it is still being read.
// The epoch is kept on the device and advanced by the kernels themselves, so
// captured CUDA graphs replay correctly.
#include <cstring>
#include <mutex>

#include "common.cuh"

struct ie_comm {
  int32_t rank = 0, world = 1, device = 0;
  int64_t slot_floats = 0;
  size_t landing_bytes = 0;     // one parity: world * slot_floats * 4
  size_t flags_offset = 0, status_offset = 0, total_bytes = 0;
  void* base = nullptr;
  void* peer_base[ie::kMaxWorld] = {};
  bool peer_opened[ie::kMaxWorld] = {};
  uint64_t timeout_ns = 2000000000ull;
  bool open = false;
  unsigned char own_handle[IE_COMM_HANDLE_BYTES] = {};
};

namespace ie {

constexpr int64_t kMaxTiles = 1 << 16;

// Smallest NVLink saving per rank (bytes) for which IE_AR_AUTO takes two-shot:
// about the cost of its second flag round trip at the measured ~770 GB/s.
constexpr double kTwoShotMinSavedBytes = 2.5e6;

int resolve_algo(int32_t world, int64_t tiles, int64_t numel, int32_t algo) {
  if (algo == IE_AR_ONESHOT) return kArOneShot;
  if (algo == IE_AR_TWOSHOT) return tiles >= world ? kArTwoShot : kArOneShot;
  if (algo != IE_AR_AUTO) return -1;
  if (world < 4 || tiles < world) return kArOneShot;
  const double saved = (double)numel * (4.0 * (world - 1) - 8.0 * (world - 1) / world);
  return saved >= kTwoShotMinSavedBytes ? kArTwoShot : kArOneShot;
}

int comm_context(ie_comm* c, ReduceCtx* rc, int64_t tiles, int64_t floats_per_rank,
                 int32_t algo) {
  IE_CHECK(c && c->open, "comm: not open (call ie_comm_open first)");
  if (algo == IE_AR_NVLS)
    return set_error(IE_ERR_UNSUPPORTED, "comm: the NVLS (multicast) all-reduce is not built");
  IE_CHECK(algo >= IE_AR_AUTO && algo <= IE_AR_TWOSHOT, "comm: unknown all-reduce algo %d", algo);
  IE_CHECK(tiles <= kMaxTiles, "comm: %lld tiles exceed the flag table (%lld)",
           (long long)tiles, (long long)kMaxTiles);
  IE_CHECK(floats_per_rank <= c->slot_floats,
           "comm: %lld f32 values exceed the landing slot (%lld); create the comm with a "
           "larger max_bytes", (long long)floats_per_rank, (long long)c->slot_floats);
  int dev = -1;
  IE_CUDA_TRY(cudaGetDevice(&dev));
  IE_CHECK(dev == c->device, "comm: current device %d is not the comm's device %d", dev,
           c->device);
  *rc = ReduceCtx{};
  for (int r = 0; r < c->world; ++r) {
    char* b = static_cast<char*>(c->peer_base[r]);
    rc->landing[r] = reinterpret_cast<float*>(b);
    rc->flags[r] = reinterpret_cast<uint32_t*>(b + c->flags_offset);
  }
  char* mine = static_cast<char*>(c->base) + c->status_offset;
  rc->status = reinterpret_cast<uint32_t*>(mine);
  rc->epoch_dev = reinterpret_cast<uint32_t*>(mine + 4);
  rc->done = reinterpret_cast<uint32_t*>(mine + 8);
  rc->timeout_ns = c->timeout_ns;
  rc->parity_stride = (int64_t)(c->landing_bytes / sizeof(float));
  rc->slot_floats = c->slot_floats;
  rc->rank = c->rank;
  rc->world = c->world;
  rc->algo = resolve_algo(c->world, tiles, floats_per_rank, algo);
  return IE_OK;
}

namespace {

constexpr int kARThreads = 256;
constexpr int kARTile = 2048;   // elements per all-reduce tile

template <typename T>
__global__ void __launch_bounds__(kARThreads)
allreduce_kernel(const T* __restrict__ in, T* __restrict__ out, int64_t n, ReduceCtx rc) {
  const uint32_t epoch = reduce_epoch(rc);
  const int64_t tiles = (n + kARTile - 1) / kARTile;
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int64_t b = t * kARTile;
    int d0, d1;
    ar_push_range(rc, t, d0, d1);
    for (int i = threadIdx.x; i < kARTile; i += kARThreads) {
      const int64_t e = b + i;
      if (e >= n) break;
      const float v = to_f32<T>(in[e]);
      for (int dst = d0; dst < d1; ++dst)
        landing_slot(rc, dst, epoch)[rc.rank * rc.slot_floats + e] = v;
    }
    __syncthreads();
    ar_publish(rc, t, epoch, threadIdx.x);
  }
  // the flat array as one token row of n values, tile t = [t * kARTile, ...)
  __shared__ int s_ok;
  const ArOut o{out, nullptr, nullptr, n, 0, 1, n, dtype_of<T>(), false, false};
  ar_finish_all<kARThreads, kARTile>(rc, epoch, o, tiles,
                            [](int64_t t, int64_t& n0, int64_t& m0, int& cols) {
                              n0 = t * kARTile;
                              m0 = 0;
                              cols = 1;
                            },
                            &s_ok);
  __syncthreads();
  reduce_finish(rc, epoch);
}

template <typename T>
int resident_allreduce_ctas(int* out) {
  int per_sm = 0, dev = 0, sms = 0;
  IE_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, allreduce_kernel<T>,
                                                            kARThreads, 0));
  IE_CUDA_TRY(cudaGetDevice(&dev));
  IE_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  *out = per_sm * sms;
  return IE_OK;
}

template <typename T>
int launch_allreduce(ie_comm* c, const void* in, void* out, int64_t n, int32_t algo,
                     cudaStream_t s) {
  const int64_t tiles = (n + kARTile - 1) / kARTile;
  ReduceCtx rc;
  int rcode = comm_context(c, &rc, tiles, n, algo);
  if (rcode) return rcode;
  int resident = 0;
  rcode = resident_allreduce_ctas<T>(&resident);
  if (rcode) return rcode;
  const int64_t grid = std::min<int64_t>(tiles, std::max(resident, 1));
  allreduce_kernel<T><<<(unsigned)grid, kARThreads, 0, s>>>(static_cast<const T*>(in),
                                                            static_cast<T*>(out), n, rc);
  return launch_status("allreduce_kernel");
}

}  // namespace
}  // namespace ie

using namespace ie;

extern "C" int ie_comm_create(int32_t rank, int32_t world, int32_t device, size_t max_bytes,
                              ie_comm** out) {
  IE_CHECK(out, "comm_create: null output");
  *out = nullptr;
  IE_CHECK(world >= 1 && world <= kMaxWorld, "comm_create: world %d outside [1, %d]", world,
           kMaxWorld);
  IE_CHECK(rank >= 0 && rank < world, "comm_create: rank %d outside world of %d", rank, world);
  IE_CHECK(max_bytes >= 4, "comm_create: max_bytes must hold at least one f32");
  ie_comm* c = new ie_comm();
  c->rank = rank;
  c->world = world;
  c->device = device;
  c->slot_floats = (int64_t)((max_bytes + 255) / 256 * 64);
  c->landing_bytes = (size_t)world * (size_t)c->slot_floats * sizeof(float);
  c->flags_offset = 2 * c->landing_bytes;
  c->status_offset = c->flags_offset + (size_t)kMaxTiles * kMaxWorld * sizeof(uint32_t);
  c->total_bytes = c->status_offset + 256;   // status, epoch, done counter
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaMalloc(&c->base, c->total_bytes);
  if (e == cudaSuccess) e = cudaMemset(c->base, 0, c->total_bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (c->base) cudaFree(c->base);
    delete c;
    return set_error(IE_ERR_CUDA, "comm_create: %s", cudaGetErrorString(e));
  }
  c->peer_base[rank] = c->base;
  *out = c;
  return IE_OK;
}

extern "C" int ie_comm_export(ie_comm* c, void* handle_out) {
  IE_CHECK(c && handle_out, "comm_export: null pointer");
  static_assert(sizeof(cudaIpcMemHandle_t) == IE_COMM_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  IE_CUDA_TRY(cudaSetDevice(c->device));
  IE_CUDA_TRY(cudaIpcGetMemHandle(&h, c->base));
  std::memcpy(handle_out, &h, sizeof(h));
  std::memcpy(c->own_handle, &h, sizeof(h));
  return IE_OK;
}

extern "C" int ie_comm_open(ie_comm* c, const void* handles) {
  IE_CHECK(c && handles, "comm_open: null pointer");
  IE_CHECK(!c->open, "comm_open: already open");
  IE_CUDA_TRY(cudaSetDevice(c->device));
  const unsigned char* hb = static_cast<const unsigned char*>(handles);
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank) continue;
    const unsigned char* h = hb + (size_t)r * IE_COMM_HANDLE_BYTES;
    if (std::memcmp(h, c->own_handle, IE_COMM_HANDLE_BYTES) == 0) {
      // Loopback: a handle equal to this rank's own maps to its own buffer.
      // Used by single-GPU tests of the wait / timeout path; no peer exists.
      c->peer_base[r] = c->base;
      continue;
    }
    cudaIpcMemHandle_t ih;
    std::memcpy(&ih, h, sizeof(ih));
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, ih, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess)
      return set_error(IE_ERR_CUDA, "comm_open: cudaIpcOpenMemHandle(rank %d): %s", r,
                       cudaGetErrorString(e));
    c->peer_base[r] = p;
    c->peer_opened[r] = true;
  }
  c->open = true;
  return IE_OK;
}

extern "C" int ie_comm_destroy(ie_comm* c) {
  if (!c) return IE_OK;
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  for (int r = 0; r < c->world; ++r)
    if (c->peer_opened[r]) cudaIpcCloseMemHandle(c->peer_base[r]);
  if (c->base) cudaFree(c->base);
  delete c;
  return IE_OK;
}

extern "C" int ie_comm_set_timeout(ie_comm* c, uint64_t ns) {
  IE_CHECK(c, "comm_set_timeout: null comm");
  IE_CHECK(ns > 0, "comm_set_timeout: timeout must be positive");
  c->timeout_ns = ns;
  return IE_OK;
}

extern "C" int ie_comm_check(ie_comm* c) {
  IE_CHECK(c, "comm_check: null comm");
  IE_CUDA_TRY(cudaSetDevice(c->device));
  uint32_t st = 0;
  uint32_t* dst = reinterpret_cast<uint32_t*>(static_cast<char*>(c->base) + c->status_offset);
  IE_CUDA_TRY(cudaDeviceSynchronize());
  IE_CUDA_TRY(cudaMemcpy(&st, dst, sizeof(st), cudaMemcpyDeviceToHost));
  if (st != 0) {
    IE_CUDA_TRY(cudaMemset(dst, 0, sizeof(uint32_t)));
    return set_error(IE_ERR_TIMEOUT, "comm: a peer wait timed out (status %u)", st);
  }
  return IE_OK;
}

extern "C" int ie_allreduce_resolve(int32_t world, int64_t tiles, int64_t numel,
                                    int32_t algo) {
  if (world < 1 || world > kMaxWorld || tiles < 0 || numel < 0) return -1;
  const int r = resolve_algo(world, tiles, numel, algo);
  return r == kArTwoShot ? IE_AR_TWOSHOT : r == kArOneShot ? IE_AR_ONESHOT : -1;
}

extern "C" int ie_allreduce(ie_comm* c, const void* in, void* out, int64_t numel, int32_t dtype,
                            int32_t algo, void* stream) {
  IE_CHECK(c, "allreduce: null comm");
  IE_CHECK(numel >= 0, "allreduce: negative size");
  if (numel == 0) return IE_OK;
  IE_CHECK(in && out, "allreduce: null pointer");
  cudaStream_t s = as_stream(stream);
  if (dtype == IE_DT_F32) return launch_allreduce<float>(c, in, out, numel, algo, s);
  if (dtype == IE_DT_BF16) return launch_allreduce<__nv_bfloat16>(c, in, out, numel, algo, s);
  if (dtype == IE_DT_F16) return launch_allreduce<__half>(c, in, out, numel, algo, s);
  return set_error(IE_ERR_INVALID, "allreduce: unsupported dtype %d", dtype);
}
