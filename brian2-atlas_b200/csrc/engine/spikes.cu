// Spike bitmap -> ascending spike index list, as a stand-alone device
// primitive of the C ABI (b2g_spikes_from_bitmap).
//
// A GPU-side caller that evaluates thresholds itself (for instance a backend
// whose threshold kernel writes one bit per neuron, the layout of the tick
// exchange between GPUs) gets the reference's `fired` list from it: neurons
// in ascending order (emit_threshold, brian2-rust/src/executor.rs:2949-3006).
// Bit b of word w is neuron 32*w + b.
//
// Two launches, no atomics, deterministic:
//   1. tile_popcounts: per tile of kWordsPerTile words, the number of set bits
//      -> tile_counts[tile] (scratch, fully overwritten: nothing to clear);
//   2. tile_write: each tile sums the counts of the tiles before it (a block
//      reduction; tiles are few), scans its words' popcounts and writes every
//      set bit at its global rank; the last tile writes the total.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>

#include "cuda_util.hpp"
#include "spikes.hpp"

namespace b2gpu {

namespace {

constexpr int kThreads = 256;
constexpr int kWordsPerThread = 4;
constexpr uint64_t kWordsPerTile = uint64_t(kThreads) * kWordsPerThread;

// Exclusive scan of one value per thread; *total gets the block sum.
__device__ __forceinline__ uint32_t block_scan(uint32_t v, uint32_t* total) {
  __shared__ uint32_t s_part[kThreads / 32 + 1];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, d);
    if (lane >= d) x += y;
  }
  if (lane == 31) s_part[warp] = x;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t acc = 0;
    for (int w = 0; w < kThreads / 32; ++w) {
      const uint32_t c = s_part[w];
      s_part[w] = acc;
      acc += c;
    }
    s_part[kThreads / 32] = acc;
  }
  __syncthreads();
  *total = s_part[kThreads / 32];
  const uint32_t r = s_part[warp] + x - v;
  __syncthreads();
  return r;
}

__device__ __forceinline__ uint32_t load_word(const uint32_t* bits, uint64_t w, uint64_t words, uint32_t last_mask) {
  if (w >= words) return 0u;
  const uint32_t v = bits[w];
  return w + 1 == words ? v & last_mask : v;
}

__global__ void __launch_bounds__(kThreads) tile_popcounts(const uint32_t* __restrict__ bits, uint64_t words,
                                                           uint32_t last_mask, uint32_t* __restrict__ tile_counts) {
  const uint64_t w0 = uint64_t(blockIdx.x) * kWordsPerTile + uint64_t(threadIdx.x) * kWordsPerThread;
  uint32_t c = 0;
#pragma unroll
  for (int k = 0; k < kWordsPerThread; ++k) c += __popc(load_word(bits, w0 + k, words, last_mask));
  uint32_t total;
  block_scan(c, &total);
  if (threadIdx.x == 0) tile_counts[blockIdx.x] = total;
}

__global__ void __launch_bounds__(kThreads) tile_write(const uint32_t* __restrict__ bits, uint64_t words,
                                                       uint32_t last_mask, const uint32_t* __restrict__ tile_counts,
                                                       uint32_t tiles, uint32_t* __restrict__ out,
                                                       uint32_t* __restrict__ count) {
  uint32_t part = 0;
  for (uint32_t t = threadIdx.x; t < blockIdx.x; t += kThreads) part += tile_counts[t];
  uint32_t base;
  block_scan(part, &base);
  const uint64_t w0 = uint64_t(blockIdx.x) * kWordsPerTile + uint64_t(threadIdx.x) * kWordsPerThread;
  uint32_t wv[kWordsPerThread];
  uint32_t c = 0;
#pragma unroll
  for (int k = 0; k < kWordsPerThread; ++k) {
    wv[k] = load_word(bits, w0 + k, words, last_mask);
    c += __popc(wv[k]);
  }
  uint32_t tile_total;
  uint32_t pos = base + block_scan(c, &tile_total);
#pragma unroll
  for (int k = 0; k < kWordsPerThread; ++k)
    for (uint32_t x = wv[k]; x; x &= x - 1u) out[pos++] = uint32_t((w0 + k) * 32u + uint32_t(__ffs(x) - 1));
  if (blockIdx.x == tiles - 1 && threadIdx.x == 0) *count = base + tile_total;
}

}  // namespace

uint64_t bitmap_tiles(uint64_t nbits) {
  const uint64_t words = (nbits + 31) / 32;
  return (words + kWordsPerTile - 1) / kWordsPerTile;
}

void bitmap_to_spikes(const uint32_t* d_bits, uint64_t nbits, uint32_t* d_out, uint32_t* d_count,
                      uint32_t* d_tile_counts, cudaStream_t stream) {
  b2ir::check(nbits <= (uint64_t(1) << 32), "bitmap larger than 2^32 neurons");
  const uint64_t words = (nbits + 31) / 32;
  const uint64_t tiles = bitmap_tiles(nbits);
  if (tiles == 0) {
    B2_CUDA(cudaMemsetAsync(d_count, 0, sizeof(uint32_t), stream));
    return;
  }
  const uint32_t tail = uint32_t(nbits % 32);
  const uint32_t last_mask = tail ? (1u << tail) - 1u : 0xffffffffu;  // bits past nbits are ignored
  tile_popcounts<<<unsigned(tiles), kThreads, 0, stream>>>(d_bits, words, last_mask, d_tile_counts);
  B2_CUDA(cudaGetLastError());
  tile_write<<<unsigned(tiles), kThreads, 0, stream>>>(d_bits, words, last_mask, d_tile_counts, uint32_t(tiles),
                                                       d_out, d_count);
  B2_CUDA(cudaGetLastError());
}

// ---------------------------------------------------------------- no-alloc variant
// Callers that must not allocate device memory around the call -- a tick
// loop that may not stall on an allocator, a host framework whose own caching
// allocator holds the device's memory budget, a process that has already
// reserved all free device memory -- get the same two launches with the
// scratch in this file-scope array instead of a caller buffer.  Its size caps
// the bitmap at kNoAllocMaxBits (2^27 neurons -> 4096 tile counts, 16 KiB).
// The tile counts are fully overwritten by the first launch, so nothing has
// to start at zero.  The array exists once per device: two calls whose
// launches overlap on one GPU (different streams, or host threads) race on it.
static __device__ __align__(256) uint32_t
    g_noalloc_tile_counts[(kNoAllocMaxBits / 32 + kWordsPerTile - 1) / kWordsPerTile];
namespace {
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mutex;
// Per device ordinal: the array's device address and the unique id of the
// CUDA context it was looked up in.  A context that the host framework tore
// down and re-created (cudaDeviceReset, primary-context release) gets a new
// id, and the address is looked up again in the new context.
struct NoAllocSlot {
  unsigned long long context_id = 0;
  uint32_t* scratch = nullptr;
};
NoAllocSlot g_noalloc_slots[kNoAllocMaxDevices];

// Unique id of the calling thread's current CUDA context (cuCtxGetCurrent +
// cuCtxGetId, reached through the runtime's driver entry points, so the
// library still links no driver library); 0 when it cannot be read, which
// makes every call look the address up again.
unsigned long long current_context_id() {
  using GetCurrent = int (*)(void**);
  using GetId = int (*)(void*, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static bool resolved = false;
  if (!resolved) {
    resolved = true;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &fn, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrent>(fn);
    fn = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &fn, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(fn);
  }
  void* ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != 0 || !ctx || get_id(ctx, &id) != 0) return 0;
  return id;
}
}  // namespace

void bitmap_to_spikes_noalloc(const uint32_t* d_bits, uint64_t nbits, uint32_t* d_out, uint32_t* d_count,
                              cudaStream_t stream) {
  b2ir::check(nbits <= kNoAllocMaxBits,
              "bitmap of " + std::to_string(nbits) + " bits exceeds the no-alloc limit of " +
                  std::to_string(kNoAllocMaxBits) + " bits; use b2g_spikes_from_bitmap with a scratch buffer");
  // The launches go to the stream's device, with that device's copy of the
  // array: make it current for the call when it is not already.
  int current = -1, device = -1;
  B2_CUDA(cudaGetDevice(&current));
  B2_CUDA(cudaStreamGetDevice(stream, &device));
  b2ir::check(device >= 0 && device < kNoAllocMaxDevices, "device ordinal out of range for the no-alloc scratch");
  struct Restore {
    int device;
    bool active;
    ~Restore() {
      if (active) cudaSetDevice(device);
    }
  } restore{current, device != current};
  if (device != current) B2_CUDA(cudaSetDevice(device));
  uint32_t* scratch = nullptr;
  {
    // Set-up, once per device and context, with that device current: the
    // address of this device's copy of the array (the first call may load
    // the module, so it belongs before any stream capture).
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    NoAllocSlot& slot = g_noalloc_slots[device];
    const unsigned long long ctx = current_context_id();
    if (!slot.scratch || ctx == 0 || slot.context_id != ctx) {
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_tile_counts);
      b2ir::check(e == cudaSuccess && p, std::string("cudaGetSymbolAddress(no-alloc scratch): ") + cudaGetErrorString(e));
      slot.scratch = static_cast<uint32_t*>(p);
      // the lookup initialises the device's context if nothing had yet
      slot.context_id = ctx ? ctx : current_context_id();
    }
    scratch = slot.scratch;
  }
  bitmap_to_spikes(d_bits, nbits, d_out, d_count, scratch, stream);
}

}  // namespace b2gpu
