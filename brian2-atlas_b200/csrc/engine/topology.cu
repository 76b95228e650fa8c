// Device construction of procedural projections (fixed in-degree and fixed
// total), producing the reference's source-major edge order directly in HBM.
//
// Semantics follow brian2-rust/src/large_topology.rs:
//   * fixed_indegree_sources (:189-208): per target, Floyd subset sampling over
//     candidates S-K .. S-1 with draw = bounded(seed, 0, target*S+candidate,
//     candidate+1), falling back to the candidate on a repeat;
//   * build_fixed_indegree_indices (:214-260): edges grouped by source, and
//     within a source in ascending target order (targets are visited in order);
//   * build_fixed_total_indices (:144-187): source = bounded(seed,0,e,S),
//     target = bounded(seed,1,e,T), grouped by source in edge order.
//
// B200 design: one warp per target resolves Floyd's picks 32 candidates at a
// time (draws are independent; only the repeat test is sequential, and it runs
// as a 32-step shuffle broadcast), then targets are processed in chunks whose
// (source, target) pairs are stably radix-sorted by source and scattered to
// their final CSR positions.  Chunks advance in target order, so each row stays
// in ascending target order without a global sort.
#include <cub/cub.cuh>

#include <algorithm>
#include <cstdint>
#include <vector>

#include "cuda_util.hpp"
#include "topology.hpp"

namespace b2gpu {

namespace {

__device__ __forceinline__ uint64_t topo_mix64(uint64_t v) {
  v += 0x9e3779b97f4a7c15ull;
  v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
  v = (v ^ (v >> 27)) * 0x94d049bb133111ebull;
  return v ^ (v >> 31);
}

__device__ __forceinline__ uint64_t topo_draw(uint64_t seed, uint64_t stream, uint64_t edge, uint64_t attempt) {
  return topo_mix64(seed ^ (stream * 0xd2b74407b1ce6e93ull) ^ (edge * 0x9e3779b97f4a7c15ull) ^
                    (attempt * 0xca5a826395121157ull));
}

__device__ __forceinline__ uint64_t topo_bounded(uint64_t seed, uint64_t stream, uint64_t edge, uint64_t upper) {
  return __umul64hi(topo_draw(seed, stream, edge, 0), upper);
}

__device__ __forceinline__ double topo_uniform_open(uint64_t seed, uint64_t stream, uint64_t edge, uint64_t attempt) {
  uint64_t mantissa = topo_draw(seed, stream, edge, attempt) >> 11;
  return ((double)mantissa + 0.5) * (1.0 / 9007199254740992.0);
}

constexpr int kWarpsPerBlock = 4;
constexpr uint32_t kMaxIndegree = 2048;  // picks held in shared memory per warp (32 KB per block)

// Floyd picks for targets [t_begin, t_end).  mode 0: count picks per source
// (counts[source]++); mode 1: also emit (source, target) pairs at
// (t - t_begin) * K + j.
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
fixed_indegree_kernel(uint64_t S, uint64_t K, uint64_t seed, uint64_t t_begin, uint64_t t_end,
                      uint32_t* __restrict__ counts, uint32_t* __restrict__ keys,
                      uint32_t* __restrict__ vals, int emit) {
  __shared__ uint32_t picks[kWarpsPerBlock][kMaxIndegree];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t warps_total = (uint64_t)gridDim.x * kWarpsPerBlock;
  for (uint64_t t = t_begin + (uint64_t)blockIdx.x * kWarpsPerBlock + warp; t < t_end; t += warps_total) {
    uint32_t* sel = picks[warp];
    for (uint64_t c0 = 0; c0 < K; c0 += 32) {
      const uint64_t j = c0 + lane;
      const bool valid = j < K;
      const uint64_t candidate = S - K + j;
      uint32_t draw = valid ? (uint32_t)topo_bounded(seed, 0, t * S + candidate, candidate + 1) : 0xffffffffu;
      bool hit = false;
      for (uint64_t x = 0; x < c0; ++x) hit |= (sel[x] == draw);
      // Resolve this chunk in candidate order: a lane's pick is visible to
      // every later lane before that lane decides.
      uint32_t pick = 0;
      for (int L = 0; L < 32; ++L) {
        uint32_t mine = hit ? (uint32_t)candidate : draw;
        uint32_t pL = __shfl_sync(0xffffffffu, mine, L);
        if (lane == L) pick = mine;
        if (lane > L && draw == pL) hit = true;
      }
      if (valid) {
        sel[j] = pick;
        if (emit) {
          uint64_t out = (t - t_begin) * K + j;
          keys[out] = pick;
          vals[out] = (uint32_t)t;
        }
        atomicAdd(&counts[pick], 1u);
      }
      __syncwarp();
    }
  }
}

// Fixed-total pairs for edges [e_begin, e_end) whose target lies in
// [t_lo, t_hi).  Counts always; emits compacted pairs in edge order when
// `emit` (positions from a per-block exclusive scan done by the caller's
// second pass: here we emit into dense slots e - e_begin and mark misses).
__global__ void fixed_total_kernel(uint64_t S, uint64_t T, uint64_t seed, uint64_t e_begin, uint64_t e_end,
                                   uint64_t t_lo, uint64_t t_hi, uint32_t* __restrict__ counts,
                                   uint32_t* __restrict__ keys, uint32_t* __restrict__ vals, int emit) {
  for (uint64_t e = e_begin + blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < e_end;
       e += (uint64_t)gridDim.x * blockDim.x) {
    uint32_t s = (uint32_t)topo_bounded(seed, 0, e, S);
    uint32_t t = (uint32_t)topo_bounded(seed, 1, e, T);
    bool local = t >= t_lo && t < t_hi;
    if (local) atomicAdd(&counts[s], 1u);
    if (emit) {
      keys[e - e_begin] = local ? s : 0xffffffffu;  // misses sort to the end
      vals[e - e_begin] = t;
    }
  }
}

__global__ void counts_to_u64(const uint32_t* __restrict__ in, uint64_t* __restrict__ out, uint64_t n) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = in[i];
}

// Scatter a source-sorted chunk to final CSR positions.
__global__ void scatter_chunk(const uint32_t* __restrict__ keys, const uint32_t* __restrict__ vals, uint64_t n,
                              const uint64_t* __restrict__ offsets, const uint64_t* __restrict__ cursor,
                              const uint64_t* __restrict__ chunk_start, uint32_t* __restrict__ row_targets) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    uint32_t s = keys[i];
    if (s == 0xffffffffu) continue;
    uint64_t pos = offsets[s] + cursor[s] + (i - chunk_start[s]);
    row_targets[pos] = vals[i];
  }
}

__global__ void advance_cursor(uint64_t* __restrict__ cursor, const uint32_t* __restrict__ chunk_counts, uint64_t S) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < S; i += (uint64_t)gridDim.x * blockDim.x)
    cursor[i] += chunk_counts[i];
}

__global__ void uniform_initializer(double* __restrict__ out, uint64_t n, uint64_t seed, uint64_t stream,
                                    double lo, double hi, uint64_t edge_base) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = lo + (hi - lo) * topo_uniform_open(seed, stream, edge_base + i, 0);
}

// Per-edge delay in ticks from a uniform delay initializer
// (materialize_delay_initializer, brian2-rust/src/executor.rs:160-188, and the
// tick rounding of its caller): d = lo + (hi - lo) * u, ticks = floor(d/dt +
// 0.5); bounds[0] / bounds[1] collect the smallest / largest tick count,
// bounds[2] is set when a delay is negative or does not fit 16 bits.
__global__ void delay_ticks_uniform(uint16_t* __restrict__ out, uint64_t n, uint64_t seed, uint64_t stream,
                                    double lo, double hi, double dt, unsigned int* __restrict__ bounds) {
  unsigned int mn = 0xffffffffu, mx = 0, bad = 0;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const double d = lo + (hi - lo) * topo_uniform_open(seed, stream, i, 0);
    const double t = floor(d / dt + 0.5);
    unsigned int k = 0;
    if (!(t >= 0.0 && t < 65535.0)) bad = 1;
    else k = (unsigned int)t;
    out[i] = (uint16_t)k;
    mn = min(mn, k);
    mx = max(mx, k);
  }
  atomicMin(bounds, mn);
  atomicMax(bounds + 1, mx);
  if (bad) atomicOr(bounds + 2, 1u);
}

int bits_for(uint64_t n) {
  int b = 1;
  while ((1ull << b) < n) ++b;
  return b;
}

unsigned grid_for(uint64_t n, unsigned block, unsigned cap = 148u * 64u) {
  uint64_t g = (n + block - 1) / block;
  return (unsigned)std::max<uint64_t>(1, std::min<uint64_t>(g, cap));
}

// Shared second phase: given per-source counts over the whole local edge set,
// build offsets, then per chunk regenerate, sort stably by source and scatter.
template <class Gen>
void build_csr(uint64_t S, uint64_t chunk_items, uint64_t chunks, Gen gen, DeviceBuffer& offsets,
               DeviceBuffer& row_targets, uint64_t& local_edges, cudaStream_t stream) {
  DeviceBuffer counts(S * sizeof(uint32_t));
  B2_CUDA(cudaMemsetAsync(counts.ptr, 0, counts.bytes, stream));
  for (uint64_t c = 0; c < chunks; ++c) gen(c, counts.as<uint32_t>(), nullptr, nullptr, 0);
  DeviceBuffer counts64(S * sizeof(uint64_t));
  counts_to_u64<<<grid_for(S, 256), 256, 0, stream>>>(counts.as<uint32_t>(), counts64.as<uint64_t>(), S);
  offsets = DeviceBuffer((S + 1) * sizeof(uint64_t));
  B2_CUDA(cudaMemsetAsync(offsets.ptr, 0, sizeof(uint64_t), stream));
  size_t temp_bytes = 0;
  cub::DeviceScan::InclusiveSum(nullptr, temp_bytes, counts64.as<uint64_t>(), offsets.as<uint64_t>() + 1, (int64_t)S, stream);
  {
    DeviceBuffer temp(std::max<size_t>(temp_bytes, 16));
    cub::DeviceScan::InclusiveSum(temp.ptr, temp_bytes, counts64.as<uint64_t>(), offsets.as<uint64_t>() + 1, (int64_t)S, stream);
  }
  B2_CUDA(cudaMemcpyAsync(&local_edges, offsets.as<uint64_t>() + S, sizeof(uint64_t), cudaMemcpyDeviceToHost, stream));
  B2_CUDA(cudaStreamSynchronize(stream));
  row_targets = DeviceBuffer(std::max<uint64_t>(local_edges, 1) * sizeof(uint32_t));
  if (local_edges == 0) return;

  DeviceBuffer keys(chunk_items * 4), vals(chunk_items * 4), keys2(chunk_items * 4), vals2(chunk_items * 4);
  DeviceBuffer cursor(S * 8), chunk_start(S * 8);
  B2_CUDA(cudaMemsetAsync(cursor.ptr, 0, cursor.bytes, stream));
  const int end_bit = bits_for(S + 1);  // 0xffffffff misses must sort last
  size_t sort_bytes = 0, scan_bytes = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, sort_bytes, keys.as<uint32_t>(), keys2.as<uint32_t>(),
                                  vals.as<uint32_t>(), vals2.as<uint32_t>(), (int64_t)chunk_items, 0, 32, stream);
  cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, counts64.as<uint64_t>(), chunk_start.as<uint64_t>(), (int64_t)S, stream);
  DeviceBuffer sort_temp(std::max<size_t>(sort_bytes, 16)), scan_temp(std::max<size_t>(scan_bytes, 16));
  (void)end_bit;
  for (uint64_t c = 0; c < chunks; ++c) {
    B2_CUDA(cudaMemsetAsync(counts.ptr, 0, counts.bytes, stream));
    uint64_t n = gen(c, counts.as<uint32_t>(), keys.as<uint32_t>(), vals.as<uint32_t>(), 1);
    if (n == 0) continue;
    size_t sb = sort_bytes;
    B2_CUDA(cub::DeviceRadixSort::SortPairs(sort_temp.ptr, sb, keys.as<uint32_t>(), keys2.as<uint32_t>(),
                                            vals.as<uint32_t>(), vals2.as<uint32_t>(), (int64_t)n, 0, 32, stream));
    counts_to_u64<<<grid_for(S, 256), 256, 0, stream>>>(counts.as<uint32_t>(), counts64.as<uint64_t>(), S);
    size_t cb = scan_bytes;
    B2_CUDA(cub::DeviceScan::ExclusiveSum(scan_temp.ptr, cb, counts64.as<uint64_t>(), chunk_start.as<uint64_t>(), (int64_t)S, stream));
    scatter_chunk<<<grid_for(n, 256), 256, 0, stream>>>(keys2.as<uint32_t>(), vals2.as<uint32_t>(), n,
                                                         offsets.as<uint64_t>(), cursor.as<uint64_t>(),
                                                         chunk_start.as<uint64_t>(), row_targets.as<uint32_t>());
    advance_cursor<<<grid_for(S, 256), 256, 0, stream>>>(cursor.as<uint64_t>(), counts.as<uint32_t>(), S);
    B2_CUDA(cudaGetLastError());
  }
  B2_CUDA(cudaStreamSynchronize(stream));
}

}  // namespace

void build_fixed_indegree_csr(uint64_t S, uint64_t T, uint64_t K, uint64_t seed, uint64_t t_lo, uint64_t t_hi,
                              DeviceBuffer& offsets, DeviceBuffer& row_targets, uint64_t& local_edges,
                              cudaStream_t stream) {
  b2ir::check(S > 0 && T > 0 && K > 0 && K <= S && T * K <= UINT32_MAX,
              "invalid fixed-indegree topology specification");
  b2ir::check(K <= kMaxIndegree, "fixed in-degree above 2048 is not supported by the device generator");
  b2ir::check(S < 0xffffffffull, "fixed-indegree source count must fit u32");
  const uint64_t targets = t_hi - t_lo;
  const uint64_t per_chunk = std::max<uint64_t>(1, std::min<uint64_t>(targets, (1ull << 27) / K));
  const uint64_t chunks = (targets + per_chunk - 1) / per_chunk;
  auto gen = [&](uint64_t c, uint32_t* counts, uint32_t* keys, uint32_t* vals, int emit) -> uint64_t {
    uint64_t b = t_lo + c * per_chunk, e = std::min(t_hi, b + per_chunk);
    unsigned grid = (unsigned)std::max<uint64_t>(1, std::min<uint64_t>((e - b + kWarpsPerBlock - 1) / kWarpsPerBlock, 148ull * 16));
    fixed_indegree_kernel<<<grid, kWarpsPerBlock * 32, 0, stream>>>(S, K, seed, b, e, counts, keys, vals, emit);
    B2_CUDA(cudaGetLastError());
    return (e - b) * K;
  };
  build_csr(S, per_chunk * K, chunks, gen, offsets, row_targets, local_edges, stream);
}

void build_fixed_total_csr(uint64_t S, uint64_t T, uint64_t E, uint64_t seed, uint64_t t_lo, uint64_t t_hi,
                           DeviceBuffer& offsets, DeviceBuffer& row_targets, uint64_t& local_edges,
                           cudaStream_t stream) {
  b2ir::check(S > 0 && T > 0 && E > 0 && E <= UINT32_MAX, "invalid fixed-total topology specification");
  const uint64_t per_chunk = std::min<uint64_t>(E, 1ull << 27);
  const uint64_t chunks = (E + per_chunk - 1) / per_chunk;
  auto gen = [&](uint64_t c, uint32_t* counts, uint32_t* keys, uint32_t* vals, int emit) -> uint64_t {
    uint64_t b = c * per_chunk, e = std::min(E, b + per_chunk);
    fixed_total_kernel<<<grid_for(e - b, 256), 256, 0, stream>>>(S, T, seed, b, e, t_lo, t_hi, counts, keys, vals, emit);
    B2_CUDA(cudaGetLastError());
    return e - b;
  };
  build_csr(S, per_chunk, chunks, gen, offsets, row_targets, local_edges, stream);
}

namespace {

// source of every source-major position (one warp per source row)
__global__ void row_sources(const uint64_t* __restrict__ offsets, uint64_t S, uint32_t* __restrict__ src) {
  const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x / 32);
  for (uint64_t s = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) / 32; s < S; s += warps)
    for (uint64_t q = offsets[s] + (threadIdx.x & 31); q < offsets[s + 1]; q += 32) src[q] = (uint32_t)s;
}

// keys = (target - t_lo) * (D + 1) + (D - delay), values = position (edges
// of non-owned targets never occur)
__global__ void target_keys(const uint32_t* __restrict__ row_other, const uint16_t* __restrict__ row_delay,
                            uint64_t E, uint32_t t_lo, uint64_t D, uint64_t* __restrict__ keys,
                            uint32_t* __restrict__ pos) {
  for (uint64_t q = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; q < E; q += (uint64_t)gridDim.x * blockDim.x) {
    keys[q] = (uint64_t)(row_other[q] - t_lo) * (D + 1) + (row_delay ? D - row_delay[q] : 0);
    pos[q] = (uint32_t)q;
  }
}

// tm_off[j] = first sorted position whose key belongs to target >= j
__global__ void target_offsets(const uint64_t* __restrict__ keys, uint64_t E, uint64_t T, uint64_t D,
                               uint64_t* __restrict__ off) {
  for (uint64_t j = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; j <= T; j += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t first = j * (D + 1);
    uint64_t lo = 0, hi = E;
    while (lo < hi) {
      const uint64_t mid = (lo + hi) / 2;
      if (keys[mid] < first) lo = mid + 1;
      else hi = mid;
    }
    off[j] = lo;
  }
}

__global__ void gather_target_major(const uint32_t* __restrict__ pos, uint64_t E, const uint32_t* __restrict__ src_of,
                                    const uint32_t* __restrict__ row_edge, const uint16_t* __restrict__ row_delay,
                                    uint32_t* __restrict__ tm_src, uint32_t* __restrict__ tm_edge,
                                    uint16_t* __restrict__ tm_delay) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < E; k += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t q = pos[k];
    tm_src[k] = src_of[q];
    tm_edge[k] = row_edge ? row_edge[q] : q;
    if (tm_delay) tm_delay[k] = row_delay[q];
  }
}

}  // namespace

void delay_ticks_uniform_device(uint64_t n, uint64_t seed, uint64_t stream, double lo, double hi, double dt,
                                DeviceBuffer& ticks, uint64_t& min_ticks, uint64_t& max_ticks, cudaStream_t stream_) {
  ticks = DeviceBuffer(std::max<uint64_t>(n, 1) * 2);
  DeviceBuffer bounds(16);
  const unsigned int init[4] = {0xffffffffu, 0u, 0u, 0u};
  B2_CUDA(cudaMemcpyAsync(bounds.ptr, init, sizeof init, cudaMemcpyHostToDevice, stream_));
  if (n) delay_ticks_uniform<<<grid_for(n, 256), 256, 0, stream_>>>(ticks.as<uint16_t>(), n, seed, stream, lo, hi, dt,
                                                                   bounds.as<unsigned int>());
  B2_CUDA(cudaGetLastError());
  unsigned int host[4];
  B2_CUDA(cudaMemcpyAsync(host, bounds.ptr, sizeof host, cudaMemcpyDeviceToHost, stream_));
  B2_CUDA(cudaStreamSynchronize(stream_));
  b2ir::check(host[2] == 0, "procedural delay outside 0 to 65534 ticks");
  min_ticks = n ? host[0] : 0;
  max_ticks = host[1];
}

void csr_row_sources(const uint64_t* d_offsets, uint64_t S, uint64_t E, DeviceBuffer& src, cudaStream_t stream) {
  b2ir::check(E <= UINT32_MAX && S <= UINT32_MAX, "row sources need u32 indices");
  src = DeviceBuffer(std::max<uint64_t>(E, 1) * 4);
  if (E == 0) return;
  row_sources<<<grid_for(S * 32, 256), 256, 0, stream>>>(d_offsets, S, src.as<uint32_t>());
  B2_CUDA(cudaGetLastError());
  B2_CUDA(cudaStreamSynchronize(stream));
}

void build_target_major(const uint64_t* d_offsets, const uint32_t* d_row_other, const uint32_t* d_row_edge,
                        const uint16_t* d_row_delay, uint64_t max_delay, uint64_t S, uint64_t E, uint64_t t_lo,
                        uint64_t T, DeviceBuffer& tm_offsets, DeviceBuffer& tm_src, DeviceBuffer& tm_edge,
                        DeviceBuffer& tm_delay, cudaStream_t stream) {
  b2ir::check(E <= UINT32_MAX && T < UINT32_MAX, "target-major view needs u32 edge and target indices");
  const uint64_t D = d_row_delay ? max_delay : 0;
  tm_offsets = DeviceBuffer((T + 1) * sizeof(uint64_t));
  tm_src = DeviceBuffer(std::max<uint64_t>(E, 1) * 4);
  tm_edge = DeviceBuffer(std::max<uint64_t>(E, 1) * 4);
  if (d_row_delay) tm_delay = DeviceBuffer(std::max<uint64_t>(E, 1) * 2);
  if (E == 0) {
    B2_CUDA(cudaMemsetAsync(tm_offsets.ptr, 0, tm_offsets.bytes, stream));
    return;
  }
  DeviceBuffer src_of(E * 4), keys(E * 8), pos(E * 4), keys2(E * 8), pos2(E * 4);
  row_sources<<<grid_for(S * 32, 256), 256, 0, stream>>>(d_offsets, S, src_of.as<uint32_t>());
  target_keys<<<grid_for(E, 256), 256, 0, stream>>>(d_row_other, d_row_delay, E, (uint32_t)t_lo, D,
                                                     keys.as<uint64_t>(), pos.as<uint32_t>());
  B2_CUDA(cudaGetLastError());
  // LSD radix sort is stable: within a target and delay, edges keep the
  // source-major order, i.e. source ascending, then creation order
  size_t temp_bytes = 0;
  const int end_bit = bits_for(T * (D + 1) + 1);
  cub::DeviceRadixSort::SortPairs(nullptr, temp_bytes, keys.as<uint64_t>(), keys2.as<uint64_t>(), pos.as<uint32_t>(),
                                  pos2.as<uint32_t>(), (int64_t)E, 0, end_bit, stream);
  {
    DeviceBuffer temp(std::max<size_t>(temp_bytes, 16));
    B2_CUDA(cub::DeviceRadixSort::SortPairs(temp.ptr, temp_bytes, keys.as<uint64_t>(), keys2.as<uint64_t>(),
                                            pos.as<uint32_t>(), pos2.as<uint32_t>(), (int64_t)E, 0, end_bit, stream));
  }
  target_offsets<<<grid_for(T + 1, 256), 256, 0, stream>>>(keys2.as<uint64_t>(), E, T, D, tm_offsets.as<uint64_t>());
  gather_target_major<<<grid_for(E, 256), 256, 0, stream>>>(pos2.as<uint32_t>(), E, src_of.as<uint32_t>(), d_row_edge,
                                                            d_row_delay, tm_src.as<uint32_t>(), tm_edge.as<uint32_t>(),
                                                            d_row_delay ? tm_delay.as<uint16_t>() : nullptr);
  B2_CUDA(cudaGetLastError());
  B2_CUDA(cudaStreamSynchronize(stream));
}

void uniform_initializer_device(double* out, uint64_t n, uint64_t seed, uint64_t stream_id, double lo, double hi,
                                uint64_t edge_base, cudaStream_t stream) {
  if (n == 0) return;
  uniform_initializer<<<grid_for(n, 256), 256, 0, stream>>>(out, n, seed, stream_id, lo, hi, edge_base);
  B2_CUDA(cudaGetLastError());
}

}  // namespace b2gpu
