// Device construction of procedural projections (see topology.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "engine.hpp"

namespace b2gpu {

// Source-major CSR of a fixed in-degree projection restricted to the targets
// [t_lo, t_hi): offsets[S+1] (u64) and row_targets[] (u32, global target
// indices in [t_lo, t_hi)), rows in ascending target order.
void build_fixed_indegree_csr(uint64_t S, uint64_t T, uint64_t K, uint64_t seed, uint64_t t_lo, uint64_t t_hi,
                              DeviceBuffer& offsets, DeviceBuffer& row_targets, uint64_t& local_edges,
                              cudaStream_t stream);

// Same for a fixed-total projection (edges sampled with replacement).
void build_fixed_total_csr(uint64_t S, uint64_t T, uint64_t E, uint64_t seed, uint64_t t_lo, uint64_t t_hi,
                           DeviceBuffer& offsets, DeviceBuffer& row_targets, uint64_t& local_edges,
                           cudaStream_t stream);

// Delays in ticks (u16 per edge, edge order) of a uniform delay initializer,
// and their smallest and largest value.
void delay_ticks_uniform_device(uint64_t n, uint64_t seed, uint64_t stream, double lo, double hi, double dt,
                                DeviceBuffer& ticks, uint64_t& min_ticks, uint64_t& max_ticks, cudaStream_t stream_);

// Row (source) index of every position of a source-major CSR with S rows and
// E entries (u32 per entry).
void csr_row_sources(const uint64_t* d_offsets, uint64_t S, uint64_t E, DeviceBuffer& src, cudaStream_t stream);

// Target-major view of a source-major CSR restricted to the targets
// [t_lo, t_lo + T): tm_offsets[T+1] (u64), and per entry the source index
// (u32), the edge index (row_edge[q], or the position q when row_edge is null)
// and, when row_delay is given, the delay (u16).  Within a target the entries
// run by delay descending (emission tick ascending), then in the source-major
// order: source ascending, then creation order.
void build_target_major(const uint64_t* d_offsets, const uint32_t* d_row_other, const uint32_t* d_row_edge,
                        const uint16_t* d_row_delay, uint64_t max_delay, uint64_t S, uint64_t E, uint64_t t_lo,
                        uint64_t T, DeviceBuffer& tm_offsets, DeviceBuffer& tm_src, DeviceBuffer& tm_edge,
                        DeviceBuffer& tm_delay, cudaStream_t stream);

// Uniform per-edge initializer (large_topology.rs:129-142) for edge ids
// edge_base .. edge_base+n-1.
void uniform_initializer_device(double* out, uint64_t n, uint64_t seed, uint64_t stream_id, double lo, double hi,
                                uint64_t edge_base, cudaStream_t stream);

}  // namespace b2gpu
