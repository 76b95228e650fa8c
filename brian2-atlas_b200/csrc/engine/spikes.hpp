// Spike bitmap -> ascending spike index list (see spikes.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace b2gpu {

// Scratch words (u32 tile counts) bitmap_to_spikes needs for `nbits` bits.
uint64_t bitmap_tiles(uint64_t nbits);

// Ascending indices of the set bits among the first `nbits` bits of d_bits
// (bit b of word w is index 32*w + b; bits past nbits are ignored) into d_out
// (room for the popcount) and their number into *d_count, all on `stream`.
// d_tile_counts: bitmap_tiles(nbits) u32 of scratch, overwritten.
void bitmap_to_spikes(const uint32_t* d_bits, uint64_t nbits, uint32_t* d_out, uint32_t* d_count,
                      uint32_t* d_tile_counts, cudaStream_t stream);

// Same result without any device allocation: the scratch is a file-scope
// device array (see spikes.cu), so nbits <= kNoAllocMaxBits and calls that
// overlap on one GPU race on it.  The first call on a device looks the array
// up (and may load the module).
constexpr uint64_t kNoAllocMaxBits = uint64_t(1) << 27;
void bitmap_to_spikes_noalloc(const uint32_t* d_bits, uint64_t nbits, uint32_t* d_out, uint32_t* d_count,
                              cudaStream_t stream);

}  // namespace b2gpu
