// Layout of one KV page (16 token slots, head_dim 128) in the pool.
//
// bf16 pages (8 KB) are stored PRE-SWIZZLED, in exactly the shared-memory
// layout the tensor-core kernels consume, so one contiguous bulk copy of a page
// (or of a 2 KB quarter) lands ready for ldmatrix / tcgen05 descriptors:
//
//   page = [half h: dims 64h..64h+63][kv: 0 = K, 1 = V][slot: 16][128 bytes]
//   the 16-byte chunk c (dims 64h + 8c .. +7) of a row sits at chunk c ^ (slot & 7)
//
// i.e. each 2 KB (half, kv) block is two 1 KB atoms of the 128-byte swizzle
// pattern (row r of an atom: chunk index XOR r).  f32 pages (16 KB) are plain
// row-major [kv][slot][dim].
#pragma once

#include <stdint.h>

namespace aoh {

constexpr int kPageBf16Bytes = 8192;
constexpr int kPageF32Bytes = 16384;
constexpr int kHalfBytes = 4096;   // one 64-dim half of K and V
constexpr int kBlockBytes = 2048;  // one (half, kv) block: 16 rows x 128 B

// Byte offset of the 16-byte chunk c8 (dims 8*c8 .. 8*c8+7) of row (kv, slot).
__host__ __device__ __forceinline__ int bf16_chunk_offset(int kv, int slot, int c8) {
  return (c8 >> 3) * kHalfBytes + kv * kBlockBytes + slot * 128 + (((c8 & 7) ^ (slot & 7)) << 4);
}

// Element offset (in bf16 elements) of dim d of row (kv, slot).
__host__ __device__ __forceinline__ int bf16_elem_offset(int kv, int slot, int d) {
  return (bf16_chunk_offset(kv, slot, d >> 3) >> 1) + (d & 7);
}

// Element offset (in floats) of dim d of row (kv, slot) in an f32 page.
__host__ __device__ __forceinline__ int f32_elem_offset(int kv, int slot, int d) {
  return (kv * 16 + slot) * 128 + d;
}

}  // namespace aoh
