// Tensor-memory-accelerator (TMA) copies of [B, T, H, D] tiles for the tensor-core kernels.
//
// A chunk's rows t0..t0+63 of one head form a 64 x D box of a 4-D tensor map
// (dims D, H, T, B).  Rows past T read as zero and are dropped on store, so ragged tails need
// no special case.  All maps use the 128-byte swizzle: a bf16 box (64 columns) is the layout
// sw64() addresses, an fp32 box covers 32 columns and a 64-column fp32 tile takes two of them
// (the layout gsw() addresses); the shared-memory tiles start on 1024-byte boundaries.  No
// copy here multicasts.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "kda_common.cuh"

namespace kda {

struct alignas(64) TmaMaps {
  CUtensorMap m[8];
};

// Encodes the map of a [B, T, H, D] tensor (bf16 or fp32) with a box of 64 rows of one head
// and 128 bytes of columns (64 for bf16, 32 for fp32; x selects the first column).  `st` gives
// the element strides of b, t, h (nullptr: dense).  Returns 0 on success, a KDA_ERR_* code
// otherwise.
int tma_map_bthd(CUtensorMap *map, const void *base, int64_t B, int64_t T, int64_t H, int64_t D, bool fp32,
                 const Str *st = nullptr);

// x: first column of the box (a multiple of 64 for bf16, of 32 for fp32)
__device__ __forceinline__ void tma_load_rows(uint32_t dst, const CUtensorMap *map, int h, int t0, int b,
                                              uint32_t mbar, int x = 0) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];\n"
      :: "r"(dst), "l"(map), "r"(x), "r"(h), "r"(t0), "r"(b), "r"(mbar) : "memory");
}
__device__ __forceinline__ void tma_store_rows(const CUtensorMap *map, uint32_t src, int h, int t0, int b, int x = 0) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];\n"
               :: "l"(map), "r"(src), "r"(x), "r"(h), "r"(t0), "r"(b) : "memory");
}
// both halves of an fp32 64 x 64 tile
__device__ __forceinline__ void tma_load_rows_f32(uint32_t dst, const CUtensorMap *map, int h, int t0, int b,
                                                  uint32_t mbar) {
  tma_load_rows(dst, map, h, t0, b, mbar, 0);
  tma_load_rows(dst + 8192, map, h, t0, b, mbar, 32);
}
__device__ __forceinline__ void tma_store_rows_f32(const CUtensorMap *map, uint32_t src, int h, int t0, int b) {
  tma_store_rows(map, src, h, t0, b, 0);
  tma_store_rows(map, src + 8192, h, t0, b, 32);
}

}  // namespace kda
