// Tensor-memory-accelerator (TMA) copies of [B, T, H, D] tiles for the tensor-core kernels.
//
// A chunk's rows t0..t0+63 of one head form a 64 x D box of a 4-D tensor map
// (dims D, H, T, B).  Rows past T read as zero and are dropped on store, so ragged tails need
// no special case.  bf16 maps use the 128-byte swizzle, which is the layout sw64() addresses
// when the shared-memory tile starts on a 1024-byte boundary; fp32 maps (g, dg) are plain
// [t][d] rows of 256 bytes.  No copy here multicasts.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace kda {

struct alignas(64) TmaMaps {
  CUtensorMap m[8];
};

// Encodes the map of a [B, T, H, D] tensor (bf16 or fp32, D = 64) with a box of 64 rows of
// one head.  Returns 0 on success, a KDA_ERR_* code otherwise.
int tma_map_bthd(CUtensorMap *map, const void *base, int64_t B, int64_t T, int64_t H, int64_t D, bool fp32);

__device__ __forceinline__ void tma_load_rows(uint32_t dst, const CUtensorMap *map, int h, int t0, int b,
                                              uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];\n"
      :: "r"(dst), "l"(map), "r"(0), "r"(h), "r"(t0), "r"(b), "r"(mbar) : "memory");
}
__device__ __forceinline__ void tma_store_rows(const CUtensorMap *map, uint32_t src, int h, int t0, int b) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];\n"
               :: "l"(map), "r"(src), "r"(0), "r"(h), "r"(t0), "r"(b) : "memory");
}

}  // namespace kda
