// Warp-level tensor-core and shared-memory helpers for the KDA tensor-core kernels.
//
// Tiles of 64 bf16 columns (128-byte rows) live in shared memory with the 128-byte XOR
// swizzle: 16-byte chunk c of row r is stored at chunk (c ^ (r & 7)).  That keeps ldmatrix /
// stmatrix conflict-free and is the same layout tcgen05 descriptors call SWIZZLE_128B.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace kda {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// byte offset of element (row, col) in a 64-column swizzled bf16 tile
__device__ __forceinline__ uint32_t sw64(int row, int col) {
  return (uint32_t)(row * 128 + ((((col >> 3) ^ row) & 7) << 4) + ((col & 7) << 1));
}

// float index of element (row t, column d) of a 64 x 64 fp32 tile kept as two 64 x 32 halves,
// each with the 128-byte swizzle (two TMA boxes of 32 columns): 8 consecutive rows of one
// column pair fall in 8 different bank groups
__device__ __forceinline__ int gsw(int t, int d) {
  return ((d >> 5) << 11) + t * 32 + ((((d >> 2) & 7) ^ (t & 7)) << 2) + (d & 3);
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}
__device__ __forceinline__ float2 unpack_bf16(uint32_t u) {
  __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162 *>(&u);
  return __bfloat1622float2(v);
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t (&r)[2]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t (&r)[2]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}
__device__ __forceinline__ void stsm_x4(uint32_t addr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1,%2,%3,%4};\n"
               :: "r"(addr), "r"(r0), "r"(r1), "r"(r2), "r"(r3));
}
__device__ __forceinline__ void stsm_x4_t(uint32_t addr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1,%2,%3,%4};\n"
               :: "r"(addr), "r"(r0), "r"(r1), "r"(r2), "r"(r3));
}

// D += A(16x16, row) * B(16x8, col), bf16 in, fp32 accumulate
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// D += A(16x8, row) * B(8x8, col), bf16 in, fp32 accumulate; A in two registers (rows g, g + 8),
// B in one (k = 2c, 2c + 1 of column g), with g = lane / 4, c = lane % 4
__device__ __forceinline__ void mma1688(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(b0));
}

// Lane address helpers for ldmatrix/stmatrix x4 on 64-column swizzled tiles.
//  A fragment of the 16x16 block at (r0, k0):
__device__ __forceinline__ uint32_t a_frag_addr(uint32_t base, int r0, int k0, int lane) {
  return base + sw64(r0 + (lane & 15), k0 + ((lane >> 4) << 3));
}
//  B fragments (two n8 tiles n0, n0+8; k16 at k0) from a tile stored [n][k] (non-trans):
__device__ __forceinline__ uint32_t bnk_frag_addr(uint32_t base, int n0, int k0, int lane) {
  return base + sw64(n0 + (lane & 7) + ((lane >> 4) << 3), k0 + (((lane >> 3) & 1) << 3));
}
//  B fragments from a tile stored [k][n] (use with ldsm_x4_t):
__device__ __forceinline__ uint32_t bkn_frag_addr(uint32_t base, int k0, int n0, int lane) {
  return base + sw64(k0 + (lane & 7) + (((lane >> 3) & 1) << 3), n0 + ((lane >> 4) << 3));
}
//  Transposed access of a tile stored [t][j] (with ldsm_x4_t / stsm_x4_t):
//   - C fragments (rows j0..j0+15, columns t0..t0+15) of X^T, registers ordered
//     (n-tile t0: c0c1, c2c3; n-tile t0+8: c0c1, c2c3);
//   - equally the A fragment of X^T for rows j0..j0+15 and k = t0..t0+15.
__device__ __forceinline__ uint32_t ct_frag_addr(uint32_t base, int t0, int j0, int lane) {
  return base + sw64(t0 + (lane & 7) + ((lane >> 4) << 3), j0 + (((lane >> 3) & 1) << 3));
}
// ldmatrix x2 on 64-column swizzled tiles (m16n8k8 operands):
//  - plain: the A fragment of the 16 x 8 block at (r0, k0) of a tile stored [m][k];
//  - with .trans, from rows r0..r0+7 and columns c0..c0+15 of a tile stored [k][x]: the A
//    fragment of its transpose (rows c0..c0+15, k = r0..r0+7), or the B fragments of the two n8
//    tiles c0 and c0 + 8 (k = r0..r0+7)
__device__ __forceinline__ uint32_t a8_frag_addr(uint32_t base, int r0, int k0, int lane) {
  return base + sw64(r0 + (lane & 15), k0);
}
__device__ __forceinline__ uint32_t t8_frag_addr(uint32_t base, int r0, int c0, int lane) {
  return base + sw64(r0 + (lane & 7), c0 + (((lane >> 3) & 1) << 3));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" :: "r"(dst), "l"(src), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }
// wait until at most N committed groups are still in flight
template <int N>
__device__ __forceinline__ void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;\n" :: "n"(N) : "memory"); }

// ---- bulk async copies (cp.async.bulk, no multicast) completed on an mbarrier ----
__device__ __forceinline__ void mbar_init(uint32_t mbar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" :: "r"(mbar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" :: "r"(mbar), "r"(bytes) : "memory");
}
// global -> shared, `bytes` a multiple of 16, both addresses 16-byte aligned
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t mbar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
               :: "r"(dst), "l"(src), "r"(bytes), "r"(mbar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t mbar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(mbar), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait for the mbarrier phase with the given parity.  Returns false (the caller
// records KDA_ERR_TIMEOUT and bails out) if it has not completed after kMbarSpinLimit polls,
// each of which already blocks for a hardware-chosen interval.
constexpr int kMbarSpinLimit = 1 << 22;
__device__ __forceinline__ bool mbar_wait(uint32_t mbar, uint32_t parity, int limit = kMbarSpinLimit) {
  for (int i = 0; i < limit; ++i)
    if (mbar_try_wait(mbar, parity)) return true;
  return false;
}

// The same bound for a wait on the latency-critical path: polls with the non-blocking test_wait, so
// the thread sees the phase complete without a suspended try_wait's wake-up delay.
__device__ __forceinline__ bool mbar_wait_spin(uint32_t mbar, uint32_t parity, int limit = kMbarSpinLimit) {
  for (int i = 0; i < limit; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok) : "r"(mbar), "r"(parity) : "memory");
    if (ok) return true;
  }
  return mbar_wait(mbar, parity, limit);
}

// shared -> global bulk copies (bulk-group completion)
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ void bulk_s2g(void *dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n"
               :: "l"(dst), "r"(src), "r"(bytes) : "memory");
}
// L2 cache policies for bulk copies: keep (a record that the next kernel reads back) or
// stream (data no kernel of this call reads again)
__device__ __forceinline__ uint64_t l2_policy_keep() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;\n" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint64_t l2_policy_stream() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void bulk_s2g_hint(void *dst, uint32_t src, uint32_t bytes, uint64_t pol) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group.L2::cache_hint [%0], [%1], %2, %3;\n"
               :: "l"(dst), "r"(src), "r"(bytes), "l"(pol) : "memory");
}
__device__ __forceinline__ void bulk_g2s_hint(uint32_t dst, const void *src, uint32_t bytes, uint32_t mbar, uint64_t pol) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;\n"
               :: "r"(dst), "l"(src), "r"(bytes), "r"(mbar), "l"(pol) : "memory");
}
// one arrival of this thread (release: its earlier shared-memory writes are visible to the thread
// that completes a wait on the phase)
__device__ __forceinline__ void mbar_arrive(uint32_t mbar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];\n" :: "r"(mbar) : "memory");
}
// wait until at most N of this thread's bulk store groups still read their shared-memory source
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;\n" :: "n"(N) : "memory");
}
// hint: bring `bytes` (a multiple of 16) at a 16-byte aligned global address into L2
__device__ __forceinline__ void prefetch_l2(const void *src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" :: "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }

__device__ __forceinline__ void bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;\n" :: "r"(id), "r"(n) : "memory");
}
// named barrier over n threads that also returns whether c held for all of them
__device__ __forceinline__ bool bar_and(int id, int n, bool c) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r) : "r"((uint32_t)c), "r"(id), "r"(n) : "memory");
  return r != 0;
}
__device__ __forceinline__ void bar_arrive(int id, int n) {
  asm volatile("bar.arrive %0, %1;\n" :: "r"(id), "r"(n) : "memory");
}

// Gate parameters staged once per CTA in shared memory (after the kernel's own layout, 16-byte
// aligned): dt_bias [H][64] then A_log [H].  Above kGateSmemMaxH heads they stay in global memory.
constexpr int kGateSmemMaxH = 64;
__host__ __device__ inline int gate_smem_bytes(int gated, int H) {
  return gated && H <= kGateSmemMaxH ? H * 65 * 4 : 0;
}
// Returns the dt_bias base (A_log follows at +H*64 when staged); the caller syncs the CTA.
template <typename P>
__device__ __forceinline__ const float *stage_gate_params(float *gs, const P &p, int tid, int nt,
                                                          const float **A_log) {
  if (!p.gated || p.H > kGateSmemMaxH) {
    *A_log = p.A_log;
    return p.dt_bias;
  }
  for (int i = tid; i < p.H * 65; i += nt) gs[i] = i < p.H * 64 ? p.dt_bias[i] : p.A_log[i - p.H * 64];
  *A_log = gs + p.H * 64;
  return gs;
}

// Fused decay gate: the bf16 tile of the gate pre-activation f (64 rows, 128-byte swizzle) at
// `raw` becomes g = -exp(A_log[h]) softplus(f + dt_bias[h, d]) in fp32 over `G` (gsw layout;
// `in_place`: the first half of G is `raw` itself).  Rows from `nvalid` on (past the sequence
// end) get g = 0.  With `sg` (the backward), {sigmoid(x), softplus(x)} of x = f + dt_bias go there
// as half2, row-major [t][d], for the gate's VJP.  Thread `tid` < 512 converts 8 elements; the
// caller synchronises the CTA after the call.
__device__ __forceinline__ void gate_to_g(const uint8_t *raw, float *G, const float *A_log,
                                          const float *dt_bias, int h, int nvalid, int tid,
                                          bool in_place, __half2 *sg = nullptr) {
  const int t = tid >> 3, c0 = (tid & 7) * 8;
  const uint4 u = *reinterpret_cast<const uint4 *>(raw + sw64(t, c0));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  const float A = __expf(A_log[h]);
  const float *db = dt_bias + h * 64 + c0;
  float g[8], sig[8];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = unpack_bf16(w[e]);
    const float x[2] = {f.x + db[2 * e], f.y + db[2 * e + 1]};
#pragma unroll
    for (int j = 0; j < 2; ++j) {  // softplus(x) = max(x, 0) + log(1 + e^-|x|), sigmoid from e^-|x|
      const float ex = __expf(-fabsf(x[j])), r = __fdividef(1.f, 1.f + ex);
      const float sp = __logf(1.f + ex) + fmaxf(x[j], 0.f);
      g[2 * e + j] = sp;
      sig[2 * e + j] = x[j] >= 0.f ? r : ex * r;
    }
  }
  if (sg) {
    uint32_t hw[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const __half2 v = __floats2half2_rn(sig[e], g[e]);
      hw[e] = *reinterpret_cast<const uint32_t *>(&v);
    }
    uint4 *dst = reinterpret_cast<uint4 *>(sg + t * 64 + c0);
    dst[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    dst[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) g[e] *= -A;
  if (t >= nvalid)  // rows past the sequence end carry no decay (their f is the TMA zero fill)
#pragma unroll
    for (int e = 0; e < 8; ++e) g[e] = 0.f;
  if (in_place) __syncthreads();  // every thread has read its f before G overwrites the tile
  *reinterpret_cast<float4 *>(G + gsw(t, c0)) = make_float4(g[0], g[1], g[2], g[3]);
  *reinterpret_cast<float4 *>(G + gsw(t, c0 + 4)) = make_float4(g[4], g[5], g[6], g[7]);
}

}  // namespace kda
