// Tensor-core KDA forward for head dim D = 128, chunk = 64, bf16 q/k/v: the streaming-inference
// configuration (long sequences carried across calls through the state, few heads per GPU).
// Forward only; a call that saves states for a backward takes the generic kernels.
//
//  kda_fwd128_chunks  one CTA per (b, h, chunk), all independent: every state-independent
//                     quantity of the chunk, written to the workspace as one record:
//                       [Qd; -W] (two K-halves of d), U (two halves of the value index j),
//                       P (zero above the diagonal), Kb^T, e^{gamma_C}
//  kda_fwd128_scan    one CTA per (b, h, value half j0 = 0 / 64): the state rows j of one half
//                     evolve independently of the other half.  Per chunk, two accumulators in
//                     TMEM (M = 128 rows, 64 columns each):
//                       MMA A:   D1  = [Qd; -W] S^T         (K = d, 128)
//                       Unew = U + rows 64-127 of D1 -> bf16 B operand
//                       MMA BO:  D1 += [P; .] Unew          rows 0-63 = O = Qd S^T + P Unew
//                       MMA BS:  DS  = e^{gamma_C} S^T (stored by the state warps) + Kb^T Unew
//                     The fp32 state slice S^T [128 d][64 j] stays in the registers of four warps.
//
// Chunk algebra as in the D = 64 kernels (the reference's chunkwise path, nope_gdn_mlx.py:549-613,
// 2318-2456): gamma = cumsum(g); A = beta * decayed K K^T (strict lower); P = decayed Q K^T
// (lower incl.); W = (I + A)^{-1} beta Kd, U = (I + A)^{-1} beta V with Kd = k e^gamma; Qd = q e^gamma,
// Kb = k e^{gamma_C - gamma}.  (I + A)^{-1} diag(beta) comes out of one block substitution on
// diag(beta), so W and U are one GEMM against [k e^gamma | v].
#include "kda_common.cuh"
#include "kda_mma.cuh"
#include "kda_tc05.cuh"
#include "kda_tma.cuh"

namespace kda {
namespace tcfwd128 {

// set to a KDA_ERR_* code by a bounded wait that gave up (read by kda_device_status)
static __device__ int g_fwd128_status;

constexpr int C = 64, D = 128;
constexpr float kSpanMax = 60.f;
// the block-pair factors e^{r_i - r_j} of a chunk that is not "big" stay above fp32's smallest
// normal (e^-87) only if gamma moves at most this much between the middle rows of the first and
// the last block; beyond it the factor would flush to zero while the decay it stands for
// (e^{gamma_t - gamma_s} for t, s close to the block boundary) is not negligible
constexpr float kMidGapMax = 80.f;

// byte offset of (row, col) in a 64 x 128 bf16 tile kept as two 64-column swizzled halves
__device__ __forceinline__ uint32_t sw128(int row, int col) { return ((col >> 6) << 13) + sw64(row, col & 63); }
// float index of (t, d) in a 64 x 128 fp32 tile kept as two 64-column gsw() halves
__device__ __forceinline__ int gsw128(int t, int d) { return ((d >> 6) << 12) + gsw(t, d & 63); }

// ---- the per-chunk record (bytes) ----
constexpr int R_A0 = 0;          // [Qd; -W] for d 0-63: Qd rows t (8 KB) then -W rows t (8 KB)
constexpr int R_A1 = 16384;      // the same for d 64-127
constexpr int R_U = 32768;       // U [t][j], j 0-63 then j 64-127 (8 KB each)
constexpr int R_P = 49152;       // P [t][s]
constexpr int R_KBT = 57344;     // Kb^T [d][t], 128 rows
constexpr int R_EG = 73728;      // e^{gamma_C}, 128 floats
constexpr int REC = R_EG + 512;  // 74240

__host__ __device__ inline size_t ws_bytes(int64_t nchunks) { return (size_t)nchunks * REC; }

// ---------------------------------------------------------------------------------------
// kda_fwd128_chunks
// ---------------------------------------------------------------------------------------
constexpr int NT1 = 512;
constexpr int OFF_QS = 0, OFF_KS = 16384, OFF_VS = 32768;  // raw tiles (TMA); QS becomes Qd
constexpr int OFF_GS = 49152;                              // g -> gamma, fp32 32 KB
constexpr int OFF_KD = 81920;                              // Kdec = k F, later U
constexpr int OFF_QD = 98304;                              // Qdec = q F, later -W
constexpr int OFF_KI = 114688;                             // Kinc of the 4 diagonal blocks, 4 KB each
constexpr int OFF_XK = 131072;                             // k e^gamma
constexpr int OFF_AB = 147456;                             // A off-diagonal blocks (bf16)
constexpr int OFF_AD = 155648;                             // A diagonal blocks (fp32, 4 x 16 x 16)
constexpr int OFF_TI = 159744;                             // (I + A_ii)^{-1} (bf16, 4 x 16 x 16)
constexpr int OFF_TF = 161792;                             // (I + A)^{-1} diag(beta) (bf16)
constexpr int OFF_RS = 169984;                             // per-warp 16 x 8 staging of the solve
constexpr int OFF_PR = 174080;                             // P (bf16)
constexpr int OFF_KBT = 182272;                            // Kb^T (bf16, 128 rows)
constexpr int OFF_VEC = 198656;
// vectors (floats): bet[64] refs[4][128] erb[4][128] egr[4][128] gij[6][128] eG[128] part[4][128] flag[4]
constexpr int V_BET = 0, V_REFS = 64, V_ERB = 576, V_EGR = 1088, V_G = 1600, V_EG = 2368, V_PART = 2496,
              V_FLAG = 3008;
constexpr int OFF_MBAR1 = OFF_VEC + (V_FLAG + 4) * 4;
constexpr int SMEM1 = OFF_MBAR1 + 8;

// gij slot of the block pair (i, j < i)
__device__ __forceinline__ int pair_index(int i, int j) { return i * (i - 1) / 2 + j; }

// Block forward substitution Y = (I + A)^{-1} diag(beta) for the 8 columns n0..n0+7, one warp:
//   Y_i = T_ii (X_i - sum_{j<i} A_ij Y_j), X = diag(beta), i = ib..3 (rows above ib are zero)
__device__ __forceinline__ void solve_columns128(uint8_t *sm, uint32_t s_base, const float *bet, int n0, int ib,
                                                 int warp, int lane) {
  const int g4 = lane >> 2, c4 = lane & 3, l15 = lane & 15;
  const uint32_t Yb = s_base + OFF_TF;
  uint8_t *Ym = sm + OFF_TF;
  const uint32_t Rs = s_base + OFF_RS + warp * 256;
  uint8_t *Rm = sm + OFF_RS + warp * 256;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (i < ib) continue;
    float acc[4] = {};
#pragma unroll
    for (int j = 0; j < i; ++j) {
      if (j < ib) continue;
      uint32_t af[4], bf[2];
      ldsm_x4(a_frag_addr(s_base + OFF_AB, 16 * i, 16 * j, lane), af);
      ldsm_x2_t(Yb + sw64(16 * j + (l15 & 7) + ((l15 >> 3) << 3), n0), bf);
      mma16816(acc, af, bf[0], bf[1]);
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int tl = g4 + 8 * hh, t = 16 * i + tl, col = n0 + 2 * c4;
      const float x0 = t == col ? bet[col] : 0.f, x1 = t == col + 1 ? bet[col + 1] : 0.f;
      *reinterpret_cast<uint32_t *>(Rm + tl * 16 + c4 * 4) = pack_bf16(x0 - acc[2 * hh], x1 - acc[2 * hh + 1]);
    }
    __syncwarp();
    uint32_t af[4], bf[2];
    ldsm_x4(s_base + OFF_TI + i * 512 + (lane & 15) * 32 + (lane >> 4) * 16, af);
    ldsm_x2_t(Rs + ((l15 & 7) + ((l15 >> 3) << 3)) * 16, bf);
    float y[4] = {};
    mma16816(y, af, bf[0], bf[1]);
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int t = 16 * i + g4 + 8 * hh, col = n0 + 2 * c4;
      *reinterpret_cast<uint32_t *>(Ym + sw64(t, col)) = pack_bf16(y[2 * hh], y[2 * hh + 1]);
    }
    __syncwarp();
  }
}

template <typename Tb>
__global__ void __launch_bounds__(NT1, 1) kda_fwd128_chunks_kernel(Params p, const __grid_constant__ TmaMaps tm) {
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g4 = lane >> 2, c4 = lane & 3;
  const int idx = blockIdx.x, nc = p.nc, T = p.T, H = p.H;
  const int bh = idx / nc, c = idx % nc, b = bh / H, h = bh % H, t0 = c * C;
  const uint32_t s_base = smem_u32(sm);
  if (s_base & 1023) {  // TMA tiles with the 128-byte swizzle need a 1024-byte aligned base
    if (tid == 0) atomicExch(&g_fwd128_status, KDA_ERR_MISALIGNED);
    return;
  }
  float *GS = reinterpret_cast<float *>(sm + OFF_GS);
  float *AD = reinterpret_cast<float *>(sm + OFF_AD);
  float *vec = reinterpret_cast<float *>(sm + OFF_VEC);
  float *bet = vec + V_BET, *refs = vec + V_REFS, *erb = vec + V_ERB, *egr = vec + V_EGR, *gij = vec + V_G;
  float *eG = vec + V_EG, *part = vec + V_PART;
  int *flag = reinterpret_cast<int *>(vec + V_FLAG);
  const uint32_t mbar = s_base + OFF_MBAR1;

  if (tid == 0) {
    mbar_init(mbar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (tid == 0) {
    mbar_expect_tx(mbar, 3 * 16384 + 32768);
#pragma unroll
    for (int x = 0; x < 2; ++x) {
      tma_load_rows(s_base + OFF_QS + 8192 * x, &tm.m[0], h, t0, b, mbar, 64 * x);
      tma_load_rows(s_base + OFF_KS + 8192 * x, &tm.m[1], h, t0, b, mbar, 64 * x);
      tma_load_rows(s_base + OFF_VS + 8192 * x, &tm.m[2], h, t0, b, mbar, 64 * x);
    }
#pragma unroll
    for (int x = 0; x < 4; ++x) tma_load_rows(s_base + OFF_GS + 8192 * x, &tm.m[3], h, t0, b, mbar, 32 * x);
  }
  if (tid < C) {
    const Tb *betag = (const Tb *)p.beta;
    bet[tid] = t0 + tid < T ? to_f(betag[at(p.sb, b, t0 + tid, h)]) : 0.f;
  }
  if (__syncthreads_or(!mbar_wait(mbar, 0))) {
    if (tid == 0) {
      atomicExch(&g_fwd128_status, KDA_ERR_TIMEOUT);
      mbar_wait(mbar, 0);  // (bounded) the loads in flight land before the CTA exits
    }
    return;
  }

  // ---- gamma = cumsum(g): 4 segments of 16 rows per channel ----
  {
    const int d = tid & 127, seg = tid >> 7;
    float acc = 0.f;
#pragma unroll
    for (int r = 0; r < 16; ++r) acc += GS[gsw128(seg * 16 + r, d)];
    part[seg * 128 + d] = acc;
    __syncthreads();
    float off = 0.f;
    for (int s2 = 0; s2 < seg; ++s2) off += part[s2 * 128 + d];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      off += GS[gsw128(seg * 16 + r, d)];
      GS[gsw128(seg * 16 + r, d)] = off;
    }
  }
  __syncthreads();
  // guard: the mid-block factoring keeps every factor within e^{kSpanMax} unless gamma moves
  // more than that across half a 16-row block.  Such a "big" chunk factors
  // e^{gamma_t - gamma_s} (t in block i > j, the block of s) as A_t G_ij B_s, every factor <= 1,
  // and computes its diagonal blocks exactly.
  if (tid < 128) {
    float span = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      span = fmaxf(span, GS[gsw128(i * 16, tid)] - GS[gsw128(i * 16 + 8, tid)]);
      span = fmaxf(span, GS[gsw128(i * 16 + 8, tid)] - GS[gsw128(i * 16 + 15, tid)]);
    }
    if (!(GS[gsw128(8, tid)] - GS[gsw128(56, tid)] <= kMidGapMax)) span = 2.f * kSpanMax;
    const int any = __any_sync(0xffffffffu, !(span <= kSpanMax));
    if (lane == 0) flag[warp] = any;
  }
  __syncthreads();
  const bool big = flag[0] | flag[1] | flag[2] | flag[3];
  {  // per-block vectors, thread (block i, channel d)
    const int d = tid & 127, i = tid >> 7, ro = big ? 0 : 8;
    const float gC = GS[gsw128(63, d)], ri = GS[gsw128(i * 16 + ro, d)];
    refs[i * 128 + d] = ri;
    erb[i * 128 + d] = __expf(ri);
    egr[i * 128 + d] = __expf(gC - ri);
    for (int j = 0; j < i; ++j) gij[pair_index(i, j) * 128 + d] = __expf(ri - GS[gsw128(j * 16 + (big ? 15 : 8), d)]);
    if (i == 0) eG[d] = __expf(gC);
  }
  __syncthreads();

  // ---- operand build: units of (row t, 8 consecutive channels); F = e^{gamma - r_b(t)} ----
  for (int u = tid; u < 1024; u += NT1) {
    const int t = u >> 4, d0 = (u & 15) * 8, blk = t >> 4;
    const uint32_t off = sw128(t, d0);
    const uint4 kq = *reinterpret_cast<const uint4 *>(sm + OFF_KS + off);
    const uint4 qq = *reinterpret_cast<const uint4 *>(sm + OFF_QS + off);
    const uint32_t kw[4] = {kq.x, kq.y, kq.z, kq.w}, qw[4] = {qq.x, qq.y, qq.z, qq.w};
    uint32_t okd[4], oqd[4], oxk[4], oki[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 kf = unpack_bf16(kw[e]), qf = unpack_bf16(qw[e]);
      const int d = d0 + 2 * e;
      float F[2], ki[2], eg[2];
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const float gm = GS[gsw128(t, d + x)];
        F[x] = __expf(gm - refs[blk * 128 + d + x]);
        if (!big) {
          ki[x] = __fdividef(1.f, F[x]);
          eg[x] = F[x] * erb[blk * 128 + d + x];
        } else {
          ki[x] = __expf(GS[gsw128(16 * blk + 15, d + x)] - gm);
          eg[x] = __expf(gm);
        }
      }
      okd[e] = pack_bf16(kf.x * F[0], kf.y * F[1]);
      oqd[e] = pack_bf16(qf.x * F[0], qf.y * F[1]);
      oxk[e] = pack_bf16(kf.x * eg[0], kf.y * eg[1]);
      oki[e] = pack_bf16(kf.x * ki[0], kf.y * ki[1]);
    }
    *reinterpret_cast<uint4 *>(sm + OFF_KD + off) = make_uint4(okd[0], okd[1], okd[2], okd[3]);
    *reinterpret_cast<uint4 *>(sm + OFF_QD + off) = make_uint4(oqd[0], oqd[1], oqd[2], oqd[3]);
    *reinterpret_cast<uint4 *>(sm + OFF_XK + off) = make_uint4(oxk[0], oxk[1], oxk[2], oxk[3]);
    *reinterpret_cast<uint4 *>(sm + OFF_KI + blk * 4096 + (d0 >> 6) * 2048 + sw64(t & 15, d0 & 63)) =
        make_uint4(oki[0], oki[1], oki[2], oki[3]);
  }
  // exact diagonal blocks of M and P for a big chunk: the 136 pairs s <= t of each block, each
  // summed over d by four adjacent lanes (32 channels each); the lane for channels 0-31 of a
  // pair below the diagonal also zeroes the mirror entry above it
  if (big) {
    for (int item = tid; item < 4 * 136 * 4; item += NT1) {
      const int qd = item & 3, pr = item >> 2, i = pr / 136, pi = pr - i * 136;
      int tl = (int)((sqrtf(8.f * pi + 1.f) - 1.f) * 0.5f);
      tl += (tl + 1) * (tl + 2) / 2 <= pi;
      tl -= tl * (tl + 1) / 2 > pi;
      const int sl = pi - tl * (tl + 1) / 2, t = 16 * i + tl, s = 16 * i + sl;
      float mk = 0.f, mq = 0.f;
#pragma unroll 4
      for (int d = 32 * qd; d < 32 * qd + 32; d += 2) {
        const float2 kt = unpack_bf16(*reinterpret_cast<const uint32_t *>(sm + OFF_KS + sw128(t, d)));
        const float2 qt = unpack_bf16(*reinterpret_cast<const uint32_t *>(sm + OFF_QS + sw128(t, d)));
        const float2 ks = unpack_bf16(*reinterpret_cast<const uint32_t *>(sm + OFF_KS + sw128(s, d)));
        const float2 gt = *reinterpret_cast<const float2 *>(GS + gsw128(t, d));
        const float2 gs = *reinterpret_cast<const float2 *>(GS + gsw128(s, d));
        const float e0 = __expf(gt.x - gs.x), e1 = __expf(gt.y - gs.y);
        mk = fmaf(kt.x * ks.x, e0, fmaf(kt.y * ks.y, e1, mk));
        mq = fmaf(qt.x * ks.x, e0, fmaf(qt.y * ks.y, e1, mq));
      }
      mk += __shfl_xor_sync(0xffffffffu, mk, 1);
      mq += __shfl_xor_sync(0xffffffffu, mq, 1);
      mk += __shfl_xor_sync(0xffffffffu, mk, 2);
      mq += __shfl_xor_sync(0xffffffffu, mq, 2);
      if (qd == 0) {
        AD[i * 256 + tl * 16 + sl] = s < t ? bet[t] * mk : 0.f;
        *reinterpret_cast<__nv_bfloat16 *>(sm + OFF_PR + sw64(t, s)) = __float2bfloat16_rn(mq);
      } else if (qd == 1 && sl < tl) {
        AD[i * 256 + sl * 16 + tl] = 0.f;
        *reinterpret_cast<__nv_bfloat16 *>(sm + OFF_PR + sw64(s, t)) = __float2bfloat16_rn(0.f);
      }
    }
  }
  // P's blocks above the diagonal are zero (the scan multiplies the whole tile)
  for (int u = tid; u < 192; u += NT1) {
    const int blk = u >> 5, r = (u >> 1) & 15, hf = u & 1;
    const int i = blk < 3 ? 0 : blk < 5 ? 1 : 2, j = blk < 3 ? blk + 1 : blk < 5 ? blk - 1 : 3;
    *reinterpret_cast<uint4 *>(sm + OFF_PR + sw64(16 * i + r, 16 * j + 8 * hf)) = make_uint4(0u, 0u, 0u, 0u);
  }
  __syncthreads();

  // ---- M = Kdec Kinc^T and P = Qdec Kinc^T per block pair (j <= i), K = d (128); T_ii ----
  auto mp_block = [&](int mat, int i, int j) {
    float acc[2][4] = {};
    const bool scale = j < i;  // the pair's factor scales the A operand along d
    const uint32_t kib = s_base + OFF_KI + j * 4096;
    const float *G = scale ? gij + pair_index(i, j) * 128 : nullptr;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t af[4], bf[4];
      ldsm_x4(a_frag_addr(s_base + (mat ? OFF_QD : OFF_KD) + (kk >> 2) * 8192, 16 * i, 16 * (kk & 3), lane), af);
      if (scale) {
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          const float2 v = unpack_bf16(af[x]);
          const float2 gg = *reinterpret_cast<const float2 *>(G + 16 * kk + (x >> 1) * 8 + 2 * c4);
          af[x] = pack_bf16(v.x * gg.x, v.y * gg.y);
        }
      }
      ldsm_x4(bnk_frag_addr(kib + (kk >> 2) * 2048, 0, 16 * (kk & 3), lane), bf);
      mma16816(acc[0], af, bf[0], bf[1]);
      mma16816(acc[1], af, bf[2], bf[3]);
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int tl = g4 + 8 * hh, t = 16 * i + tl;
        const int sl = nt * 8 + 2 * c4, s = 16 * j + sl;
        float v0 = acc[nt][2 * hh], v1 = acc[nt][2 * hh + 1];
        if (mat == 0) {
          v0 = s < t ? bet[t] * v0 : 0.f;
          v1 = s + 1 < t ? bet[t] * v1 : 0.f;
          if (j == i)
            *reinterpret_cast<float2 *>(AD + i * 256 + tl * 16 + sl) = make_float2(v0, v1);
          else
            *reinterpret_cast<uint32_t *>(sm + OFF_AB + sw64(t, s)) = pack_bf16(v0, v1);
        } else {
          v0 = s <= t ? v0 : 0.f;
          v1 = s + 1 <= t ? v1 : 0.f;
          *reinterpret_cast<uint32_t *>(sm + OFF_PR + sw64(t, s)) = pack_bf16(v0, v1);
        }
      }
  };
  if (warp < 4) {
    const int i = warp;
    if (!big) mp_block(0, i, i);  // (a big chunk's diagonal blocks are already exact)
    __syncwarp();
    if (lane < 16) {  // T_ii = (I + A_ii)^{-1}, one column per lane
      const int u = lane;
      const float *A = AD + i * 256;
      float x[16];
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        float v = t == u ? 1.f : 0.f;
#pragma unroll
        for (int s2 = 0; s2 < t; ++s2) v = fmaf(-A[t * 16 + s2], x[s2], v);
        x[t] = v;
      }
      __nv_bfloat16 *Ti = reinterpret_cast<__nv_bfloat16 *>(sm + OFF_TI + i * 512);
#pragma unroll
      for (int t = 0; t < 16; ++t) Ti[t * 16 + u] = __float2bfloat16_rn(x[t]);
    }
  } else {
    for (int q = warp - 4; q < 16; q += 12) {
      // q < 10: P block number q of the 10 pairs (i, j <= i); else off-diagonal M block q - 10
      const int pr = q < 10 ? q : (q == 10 ? 1 : q == 11 ? 3 : q == 12 ? 4 : q - 7);
      const int i = pr < 1 ? 0 : pr < 3 ? 1 : pr < 6 ? 2 : 3;
      const int j = pr - i * (i + 1) / 2;
      if (big && j == i) continue;
      mp_block(q < 10 ? 1 : 0, i, j);
    }
  }
  __syncthreads();

  // ---- (I + A)^{-1} diag(beta): 8 columns per warp (warps 0-7) ----
  if (warp < 8) solve_columns128(sm, s_base, bet, warp * 8, warp >> 1, warp, lane);
  __syncthreads();

  // ---- [W | U] = (I + A)^{-1} diag(beta) [k e^gamma | v]: warp w takes 16 of the 256
  //      columns (W stored negated over Qdec, U over Kdec); meanwhile Qd = q e^gamma over the
  //      raw q tile and Kb^T = (k e^{gamma_C - gamma})^T ----
  {
    const int cw = 16 * warp, isW = cw < 128, cc = cw & 127;
    const uint32_t src = s_base + (isW ? OFF_XK : OFF_VS) + (cc >> 6) * 8192;
    uint8_t *dst = sm + (isW ? OFF_QD : OFF_KD) + (cc >> 6) * 8192;
    const float so = isW ? -1.f : 1.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float acc[2][4] = {};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (k > i) break;
        uint32_t af[4], bf[4];
        ldsm_x4(a_frag_addr(s_base + OFF_TF, 16 * i, 16 * k, lane), af);
        ldsm_x4_t(bkn_frag_addr(src, 16 * k, cc & 63, lane), bf);
        mma16816(acc[0], af, bf[0], bf[1]);
        mma16816(acc[1], af, bf[2], bf[3]);
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
          *reinterpret_cast<uint32_t *>(dst + sw64(16 * i + g4 + 8 * hh, (cc & 63) + 8 * nt + 2 * c4)) =
              pack_bf16(so * acc[nt][2 * hh], so * acc[nt][2 * hh + 1]);
    }
  }
  for (int u = tid; u < 1024; u += NT1) {
    const int t = u >> 4, d0 = (u & 15) * 8;
    const uint32_t off = sw128(t, d0);
    const uint4 kq = *reinterpret_cast<const uint4 *>(sm + OFF_KS + off);
    const uint4 qq = *reinterpret_cast<const uint4 *>(sm + OFF_QS + off);
    const uint32_t kw[4] = {kq.x, kq.y, kq.z, kq.w}, qw[4] = {qq.x, qq.y, qq.z, qq.w};
    uint32_t oq[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int d = d0 + 2 * e;
      const float2 kf = unpack_bf16(kw[e]), qf = unpack_bf16(qw[e]);
      const float g0 = GS[gsw128(t, d)], g1 = GS[gsw128(t, d + 1)];
      oq[e] = pack_bf16(qf.x * __expf(g0), qf.y * __expf(g1));
      const float gc0 = GS[gsw128(63, d)], gc1 = GS[gsw128(63, d + 1)];
      *reinterpret_cast<__nv_bfloat16 *>(sm + OFF_KBT + sw64(d, t)) = __float2bfloat16_rn(kf.x * __expf(gc0 - g0));
      *reinterpret_cast<__nv_bfloat16 *>(sm + OFF_KBT + sw64(d + 1, t)) = __float2bfloat16_rn(kf.y * __expf(gc1 - g1));
    }
    *reinterpret_cast<uint4 *>(sm + OFF_QS + off) = make_uint4(oq[0], oq[1], oq[2], oq[3]);
  }
  fence_proxy_async_smem();  // this thread's smem writes are read by the bulk copies
  __syncthreads();
  if (tid == 0) {  // the record, kept in L2 for the scan
    uint8_t *rec = (uint8_t *)p.ws + (int64_t)idx * REC;
    const uint64_t pol = l2_policy_keep();
    bulk_s2g_hint(rec + R_A0, s_base + OFF_QS, 8192, pol);
    bulk_s2g_hint(rec + R_A0 + 8192, s_base + OFF_QD, 8192, pol);
    bulk_s2g_hint(rec + R_A1, s_base + OFF_QS + 8192, 8192, pol);
    bulk_s2g_hint(rec + R_A1 + 8192, s_base + OFF_QD + 8192, 8192, pol);
    bulk_s2g_hint(rec + R_U, s_base + OFF_KD, 16384, pol);
    bulk_s2g_hint(rec + R_P, s_base + OFF_PR, 8192, pol);
    bulk_s2g_hint(rec + R_KBT, s_base + OFF_KBT, 16384, pol);
    bulk_s2g_hint(rec + R_EG, s_base + OFF_VEC + V_EG * 4, 512, pol);
    bulk_commit();
    bulk_wait_all();  // shared memory stays valid until the stores have read it
  }
}

// ---------------------------------------------------------------------------------------
// kda_fwd128_scan
// ---------------------------------------------------------------------------------------
// warps 0-1: O rows (TMEM lanes 0-63 of D1); warps 2-3: Unew rows (lanes 64-127 of D1);
// warps 4-7: the state slice (all 128 lanes of DS, one row d per thread); thread 256 (warp 8)
// issues the record loads, the MMAs and the O stores, and warp 8 owns the TMEM allocation.
constexpr int NT2 = 288;
constexpr int SLOT = 66560;                          // record slot: A0 A1 U(half) P KbT eG, 1 KB aligned
constexpr int S_A0 = 0, S_U = 32768, S_P = 40960, S_KBT = 49152, S_EG = 65536;
constexpr int OFF2_SLOT = 0;                         // 2 slots
constexpr int OFF2_SV = 2 * SLOT;                    // S^T [d][j] bf16 (128 rows), 2 x 16 KB
constexpr int OFF2_UN = OFF2_SV + 2 * 16384;         // Unew [t][j] bf16
constexpr int OFF2_O = OFF2_UN + 8192;               // O staging, 2 x 8 KB
constexpr int OFF2_MBAR = OFF2_O + 2 * 8192;         // 2 slot mbarriers, mA, mB, TMEM slot
constexpr int SMEM2 = OFF2_MBAR + 64;
constexpr uint32_t kIdesc = idesc_bf16(128, 64, 0, 1);  // A K-major, B MN-major

__device__ __forceinline__ void store_row_bf16_128(uint8_t *tile, int row, const float *x) {
#pragma unroll
  for (int ch = 0; ch < 8; ++ch)
    *reinterpret_cast<uint4 *>(tile + sw64(row, ch * 8)) =
        make_uint4(pack_bf16(x[8 * ch], x[8 * ch + 1]), pack_bf16(x[8 * ch + 2], x[8 * ch + 3]),
                   pack_bf16(x[8 * ch + 4], x[8 * ch + 5]), pack_bf16(x[8 * ch + 6], x[8 * ch + 7]));
}
__device__ __forceinline__ void tmem_row64_128(uint32_t taddr, float *x) {
  uint32_t v[32], w[32];
  tmem_ld32(taddr, v);
  tmem_ld32(taddr + 32, w);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    x[i] = __uint_as_float(v[i]);
    x[32 + i] = __uint_as_float(w[i]);
  }
}

__global__ void __launch_bounds__(NT2, 1) kda_fwd128_scan_kernel(Params p, const __grid_constant__ TmaMaps tm) {
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int bh = blockIdx.x >> 1, jh = blockIdx.x & 1, j0 = 64 * jh, b = bh / p.H, h = bh % p.H;
  const int nc = p.nc;
  const uint32_t s_base = smem_u32(sm);
  if (s_base & 1023) {
    if (tid == 0) atomicExch(&g_fwd128_status, KDA_ERR_MISALIGNED);
    return;
  }
  const uint32_t mrec = s_base + OFF2_MBAR, mA = mrec + 16, mB = mrec + 24;
  uint32_t *tslot = reinterpret_cast<uint32_t *>(sm + OFF2_MBAR + 32);
  const bool leader = tid == 256, owarp = warp < 2, uwarp = warp >= 2 && warp < 4, swarp = warp >= 4 && warp < 8;
  const int q = warp & 3;
  const int m = 32 * q + lane;  // TMEM lane: O row t (warps 0-1), 64 + Unew row (warps 2-3), state row d (4-7)

  if (leader) {
    for (int i = 0; i < 4; ++i) mbar_init(mrec + 8 * i, 1);
    mbar_fence_init();
  }
  float S[64];  // state warps: S^T[m][jj] = S[j0 + jj][m]
#pragma unroll
  for (int jj = 0; jj < 64; ++jj) S[jj] = 0.f;
  if (swarp && p.state0) {
#pragma unroll
    for (int jj = 0; jj < 64; ++jj) S[jj] = p.state0[(int64_t)bh * D * D + (int64_t)(j0 + jj) * D + m];
  }
  if (swarp) store_row_bf16_128(sm + OFF2_SV, m, S);
  if (warp == 8) {
    tmem_alloc(smem_u32(tslot), 128);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tD = *tslot;
  const uint32_t lq = (uint32_t)(32 * q) << 16;
  const uint32_t t1 = tD + lq, tS = tD + 64 + lq;  // this warp's lane quarter of D1 / DS

  auto issue = [&](int c) {  // leader: this CTA's part of chunk c's record, three bulk copies
    const uint8_t *rec = (const uint8_t *)p.ws + ((int64_t)bh * nc + c) * REC;
    const int s = c & 1;
    const uint32_t dst = s_base + OFF2_SLOT + s * SLOT, mb = mrec + 8 * s;
    mbar_expect_tx(mb, 32768 + 8192 + (REC - R_P));
    bulk_g2s(dst + S_A0, rec + R_A0, 32768, mb);
    bulk_g2s(dst + S_U, rec + R_U + 8192 * jh, 8192, mb);
    bulk_g2s(dst + S_P, rec + R_P, REC - R_P, mb);
  };
  if (leader) issue(0);
  int issued = 1, landed = 0;  // leader: record copies issued / seen complete
  bool failed = false;
  for (int c = 0; c < nc; ++c) {
    const int s = c & 1, buf = c & 1;
    const uint32_t slot = s_base + OFF2_SLOT + s * SLOT;
    const uint8_t *slotm = sm + OFF2_SLOT + s * SLOT;
    const uint32_t sv = s_base + OFF2_SV + (c & 1) * 16384;
    uint8_t *svn = sm + OFF2_SV + ((c + 1) & 1) * 16384;
    // the O store of chunk c - 2 (same staging buffer) has read its source
    if (leader) asm volatile("cp.async.bulk.wait_group.read 1;\n" ::: "memory");
    if (__syncthreads_or(!mbar_wait(mrec + 8 * s, (c >> 1) & 1))) { failed = true; break; }
    landed = c + 1;
    if (leader) {
      if (c + 1 < nc) {
        issue(c + 1);
        issued = c + 2;
      }
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < 8; ++k)
        tc_mma(tD, desc_k(slot + S_A0 + (k >> 2) * 16384, k & 3), desc_mn(sv, k), kIdesc, k > 0);
      tc_commit(mA);
    }
    bool ok = true;
    if (swarp) {  // DS <- e^{gamma_C} S^T (the previous chunk's MMA BS has been read)
      const float e = reinterpret_cast<const float *>(slotm + S_EG)[m];
      uint32_t v[32], w[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        v[j] = __float_as_uint(e * S[j]);
        w[j] = __float_as_uint(e * S[32 + j]);
      }
      tmem_st32(tS, v);
      tmem_st32(tS + 32, w);
      tmem_wait_st();
      tc_fence_before();
    } else if (uwarp) {  // Unew = U - W S^T
      ok = mbar_wait(mA, c & 1);
      tc_fence_after();
      float x[64];
      tmem_row64_128(t1, x);
      const int r = m - 64;
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        const uint4 u = *reinterpret_cast<const uint4 *>(slotm + S_U + sw64(r, ch * 8));
        const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = unpack_bf16(uw[e]);
          x[8 * ch + 2 * e] += f.x;
          x[8 * ch + 2 * e + 1] += f.y;
        }
      }
      store_row_bf16_128(sm + OFF2_UN, r, x);
      fence_proxy_async_smem();
      tc_fence_before();
    }
    if (__syncthreads_or(!ok)) { failed = true; break; }
    if (leader) {
      tc_fence_after();
      const uint32_t un = s_base + OFF2_UN;
#pragma unroll
      for (int k = 0; k < 4; ++k) tc_mma(tD, desc_k(slot + S_P, k), desc_mn(un, k), kIdesc, 1);
#pragma unroll
      for (int k = 0; k < 4; ++k) tc_mma(tD + 64, desc_k(slot + S_KBT, k), desc_mn(un, k), kIdesc, 1);
      tc_commit(mB);
    }
    if (owarp || swarp) {
      ok = mbar_wait(mB, c & 1);
      tc_fence_after();
      float x[64];
      if (owarp) {
        tmem_row64_128(t1, x);
        store_row_bf16_128(sm + OFF2_O + buf * 8192, m, x);  // O row t
      } else {
        tmem_row64_128(tS, x);
#pragma unroll
        for (int j = 0; j < 64; ++j) S[j] = x[j];
        store_row_bf16_128(svn, m, S);  // S^T(c + 1) row d
      }
      fence_proxy_async_smem();
      tc_fence_before();
    }
    if (__syncthreads_or(!ok)) { failed = true; break; }
    if (leader) {  // O by TMA (rows past T dropped)
      tma_store_rows(&tm.m[0], s_base + OFF2_O + buf * 8192, h, c * C, b, j0);
      bulk_commit();
    }
  }
  if (failed && leader) atomicExch(&g_fwd128_status, KDA_ERR_TIMEOUT);
  if (!failed && swarp) {
#pragma unroll
    for (int jj = 0; jj < 64; ++jj) p.stateT[(int64_t)bh * D * D + (int64_t)(j0 + jj) * D + m] = S[jj];
  }
  if (leader) {
    bulk_wait_all();
    if (failed) {  // no copy may still land and no MMA may still write TMEM (bounded waits)
      for (int c = landed; c < issued; ++c) mbar_wait(mrec + 8 * (c & 1), (c >> 1) & 1);
      mbar_wait(mA, 0);
      mbar_wait(mA, 1);
      mbar_wait(mB, 0);
      mbar_wait(mB, 1);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 8) tmem_dealloc(tD, 128);
}

template <typename Tb>
int launch(const Params &p, cudaStream_t st) {
  auto k1 = kda_fwd128_chunks_kernel<Tb>;
  if (cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM1)) return KDA_ERR_CUDA;
  const int nchunks = p.B * p.H * p.nc;
  TmaMaps tm;
  const void *srcs[4] = {p.q, p.k, p.v, p.g};
  const Str in_str[4] = {p.sq, p.sk, p.sv, p.sg};
  for (int i = 0; i < 4; ++i)
    if (int e = tma_map_bthd(&tm.m[i], srcs[i], p.B, p.T, p.H, D, i == 3, &in_str[i])) return e;
  k1<<<nchunks, NT1, SMEM1, st>>>(p, tm);
  count_launch();
  if (cudaFuncSetAttribute(kda_fwd128_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2))
    return KDA_ERR_CUDA;
  TmaMaps to;
  if (int e = tma_map_bthd(&to.m[0], p.o, p.B, p.T, p.H, D, false)) return e;
  kda_fwd128_scan_kernel<<<p.B * p.H * 2, NT2, SMEM2, st>>>(p, to);
  count_launch();
  return cudaPeekAtLastError() == cudaSuccess ? KDA_OK : KDA_ERR_CUDA;
}

}  // namespace tcfwd128

bool tc128_supported(const KdaDesc *d) {
  return d->Dk == 128 && d->Dv == 128 && d->chunk == 64 && d->dtype_qkv == KDA_BF16 &&
         (d->dtype_beta == KDA_BF16 || d->dtype_beta == KDA_F32);
}
size_t tc128_workspace_bytes(const KdaDesc *d) {
  const int64_t nc = (d->T + d->chunk - 1) / d->chunk;
  return tcfwd128::ws_bytes(d->B * d->H * nc);
}
int tc128_fwd(const Params &p, int dtype_beta, cudaStream_t st) {
  return dtype_beta == KDA_BF16 ? tcfwd128::launch<__nv_bfloat16>(p, st) : tcfwd128::launch<float>(p, st);
}
int tc128_fwd_device_status(bool reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, tcfwd128::g_fwd128_status, sizeof(int)) != cudaSuccess) return KDA_ERR_CUDA;
  if (reset && v) {
    const int z = 0;
    cudaMemcpyToSymbol(tcfwd128::g_fwd128_status, &z, sizeof(int));
  }
  return v;
}

}  // namespace kda
