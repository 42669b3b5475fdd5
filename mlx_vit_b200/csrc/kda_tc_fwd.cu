// Tensor-core KDA forward for D = 64, chunk = 64, bf16 q/k/v, in two kernels.
//
//  kda_fwd_chunks  one CTA per (b, h, chunk), two CTAs per SM; chunks are independent: every
//                  state-independent quantity of the chunk, written as a per-chunk record to the
//                  forward workspace (-W, U, O_intra = P U, N = Kb^T U) and, for training, the
//                  backward's record (P, M, Tinv = (I+A)^{-1}, Mneg = -Kb^T W, Qt = Qd - P W,
//                  e^{gamma_C}; without one, Mneg, Qt and e^{gamma_C} go to the workspace).
//  kda_fwd_scan    one CTA per (b, h): the state recurrence S^T <- diag(e^{gamma_C}) S^T +
//                  Mneg S^T + N, one tcgen05 MMA per chunk on the chain, with O = Qt S^T +
//                  O_intra and Unew = U - W S^T formed beside it (see the kernel's comment).
//
// Chunk quantities (gamma = cumsum(g) inside the chunk, rows t, 16-row blocks b(t), r_i = gamma
// at the middle row of block i):
//  1. operand build (elementwise): Kdec = k e^{gamma - r_b(t)}, Qdec = q e^{...},
//     Kinc[i][j] = k_s e^{r_i - gamma_s} (s in block j <= i), beta k e^gamma, beta v,
//     Qd = q e^gamma, Kb = k e^{gamma_C - gamma}; one exp and one reciprocal per element, the
//     other factors are products with per-block vectors e^{r_i}, e^{gamma_C - r_i}, e^{r_i - r_j}
//  2. M = Kdec Kinc^T, P = Qdec Kinc^T per block pair (mma.sync): the decay-weighted K K^T and
//     Q K^T with both factors of e^{gamma_t - gamma_s} bounded; A = beta M (strict lower)
//  3. T_ii = (I + A_ii)^{-1} for the four 16x16 diagonal blocks (fp32 substitution)
//  4. Tinv = (I+A)^{-1} by block forward substitution (mma.sync), then W = Tinv beta Kd,
//     U = Tinv beta V as one GEMM
// This is the chunkwise WY algebra of the reference's chunkwise path (nope_gdn_mlx.py:549-613,
// 2318-2456) with U = (I+A)^{-1} beta (V - K_proj S^T) split into U - W S^T.
#include "kda_common.cuh"
#include "kda_mma.cuh"
#include "kda_tc05.cuh"
#include "kda_tma.cuh"

namespace kda {
namespace tcfwd {

// set to a KDA_ERR_* code by a bounded wait that gave up (read by kda_device_status)
static __device__ int g_fwd_status;

// Optional event trace of the forward scan (builds with -DKDA_SCAN_TRACE only): SM clock at
// fixed points of the first 64 chunks of (b, h) = 0, read back by kda_scan_trace().
#ifdef KDA_SCAN_TRACE
__device__ long long g_scan_trace[20][64];
#define SCAN_TR(slot, c) do { if (bh == 0 && (c) < 64) g_scan_trace[slot][c] = clock64(); } while (0)
__device__ long long g_chunk_trace[12][64];
#define CHUNK_TR(slot) do { if (threadIdx.x == 0 && (int)blockIdx.x < 64) g_chunk_trace[slot][blockIdx.x] = clock64(); } while (0)
#else
#define SCAN_TR(slot, c) do { } while (0)
#define CHUNK_TR(slot) do { } while (0)
#endif

constexpr int C = 64, D = 64;
constexpr float kSpanMax = 60.f;
// the block-pair factors e^{r_i - r_j} of a chunk that is not "big" stay above fp32's smallest
// normal (e^-87) only if gamma moves at most this much between the middle rows of the first and
// the last block; beyond it the factor would flush to zero while the decay it stands for
// (e^{gamma_t - gamma_s} for t, s close to the block boundary) is not negligible
constexpr float kMidGapMax = 80.f;

// the chunk kernel's tiles of per-chunk values in shared memory (bf16, swizzled): Qd = q e^gamma
// [t][d], -W [t][d], U [t][j], P [t][s] (zero above the diagonal), e^{gamma_C} (fp32)
constexpr int HO_QD = 0, HO_W = 8192, HO_U = 16384, HO_P = 24576, HO_EG = 32768;
// per-chunk record handed from kda_fwd_chunks to kda_fwd_scan in the forward workspace (bf16
// tiles, swizzled as in shared memory): Mneg = -Kb^T W [d][d'], Qt = Qd - P W [t][d], -W [t][d],
// U [t][j], O_intra = P U [t][j], N = Kb^T U [d][j], e^{gamma_C} (fp32).  With a saved record
// (training) Mneg, Qt and e^{gamma_C} go there instead and the scan reads them from it.
constexpr int WS_MN = 0, WS_QT = 8192, WS_W = 16384, WS_U = 24576, WS_OI = 32768, WS_N = 40960,
              WS_EG = 49152;
constexpr int WS_SIZE = 49152 + 256;

// ---------------------------------------------------------------------------------------
// kda_fwd_chunks
// ---------------------------------------------------------------------------------------
// One CTA of 8 warps per chunk, with about 107 KB of shared memory so that two CTAs share an SM:
// each chunk's phases meet at CTA barriers, and the other CTA's work fills those gaps.  Tiles are
// reused as their contents die (the phase that frees each is noted).
constexpr int NT1 = 256;
constexpr int R_QS = 0;                // q (TMA) -> Qdec (operand build, in place) -> N staging (6)
constexpr int R_KS = 8192;             // k (TMA) -> Kdec (in place) -> Tinv (4)
constexpr int R_VS = 16384;            // v (TMA) -> beta V (in place) -> Qt staging (6)
constexpr int R_GS = 24576;            // g (TMA, fp32) or f -> gamma -> beta Kd | Kb (operand build)
constexpr int R_XK = R_GS, R_KB = R_GS + 8192;   //   beta Kd -> Mneg staging (6);  Kb [t][d]
constexpr int OFF_OUT = 40960;         // Qd, -W, U, P tiles and e^{gamma_C} (HO_*); Kinc's four
                                       //   diagonal 16 x 64 tiles sit in -W | U until (2) is done
constexpr int R_KI = OFF_OUT + HO_W;
constexpr int R_MK = OFF_OUT + 33 * 1024;   // M = Kdec Kinc^T strict lower (bf16), saved
constexpr int R_AB = R_MK + 8192;      // A off-diagonal blocks (bf16) -> O_intra staging (6)
constexpr int R_AD = R_AB + 8192;      // A diagonal blocks fp32 4 x 16 x 16
constexpr int R_TI = R_AD + 4096;      // T_ii bf16 4 x 16 x 16
constexpr int R_RS = R_TI + 2048;      // per-warp 16 x 16 staging of the block solve
constexpr int OFF_VEC = R_RS + 8 * 256;
// vectors (floats): bet[64] refs[4][64] part[4][64] erb[4][64] egr[4][64] gij[16][64] gend[4][64]
// gC[64] flag[4]
constexpr int V_BET = 0, V_REFS = 64, V_PART = 320, V_ERB = 576, V_EGR = 832, V_G = 1088, V_GEND = 2112,
              V_GC = 2368, V_FLAG = 2432;
constexpr int OFF_MBAR1 = OFF_VEC + (2432 + 4) * 4;  // mbarrier of the TMA loads
constexpr int SMEM1 = OFF_MBAR1 + 8;

// Block forward substitution Tinv = (I+A)^{-1} for the 8 columns n0..n0+7, by one warp:
//   Y_i = T_ii (E_i - sum_{j<i} A_ij Y_j),  i = ib..3  (rows of blocks below ib are zero).
__device__ __forceinline__ void solve_columns(uint8_t *sm, uint32_t s_base, int n0, int ib, int warp, int lane) {
  const int g4 = lane >> 2, c4 = lane & 3, l15 = lane & 15;
  const uint32_t Yb = s_base + R_KS;
  uint8_t *Ym = sm + R_KS;
  const uint32_t Rs = s_base + R_RS + warp * 256;
  uint8_t *Rm = sm + R_RS + warp * 256;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (i < ib) continue;
    float acc[4] = {};
#pragma unroll
    for (int j = 0; j < i; ++j) {
      if (j < ib) continue;
      uint32_t af[4], bf[2];
      ldsm_x4(a_frag_addr(s_base + R_AB, 16 * i, 16 * j, lane), af);
      ldsm_x2_t(Yb + sw64(16 * j + (l15 & 7) + ((l15 >> 3) << 3), n0), bf);
      mma16816(acc, af, bf[0], bf[1]);
    }
    // R = E_i - acc -> bf16 staging [t][col] 16x8
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int tl = g4 + 8 * hh, col = n0 + 2 * c4;
      const float x0 = 16 * i + tl == col ? 1.f : 0.f, x1 = 16 * i + tl == col + 1 ? 1.f : 0.f;
      *reinterpret_cast<uint32_t *>(Rm + tl * 16 + c4 * 4) = pack_bf16(x0 - acc[2 * hh], x1 - acc[2 * hh + 1]);
    }
    __syncwarp();
    uint32_t af[4], bf[2];
    ldsm_x4(s_base + R_TI + i * 512 + (lane & 15) * 32 + (lane >> 4) * 16, af);
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
__global__ void __launch_bounds__(NT1, 2) kda_fwd_chunks_kernel(Params p, const __grid_constant__ TmaMaps tm) {
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g4 = lane >> 2, c4 = lane & 3;
  const int nc = p.nc, T = p.T, H = p.H;
  const int idx = blockIdx.x, bh = idx / nc, c = idx % nc, b = bh / H, h = bh % H, t0 = c * C;
  const uint32_t s_base = smem_u32(sm);
  if (s_base & 1023) {  // TMA tiles with the 128-byte swizzle need a 1024-byte aligned base
    if (tid == 0) atomicExch(&g_fwd_status, KDA_ERR_MISALIGNED);
    return;
  }
  float *GS = reinterpret_cast<float *>(sm + R_GS);
  float *AD = reinterpret_cast<float *>(sm + R_AD);
  float *vec = reinterpret_cast<float *>(sm + OFF_VEC);
  float *bet = vec + V_BET, *refs = vec + V_REFS, *part = vec + V_PART;
  float *erb = vec + V_ERB, *egr = vec + V_EGR, *gij = vec + V_G, *gend = vec + V_GEND, *gCv = vec + V_GC;
  int *flag = reinterpret_cast<int *>(vec + V_FLAG);
  uint8_t *hom = sm + OFF_OUT;
  const uint32_t ho = s_base + OFF_OUT;
  float *eG = reinterpret_cast<float *>(hom + HO_EG);
  const int nvalid = min(C, T - t0);

  const uint32_t mbar = s_base + OFF_MBAR1;
  if (tid == 0) {
    mbar_init(mbar, 1);
    mbar_fence_init();
    mbar_expect_tx(mbar, 3 * 8192 + (p.gated ? 8192 : 16384));
    tma_load_rows(s_base + R_QS, &tm.m[0], h, t0, b, mbar);
    tma_load_rows(s_base + R_KS, &tm.m[1], h, t0, b, mbar);
    tma_load_rows(s_base + R_VS, &tm.m[2], h, t0, b, mbar);
    if (p.gated)  // the gate pre-activation f (bf16) into the first half of GS, converted in place
      tma_load_rows(s_base + R_GS, &tm.m[3], h, t0, b, mbar);
    else
      tma_load_rows_f32(s_base + R_GS, &tm.m[3], h, t0, b, mbar);
  }
  Tb beta_raw = from_f<Tb>(0.f);
  if (tid < C && tid < nvalid) beta_raw = ((const Tb *)p.beta)[at(p.sb, b, t0 + tid, h)];
  // P's blocks above the diagonal are zero (the scan's products read whole tiles)
  for (int u = tid; u < 192; u += NT1) {
    const int blk = u >> 5, r = (u >> 1) & 15, hf = u & 1;
    const int i = blk < 3 ? 0 : blk < 5 ? 1 : 2, j = blk < 3 ? blk + 1 : blk < 5 ? blk - 1 : 3;
    *reinterpret_cast<uint4 *>(hom + HO_P + sw64(16 * i + r, 16 * j + 8 * hf)) = make_uint4(0u, 0u, 0u, 0u);
  }
  __syncthreads();  // the mbarrier is initialised before anyone waits on it
  if (__syncthreads_or(!mbar_wait(mbar, 0))) {
    if (tid == 0) {
      atomicExch(&g_fwd_status, KDA_ERR_TIMEOUT);
      mbar_wait(mbar, 0);  // (bounded) the loads in flight land before the CTA exits
    }
    return;
  }
  if (tid < C)
    bet[tid] = !p.gated ? to_f(beta_raw) : tid < nvalid ? p.beta_scale * sigmoid_f(to_f(beta_raw)) : 0.f;
  if (p.gated) {  // rows 0-31, then 32-63 (each call reads its rows of f before writing them)
    gate_to_g(sm + R_GS, GS, p.A_log, p.dt_bias, h, nvalid, tid, true);
    gate_to_g(sm + R_GS, GS, p.A_log, p.dt_bias, h, nvalid, tid + NT1, true);
  }
  __syncthreads();
  CHUNK_TR(0);

  // ---- (1a) gamma = cumsum(g): 4 segments of 16 rows per channel ----
  {
    const int d = tid & 63, seg = tid >> 6;
    float acc = 0.f;
#pragma unroll
    for (int r = 0; r < 16; ++r) acc += GS[gsw(seg * 16 + r, d)];
    part[seg * 64 + d] = acc;
    __syncthreads();
    float off = 0.f;
    for (int s2 = 0; s2 < seg; ++s2) off += part[s2 * 64 + d];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      off += GS[gsw(seg * 16 + r, d)];
      GS[gsw(seg * 16 + r, d)] = off;
    }
    __syncthreads();
  }
  // guard: factored decay stays within e^{kSpanMax} unless gamma moves more than that across
  // half a 16-row block (or the block-pair factors would leave fp32's range, kMidGapMax).  Such a
  // "big" chunk factors e^{gamma_t - gamma_s} (t in block i > j, the block of s) as A_t G_ij B_s
  // with A_t = e^{gamma_t - gamma(start of i)}, G_ij = e^{gamma(start of i) - gamma(end of j)},
  // B_s = e^{gamma(end of j) - gamma_s}, every factor <= 1, and computes its diagonal blocks exactly.
  if (tid < 64) {
    float span = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      span = fmaxf(span, GS[gsw(i * 16, tid)] - GS[gsw(i * 16 + 8, tid)]);
      span = fmaxf(span, GS[gsw(i * 16 + 8, tid)] - GS[gsw(i * 16 + 15, tid)]);
    }
    if (!(GS[gsw(8, tid)] - GS[gsw(56, tid)] <= kMidGapMax)) span = 2.f * kSpanMax;
    const int any = __any_sync(0xffffffffu, !(span <= kSpanMax));
    if (lane == 0) flag[warp] = any;
  }
  __syncthreads();
  CHUNK_TR(1);
  const bool big = flag[0] | flag[1];
  // per-block vectors, item (slot, d): slot i < 4 -> block i's entries, slot 4 -> gamma_C
  for (int u = tid; u < 320; u += NT1) {
    const int d = u & 63, slot = u >> 6, ro = big ? 0 : 8;
    const float gC = GS[gsw(63, d)];
    if (slot < 4) {
      const int i = slot;
      const float ri = GS[gsw(i * 16 + ro, d)];
      refs[i * 64 + d] = ri;
      erb[i * 64 + d] = __expf(ri);
      egr[i * 64 + d] = __expf(gC - ri);
      gend[i * 64 + d] = GS[gsw(i * 16 + 15, d)];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        gij[(i * 4 + j) * 64 + d] = j < i ? __expf(ri - GS[gsw(j * 16 + (big ? 15 : ro), d)]) : (j == i ? 1.f : 0.f);
    } else {
      eG[d] = __expf(gC);
      gCv[d] = gC;
    }
  }
  __syncthreads();
  CHUNK_TR(2);

  // diagonal blocks of M and P for a "big" chunk, from the raw q / k tiles (so before the operand
  // build reuses them), each 16-row block split into 8-row halves:
  //  - t in the upper half, s in the lower half: e^{gamma_t - gamma_s} = A_t B_s with A_t =
  //    e^{gamma_t - gamma_8} and B_s = e^{gamma_8 - gamma_s} (row 8 of the block), both <= 1, so
  //    this quadrant is a tensor-core product of X = k A (upper rows) / k B (lower rows) and
  //    Y = q A (upper rows), built in the Qd / -W tiles that the operand build fills later;
  //  - t in the lower half, s in the upper half: zero (above the diagonal);
  //  - the two 8 x 8 triangles on the diagonal: exact, per-element factors (s <= t, so <= 1).
  if (big) {
    uint8_t *XT = hom + HO_QD, *YT = hom + HO_W;
    for (int u = tid; u < 512; u += NT1) {
      const int t = u >> 3, d0 = (u & 7) * 8, up = (t >> 3) & 1, rr = (t & ~15) + 8;
      const uint32_t off = sw64(t, d0);
      const uint4 kq = *reinterpret_cast<const uint4 *>(sm + R_KS + off);
      const uint4 qq = *reinterpret_cast<const uint4 *>(sm + R_QS + off);
      const uint32_t kw[4] = {kq.x, kq.y, kq.z, kq.w}, qw[4] = {qq.x, qq.y, qq.z, qq.w};
      uint32_t ox[4], oy[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d = d0 + 2 * e;
        const float2 gt = *reinterpret_cast<const float2 *>(GS + gsw(t, d));
        const float2 gr = *reinterpret_cast<const float2 *>(GS + gsw(rr, d));
        const float f0 = __expf(up ? gt.x - gr.x : gr.x - gt.x), f1 = __expf(up ? gt.y - gr.y : gr.y - gt.y);
        const float2 kf = unpack_bf16(kw[e]), qf = unpack_bf16(qw[e]);
        ox[e] = pack_bf16(kf.x * f0, kf.y * f1);
        oy[e] = pack_bf16(qf.x * f0, qf.y * f1);
      }
      *reinterpret_cast<uint4 *>(XT + off) = make_uint4(ox[0], ox[1], ox[2], ox[3]);
      if (up) *reinterpret_cast<uint4 *>(YT + off) = make_uint4(oy[0], oy[1], oy[2], oy[3]);
    }
    __syncthreads();
    CHUNK_TR(9);
    {  // warp (block i, M or P): the quadrant t upper / s lower, and the zero quadrant above it
      const int i = warp >> 1, isP = warp & 1;
      float acc[4] = {};
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t af[4], bf[2];
        ldsm_x4(a_frag_addr(ho + (isP ? HO_W : HO_QD), 16 * i, 16 * kk, lane), af);
        ldsm_x2(t8_frag_addr(ho + HO_QD, 16 * i, 16 * kk, lane), bf);  // X rows s, k = d
        mma16816(acc, af, bf[0], bf[1]);
      }
      const int tl = 8 + g4, t = 16 * i + tl, sl = 2 * c4;  // rows g4 + 8 of the fragment
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const float v = acc[2 + x];
        if (isP) {
          *reinterpret_cast<__nv_bfloat16 *>(hom + HO_P + sw64(t, 16 * i + sl + x)) = __float2bfloat16_rn(v);
          *reinterpret_cast<__nv_bfloat16 *>(hom + HO_P + sw64(16 * i + sl + x, t)) = __float2bfloat16_rn(0.f);
        } else {
          AD[i * 256 + tl * 16 + sl + x] = bet[t] * v;
          AD[i * 256 + (sl + x) * 16 + tl] = 0.f;
          *reinterpret_cast<__nv_bfloat16 *>(sm + R_MK + sw64(t, 16 * i + sl + x)) = __float2bfloat16_rn(v);
          *reinterpret_cast<__nv_bfloat16 *>(sm + R_MK + sw64(16 * i + sl + x, t)) = __float2bfloat16_rn(0.f);
        }
      }
    }
    CHUNK_TR(10);
    {  // warp w: the triangle of half w & 1 of block w >> 1 (36 pairs t >= s).  Lane l sums pair
       // l over all 64 channels; a column read then touches one address per row, each row in
       // its own bank (or the same address: broadcast).  The last four pairs (row 7, columns
       // 4-7) take eight lanes each, one eighth of the channels per lane.
      const int i = warp >> 1, hb = 16 * i + 8 * (warp & 1);
      auto store = [&](int t, int s, float mk, float mq, bool mirror) {
        const int tb = t - 16 * i, sb = s - 16 * i;  // positions in the 16 x 16 block
        AD[i * 256 + tb * 16 + sb] = s < t ? bet[t] * mk : 0.f;
        *reinterpret_cast<__nv_bfloat16 *>(sm + R_MK + sw64(t, s)) = __float2bfloat16_rn(s < t ? mk : 0.f);
        *reinterpret_cast<__nv_bfloat16 *>(hom + HO_P + sw64(t, s)) = __float2bfloat16_rn(mq);
        if (mirror && s < t) {  // the mirror (s, t) above the diagonal
          AD[i * 256 + sb * 16 + tb] = 0.f;
          *reinterpret_cast<__nv_bfloat16 *>(sm + R_MK + sw64(s, t)) = __float2bfloat16_rn(0.f);
          *reinterpret_cast<__nv_bfloat16 *>(hom + HO_P + sw64(s, t)) = __float2bfloat16_rn(0.f);
        }
      };
      auto dot = [&](int t, int s, int d0, int nd, float &mk, float &mq) {
#pragma unroll 8
        for (int d = d0; d < d0 + nd; d += 2) {
          const float2 kt = unpack_bf16(*reinterpret_cast<const uint32_t *>(sm + R_KS + sw64(t, d)));
          const float2 qt = unpack_bf16(*reinterpret_cast<const uint32_t *>(sm + R_QS + sw64(t, d)));
          const float2 ks = unpack_bf16(*reinterpret_cast<const uint32_t *>(sm + R_KS + sw64(s, d)));
          const float2 gt = *reinterpret_cast<const float2 *>(GS + gsw(t, d));
          const float2 gs = *reinterpret_cast<const float2 *>(GS + gsw(s, d));
          const float e0 = __expf(gt.x - gs.x), e1 = __expf(gt.y - gs.y);
          mk = fmaf(kt.x * ks.x, e0, fmaf(kt.y * ks.y, e1, mk));
          mq = fmaf(qt.x * ks.x, e0, fmaf(qt.y * ks.y, e1, mq));
        }
      };
      {  // pairs 0-31: row tl, column sl with lane = tl (tl + 1) / 2 + sl
        int tl = (int)((sqrtf(8.f * lane + 1.f) - 1.f) * 0.5f);
        tl += (tl + 1) * (tl + 2) / 2 <= lane;
        tl -= tl * (tl + 1) / 2 > lane;
        const int sl = lane - tl * (tl + 1) / 2;
        float mk = 0.f, mq = 0.f;
        dot(hb + tl, hb + sl, 0, 64, mk, mq);
        store(hb + tl, hb + sl, mk, mq, true);
      }
      {  // pairs 32-35: row 7, columns 4 + (lane >> 3)
        const int e8 = lane & 7, t = hb + 7, s = hb + 4 + (lane >> 3);
        float mk = 0.f, mq = 0.f;
        dot(t, s, 8 * e8, 8, mk, mq);
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
          mk += __shfl_xor_sync(0xffffffffu, mk, o);
          mq += __shfl_xor_sync(0xffffffffu, mq, o);
        }
        if (e8 == 0) store(t, s, mk, mq, true);
      }
    }
    __syncthreads();
    CHUNK_TR(3);
  }

  // ---- (1b) operand build: 512 units of (row t, 8 consecutive channels), two per thread; all
  //      reads first, then (after a barrier) the writes, several of which go over the inputs ----
  {
    uint4 okd[2], oqd[2], oxk[2], oqe[2], oxv[2], okb[2], oki[2];
#pragma unroll
    for (int w2 = 0; w2 < 2; ++w2) {
      const int u = tid + NT1 * w2;
      const int t = u >> 3, ch = u & 7, d0 = ch * 8, blk = t >> 4;
      const uint32_t off = sw64(t, d0);
      const uint4 kq = *reinterpret_cast<const uint4 *>(sm + R_KS + off);
      const uint4 qq = *reinterpret_cast<const uint4 *>(sm + R_QS + off);
      const uint4 vq = *reinterpret_cast<const uint4 *>(sm + R_VS + off);
      const uint32_t kw[4] = {kq.x, kq.y, kq.z, kq.w}, qw[4] = {qq.x, qq.y, qq.z, qq.w},
                     vw[4] = {vq.x, vq.y, vq.z, vq.w};
      const float bt = bet[t];
      const float4 ga4 = *reinterpret_cast<const float4 *>(GS + gsw(t, d0));
      const float4 gb4 = *reinterpret_cast<const float4 *>(GS + gsw(t, d0 + 4));
      const float gam[8] = {ga4.x, ga4.y, ga4.z, ga4.w, gb4.x, gb4.y, gb4.z, gb4.w};
      uint32_t a_kd[4], a_qd[4], a_xk[4], a_xv[4], a_qe[4], a_kb[4], a_ki[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 kf = unpack_bf16(kw[e]), qf = unpack_bf16(qw[e]), vf = unpack_bf16(vw[e]);
        const int d = d0 + 2 * e;
        const float2 rf2 = *reinterpret_cast<const float2 *>(refs + blk * 64 + d);
        const float2 er2 = *reinterpret_cast<const float2 *>(erb + blk * 64 + d);
        const float2 eq2 = *reinterpret_cast<const float2 *>(egr + blk * 64 + d);
        const float rf[2] = {rf2.x, rf2.y}, er[2] = {er2.x, er2.y}, eq[2] = {eq2.x, eq2.y};
        float F[2], iF[2], eg[2], eb[2];
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          const float gm = gam[2 * e + x];
          F[x] = __expf(gm - rf[x]);
          if (!big) {
            iF[x] = __fdividef(1.f, F[x]);
            eg[x] = F[x] * er[x];
            eb[x] = iF[x] * eq[x];
          } else {
            iF[x] = __expf(gend[blk * 64 + d + x] - gm);  // B_s = e^{gamma(end of block) - gamma_s}
            eg[x] = __expf(gm);
            eb[x] = __expf(gCv[d + x] - gm);
          }
        }
        a_kd[e] = pack_bf16(kf.x * F[0], kf.y * F[1]);
        a_qd[e] = pack_bf16(qf.x * F[0], qf.y * F[1]);
        a_xk[e] = pack_bf16(bt * kf.x * eg[0], bt * kf.y * eg[1]);
        a_qe[e] = pack_bf16(qf.x * eg[0], qf.y * eg[1]);
        a_xv[e] = pack_bf16(bt * vf.x, bt * vf.y);
        a_kb[e] = pack_bf16(kf.x * eb[0], kf.y * eb[1]);
        // Kinc of the diagonal block only: k / F (the GEMMs rescale it per block pair), or k B_s
        a_ki[e] = pack_bf16(kf.x * iF[0], kf.y * iF[1]);
      }
      okd[w2] = make_uint4(a_kd[0], a_kd[1], a_kd[2], a_kd[3]);
      oqd[w2] = make_uint4(a_qd[0], a_qd[1], a_qd[2], a_qd[3]);
      oxk[w2] = make_uint4(a_xk[0], a_xk[1], a_xk[2], a_xk[3]);
      oqe[w2] = make_uint4(a_qe[0], a_qe[1], a_qe[2], a_qe[3]);
      oxv[w2] = make_uint4(a_xv[0], a_xv[1], a_xv[2], a_xv[3]);
      okb[w2] = make_uint4(a_kb[0], a_kb[1], a_kb[2], a_kb[3]);
      oki[w2] = make_uint4(a_ki[0], a_ki[1], a_ki[2], a_ki[3]);
    }
    __syncthreads();
#pragma unroll
    for (int w2 = 0; w2 < 2; ++w2) {
      const int u = tid + NT1 * w2;
      const int t = u >> 3, d0 = (u & 7) * 8, blk = t >> 4;
      const uint32_t off = sw64(t, d0);
      *reinterpret_cast<uint4 *>(sm + R_KS + off) = okd[w2];
      *reinterpret_cast<uint4 *>(sm + R_QS + off) = oqd[w2];
      *reinterpret_cast<uint4 *>(sm + R_XK + off) = oxk[w2];
      *reinterpret_cast<uint4 *>(sm + R_VS + off) = oxv[w2];
      *reinterpret_cast<uint4 *>(hom + HO_QD + off) = oqe[w2];
      *reinterpret_cast<uint4 *>(sm + R_KB + off) = okb[w2];
      *reinterpret_cast<uint4 *>(sm + R_KI + blk * 2048 + sw64(t & 15, d0)) = oki[w2];
    }
  }
  __syncthreads();
  CHUNK_TR(4);

  // ---- (2) M = Kdec Kinc^T and P = Qdec Kinc^T per (block row i, block column j <= i), and
  //      (3) T_ii = (I + A_ii)^{-1}.  Warps 0-3 take the diagonal M block i = warp and invert it
  //      right away (one column per lane, fp32 substitution), then one of the 16 other blocks
  //      each; warps 4-7 take three each ----
  auto mp_block = [&](int mat, int i, int j) {
    float acc[2][4] = {};
    // only the diagonal Kinc tiles exist (k / F, or k B for a big chunk); the block pair's
    // factor (e^{r_i - r_j}, or G_ij) scales the A operand along d
    const bool scale = j < i;
    const uint32_t kib = s_base + R_KI + j * 2048;
    const float *G = gij + (i * 4 + j) * 64;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t af[4], bf[4];
      ldsm_x4(a_frag_addr(s_base + (mat ? R_QS : R_KS), 16 * i, 16 * kk, lane), af);
      if (scale) {
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          const float2 v = unpack_bf16(af[x]);
          const float2 gg = *reinterpret_cast<const float2 *>(G + 16 * kk + (x >> 1) * 8 + 2 * c4);
          af[x] = pack_bf16(v.x * gg.x, v.y * gg.y);
        }
      }
      ldsm_x4(bnk_frag_addr(kib, 0, 16 * kk, lane), bf);
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
          v0 = s < t ? v0 : 0.f;
          v1 = s + 1 < t ? v1 : 0.f;
          *reinterpret_cast<uint32_t *>(sm + R_MK + sw64(t, s)) = pack_bf16(v0, v1);
          v0 *= bet[t];
          v1 *= bet[t];
          if (j == i) {
            *reinterpret_cast<float2 *>(AD + i * 256 + tl * 16 + sl) = make_float2(v0, v1);
          } else {
            *reinterpret_cast<uint32_t *>(sm + R_AB + sw64(t, s)) = pack_bf16(v0, v1);
          }
        } else {
          v0 = s <= t ? v0 : 0.f;
          v1 = s + 1 <= t ? v1 : 0.f;
          *reinterpret_cast<uint32_t *>(hom + HO_P + sw64(t, s)) = pack_bf16(v0, v1);
        }
      }
  };
  // task q < 10: P block number q of the 10 pairs (i, j <= i); else off-diagonal M block q - 10
  auto mp_task = [&](int q) {
    const int pr = q < 10 ? q : (q == 10 ? 1 : q == 11 ? 3 : q == 12 ? 4 : q - 7);
    const int i = pr < 1 ? 0 : pr < 3 ? 1 : pr < 6 ? 2 : 3;
    const int j = pr - i * (i + 1) / 2;
    if (big && j == i && q < 10) return;  // diagonal block already computed exactly
    mp_block(q < 10 ? 1 : 0, i, j);
  };
  if (warp < 4) {
    const int i = warp;
    if (!big) mp_block(0, i, i);  // (a big chunk's diagonal blocks are already exact)
    __syncwarp();
    if (lane < 16) {
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
      __nv_bfloat16 *Ti = reinterpret_cast<__nv_bfloat16 *>(sm + R_TI + i * 512);
#pragma unroll
      for (int t = 0; t < 16; ++t) Ti[t * 16 + u] = __float2bfloat16_rn(x[t]);
    }
    mp_task(12 + warp);
  } else {
    for (int q = warp - 4; q < 12; q += 4) mp_task(q);
  }
  __syncthreads();
  CHUNK_TR(5);

  // ---- (4) Tinv = (I+A)^{-1} (into the Kdec tile): block forward substitution on the identity,
  //      8 columns per warp (the rows above a column's diagonal block are zero and skipped) ----
  solve_columns(sm, s_base, warp * 8, warp >> 1, warp, lane);
  __syncthreads();
  CHUNK_TR(6);
  // ---- (5) W = Tinv beta Kd (stored negated) and U = Tinv beta V as one block-triangular GEMM;
  //      warp w takes 16 of the 128 columns of [W | U] for all four row blocks ----
  {
    const int c0 = 16 * (warp & 3);
    const bool isW = warp < 4;
    const uint32_t xb = s_base + (isW ? R_XK : R_VS);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float acc[2][4] = {};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (k > i) break;
        uint32_t af[4], bf[4];
        ldsm_x4(a_frag_addr(s_base + R_KS, 16 * i, 16 * k, lane), af);
        ldsm_x4_t(bkn_frag_addr(xb, 16 * k, c0, lane), bf);
        mma16816(acc[0], af, bf[0], bf[1]);
        mma16816(acc[1], af, bf[2], bf[3]);
      }
      const float so = isW ? -1.f : 1.f;  // -W [t][d], U [t][j]
      uint8_t *Y = hom + (isW ? HO_W : HO_U);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
          *reinterpret_cast<uint32_t *>(Y + sw64(16 * i + g4 + 8 * hh, c0 + 8 * nt + 2 * c4)) =
              pack_bf16(so * acc[nt][2 * hh], so * acc[nt][2 * hh + 1]);
    }
  }
  __syncthreads();
  CHUNK_TR(7);
  // ---- (6) the state-independent products the scan and the backward need, 16 tasks of 16 rows
  //      x 64 columns, two per warp:
  //        [Mneg | N]       = Kb^T [-W | U]          (tasks 0-7, rows d)
  //        [Qt | O_intra]   = [Qd | 0] + P [-W | U]  (tasks 8-15, rows t; P is lower triangular)
  //      so that the scan advances S^T <- diag(e^{gamma_C}) S^T + Mneg S^T + N with one MMA per
  //      chunk and forms O = Qt S^T + O_intra and Unew = U - W S^T beside it ----
#pragma unroll 1
  for (int r = 0; r < 2; ++r) {
    const int q = warp + 8 * r;
    const int rb = (q >> 1) & 3, jb = rb * 16, nh = q & 1;
    const uint32_t bsrc = ho + (nh ? HO_U : HO_W);
    float X[8][4];
    if (q >= 8 && nh == 0) {  // Qt starts from Qd
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const float2 v = unpack_bf16(*reinterpret_cast<const uint32_t *>(
              hom + HO_QD + sw64(jb + g4 + 8 * hh, nt * 8 + 2 * c4)));
          X[nt][2 * hh] = v.x;
          X[nt][2 * hh + 1] = v.y;
        }
    } else {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) X[nt][e] = 0.f;
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      if (q >= 8 && kk > rb) break;
      uint32_t af[4];
      if (q < 8)
        ldsm_x4_t(ct_frag_addr(s_base + R_KB, 16 * kk, jb, lane), af);  // Kb^T rows d, k = t
      else
        ldsm_x4(a_frag_addr(ho + HO_P, jb, 16 * kk, lane), af);          // P rows t, k = s
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bf[4];
        ldsm_x4_t(bkn_frag_addr(bsrc, 16 * kk, 16 * np, lane), bf);
        mma16816(X[2 * np], af, bf[0], bf[1]);
        mma16816(X[2 * np + 1], af, bf[2], bf[3]);
      }
    }
    // staged in tiles that are free by now: Mneg -> beta-Kd, N -> Qdec, Qt -> beta-V, O_intra -> A
    uint8_t *dst = sm + (q < 8 ? (nh ? R_QS : R_XK) : (nh ? R_AB : R_VS));
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh)
        *reinterpret_cast<uint32_t *>(dst + sw64(jb + g4 + 8 * hh, nt * 8 + 2 * c4)) =
            pack_bf16(X[nt][2 * hh], X[nt][2 * hh + 1]);
  }
  fence_proxy_async_smem();  // make this thread's smem writes visible to the bulk copies
  __syncthreads();
  CHUNK_TR(8);
  // ---- the scan's record (ws) and, for training, the backward's record (saved): bulk copies
  //      of the swizzled tiles as they lie in shared memory ----
  if (tid == 0) {
    uint8_t *wr = (uint8_t *)p.ws + (int64_t)idx * WS_SIZE;
    const uint64_t keep = l2_policy_keep(), stream = l2_policy_stream();
    bulk_s2g_hint(wr + WS_W, ho + HO_W, 2 * 8192, keep);          // -W | U
    bulk_s2g_hint(wr + WS_OI, s_base + R_AB, 8192, keep);         // O_intra
    bulk_s2g_hint(wr + WS_N, s_base + R_QS, 8192, keep);          // N
    if (p.saved) {  // Mneg, Qt and e^{gamma_C} live in the saved record, where the scan reads them
      uint8_t *sv = (uint8_t *)p.saved + (int64_t)idx * kSavedChunk;
      bulk_s2g_hint(sv + kSavedM, s_base + R_XK, 8192, keep);
      bulk_s2g_hint(sv + kSavedQt, s_base + R_VS, 8192, keep);
      bulk_s2g_hint(sv + kSavedEG, ho + HO_EG, 256, keep);
      bulk_s2g_hint(sv + kSavedP, ho + HO_P, 8192, stream);
      bulk_s2g_hint(sv + kSavedMkk, s_base + R_MK, 8192, stream);   // M
      bulk_s2g_hint(sv + kSavedTinv, s_base + R_KS, 8192, stream);  // Tinv
    } else {
      bulk_s2g_hint(wr + WS_MN, s_base + R_XK, 8192, keep);
      bulk_s2g_hint(wr + WS_QT, s_base + R_VS, 8192, keep);
      bulk_s2g_hint(wr + WS_EG, ho + HO_EG, 256, keep);
    }
    bulk_commit();
    bulk_wait_read_all();  // shared memory stays valid until the stores have read it
  }
}

// ---------------------------------------------------------------------------------------
// kda_fwd_scan
// ---------------------------------------------------------------------------------------
// One CTA per (b, h) walks the chunks in order.  The state recurrence of a chunk is linear in
// the state, with every other term precomputed by the chunk kernel:
//     S^T <- diag(e^{gamma_C}) S^T + Mneg S^T + N          (Mneg = -Kb^T W, N = Kb^T U)
// so only ONE tcgen05 MMA (Mneg S^T, K = 64) lies on the chain from one chunk's state to the
// next; the fp32 state stays in registers (the diagonal decay is applied there exactly) and a
// bf16 copy of S^T is the MMA's B operand.  The outputs come off the chain:
//     O = Qt S^T + O_intra,   Unew = U - W S^T             (Qt = Qd - P W, O_intra = P U)
// Per chunk two MMAs read S^T: MMA1 = [Mneg; -W] S^T into accumulator D1 (rows 0-63 the state
// product, rows 64-127 -W S^T) and MMA2 = [-W; Qt] S^T into D2 (rows 64-127 Qt S^T; rows 0-63
// repeat -W S^T and are not read).  NB = 3 sets of both accumulators rotate in TMEM (512 columns
// allocated), so the output roles may finish a chunk up to two chunks behind the state chain.
// Warp roles (a warp reaches TMEM lanes 32 (warp % 4) ..):
//   warps 0, 1, 4, 5  state rows d (lanes 0-63 of D1), warps 0-1 columns 0-31, warps 4-5
//              columns 32-63: S <- D1 + e^{gamma_C} S + N, bf16 S^T tile for the next MMA;
//              thread 0 then issues the next chunk's MMA1 itself (no hand-off on the chain);
//   warps 2-3, 10-11  Unew rows t (training only): D1 rows 64-127 + U, columns 0-31 / 32-63;
//   warps 6-7, 14-15  O rows t: D2 rows 64-127 + O_intra, columns 0-31 / 32-63;
//              each of these two roles keeps a ring of NIO tiles: one thread bulk-loads the
//              chunk's U / O_intra tile NIO - 1 chunks ahead, every thread adds its TMEM row in
//              place, and the tile then leaves by a bulk / TMA store;
//   warp 8     one thread issues MMA2 as soon as thread 0 hands a chunk over (go2) and stores
//              S^T (the saved chunk-entry state) from its tile;
//   warp 9     one thread keeps the ring of chunk operands (Mneg, -W, Qt, N, e^{gamma_C}: bulk
//              copies) NREC chunks deep, refilling a slot once the MMAs that read it are done.
//
// Every wait is bounded; a role that gives up raises `abort`, which the others poll, and the
// teardown drains copies, MMAs and stores before TMEM is freed.
constexpr int NT2 = 512;                       // warps 9, 12, 13 have no role
constexpr int NREC = 4;                        // ring of chunk operand slots
constexpr int R_MN = 0, R_W = 8192, R_QT = 16384, R_N = 24576, R_EG = 32768;
constexpr int SLOT_BYTES = 32768 + 256;        // what one slot's copies bring
constexpr int SLOT = 33 * 1024;                // slot stride (1024-byte aligned)
constexpr int NB = 3;                          // TMEM accumulator sets (D1, D2) in flight
constexpr int NST = NB + 2;                    // bf16 S^T tiles (MMA B operand, saved-record staging)
constexpr int NIO = 3;                         // U -> Unew and O_intra -> O tiles per role
constexpr int OFF2_REC = 0;
constexpr int OFF2_ST = OFF2_REC + NREC * SLOT;   // NST x 8 KB
constexpr int OFF2_UN = OFF2_ST + NST * 8192;     // NIO x 8 KB
constexpr int OFF2_O = OFF2_UN + NIO * 8192;      // NIO x 8 KB
constexpr int OFF2_MBAR = OFF2_O + NIO * 8192;    // mrec[NREC] sfree[NREC] mA[NB] mB[NB] done[NB] io[2][NIO] go2[NB], TMEM slot, abort
constexpr int NMBAR2 = 2 * NREC + 4 * NB + 2 * NIO;
constexpr int SMEM2 = OFF2_MBAR + 8 * NMBAR2 + 16;
constexpr uint32_t kIdescScan = idesc_bf16(128, 64, 0, 1);  // A K-major, B MN-major

// 32 fp32 values -> columns c0 .. c0 + 31 of a row of a swizzled bf16 tile
__device__ __forceinline__ void store_half_row_bf16(uint8_t *tile, int row, int c0, const float *x) {
#pragma unroll
  for (int ch = 0; ch < 4; ++ch)
    *reinterpret_cast<uint4 *>(tile + sw64(row, c0 + ch * 8)) =
        make_uint4(pack_bf16(x[8 * ch], x[8 * ch + 1]), pack_bf16(x[8 * ch + 2], x[8 * ch + 3]),
                   pack_bf16(x[8 * ch + 4], x[8 * ch + 5]), pack_bf16(x[8 * ch + 6], x[8 * ch + 7]));
}
__global__ void __launch_bounds__(NT2, 1) kda_fwd_scan_kernel(Params p, const __grid_constant__ TmaMaps tm) {
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.x, b = bh / p.H, h = bh % p.H;
  const int nc = p.nc;
  const uint32_t s_base = smem_u32(sm);
  if (s_base & 1023) {  // swizzled tiles need a 1024-byte aligned base
    if (tid == 0) atomicExch(&g_fwd_status, KDA_ERR_MISALIGNED);
    return;
  }
  const uint32_t mrec = s_base + OFF2_MBAR, sfree = mrec + 8 * NREC, mA = sfree + 8 * NREC, mB = mA + 8 * NB,
                 done = mB + 8 * NB, mio = done + 8 * NB, go2 = mio + 16 * NIO;
  uint32_t *tslot = reinterpret_cast<uint32_t *>(sm + OFF2_MBAR + 8 * NMBAR2);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(sm + OFF2_MBAR + 8 * NMBAR2 + 4);
  const bool leader = tid == 256;
  const bool state_warp = warp == 0 || warp == 1 || warp == 4 || warp == 5;
  const int d = 32 * (warp & 1) + lane;   // state warps: row d of S^T
  const int half = warp >= 4 ? 32 : 0;    // state warps: first column of their half
  // per-chunk sources: -W, U, O_intra, N in the workspace; Mneg, Qt, e^{gamma_C} in the saved
  // record when there is one, else in the workspace
  const uint8_t *wsb = (const uint8_t *)p.ws + (int64_t)bh * nc * WS_SIZE;
  const uint8_t *svb = p.saved ? (const uint8_t *)p.saved + (int64_t)bh * nc * kSavedChunk : nullptr;
  auto rec_ws = [&](int c) { return wsb + (int64_t)c * WS_SIZE; };
  auto mq_src = [&](int c, int which) -> const uint8_t * {  // which: 0 Mneg, 1 Qt, 2 e^{gamma_C}
    if (svb) return svb + (int64_t)c * kSavedChunk + (which == 0 ? kSavedM : which == 1 ? kSavedQt : kSavedEG);
    return rec_ws(c) + (which == 0 ? WS_MN : which == 1 ? WS_QT : WS_EG);
  };

  if (leader) {
    for (int i = 0; i < NREC; ++i) {
      mbar_init(mrec + 8 * i, 1);
      mbar_init(sfree + 8 * i, 1);
    }
    for (int i = 0; i < NB; ++i) {
      mbar_init(mA + 8 * i, 1);
      mbar_init(mB + 8 * i, 1);
      mbar_init(done + 8 * i, 256);
      mbar_init(go2 + 8 * i, 1);
    }
    for (int i = 0; i < 2 * NIO; ++i) mbar_init(mio + 8 * i, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (p.debug_wait_polls > 0) {  // test hook: a bounded wait on a barrier nothing completes,
    __syncthreads();             // entered before any copy is issued or tensor memory is held
    const bool ok = !leader || mbar_wait(mA, 0, p.debug_wait_polls);
    if (__syncthreads_or(!ok)) {
      if (leader) atomicExch(&g_fwd_status, KDA_ERR_TIMEOUT);
      return;
    }
  }
  float S[32];  // state warps: S^T[d][half + j] = S[half + j][d]
  if (state_warp) {
#pragma unroll
    for (int j = 0; j < 32; ++j) S[j] = p.state0 ? p.state0[(int64_t)bh * D * D + (half + j) * D + d] : 0.f;
    store_half_row_bf16(sm + OFF2_ST, d, half, S);
  }
  if (warp == 8) {
    tmem_alloc(smem_u32(tslot), 512);
    tmem_relinquish();
  }
  fence_proxy_async_smem();  // the S^T tile is read by the tensor cores
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tD = *tslot;
  const uint32_t lq = (uint32_t)(32 * (warp & 3)) << 16;  // this warp's TMEM lane quarter
  bool failed = false;
  // MMA1 of chunk c (thread 0, on the chain): D1[c % NB] = [Mneg; -W] S^T(c); then thread 0 hands
  // chunk c to the leader (go2), which issues MMA2: D2[c % NB] = [-W; Qt] S^T(c).  TMEM columns:
  // D1[i] at 64 i, D2[i] at 64 (NB + i)
  auto issue_mma1 = [&](int c) {
    const int bb = c % NB;
    const uint32_t st = s_base + OFF2_ST + (c % NST) * 8192, rec = s_base + OFF2_REC + (c % NREC) * SLOT;
    tc_fence_after();
    SCAN_TR(2, c - 1);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      tc_mma(tD + 64 * bb, desc_k(rec + R_MN, k), desc_mn(st, k), kIdescScan, k > 0);
      if (k == 0) SCAN_TR(3, c - 1);
    }
    tc_commit(mA + 8 * bb);
    SCAN_TR(16, c - 1);
    mbar_arrive(go2 + 8 * bb);
  };
  if (leader) {
    // ---- MMA2 of every chunk, issued as soon as thread 0 hands the chunk over (go2 follows
    //      MMA1(c), which thread 0 issued after chunk c's operands were seen to land), so that
    //      the tensor pipe runs it while the state rows are updated, not after the next MMA1 ----
    for (int c = 0; c < nc; ++c) {
      const int bb = c % NB;
      const bool ok = mbar_wait_spin(go2 + 8 * bb, (c / NB) & 1);
      SCAN_TR(6, c);
      if (!ok || *abort_flag) {
        failed = true;
        *abort_flag = 1;
        break;
      }
      const uint32_t st = s_base + OFF2_ST + (c % NST) * 8192, rec = s_base + OFF2_REC + (c % NREC) * SLOT;
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < 4; ++k) tc_mma(tD + 64 * (NB + bb), desc_k(rec + R_W, k), desc_mn(st, k), kIdescScan, k > 0);
      tc_commit(mB + 8 * bb);
      if (p.saved) {  // S^T(c), the chunk-entry state of the saved record
        bulk_s2g((uint8_t *)svb + (int64_t)c * kSavedChunk + kSavedS0, st, 8192);
        bulk_commit();
        bulk_wait_read<1>();  // S^T(c - 1)'s store has read its tile (see the state warps)
      }
      SCAN_TR(7, c);
    }
  } else if (tid == 288) {
    // ---- the operand ring: a slot is refilled once both MMAs of its chunk are complete and the
    //      state warps have read it (thread 0 commits the next chunk's MMA1 to sfree[slot]) ----
    int issued = 0;
    auto issue = [&](int c) {
      const int s = c % NREC;
      const uint32_t dst = s_base + OFF2_REC + s * SLOT, mb = mrec + 8 * s;
      mbar_expect_tx(mb, SLOT_BYTES);
      bulk_g2s(dst + R_MN, mq_src(c, 0), 8192, mb);
      bulk_g2s(dst + R_W, rec_ws(c) + WS_W, 8192, mb);
      bulk_g2s(dst + R_QT, mq_src(c, 1), 8192, mb);
      bulk_g2s(dst + R_N, rec_ws(c) + WS_N, 8192, mb);
      bulk_g2s(dst + R_EG, mq_src(c, 2), 256, mb);
      issued = c + 1;
    };
    for (int c = 0; c < nc && c < NREC; ++c) issue(c);
    for (int c = 0; c + NREC < nc; ++c) {
      const bool ok = mbar_wait(mB + 8 * (c % NB), (c / NB) & 1) && mbar_wait(sfree + 8 * (c % NREC), (c / NREC) & 1);
      if (!ok || *abort_flag) {
        failed = true;
        *abort_flag = 1;
        break;
      }
      issue(c + NREC);
    }
    if (*abort_flag)  // (bounded) the last copy issued into each slot lands before the CTA exits
      for (int c = issued > NREC ? issued - NREC : 0; c < issued; ++c) mbar_wait(mrec + 8 * (c % NREC), (c / NREC) & 1);
  } else if (state_warp) {
    // ---- state rows: S <- D1 + e^{gamma_C} S + N, 32 columns per thread ----
    // One thread per condition waits and the named-barrier vote passes the outcome on: thread 0
    // polls MMA1(c) (the chain), thread 32 the barriers MMA1(c + 1) needs besides S^T(c + 1).
    {
      const bool ok0 = tid != 0 || mbar_wait(mrec, 0);  // chunk 0's operands
      if (!bar_and(1, 128, ok0)) {
        failed = true;
        *abort_flag = 1;
      } else if (tid == 0) {
        issue_mma1(0);
      }
    }
    for (int c = 0; c < nc && !failed; ++c) {
      const int bb = c % NB, s = c % NREC;
      const uint8_t *recm = sm + OFF2_REC + s * SLOT;
      // e^{gamma_C} S + N while MMA1(c) runs: chunk c's operands are in (vote of the step before)
      {
        const float e = reinterpret_cast<const float *>(recm + R_EG)[d];
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          const uint4 nw = *reinterpret_cast<const uint4 *>(recm + R_N + sw64(d, half + 8 * ch));
          const uint32_t u[4] = {nw.x, nw.y, nw.z, nw.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = unpack_bf16(u[q]);
            const int j = 8 * ch + 2 * q;
            S[j] = fmaf(e, S[j], f.x);
            S[j + 1] = fmaf(e, S[j + 1], f.y);
          }
        }
      }
      bool ok = true;
      if (tid == 32 && c + 1 < nc) {
        // D1 / D2[(c + 1) % NB] (chunk c + 1 - NB) are drained.  This also frees the tile of
        // S^T(c + 1), which last held S^T(c + 1 - NST) = S^T(c - 1 - NB): the leader saw that
        // state's saved-record store read its tile before it issued MMA2(c + 1 - NB), and
        // done(c + 1 - NB) follows MMA2(c + 1 - NB).  And chunk c + 1's operands have landed.
        if (c + 1 >= NB) ok = mbar_wait(done + 8 * ((c + 1) % NB), ((c + 1 - NB) / NB) & 1);
        ok = ok && mbar_wait(mrec + 8 * ((c + 1) % NREC), ((c + 1) / NREC) & 1);
      }
      if (tid == 0) ok = mbar_wait_spin(mA + 8 * bb, (c / NB) & 1);
      if (!bar_and(1, 128, ok && !*abort_flag)) {
        failed = true;
        *abort_flag = 1;
        break;
      }
      if (tid == 0) SCAN_TR(0, c);
      tc_fence_after();
      {
        uint32_t v[32];
        tmem_ld32(tD + 64 * bb + lq + half, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) S[j] += __uint_as_float(v[j]);
      }
      if (tid == 0) SCAN_TR(1, c);
      if (c + 1 < nc) {
        store_half_row_bf16(sm + OFF2_ST + ((c + 1) % NST) * 8192, d, half, S);
        fence_proxy_async_smem();
        tc_fence_before();
        bar_sync(1, 128);
        if (tid == 0) {
          SCAN_TR(4, c);
          issue_mma1(c + 1);
          tc_commit(sfree + 8 * s);  // slot s (chunk c) is free once MMA1(c + 1) completes
          SCAN_TR(5, c);
        }
      }
    }
    if (!failed) {
#pragma unroll
      for (int j = 0; j < 32; ++j) p.stateT[(int64_t)bh * D * D + (half + j) * D + d] = S[j];
    }
  } else if ((warp & 3) >= 2) {
    // ---- warps 2-3, 10-11: Unew rows (training); warps 6-7, 14-15: O rows ----
    const bool un = (warp & 4) == 0;
    const int t = 32 * (warp & 1) + lane, bar = un ? 2 : 3, c0 = warp >= 8 ? 32 : 0;
    const bool lead = t == 0 && c0 == 0;
    const uint32_t macc = un ? mA : mB, tcol = un ? 0 : 64 * NB, mb0 = mio + (un ? 0 : 8 * NIO);
    const int src_off = un ? WS_U : WS_OI;
    const int ring = un ? OFF2_UN : OFF2_O;
    const bool active = !un || p.saved;
    int io_issued = 0;
    auto load_tile = [&](int c) {
      const int s = c % NIO;
      io_issued = c + 1;
      mbar_expect_tx(mb0 + 8 * s, 8192);
      bulk_g2s(s_base + ring + s * 8192, rec_ws(c) + src_off, 8192, mb0 + 8 * s);
    };
    if (active && lead)
      for (int c = 0; c < nc && c < NIO - 1; ++c) load_tile(c);
    for (int c = 0; c < nc; ++c) {
      const int bb = c % NB, s = c % NIO;
      // the lead thread waits, the vote passes the outcome on
      const bool ok = !lead || (mbar_wait(macc + 8 * bb, (c / NB) & 1) && (!active || mbar_wait(mb0 + 8 * s, (c / NIO) & 1)));
      if (lead) SCAN_TR(un ? 8 : 10, c);
      if (!bar_and(bar, 128, ok && !*abort_flag)) {
        failed = true;
        *abort_flag = 1;
        if (lead)  // (bounded) the last tile load issued into each slot lands before the CTA exits
          for (int c2 = io_issued > NIO ? io_issued - NIO : 0; c2 < io_issued; ++c2)
            mbar_wait(mb0 + 8 * (c2 % NIO), (c2 / NIO) & 1);
        break;
      }
      tc_fence_after();
      if (active) {
        // + this thread's half row of U / O_intra, written back in place: its four 16-byte
        // pieces are all read (while the TMEM load runs) before any is written
        uint8_t *tile = sm + ring + s * 8192;
        uint32_t v[32];
        tmem_ld32(tD + tcol + 64 * bb + lq + c0, v);
        uint4 u[4];
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) u[ch] = *reinterpret_cast<const uint4 *>(tile + sw64(t, c0 + 8 * ch));
        tmem_wait_ld();
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          const uint32_t uw[4] = {u[ch].x, u[ch].y, u[ch].z, u[ch].w};
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = 8 * ch + 2 * e;
            const float2 f = unpack_bf16(uw[e]);
            o[e] = pack_bf16(__uint_as_float(v[j]) + f.x, __uint_as_float(v[j + 1]) + f.y);
          }
          u[ch] = make_uint4(o[0], o[1], o[2], o[3]);
        }
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) *reinterpret_cast<uint4 *>(tile + sw64(t, c0 + 8 * ch)) = u[ch];
        if (lead) SCAN_TR(un ? 12 : 14, c);
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(done + 8 * bb);
        if (lead) SCAN_TR(un ? 9 : 11, c);
        bar_sync(bar, 128);
        if (lead) {
          const uint32_t src = s_base + ring + s * 8192;
          if (un)
            bulk_s2g((uint8_t *)svb + (int64_t)c * kSavedChunk + kSavedUnT, src, 8192);
          else
            tma_store_rows(&tm.m[0], src, h, c * C, b);  // rows past T are dropped
          bulk_commit();
          // refill the tile of chunk c - 1 with chunk c - 1 + NIO once its store has read it
          if (c + NIO - 1 < nc) {
            bulk_wait_read<1>();
            load_tile(c + NIO - 1);
          }
          SCAN_TR(un ? 13 : 15, c);
        }
      } else {
        tc_fence_before();
        mbar_arrive(done + 8 * bb);
      }
    }
  }
  const bool storer = leader || tid == 64 || tid == 192;  // threads that issue bulk stores
  if (failed && (tid == 288 || storer)) atomicExch(&g_fwd_status, KDA_ERR_TIMEOUT);
  if (storer) bulk_wait_all();  // the stores this thread issued have completed
  if (tid == 0 && *abort_flag) {  // (bounded) no MMA may still write TMEM when it is freed
    for (int i = 0; i < NB; ++i) {
      mbar_wait(mA + 8 * i, 0);
      mbar_wait(mA + 8 * i, 1);
      mbar_wait(mB + 8 * i, 0);
      mbar_wait(mB + 8 * i, 1);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 8) tmem_dealloc(tD, 512);
}

template <typename Tb>
int launch(const Params &p, cudaStream_t st) {
  auto k1 = kda_fwd_chunks_kernel<Tb>;
  if (cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM1) ||
      cudaFuncSetAttribute(k1, cudaFuncAttributePreferredSharedMemoryCarveout, 100))
    return KDA_ERR_CUDA;
  const int nchunks = p.B * p.H * p.nc;
  TmaMaps tm;
  const void *srcs[4] = {p.q, p.k, p.v, p.gated ? p.f : (const void *)p.g};
  const Str in_str[4] = {p.sq, p.sk, p.sv, p.sg};
  for (int i = 0; i < 4; ++i)
    if (int e = tma_map_bthd(&tm.m[i], srcs[i], p.B, p.T, p.H, D, i == 3 && !p.gated, &in_str[i])) return e;
  k1<<<nchunks, NT1, SMEM1, st>>>(p, tm);
  count_launch();
  if (cudaFuncSetAttribute(kda_fwd_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2))
    return KDA_ERR_CUDA;
  TmaMaps to;
  if (int e = tma_map_bthd(&to.m[0], p.o, p.B, p.T, p.H, D, false)) return e;
  kda_fwd_scan_kernel<<<p.B * p.H, NT2, SMEM2, st>>>(p, to);
  count_launch();
  return cudaPeekAtLastError() == cudaSuccess ? KDA_OK : KDA_ERR_CUDA;
}

}  // namespace tcfwd


int tc_fwd_device_status(bool reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, tcfwd::g_fwd_status, sizeof(int)) != cudaSuccess) return KDA_ERR_CUDA;
  if (reset && v) {
    const int z = 0;
    if (cudaMemcpyToSymbol(tcfwd::g_fwd_status, &z, sizeof(int)) != cudaSuccess) return KDA_ERR_CUDA;
  }
  return v;
}

size_t tc_fwd_workspace_bytes(const KdaDesc *d) {
  return (size_t)(d->B * d->H * ((d->T + d->chunk - 1) / d->chunk)) * tcfwd::WS_SIZE;
}

int tc_fwd(const Params &p, int dtype_beta, cudaStream_t st) {
  if (dtype_beta == KDA_BF16) return tcfwd::launch<__nv_bfloat16>(p, st);
  if (dtype_beta == KDA_F32) return tcfwd::launch<float>(p, st);
  return KDA_ERR_DTYPE;
}

}  // namespace kda

#ifdef KDA_SCAN_TRACE
extern "C" __attribute__((visibility("default"))) int kda_chunk_trace(long long *out) {
  return cudaMemcpyFromSymbol(out, kda::tcfwd::g_chunk_trace, sizeof(long long) * 12 * 64) == cudaSuccess ? 0 : -1;
}
extern "C" __attribute__((visibility("default"))) int kda_scan_trace(long long *out) {
  return cudaMemcpyFromSymbol(out, kda::tcfwd::g_scan_trace, sizeof(long long) * 20 * 64) == cudaSuccess ? 0 : -1;
}
#endif
