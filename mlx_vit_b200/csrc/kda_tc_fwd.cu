// Tensor-core KDA forward for D = 64, chunk = 64, bf16 q/k/v, in two kernels.
//
//  kda_fwd_chunks  one persistent CTA per SM walking all (b, h, chunk), which are independent:
//                  every state-independent quantity of the chunk, written as a per-chunk record
//                  (-W, U, Qd, Kb, P as bf16 tiles, e^{gamma_C}) to the forward workspace,
//                  and, for training, the state-independent part of the backward's record
//                  (P, M, Tinv = (I+A)^{-1}, Mneg = -Kb^T W, Qt = Qd - P W).
//  kda_fwd_scan    one CTA of 5 warps per (b, h): streams the chunk records (bulk copies, two
//                  chunks ahead) and advances the state with two tcgen05 MMAs per chunk into one
//                  M = 128 TMEM accumulator (the fp32 state itself stays in registers):
//                    Unew = U - W S^T;  O = Qd S^T + P Unew;  S^T <- diag(e^{gamma_C}) S^T + Kb^T Unew
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

constexpr int C = 64, D = 64;
constexpr float kSpanMax = 60.f;

// per-chunk record handed from kda_fwd_chunks to kda_fwd_scan (bf16 tiles, swizzled): Qd [t][d]
// and -W [t][d] (together the 128-row A operand of the scan's first MMA), U [t][j], P [t][s]
// (zero above the diagonal) and Kb^T [d][t] (together the A operand of its second MMA), and
// e^{gamma_C} (fp32)
constexpr int HO_QD = 0, HO_W = 8192, HO_U = 16384, HO_P = 24576, HO_KBT = 32768, HO_EG = 40960;
constexpr int HO_SIZE = 40960 + 256;

// ---------------------------------------------------------------------------------------
// kda_fwd_chunks
// ---------------------------------------------------------------------------------------
constexpr int NT1 = 512;  // 16 warps: every phase splits into more independent pieces
constexpr int OFF_QS = 0;                                // raw q/k/v tiles (TMA, 128-byte swizzle,
constexpr int OFF_KS = OFF_QS + 8192;                    //   1024-byte aligned)
constexpr int OFF_VS = OFF_KS + 8192;
constexpr int OFF_GS = OFF_VS + 8192;                    // g (TMA) -> gamma (fp32, gsw layout) 16 KB
constexpr int OFF_OUT = OFF_GS + 16384;                  // the record, swizzled tiles
constexpr int OFF_KD = OFF_OUT + HO_SIZE;                // Kdec
constexpr int OFF_QD = OFF_KD + 8192;                    // Qdec
constexpr int OFF_KI = OFF_QD + 8192;                    // Kinc, 10 tiles of 16x64
constexpr int OFF_AB = OFF_KI + 10 * 2048;               // A off-diagonal blocks (bf16)
constexpr int OFF_AD = OFF_AB + 8192;                    // A diagonal blocks fp32 4x16x16
constexpr int OFF_TI = OFF_AD + 4096;                    // T_ii bf16 4x16x16
constexpr int OFF_XK = OFF_TI + 2048;                    // beta Kd
constexpr int OFF_XV = OFF_XK + 8192;                    // beta V
constexpr int OFF_MK = OFF_XV + 8192;                    // M = Kdec Kinc^T strict lower (bf16)
constexpr int OFF_TF = OFF_MK + 8192;                    // Tinv = (I + A)^{-1} (bf16), after OFF_MK
constexpr int OFF_KBS = OFF_TF + 8192;                   // Kb [t][d] (bf16)
constexpr int OFF_RS = OFF_KBS + 8192;                   // per-warp 16x16 staging
constexpr int OFF_VEC = OFF_RS + 16 * 256;
// vectors (floats): bet[64] refs[4][64] part[8][64] erb[4][64] egr[4][64] gij[16][64] flag[4]
constexpr int V_BET = 0, V_REFS = 64, V_PART = 320, V_ERB = 832, V_EGR = 1088, V_G = 1344,
              V_FLAG = 2368;
constexpr int OFF_MBAR1 = OFF_VEC + (2368 + 4) * 4;      // mbarrier of the TMA loads
constexpr int SMEM1 = OFF_MBAR1 + 8;
// fused gates only: the raw f tile (TMA, bf16), then the staged gate parameters
constexpr int OFF_FS1 = (SMEM1 + 1023) & ~1023;
constexpr int SMEM1_GP = OFF_FS1 + 8192;

__device__ __forceinline__ int ki_index(int i, int j) { return i * (i + 1) / 2 + j; }

// Block forward substitution Y = (I+A)^{-1} X for the 8 columns n0..n0+7, by one warp:
//   Y_i = T_ii (X_i - sum_{j<i} A_ij Y_j),  i = ib..3  (rows of blocks below ib are zero).
// Y is a swizzled tile at byte offset y_off from OFF_OUT, stored as so * Y; the stored values
// of earlier blocks are read back with the sign sg = -so.  X is a swizzled tile at x_off, or the
// identity when x_off < 0 (Y is then Tinv).
__device__ __forceinline__ void solve_columns(uint8_t *sm, uint32_t s_base, int y_off, int x_off, int n0,
                                              int ib, float sg, float so, int warp, int lane) {
  const int g4 = lane >> 2, c4 = lane & 3, l15 = lane & 15;
  const uint32_t Yb = s_base + OFF_OUT + y_off;
  uint8_t *Ym = sm + OFF_OUT + y_off;
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
    // R = X_i + sg * acc -> bf16 staging [t][col] 16x8
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int tl = g4 + 8 * hh, col = n0 + 2 * c4;
      float2 x;
      if (x_off >= 0) {
        x = unpack_bf16(*reinterpret_cast<const uint32_t *>(sm + x_off + sw64(16 * i + tl, col)));
      } else {
        x.x = 16 * i + tl == col ? 1.f : 0.f;
        x.y = 16 * i + tl == col + 1 ? 1.f : 0.f;
      }
      *reinterpret_cast<uint32_t *>(Rm + tl * 16 + c4 * 4) =
          pack_bf16(x.x + sg * acc[2 * hh], x.y + sg * acc[2 * hh + 1]);
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
      *reinterpret_cast<uint32_t *>(Ym + sw64(t, col)) = pack_bf16(so * y[2 * hh], so * y[2 * hh + 1]);
    }
    __syncwarp();
  }
}

template <typename Tb>
__global__ void __launch_bounds__(NT1, 1) kda_fwd_chunks_kernel(Params p, const __grid_constant__ TmaMaps tm) {
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g4 = lane >> 2, c4 = lane & 3;
  const int nc = p.nc, T = p.T, H = p.H, nchunks = p.B * p.H * nc;
  const uint32_t s_base = smem_u32(sm);
  if (s_base & 1023) {  // TMA tiles with the 128-byte swizzle need a 1024-byte aligned base
    if (tid == 0) atomicExch(&g_fwd_status, KDA_ERR_MISALIGNED);
    return;
  }
  float *GS = reinterpret_cast<float *>(sm + OFF_GS);
  float *AD = reinterpret_cast<float *>(sm + OFF_AD);
  float *vec = reinterpret_cast<float *>(sm + OFF_VEC);
  float *bet = vec + V_BET, *refs = vec + V_REFS, *part = vec + V_PART;
  float *erb = vec + V_ERB, *egr = vec + V_EGR, *gij = vec + V_G;
  int *flag = reinterpret_cast<int *>(vec + V_FLAG);
  uint8_t *hom = sm + OFF_OUT;
  const uint32_t ho = s_base + OFF_OUT;
  float *eG = reinterpret_cast<float *>(hom + HO_EG);
  const Tb *betag = (const Tb *)p.beta;

  // the CTA is persistent: it walks chunks idx = blockIdx.x, + gridDim.x, ...; the TMA loads of
  // the next chunk are issued as soon as this chunk's raw tiles are consumed
  const uint32_t mbar = s_base + OFF_MBAR1;
  if (tid == 0) {
    mbar_init(mbar, 1);
    mbar_fence_init();
  }
  const float *gA_log;
  const float *gdtb = stage_gate_params(reinterpret_cast<float *>(sm + SMEM1_GP), p, tid, NT1, &gA_log);
  __syncthreads();
  auto issue_loads = [&](int i) {  // q, k, v tiles (swizzled) and g (fp32) of chunk i
    if (tid == 0) {
      const int bh_ = i / nc, t0_ = (i % nc) * C, b_ = bh_ / H, h_ = bh_ % H;
      mbar_expect_tx(mbar, 3 * 8192 + (p.gated ? 8192 : 16384));
      tma_load_rows(s_base + OFF_QS, &tm.m[0], h_, t0_, b_, mbar);
      tma_load_rows(s_base + OFF_KS, &tm.m[1], h_, t0_, b_, mbar);
      tma_load_rows(s_base + OFF_VS, &tm.m[2], h_, t0_, b_, mbar);
      if (p.gated)  // the gate pre-activation f (bf16), converted into GS
        tma_load_rows(s_base + OFF_FS1, &tm.m[3], h_, t0_, b_, mbar);
      else
        tma_load_rows_f32(s_base + OFF_GS, &tm.m[3], h_, t0_, b_, mbar);
    }
  };
  // beta of the next chunk, kept raw until its use so that the load does not stall anyone
  auto load_beta = [&](int i) -> Tb {
    const int bh_ = i / nc, c_ = i % nc, t = c_ * C + tid;
    return t < T ? betag[((int64_t)(bh_ / H) * T + t) * H + bh_ % H] : from_f<Tb>(0.f);
  };
  // P's blocks above the diagonal are zero (the scan multiplies the whole tile); nothing else
  // writes them, so they are cleared once
  for (int u = tid; u < 192; u += NT1) {
    const int blk = u >> 5, r = (u >> 1) & 15, half = u & 1;
    const int i = blk < 3 ? 0 : blk < 5 ? 1 : 2, j = blk < 3 ? blk + 1 : blk < 5 ? blk - 1 : 3;
    *reinterpret_cast<uint4 *>(hom + HO_P + sw64(16 * i + r, 16 * j + 8 * half)) = make_uint4(0u, 0u, 0u, 0u);
  }
  int idx = blockIdx.x;
  if (idx < nchunks) issue_loads(idx);
  Tb beta_next = (idx < nchunks && tid < C) ? load_beta(idx) : from_f<Tb>(0.f);

  for (int it = 0; idx < nchunks; idx += gridDim.x, ++it) {
  if (__syncthreads_or(!mbar_wait(mbar, it & 1))) {  // this chunk's q, k, v, g
    if (tid == 0) atomicExch(&g_fwd_status, KDA_ERR_TIMEOUT);
    break;
  }
  const int nvalid = min(C, T - (idx % nc) * C);
  if (tid < C)
    bet[tid] = !p.gated ? to_f(beta_next) : tid < nvalid ? p.beta_scale * sigmoid_f(to_f(beta_next)) : 0.f;
  if (p.gated) gate_to_g(sm + OFF_FS1, GS, gA_log, gdtb, idx / nc % H, nvalid, tid, false);
  __syncthreads();

  // ---- (1a) gamma = cumsum(g): 8 segments of 8 rows per channel ----
  {
    const int d = tid & 63, seg = tid >> 6;
    float acc = 0.f;
#pragma unroll
    for (int r = 0; r < 8; ++r) acc += GS[gsw(seg * 8 + r, d)];
    part[seg * 64 + d] = acc;
    __syncthreads();
    float off = 0.f;
    for (int s2 = 0; s2 < seg; ++s2) off += part[s2 * 64 + d];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      off += GS[gsw(seg * 8 + r, d)];
      GS[gsw(seg * 8 + r, d)] = off;
    }
    __syncthreads();
  }
  // guard: factored decay stays within e^{kSpanMax} unless gamma moves more than that across
  // half a 16-row block.  Such a "big" chunk factors e^{gamma_t - gamma_s} (t in block i > j,
  // the block of s) as A_t G_ij B_s with A_t = e^{gamma_t - gamma(start of i)},
  // G_ij = e^{gamma(start of i) - gamma(end of j)}, B_s = e^{gamma(end of j) - gamma_s}, every
  // factor <= 1, and computes its diagonal blocks exactly.
  if (tid < 64) {
    float span = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      span = fmaxf(span, GS[gsw(i * 16, tid)] - GS[gsw(i * 16 + 8, tid)]);
      span = fmaxf(span, GS[gsw(i * 16 + 8, tid)] - GS[gsw(i * 16 + 15, tid)]);
    }
    const int any = __any_sync(0xffffffffu, !(span <= kSpanMax));
    if (lane == 0) flag[warp] = any;
  }
  // the previous chunk's bulk stores have read the record and staging tiles written from here on
  if (tid == 0) bulk_wait_read_all();
  __syncthreads();
  const bool big = flag[0] | flag[1];
  {  // per-block vectors, thread (slot, d): slot i < 4 -> block i's entries, slot 4 -> e^{gamma_C}
    const int d = tid & 63, slot = tid >> 6, ro = big ? 0 : 8;
    const float gC = GS[gsw(63, d)];
    if (slot < 4) {
      const int i = slot;
      const float ri = GS[gsw(i * 16 + ro, d)];
      refs[i * 64 + d] = ri;
      erb[i * 64 + d] = __expf(ri);
      egr[i * 64 + d] = __expf(gC - ri);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        gij[(i * 4 + j) * 64 + d] = j < i ? __expf(ri - GS[gsw(j * 16 + (big ? 15 : ro), d)]) : (j == i ? 1.f : 0.f);
    } else if (slot == 4) {
      eG[d] = __expf(gC);
    }
  }
  __syncthreads();

  // ---- (1b) operand build: 512 units of (row t, 8 consecutive channels) ----
  for (int u = tid; u < 512; u += NT1) {
    const int t = u >> 3, ch = u & 7, d0 = ch * 8, blk = t >> 4;
    const uint32_t off = sw64(t, d0);
    const uint4 kq = *reinterpret_cast<const uint4 *>(sm + OFF_KS + off);
    const uint4 qq = *reinterpret_cast<const uint4 *>(sm + OFF_QS + off);
    const uint4 vq = *reinterpret_cast<const uint4 *>(sm + OFF_VS + off);
    const uint32_t kw[4] = {kq.x, kq.y, kq.z, kq.w}, qw[4] = {qq.x, qq.y, qq.z, qq.w},
                   vw[4] = {vq.x, vq.y, vq.z, vq.w};
    const float bt = bet[t];
    const float4 ga4 = *reinterpret_cast<const float4 *>(GS + gsw(t, d0));
    const float4 gb4 = *reinterpret_cast<const float4 *>(GS + gsw(t, d0 + 4));
    const float gam[8] = {ga4.x, ga4.y, ga4.z, ga4.w, gb4.x, gb4.y, gb4.z, gb4.w};
    uint32_t okd[4], oqd[4], oxk[4], oxv[4], oqe[4], okb[4], oki[1][4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 kf = unpack_bf16(kw[e]), qf = unpack_bf16(qw[e]), vf = unpack_bf16(vw[e]);
      const int d = d0 + 2 * e;
      float F[2], iF[2], eg[2], eb[2];
      const float2 rf2 = *reinterpret_cast<const float2 *>(refs + blk * 64 + d);
      const float2 er2 = *reinterpret_cast<const float2 *>(erb + blk * 64 + d);
      const float2 eq2 = *reinterpret_cast<const float2 *>(egr + blk * 64 + d);
      const float rf[2] = {rf2.x, rf2.y}, er[2] = {er2.x, er2.y}, eq[2] = {eq2.x, eq2.y};
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const float gm = gam[2 * e + x];
        F[x] = __expf(gm - rf[x]);
        if (!big) {
          iF[x] = __fdividef(1.f, F[x]);
          eg[x] = F[x] * er[x];
          eb[x] = iF[x] * eq[x];
        } else {
          iF[x] = 0.f;
          eg[x] = __expf(gm);
          eb[x] = __expf(GS[gsw(63, d + x)] - gm);
        }
      }
      okd[e] = pack_bf16(kf.x * F[0], kf.y * F[1]);
      oqd[e] = pack_bf16(qf.x * F[0], qf.y * F[1]);
      oxk[e] = pack_bf16(bt * kf.x * eg[0], bt * kf.y * eg[1]);
      oqe[e] = pack_bf16(qf.x * eg[0], qf.y * eg[1]);
      oxv[e] = pack_bf16(bt * vf.x, bt * vf.y);
      okb[e] = pack_bf16(kf.x * eb[0], kf.y * eb[1]);
      if (!big) {  // Kinc of the diagonal block only: k / F (the GEMMs rescale it per block pair)
        oki[0][e] = pack_bf16(kf.x * iF[0], kf.y * iF[1]);
      } else {  // k B_s
        const float ge0 = GS[gsw(16 * blk + 15, d)], ge1 = GS[gsw(16 * blk + 15, d + 1)];
        oki[0][e] = pack_bf16(kf.x * __expf(ge0 - gam[2 * e]), kf.y * __expf(ge1 - gam[2 * e + 1]));
      }
    }
    *reinterpret_cast<uint4 *>(sm + OFF_KD + off) = make_uint4(okd[0], okd[1], okd[2], okd[3]);
    *reinterpret_cast<uint4 *>(sm + OFF_QD + off) = make_uint4(oqd[0], oqd[1], oqd[2], oqd[3]);
    *reinterpret_cast<uint4 *>(sm + OFF_XK + off) = make_uint4(oxk[0], oxk[1], oxk[2], oxk[3]);
    *reinterpret_cast<uint4 *>(sm + OFF_XV + off) = make_uint4(oxv[0], oxv[1], oxv[2], oxv[3]);
    *reinterpret_cast<uint4 *>(hom + HO_QD + off) = make_uint4(oqe[0], oqe[1], oqe[2], oqe[3]);
    *reinterpret_cast<uint4 *>(sm + OFF_KBS + off) = make_uint4(okb[0], okb[1], okb[2], okb[3]);
    *reinterpret_cast<uint4 *>(sm + OFF_KI + ki_index(blk, blk) * 2048 + sw64(t & 15, d0)) =
        make_uint4(oki[0][0], oki[0][1], oki[0][2], oki[0][3]);
  }
  __syncthreads();

  // exact diagonal blocks of M and P for a "big" chunk (per-element decay factors): the 136
  // pairs s <= t of each block, each summed over d by four adjacent lanes (16 channels each);
  // the pair's lane for channels 0-15 also zeroes the mirror entry above the diagonal
  if (big) {
    for (int item = tid; item < 4 * 136 * 4; item += NT1) {
      const int qd = item & 3, pr = item >> 2, i = pr / 136, pi = pr - i * 136;
      int tl = (int)((sqrtf(8.f * pi + 1.f) - 1.f) * 0.5f);
      tl += (tl + 1) * (tl + 2) / 2 <= pi;
      tl -= tl * (tl + 1) / 2 > pi;
      const int sl = pi - tl * (tl + 1) / 2, t = 16 * i + tl, s = 16 * i + sl;
      float mk = 0.f, mq = 0.f;
#pragma unroll 4
      for (int d = 16 * qd; d < 16 * qd + 16; d += 2) {
        const float2 kt = unpack_bf16(*reinterpret_cast<const uint32_t *>(sm + OFF_KS + sw64(t, d)));
        const float2 qt = unpack_bf16(*reinterpret_cast<const uint32_t *>(sm + OFF_QS + sw64(t, d)));
        const float2 ks = unpack_bf16(*reinterpret_cast<const uint32_t *>(sm + OFF_KS + sw64(s, d)));
        const float2 gt = *reinterpret_cast<const float2 *>(GS + gsw(t, d));
        const float2 gs = *reinterpret_cast<const float2 *>(GS + gsw(s, d));
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
        *reinterpret_cast<__nv_bfloat16 *>(sm + OFF_MK + sw64(t, s)) = __float2bfloat16_rn(s < t ? mk : 0.f);
        *reinterpret_cast<__nv_bfloat16 *>(hom + HO_P + sw64(t, s)) = __float2bfloat16_rn(mq);
      } else if (qd == 1 && sl < tl) {  // the mirror (sl, tl) above the diagonal
        AD[i * 256 + sl * 16 + tl] = 0.f;
        *reinterpret_cast<__nv_bfloat16 *>(sm + OFF_MK + sw64(s, t)) = __float2bfloat16_rn(0.f);
        *reinterpret_cast<__nv_bfloat16 *>(hom + HO_P + sw64(s, t)) = __float2bfloat16_rn(0.f);
      }
    }
    __syncthreads();
  }

  __syncthreads();  // the raw tiles are consumed: prefetch the next chunk behind the GEMMs
  if (idx + (int)gridDim.x < nchunks) {
    issue_loads(idx + gridDim.x);
    if (tid < C) beta_next = load_beta(idx + gridDim.x);
  }

  // ---- (2) M = Kdec Kinc^T and P = Qdec Kinc^T per (block row i, block column j <= i), and
  //      (3) T_ii = (I + A_ii)^{-1}.  Warps 0-3 take the diagonal M block i = warp and invert
  //      it right away (one column per lane, fp32 substitution); warps 4-15 take the 10 P
  //      blocks and the 6 off-diagonal M blocks. ----
  auto mp_block = [&](int mat, int i, int j) {
    float acc[2][4] = {};
    // only the diagonal Kinc tiles exist (k / F, or k B for a big chunk); the block pair's
    // factor (e^{r_i - r_j}, or G_ij) scales the A operand along d
    const bool scale = j < i;
    const uint32_t kib = s_base + OFF_KI + ki_index(scale ? j : i, j) * 2048;
    const float *G = gij + (i * 4 + j) * 64;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t af[4], bf[4];
      ldsm_x4(a_frag_addr(s_base + (mat ? OFF_QD : OFF_KD), 16 * i, 16 * kk, lane), af);
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
          *reinterpret_cast<uint32_t *>(sm + OFF_MK + sw64(t, s)) = pack_bf16(v0, v1);
          v0 *= bet[t];
          v1 *= bet[t];
          if (j == i) {
            *reinterpret_cast<float2 *>(AD + i * 256 + tl * 16 + sl) = make_float2(v0, v1);
          } else {
            *reinterpret_cast<uint32_t *>(sm + OFF_AB + sw64(t, s)) = pack_bf16(v0, v1);
          }
        } else {
          v0 = s <= t ? v0 : 0.f;
          v1 = s + 1 <= t ? v1 : 0.f;
          *reinterpret_cast<uint32_t *>(hom + HO_P + sw64(t, s)) = pack_bf16(v0, v1);
        }
      }
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
      const int mat = q < 10 ? 1 : 0;
      if (big && j == i) continue;  // diagonal block already computed exactly
      mp_block(mat, i, j);
    }
  }
  __syncthreads();

  // ---- (4) Tinv = (I+A)^{-1}: block forward substitution on the identity, 8 columns per warp
  //      (warps 0-7; the rows above a column's diagonal block are zero and skipped) ----
  if (warp < 8) solve_columns(sm, s_base, OFF_TF - OFF_OUT, -1, warp * 8, warp >> 1, -1.f, 1.f, warp, lane);
  __syncthreads();
  // ---- (5) W = Tinv beta Kd (stored negated) and U = Tinv beta V as one block-triangular GEMM;
  //      warp w takes 16 of the 128 columns of [W | U] for the row blocks {0, 3} or {1, 2}, so
  //      every warp does 5 of the 10 nonzero blocks of a column ----
  {
    const int cg = warp & 7, c0 = 16 * (cg & 3);
    const bool isW = cg < 4;
    const uint32_t xb = s_base + (isW ? OFF_XK : OFF_XV);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int i = half == 0 ? (warp >> 3) : 3 - (warp >> 3);
      float acc[2][4] = {};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (k > i) break;
        uint32_t af[4], bf[4];
        ldsm_x4(a_frag_addr(s_base + OFF_TF, 16 * i, 16 * k, lane), af);
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
    {  // Kb^T: warp (i, q) transposes the 16 x 16 block (rows 16 i, columns 16 q) of Kb
      const int i = warp >> 2, q = warp & 3;
      uint32_t r[4];
      ldsm_x4_t(ct_frag_addr(s_base + OFF_KBS, 16 * i, 16 * q, lane), r);
      stsm_x4(ho + HO_KBT + sw64(16 * q + (lane & 7) + ((lane >> 3) & 1) * 8, 16 * i + (lane >> 4) * 8), r[0], r[1],
              r[2], r[3]);
    }
  }

  fence_proxy_async_smem();  // make this thread's smem writes visible to the bulk copies
  __syncthreads();
  // ---- the record for kda_fwd_scan: one bulk copy, same swizzled layout as in smem ----
  if (tid == 0) {
    // the record stays in L2 for kda_fwd_scan; the saved record streams out
    bulk_s2g_hint((uint8_t *)p.ws + (int64_t)idx * HO_SIZE, ho, HO_SIZE, l2_policy_keep());
    if (p.saved) {  // P, M, Tinv for the backward
      uint8_t *sv = (uint8_t *)p.saved + (int64_t)idx * kSavedChunk;
      const uint64_t pol = l2_policy_stream();
      bulk_s2g_hint(sv + kSavedP, ho + HO_P, 8192, pol);
      bulk_s2g_hint(sv + kSavedMkk, s_base + OFF_MK, 2 * 8192, pol);
    }
    bulk_commit();
  }
  // ---- the state-independent part of the backward's record: Mneg = Kb^T (-W) (warps 0-7) and
  //      Qt = Qd + P (-W) (warps 8-15), each warp 16 rows x 32 columns ----
  if (p.saved) {
    uint8_t *sv = (uint8_t *)p.saved + (int64_t)idx * kSavedChunk;
    const int rb = (warp >> 1) & 3, jb = rb * 16, nh = warp & 1;
    float X[4][4];
    if (warp < 8) {  // Mneg rows d' in [jb, jb+16)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) X[nt][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t af[4];
        ldsm_x4_t(ct_frag_addr(s_base + OFF_KBS, 16 * kk, jb, lane), af);
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          uint32_t bf[4];
          ldsm_x4_t(bkn_frag_addr(ho + HO_W, 16 * kk, 32 * nh + 16 * np, lane), bf);
          mma16816(X[2 * np], af, bf[0], bf[1]);
          mma16816(X[2 * np + 1], af, bf[2], bf[3]);
        }
      }
    } else {  // Qt rows t in [jb, jb+16)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const float2 v = unpack_bf16(*reinterpret_cast<const uint32_t *>(
              hom + HO_QD + sw64(jb + g4 + 8 * hh, 32 * nh + nt * 8 + 2 * c4)));
          X[nt][2 * hh] = v.x;
          X[nt][2 * hh + 1] = v.y;
        }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        if (kk > rb) break;
        uint32_t af[4];
        ldsm_x4(a_frag_addr(ho + HO_P, jb, 16 * kk, lane), af);
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          uint32_t bf[4];
          ldsm_x4_t(bkn_frag_addr(ho + HO_W, 16 * kk, 32 * nh + 16 * np, lane), bf);
          mma16816(X[2 * np], af, bf[0], bf[1]);
          mma16816(X[2 * np + 1], af, bf[2], bf[3]);
        }
      }
    }
    uint8_t *dst = sm + (warp < 8 ? OFF_XK : OFF_XV);  // staged in the free beta-Kd / beta-V tiles
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh)
        *reinterpret_cast<uint32_t *>(dst + sw64(jb + g4 + 8 * hh, 32 * nh + nt * 8 + 2 * c4)) =
            pack_bf16(X[nt][2 * hh], X[nt][2 * hh + 1]);
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {  // Mneg, Qt (staged in the free beta-Kd / beta-V tiles) and e^{gamma_C}
      const uint64_t pol = l2_policy_stream();
      bulk_s2g_hint(sv + kSavedM, s_base + OFF_XK, 8192, pol);
      bulk_s2g_hint(sv + kSavedQt, s_base + OFF_XV, 8192, pol);
      bulk_s2g_hint(sv + kSavedEG, ho + HO_EG, 256, pol);
      bulk_commit();
    }
  }
  }  // chunk loop
  if (tid == 0) bulk_wait_all();
}

// ---------------------------------------------------------------------------------------
// kda_fwd_scan
// ---------------------------------------------------------------------------------------
// One CTA of 5 warps per (b, h), on the tcgen05 tensor cores with one M = 128 accumulator in
// TMEM (64 columns).  Per chunk, with Sᵀ [d][j] and Unew [t][j] as bf16 B operands in shared
// memory and the record's stacked A operands [Qd; -W] and [P; Kb^T]:
//   MMA A:  D = [Qd; -W] S^T            rows 0-63: Qd S^T,  rows 64-127: -W S^T
//   warps 2-3 (rows 64-127): Unew = U - W S^T -> bf16 tile; then put e^{gamma_C} S^T (fp32
//   state rows d, kept in registers) into rows 64-127 of D
//   MMA B:  D += [P; Kb^T] Unew         rows 0-63: O = Qd S^T + P Unew,
//                                       rows 64-127: S^T <- diag(e^{gamma_C}) S^T + Kb^T Unew
//   warps 0-1 drain O (bf16, TMA store); warps 2-3 take the new state.
// One thread of warp 4 issues the MMAs, the record loads (a three-slot ring of bulk copies, two
// chunks ahead) and the stores; S^T | Unew of each chunk leave by one bulk store for the
// backward.  Every CTA-wide barrier votes on failures, so a bounded wait that gives up takes
// all warps out together.
constexpr int NT2 = 160;
constexpr int NREC = 3;                       // record ring
constexpr int NSV = 3;                        // S^T | Unew tiles (B operands and saved-record staging)
constexpr int REC_STRIDE = 41 * 1024;         // ring slot (HO_SIZE rounded up to 1024 bytes)
constexpr int OFF2_O = 0;                     // O staging, 2 x 8 KB (TMA stores)
constexpr int OFF2_SV = 2 * 8192;             // NSV x 16 KB
constexpr int OFF2_REC = OFF2_SV + NSV * 16384;  // NREC x REC_STRIDE
constexpr int OFF2_MBAR = OFF2_REC + NREC * REC_STRIDE;  // NREC record mbarriers, 2 MMA mbarriers, TMEM slot
constexpr int SMEM2 = OFF2_MBAR + 64;
constexpr uint32_t kIdescScan = idesc_bf16(128, 64, 0, 1);  // A K-major, B MN-major

// 64 fp32 values -> one 128-byte bf16 row of a swizzled tile
__device__ __forceinline__ void store_row_bf16(uint8_t *tile, int row, const float *x) {
#pragma unroll
  for (int ch = 0; ch < 8; ++ch)
    *reinterpret_cast<uint4 *>(tile + sw64(row, ch * 8)) =
        make_uint4(pack_bf16(x[8 * ch], x[8 * ch + 1]), pack_bf16(x[8 * ch + 2], x[8 * ch + 3]),
                   pack_bf16(x[8 * ch + 4], x[8 * ch + 5]), pack_bf16(x[8 * ch + 6], x[8 * ch + 7]));
}
// this thread's TMEM lane, 64 columns from taddr
__device__ __forceinline__ void tmem_row64(uint32_t taddr, float *x) {
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

__global__ void __launch_bounds__(NT2, 1) kda_fwd_scan_kernel(Params p, const __grid_constant__ TmaMaps tm) {
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int bh = blockIdx.x, b = bh / p.H, h = bh % p.H;
  const int nc = p.nc;
  const uint32_t s_base = smem_u32(sm);
  if (s_base & 1023) {  // swizzled tiles need a 1024-byte aligned base
    if (tid == 0) atomicExch(&g_fwd_status, KDA_ERR_MISALIGNED);
    return;
  }
  const uint32_t mrec = s_base + OFF2_MBAR, mA = mrec + 8 * NREC, mB = mA + 8;
  uint32_t *tslot = reinterpret_cast<uint32_t *>(sm + OFF2_MBAR + 8 * NREC + 16);
  const bool leader = tid == 128, lower = warp >= 2 && warp < 4, upper = warp < 2;
  const int m = 32 * warp + lane;  // TMEM lane / accumulator row of warps 0-3
  const int r = m - 64;            // warps 2-3: row t of Unew, row d of S^T

  if (leader) {
    for (int i = 0; i < NREC + 2; ++i) mbar_init(mrec + 8 * i, 1);
    mbar_fence_init();
  }
  float S[64];  // warps 2-3: S^T[r][j] = S[j][r]
#pragma unroll
  for (int j = 0; j < 64; ++j) S[j] = 0.f;
  if (lower && p.state0) {
#pragma unroll
    for (int j = 0; j < 64; ++j) S[j] = p.state0[(int64_t)bh * D * D + j * D + r];
  }
  if (lower) store_row_bf16(sm + OFF2_SV, r, S);
  if (warp == 4) {
    tmem_alloc(smem_u32(tslot), 64);
    tmem_relinquish();
  }
  fence_proxy_async_smem();  // the S^T tile is read by the tensor cores
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tD = *tslot;
  const uint32_t tl = tD + ((uint32_t)(32 * (warp & 3)) << 16);  // this warp's lane quarter

  auto issue = [&](int c) {  // leader: one bulk copy of the chunk's whole record
    const uint8_t *rec = (const uint8_t *)p.ws + ((int64_t)bh * nc + c) * HO_SIZE;
    const int s = c % NREC;
    mbar_expect_tx(mrec + s * 8, HO_SIZE);
    bulk_g2s(s_base + OFF2_REC + s * REC_STRIDE, rec, HO_SIZE, mrec + s * 8);
  };
  if (leader)
    for (int c = 0; c < nc && c < NREC - 1; ++c) issue(c);
  bool failed = false;
  for (int c = 0; c < nc; ++c) {
    const int buf = c & 1, slot = c % NREC;
    const uint32_t rec = s_base + OFF2_REC + slot * REC_STRIDE;
    const uint8_t *recm = sm + OFF2_REC + slot * REC_STRIDE;
    const float *eG = reinterpret_cast<const float *>(recm + HO_EG);
    const uint32_t sv = s_base + OFF2_SV + (c % NSV) * 16384;
    uint8_t *svm = sm + OFF2_SV + (c % NSV) * 16384, *svnm = sm + OFF2_SV + ((c + 1) % NSV) * 16384;
    // chunk c's record landed; the barrier also publishes S^T(c); the leader has seen the stores
    // of chunk c-2 (same O staging, same S^T | Unew tiles as chunk c+1) read their sources
    if (leader) asm volatile("cp.async.bulk.wait_group.read 1;\n" ::: "memory");
    if (__syncthreads_or(!mbar_wait(mrec + slot * 8, (c / NREC) & 1))) { failed = true; break; }
    if (leader) {
      if (c + NREC - 1 < nc) issue(c + NREC - 1);
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < 4; ++k) tc_mma(tD, desc_k(rec + HO_QD, k), desc_mn(sv, k), kIdescScan, k > 0);
      tc_commit(mA);
    }
    bool ok = true;
    if (lower) {  // Unew = U - W S^T; then rows 64-127 of D <- e^{gamma_C} S^T
      ok = mbar_wait(mA, c & 1);
      tc_fence_after();
      float x[64];
      tmem_row64(tl, x);
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        const uint4 u = *reinterpret_cast<const uint4 *>(recm + HO_U + sw64(r, ch * 8));
        const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = unpack_bf16(uw[e]);
          x[8 * ch + 2 * e] += f.x;
          x[8 * ch + 2 * e + 1] += f.y;
        }
      }
      store_row_bf16(svm + 8192, r, x);
      const float e = eG[r];
      uint32_t v[32], w[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        v[j] = __float_as_uint(e * S[j]);
        w[j] = __float_as_uint(e * S[32 + j]);
      }
      tmem_st32(tl, v);
      tmem_st32(tl + 32, w);
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
    }
    if (__syncthreads_or(!ok)) { failed = true; break; }
    if (leader) {
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < 4; ++k) tc_mma(tD, desc_k(rec + HO_P, k), desc_mn(sv + 8192, k), kIdescScan, 1);
      tc_commit(mB);
    }
    if (warp < 4) {
      ok = mbar_wait(mB, c & 1);
      tc_fence_after();
      float x[64];
      tmem_row64(tl, x);
      if (upper) {
        store_row_bf16(sm + OFF2_O + buf * 8192, m, x);  // O row t
      } else {
#pragma unroll
        for (int j = 0; j < 64; ++j) S[j] = x[j];
        store_row_bf16(svnm, r, S);  // S^T(c+1) row d
      }
      fence_proxy_async_smem();
      tc_fence_before();
    }
    if (__syncthreads_or(!ok)) { failed = true; break; }
    if (leader) {  // O by TMA (rows past T dropped); S^T | Unew of chunk c for the backward
      tma_store_rows(&tm.m[0], s_base + OFF2_O + buf * 8192, h, c * C, b);
      if (p.saved) bulk_s2g((uint8_t *)p.saved + ((int64_t)bh * nc + c) * kSavedChunk + kSavedS0, sv, 16384);
      bulk_commit();
    }
  }
  if (failed && leader) atomicExch(&g_fwd_status, KDA_ERR_TIMEOUT);
  if (!failed && lower) {
#pragma unroll
    for (int j = 0; j < 64; ++j) p.stateT[(int64_t)bh * D * D + j * D + r] = S[j];
  }
  if (leader) {
    bulk_wait_all();
    if (failed) {  // no MMA may still write TMEM when it is freed
      mbar_wait(mA, 0);
      mbar_wait(mA, 1);
      mbar_wait(mB, 0);
      mbar_wait(mB, 1);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 4) tmem_dealloc(tD, 64);
}

template <typename Tb>
int launch(const Params &p, cudaStream_t st) {
  auto k1 = kda_fwd_chunks_kernel<Tb>;
  const int smem1 = p.gated ? SMEM1_GP + gate_smem_bytes(p.gated, p.H) : SMEM1;
  if (cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, smem1)) return KDA_ERR_CUDA;
  int dev = 0, nsm = 148;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return KDA_ERR_CUDA;
  const int nchunks = p.B * p.H * p.nc;
  TmaMaps tm;
  const void *srcs[4] = {p.q, p.k, p.v, p.gated ? p.f : (const void *)p.g};
  for (int i = 0; i < 4; ++i)
    if (int e = tma_map_bthd(&tm.m[i], srcs[i], p.B, p.T, p.H, D, i == 3 && !p.gated)) return e;
  k1<<<nchunks < nsm ? nchunks : nsm, NT1, smem1, st>>>(p, tm);
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
  return (size_t)(d->B * d->H * ((d->T + d->chunk - 1) / d->chunk)) * tcfwd::HO_SIZE;
}

int tc_fwd(const Params &p, int dtype_beta, cudaStream_t st) {
  if (dtype_beta == KDA_BF16) return tcfwd::launch<__nv_bfloat16>(p, st);
  if (dtype_beta == KDA_F32) return tcfwd::launch<float>(p, st);
  return KDA_ERR_DTYPE;
}

}  // namespace kda
