// Tensor-core KDA backward for D = 64, chunk = 64, bf16 q/k/v (mma.sync, fp32 accumulate).
//
// Per chunk (gamma = cumsum(g) in the chunk, T_ = (I + A)^{-1}, W = T_ beta Kd, Unew the solved
// WY values of the forward, S0 the chunk-entry state, dS1 the cotangent of the chunk-exit state):
//   dU  = P^T dO + Kb dS1^T          dR = T_^T dU               dv = beta dR
//   dS0 = dS1 diag(e^{gamma_C}) - dS1 Kb^T W + dO^T (Qd - P W)
//   dq  = (dO S0) e^gamma + decayed(dP, k)            dP  = dO Unew^T (s <= t)
//   dk  = -beta (dR S0) e^gamma + decayed(dKK, k)     dKK = -beta_t dR Unew^T (s < t)
//         + (Unew dS1) e^{gamma_C - gamma} + decayed^T(dKK, k) + decayed^T(dP, q)
//   dbeta = dR.V - (dR S0).Kd + sum_s dA M;  dgamma = q dq + k (dk_row - dk_col), + dGamma_C on
//   the last row;  dg = reverse cumsum of dgamma.
// (decayed(X, k)_t = sum_s X[t,s] k_s e^{gamma_t - gamma_s}; decayed^T the same over t >= s.)
// These are the VJPs of the forward's chunk algebra (the quantities of the reference's
// _chunkwise_kda_backward, nope_gdn_mlx.py:2579-2720, derived independently).
//
// Two kernels:
//   kda_bwd_state_scan  one CTA per (b, h) walks the chunks backwards carrying dS in mma
//                       registers, using the forward's saved Mneg = -Kb^T W and Qt = Qd - P W;
//                       it writes every chunk's exit cotangent dS1 (bf16) to the workspace.
//   kda_bwd_chunks      one CTA per (b, h, chunk), independent of each other: takes the
//                       chunk's decay-weighted P, M and Tinv from the saved record, forms
//                       dR = Tinv^T dU as one GEMM, and produces all gradients.
// Chunks whose decay is too strong for the factored form ("big": gamma moves more than
// kSpanMax across half a 16-row block in some channel) take exact per-element decay factors in
// the same kernel.
#include <mutex>
#include <type_traits>

#include "kda_common.cuh"
#include "kda_mma.cuh"
#include "kda_tma.cuh"

namespace kda {


namespace tcbwd {

// set to a KDA_ERR_* code by a bounded wait that gave up (read by kda_device_status)
static __device__ int g_bwd_status;

// Optional phase trace of the chunk kernel (builds with -DKDA_SCAN_TRACE only): SM clock after
// each phase of the first 16 chunks that CTA 0 walks, read back by kda_bwd_trace().
#ifdef KDA_SCAN_TRACE
__device__ long long g_bwd_trace[12][16];
#define BWD_TR(slot) do { if (tid == 0 && blockIdx.x == 0 && it < 16) g_bwd_trace[slot][it] = clock64(); } while (0)
#else
#define BWD_TR(slot) do { } while (0)
#endif

constexpr int C = 64, D = 64;
constexpr float kSpanMax = 60.f;
// the block-pair factors e^{r_i - r_j} of a chunk that is not "big" stay above fp32's smallest
// normal (e^-87) only if gamma moves at most this much between the middle rows of the first and
// the last block; beyond it the factor would flush to zero while the decay it stands for
// (e^{gamma_t - gamma_s} for t, s close to the block boundary) is not negligible
constexpr float kMidGapMax = 80.f;
constexpr float kLog2e = 1.4426950408889634f;  // the big-chunk copy of gamma is kept in log2 units

// workspace: the exit cotangent of every chunk (bf16 [j][d], swizzled)
__host__ __device__ inline size_t ws_bytes(int64_t nchunks) { return (size_t)nchunks * 8192; }

// ---------------------------------------------------------------------------------------
// state-cotangent scan
// ---------------------------------------------------------------------------------------
constexpr int SC_NT = 128;
// a ring of SC_NB chunk buffers, loads running two chunks ahead: per slot the dO tile (TMA,
// 1024-byte aligned) at SC_DO + slot * 8192 and the record span Mneg, Qt, e^{gamma_C} at
// SC_RC + slot * SC_RCB; the exit-cotangent staging (two 8 KB tiles) at SC_DSX
constexpr int SC_NB = 3;
constexpr int SC_DO = 0, SC_DSX = SC_NB * 8192, SC_RC = SC_DSX + 2 * 8192, SC_RCB = 16384 + 256;
constexpr int SC_MN = 0, SC_QT = 8192, SC_EG = 16384;
constexpr int SC_MBAR = SC_RC + SC_NB * SC_RCB;
constexpr int SC_SMEM = SC_MBAR + 8 * SC_NB;

__global__ void __launch_bounds__(SC_NT, 1) kda_bwd_state_scan_kernel(Params p, const __grid_constant__ TmaMaps tm) {
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g4 = lane >> 2, c4 = lane & 3, jb = warp * 16;
  const int bh = blockIdx.x, b = bh / p.H, h = bh % p.H;
  const int nc = p.nc;
  const uint32_t s_base = smem_u32(sm);
  __nv_bfloat16 *ds_exit = (__nv_bfloat16 *)p.ws;
  if (p.gated && bh == 0)  // the gate-parameter gradients are accumulated by the chunk kernel,
    for (int i = tid; i < p.H * 65; i += SC_NT)  // which runs after this one on the stream
      (i < p.H * 64 ? p.ddt_bias[i] : p.dA_log[i - p.H * 64]) = 0.f;
  if (s_base & 1023) {  // TMA tiles with the 128-byte swizzle need a 1024-byte aligned base
    if (tid == 0) atomicExch(&g_bwd_status, KDA_ERR_MISALIGNED);
    return;
  }

  const uint32_t mbar = s_base + SC_MBAR;
  if (tid == 0) {
    for (int i = 0; i < SC_NB; ++i) mbar_init(mbar + 8 * i, 1);
    mbar_fence_init();
  }
  __syncthreads();
  // dO tile by TMA; Mneg, Qt, e^{gamma_C} (one contiguous, already swizzled span of the saved
  // record) by one bulk copy; both complete on the buffer's mbarrier
  int issued = 0;  // thread 0: steps whose loads are issued
  auto issue = [&](int c, int buf) {
    const uint8_t *rec = (const uint8_t *)p.saved_in + ((int64_t)bh * nc + c) * kSavedChunk;
    if (tid == 0) {
      issued = nc - c;
      mbar_expect_tx(mbar + buf * 8, 8192 + kSavedChunk - kSavedM);
      tma_load_rows(s_base + SC_DO + buf * 8192, &tm.m[0], h, c * C, b, mbar + buf * 8);
      bulk_g2s(s_base + SC_RC + buf * SC_RCB, rec + kSavedM, kSavedChunk - kSavedM, mbar + buf * 8);
    }
  };
  auto store_exit = [&](int i) {  // thread 0: the staged exit cotangent of step i (chunk nc-1-i)
    if (tid == 0) {
      bulk_s2g(ds_exit + ((int64_t)bh * nc + nc - 1 - i) * D * D, s_base + SC_DSX + (i & 1) * 8192, 8192);
      bulk_commit();
    }
  };

  float dS[8][4];
#pragma unroll
  for (int nt = 0; nt < 8; ++nt)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float2 v = make_float2(0.f, 0.f);
      if (p.dstateT)
        v = *reinterpret_cast<const float2 *>(p.dstateT + (int64_t)bh * D * D + (jb + g4 + 8 * hh) * D + nt * 8 + 2 * c4);
      dS[nt][2 * hh] = v.x;
      dS[nt][2 * hh + 1] = v.y;
    }
  issue(nc - 1, 0);
  if (nc > 1) issue(nc - 2, 1);
  for (int i = 0; i < nc; ++i) {
    const int c = nc - 1 - i, buf = i % SC_NB;
    if (tid == 0) bulk_wait_read_all();  // the exit-cotangent store of step i - 2 has read its staging
    if (__syncthreads_or(!mbar_wait(mbar + buf * 8, (i / SC_NB) & 1))) {
      if (tid == 0) {  // (bounded) the loads in flight land and the stores read their staging
        atomicExch(&g_bwd_status, KDA_ERR_TIMEOUT);
        for (int s2 = i; s2 < issued; ++s2) mbar_wait(mbar + (s2 % SC_NB) * 8, (s2 / SC_NB) & 1);
        bulk_wait_all();
      }
      return;
    }
    if (i + 2 < nc) issue(c - 2, (i + 2) % SC_NB);
    if (i > 0) store_exit(i - 1);
    const uint32_t base = s_base + SC_RC + buf * SC_RCB, dob = s_base + SC_DO + buf * 8192;
    const float *eG = reinterpret_cast<const float *>(sm + SC_RC + buf * SC_RCB + SC_EG);
    uint32_t da[4][4];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      da[kk][0] = pack_bf16(dS[2 * kk][0], dS[2 * kk][1]);
      da[kk][1] = pack_bf16(dS[2 * kk][2], dS[2 * kk][3]);
      da[kk][2] = pack_bf16(dS[2 * kk + 1][0], dS[2 * kk + 1][1]);
      da[kk][3] = pack_bf16(dS[2 * kk + 1][2], dS[2 * kk + 1][3]);
    }
    {  // stage the exit cotangent (bf16, swizzled) for one bulk store at the next step
      const uint32_t dsx = s_base + SC_DSX + (i & 1) * 8192;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        stsm_x4(dsx + sw64(jb + (lane & 7) + ((lane >> 3) & 1) * 8, 16 * kk + (lane >> 4) * 8), da[kk][0],
                da[kk][1], da[kk][2], da[kk][3]);
      fence_proxy_async_smem();
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float e0 = eG[nt * 8 + 2 * c4], e1 = eG[nt * 8 + 2 * c4 + 1];
      dS[nt][0] *= e0; dS[nt][1] *= e1; dS[nt][2] *= e0; dS[nt][3] *= e1;
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t ao[4];
      ldsm_x4_t(ct_frag_addr(dob, 16 * kk, jb, lane), ao);  // dO^T rows j, k = t
#pragma unroll
      for (int nd = 0; nd < 4; ++nd) {
        uint32_t bm[4], bq[4];
        ldsm_x4_t(bkn_frag_addr(base + SC_MN, 16 * kk, 16 * nd, lane), bm);
        ldsm_x4_t(bkn_frag_addr(base + SC_QT, 16 * kk, 16 * nd, lane), bq);
        mma16816(dS[2 * nd], da[kk], bm[0], bm[1]);
        mma16816(dS[2 * nd + 1], da[kk], bm[2], bm[3]);
        mma16816(dS[2 * nd], ao, bq[0], bq[1]);
        mma16816(dS[2 * nd + 1], ao, bq[2], bq[3]);
      }
    }
  }
  __syncthreads();
  store_exit(nc - 1);
  if (tid == 0) bulk_wait_all();
  if (p.dstate0) {
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh)
        *reinterpret_cast<float2 *>(p.dstate0 + (int64_t)bh * D * D + (jb + g4 + 8 * hh) * D + nt * 8 + 2 * c4) =
            make_float2(dS[nt][2 * hh], dS[nt][2 * hh + 1]);
  }
}

// ---------------------------------------------------------------------------------------
// chunk-parallel gradients
// ---------------------------------------------------------------------------------------
constexpr int CK_NT = 512;  // 16 warps; warp w owns row block mt = w / 4, columns 16 * (w % 4)..
constexpr int O_QS = 0, O_KS = 8192, O_VS = 16384, O_DO = 24576;   // raw bf16 tiles [t][d]
constexpr int O_GS = 32768;                                         // g -> gamma -> F -> dgamma fp32
// S0^T [d][j], Unew [t][j], P [t][s], M [t][s], Tinv [t][s]: one bulk copy of the saved record
constexpr int O_S0 = 49152, O_UN = 57344, O_PB = 65536, O_MK = 73728, O_TF = 81920;
constexpr int O_DS = 90112;                                         // dS1 [j][d]
constexpr int O_KD = 98304, O_QD = 106496, O_KF = 114688, O_KB = 122880;
constexpr int O_DR = 131072, O_DP = 139264, O_DK = 147456;
constexpr int O_SG = 155648;                                        // fused gates: {sigmoid, softplus}(x) half2 [t][d]
constexpr int O_GB = 172032;                                        // big chunks: gamma (fp32, gsw) for P8
constexpr int O_VEC = 188416;
constexpr int V_BET = 0, V_REFS = 64, V_PART = 320, V_ERB = 832, V_EGR = 1088, V_G = 1344,
              V_EG = 2368, V_PDB = 2432, V_PDG = 3200, V_GPT = 3968, V_GPA = 4480,
              V_FLAG = 4496;
// partial sums, each slot written by exactly one thread (no atomics): dbeta rows from P5, P6, P7
// [3][4 column warps][64], dGamma_C columns from the state term [8] and P6 [4] ([12][64])
constexpr int O_MBAR = O_VEC + (V_FLAG + 4) * 4;                    // three mbarriers
constexpr int CK_SMEM = O_MBAR + 24;
constexpr int CK_SMEM_GP = (CK_SMEM + 15) & ~15;                  // staged gate parameters

// out[r] = in[(r - s) mod 8] for a run-time s in [0, 8): three conditional rotations, so that the
// arrays stay in registers
__device__ __forceinline__ void rot8(const float (&in)[8], float (&out)[8], int s) {
  float a[8], b[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) a[r] = (s & 1) ? in[(r + 7) & 7] : in[r];
#pragma unroll
  for (int r = 0; r < 8; ++r) b[r] = (s & 2) ? a[(r + 6) & 7] : a[r];
#pragma unroll
  for (int r = 0; r < 8; ++r) out[r] = (s & 4) ? b[(r + 4) & 7] : b[r];
}

template <typename Tb>
__global__ void __launch_bounds__(CK_NT, 1) kda_bwd_chunks_kernel(Params p, const __grid_constant__ TmaMaps tm) {
  extern __shared__ __align__(1024) uint8_t sm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g4 = lane >> 2, c4 = lane & 3;
  const int mt = warp >> 2, nq = warp & 3, n0 = 16 * nq;
  const int nc = p.nc, T = p.T, H = p.H, nchunks = p.B * p.H * nc;
  const uint32_t s_base = smem_u32(sm);
  const int64_t row_stride = (int64_t)H * D;
  float *GS = reinterpret_cast<float *>(sm + O_GS);
  float *vec = reinterpret_cast<float *>(sm + O_VEC);
  float *bet = vec + V_BET, *refs = vec + V_REFS, *part = vec + V_PART, *erb = vec + V_ERB;
  float *egr = vec + V_EGR, *gij = vec + V_G, *eG = vec + V_EG, *pdb = vec + V_PDB, *pdg = vec + V_PDG;
  const Tb *betag = (const Tb *)p.beta;

  // The CTA is persistent: it walks chunks idx = blockIdx.x, + gridDim.x, ...  The next
  // chunk's inputs are loaded in three stages, each issued (by one thread: TMA tiles of
  // q/k/v/dO/g, bulk copies of the saved record and dS1) as soon as the tiles it fills are dead:
  //   0 (after P5): v, P, Tinv;  1 (after P7): dO, g, S0, Unew^T, M, dS1;  2 (after P8): q, k.
  // Each stage completes on its own mbarrier.  The outputs dq, dk, dg leave by TMA stores
  // from tiles that no load touches.
  const uint32_t mbar = s_base + O_MBAR;
  if (s_base & 1023) {  // TMA tiles with the 128-byte swizzle need a 1024-byte aligned base
    if (tid == 0) atomicExch(&g_bwd_status, KDA_ERR_MISALIGNED);
    return;
  }
  auto issue_loads = [&](int i, int stage) {
    if (tid != 0) return;
    const int bh_ = i / nc, t0_ = (i % nc) * C, b_ = bh_ / H, h_ = bh_ % H;
    const uint8_t *rec_ = (const uint8_t *)p.saved_in + (int64_t)i * kSavedChunk;
    const uint32_t mb = mbar + 8 * stage;
    if (stage == 0) {
      mbar_expect_tx(mb, 3 * 8192);
      tma_load_rows(s_base + O_VS, &tm.m[2], h_, t0_, b_, mb);
      bulk_g2s(s_base + O_PB, rec_ + kSavedP, 8192, mb);
      bulk_g2s(s_base + O_TF, rec_ + kSavedTinv, 8192, mb);
    } else if (stage == 1) {
      mbar_expect_tx(mb, 5 * 8192 + (p.gated ? 8192 : 16384));
      tma_load_rows(s_base + O_DO, &tm.m[3], h_, t0_, b_, mb);
      if (p.gated)  // the gate pre-activation f (bf16) into the first half of GS
        tma_load_rows(s_base + O_GS, &tm.m[4], h_, t0_, b_, mb);
      else
        tma_load_rows_f32(s_base + O_GS, &tm.m[4], h_, t0_, b_, mb);
      bulk_g2s(s_base + O_S0, rec_ + kSavedS0, 2 * 8192, mb);
      bulk_g2s(s_base + O_MK, rec_ + kSavedMkk, 8192, mb);
      bulk_g2s(s_base + O_DS, (const __nv_bfloat16 *)p.ws + (int64_t)i * D * D, 8192, mb);
    } else {
      mbar_expect_tx(mb, 2 * 8192);
      tma_load_rows(s_base + O_QS, &tm.m[0], h_, t0_, b_, mb);
      tma_load_rows(s_base + O_KS, &tm.m[1], h_, t0_, b_, mb);
    }
  };
  // beta of the next chunk, kept raw until its use so that the load does not stall anyone
  auto load_beta = [&](int i) -> Tb {
    const int bh_ = i / nc, t = (i % nc) * C + tid;
    return t < T ? betag[at(p.sb, bh_ / H, t, bh_ % H)] : from_f<Tb>(0.f);
  };
  if (tid == 0) {
    for (int i = 0; i < 3; ++i) mbar_init(mbar + 8 * i, 1);
    mbar_fence_init();
  }
  const float *gA_log;
  const float *gdtb = stage_gate_params(reinterpret_cast<float *>(sm + CK_SMEM_GP), p, tid, CK_NT, &gA_log);
  __syncthreads();
  int idx = blockIdx.x;
  if (idx < nchunks)
    for (int stage = 0; stage < 3; ++stage) issue_loads(idx, stage);
  Tb beta_next = (idx < nchunks && tid < C) ? load_beta(idx) : from_f<Tb>(0.f);

  for (int it = 0; idx < nchunks; idx += gridDim.x, ++it) {
  const int bh = idx / nc, c = idx % nc, b = bh / H, h = bh % H, t0 = c * C;
  const int64_t base_bh = ((int64_t)b * T * H + h) * D;
  const int inext = idx + gridDim.x;
  // ---- P0: this chunk's inputs (bounded waits) ----
  if (__syncthreads_or(!mbar_wait(mbar, it & 1) || !mbar_wait(mbar + 8, it & 1) ||
                       !mbar_wait(mbar + 16, it & 1))) {
    if (tid == 0) {  // (bounded) the loads in flight land before the CTA exits
      atomicExch(&g_bwd_status, KDA_ERR_TIMEOUT);
      for (int s2 = 0; s2 < 3; ++s2) mbar_wait(mbar + 8 * s2, it & 1);
    }
    break;
  }
  const int nvalid = min(C, T - t0);
  BWD_TR(0);
  if (tid < C)
    bet[tid] = !p.gated ? to_f(beta_next) : tid < nvalid ? p.beta_scale * sigmoid_f(to_f(beta_next)) : 0.f;
  if (p.gated) {  // g over GS; sigmoid and softplus of the gate input kept for the VJP
    gate_to_g(sm + O_GS, GS, gA_log, gdtb, h, nvalid, tid, true, reinterpret_cast<__half2 *>(sm + O_SG));
    __syncthreads();
  }
  if (inext < nchunks && tid < C) beta_next = load_beta(inext);
  // ---- P1: gamma = cumsum(g) per channel without a CTA barrier: warp w owns channels 4 w ..
  //      4 w + 3, lane (segment sg = lane / 4 of 8 rows, channel 4 w + lane % 4) adds up its
  //      segment in registers, and the segments' offsets come from a shuffle scan.  Lane sg
  //      visits its rows rotated by sg, so that the 8 lanes of a channel read and write 8 different
  //      swizzle phases (no bank conflicts).  The big-chunk guard comes from the same registers ----
  int bigloc;
  {
    const int sg = lane >> 2, d = 4 * warp + (lane & 3);
    float v[8], w[8], q[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = GS[gsw(8 * sg + ((k + sg) & 7), d)];  // row 8 sg + (k + sg) % 8
    rot8(v, w, sg);  // w[r]: row 8 sg + r
    float tot = 0.f;
#pragma unroll
    for (int r = 0; r < 8; ++r) tot += w[r];
    float inc = tot;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      const float x = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += x;
    }
    float run = inc - tot;  // the segments before this one
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      run += w[r];
      w[r] = run;
    }
    rot8(w, q, (8 - sg) & 7);  // back to the visiting order
#pragma unroll
    for (int k = 0; k < 8; ++k) GS[gsw(8 * sg + ((k + sg) & 7), d)] = q[k];
    // guard: gamma may move at most kSpanMax across either half of a 16-row block (rows 0-8 and
    // 8-15 of block i: lanes of the odd segment 2 i + 1 see both), and at most kMidGapMax between
    // rows 8 and 56 (the block-pair factors), or the chunk is "big"
    const float g_prev = __shfl_up_sync(0xffffffffu, w[0], 4);  // first row of the segment before
    const float g8 = __shfl_sync(0xffffffffu, w[0], 4 + (lane & 3));
    const float g56 = __shfl_sync(0xffffffffu, w[0], 28 + (lane & 3));
    const float span = (sg & 1) ? fmaxf(g_prev - w[0], w[0] - w[7]) : 0.f;
    bigloc = !(span <= kSpanMax) || !(g8 - g56 <= kMidGapMax);
  }
  // a "big" chunk (decay too strong for the factored form) keeps gamma itself and takes exact
  // per-element decay factors in P2, P6 and P8; everything else is the same
  const int big = __syncthreads_or(bigloc);
  {  // per-block vectors, thread (slot, d): slot i < 4 -> block i's entries, slot 4 -> e^{gamma_C}
    const int d = tid & 63, slot = tid >> 6;
    if (slot < 4 && !big) {
      const int i = slot;
      const float gC = GS[gsw(63, d)], ri = GS[gsw(i * 16 + 8, d)];
      refs[i * 64 + d] = ri;
      erb[i * 64 + d] = __expf(ri);
      egr[i * 64 + d] = __expf(gC - ri);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        gij[(i * 4 + j) * 64 + d] = j < i ? __expf(ri - GS[gsw(j * 16 + 8, d)]) : (j == i ? 1.f : 0.f);
    } else if (slot < 4) {  // big: G_ij = e^{gamma(start of i) - gamma(end of j)} <= 1, j < i
      const int i = slot;
      const float si = GS[gsw(i * 16, d)];
#pragma unroll
      for (int j = 0; j < 4; ++j) gij[(i * 4 + j) * 64 + d] = j < i ? __expf(si - GS[gsw(j * 16 + 15, d)]) : 0.f;
    } else if (slot == 4) {
      eG[d] = __expf(GS[gsw(63, d)]);
    }
  }
  if (tid == 0) bulk_wait_read_all();  // the previous chunk's output stores have read KD, QD, KF
  __syncthreads();
  BWD_TR(1);

  // ---- P2: operand build: KD = k F, QD = q F, KF = k / F, KB = k e^{gamma_C - gamma}.
  //      A big chunk factors e^{gamma_t - gamma_s} (t in block i > j, the block of s) as
  //      A_t G_ij B_s, every factor <= 1: KD = k A, QD = q A with A_t = e^{gamma_t - gamma(start
  //      of t's block)}, KF = k B with B_s = e^{gamma(end of s's block) - gamma_s}; its diagonal
  //      blocks take exact factors in P8 from a copy of gamma (GS is reloaded before P8) ----
  float *GB = reinterpret_cast<float *>(sm + O_GB);
  if (big) {
    for (int u = tid; u < 512; u += CK_NT) {
      const int t = u >> 3, ch = u & 7, d0 = ch * 8, blk = t >> 4;
      const uint32_t off = sw64(t, d0);
      const uint4 kq = *reinterpret_cast<const uint4 *>(sm + O_KS + off);
      const uint4 qq = *reinterpret_cast<const uint4 *>(sm + O_QS + off);
      const uint32_t kw[4] = {kq.x, kq.y, kq.z, kq.w}, qw[4] = {qq.x, qq.y, qq.z, qq.w};
      uint32_t okd[4], oqd[4], okf[4], okb[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 kf = unpack_bf16(kw[e]), qf = unpack_bf16(qw[e]);
        const int d = d0 + 2 * e;
        const float2 gm = *reinterpret_cast<const float2 *>(GS + gsw(t, d));
        const float2 gc = *reinterpret_cast<const float2 *>(GS + gsw(63, d));
        const float2 gs = *reinterpret_cast<const float2 *>(GS + gsw(16 * blk, d));
        const float2 ge = *reinterpret_cast<const float2 *>(GS + gsw(16 * blk + 15, d));
        *reinterpret_cast<float2 *>(GB + gsw(t, d)) = make_float2(gm.x * kLog2e, gm.y * kLog2e);
        const float a0 = __expf(gm.x - gs.x), a1 = __expf(gm.y - gs.y);
        const float b0 = __expf(ge.x - gm.x), b1 = __expf(ge.y - gm.y);
        okd[e] = pack_bf16(kf.x * a0, kf.y * a1);
        oqd[e] = pack_bf16(qf.x * a0, qf.y * a1);
        okf[e] = pack_bf16(kf.x * b0, kf.y * b1);
        okb[e] = pack_bf16(kf.x * __expf(gc.x - gm.x), kf.y * __expf(gc.y - gm.y));
      }
      *reinterpret_cast<uint4 *>(sm + O_KD + off) = make_uint4(okd[0], okd[1], okd[2], okd[3]);
      *reinterpret_cast<uint4 *>(sm + O_QD + off) = make_uint4(oqd[0], oqd[1], oqd[2], oqd[3]);
      *reinterpret_cast<uint4 *>(sm + O_KF + off) = make_uint4(okf[0], okf[1], okf[2], okf[3]);
      *reinterpret_cast<uint4 *>(sm + O_KB + off) = make_uint4(okb[0], okb[1], okb[2], okb[3]);
    }
  } else
  for (int u = tid; u < 512; u += CK_NT) {
    const int t = u >> 3, ch = u & 7, d0 = ch * 8, blk = t >> 4;
    const uint32_t off = sw64(t, d0);
    const uint4 kq = *reinterpret_cast<const uint4 *>(sm + O_KS + off);
    const uint4 qq = *reinterpret_cast<const uint4 *>(sm + O_QS + off);
    const uint32_t kw[4] = {kq.x, kq.y, kq.z, kq.w}, qw[4] = {qq.x, qq.y, qq.z, qq.w};
    uint32_t okd[4], oqd[4], okf[4], okb[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 kf = unpack_bf16(kw[e]), qf = unpack_bf16(qw[e]);
      const int d = d0 + 2 * e;
      const float2 gm = *reinterpret_cast<const float2 *>(GS + gsw(t, d));
      const float2 rf = *reinterpret_cast<const float2 *>(refs + blk * 64 + d);
      const float2 er = *reinterpret_cast<const float2 *>(egr + blk * 64 + d);
      const float F0 = __expf(gm.x - rf.x), F1 = __expf(gm.y - rf.y);
      *reinterpret_cast<float2 *>(GS + gsw(t, d)) = make_float2(F0, F1);  // GS holds F = e^{gamma - r_b(t)}
      const float i0 = __fdividef(1.f, F0), i1 = __fdividef(1.f, F1);
      okd[e] = pack_bf16(kf.x * F0, kf.y * F1);
      oqd[e] = pack_bf16(qf.x * F0, qf.y * F1);
      okf[e] = pack_bf16(kf.x * i0, kf.y * i1);
      okb[e] = pack_bf16(kf.x * i0 * er.x, kf.y * i1 * er.y);
    }
    *reinterpret_cast<uint4 *>(sm + O_KD + off) = make_uint4(okd[0], okd[1], okd[2], okd[3]);
    *reinterpret_cast<uint4 *>(sm + O_QD + off) = make_uint4(oqd[0], oqd[1], oqd[2], oqd[3]);
    *reinterpret_cast<uint4 *>(sm + O_KF + off) = make_uint4(okf[0], okf[1], okf[2], okf[3]);
    *reinterpret_cast<uint4 *>(sm + O_KB + off) = make_uint4(okb[0], okb[1], okb[2], okb[3]);
  }

  __syncthreads();
  BWD_TR(2);
  // dGamma_C, state part: e^{gamma_C} sum_j S0[j,d] dS1[j,d]
  {
    const int d = tid & 63, jq = tid >> 6;
    float a = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int row = jq * 8 + j;
      a += __bfloat162float(*reinterpret_cast<const __nv_bfloat16 *>(sm + O_S0 + sw64(d, row))) *
           __bfloat162float(*reinterpret_cast<const __nv_bfloat16 *>(sm + O_DS + sw64(row, d)));
    }
    pdg[jq * 64 + d] = a * eG[d];
  }
  // ---- P5: dU = P^T dO + Kb dS1^T (staged bf16 in the DP tile), dR = Tinv^T dU ----
  {
    float du[2][4] = {};
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t af[4], bf[4];
      if (kk >= mt) {
        ldsm_x4_t(ct_frag_addr(s_base + O_PB, 16 * kk, 16 * mt, lane), af);  // P^T
        ldsm_x4_t(bkn_frag_addr(s_base + O_DO, 16 * kk, n0, lane), bf);
        mma16816(du[0], af, bf[0], bf[1]);
        mma16816(du[1], af, bf[2], bf[3]);
      }
      ldsm_x4(a_frag_addr(s_base + O_KB, 16 * mt, 16 * kk, lane), af);
      ldsm_x4(bnk_frag_addr(s_base + O_DS, n0, 16 * kk, lane), bf);
      mma16816(du[0], af, bf[0], bf[1]);
      mma16816(du[1], af, bf[2], bf[3]);
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh)
        *reinterpret_cast<uint32_t *>(sm + O_DP + sw64(16 * mt + g4 + 8 * hh, n0 + 8 * nt + 2 * c4)) =
            pack_bf16(du[nt][2 * hh], du[nt][2 * hh + 1]);
  }
  __syncthreads();
  BWD_TR(3);
  {
    float y[2][4] = {};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (k < mt) continue;
      uint32_t af[4], bf[4];
      ldsm_x4_t(ct_frag_addr(s_base + O_TF, 16 * k, 16 * mt, lane), af);  // Tinv_k,mt^T
      ldsm_x4_t(bkn_frag_addr(s_base + O_DP, 16 * k, n0, lane), bf);
      mma16816(y[0], af, bf[0], bf[1]);
      mma16816(y[1], af, bf[2], bf[3]);
    }
    __nv_bfloat16 *dvg = (__nv_bfloat16 *)p.dv;
    float dbv[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int t = 16 * mt + g4 + 8 * hh, col = n0 + 8 * nt + 2 * c4;
        *reinterpret_cast<uint32_t *>(sm + O_DR + sw64(t, col)) = pack_bf16(y[nt][2 * hh], y[nt][2 * hh + 1]);
        const float2 vv = unpack_bf16(*reinterpret_cast<const uint32_t *>(sm + O_VS + sw64(t, col)));
        dbv[hh] += y[nt][2 * hh] * vv.x + y[nt][2 * hh + 1] * vv.y;
        if (t0 + t < T)
          *reinterpret_cast<uint32_t *>(dvg + base_bh + (int64_t)(t0 + t) * row_stride + col) =
              pack_bf16(bet[t] * y[nt][2 * hh], bet[t] * y[nt][2 * hh + 1]);
      }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float v = dbv[hh];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      if (c4 == 0) pdb[(0 * 4 + nq) * 64 + 16 * mt + g4 + 8 * hh] = v;
    }
  }
  __syncthreads();
  if (inext < nchunks) issue_loads(inext, 0);  // v, P and Tinv are dead from here on
  BWD_TR(4);

  // ---- P6..P8: per warp rows 16 * mt.. and columns n0.. of dq, dk ----
  float DQ[2][4], DKp[2][4], DKm[2][4], Fv[2][4];
  {
    float dRS[2][4] = {}, dOS[2][4] = {}, dKb[2][4] = {};
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t aR[4], aO[4], aU[4], bS[4], bD[4];
      ldsm_x4(a_frag_addr(s_base + O_DR, 16 * mt, 16 * kk, lane), aR);
      ldsm_x4(a_frag_addr(s_base + O_DO, 16 * mt, 16 * kk, lane), aO);
      ldsm_x4(a_frag_addr(s_base + O_UN, 16 * mt, 16 * kk, lane), aU);  // Unew rows t, k = j
      ldsm_x4(bnk_frag_addr(s_base + O_S0, n0, 16 * kk, lane), bS);     // S0^T rows d, k = j
      ldsm_x4_t(bkn_frag_addr(s_base + O_DS, 16 * kk, n0, lane), bD);
      mma16816(dRS[0], aR, bS[0], bS[1]);
      mma16816(dRS[1], aR, bS[2], bS[3]);
      mma16816(dOS[0], aO, bS[0], bS[1]);
      mma16816(dOS[1], aO, bS[2], bS[3]);
      mma16816(dKb[0], aU, bD[0], bD[1]);
      mma16816(dKb[1], aU, bD[2], bD[3]);
    }
    float dbr[2] = {0.f, 0.f}, dgc[2][2] = {};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int d = n0 + 8 * nt + 2 * c4;
      const float2 er = *reinterpret_cast<const float2 *>(erb + mt * 64 + d);
      const float2 eq = *reinterpret_cast<const float2 *>(egr + mt * 64 + d);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int t = 16 * mt + g4 + 8 * hh;
        const float2 F = *reinterpret_cast<const float2 *>(GS + gsw(t, d));  // F, or gamma if big
        const float2 kv = unpack_bf16(*reinterpret_cast<const uint32_t *>(sm + O_KS + sw64(t, d)));
        const float nb = -bet[t];
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          const int e = 2 * hh + x;
          const float fg = x ? F.y : F.x, k_ = x ? kv.y : kv.x;
          float f, eg, eb;  // e^{gamma_t} = f e^{r}, e^{gamma_C - gamma_t} = e^{gamma_C - r} / f
          if (!big) {
            f = fg;
            eg = f * (x ? er.y : er.x);
            eb = __fdividef(x ? eq.y : eq.x, f);
          } else {  // (A_t is applied in P8 from the copy of gamma)
            f = 1.f;
            eg = __expf(fg);
            eb = __expf(GS[gsw(63, d + x)] - fg);  // gamma_C - gamma_t
          }
          Fv[nt][e] = f;
          DQ[nt][e] = dOS[nt][e] * eg;
          DKp[nt][e] = nb * dRS[nt][e] * eg;
          DKm[nt][e] = dKb[nt][e] * eb;
          dbr[hh] -= dRS[nt][e] * k_ * eg;
          dgc[nt][x] += k_ * DKm[nt][e];
        }
      }
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float v = dbr[hh];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      if (c4 == 0) pdb[(1 * 4 + nq) * 64 + 16 * mt + g4 + 8 * hh] = v;
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        float v = dgc[nt][x];
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        if (g4 == 0) pdg[(8 + mt) * 64 + n0 + 8 * nt + 2 * c4 + x] = v;
      }
  }
  // ---- P7: block (mt, sb = nq) of dP = dO Unew^T (s <= t) and dKK = -beta dR Unew^T (s < t),
  //      dbeta += dA . M ----
  if (nq <= mt) {
    const int sb = nq;
    float aP[2][4] = {}, aA[2][4] = {};
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t aO[4], aR[4], bU[4];
      ldsm_x4(a_frag_addr(s_base + O_DO, 16 * mt, 16 * kk, lane), aO);
      ldsm_x4(a_frag_addr(s_base + O_DR, 16 * mt, 16 * kk, lane), aR);
      ldsm_x4(bnk_frag_addr(s_base + O_UN, 16 * sb, 16 * kk, lane), bU);
      mma16816(aP[0], aO, bU[0], bU[1]);
      mma16816(aP[1], aO, bU[2], bU[3]);
      mma16816(aA[0], aR, bU[0], bU[1]);
      mma16816(aA[1], aR, bU[2], bU[3]);
    }
    float dbr[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int t = 16 * mt + g4 + 8 * hh, s = 16 * sb + 8 * nt + 2 * c4;
        const float p0 = s <= t ? aP[nt][2 * hh] : 0.f, p1 = s + 1 <= t ? aP[nt][2 * hh + 1] : 0.f;
        const float a0 = s < t ? -aA[nt][2 * hh] : 0.f, a1 = s + 1 < t ? -aA[nt][2 * hh + 1] : 0.f;
        *reinterpret_cast<uint32_t *>(sm + O_DP + sw64(t, s)) = pack_bf16(p0, p1);
        *reinterpret_cast<uint32_t *>(sm + O_DK + sw64(t, s)) = pack_bf16(bet[t] * a0, bet[t] * a1);
        const float2 m = unpack_bf16(*reinterpret_cast<const uint32_t *>(sm + O_MK + sw64(t, s)));
        dbr[hh] += a0 * m.x + a1 * m.y;
      }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float v = dbr[hh];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      if (c4 == 0) pdb[(2 * 4 + nq) * 64 + 16 * mt + g4 + 8 * hh] = v;
    }
  } else if (c4 == 0) {  // blocks above the diagonal contribute nothing
    pdb[(2 * 4 + nq) * 64 + 16 * mt + g4] = 0.f;
    pdb[(2 * 4 + nq) * 64 + 16 * mt + g4 + 8] = 0.f;
  }
  __syncthreads();
  if (inext < nchunks) issue_loads(inext, 1);  // so are dO, g, S0, Unew^T, M and dS1
  BWD_TR(5);
  // ---- P8: decayed products.  Block pairs go through the tensor cores with the factors of P2;
  //      a big chunk's diagonal block (mt, mt) is summed here with exact factors ----
  // block pairs; compiled once per case (`Big`: without the diagonal block, B_s for the columns)
  auto p8_pairs = [&](auto big_tag) {
    constexpr bool Big = decltype(big_tag)::value;
    float Q2[2][4] = {}, K2[2][4] = {}, M2[2][4] = {};
    for (int j = 0; j < mt + (Big ? 0 : 1); ++j) {  // rows t in block mt, columns s in block j
      float T1[2][4] = {}, T2[2][4] = {};
      uint32_t aP[4], aK[4], bK[4];
      ldsm_x4(a_frag_addr(s_base + O_DP, 16 * mt, 16 * j, lane), aP);
      ldsm_x4(a_frag_addr(s_base + O_DK, 16 * mt, 16 * j, lane), aK);
      ldsm_x4_t(bkn_frag_addr(s_base + O_KF, 16 * j, n0, lane), bK);
      mma16816(T1[0], aP, bK[0], bK[1]);
      mma16816(T1[1], aP, bK[2], bK[3]);
      mma16816(T2[0], aK, bK[0], bK[1]);
      mma16816(T2[1], aK, bK[2], bK[3]);
      const float *G = gij + (mt * 4 + j) * 64;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const float2 g2 = *reinterpret_cast<const float2 *>(G + n0 + 8 * nt + 2 * c4);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float gv = (e & 1) ? g2.y : g2.x;
          Q2[nt][e] += gv * T1[nt][e];
          K2[nt][e] += gv * T2[nt][e];
        }
      }
    }
    for (int i = mt + (Big ? 1 : 0); i < 4; ++i) {  // rows s in block mt, sum over t in block i
      float T3[2][4] = {};
      uint32_t aKt[4], aPt[4], bK[4], bQ[4];
      ldsm_x4_t(ct_frag_addr(s_base + O_DK, 16 * i, 16 * mt, lane), aKt);
      ldsm_x4_t(ct_frag_addr(s_base + O_DP, 16 * i, 16 * mt, lane), aPt);
      ldsm_x4_t(bkn_frag_addr(s_base + O_KD, 16 * i, n0, lane), bK);
      ldsm_x4_t(bkn_frag_addr(s_base + O_QD, 16 * i, n0, lane), bQ);
      mma16816(T3[0], aKt, bK[0], bK[1]);
      mma16816(T3[1], aKt, bK[2], bK[3]);
      mma16816(T3[0], aPt, bQ[0], bQ[1]);
      mma16816(T3[1], aPt, bQ[2], bQ[3]);
      const float *G = gij + (i * 4 + mt) * 64;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const float2 g2 = *reinterpret_cast<const float2 *>(G + n0 + 8 * nt + 2 * c4);
#pragma unroll
        for (int e = 0; e < 4; ++e) M2[nt][e] += ((e & 1) ? g2.y : g2.x) * T3[nt][e];
      }
    }
    if (!Big) {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          DQ[nt][e] += Fv[nt][e] * Q2[nt][e];
          DKp[nt][e] += Fv[nt][e] * K2[nt][e];
          DKm[nt][e] += __fdividef(M2[nt][e], Fv[nt][e]);
        }
    } else {  // A_t = e^{gamma_t - gamma(start of block mt)}, B_s = e^{gamma(end of it) - gamma_s}
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int d = n0 + 8 * nt + 2 * c4 + (e & 1);
          const float b = exp2f(GB[gsw(16 * mt + 15, d)] - GB[gsw(16 * mt + g4 + 8 * (e >> 1), d)]);
          DKm[nt][e] += M2[nt][e] * b;
        }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int d = n0 + 8 * nt + 2 * c4 + (e & 1);
          const float a = exp2f(GB[gsw(16 * mt + g4 + 8 * (e >> 1), d)] - GB[gsw(16 * mt, d)]);
          DQ[nt][e] += a * Q2[nt][e];
          DKp[nt][e] += a * K2[nt][e];
        }
    }
  };
  if (big) {
    // A big chunk's diagonal blocks, split into 8-row halves.  The block of t in the upper half
    // and s in the lower half goes through the tensor cores as A'_t G B'_s, every factor <= 1:
    // A'_t = e^{gamma_t - gamma_8}, G = e^{gamma_8 - gamma_7}, B'_s = e^{gamma_7 - gamma_s} (rows
    // 7 and 8 of the block).  The two 8 x 8 triangles on the diagonal are summed exactly, over
    // the terms with s <= t only, where e^{gamma_t - gamma_s} <= 1 (gamma is a running sum of
    // g <= 0; the DP / DK tiles are zero above the diagonal).
    {  // X = k B' (lower-half rows), k A' (upper-half rows) in the dead dR tile; Y = q A' (upper-half
       // rows) in the dead Kb tile
      const int t = tid >> 3, d0 = (tid & 7) * 8, up = (t >> 3) & 1, rr = (t & ~15) + 7 + up;
      const uint32_t off = sw64(t, d0);
      const uint4 kq = *reinterpret_cast<const uint4 *>(sm + O_KS + off);
      const uint4 qq = *reinterpret_cast<const uint4 *>(sm + O_QS + off);
      const uint32_t kw[4] = {kq.x, kq.y, kq.z, kq.w}, qw[4] = {qq.x, qq.y, qq.z, qq.w};
      uint32_t ox[4], oy[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d = d0 + 2 * e;
        const float2 gt = *reinterpret_cast<const float2 *>(GB + gsw(t, d));
        const float2 gr = *reinterpret_cast<const float2 *>(GB + gsw(rr, d));
        const float f0 = exp2f(up ? gt.x - gr.x : gr.x - gt.x), f1 = exp2f(up ? gt.y - gr.y : gr.y - gt.y);
        const float2 kf = unpack_bf16(kw[e]), qf = unpack_bf16(qw[e]);
        ox[e] = pack_bf16(kf.x * f0, kf.y * f1);
        oy[e] = pack_bf16(qf.x * f0, qf.y * f1);
      }
      *reinterpret_cast<uint4 *>(sm + O_DR + off) = make_uint4(ox[0], ox[1], ox[2], ox[3]);
      if (up) *reinterpret_cast<uint4 *>(sm + O_KB + off) = make_uint4(oy[0], oy[1], oy[2], oy[3]);
    }
    __syncthreads();
    BWD_TR(8);
    auto bf = [&](int tile, int r, int c) {
      return __bfloat162float(*reinterpret_cast<const __nv_bfloat16 *>(sm + tile + sw64(r, c)));
    };
    const int r0 = 16 * mt + g4, r1 = r0 + 8;  // this thread's two rows: lower and upper half
    float gw[2][4];                              // this thread's own gamma (log2 units)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) gw[nt][e] = GB[gsw(e < 2 ? r0 : r1, n0 + 8 * nt + 2 * c4 + (e & 1))];
    {  // rows t = r1 over s in the lower half: dq += A'G (dP X), dk_row += A'G (dKK X)
      float T1[2][4] = {}, T2[2][4] = {};
      uint32_t aP[2], aK[2], bX[2];
      ldsm_x2(a8_frag_addr(s_base + O_DP, 16 * mt, 16 * mt, lane), aP);
      ldsm_x2(a8_frag_addr(s_base + O_DK, 16 * mt, 16 * mt, lane), aK);
      ldsm_x2_t(t8_frag_addr(s_base + O_DR, 16 * mt, n0, lane), bX);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        mma1688(T1[nt], aP[0], aP[1], bX[nt]);
        mma1688(T2[nt], aK[0], aK[1], bX[nt]);
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          const float ag = exp2f(gw[nt][2 + x] - GB[gsw(16 * mt + 7, n0 + 8 * nt + 2 * c4 + x)]);
          DQ[nt][2 + x] = fmaf(ag, T1[nt][2 + x], DQ[nt][2 + x]);
          DKp[nt][2 + x] = fmaf(ag, T2[nt][2 + x], DKp[nt][2 + x]);
        }
    }
    {  // columns s = r0 over t in the upper half: dk_col += G B' (dKK^T X + dP^T Y)
      float T3[2][4] = {};
      uint32_t aK[2], aP[2], bX[2], bY[2];
      ldsm_x2_t(t8_frag_addr(s_base + O_DK, 16 * mt + 8, 16 * mt, lane), aK);
      ldsm_x2_t(t8_frag_addr(s_base + O_DP, 16 * mt + 8, 16 * mt, lane), aP);
      ldsm_x2_t(t8_frag_addr(s_base + O_DR, 16 * mt + 8, n0, lane), bX);
      ldsm_x2_t(t8_frag_addr(s_base + O_KB, 16 * mt + 8, n0, lane), bY);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        mma1688(T3[nt], aK[0], aK[1], bX[nt]);
        mma1688(T3[nt], aP[0], aP[1], bY[nt]);
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          const float bg = exp2f(GB[gsw(16 * mt + 8, n0 + 8 * nt + 2 * c4 + x)] - gw[nt][x]);
          DKm[nt][x] = fmaf(bg, T3[nt][x], DKm[nt][x]);
        }
    }
    BWD_TR(9);
    // The triangles, exactly, balanced over the lanes: lane row g (g = g4) takes lower-half row
    // 16 mt + g (g + 1 terms) and upper-half row tu = 16 mt + 15 - g (8 - g terms), nine steps on
    // every lane; the upper row's sums belong to lane row 7 - g, which holds tu's fragments, and
    // move there by one shuffle (lane ^ 28).
    const int tu = 16 * mt + 15 - g4;
    {  // dq, dk rows over s <= t in t's half
      float TQ[2][2] = {}, TK[2][2] = {};
#pragma unroll
      for (int j = 0; j < 9; ++j) {
        const bool lo = j <= g4;
        const int t = lo ? r0 : tu, s = lo ? 16 * mt + j : 16 * mt + 7 + j - g4;
        const float dp = bf(O_DP, t, s), dk = bf(O_DK, t, s);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const int d = n0 + 8 * nt + 2 * c4;
          const float2 gt = *reinterpret_cast<const float2 *>(GB + gsw(t, d));
          const float2 gs = *reinterpret_cast<const float2 *>(GB + gsw(s, d));
          const float2 ks = unpack_bf16(*reinterpret_cast<const uint32_t *>(sm + O_KS + sw64(s, d)));
#pragma unroll
          for (int x = 0; x < 2; ++x) {
            const float w = (x ? ks.y : ks.x) * exp2f((x ? gt.y : gt.x) - (x ? gs.y : gs.x));
            const float wl = lo ? w : 0.f, wh = lo ? 0.f : w;
            DQ[nt][x] = fmaf(dp, wl, DQ[nt][x]);
            DKp[nt][x] = fmaf(dk, wl, DKp[nt][x]);
            TQ[nt][x] = fmaf(dp, wh, TQ[nt][x]);
            TK[nt][x] = fmaf(dk, wh, TK[nt][x]);
          }
        }
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          DQ[nt][2 + x] += __shfl_xor_sync(0xffffffffu, TQ[nt][x], 28);
          DKp[nt][2 + x] += __shfl_xor_sync(0xffffffffu, TK[nt][x], 28);
        }
    }
    BWD_TR(10);
    {  // dk columns over t >= s in s's half: column 16 mt + g (8 - g terms), column tu (g + 1 terms)
      float TM[2][2] = {};
#pragma unroll
      for (int j = 0; j < 9; ++j) {
        const bool lo = j < 8 - g4;
        const int sc = lo ? r0 : tu, t = lo ? r0 + j : tu + j - (8 - g4);
        const float dp = bf(O_DP, t, sc), dk = bf(O_DK, t, sc);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const int d = n0 + 8 * nt + 2 * c4;
          const float2 gt = *reinterpret_cast<const float2 *>(GB + gsw(t, d));
          const float2 gs = *reinterpret_cast<const float2 *>(GB + gsw(sc, d));
          const float2 kt = unpack_bf16(*reinterpret_cast<const uint32_t *>(sm + O_KS + sw64(t, d)));
          const float2 qt = unpack_bf16(*reinterpret_cast<const uint32_t *>(sm + O_QS + sw64(t, d)));
#pragma unroll
          for (int x = 0; x < 2; ++x) {
            const float v = (dk * (x ? kt.y : kt.x) + dp * (x ? qt.y : qt.x)) *
                            exp2f((x ? gt.y : gt.x) - (x ? gs.y : gs.x));
            DKm[nt][x] += lo ? v : 0.f;
            TM[nt][x] += lo ? 0.f : v;
          }
        }
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int x = 0; x < 2; ++x) DKm[nt][2 + x] += __shfl_xor_sync(0xffffffffu, TM[nt][x], 28);
    }
    BWD_TR(11);
    p8_pairs(std::true_type{});
  } else {
    p8_pairs(std::false_type{});
  }
  // ---- P9: dgamma, dg = reverse cumsum, outputs ----
  // ---- P9: dgamma = q dq + k (dk_row - dk_col) in registers while q, k are still resident ----
  float dgm[2][4];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int t = 16 * mt + g4 + 8 * hh, d = n0 + 8 * nt + 2 * c4, e = 2 * hh;
      const float2 qv = unpack_bf16(*reinterpret_cast<const uint32_t *>(sm + O_QS + sw64(t, d)));
      const float2 kv = unpack_bf16(*reinterpret_cast<const uint32_t *>(sm + O_KS + sw64(t, d)));
      dgm[nt][e] = qv.x * DQ[nt][e] + kv.x * (DKp[nt][e] - DKm[nt][e]);
      dgm[nt][e + 1] = qv.y * DQ[nt][e + 1] + kv.y * (DKp[nt][e + 1] - DKm[nt][e + 1]);
    }
  __syncthreads();  // every warp is done with q, k and the P8 operand tiles
  BWD_TR(6);
  if (inext < nchunks) issue_loads(inext, 2);
  // staging: dq (bf16) in KD, dk (bf16) in QD, dgamma (fp32, gsw layout) over KF and KB
  float *DG = reinterpret_cast<float *>(sm + O_KF);
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int t = 16 * mt + g4 + 8 * hh, d = n0 + 8 * nt + 2 * c4, e = 2 * hh;
      *reinterpret_cast<float2 *>(DG + gsw(t, d)) = make_float2(dgm[nt][e], dgm[nt][e + 1]);
      *reinterpret_cast<uint32_t *>(sm + O_KD + sw64(t, d)) = pack_bf16(DQ[nt][e], DQ[nt][e + 1]);
      *reinterpret_cast<uint32_t *>(sm + O_QD + sw64(t, d)) =
          pack_bf16(DKp[nt][e] + DKm[nt][e], DKp[nt][e + 1] + DKm[nt][e + 1]);
    }
  fence_proxy_async_smem();
  __syncthreads();
  if (tid == 0) {  // dq, dk: TMA stores of the staged tiles (rows past T are dropped)
    tma_store_rows(&tm.m[5], s_base + O_KD, h, t0, b);
    tma_store_rows(&tm.m[6], s_base + O_QD, h, t0, b);
    bulk_commit();
  }
  {  // dg = reverse cumsum of dgamma (+ dGamma_C from the last row up), in place:
     // 8 segments of 8 rows
    const int d = tid & 63, seg = tid >> 6;
    float ssum = 0.f;
#pragma unroll
    for (int r = 0; r < 8; ++r) ssum += DG[gsw(seg * 8 + r, d)];
    part[seg * 64 + d] = ssum;
    __syncthreads();
    float acc = 0.f;  // dGamma_C
#pragma unroll
    for (int s2 = 0; s2 < 12; ++s2) acc += pdg[s2 * 64 + d];
    for (int s2 = seg + 1; s2 < 8; ++s2) acc += part[s2 * 64 + d];
    if (!p.gated) {
#pragma unroll
      for (int r = 7; r >= 0; --r) {
        const int t = seg * 8 + r;
        acc += DG[gsw(t, d)];
        DG[gsw(t, d)] = acc;
      }
    } else {  // through the gate: df = dg (-A) sigmoid(x), dA_log += dg g, ddt_bias += df
      // (partials into their own slots; summed after the barrier below)
      const __half2 *sgt = reinterpret_cast<const __half2 *>(sm + O_SG);
      const float A = __expf(gA_log[h]);
      float pa = 0.f, pt = 0.f;
#pragma unroll
      for (int r = 7; r >= 0; --r) {
        const int t = seg * 8 + r;
        acc += DG[gsw(t, d)];
        const float2 ss = __half22float2(sgt[t * 64 + d]);
        const float df = t0 + t < T ? -A * acc * ss.x : 0.f;
        pa += t0 + t < T ? acc * ss.y : 0.f;
        pt += df;
        *reinterpret_cast<__nv_bfloat16 *>(sm + O_DR + sw64(t, d)) = __float2bfloat16_rn(df);
      }
      vec[V_GPT + seg * 64 + d] = pt;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) pa += __shfl_xor_sync(0xffffffffu, pa, o);
      if (lane == 0) vec[V_GPA + warp] = -A * pa;
    }
    if (tid < 64 && t0 + tid < T) {
      float db = 0.f;
#pragma unroll
      for (int s2 = 0; s2 < 12; ++s2) db += pdb[s2 * 64 + tid];
      if (p.gated) db *= bet[tid] * (1.f - bet[tid] / p.beta_scale);  // through beta = s sigmoid(b)
      ((Tb *)p.dbeta)[((int64_t)b * T + t0 + tid) * H + h] = from_f<Tb>(db);
    }
  }
  fence_proxy_async_smem();
  __syncthreads();
  if (tid == 0) {
    if (p.gated)
      tma_store_rows(&tm.m[7], s_base + O_DR, h, t0, b);  // df (bf16)
    else
      tma_store_rows_f32(&tm.m[7], s_base + O_KF, h, t0, b);
    bulk_commit();
  }
  if (p.gated) {  // this chunk's shares of ddt_bias and dA_log
    if (tid >= 64 && tid < 128) {
      float sdt = 0.f;
#pragma unroll
      for (int s2 = 0; s2 < 8; ++s2) sdt += vec[V_GPT + s2 * 64 + tid - 64];
      atomicAdd(p.ddt_bias + h * 64 + tid - 64, sdt);
    } else if (tid == 128) {
      float sa = 0.f;
#pragma unroll
      for (int w = 0; w < CK_NT / 32; ++w) sa += vec[V_GPA + w];
      atomicAdd(p.dA_log + h, sa);
    }
  }
  BWD_TR(7);
  }  // chunk loop
  if (tid == 0) bulk_wait_all();  // shared memory stays valid until the stores have read it
}

template <typename Tb>
int launch(const Params &p, cudaStream_t st) {
  TmaMaps tm;  // 0 q, 1 k, 2 v, 3 dO, 4 g (loads); 5 dq, 6 dk, 7 dg (stores)
  const void *base[8] = {p.q, p.k, p.v, p.dO, p.gated ? p.f : (const void *)p.g, p.dq, p.dk,
                         p.gated ? p.df : (void *)p.dg};
  const Str in_str[5] = {p.sq, p.sk, p.sv, p.sdo, p.sg};  // the loads read strided inputs
  for (int i = 0; i < 8; ++i)
    if (int e = tma_map_bthd(&tm.m[i], base[i], p.B, p.T, p.H, D, (i == 4 || i == 7) && !p.gated,
                             i < 5 ? &in_str[i] : nullptr))
      return e;
  TmaMaps tms;
  tms.m[0] = tm.m[3];
  if (cudaFuncSetAttribute(kda_bwd_state_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SC_SMEM))
    return KDA_ERR_CUDA;
  kda_bwd_state_scan_kernel<<<p.B * p.H, SC_NT, SC_SMEM, st>>>(p, tms);
  count_launch();
  auto kern = kda_bwd_chunks_kernel<Tb>;
  const int ck_smem = CK_SMEM_GP + gate_smem_bytes(p.gated, p.H);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, ck_smem)) return KDA_ERR_CUDA;
  const int n = p.B * p.H * p.nc;
  int dev = 0, nsm = 148;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return KDA_ERR_CUDA;
  kern<<<n < nsm ? n : nsm, CK_NT, ck_smem, st>>>(p, tm);
  count_launch();
  return cudaPeekAtLastError() == cudaSuccess ? KDA_OK : KDA_ERR_CUDA;
}

}  // namespace tcbwd

int tc_bwd_device_status(bool reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, tcbwd::g_bwd_status, sizeof(int)) != cudaSuccess) return KDA_ERR_CUDA;
  if (reset && v) {
    const int z = 0;
    if (cudaMemcpyToSymbol(tcbwd::g_bwd_status, &z, sizeof(int)) != cudaSuccess) return KDA_ERR_CUDA;
  }
  return v;
}

size_t tc_bwd_workspace_bytes(const KdaDesc *d) {
  const int64_t n = d->B * d->H * ((d->T + d->chunk - 1) / d->chunk);
  return tcbwd::ws_bytes(n);
}

int tc_bwd(const Params &p, int dtype_beta, cudaStream_t st) {
  if (dtype_beta == KDA_BF16) return tcbwd::launch<__nv_bfloat16>(p, st);
  if (dtype_beta == KDA_F32) return tcbwd::launch<float>(p, st);
  return KDA_ERR_DTYPE;
}

}  // namespace kda

// ---------------------------------------------------------------------------------------
// kda_bwd_noalloc: kda_bwd with the workspace taken from a static device array.
//
// Some callers cannot allocate device memory: a host that owns all GPU memory through its own
// fixed pool and forbids other allocations, or one calling from a context where a cudaMalloc
// (which may synchronise the device) is not allowed.  This entry point needs no workspace from
// them.  Its scratch is the file-scope array below, KDA_NOALLOC_SCRATCH_BYTES bytes that every
// GPU that loads the library keeps until the process exits.  The first call on a device
// resolves the array's device address (cudaGetSymbolAddress, with that device current); make
// that first call before any stream capture.  All calls share the one array: calls whose
// kernels overlap on the GPU (different streams, or two host threads) race on it.  Nothing in
// it has to start at zero: each call overwrites every byte it reads back.
// ---------------------------------------------------------------------------------------

static __device__ __align__(256) uint8_t kda_noalloc_scratch[KDA_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void *g_noalloc_ptr[kMaxDevices] = {};
}  // namespace

extern "C" int kda_bwd_noalloc(const KdaDesc *d, const void *q, const void *k, const void *v,
                               const float *g, const void *beta, const float *state0,
                               const void *saved, const void *dO, const float *dstateT, void *dq,
                               void *dk, void *dv, float *dg, void *dbeta, float *dstate0,
                               void *stream) {
  const int s = kda_check_desc(d, 1);
  if (s) return s;
  const size_t need = kda_workspace_bytes(d, 1);
  if (need > (size_t)KDA_NOALLOC_SCRATCH_BYTES) return KDA_ERR_SCRATCH_LIMIT;
  void *scratch = nullptr;
  if (need) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return KDA_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
      void *ptr = nullptr;
      if (cudaGetSymbolAddress(&ptr, kda_noalloc_scratch) != cudaSuccess || !ptr) return KDA_ERR_CUDA;
      g_noalloc_ptr[dev] = ptr;
    }
    scratch = g_noalloc_ptr[dev];
  }
  return kda_bwd(d, q, k, v, g, beta, state0, saved, dO, dstateT, dq, dk, dv, dg, dbeta, dstate0,
                 scratch, need ? (size_t)KDA_NOALLOC_SCRATCH_BYTES : 0, stream);
}

#ifdef KDA_SCAN_TRACE
extern "C" __attribute__((visibility("default"))) int kda_bwd_trace(long long *out) {
  return cudaMemcpyFromSymbol(out, kda::tcbwd::g_bwd_trace, sizeof(long long) * 12 * 16) == cudaSuccess ? 0 : -1;
}
#endif
