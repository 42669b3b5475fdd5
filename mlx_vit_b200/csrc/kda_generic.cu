// Generic fp32 SIMT KDA kernels: any chunk C <= 64 and head dim D <= 128 (forward) /
// D <= 64 (backward), any I/O dtype, arithmetic in fp32 FFMA with accurate expf.
//
// These are the fp32-exact kernels (the north-star fp32 tolerance is 1e-4 relative, which
// bf16/tf32 tensor-core products cannot meet) and the kernels for shapes the tensor-core
// kernels do not cover.  One CTA walks the chunks of one (b, h) sequentially, with the
// chunk's tiles, the state and the C x C chunk matrices resident in shared memory.
//
// Algebra per chunk (nope_gdn_mlx.py:549-613, 2318-2456), gamma = cumsum(g) inside the chunk:
//   A[t,s] = beta_t sum_d k_t k_s e^{min(gamma_t-gamma_s,0)}  (s <  t)   (kernel 3, :1301-1336)
//   P[t,s] =        sum_d q_t k_s e^{min(gamma_t-gamma_s,0)}  (s <= t)
//   U      = (I + A)^{-1} beta (V - (e^gamma k) S^T)                    (:600-603, kernel 1)
//   O      = (e^gamma q) S^T + P U                                      (:606-613)
//   S'     = S diag(e^{gamma_C}) + U^T (e^{gamma_C - gamma} k)
// The backward recomputes these per chunk from the saved chunk-entry states and applies
// the hand-derived VJP (the same quantities as :2579-2720, derived independently).
#include "kda_common.cuh"

namespace kda {

static constexpr int kGenThreads = 256;

// ---------------------------------------------------------------------------------------
// forward: grid (B*H, D / DVS), block kGenThreads
// smem floats: S[DVS*D] K[C*D] Q[C*D] Gm[C*D] V[C*DVS] A[C*C] P[C*C] U[C*DVS] bet[C] eG[D]
// ---------------------------------------------------------------------------------------
template <typename Tio, typename Tb>
__global__ void __launch_bounds__(kGenThreads)
kda_fwd_generic_kernel(Params p, int DVS) {
  extern __shared__ float sm[];
  const int D = p.D, C = p.C, T = p.T, H = p.H;
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const int j0 = blockIdx.y * DVS;
  const int tid = threadIdx.x, nt = blockDim.x;
  float *S = sm, *K = S + DVS * D, *Q = K + C * D, *Gm = Q + C * D, *V = Gm + C * D;
  float *A = V + C * DVS, *P = A + C * C, *U = P + C * C, *bet = U + C * DVS, *eG = bet + C;

  const Tio *q = (const Tio *)p.q, *k = (const Tio *)p.k, *v = (const Tio *)p.v;
  const Tb *beta = (const Tb *)p.beta;
  const int64_t sbase = (int64_t)bh * D * D;

  for (int i = tid; i < DVS * D; i += nt) {
    int j = i / D, d = i % D;
    S[i] = p.state0 ? p.state0[sbase + (int64_t)(j0 + j) * D + d] : 0.f;
  }
  __syncthreads();

  for (int c = 0; c < p.nc; ++c) {
    const int t0 = c * C;
    if (p.saved) {  // generic saved layout: fp32 chunk-entry state [bh][c][Dv][Dk]
      float *cs = (float *)p.saved + ((int64_t)bh * p.nc + c) * D * D;
      for (int i = tid; i < DVS * D; i += nt) cs[(int64_t)(j0 + i / D) * D + (i % D)] = S[i];
    }
    for (int i = tid; i < C * D; i += nt) {
      int t = i / D, d = i % D, tt = t0 + t;
      bool in = tt < T;
      K[i] = in ? to_f(k[at(p.sk, b, tt, h, d)]) : 0.f;
      Q[i] = in ? to_f(q[at(p.sq, b, tt, h, d)]) : 0.f;
      Gm[i] = in ? p.g[at(p.sg, b, tt, h, d)] : 0.f;
    }
    for (int i = tid; i < C * DVS; i += nt) {
      int t = i / DVS, j = i % DVS, tt = t0 + t;
      V[i] = tt < T ? to_f(v[at(p.sv, b, tt, h, j0 + j)]) : 0.f;
    }
    for (int t = tid; t < C; t += nt) {
      int tt = t0 + t;
      bet[t] = tt < T ? to_f(beta[at(p.sb, b, tt, h)]) : 0.f;
    }
    __syncthreads();
    for (int d = tid; d < D; d += nt) {  // gamma = cumsum(g) over the chunk
      float acc = 0.f;
      for (int t = 0; t < C; ++t) { acc += Gm[t * D + d]; Gm[t * D + d] = acc; }
      eG[d] = expf(acc);
    }
    __syncthreads();
    // A, P (C x C) and the right-hand side beta (V - K_proj S^T) into U
    for (int i = tid; i < C * C; i += nt) {
      int t = i / C, s = i % C;
      float sk = 0.f, sq = 0.f;
      if (s <= t) {
        for (int d = 0; d < D; ++d) {
          float e = expf(fminf(Gm[t * D + d] - Gm[s * D + d], 0.f));
          float ks = K[s * D + d] * e;
          sk = fmaf(K[t * D + d], ks, sk);
          sq = fmaf(Q[t * D + d], ks, sq);
        }
      }
      A[i] = s < t ? bet[t] * sk : 0.f;
      P[i] = sq;
    }
    for (int i = tid; i < C * DVS; i += nt) {
      int t = i / DVS, j = i % DVS;
      float acc = 0.f;
      for (int d = 0; d < D; ++d) acc = fmaf(K[t * D + d] * expf(Gm[t * D + d]), S[j * D + d], acc);
      U[i] = bet[t] * (V[i] - acc);
    }
    __syncthreads();
    // unit-lower forward substitution, one value column per thread
    for (int j = tid; j < DVS; j += nt) {
      for (int t = 1; t < C; ++t) {
        float u = U[t * DVS + j];
        for (int s = 0; s < t; ++s) u = fmaf(-A[t * C + s], U[s * DVS + j], u);
        U[t * DVS + j] = u;
      }
    }
    __syncthreads();
    // O = (e^gamma q) S^T + P U
    Tio *o = (Tio *)p.o;
    for (int i = tid; i < C * DVS; i += nt) {
      int t = i / DVS, j = i % DVS, tt = t0 + t;
      if (tt >= T) continue;
      float acc = 0.f;
      for (int d = 0; d < D; ++d) acc = fmaf(Q[t * D + d] * expf(Gm[t * D + d]), S[j * D + d], acc);
      for (int s = 0; s <= t; ++s) acc = fmaf(P[t * C + s], U[s * DVS + j], acc);
      o[off_bthd(b, tt, h, j0 + j, T, H, D)] = from_f<Tio>(acc);
    }
    __syncthreads();
    // S' = S diag(e^gamma_C) + U^T (e^{gamma_C - gamma} k)
    for (int i = tid; i < DVS * D; i += nt) {
      int j = i / D, d = i % D;
      float gl = Gm[(C - 1) * D + d];
      float acc = eG[d] * S[i];
      for (int t = 0; t < C; ++t) acc = fmaf(U[t * DVS + j], K[t * D + d] * expf(gl - Gm[t * D + d]), acc);
      S[i] = acc;
    }
    __syncthreads();
  }
  for (int i = tid; i < DVS * D; i += nt)
    p.stateT[sbase + (int64_t)(j0 + i / D) * D + (i % D)] = S[i];
}

// One chunk of the generic backward: S0 (chunk-entry state) and dS (state cotangent at the
// chunk's end) are already in shared memory; writes dq, dk, dv, dg, dbeta for the chunk's
// rows and, if update_dS, replaces dS by the cotangent of the chunk-entry state.
// smem floats: S0 dS [D*D]; K Q Gm Y(->DKp) dO U X1(dU->dR) DQ DKm [C*D]; M(->dKK) P(->dP)
// [C*C]; bet dbet [C]; eG dGam [D]
template <typename Tio, typename Tb>
__device__ void bwd_chunk_body(const Params &p, float *sm, int bh, int c, bool update_dS) {
  const int D = p.D, C = p.C, T = p.T, H = p.H;
  const int b = bh / H, h = bh % H;
  const int tid = threadIdx.x, nt = blockDim.x;
  float *S0 = sm, *dS = S0 + D * D;
  float *K = dS + D * D, *Q = K + C * D, *Gm = Q + C * D, *Y = Gm + C * D, *dO = Y + C * D;
  float *U = dO + C * D, *X1 = U + C * D, *DQ = X1 + C * D, *DKm = DQ + C * D;
  float *M = DKm + C * D, *P = M + C * C, *bet = P + C * C, *dbet = bet + C, *eG = dbet + C;
  float *dGam = eG + D;
  const Tio *q = (const Tio *)p.q, *k = (const Tio *)p.k, *v = (const Tio *)p.v;
  const Tio *dOg = (const Tio *)p.dO;
  const Tb *beta = (const Tb *)p.beta;
  const int t0 = c * C;
  for (int i = tid; i < C * D; i += nt) {
    int t = i / D, d = i % D, tt = t0 + t;
    bool in = tt < T;
    K[i] = in ? to_f(k[at(p.sk, b, tt, h, d)]) : 0.f;
    Q[i] = in ? to_f(q[at(p.sq, b, tt, h, d)]) : 0.f;
    Gm[i] = in ? p.g[at(p.sg, b, tt, h, d)] : 0.f;
    Y[i] = in ? to_f(v[at(p.sv, b, tt, h, d)]) : 0.f;
    dO[i] = in ? to_f(dOg[at(p.sdo, b, tt, h, d)]) : 0.f;
  }
  for (int t = tid; t < C; t += nt) {
    int tt = t0 + t;
    bet[t] = tt < T ? to_f(beta[at(p.sb, b, tt, h)]) : 0.f;
  }
  __syncthreads();
  for (int d = tid; d < D; d += nt) {
    float acc = 0.f;
    for (int t = 0; t < C; ++t) { acc += Gm[t * D + d]; Gm[t * D + d] = acc; }
    eG[d] = expf(acc);
  }
  __syncthreads();
  // M[t,s] = sum_d k_t k_s E (s<t), P[t,s] = sum_d q_t k_s E (s<=t); Y = V - Kd S0^T
  for (int i = tid; i < C * C; i += nt) {
    int t = i / C, s = i % C;
    float sk = 0.f, sq = 0.f;
    if (s <= t) {
      for (int d = 0; d < D; ++d) {
        float e = expf(fminf(Gm[t * D + d] - Gm[s * D + d], 0.f));
        float ks = K[s * D + d] * e;
        sk = fmaf(K[t * D + d], ks, sk);
        sq = fmaf(Q[t * D + d], ks, sq);
      }
    }
    M[i] = s < t ? sk : 0.f;
    P[i] = sq;
  }
  for (int i = tid; i < C * D; i += nt) {
    int t = i / D, j = i % D;
    float acc = 0.f;
    for (int d = 0; d < D; ++d) acc = fmaf(K[t * D + d] * expf(Gm[t * D + d]), S0[j * D + d], acc);
    float y = Y[i] - acc;
    Y[i] = y;
    U[i] = bet[t] * y;
  }
  __syncthreads();
  for (int j = tid; j < D; j += nt) {  // U = (I + diag(beta) M)^{-1} beta Y
    for (int t = 1; t < C; ++t) {
      float u = U[t * D + j];
      for (int s = 0; s < t; ++s) u = fmaf(-bet[t] * M[t * C + s], U[s * D + j], u);
      U[t * D + j] = u;
    }
  }
  __syncthreads();
  // dU = P^T dO + Kb dS^T ;  DQ = (dO S0) e^gamma
  for (int i = tid; i < C * D; i += nt) {
    int t = i / D, j = i % D;
    float acc = 0.f;
    for (int tp = t; tp < C; ++tp) acc = fmaf(P[tp * C + t], dO[tp * D + j], acc);
    for (int d = 0; d < D; ++d)
      acc = fmaf(K[t * D + d] * expf(Gm[(C - 1) * D + d] - Gm[t * D + d]), dS[j * D + d], acc);
    X1[i] = acc;
    int dd = j;  // reuse the same (t, d) index for DQ
    float aq = 0.f;
    for (int jj = 0; jj < D; ++jj) aq = fmaf(dO[t * D + jj], S0[jj * D + dd], aq);
    DQ[i] = aq * expf(Gm[t * D + dd]);
  }
  __syncthreads();
  // dP[t,s] = dO_t . U_s (s <= t), overwrites P;  then dR = (I + A)^{-T} dU in X1
  for (int i = tid; i < C * C; i += nt) {
    int t = i / C, s = i % C;
    float acc = 0.f;
    if (s <= t)
      for (int j = 0; j < D; ++j) acc = fmaf(dO[t * D + j], U[s * D + j], acc);
    P[i] = acc;
  }
  for (int j = tid; j < D; j += nt) {
    for (int t = C - 2; t >= 0; --t) {
      float r = X1[t * D + j];
      for (int tp = t + 1; tp < C; ++tp) r = fmaf(-bet[tp] * M[tp * C + t], X1[tp * D + j], r);
      X1[t * D + j] = r;
    }
  }
  __syncthreads();
  // dbeta_t = dR_t . Y_t + sum_s dA[t,s] M[t,s] with dA = -(dR U^T) strict-lower;
  // M row t becomes dKK[t,s] = beta_t dA[t,s]
  for (int t = tid; t < C; t += nt) {
    float db = 0.f;
    for (int j = 0; j < D; ++j) db = fmaf(X1[t * D + j], Y[t * D + j], db);
    for (int s = 0; s < t; ++s) {
      float da = 0.f;
      for (int j = 0; j < D; ++j) da = fmaf(X1[t * D + j], U[s * D + j], da);
      da = -da;
      db = fmaf(da, M[t * C + s], db);
      M[t * C + s] = bet[t] * da;
    }
    dbet[t] = db;
  }
  __syncthreads();
  // DQ += sum_{s<=t} dP[t,s] k_s E_ts
  // DKp (into Y) = -beta_t e^gamma_t (dR_t S0) + sum_{s<t} dKK[t,s] k_s E_ts
  // DKm first term = e^{gamma_C-gamma_t} (U_t dS)
  for (int i = tid; i < C * D; i += nt) {
    int t = i / D, d = i % D;
    const float gt = Gm[t * D + d];
    float aq = DQ[i], ap = 0.f;
    for (int s = 0; s <= t; ++s) {
      float ks = K[s * D + d] * expf(fminf(gt - Gm[s * D + d], 0.f));
      aq = fmaf(P[t * C + s], ks, aq);
      ap = fmaf(M[t * C + s], ks, ap);  // M[t,t] == 0
    }
    float rs = 0.f, us = 0.f;
    for (int j = 0; j < D; ++j) {
      rs = fmaf(X1[t * D + j], S0[j * D + d], rs);
      us = fmaf(U[t * D + j], dS[j * D + d], us);
    }
    DQ[i] = aq;
    Y[i] = ap - bet[t] * expf(gt) * rs;
    DKm[i] = us * expf(Gm[(C - 1) * D + d] - gt);
  }
  __syncthreads();
  // dGamma_C[d] = sum_t k_t DKm_t + e^{gamma_C} sum_j S0[j,d] dS[j,d]
  for (int d = tid; d < D; d += nt) {
    float a = 0.f, s2 = 0.f;
    for (int t = 0; t < C; ++t) a = fmaf(K[t * D + d], DKm[t * D + d], a);
    for (int j = 0; j < D; ++j) s2 = fmaf(S0[j * D + d], dS[j * D + d], s2);
    dGam[d] = a + eG[d] * s2;
  }
  __syncthreads();
  // DKm += sum_{t'>t} dKK[t',t] k_t' E + sum_{t'>=t} dP[t',t] q_t' E
  for (int i = tid; i < C * D; i += nt) {
    int t = i / D, d = i % D;
    const float gt = Gm[t * D + d];
    float a = DKm[i];
    for (int tp = t; tp < C; ++tp) {
      float e = expf(fminf(Gm[tp * D + d] - gt, 0.f));
      a = fmaf((M[tp * C + t] * K[tp * D + d] + P[tp * C + t] * Q[tp * D + d]), e, a);
    }
    DKm[i] = a;
  }
  __syncthreads();
  // dgamma = q dq + k DKp - k DKm (+ dGamma_C on the last row); dg = reverse cumsum;
  // write dq, dk, dv, dg, dbeta for the chunk's valid rows
  {
    Tio *dqg = (Tio *)p.dq, *dkg = (Tio *)p.dk, *dvg = (Tio *)p.dv;
    for (int d = tid; d < D; d += nt) {
      float acc = 0.f;
      for (int t = C - 1; t >= 0; --t) {
        int i = t * D + d;
        float dgam = Q[i] * DQ[i] + K[i] * (Y[i] - DKm[i]) + (t == C - 1 ? dGam[d] : 0.f);
        acc += dgam;
        int tt = t0 + t;
        if (tt < T) p.dg[off_bthd(b, tt, h, d, T, H, D)] = acc;
      }
    }
    for (int i = tid; i < C * D; i += nt) {
      int t = i / D, d = i % D, tt = t0 + t;
      if (tt >= T) continue;
      int64_t o = off_bthd(b, tt, h, d, T, H, D);
      dqg[o] = from_f<Tio>(DQ[i]);
      dkg[o] = from_f<Tio>(Y[i] + DKm[i]);
      dvg[o] = from_f<Tio>(bet[t] * X1[i]);
    }
    Tb *dbg = (Tb *)p.dbeta;
    for (int t = tid; t < C; t += nt)
      if (t0 + t < T) dbg[((int64_t)b * T + t0 + t) * H + h] = from_f<Tb>(dbet[t]);
  }
  if (!update_dS) return;
  // dS <- dS diag(e^gamma_C) + dO^T (e^gamma q) - (beta dR)^T (e^gamma k)
  for (int i = tid; i < D * D; i += nt) {
    int j = i / D, d = i % D;
    float acc = eG[d] * dS[i];
    for (int t = 0; t < C; ++t) {
      float eg = expf(Gm[t * D + d]);
      acc = fmaf(dO[t * D + j], Q[t * D + d] * eg, acc);
      acc = fmaf(-bet[t] * X1[t * D + j], K[t * D + d] * eg, acc);
    }
    dS[i] = acc;
  }
  __syncthreads();
}

template <typename Tio, typename Tb>
__global__ void __launch_bounds__(kGenThreads)
kda_bwd_generic_kernel(Params p) {
  extern __shared__ float sm[];
  const int D = p.D;
  const int bh = blockIdx.x;
  const int tid = threadIdx.x, nt = blockDim.x;
  float *S0 = sm, *dS = S0 + D * D;
  const int64_t sbase = (int64_t)bh * D * D;
  for (int i = tid; i < D * D; i += nt) dS[i] = p.dstateT ? p.dstateT[sbase + i] : 0.f;
  for (int c = p.nc - 1; c >= 0; --c) {
    const float *cs = (const float *)p.saved_in + ((int64_t)bh * p.nc + c) * D * D;
    for (int i = tid; i < D * D; i += nt) S0[i] = cs[i];
    bwd_chunk_body<Tio, Tb>(p, sm, bh, c, true);
  }
  if (p.dstate0)
    for (int i = tid; i < D * D; i += nt) p.dstate0[sbase + i] = dS[i];
}

// ---------------------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------------------
size_t generic_fwd_smem(int D, int C, int dvs) {
  return sizeof(float) * ((size_t)dvs * D + 3 * C * D + 2 * C * dvs + 2 * C * C + C + D);
}
size_t generic_bwd_smem(int D, int C) {
  return sizeof(float) * ((size_t)2 * D * D + 9 * C * D + 2 * C * C + 2 * C + 2 * D);
}
static constexpr size_t kMaxSmem = 227 * 1024;

// The chunk the fp32 kernels run at: the caller's chunk C, or the largest smaller one whose
// backward working set fits shared memory, halving C (D = 96 runs at 32, D = 128 at 16).  The chunkwise
// algebra gives the recurrence's values at any chunk size, so this changes only rounding; the
// forward and the backward of one descriptor use the same chunk, so the saved per-chunk states
// line up.  0 if none fits.
int generic_fwd_split(int D, int C);
int generic_chunk(int D, int C) {
  for (int c = C; c >= 1; c /= 2)
    if (generic_bwd_smem(D, c) <= kMaxSmem && generic_fwd_split(D, c)) return c;
  return 0;
}
int generic_fwd_split(int D, int C) {
  for (int dvs = D; dvs >= 1; --dvs) {
    if (D % dvs) continue;
    if (dvs > 64) continue;
    if (generic_fwd_smem(D, C, dvs) <= kMaxSmem) return dvs;
  }
  return 0;
}

template <typename Tio, typename Tb>
static int launch_fwd_t(const Params &p, cudaStream_t st) {
  int dvs = generic_fwd_split(p.D, p.C);
  if (!dvs) return KDA_ERR_UNSUPPORTED;
  size_t smem = generic_fwd_smem(p.D, p.C, dvs);
  auto kern = kda_fwd_generic_kernel<Tio, Tb>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return KDA_ERR_CUDA;
  dim3 grid(p.B * p.H, p.D / dvs);
  kern<<<grid, kGenThreads, smem, st>>>(p, dvs);
  count_launch();
  return cudaPeekAtLastError() == cudaSuccess ? KDA_OK : KDA_ERR_CUDA;
}

template <typename Tio, typename Tb>
static int launch_bwd_t(const Params &p, cudaStream_t st) {
  size_t smem = generic_bwd_smem(p.D, p.C);
  if (smem > kMaxSmem) return KDA_ERR_UNSUPPORTED;
  auto kern = kda_bwd_generic_kernel<Tio, Tb>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return KDA_ERR_CUDA;
  kern<<<p.B * p.H, kGenThreads, smem, st>>>(p);
  count_launch();
  return cudaPeekAtLastError() == cudaSuccess ? KDA_OK : KDA_ERR_CUDA;
}

#define KDA_DISPATCH_IO(dq, db, FN, ...)                                                   \
  do {                                                                                     \
    if (dq == KDA_F32 && db == KDA_F32) return FN<float, float>(__VA_ARGS__);               \
    if (dq == KDA_BF16 && db == KDA_BF16) return FN<__nv_bfloat16, __nv_bfloat16>(__VA_ARGS__); \
    if (dq == KDA_BF16 && db == KDA_F32) return FN<__nv_bfloat16, float>(__VA_ARGS__);      \
    if (dq == KDA_F16 && db == KDA_F16) return FN<__half, __half>(__VA_ARGS__);             \
    if (dq == KDA_F16 && db == KDA_F32) return FN<__half, float>(__VA_ARGS__);              \
    if (dq == KDA_F32 && db == KDA_BF16) return FN<float, __nv_bfloat16>(__VA_ARGS__);      \
    return KDA_ERR_DTYPE;                                                                  \
  } while (0)

int generic_fwd(const Params &p, int dq, int db, cudaStream_t st) {
  KDA_DISPATCH_IO(dq, db, launch_fwd_t, p, st);
}
int generic_bwd(const Params &p, int dq, int db, cudaStream_t st) {
  KDA_DISPATCH_IO(dq, db, launch_bwd_t, p, st);
}

}  // namespace kda
