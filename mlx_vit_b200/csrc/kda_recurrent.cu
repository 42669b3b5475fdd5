// Token-by-token KDA forward for decoding and short segments: the reference's step form
// (_kda_step_fused, nope_gdn_mlx.py:616-638, looped as in _loop_compiled_kda :890-917), exact
// in fp32.  No chunk padding, one launch, cost = reading and writing the state plus D^2 FMAs per
// token.
//
// Row j of the state (value index j, decay on the key columns d) evolves on its own:
//   S_j <- S_j * e^{g_t};   u_j = beta_t (v_tj - S_j . k_t);   S_j <- S_j + u_j k_t;   o_tj = S_j . q_t
// which is S (I - beta k k^T) + beta v k^T row by row.  A row lives in the registers of one thread
// (two at D = 128); a CTA holds up to 32 rows of one (b, h).  Each token's k, q and e^{g} go through a double-buffered
// shared vector (one barrier per token); the next token's inputs are loaded while this one
// computes.
#include "kda_common.cuh"

namespace kda {
namespace rec {

// One CTA owns R = min(D, 32) consecutive rows of one (b, h) state, with P = D / 64 threads per
// row at D = 128 (each holding 64 columns; the two halves' dot products meet through a shuffle)
// and one thread per row otherwise.  The rows are contiguous in memory, so the state moves between
// HBM and registers through a padded shared slab with coalesced loads and stores.
template <typename Tio, typename Tb, int D>
__global__ void __launch_bounds__((D < 32 ? D : 32) * (D > 64 ? 2 : 1)) kda_recurrent_kernel(Params p) {
  constexpr int R = D < 32 ? D : 32, P = D > 64 ? 2 : 1, NT = R * P, W = D / P, PER = (D + NT - 1) / NT;
  __shared__ float slab[R][D + 1];
  __shared__ float kb[2][D], qb[2][D], eb[2][D];
  const int tid = threadIdx.x, r = tid / P, part = tid % P, c0 = part * W;
  const int bh = blockIdx.x, b = bh / p.H, h = bh % p.H;
  const int j = blockIdx.y * R + r;
  const int T = p.T, H = p.H;
  const Tio *q = (const Tio *)p.q, *k = (const Tio *)p.k, *v = (const Tio *)p.v;
  const Tb *beta = (const Tb *)p.beta;
  Tio *o = (Tio *)p.o;
  const int64_t sbase = ((int64_t)bh * D + blockIdx.y * R) * D;  // first element of the slab
  for (int i = tid; i < R * D; i += NT) slab[i / D][i % D] = p.state0 ? p.state0[sbase + i] : 0.f;
  __syncthreads();
  float S[W];
#pragma unroll
  for (int d = 0; d < W; ++d) S[d] = slab[r][c0 + d];

  // this thread's share of token t: elements tid, tid + NT, ... of k, q, g; v of its row; beta
  float nk[PER], nq[PER], ng[PER], nv = 0.f, nb = 0.f;
  auto load = [&](int t) {
#pragma unroll
    for (int m = 0; m < PER; ++m) {
      const int d = tid + NT * m;
      if (d < D) {
        nk[m] = to_f(k[at(p.sk, b, t, h, d)]);
        nq[m] = to_f(q[at(p.sq, b, t, h, d)]);
        ng[m] = p.g[at(p.sg, b, t, h, d)];
      }
    }
    nv = to_f(v[at(p.sv, b, t, h, j)]);
    nb = to_f(beta[at(p.sb, b, t, h)]);
  };
  if (T > 0) load(0);
  for (int t = 0; t < T; ++t) {
    const int s = t & 1;
#pragma unroll
    for (int m = 0; m < PER; ++m) {
      const int d = tid + NT * m;
      if (d < D) {
        kb[s][d] = nk[m];
        qb[s][d] = nq[m];
        eb[s][d] = expf(ng[m]);
      }
    }
    const float vt = nv, bt = nb;
    __syncthreads();  // (the buffer written here was last read two tokens ago)
    if (t + 1 < T) load(t + 1);
    float dot = 0.f;
#pragma unroll
    for (int d = 0; d < W; ++d) {
      S[d] *= eb[s][c0 + d];
      dot = fmaf(S[d], kb[s][c0 + d], dot);
    }
    if (P == 2) dot += __shfl_xor_sync(0xffffffffu, dot, 1);
    const float u = bt * (vt - dot);
    float out = 0.f;
#pragma unroll
    for (int d = 0; d < W; ++d) {
      S[d] = fmaf(u, kb[s][c0 + d], S[d]);
      out = fmaf(S[d], qb[s][c0 + d], out);
    }
    if (P == 2) out += __shfl_xor_sync(0xffffffffu, out, 1);
    if (part == 0) o[off_bthd(b, t, h, j, T, H, D)] = from_f<Tio>(out);
  }
  __syncthreads();  // every thread is done reading the slab it was loaded from
#pragma unroll
  for (int d = 0; d < W; ++d) slab[r][c0 + d] = S[d];
  __syncthreads();
  for (int i = tid; i < R * D; i += NT) p.stateT[sbase + i] = slab[i / D][i % D];
}

template <typename Tio, typename Tb>
int launch_d(const Params &p, cudaStream_t st) {
  switch (p.D) {
    case 16: kda_recurrent_kernel<Tio, Tb, 16><<<dim3(p.B * p.H, 16 / 16), 16, 0, st>>>(p); break;
    case 32: kda_recurrent_kernel<Tio, Tb, 32><<<dim3(p.B * p.H, 32 / 32), 32, 0, st>>>(p); break;
    case 64: kda_recurrent_kernel<Tio, Tb, 64><<<dim3(p.B * p.H, 64 / 32), 32, 0, st>>>(p); break;
    case 128: kda_recurrent_kernel<Tio, Tb, 128><<<dim3(p.B * p.H, 128 / 32), 64, 0, st>>>(p); break;
    default: return KDA_ERR_UNSUPPORTED;
  }
  count_launch();
  return cudaPeekAtLastError() == cudaSuccess ? KDA_OK : KDA_ERR_CUDA;
}
template <typename Tio>
int launch_b(const Params &p, int db, cudaStream_t st) {
  switch (db) {
    case KDA_F32: return launch_d<Tio, float>(p, st);
    case KDA_BF16: return launch_d<Tio, __nv_bfloat16>(p, st);
    case KDA_F16: return launch_d<Tio, __half>(p, st);
  }
  return KDA_ERR_DTYPE;
}

}  // namespace rec

bool recurrent_supported(int D) { return D == 16 || D == 32 || D == 64 || D == 128; }

int recurrent_fwd(const Params &p, int dq, int db, cudaStream_t st) {
  switch (dq) {
    case KDA_F32: return rec::launch_b<float>(p, db, st);
    case KDA_BF16: return rec::launch_b<__nv_bfloat16>(p, db, st);
    case KDA_F16: return rec::launch_b<__half>(p, db, st);
  }
  return KDA_ERR_DTYPE;
}

}  // namespace kda
