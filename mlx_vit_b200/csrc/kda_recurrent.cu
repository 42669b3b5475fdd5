// Token-by-token KDA forward for decoding and short segments: the reference's step form
// (_kda_step_fused, nope_gdn_mlx.py:616-638, looped as in _loop_compiled_kda :890-917), exact
// in fp32.  No chunk padding, one launch, cost = reading and writing the state plus D^2 FMAs per
// token.
//
// Row j of the state (value index j, decay on the key columns d) evolves on its own:
//   S_j <- S_j * e^{g_t};   u_j = beta_t (v_tj - S_j . k_t);   S_j <- S_j + u_j k_t;   o_tj = S_j . q_t
// which is S (I - beta k k^T) + beta v k^T row by row.  One thread owns one row in registers; a
// CTA holds the D rows of one (b, h).  Each token's k, q and e^{g} go through a double-buffered
// shared vector (one barrier per token); the next token's inputs are loaded while this one
// computes.
#include "kda_common.cuh"

namespace kda {
namespace rec {

template <typename Tio, typename Tb, int D>
__global__ void __launch_bounds__(D) kda_recurrent_kernel(Params p) {
  __shared__ float kb[2][D], qb[2][D], eb[2][D];
  const int j = threadIdx.x, bh = blockIdx.x, b = bh / p.H, h = bh % p.H;
  const int T = p.T, H = p.H;
  const Tio *q = (const Tio *)p.q, *k = (const Tio *)p.k, *v = (const Tio *)p.v;
  const Tb *beta = (const Tb *)p.beta;
  Tio *o = (Tio *)p.o;
  float S[D];
  const int64_t srow = ((int64_t)bh * D + j) * D;
#pragma unroll
  for (int d = 0; d < D; ++d) S[d] = p.state0 ? p.state0[srow + d] : 0.f;

  // this thread's share of token t: element j of k, q, g and v, and beta
  float nk = 0.f, nq = 0.f, ng = 0.f, nv = 0.f, nb = 0.f;
  auto load = [&](int t) {
    const int64_t off = off_bthd(b, t, h, j, T, H, D);
    nk = to_f(k[off]);
    nq = to_f(q[off]);
    ng = p.g[off];
    nv = to_f(v[off]);
    nb = to_f(beta[((int64_t)b * T + t) * H + h]);
  };
  if (T > 0) load(0);
  for (int t = 0; t < T; ++t) {
    const int s = t & 1;
    kb[s][j] = nk;
    qb[s][j] = nq;
    eb[s][j] = expf(ng);
    const float vt = nv, bt = nb;
    __syncthreads();  // (the buffer written here was last read two tokens ago)
    if (t + 1 < T) load(t + 1);
    float dot = 0.f;
#pragma unroll
    for (int d = 0; d < D; ++d) {
      S[d] *= eb[s][d];
      dot = fmaf(S[d], kb[s][d], dot);
    }
    const float u = bt * (vt - dot);
    float out = 0.f;
#pragma unroll
    for (int d = 0; d < D; ++d) {
      S[d] = fmaf(u, kb[s][d], S[d]);
      out = fmaf(S[d], qb[s][d], out);
    }
    o[off_bthd(b, t, h, j, T, H, D)] = from_f<Tio>(out);
  }
#pragma unroll
  for (int d = 0; d < D; ++d) p.stateT[srow + d] = S[d];
}

template <typename Tio, typename Tb>
int launch_d(const Params &p, cudaStream_t st) {
  switch (p.D) {
    case 16: kda_recurrent_kernel<Tio, Tb, 16><<<p.B * p.H, 16, 0, st>>>(p); break;
    case 32: kda_recurrent_kernel<Tio, Tb, 32><<<p.B * p.H, 32, 0, st>>>(p); break;
    case 64: kda_recurrent_kernel<Tio, Tb, 64><<<p.B * p.H, 64, 0, st>>>(p); break;
    case 128: kda_recurrent_kernel<Tio, Tb, 128><<<p.B * p.H, 128, 0, st>>>(p); break;
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
