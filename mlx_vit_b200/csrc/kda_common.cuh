// Shared device helpers for the KDA kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/kda_b200.h"

namespace kda {

// Kernel launch counter behind kda_launch_counter(); every launch site bumps it.
void count_launch();

// Element strides (batch, time, head) of one input; the last axis is unit-stride.
struct Str {
  int64_t b, t, h;
};
__device__ __forceinline__ int64_t at(const Str &s, int b, int t, int h, int d = 0) {
  return (int64_t)b * s.b + (int64_t)t * s.t + (int64_t)h * s.h + d;
}

// Kernel parameter block shared by every KDA kernel.  Outputs, states and records use the dense
// [B, T, H, D] / [B, T, H] / [B, H, Dv, Dk] layouts of the C ABI; the inputs carry strides.
struct Params {
  Str sq, sk, sv, sg, sb, sdo;  // input strides (f uses sg, the gate logits sb)
  int B, T, H, D, C, nc;       // D = Dk = Dv, C = chunk, nc = ceil(T / C)
  const void *q, *k, *v, *beta;
  const float *g, *state0, *dstateT;
  const void *saved_in;        // backward: what the forward saved
  void *ws;                    // workspace (caller-provided)
  const void *dO;
  void *o, *dq, *dk, *dv, *dbeta;
  float *stateT, *dg, *dstate0;
  void *saved;                 // forward: per-chunk record for the backward (may be null)
  int *err;                    // optional device error word
  // fused gates (kda_fwd_gated / kda_bwd_gated): g and beta come from f (dtype_qkv) and the
  // logits in `beta`; the backward writes df, the logit gradient in `dbeta`, dA_log, ddt_bias
  int gated, beta_scale;       // beta_scale: 2 with allow_neg_eigval, else 1
  const void *f;
  const float *A_log, *dt_bias;
  void *df;
  float *dA_log, *ddt_bias;
  // test hook (KDA_FLAG_DEBUG_WAIT_TIMEOUT): > 0 makes the forward's state scan first wait this
  // many polls on a barrier that nothing completes, so that its bounded-wait failure path runs
  int debug_wait_polls;
};

// softplus as the reference's (nope_gdn_mlx.py:83-86): log1p(e^{-|x|}) + max(x, 0)
// softplus(x) = max(x, 0) + log(1 + e^-|x|) with the fast intrinsics: the log argument is in
// (1, 2], where __logf's absolute error is about 2^-21, so g = -A softplus(.) carries an absolute
// error of a few 1e-7 A (the terms below 2^-24 that 1 + e^-|x| drops are smaller still)
__device__ __forceinline__ float softplus_f(float x) { return __logf(1.f + __expf(-fabsf(x))) + fmaxf(x, 0.f); }
__device__ __forceinline__ float sigmoid_f(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

// Per-chunk record the tensor-core forward saves for the tensor-core backward (D = C = 64):
// S0^T = transposed chunk-entry state [d][j], Unew [t][j], the decay-weighted P = Q K^T (lower incl.) and
// M = K K^T (strict lower) [t][s], Tinv = (I + beta M)^{-1} [t][s], Mneg = -Kb^T W [d'][d],
// Qt = Qd - P W [t][d] (all bf16, 64 x 64 with the 128-byte row swizzle of the shared-memory
// tiles, so that one bulk copy lands them ready for ldmatrix) and e^{gamma_C} [d] (fp32).
// With them the state cotangent obeys
//   dS_entry = dS_exit diag(e^{gamma_C}) + dS_exit Mneg + dO^T Qt
// and the chunk gradients need no triangular solve.
constexpr int kSavedS0 = 0, kSavedUnT = 8192, kSavedP = 16384, kSavedMkk = 24576, kSavedTinv = 32768;
constexpr int kSavedM = 40960, kSavedQt = 49152, kSavedEG = 57344;
constexpr int kSavedChunk = 57344 + 256;

template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

// Offset of element (b, t, h, d) in a dense [B, T, H, D] tensor.
__device__ __forceinline__ int64_t off_bthd(int b, int t, int h, int d, int T, int H, int D) {
  return (((int64_t)b * T + t) * H + h) * D + d;
}

}  // namespace kda
