// The GDN layer's row operations around the recurrence, fused into one pass each (bf16 I/O,
// fp32 arithmetic):
//
//   prologue  y = l2norm(silu(x)) * scale     q and k after the short convolutions, the norm
//             taken over the whole H*D channel row as the reference does before its head
//             reshape (nope_gdn_mlx.py:797-799 with l2_normalize :76-79: x / max(||x||, 1e-12);
//             reshape :818-821); one CTA per row, a block reduction
//   epilogue  y = rmsnorm(o) * w * sigmoid(gate)   the output's gated RMSNorm over each head's
//             D channels (RMSNormGated(D) / _gated_rms_norm :340-371 on the (B, L, H, D)
//             output, :880-885); one warp per row
//
// and their VJPs.  The backward of the prologue recomputes silu(x) and the norm from x; the
// backward of the epilogue recomputes the RMS from o and reduces dw over rows with one atomic
// per channel per CTA.
#include <initializer_list>
#include <mutex>

#include "kda_common.cuh"

namespace kda {
namespace rowops {

constexpr int kWarps = 8;  // rows per CTA pass

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float sigm(float x) { return 1.f / (1.f + __expf(-x)); }

// E = elements per lane (D / 32): lane l holds columns l*E .. l*E+E-1
template <int E>
__device__ __forceinline__ void load_row(const __nv_bfloat16 *p, int lane, float (&x)[E]) {
  const __nv_bfloat162 *q = reinterpret_cast<const __nv_bfloat162 *>(p + lane * E);
#pragma unroll
  for (int i = 0; i < E / 2; ++i) {
    const float2 f = __bfloat1622float2(q[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}
template <int E>
__device__ __forceinline__ void store_row(__nv_bfloat16 *p, int lane, const float (&x)[E]) {
  __nv_bfloat162 *q = reinterpret_cast<__nv_bfloat162 *>(p + lane * E);
#pragma unroll
  for (int i = 0; i < E / 2; ++i) q[i] = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
}

// ---- row-wide L2 norm: one CTA of kRowThreads per row of n channels (the layer's whole H*D
// row, which the reference normalises before its head reshape, nope_gdn_mlx.py:797-799 then
// :818-821).  A thread owns chunks of 8 consecutive channels (16-byte loads), chunk
// tid + kRowThreads * k for k < KC, so n <= 8 * kRowThreads * KC. ----
constexpr int kRowThreads = 128;
constexpr int kRowMaxChunks = 8;  // n <= 8192

// sum over the CTA; `red` holds two slots per warp so that consecutive rows need one barrier each
__device__ __forceinline__ float2 block_sum2(float2 v, float2 (*red)[kRowThreads / 32], int parity) {
  v.x = warp_sum(v.x);
  v.y = warp_sum(v.y);
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  if (lane == 0) red[parity][wp] = v;
  __syncthreads();
  float2 s = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < kRowThreads / 32; ++i) {
    s.x += red[parity][i].x;
    s.y += red[parity][i].y;
  }
  return s;
}

__device__ __forceinline__ void load8(const __nv_bfloat16 *p, float (&x)[8]) {
  const uint4 u = *reinterpret_cast<const uint4 *>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[e]));
    x[2 * e] = f.x;
    x[2 * e + 1] = f.y;
  }
}
__device__ __forceinline__ void store8(__nv_bfloat16 *p, const float (&x)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    __nv_bfloat162 v = __floats2bfloat162_rn(x[2 * e], x[2 * e + 1]);
    w[e] = *reinterpret_cast<uint32_t *>(&v);
  }
  *reinterpret_cast<uint4 *>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}

template <int KC>
__global__ void __launch_bounds__(kRowThreads) l2norm_silu_fwd_kernel(int64_t rows, int n, const __nv_bfloat16 *x,
                                                                      __nv_bfloat16 *y, float scale) {
  __shared__ float2 red[2][kRowThreads / 32];
  const int nch = n >> 3;
  int parity = 0;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x, parity ^= 1) {
    float v[KC][8];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < KC; ++k) {
      const int c = threadIdx.x + kRowThreads * k;
      if (c < nch) {
        load8(x + r * n + 8 * c, v[k]);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          v[k][i] *= sigm(v[k][i]);
          ss += v[k][i] * v[k][i];
        }
      }
    }
    const float inv = scale / fmaxf(sqrtf(block_sum2(make_float2(ss, 0.f), red, parity).x), 1e-12f);
#pragma unroll
    for (int k = 0; k < KC; ++k) {
      const int c = threadIdx.x + kRowThreads * k;
      if (c < nch) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[k][i] *= inv;
        store8(y + r * n + 8 * c, v[k]);
      }
    }
  }
}

// y = scale s / max(N, eps), s = silu(x), N = ||s|| over the row:
//   ds = scale (dy - s (s . dy) / N^2) / N  (N > eps; else scale dy / eps);  dx = ds silu'(x)
template <int KC>
__global__ void __launch_bounds__(kRowThreads) l2norm_silu_bwd_kernel(int64_t rows, int n, const __nv_bfloat16 *x,
                                                                      const __nv_bfloat16 *dy,
                                                                      __nv_bfloat16 *dx, float scale) {
  __shared__ float2 red[2][kRowThreads / 32];
  const int nch = n >> 3;
  int parity = 0;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x, parity ^= 1) {
    float v[KC][8], g[KC][8];
    float ss = 0.f, sg = 0.f;
#pragma unroll
    for (int k = 0; k < KC; ++k) {
      const int c = threadIdx.x + kRowThreads * k;
      if (c < nch) {
        load8(x + r * n + 8 * c, v[k]);
        load8(dy + r * n + 8 * c, g[k]);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float s = v[k][i] * sigm(v[k][i]);
          ss += s * s;
          sg += s * g[k][i];
        }
      }
    }
    const float2 red2 = block_sum2(make_float2(ss, sg), red, parity);
    const float N = sqrtf(red2.x);
    const bool clamp = !(N > 1e-12f);
    const float inv = scale / (clamp ? 1e-12f : N), proj = clamp ? 0.f : red2.y / red2.x;
#pragma unroll
    for (int k = 0; k < KC; ++k) {
      const int c = threadIdx.x + kRowThreads * k;
      if (c < nch) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float sgm = sigm(v[k][i]), s = v[k][i] * sgm;
          const float ds = inv * (g[k][i] - s * proj);
          g[k][i] = ds * sgm * (1.f + v[k][i] * (1.f - sgm));
        }
        store8(dx + r * n + 8 * c, g[k]);
      }
    }
  }
}

template <int E>
__global__ void __launch_bounds__(32 * kWarps) gated_rmsnorm_fwd_kernel(int64_t rows, const __nv_bfloat16 *o,
                                                                        const __nv_bfloat16 *gate, const float *w,
                                                                        __nv_bfloat16 *y, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t stride = (int64_t)gridDim.x * kWarps;
  float wl[E];
#pragma unroll
  for (int i = 0; i < E; ++i) wl[i] = w[lane * E + i];
  for (int64_t r = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); r < rows; r += stride) {
    float v[E], g[E];
    load_row<E>(o + r * 32 * E, lane, v);
    load_row<E>(gate + r * 32 * E, lane, g);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < E; ++i) ss += v[i] * v[i];
    const float rr = rsqrtf(warp_sum(ss) / (32 * E) + eps);
#pragma unroll
    for (int i = 0; i < E; ++i) v[i] = v[i] * rr * wl[i] * sigm(g[i]);
    store_row<E>(y + r * 32 * E, lane, v);
  }
}

// n = o r, r = rsqrt(mean(o^2) + eps), y = n w sigmoid(gate):
//   dgate = dy n w s (1 - s);  dw += dy n s;  dn = dy w s;  do = r (dn - n mean(dn n))
template <int E>
__global__ void __launch_bounds__(32 * kWarps) gated_rmsnorm_bwd_kernel(int64_t rows, const __nv_bfloat16 *o,
                                                                        const __nv_bfloat16 *gate, const float *w,
                                                                        const __nv_bfloat16 *dy, __nv_bfloat16 *dout,
                                                                        __nv_bfloat16 *dgate, float *dw, float eps) {
  __shared__ float red[kWarps][32 * E];
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  const int64_t stride = (int64_t)gridDim.x * kWarps;
  float wl[E], dwl[E];
#pragma unroll
  for (int i = 0; i < E; ++i) {
    wl[i] = w[lane * E + i];
    dwl[i] = 0.f;
  }
  for (int64_t r = (int64_t)blockIdx.x * kWarps + wp; r < rows; r += stride) {
    float v[E], g[E], d[E];
    load_row<E>(o + r * 32 * E, lane, v);
    load_row<E>(gate + r * 32 * E, lane, g);
    load_row<E>(dy + r * 32 * E, lane, d);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < E; ++i) ss += v[i] * v[i];
    const float rr = rsqrtf(warp_sum(ss) / (32 * E) + eps);
    float dnn = 0.f;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const float n = v[i] * rr, s = sigm(g[i]);
      dwl[i] += d[i] * n * s;
      const float dn = d[i] * wl[i] * s;
      g[i] = d[i] * n * wl[i] * s * (1.f - s);  // dgate
      v[i] = n;
      d[i] = dn;
      dnn += dn * n;
    }
    const float m = warp_sum(dnn) / (32 * E);
#pragma unroll
    for (int i = 0; i < E; ++i) d[i] = rr * (d[i] - v[i] * m);
    store_row<E>(dout + r * 32 * E, lane, d);
    store_row<E>(dgate + r * 32 * E, lane, g);
  }
#pragma unroll
  for (int i = 0; i < E; ++i) red[wp][lane * E + i] = dwl[i];
  __syncthreads();
  for (int c = threadIdx.x; c < 32 * E; c += 32 * kWarps) {
    float a = 0.f;
#pragma unroll
    for (int k = 0; k < kWarps; ++k) a += red[k][c];
    atomicAdd(dw + c, a);
  }
}

// Short causal depthwise convolution (kernel 4, the reference's ShortCausalConv1d,
// nope_gdn_mlx.py:400-431: z[t, c] = b[c] + sum_j w[c, j] x[t - 3 + j, c], zeros before t = 0)
// followed by SiLU, and for q / k by the L2 norm over the whole C = H D channel row (the
// reference normalises before its head reshape, :797-799 then :818-821) and the scale.  x, y:
// [B, T, C] bf16 (C at most kConvMaxC); w [C][4], b [C] fp32.  A CTA walks kConvRows consecutive
// rows of one sequence with one thread per 4 channels (blockDim = C / 4 rounded up to a warp):
// the thread keeps its weights and the last three input rows in registers (a sliding window, so
// every input row is read once) and the rows go kConvG at a time through one block reduction of
// their norms.
constexpr int kConvRows = 16, kConvG = 4, kConvV = 4;  // rows per CTA, per reduction; channels per thread
constexpr int kConvMaxC = 2048;                         // 512 threads of 4 channels

__device__ __forceinline__ void load4(const __nv_bfloat16 *p, float (&x)[4]) {
  const uint2 u = *reinterpret_cast<const uint2 *>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.y));
  x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
}
__device__ __forceinline__ void store4(__nv_bfloat16 *p, const float (&x)[4]) {
  __nv_bfloat162 a = __floats2bfloat162_rn(x[0], x[1]), b = __floats2bfloat162_rn(x[2], x[3]);
  *reinterpret_cast<uint2 *>(p) = make_uint2(*reinterpret_cast<uint32_t *>(&a), *reinterpret_cast<uint32_t *>(&b));
}

// sums of G per-row partials over the CTA (nw warps, at most 16); red holds two slots per warp
template <int G>
__device__ __forceinline__ void block_sums(const float (&v)[G], float (&out)[G], float (*red)[16][G], int parity,
                                           int nw) {
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float x = warp_sum(v[g]);
    if (lane == 0) red[parity][wp][g] = x;
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float s = 0.f;
    for (int i = 0; i < nw; ++i) s += red[parity][i][g];
    out[g] = s;
  }
}

struct ConvThread {  // one thread's channels: weights, bias and the input window
  float w[kConvV][4], bias[kConvV], win[3][kConvV];
  __device__ __forceinline__ void init(int b, int t0, int T, int C, int c0, const __nv_bfloat16 *x,
                                       const float *wg, const float *bg) {
#pragma unroll
    for (int i = 0; i < kConvV; ++i) {
      const float4 q = *reinterpret_cast<const float4 *>(wg + (c0 + i) * 4);
      w[i][0] = q.x; w[i][1] = q.y; w[i][2] = q.z; w[i][3] = q.w;
      bias[i] = bg[c0 + i];
    }
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int t = t0 - 3 + j;
      if (t >= 0) load4(x + ((int64_t)b * T + t) * C + c0, win[j]);
      else
#pragma unroll
        for (int i = 0; i < kConvV; ++i) win[j][i] = 0.f;
    }
  }
  // z of row t (whose input is xt), then slide the window
  __device__ __forceinline__ void step(const float (&xt)[kConvV], float (&z)[kConvV]) {
#pragma unroll
    for (int i = 0; i < kConvV; ++i) {
      z[i] = fmaf(w[i][3], xt[i], fmaf(w[i][2], win[2][i], fmaf(w[i][1], win[1][i], fmaf(w[i][0], win[0][i], bias[i]))));
      win[0][i] = win[1][i];
      win[1][i] = win[2][i];
      win[2][i] = xt[i];
    }
  }
};

template <bool NORM>
__global__ void __launch_bounds__(512) conv_silu_fwd_kernel(int B, int T, int C, const __nv_bfloat16 *x,
                                                            const float *w, const float *bias,
                                                            __nv_bfloat16 *y, float scale) {
  __shared__ float red[2][16][kConvG];
  const int nch = C / kConvV, nw = (blockDim.x + 31) >> 5, c = threadIdx.x, c0 = kConvV * c;
  const bool act = c < nch;
  const int nseg = (T + kConvRows - 1) / kConvRows;
  const int b = blockIdx.x / nseg, t0 = (blockIdx.x % nseg) * kConvRows;
  const int t1 = min(T, t0 + kConvRows);
  ConvThread th;
  if (act) th.init(b, t0, T, C, c0, x, w, bias);
  int parity = 0;
  for (int tg = t0; tg < t1; tg += kConvG, parity ^= 1) {
    float z[kConvG][kConvV], ss[kConvG];
    float xt[kConvG][kConvV];
#pragma unroll
    for (int g = 0; g < kConvG; ++g)  // all loads first
      if (act && tg + g < t1) load4(x + ((int64_t)b * T + tg + g) * C + c0, xt[g]);
#pragma unroll
    for (int g = 0; g < kConvG; ++g) {
      ss[g] = 0.f;
      if (act && tg + g < t1) {
        th.step(xt[g], z[g]);
#pragma unroll
        for (int i = 0; i < kConvV; ++i) {
          z[g][i] *= sigm(z[g][i]);
          ss[g] += z[g][i] * z[g][i];
        }
      }
    }
    float inv[kConvG];
#pragma unroll
    for (int g = 0; g < kConvG; ++g) inv[g] = 1.f;
    if (NORM) {
      float tot[kConvG];
      block_sums<kConvG>(ss, tot, red, parity, nw);
#pragma unroll
      for (int g = 0; g < kConvG; ++g) inv[g] = scale / fmaxf(sqrtf(tot[g]), 1e-12f);
    }
#pragma unroll
    for (int g = 0; g < kConvG; ++g)
      if (act && tg + g < t1) {
#pragma unroll
        for (int i = 0; i < kConvV; ++i) z[g][i] *= inv[g];
        store4(y + ((int64_t)b * T + tg + g) * C + c0, z[g]);
      }
  }
}

// backward, part 1: per row, dz = d/dz of silu (and the row-wide L2 norm) at z = conv(x), into
// fp32 dz; the same walk as the forward
template <bool NORM>
__global__ void __launch_bounds__(512) conv_silu_bwd_rows_kernel(int B, int T, int C, const __nv_bfloat16 *x,
                                                                 const float *w, const float *bias,
                                                                 const __nv_bfloat16 *dy, float *dz, float scale) {
  __shared__ float red[2][16][kConvG];
  __shared__ float red2[2][16][kConvG];
  const int nch = C / kConvV, nw = (blockDim.x + 31) >> 5, c = threadIdx.x, c0 = kConvV * c;
  const bool act = c < nch;
  const int nseg = (T + kConvRows - 1) / kConvRows;
  const int b = blockIdx.x / nseg, t0 = (blockIdx.x % nseg) * kConvRows;
  const int t1 = min(T, t0 + kConvRows);
  ConvThread th;
  if (act) th.init(b, t0, T, C, c0, x, w, bias);
  int parity = 0;
  for (int tg = t0; tg < t1; tg += kConvG, parity ^= 1) {
    float z[kConvG][kConvV], g4v[kConvG][kConvV], xt[kConvG][kConvV];
    float ss[kConvG], sg[kConvG];
#pragma unroll
    for (int g = 0; g < kConvG; ++g)
      if (act && tg + g < t1) {
        load4(x + ((int64_t)b * T + tg + g) * C + c0, xt[g]);
        load4(dy + ((int64_t)b * T + tg + g) * C + c0, g4v[g]);
      }
#pragma unroll
    for (int g = 0; g < kConvG; ++g) {
      ss[g] = sg[g] = 0.f;
      if (act && tg + g < t1) {
        th.step(xt[g], z[g]);
#pragma unroll
        for (int i = 0; i < kConvV; ++i) {
          const float sv = z[g][i] * sigm(z[g][i]);
          ss[g] += sv * sv;
          sg[g] += sv * g4v[g][i];
        }
      }
    }
    float inv[kConvG], proj[kConvG];
#pragma unroll
    for (int g = 0; g < kConvG; ++g) {
      inv[g] = 1.f;
      proj[g] = 0.f;
    }
    if (NORM) {
      float ta[kConvG], tb[kConvG];
      block_sums<kConvG>(ss, ta, red, parity, nw);
      block_sums<kConvG>(sg, tb, red2, parity, nw);
#pragma unroll
      for (int g = 0; g < kConvG; ++g) {
        const float N = sqrtf(ta[g]);
        const bool clamp = !(N > 1e-12f);
        inv[g] = scale / (clamp ? 1e-12f : N);
        proj[g] = clamp ? 0.f : tb[g] / ta[g];
      }
    }
#pragma unroll
    for (int g = 0; g < kConvG; ++g)
      if (act && tg + g < t1) {
        float o[kConvV];
#pragma unroll
        for (int i = 0; i < kConvV; ++i) {
          const float sgm = sigm(z[g][i]), sv = z[g][i] * sgm;
          o[i] = inv[g] * (g4v[g][i] - sv * proj[g]) * sgm * (1.f + z[g][i] * (1.f - sgm));
        }
        *reinterpret_cast<float4 *>(dz + ((int64_t)b * T + tg + g) * C + c0) = make_float4(o[0], o[1], o[2], o[3]);
      }
  }
}

// backward, part 2: dx[t, c] = sum_j w[c, j] dz[t + 3 - j, c]; dw[c, j] += sum_t dz[t, c] x[t - 3 + j, c];
// db[c] += sum_t dz[t, c].  Thread = channel, walking a segment of t with sliding windows.
__global__ void __launch_bounds__(128) conv_bwd_cols_kernel(int B, int T, int C, int seg, const __nv_bfloat16 *x,
                                                            const float *w, const float *dz, __nv_bfloat16 *dx,
                                                            float *dw, float *db) {
  const int c = blockIdx.x * 128 + threadIdx.x;
  const int b = blockIdx.z, t0 = blockIdx.y * seg, t1 = min(T, t0 + seg);
  if (c >= C || t0 >= T) return;
  const float w0 = w[c * 4], w1 = w[c * 4 + 1], w2 = w[c * 4 + 2], w3 = w[c * 4 + 3];
  const int64_t base = (int64_t)b * T * C + c;
  auto X = [&](int t) { return t >= 0 ? __bfloat162float(x[base + (int64_t)t * C]) : 0.f; };
  auto Z = [&](int t) { return t < T ? dz[base + (int64_t)t * C] : 0.f; };
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f, ab = 0.f;
  // window: dz[t .. t+3], x[t-3 .. t]
  float z0 = Z(t0), z1 = Z(t0 + 1), z2 = Z(t0 + 2), z3 = Z(t0 + 3);
  float xm3 = X(t0 - 3), xm2 = X(t0 - 2), xm1 = X(t0 - 1), x0 = X(t0);
  for (int t = t0; t < t1; ++t) {
    dx[base + (int64_t)t * C] = __float2bfloat16_rn(w3 * z0 + w2 * z1 + w1 * z2 + w0 * z3);
    a0 = fmaf(z0, xm3, a0);
    a1 = fmaf(z0, xm2, a1);
    a2 = fmaf(z0, xm1, a2);
    a3 = fmaf(z0, x0, a3);
    ab += z0;
    z0 = z1; z1 = z2; z2 = z3; z3 = Z(t + 4);
    xm3 = xm2; xm2 = xm1; xm1 = x0; x0 = X(t + 1 < T ? t + 1 : -1);
  }
  atomicAdd(dw + c * 4, a0);
  atomicAdd(dw + c * 4 + 1, a1);
  atomicAdd(dw + c * 4 + 2, a2);
  atomicAdd(dw + c * 4 + 3, a3);
  atomicAdd(db + c, ab);
}

// grid-stride launches: at most 8 CTAs per SM of the device current at the first call
static int grid_for(int64_t rows) {
  static int nsm = 148;
  static std::once_flag once;
  std::call_once(once, [] {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0)
      nsm = n;
  });
  const int64_t need = (rows + kWarps - 1) / kWarps;
  return (int)(need < 8LL * nsm ? need : 8LL * nsm);
}

}  // namespace rowops
}  // namespace kda

using namespace kda::rowops;

static bool row_args_ok(int64_t rows, int D, std::initializer_list<const void *> ptrs) {
  if (rows <= 0 || !(D == 64 || D == 128)) return false;
  for (const void *p : ptrs)
    if (!p || ((uintptr_t)p & 15u)) return false;
  return true;
}

#define KDA_ROW_LAUNCH(kern, rows, D, st, ...)                                                 \
  do {                                                                                         \
    const int g = grid_for(rows);                                                              \
    if (D == 64) kern<2><<<g, 32 * kWarps, 0, st>>>(rows, __VA_ARGS__);                        \
    else kern<4><<<g, 32 * kWarps, 0, st>>>(rows, __VA_ARGS__);                                \
    kda::count_launch();                                                                       \
  } while (0)

extern "C" {

// row-wide kernels: chunks of 8 channels per thread, KC chunks at most
static int row_chunks(int n) {
  const int per = (n / 8 + kRowThreads - 1) / kRowThreads;
  return per <= 1 ? 1 : per <= 2 ? 2 : per <= 4 ? 4 : per <= kRowMaxChunks ? 8 : 0;
}
static bool wide_row_ok(int64_t rows, int n, std::initializer_list<const void *> ptrs) {
  if (rows <= 0 || n <= 0 || (n & 7) || !row_chunks(n)) return false;
  for (const void *p : ptrs)
    if (!p || ((uintptr_t)p & 15u)) return false;
  return true;
}
static int wide_grid(int64_t rows) { return (int)(rows < 8LL * 148 * 4 ? rows : 8LL * 148 * 4); }

#define KDA_WIDE_LAUNCH(kern, kc, g, st, ...)                                     \
  do {                                                                            \
    switch (kc) {                                                                 \
      case 1: kern<1><<<g, kRowThreads, 0, st>>>(__VA_ARGS__); break;             \
      case 2: kern<2><<<g, kRowThreads, 0, st>>>(__VA_ARGS__); break;             \
      case 4: kern<4><<<g, kRowThreads, 0, st>>>(__VA_ARGS__); break;             \
      default: kern<8><<<g, kRowThreads, 0, st>>>(__VA_ARGS__); break;            \
    }                                                                             \
    kda::count_launch();                                                          \
  } while (0)

int kda_l2norm_silu_fwd(int64_t rows, int n, const void *x, void *y, float scale, void *stream) {
  if (!wide_row_ok(rows, n, {x, y})) return KDA_ERR_INVALID_ARG;
  KDA_WIDE_LAUNCH(l2norm_silu_fwd_kernel, row_chunks(n), wide_grid(rows), (cudaStream_t)stream, rows, n,
                  (const __nv_bfloat16 *)x, (__nv_bfloat16 *)y, scale);
  return cudaPeekAtLastError() == cudaSuccess ? KDA_OK : KDA_ERR_CUDA;
}

int kda_l2norm_silu_bwd(int64_t rows, int n, const void *x, const void *dy, void *dx, float scale, void *stream) {
  if (!wide_row_ok(rows, n, {x, dy, dx})) return KDA_ERR_INVALID_ARG;
  KDA_WIDE_LAUNCH(l2norm_silu_bwd_kernel, row_chunks(n), wide_grid(rows), (cudaStream_t)stream, rows, n,
                  (const __nv_bfloat16 *)x, (const __nv_bfloat16 *)dy, (__nv_bfloat16 *)dx, scale);
  return cudaPeekAtLastError() == cudaSuccess ? KDA_OK : KDA_ERR_CUDA;
}

int kda_gated_rmsnorm_fwd(int64_t rows, int D, const void *o, const void *gate, const float *w, void *y,
                          float eps, void *stream) {
  if (!row_args_ok(rows, D, {o, gate, w, y})) return KDA_ERR_INVALID_ARG;
  KDA_ROW_LAUNCH(gated_rmsnorm_fwd_kernel, rows, D, (cudaStream_t)stream, (const __nv_bfloat16 *)o,
                 (const __nv_bfloat16 *)gate, w, (__nv_bfloat16 *)y, eps);
  return cudaPeekAtLastError() == cudaSuccess ? KDA_OK : KDA_ERR_CUDA;
}

int kda_gated_rmsnorm_bwd(int64_t rows, int D, const void *o, const void *gate, const float *w, const void *dy,
                          void *dout, void *dgate, float *dw, float eps, void *stream) {
  if (!row_args_ok(rows, D, {o, gate, w, dy, dout, dgate, dw})) return KDA_ERR_INVALID_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemsetAsync(dw, 0, sizeof(float) * D, st) != cudaSuccess) return KDA_ERR_CUDA;
  KDA_ROW_LAUNCH(gated_rmsnorm_bwd_kernel, rows, D, st, (const __nv_bfloat16 *)o, (const __nv_bfloat16 *)gate, w,
                 (const __nv_bfloat16 *)dy, (__nv_bfloat16 *)dout, (__nv_bfloat16 *)dgate, dw, eps);
  return cudaPeekAtLastError() == cudaSuccess ? KDA_OK : KDA_ERR_CUDA;
}


int kda_conv_silu_fwd(int64_t B, int64_t T, int H, int D, const void *x, const float *w, const float *bias,
                      void *y, int norm, float scale, void *stream) {
  const int C = H * D;
  if (H <= 0 || D <= 0 || C > kConvMaxC || !wide_row_ok(B * T, C, {x, w, bias, y})) return KDA_ERR_INVALID_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const int threads = ((C / kConvV + 31) / 32) * 32;
  const int grid = (int)(B * ((T + kConvRows - 1) / kConvRows));
  const __nv_bfloat16 *xb = (const __nv_bfloat16 *)x;
  __nv_bfloat16 *yb = (__nv_bfloat16 *)y;
  if (norm) conv_silu_fwd_kernel<true><<<grid, threads, 0, st>>>((int)B, (int)T, C, xb, w, bias, yb, scale);
  else conv_silu_fwd_kernel<false><<<grid, threads, 0, st>>>((int)B, (int)T, C, xb, w, bias, yb, scale);
  kda::count_launch();
  return cudaPeekAtLastError() == cudaSuccess ? KDA_OK : KDA_ERR_CUDA;
}

int kda_conv_silu_bwd(int64_t B, int64_t T, int H, int D, const void *x, const float *w, const float *bias,
                      const void *dy, void *dx, float *dw, float *db, int norm, float scale, float *dz_ws,
                      void *stream) {
  const int C = H * D;
  if (H <= 0 || D <= 0 || C > kConvMaxC || !wide_row_ok(B * T, C, {x, w, bias, dy, dx, dw, db, dz_ws}))
    return KDA_ERR_INVALID_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemsetAsync(dw, 0, sizeof(float) * C * 4, st) != cudaSuccess ||
      cudaMemsetAsync(db, 0, sizeof(float) * C, st) != cudaSuccess)
    return KDA_ERR_CUDA;
  const int threads = ((C / kConvV + 31) / 32) * 32;
  const int grid = (int)(B * ((T + kConvRows - 1) / kConvRows));
  const __nv_bfloat16 *xb = (const __nv_bfloat16 *)x, *dyb = (const __nv_bfloat16 *)dy;
  if (norm) conv_silu_bwd_rows_kernel<true><<<grid, threads, 0, st>>>((int)B, (int)T, C, xb, w, bias, dyb, dz_ws, scale);
  else conv_silu_bwd_rows_kernel<false><<<grid, threads, 0, st>>>((int)B, (int)T, C, xb, w, bias, dyb, dz_ws, scale);
  kda::count_launch();
  const int seg = 64;
  dim3 grid2((C + 127) / 128, (int)((T + seg - 1) / seg), (int)B);
  conv_bwd_cols_kernel<<<grid2, 128, 0, st>>>((int)B, (int)T, C, seg, xb, w, dz_ws, (__nv_bfloat16 *)dx, dw, db);
  kda::count_launch();
  return cudaPeekAtLastError() == cudaSuccess ? KDA_OK : KDA_ERR_CUDA;
}

}  // extern "C"
