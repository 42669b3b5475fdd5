// C-ABI entry points of libkda_b200.so: descriptor validation and kernel dispatch.
// Declarations and the reference interface each entry point replaces: include/kda_b200.h.
#include <stdio.h>

#include <atomic>

#include "kda_common.cuh"

namespace kda {
int generic_fwd(const Params &p, int dq, int db, cudaStream_t st);
int generic_bwd(const Params &p, int dq, int db, cudaStream_t st);
int generic_fwd_split(int D, int C);
size_t generic_bwd_smem(int D, int C);
int generic_chunk(int D, int C);
bool tc_supported(const KdaDesc *d, int backward);
size_t tc_workspace_bytes(const KdaDesc *d, int backward);
size_t tc_saved_bytes(const KdaDesc *d);
int tc_fwd_device_status(bool reset);
int tc_bwd_device_status(bool reset);
int tc_fwd(const Params &p, int dtype_beta, cudaStream_t st);
int tc_bwd(const Params &p, int dtype_beta, cudaStream_t st);
bool tc128_supported(const KdaDesc *d);
bool recurrent_supported(int D);
int recurrent_fwd(const Params &p, int dq, int db, cudaStream_t st);
size_t tc128_workspace_bytes(const KdaDesc *d);
int tc128_fwd(const Params &p, int dtype_beta, cudaStream_t st);
int tc128_fwd_device_status(bool reset);
static std::atomic<uint64_t> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
}  // namespace kda

using kda::Params;

static bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

static bool strides_ok(const KdaStrides &s) { return s.b >= 0 && s.t >= 0 && s.h >= 0; }

static int dtype_ok(int dt) { return dt == KDA_F32 || dt == KDA_BF16 || dt == KDA_F16; }

static int check_desc_shape(const KdaDesc *d) {
  if (!d) return KDA_ERR_INVALID_ARG;
  if (d->B <= 0 || d->T <= 0 || d->H <= 0 || d->Dk <= 0 || d->Dv <= 0 || d->chunk <= 0)
    return KDA_ERR_INVALID_ARG;
  if (!dtype_ok(d->dtype_qkv) || !dtype_ok(d->dtype_beta)) return KDA_ERR_DTYPE;
  if (d->B * d->H > (1ll << 30) || d->T > (1ll << 30) || d->B * d->T * d->H * d->Dk > (1ll << 40))
    return KDA_ERR_UNSUPPORTED;
  if (d->Dk != d->Dv) return KDA_ERR_UNSUPPORTED;  // the reference state is D x D
  if (d->chunk > 64 || d->Dk > 128) return KDA_ERR_UNSUPPORTED;
  if (!strides_ok(d->q) || !strides_ok(d->k) || !strides_ok(d->v) || !strides_ok(d->g) ||
      !strides_ok(d->beta) || !strides_ok(d->dO))
    return KDA_ERR_INVALID_ARG;
  return KDA_OK;
}

static bool use_tc(const KdaDesc *d, int backward) {
  if (d->flags & KDA_FLAG_FORCE_GENERIC) return false;
  return kda::tc_supported(d, backward);
}
// D = 128: tensor-core forward without saved states (streaming inference)
static bool use_tc128(const KdaDesc *d, int backward) {
  if (backward || (d->flags & KDA_FLAG_FORCE_GENERIC)) return false;
  return kda::tc128_supported(d);
}

extern "C" {

int kda_abi_version(void) { return KDA_ABI_VERSION; }

int kda_device_status(int reset) {
  const int f = kda::tc_fwd_device_status(reset != 0);
  const int b = kda::tc_bwd_device_status(reset != 0);
  const int f128 = kda::tc128_fwd_device_status(reset != 0);
  return f ? f : b ? b : f128;
}

uint64_t kda_launch_counter(void) { return kda::g_launches.load(std::memory_order_relaxed); }

const char *kda_strerror(int s) {
  switch (s) {
    case KDA_OK: return "ok";
    case KDA_ERR_INVALID_ARG: return "invalid argument (null pointer, non-positive size or bad descriptor)";
    case KDA_ERR_UNSUPPORTED: return "unsupported shape: needs Dk == Dv, chunk <= 64, D <= 128";
    case KDA_ERR_DTYPE: return "unsupported dtype code";
    case KDA_ERR_MISALIGNED: return "pointer not 16-byte aligned";
    case KDA_ERR_WORKSPACE: return "workspace missing or too small (see kda_workspace_bytes)";
    case KDA_ERR_CUDA: return "CUDA launch or runtime error";
    case KDA_ERR_TIMEOUT: return "a bounded device-side wait timed out";
    case KDA_ERR_SCRATCH_LIMIT: return "problem needs more workspace than kda_bwd_noalloc's static scratch (KDA_NOALLOC_SCRATCH_BYTES)";
    default: return "unknown status";
  }
}

int kda_check_desc(const KdaDesc *d, int backward) {
  int s = check_desc_shape(d);
  if (s) return s;
  if (use_tc(d, backward) || use_tc128(d, backward)) return KDA_OK;
  return kda::generic_chunk((int)d->Dk, (int)d->chunk) ? KDA_OK : KDA_ERR_UNSUPPORTED;
}

size_t kda_workspace_bytes(const KdaDesc *d, int backward) {
  if (kda_check_desc(d, backward)) return 0;
  if (use_tc128(d, backward)) return kda::tc128_workspace_bytes(d);
  return use_tc(d, backward) ? kda::tc_workspace_bytes(d, backward) : 0;
}

// The saved record's layout belongs to the backward that reads it: a forward that saves
// for the backward uses the tensor-core forward only where the tensor-core backward runs too.
size_t kda_saved_bytes(const KdaDesc *d) {
  if (kda_check_desc(d, 0)) return 0;
  if (use_tc(d, 1)) return kda::tc_saved_bytes(d);
  const int64_t gc = kda::generic_chunk((int)d->Dk, (int)d->chunk);
  const int64_t nc = (d->T + gc - 1) / gc;
  return (size_t)(d->B * d->H * nc * d->Dk * d->Dv) * sizeof(float);
}

// an input's strides: the descriptor's, or the dense layout when all three are zero
static kda::Str input_strides(const KdaStrides &s, const KdaDesc *d, bool per_head_vector) {
  if (s.b == 0 && s.t == 0 && s.h == 0) {
    const int64_t D = per_head_vector ? d->Dk : 1;
    return kda::Str{d->T * d->H * D, d->H * D, D};
  }
  return kda::Str{s.b, s.t, s.h};
}

// TMA reads need every stride of a tile-loaded input to span a multiple of 16 bytes
static bool tma_strides_ok(const kda::Str &s, int elem_bytes) {
  return (s.b * elem_bytes) % 16 == 0 && (s.t * elem_bytes) % 16 == 0 && (s.h * elem_bytes) % 16 == 0;
}

static Params make_params(const KdaDesc *d) {
  Params p = {};
  p.B = (int)d->B; p.T = (int)d->T; p.H = (int)d->H; p.D = (int)d->Dk; p.C = (int)d->chunk;
  p.nc = (int)((d->T + d->chunk - 1) / d->chunk);
  p.sq = input_strides(d->q, d, true);
  p.sk = input_strides(d->k, d, true);
  p.sv = input_strides(d->v, d, true);
  p.sg = input_strides(d->g, d, true);
  p.sb = input_strides(d->beta, d, false);
  p.sdo = input_strides(d->dO, d, true);
  p.debug_wait_polls = (d->flags & KDA_FLAG_DEBUG_WAIT_TIMEOUT) ? 64 : 0;
  return p;
}

int kda_fwd(const KdaDesc *d, const void *q, const void *k, const void *v, const float *g,
            const void *beta, const float *state0, void *o, float *stateT, void *saved,
            void *ws, size_t ws_bytes, void *stream) {
  int s = kda_check_desc(d, 0);
  if (s) return s;
  if (!q || !k || !v || !g || !beta || !o || !stateT) return KDA_ERR_INVALID_ARG;
  const void *ptrs[] = {q, k, v, g, o, stateT};
  for (const void *ptr : ptrs) if (!aligned16(ptr)) return KDA_ERR_MISALIGNED;
  if ((state0 && !aligned16(state0)) || (saved && !aligned16(saved))) return KDA_ERR_MISALIGNED;
  size_t need = kda_workspace_bytes(d, 0);
  if (need && (!ws || ws_bytes < need || !aligned16(ws))) return KDA_ERR_WORKSPACE;
  Params p = make_params(d);
  p.q = q; p.k = k; p.v = v; p.g = g; p.beta = beta; p.state0 = state0;
  p.o = o; p.stateT = stateT; p.saved = saved; p.ws = ws;
  cudaStream_t st = (cudaStream_t)stream;
  const bool tc = use_tc(d, 0) && (!saved || use_tc(d, 1)), tc128 = !tc && use_tc128(d, 0) && !saved;
  if ((tc || tc128) && !(tma_strides_ok(p.sq, 2) && tma_strides_ok(p.sk, 2) && tma_strides_ok(p.sv, 2) &&
                         tma_strides_ok(p.sg, 4)))
    return KDA_ERR_MISALIGNED;
  if (tc) return kda::tc_fwd(p, d->dtype_beta, st);
  if (tc128) return kda::tc128_fwd(p, d->dtype_beta, st);
  p.C = kda::generic_chunk(p.D, p.C);  // the fp32 kernels' chunk (see generic_chunk)
  p.nc = (p.T + p.C - 1) / p.C;
  return kda::generic_fwd(p, d->dtype_qkv, d->dtype_beta, st);
}

int kda_bwd(const KdaDesc *d, const void *q, const void *k, const void *v, const float *g,
            const void *beta, const float *state0, const void *saved, const void *dO,
            const float *dstateT, void *dq, void *dk, void *dv, float *dg, void *dbeta,
            float *dstate0, void *ws, size_t ws_bytes, void *stream) {
  int s = kda_check_desc(d, 1);
  if (s) return s;
  if (!q || !k || !v || !g || !beta || !saved || !dO || !dq || !dk || !dv || !dg || !dbeta)
    return KDA_ERR_INVALID_ARG;
  const void *ptrs[] = {q, k, v, g, saved, dO, dq, dk, dv, dg};
  for (const void *ptr : ptrs) if (!aligned16(ptr)) return KDA_ERR_MISALIGNED;
  if ((state0 && !aligned16(state0)) || (dstateT && !aligned16(dstateT)) ||
      (dstate0 && !aligned16(dstate0)))
    return KDA_ERR_MISALIGNED;
  size_t need = kda_workspace_bytes(d, 1);
  if (need && (!ws || ws_bytes < need || !aligned16(ws))) return KDA_ERR_WORKSPACE;
  Params p = make_params(d);
  p.q = q; p.k = k; p.v = v; p.g = g; p.beta = beta; p.state0 = state0;
  p.saved_in = saved; p.dO = dO; p.dstateT = dstateT; p.ws = ws;
  p.dq = dq; p.dk = dk; p.dv = dv; p.dg = dg; p.dbeta = dbeta; p.dstate0 = dstate0;
  cudaStream_t st = (cudaStream_t)stream;
  if (use_tc(d, 1)) {
    if (!(tma_strides_ok(p.sq, 2) && tma_strides_ok(p.sk, 2) && tma_strides_ok(p.sv, 2) &&
          tma_strides_ok(p.sg, 4) && tma_strides_ok(p.sdo, 2)))
      return KDA_ERR_MISALIGNED;
    return kda::tc_bwd(p, d->dtype_beta, st);
  }
  p.C = kda::generic_chunk(p.D, p.C);
  p.nc = (p.T + p.C - 1) / p.C;
  return kda::generic_bwd(p, d->dtype_qkv, d->dtype_beta, st);
}

int kda_fwd_recurrent(const KdaDesc *d, const void *q, const void *k, const void *v, const float *g,
                      const void *beta, const float *state0, void *o, float *stateT, void *stream) {
  int s = check_desc_shape(d);
  if (s) return s;
  if (!kda::recurrent_supported((int)d->Dk)) return KDA_ERR_UNSUPPORTED;
  if (!q || !k || !v || !g || !beta || !o || !stateT) return KDA_ERR_INVALID_ARG;
  Params p = make_params(d);
  p.q = q; p.k = k; p.v = v; p.g = g; p.beta = beta; p.state0 = state0;
  p.o = o; p.stateT = stateT;
  return kda::recurrent_fwd(p, d->dtype_qkv, d->dtype_beta, (cudaStream_t)stream);
}

static int check_gate(const KdaDesc *d, const KdaGate *gate) {
  if (!gate || !gate->f || !gate->A_log || !gate->dt_bias || !gate->b) return KDA_ERR_INVALID_ARG;
  if (!use_tc(d, 1)) return KDA_ERR_UNSUPPORTED;  // the gates are fused into the tensor-core kernels only
  if (!aligned16(gate->f)) return KDA_ERR_MISALIGNED;
  const Params p = make_params(d);
  if (!(tma_strides_ok(p.sq, 2) && tma_strides_ok(p.sk, 2) && tma_strides_ok(p.sv, 2) &&
        tma_strides_ok(p.sg, 2) && tma_strides_ok(p.sdo, 2)))
    return KDA_ERR_MISALIGNED;
  return KDA_OK;
}

static void set_gate(Params &p, const KdaGate *gate) {
  p.gated = 1;
  p.beta_scale = gate->allow_neg_eigval ? 2 : 1;
  p.f = gate->f; p.A_log = gate->A_log; p.dt_bias = gate->dt_bias;
  p.beta = gate->b;
}

int kda_fwd_gated(const KdaDesc *d, const void *q, const void *k, const void *v, const KdaGate *gate,
                  const float *state0, void *o, float *stateT, void *saved, void *ws, size_t ws_bytes,
                  void *stream) {
  int s = kda_check_desc(d, 0);
  if (s) return s;
  if ((s = check_gate(d, gate))) return s;
  if (!q || !k || !v || !o || !stateT) return KDA_ERR_INVALID_ARG;
  const void *ptrs[] = {q, k, v, o, stateT};
  for (const void *ptr : ptrs) if (!aligned16(ptr)) return KDA_ERR_MISALIGNED;
  if ((state0 && !aligned16(state0)) || (saved && !aligned16(saved))) return KDA_ERR_MISALIGNED;
  size_t need = kda_workspace_bytes(d, 0);
  if (need && (!ws || ws_bytes < need || !aligned16(ws))) return KDA_ERR_WORKSPACE;
  Params p = make_params(d);
  p.q = q; p.k = k; p.v = v; p.state0 = state0;
  p.o = o; p.stateT = stateT; p.saved = saved; p.ws = ws;
  set_gate(p, gate);
  return kda::tc_fwd(p, d->dtype_beta, (cudaStream_t)stream);
}

int kda_bwd_gated(const KdaDesc *d, const void *q, const void *k, const void *v, const KdaGate *gate,
                  const float *state0, const void *saved, const void *dO, const float *dstateT,
                  void *dq, void *dk, void *dv, void *df, void *db, float *dA_log, float *ddt_bias,
                  float *dstate0, void *ws, size_t ws_bytes, void *stream) {
  int s = kda_check_desc(d, 1);
  if (s) return s;
  if ((s = check_gate(d, gate))) return s;
  if (!q || !k || !v || !saved || !dO || !dq || !dk || !dv || !df || !db || !dA_log || !ddt_bias)
    return KDA_ERR_INVALID_ARG;
  const void *ptrs[] = {q, k, v, saved, dO, dq, dk, dv, df};
  for (const void *ptr : ptrs) if (!aligned16(ptr)) return KDA_ERR_MISALIGNED;
  if ((state0 && !aligned16(state0)) || (dstateT && !aligned16(dstateT)) ||
      (dstate0 && !aligned16(dstate0)))
    return KDA_ERR_MISALIGNED;
  size_t need = kda_workspace_bytes(d, 1);
  if (need && (!ws || ws_bytes < need || !aligned16(ws))) return KDA_ERR_WORKSPACE;
  Params p = make_params(d);
  p.q = q; p.k = k; p.v = v; p.state0 = state0;
  p.saved_in = saved; p.dO = dO; p.dstateT = dstateT; p.ws = ws;
  p.dq = dq; p.dk = dk; p.dv = dv; p.dbeta = db; p.dstate0 = dstate0;
  set_gate(p, gate);
  p.df = df; p.dA_log = dA_log; p.ddt_bias = ddt_bias;
  return kda::tc_bwd(p, d->dtype_beta, (cudaStream_t)stream);
}

}  // extern "C"
