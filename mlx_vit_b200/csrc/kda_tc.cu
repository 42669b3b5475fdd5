// Dispatch rules for the tensor-core KDA kernels (D = 64, chunk = 64, bf16 q/k/v).
#include "kda_common.cuh"

namespace kda {

// set once the tensor-core backward is in place: the saved-record layout follows it
static constexpr bool kTcBackward = true;

bool tc_supported(const KdaDesc *d, int backward) {
  if (backward && !kTcBackward) return false;
  return d->Dk == 64 && d->Dv == 64 && d->chunk == 64 && d->dtype_qkv == KDA_BF16 &&
         (d->dtype_beta == KDA_BF16 || d->dtype_beta == KDA_F32);
}
size_t tc_bwd_workspace_bytes(const KdaDesc *d);
size_t tc_fwd_workspace_bytes(const KdaDesc *d);
size_t tc_workspace_bytes(const KdaDesc *d, int backward) {
  return backward ? tc_bwd_workspace_bytes(d) : tc_fwd_workspace_bytes(d);
}
size_t tc_saved_bytes(const KdaDesc *d) {
  const int64_t nc = (d->T + d->chunk - 1) / d->chunk;
  return (size_t)(d->B * d->H * nc) * kSavedChunk;
}
}  // namespace kda

// ---- tensor maps ----
#include <mutex>

#include <cudaTypedefs.h>

#include "kda_tma.cuh"

namespace kda {

static PFN_cuTensorMapEncodeTiled encode_fn() {
  static PFN_cuTensorMapEncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(p);
  });
  return fn;
}

// The tensor-map encoder is a driver call: it needs a current context on the calling thread.  A
// host thread that has made no runtime call yet (e.g. an autograd worker thread on device 0, where
// the runtime's default device already matches and nothing binds a context) has none, so bind the
// current device's primary context first.  Host-only and allowed during stream capture.
static bool ensure_context() {
  static PFN_cuCtxGetCurrent get_cur = nullptr;
  static PFN_cuCtxSetCurrent set_cur = nullptr;
  static PFN_cuDevicePrimaryCtxRetain retain = nullptr;
  static PFN_cuDeviceGet dev_get = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void *p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
      get_cur = reinterpret_cast<PFN_cuCtxGetCurrent>(p);
    if (cudaGetDriverEntryPoint("cuCtxSetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
      set_cur = reinterpret_cast<PFN_cuCtxSetCurrent>(p);
    if (cudaGetDriverEntryPoint("cuDevicePrimaryCtxRetain", &p, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
      retain = reinterpret_cast<PFN_cuDevicePrimaryCtxRetain>(p);
    if (cudaGetDriverEntryPoint("cuDeviceGet", &p, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
      dev_get = reinterpret_cast<PFN_cuDeviceGet>(p);
  });
  if (!get_cur || !set_cur || !retain || !dev_get) return false;
  CUcontext ctx = nullptr;
  if (get_cur(&ctx) == CUDA_SUCCESS && ctx) return true;
  int dev = 0;
  CUdevice cu = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev_get(&cu, dev) != CUDA_SUCCESS) return false;
  // one reference to the primary context is kept until exit (the runtime holds one as well)
  return retain(&ctx, cu) == CUDA_SUCCESS && set_cur(ctx) == CUDA_SUCCESS;
}

int tma_map_bthd(CUtensorMap *map, const void *base, int64_t B, int64_t T, int64_t H, int64_t D, bool fp32,
                 const Str *st) {
  PFN_cuTensorMapEncodeTiled fn = encode_fn();
  if (!fn || !ensure_context()) return KDA_ERR_CUDA;
  const int64_t es = fp32 ? 4 : 2;
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  const Str dense = {T * H * D, H * D, D};
  const Str &s = st ? *st : dense;
  const cuuint64_t strides[3] = {(cuuint64_t)(s.h * es), (cuuint64_t)(s.t * es), (cuuint64_t)(s.b * es)};
  for (int i = 0; i < 3; ++i)
    if (strides[i] % 16) return KDA_ERR_MISALIGNED;
  const cuuint32_t box[4] = {(cuuint32_t)(fp32 ? 32 : 64), 1, 64, 1};  // 128 bytes per box row
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = fn(map, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                        const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? KDA_OK : KDA_ERR_INVALID_ARG;
}

}  // namespace kda
