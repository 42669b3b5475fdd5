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
