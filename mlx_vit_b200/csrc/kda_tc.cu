// Tensor-core KDA kernels (placeholder until the sm_100a kernels land).
#include "kda_common.cuh"

namespace kda {
bool tc_supported(const KdaDesc *, int) { return false; }
size_t tc_workspace_bytes(const KdaDesc *, int) { return 0; }
int tc_fwd(const Params &, void *, size_t, cudaStream_t) { return KDA_ERR_UNSUPPORTED; }
int tc_bwd(const Params &, void *, size_t, cudaStream_t) { return KDA_ERR_UNSUPPORTED; }
}  // namespace kda
