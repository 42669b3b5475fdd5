"""B200-native (sm_100a) chunkwise KDA recurrence: the ``cuda_kda`` drop-in for the
reference's GatedDeltaLayer compute paths.  See ``mlx_vit_b200.kda``."""
from .kda import cuda_kda, kda_forward, kda_backward, validate_compute_path, CudaKdaFunction  # noqa: F401
from .kda import kda_recurrent  # noqa: F401
from .kda import cuda_kda_gated, kda_forward_gated, kda_backward_gated, CudaKdaGatedFunction  # noqa: F401

__all__ = ["cuda_kda", "kda_forward", "kda_backward", "validate_compute_path", "CudaKdaFunction",
           "cuda_kda_gated", "kda_forward_gated", "kda_backward_gated", "CudaKdaGatedFunction", "kda_recurrent"]
