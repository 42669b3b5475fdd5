"""CPU: host-side logic of the cuda_kda drop-in (path validation, argument checks, no CPU
fallback)."""
import pytest
import torch

from mlx_vit_b200 import cuda_kda, validate_compute_path
from mlx_vit_b200.kda import num_chunks


def test_compute_path_validation_mirrors_reference():
    assert validate_compute_path("cuda_kda", True) == "cuda_kda"
    with pytest.raises(ValueError, match="channel-wise"):
        validate_compute_path("cuda_kda", False)
    with pytest.raises(ValueError, match="Unknown compute_path"):
        validate_compute_path("cuda_kdaa", True)
    for p in ("chunkwise_kda_vjp", "compiled", "naive", "metal_vjp"):
        assert validate_compute_path(p, True) == p


def _inputs(B=1, T=8, H=2, D=16, dev="cpu"):
    q = torch.randn(B, T, H, D, device=dev)
    return q, q.clone(), q.clone(), -torch.rand(B, T, H, D, device=dev), torch.rand(B, T, H, device=dev)


def test_cpu_tensors_raise_no_fallback():
    with pytest.raises(ValueError, match="no CPU path"):
        cuda_kda(*_inputs())


def test_non_array_rejected():
    q, k, v, g, b = _inputs()
    with pytest.raises(TypeError):
        cuda_kda(q.numpy().tolist(), k, v, g, b)


def test_num_chunks():
    assert num_chunks(1568, 64) == 25
    assert num_chunks(64, 64) == 1
    assert num_chunks(1, 64) == 1
