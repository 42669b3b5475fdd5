"""Checkpoint interop (CPU): the reference's safetensors format (train_mlx_k400.py:273-325) for the
PyTorch model: key paths of the reference classifier's tree, MLX channels-last conv layouts,
``__ema__`` shadow keys and the ``.meta.json`` side file; save -> load round trip is exact."""
import json

import torch
from safetensors.torch import load_file

from mlx_vit_b200.checkpoint import (from_reference_key, load_checkpoint, save_checkpoint,
                                     to_reference_key)
from mlx_vit_b200.nope_gdn import NoPEGDNVideo


def small():
    torch.manual_seed(0)
    return NoPEGDNVideo(img_size=32, frames=4, dim=64, depth=2, heads=1, num_classes=5)


def test_key_mapping_follows_reference_tree():
    cases = {
        "embed.weight": "backbone.encoder.tubelet_embed.projection.weight",
        "blocks.1.layer.q_proj.weight": "backbone.processor_blocks.1.layer.q_proj.weight",
        "blocks.0.layer.q_conv1d.weight": "backbone.processor_blocks.0.layer.q_conv1d.weight",
        "blocks.0.layer.A_log": "backbone.processor_blocks.0.layer.A_log",
        "blocks.0.layer.o_norm.weight": "backbone.processor_blocks.0.layer.o_norm.weight",
        "blocks.11.mlp.0.weight": "backbone.processor_blocks.11.mlp.layers.0.weight",
        "blocks.11.mlp.2.bias": "backbone.processor_blocks.11.mlp.layers.3.bias",
        "norm.weight": "backbone.processor_norm.weight",
        "head.bias": "head.fc.bias",
    }
    for ours, ref in cases.items():
        assert to_reference_key(ours) == ref
        assert from_reference_key(ref) == ours


def test_round_trip_with_ema_and_meta(tmp_path):
    m1 = small()
    ema = {n: p.detach().clone() * 0.5 for n, p in m1.named_parameters()}
    path = str(tmp_path / "ckpt.safetensors")
    n = save_checkpoint(path, m1, ema=ema, epoch=3, best_acc=0.42, ema_decay=0.999)
    raw = load_file(path)
    assert n == len(raw)
    assert sum(k.startswith("__ema__") for k in raw) == len(ema)
    # MLX layouts: depthwise conv (C, K, 1), Conv3d channels-last (O, kt, kh, kw, I)
    assert tuple(raw["backbone.processor_blocks.0.layer.q_conv1d.weight"].shape) == (64, 4, 1)
    assert tuple(raw["backbone.encoder.tubelet_embed.projection.weight"].shape) == (64, 2, 16, 16, 3)
    meta = json.load(open(tmp_path / "ckpt.meta.json"))
    assert meta == {"epoch": 3, "best_acc": 0.42, "ema_decay": 0.999}

    m2 = small()
    for p in m2.parameters():
        torch.nn.init.zeros_(p)
    ema2 = {n: torch.zeros_like(p) for n, p in m2.named_parameters()}
    info = load_checkpoint(path, m2, ema=ema2)
    assert info["missing"] == [] and info["unexpected"] == []
    assert info["ema_loaded"] == len(ema2) and info["meta"]["epoch"] == 3
    for (n, a), b in zip(m1.state_dict().items(), m2.state_dict().values()):
        assert torch.equal(a, b), n
    for n in ema:
        assert torch.equal(ema[n], ema2[n]), n


def test_load_reports_missing_and_unexpected(tmp_path):
    m1 = small()
    path = str(tmp_path / "c.safetensors")
    save_checkpoint(path, m1)
    raw = load_file(path)
    raw.pop("head.fc.weight")
    raw["head.norm.weight"] = torch.ones(64)  # the reference head's own norm
    from safetensors.torch import save_file
    save_file(raw, path)
    info = load_checkpoint(path, small())
    assert info["missing"] == ["head.weight"]
    assert info["unexpected"] == ["head.norm.weight"]
