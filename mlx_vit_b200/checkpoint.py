"""Checkpoint interop with the reference trainers (train_mlx_k400.py:273-325).

The reference saves one safetensors file of the MLX parameter tree (keys are dotted tree paths,
``_flatten_params``, nope_gdn_mlx.py:5124-5133), with the EMA shadow in the same file under an
``__ema__`` prefix, plus ``<name>.meta.json`` holding {"epoch", "best_acc", "ema_decay"}.  This
module writes and reads that format for the PyTorch model in ``nope_gdn.py``:

* key paths map onto the reference classifier's tree: ``embed`` ->
  ``backbone.encoder.tubelet_embed.projection``, ``blocks.i`` -> ``backbone.processor_blocks.i``,
  ``norm`` -> ``backbone.processor_norm``, ``head`` -> ``head.fc``; inside a block, the MLP's
  ``mlp.0`` / ``mlp.2`` are the reference's ``mlp.layers.0`` / ``mlp.layers.3`` (its Sequential
  holds dropouts between); every GatedDeltaLayer name is the reference's own;
* tensor layouts follow MLX's channels-last convolutions: depthwise Conv1d weights are
  (C, K, 1) (torch: (C, 1, K)), Conv3d weights (O, kt, kh, kw, I) (torch: (O, I, kt, kh, kw)).

Loading, like the reference's ``load_checkpoint``, applies the model keys present, reports the
missing and unexpected ones, and hands ``__ema__`` tensors to an EMA shadow dict if given.
"""
from __future__ import annotations

import json
import os
import re
from typing import Dict, Optional

import torch
from safetensors.torch import load_file, save_file

EMA_PREFIX = "__ema__"

_OUTER = [(r"^embed\.", "backbone.encoder.tubelet_embed.projection."),
          (r"^blocks\.(\d+)\.", r"backbone.processor_blocks.\1."),
          (r"^norm\.", "backbone.processor_norm."),
          (r"^head\.", "head.fc.")]
_INNER = [(r"\.mlp\.0\.", ".mlp.layers.0."), (r"\.mlp\.2\.", ".mlp.layers.3.")]


def to_reference_key(name: str) -> str:
    for a, b in _OUTER:
        if re.match(a, name):
            name = re.sub(a, b, name)
            break
    for a, b in _INNER:
        name = re.sub(a, b, name)
    return name


_OUTER_REV = [(r"^backbone\.encoder\.tubelet_embed\.projection\.", "embed."),
              (r"^backbone\.processor_blocks\.(\d+)\.", r"blocks.\1."),
              (r"^backbone\.processor_norm\.", "norm."),
              (r"^head\.fc\.", "head.")]
_INNER_REV = [(r"\.mlp\.layers\.0\.", ".mlp.0."), (r"\.mlp\.layers\.3\.", ".mlp.2.")]


def from_reference_key(key: str) -> str:
    for a, b in _OUTER_REV:
        if re.match(a, key):
            key = re.sub(a, b, key)
            break
    for a, b in _INNER_REV:
        key = re.sub(a, b, key)
    return key


def _is_conv1d(name: str) -> bool:
    return name.endswith("conv1d.weight")


def _is_conv3d(name: str, t: torch.Tensor) -> bool:
    return t.dim() == 5 and name.endswith(".weight")


def to_reference_tensor(name: str, t: torch.Tensor) -> torch.Tensor:
    if _is_conv1d(name):
        return t.permute(0, 2, 1).contiguous()       # (C, 1, K) -> (C, K, 1)
    if _is_conv3d(name, t):
        return t.permute(0, 2, 3, 4, 1).contiguous()  # (O, I, kt, kh, kw) -> (O, kt, kh, kw, I)
    return t.contiguous()


def from_reference_tensor(name: str, t: torch.Tensor) -> torch.Tensor:
    if _is_conv1d(name):
        return t.permute(0, 2, 1).contiguous()
    if t.dim() == 5 and name.endswith(".weight"):
        return t.permute(0, 4, 1, 2, 3).contiguous()
    return t


def save_checkpoint(path: str, model: torch.nn.Module, ema: Optional[Dict[str, torch.Tensor]] = None,
                    epoch: int = 0, best_acc: float = 0.0, ema_decay: Optional[float] = None) -> int:
    """Writes ``path`` (safetensors, reference key paths and layouts) and ``path``'s
    ``.meta.json``.  ``ema`` maps this model's parameter names to shadow tensors.  Returns the
    number of tensors written."""
    tensors = {}
    for n, p in model.state_dict().items():
        tensors[to_reference_key(n)] = to_reference_tensor(n, p.detach().cpu())
    for n, t in (ema or {}).items():
        tensors[EMA_PREFIX + to_reference_key(n)] = to_reference_tensor(n, t.detach().cpu())
    d = os.path.dirname(os.path.abspath(path))
    os.makedirs(d, exist_ok=True)
    save_file(tensors, path)
    with open(os.path.splitext(path)[0] + ".meta.json", "w") as f:
        json.dump({"epoch": epoch, "best_acc": best_acc, "ema_decay": ema_decay}, f)
    return len(tensors)


def load_checkpoint(path: str, model: torch.nn.Module,
                    ema: Optional[Dict[str, torch.Tensor]] = None) -> dict:
    """Loads the model tensors of ``path`` into ``model`` (keys present in both), and the
    ``__ema__`` tensors into ``ema`` where it has the key.  Returns {"loaded", "missing",
    "unexpected", "ema_loaded", "meta"} with missing / unexpected in this model's names."""
    raw = load_file(path)
    own = model.state_dict()
    model_w = {from_reference_key(k): v for k, v in raw.items() if not k.startswith(EMA_PREFIX)}
    ema_w = {from_reference_key(k[len(EMA_PREFIX):]): v for k, v in raw.items() if k.startswith(EMA_PREFIX)}
    missing = sorted(set(own) - set(model_w))
    unexpected = sorted(set(model_w) - set(own))
    with torch.no_grad():
        for n, v in model_w.items():
            if n in own:
                own[n].copy_(from_reference_tensor(n, v).to(own[n].dtype))
    n_ema = 0
    if ema is not None:
        for n, v in ema_w.items():
            if n in ema:
                ema[n] = from_reference_tensor(n, v).to(ema[n].dtype)
                n_ema += 1
    meta_path = os.path.splitext(path)[0] + ".meta.json"
    meta = json.load(open(meta_path)) if os.path.exists(meta_path) else None
    return {"loaded": len(model_w) - len(unexpected), "missing": missing, "unexpected": unexpected,
            "ema_loaded": n_ema, "meta": meta}
