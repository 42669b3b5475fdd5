"""Minimal torch-backed stand-in for the ``mlx`` package (test infrastructure only).

MLX is not installable in this container (no wheel, no network), but the reference's KDA
oracle paths -- ``GatedDeltaLayer._loop_compiled_kda`` / ``_kda_step_fused`` and the
hand-written step backward ``GatedDeltaLayer._kda_python_backward_full`` in
``nope_gdn_mlx.py`` -- only use a handful of array primitives (``exp``, ``@``, ``zeros``,
``eye``, ``stack``, ``sum``, ``einsum``, ``astype``, broadcasting and indexing).  This module
implements exactly those primitives on top of torch CPU tensors so that the reference's *own
source* for the path can be executed here to produce golden vectors.  ``mx.compile`` is the
identity (it only fuses, it does not change values) and gradients of the ``compiled`` path,
which MLX obtains with autograd, are obtained with torch autograd through the same ops.

``install(float_dtype)`` registers the fake modules in ``sys.modules``.  ``mx.float32`` is
mapped to ``float_dtype`` so that the golden run can be carried out in float64 while running
the reference's code unmodified.

Only ``tests/golden/make_golden.py`` imports this file.
"""
from __future__ import annotations

import sys
import types

import torch


class _Unavailable:
    """Placeholder for MLX symbols that the KDA oracle paths never call."""

    def __init__(self, name):
        self._name = name

    def __call__(self, *a, **k):
        raise NotImplementedError(f"mlx emulator: {self._name} is not emulated")

    def __getattr__(self, item):
        return _Unavailable(f"{self._name}.{item}")


class _EmuModule(types.ModuleType):
    def __getattr__(self, item):  # only reached for names not set explicitly
        if item.startswith("__"):
            raise AttributeError(item)
        return _Unavailable(f"{self.__name__}.{item}")


def _identity_decorator(fn=None, **_kw):
    if fn is None:
        return lambda f: f
    return fn


class _CustomFunction:
    def __init__(self, fn):
        self.fn = fn

    def vjp(self, f):
        self._vjp = f
        return f

    def __call__(self, *a, **k):
        return self.fn(*a, **k)


def install(float_dtype=torch.float64):
    """Register fake ``mlx``, ``mlx.core``, ``mlx.nn``, ``mlx.utils``, ``mlx.optimizers``."""
    if not hasattr(torch.Tensor, "astype"):
        torch.Tensor.astype = lambda self, dt: self.to(dt)

    mlx = _EmuModule("mlx")
    core = _EmuModule("mlx.core")
    nn = _EmuModule("mlx.nn")
    utils = _EmuModule("mlx.utils")
    optim = _EmuModule("mlx.optimizers")
    mlx.core, mlx.nn, mlx.utils, mlx.optimizers = core, nn, utils, optim

    core.array = torch.Tensor
    core.float32 = float_dtype
    core.float16 = torch.float16
    core.bfloat16 = torch.bfloat16
    core.int32 = torch.int32
    core.compile = _identity_decorator
    core.custom_function = _CustomFunction
    core.eval = lambda *a, **k: None
    core.zeros = lambda shape, dtype=float_dtype: torch.zeros(shape, dtype=dtype)
    core.ones = lambda shape, dtype=float_dtype: torch.ones(shape, dtype=dtype)
    core.eye = lambda n, dtype=float_dtype: torch.eye(n, dtype=dtype)
    core.exp = torch.exp
    core.log = torch.log
    core.sqrt = torch.sqrt
    core.abs = torch.abs
    core.maximum = lambda a, b: torch.maximum(a, torch.as_tensor(b, dtype=a.dtype))
    core.minimum = lambda a, b: torch.minimum(a, torch.as_tensor(b, dtype=a.dtype))
    core.stack = lambda xs, axis=0: torch.stack(list(xs), dim=axis)
    core.concatenate = lambda xs, axis=0: torch.cat(list(xs), dim=axis)
    core.sum = lambda x, axis=None, keepdims=False: (
        x.sum() if axis is None else x.sum(dim=axis, keepdim=keepdims))
    core.einsum = torch.einsum
    core.swapaxes = lambda x, a, b: x.transpose(a, b)
    core.transpose = lambda x, axes: x.permute(*axes)
    core.tril = lambda x, k=0: torch.tril(x, diagonal=k)
    core.triu = lambda x, k=0: torch.triu(x, diagonal=k)

    class Module:  # the reference subclasses nn.Module at import time
        pass

    nn.Module = Module
    utils.tree_map = lambda fn, tree, *rest: tree

    for name, mod in (("mlx", mlx), ("mlx.core", core), ("mlx.nn", nn),
                      ("mlx.utils", utils), ("mlx.optimizers", optim)):
        sys.modules[name] = mod
    return core
