"""``cuda_kda``: the reference KDA operator's drop-in, backed by libkda_b200.so.

Host-side mirror of the reference's compute-path interface (HananKibria/MLX_VIT,
nope_gdn_mlx.py):

* ``cuda_kda(q, k, v, g, beta, state=None, chunk_size=64) -> (output, new_state)`` has the
  signature and dtype contract of the ``GatedDeltaLayer`` path methods (e.g.
  ``_chunkwise_kda_vjp_path`` :2829-2865, ``_loop_compiled_kda`` :890-917): q, k, v, g are
  (B, L, H, D), beta (B, L, H), state (B, H, D, D) float32 or None (zeros); the output is in
  q's dtype and the new state float32.  g is used as float32 (nope_gdn_mlx.py:804).
* Its VJP returns one gradient per primal, like the ``mx.custom_function`` vjp at
  :2746-2809: dq, dk, dv in the primal dtype, dg float32, dbeta in beta's dtype, dstate
  float32 (None when no state was passed).  The final-state cotangent may be absent.
* ``validate_compute_path`` mirrors the constructor checks at :693-735 with ``"cuda_kda"``
  added (channel-wise KDA only).

Arrays cross the boundary as raw device pointers (any DLPack-capable CUDA array is accepted
and viewed without a copy through ``torch.from_dlpack``); all launches go on the current torch
CUDA stream.  There is no CPU or eager fallback: a missing library, a CPU tensor or an
unsupported shape raises.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _lib

_DT = {torch.float32: _lib.KDA_F32, torch.bfloat16: _lib.KDA_BF16, torch.float16: _lib.KDA_F16}

KDA_COMPUTE_PATHS = ("metal_vjp", "chunkwise_kda_vjp", "chunkwise_kda", "metal_sg", "metal",
                     "compiled", "naive", "cuda_kda")


def validate_compute_path(compute_path: str, channel_wise_decay: bool = True) -> str:
    """Constructor-time check of a GDN compute path (nope_gdn_mlx.py:693-735) extended with
    ``"cuda_kda"``, which exists for channel-wise KDA only."""
    if compute_path == "cuda_kda" and not channel_wise_decay:
        raise ValueError("cuda_kda is only valid for channel-wise KDA (channel_wise_decay=True). "
                         "For scalar-alpha use 'chunkwise_wy'.")
    if compute_path not in KDA_COMPUTE_PATHS + ("chunkwise_wy",):
        raise ValueError(f"Unknown compute_path: {compute_path}")
    return compute_path


def _as_torch(x, name):
    if x is None:
        return None
    if not isinstance(x, torch.Tensor):
        if hasattr(x, "__dlpack__"):
            x = torch.from_dlpack(x)
        else:
            raise TypeError(f"{name}: expected a CUDA array (torch tensor or DLPack), got {type(x)}")
    if not x.is_cuda:
        raise ValueError(f"{name}: cuda_kda needs device arrays (got a {x.device} tensor); "
                         "there is no CPU path")
    return x


def _ptr(x):
    return ctypes.c_void_p(x.data_ptr()) if x is not None else ctypes.c_void_p(0)


def _strides(x):
    """KdaStrides of an input view (b, t, h element strides; zeros for a dense tensor)."""
    if x is None or x.is_contiguous():
        return _lib.KdaStrides(0, 0, 0)
    st = x.stride()
    return _lib.KdaStrides(st[0], st[1], st[2])


def _desc(q, beta, chunk_size, flags, k=None, v=None, g=None, do=None):
    """The call's descriptor; the strides of any strided input view go along with it."""
    B, T, H, D = q.shape
    if q.dtype not in _DT or beta.dtype not in _DT:
        raise ValueError(f"unsupported dtypes q={q.dtype} beta={beta.dtype}")
    return _lib.KdaDesc(B, T, H, D, D, int(chunk_size), _DT[q.dtype], _DT[beta.dtype], flags, 0,
                        _strides(q), _strides(k), _strides(v), _strides(g), _strides(beta),
                        _strides(do))


def _in_place_ok(x):
    """Whether the kernels can read a (B, T, H[, D]) input view where it lies: the last axis
    unit-stride (for 4-D views), non-negative strides that span whole 16-byte units and a
    16-byte aligned base (what the tensor-core kernels' TMA loads need).  Anything else is
    copied into a dense tensor first."""
    if x.is_contiguous():
        return True
    st, es = x.stride(), x.element_size()
    if x.dim() == 4 and st[3] != 1:
        return False
    if any(s < 0 for s in st):
        return False
    if x.dim() == 3:  # beta: read element by element
        return True
    return all((s * es) % 16 == 0 for s in st[:3]) and x.data_ptr() % 16 == 0


def _dense_unless_readable(x):
    return x if _in_place_ok(x) else x.contiguous()


def _check_shapes(q, k, v, g, beta, state):
    if q.dim() != 4:
        raise ValueError(f"q must be (B, L, H, D), got {tuple(q.shape)}")
    B, T, H, D = q.shape
    for n, x in (("k", k), ("v", v), ("g", g)):
        if tuple(x.shape) != (B, T, H, D):
            raise ValueError(f"{n} shape {tuple(x.shape)} != q shape {(B, T, H, D)}")
    if tuple(beta.shape) != (B, T, H):
        raise ValueError(f"beta shape {tuple(beta.shape)} != {(B, T, H)}")
    if state is not None and tuple(state.shape) != (B, H, D, D):
        raise ValueError(f"state shape {tuple(state.shape)} != {(B, H, D, D)}")
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q, k, v must share one dtype")
    devs = {x.device for x in (q, k, v, g, beta) + ((state,) if state is not None else ())}
    if len(devs) != 1:
        raise ValueError(f"all operands must be on one device, got {devs}")


def _canonical(q, k, v, g, beta, state):
    """Checks shapes, dtypes and devices, and returns the operands as the kernels read them:
    q, k, v, beta in their own dtype and g float32, as the caller's views where the kernels can
    read those in place (strides passed in the descriptor), else dense copies; the state dense
    float32."""
    q, k, v, g, beta, state = (_as_torch(x, n) for x, n in
                               ((q, "q"), (k, "k"), (v, "v"), (g, "g"), (beta, "beta"),
                                (state, "state")))
    _check_shapes(q, k, v, g, beta, state)
    q, k, v, beta = (_dense_unless_readable(x) for x in (q, k, v, beta))
    g = _dense_unless_readable(g) if g.dtype == torch.float32 else g.to(torch.float32).contiguous()
    if state is not None:
        state = state.to(torch.float32).contiguous()
    return q, k, v, g, beta, state


def _workspace(desc, backward, device):
    n = _lib.lib().kda_workspace_bytes(ctypes.byref(desc), backward)
    if n == 0:
        return None, 0
    return torch.empty(n, dtype=torch.uint8, device=device), n


def num_chunks(T: int, chunk_size: int) -> int:
    return (T + chunk_size - 1) // chunk_size


def kda_forward(q, k, v, g, beta, state=None, chunk_size=64, save_states=False, flags=0):
    """One ``kda_fwd`` call.  Returns (o, S_T, saved | None); ``saved`` is the opaque
    per-chunk record (uint8 device tensor) that ``kda_backward`` consumes."""
    L = _lib.lib()
    q, k, v, g, beta, state = _canonical(q, k, v, g, beta, state)
    B, T, H, D = q.shape
    desc = _desc(q, beta, chunk_size, flags, k, v, g)
    o = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    S_T = torch.empty((B, H, D, D), dtype=torch.float32, device=q.device)
    cs = None
    if save_states:
        n = L.kda_saved_bytes(ctypes.byref(desc))
        if n == 0:
            _lib.check(L.kda_check_desc(ctypes.byref(desc), 0) or -1, "kda_saved_bytes")
        cs = torch.empty(n, dtype=torch.uint8, device=q.device)
    ws, nws = _workspace(desc, 0, q.device)
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream().cuda_stream
        st = L.kda_fwd(ctypes.byref(desc), _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta),
                       _ptr(state), _ptr(o), _ptr(S_T), _ptr(cs), _ptr(ws), nws,
                       ctypes.c_void_p(stream))
    _lib.check(st, "kda_fwd")
    return o, S_T, cs


def kda_backward(q, k, v, g, beta, state, saved, do, dstate=None, chunk_size=64,
                 flags=0, want_dstate0=True):
    """One ``kda_bwd`` call.  Returns (dq, dk, dv, dg, dbeta, dstate0 | None)."""
    L = _lib.lib()
    q, k, v, g, beta, state = _canonical(q, k, v, g, beta, state)
    saved = _as_torch(saved, "saved")
    if saved is None or saved.dtype != torch.uint8 or not saved.is_contiguous():
        raise ValueError("saved must be the uint8 record kda_forward(save_states=True) returned")
    do = _as_torch(do, "do")
    if tuple(do.shape) != tuple(q.shape):
        raise ValueError(f"do shape {tuple(do.shape)} != q shape {tuple(q.shape)}")
    do = _dense_unless_readable(do.to(q.dtype))
    if dstate is not None:
        dstate = _as_torch(dstate, "dstate")
        if tuple(dstate.shape) != (q.shape[0], q.shape[2], q.shape[3], q.shape[3]):
            raise ValueError(f"dstate shape {tuple(dstate.shape)} != state shape")
        dstate = dstate.to(torch.float32).contiguous()
    B, T, H, D = q.shape
    desc = _desc(q, beta, chunk_size, flags, k, v, g, do)
    dq, dk, dv = (torch.empty(q.shape, dtype=q.dtype, device=q.device) for _ in range(3))
    dg = torch.empty((B, T, H, D), dtype=torch.float32, device=q.device)
    db = torch.empty(beta.shape, dtype=beta.dtype, device=q.device)
    ds0 = torch.empty((B, H, D, D), dtype=torch.float32, device=q.device) if want_dstate0 else None
    ws, nws = _workspace(desc, 1, q.device)
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream().cuda_stream
        st = L.kda_bwd(ctypes.byref(desc), _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta),
                       _ptr(state), _ptr(saved), _ptr(do), _ptr(dstate), _ptr(dq),
                       _ptr(dk), _ptr(dv), _ptr(dg), _ptr(db), _ptr(ds0), _ptr(ws), nws,
                       ctypes.c_void_p(stream))
    _lib.check(st, "kda_bwd")
    return dq, dk, dv, dg, db, ds0


RECURRENT_MAX_T = 16  # cuda_kda without gradients steps token by token up to this length


def kda_recurrent(q, k, v, g, beta, state=None):
    """One ``kda_fwd_recurrent`` call: the step form token by token (exact fp32 arithmetic, one
    launch), for decoding and short segments.  Returns (o, S_T); no gradients."""
    L = _lib.lib()
    q, k, v, g, beta, state = _canonical(q, k, v, g, beta, state)
    B, T, H, D = q.shape
    desc = _desc(q, beta, 64, 0, k, v, g)
    o = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    S_T = torch.empty((B, H, D, D), dtype=torch.float32, device=q.device)
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream().cuda_stream
        st = L.kda_fwd_recurrent(ctypes.byref(desc), _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta),
                                 _ptr(state), _ptr(o), _ptr(S_T), ctypes.c_void_p(stream))
    _lib.check(st, "kda_fwd_recurrent")
    return o, S_T


class CudaKdaFunction(torch.autograd.Function):
    """Autograd wiring of the forward/VJP pair (the torch counterpart of the reference's
    ``mx.custom_function`` + ``.vjp`` at nope_gdn_mlx.py:2734-2809).  The forward saves one
    record per chunk (the chunk-entry state and solved WY values, as the reference's U_traj /
    S_traj); the backward recomputes every other intra-chunk quantity from the inputs."""

    @staticmethod
    def forward(ctx, q, k, v, g, beta, state, chunk_size, flags):
        o, S_T, cs = kda_forward(q, k, v, g, beta, state, chunk_size, save_states=True, flags=flags)
        ctx.save_for_backward(q, k, v, g, beta, state, cs)
        ctx.chunk_size, ctx.flags = chunk_size, flags
        ctx.has_state = state is not None
        return o, S_T

    @staticmethod
    def backward(ctx, do, dS_T):
        q, k, v, g, beta, state, cs = ctx.saved_tensors
        do = torch.zeros(q.shape, dtype=q.dtype, device=q.device) if do is None else do.to(q.dtype)
        dS_T = None if dS_T is None else dS_T.float().contiguous()
        dq, dk, dv, dg, db, ds0 = kda_backward(q, k, v, g, beta, state, cs, do, dS_T,
                                               ctx.chunk_size, ctx.flags,
                                               want_dstate0=ctx.has_state)
        return dq, dk, dv, dg, db, ds0, None, None


def cuda_kda(q, k, v, g, beta, state: Optional[torch.Tensor] = None, chunk_size: int = 64,
             *, force_generic: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """Chunkwise KDA on the GPU: returns (output in q.dtype, final state float32).

    ``force_generic`` selects the fp32 SIMT kernels even where a tensor-core kernel exists.
    fp32 inputs always run on the fp32 kernels.
    """
    q, k, v, g, beta, state = _canonical(q, k, v, g, beta, state)
    flags = _lib.KDA_FLAG_FORCE_GENERIC if force_generic else 0
    need_grad = torch.is_grad_enabled() and any(
        x is not None and x.requires_grad for x in (q, k, v, g, beta, state))
    if need_grad:
        # fail before the forward runs if no backward kernel covers the shape (e.g. D = 128)
        st = _lib.lib().kda_check_desc(ctypes.byref(_desc(q, beta, chunk_size, flags, k, v, g)), 1)
        if st:
            raise ValueError(f"cuda_kda: gradients need a backward for this shape, which is not "
                             f"available ({_lib.lib().kda_strerror(st).decode()})")
        return CudaKdaFunction.apply(q, k, v, g, beta, state, chunk_size, flags)
    if q.shape[1] <= RECURRENT_MAX_T and q.shape[3] in (16, 32, 64, 128) and not force_generic:
        return kda_recurrent(q, k, v, g, beta, state)
    o, S_T, _ = kda_forward(q, k, v, g, beta, state, chunk_size, save_states=False, flags=flags)
    return o, S_T


def _gate_struct(f, A_log, dt_bias, b, allow_neg_eigval):
    return _lib.KdaGate(ctypes.c_void_p(f.data_ptr()), ctypes.c_void_p(A_log.data_ptr()),
                        ctypes.c_void_p(dt_bias.data_ptr()), ctypes.c_void_p(b.data_ptr()),
                        int(bool(allow_neg_eigval)), 0)


def _canonical_gated(q, k, v, f, A_log, dt_bias, b, state):
    """The gated entry points' operand checks; returns dense operands (A_log, dt_bias and the
    state as float32)."""
    q, k, v, f, A_log, dt_bias, b, state = (
        _as_torch(x, n) for x, n in ((q, "q"), (k, "k"), (v, "v"), (f, "f"), (A_log, "A_log"),
                                     (dt_bias, "dt_bias"), (b, "b"), (state, "state")))
    if q.dim() != 4:
        raise ValueError(f"q must be (B, L, H, D), got {tuple(q.shape)}")
    B, T, H, D = q.shape
    _check_shapes(q, k, v, f, b, state)
    if q.dtype != torch.bfloat16 or f.dtype != torch.bfloat16:
        raise ValueError("the fused-gate path needs bf16 q, k, v and f")
    if tuple(A_log.shape) != (H,) or tuple(dt_bias.shape) not in ((H * D,), (H, D)):
        raise ValueError(f"A_log must be ({H},) and dt_bias ({H * D},)")
    q, k, v, f, b = (_dense_unless_readable(x) for x in (q, k, v, f, b))
    A_log = A_log.to(torch.float32).contiguous()
    dt_bias = dt_bias.to(torch.float32).reshape(H * D).contiguous()
    if state is not None:
        state = state.to(torch.float32).contiguous()
    return q, k, v, f, A_log, dt_bias, b, state


def kda_forward_gated(q, k, v, f, A_log, dt_bias, b, state=None, chunk_size=64,
                      allow_neg_eigval=False, save_states=False):
    """One ``kda_fwd_gated`` call: the decay gate g = -exp(A_log) softplus(f + dt_bias) and
    the write gate beta = s sigmoid(b) are computed inside the chunk kernel
    (nope_gdn_mlx.py:802-816).  Returns (o, S_T, saved | None)."""
    L = _lib.lib()
    q, k, v, f, A_log, dt_bias, b, state = _canonical_gated(q, k, v, f, A_log, dt_bias, b, state)
    desc = _desc(q, b, chunk_size, 0, k, v, f)  # f takes g's place in the descriptor
    o = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    B, T, H, D = q.shape
    S_T = torch.empty((B, H, D, D), dtype=torch.float32, device=q.device)
    cs = None
    if save_states:
        n = L.kda_saved_bytes(ctypes.byref(desc))
        if n == 0:
            _lib.check(L.kda_check_desc(ctypes.byref(desc), 0) or -1, "kda_saved_bytes")
        cs = torch.empty(n, dtype=torch.uint8, device=q.device)
    ws, nws = _workspace(desc, 0, q.device)
    gate = _gate_struct(f, A_log, dt_bias, b, allow_neg_eigval)
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream().cuda_stream
        st = L.kda_fwd_gated(ctypes.byref(desc), _ptr(q), _ptr(k), _ptr(v), ctypes.byref(gate),
                             _ptr(state), _ptr(o), _ptr(S_T), _ptr(cs), _ptr(ws), nws,
                             ctypes.c_void_p(stream))
    _lib.check(st, "kda_fwd_gated")
    return o, S_T, cs


def kda_backward_gated(q, k, v, f, A_log, dt_bias, b, state, saved, do, dstate=None,
                       chunk_size=64, allow_neg_eigval=False, want_dstate0=True):
    """One ``kda_bwd_gated`` call.  Returns (dq, dk, dv, df, db, dA_log, ddt_bias,
    dstate0 | None): the VJP of the recurrence chained through both gates."""
    L = _lib.lib()
    q, k, v, f, A_log, dt_bias, b, state = _canonical_gated(q, k, v, f, A_log, dt_bias, b, state)
    saved = _as_torch(saved, "saved")
    if saved is None or saved.dtype != torch.uint8 or not saved.is_contiguous():
        raise ValueError("saved must be the uint8 record kda_forward_gated(save_states=True) returned")
    do = _as_torch(do, "do")
    if tuple(do.shape) != tuple(q.shape):
        raise ValueError(f"do shape {tuple(do.shape)} != q shape {tuple(q.shape)}")
    do = _dense_unless_readable(do.to(q.dtype))
    if dstate is not None:
        dstate = _as_torch(dstate, "dstate").to(torch.float32).contiguous()
    desc = _desc(q, b, chunk_size, 0, k, v, f, do)
    B, T, H, D = q.shape
    dq, dk, dv, df = (torch.empty(q.shape, dtype=q.dtype, device=q.device) for _ in range(4))
    db = torch.empty(b.shape, dtype=b.dtype, device=q.device)
    dA = torch.empty((H,), dtype=torch.float32, device=q.device)
    ddtb = torch.empty((H * D,), dtype=torch.float32, device=q.device)
    ds0 = torch.empty((B, H, D, D), dtype=torch.float32, device=q.device) if want_dstate0 else None
    ws, nws = _workspace(desc, 1, q.device)
    gate = _gate_struct(f, A_log, dt_bias, b, allow_neg_eigval)
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream().cuda_stream
        st = L.kda_bwd_gated(ctypes.byref(desc), _ptr(q), _ptr(k), _ptr(v), ctypes.byref(gate),
                             _ptr(state), _ptr(saved), _ptr(do), _ptr(dstate), _ptr(dq), _ptr(dk),
                             _ptr(dv), _ptr(df), _ptr(db), _ptr(dA), _ptr(ddtb), _ptr(ds0),
                             _ptr(ws), nws, ctypes.c_void_p(stream))
    _lib.check(st, "kda_bwd_gated")
    return dq, dk, dv, df, db, dA, ddtb, ds0


class CudaKdaGatedFunction(torch.autograd.Function):
    """Autograd wiring of ``kda_fwd_gated`` / ``kda_bwd_gated``: the gate lines of
    ``GatedDeltaLayer.__call__`` (nope_gdn_mlx.py:802-816) and the recurrence as one op."""

    @staticmethod
    def forward(ctx, q, k, v, f, A_log, dt_bias, b, state, chunk_size, allow_neg_eigval):
        o, S_T, cs = kda_forward_gated(q, k, v, f, A_log, dt_bias, b, state, chunk_size,
                                       allow_neg_eigval, save_states=True)
        ctx.save_for_backward(q, k, v, f, A_log, dt_bias, b, state, cs)
        ctx.chunk_size, ctx.allow_neg = chunk_size, allow_neg_eigval
        ctx.has_state = state is not None
        return o, S_T

    @staticmethod
    def backward(ctx, do, dS_T):
        q, k, v, f, A_log, dt_bias, b, state, cs = ctx.saved_tensors
        do = torch.zeros(q.shape, dtype=q.dtype, device=q.device) if do is None else do.to(q.dtype)
        dS_T = None if dS_T is None else dS_T.float().contiguous()
        dq, dk, dv, df, db, dA, ddtb, ds0 = kda_backward_gated(
            q, k, v, f, A_log, dt_bias, b, state, cs, do, dS_T, ctx.chunk_size, ctx.allow_neg,
            want_dstate0=ctx.has_state)
        return dq, dk, dv, df, dA, ddtb, db, ds0, None, None


def cuda_kda_gated(q, k, v, f, A_log, dt_bias, b, state: Optional[torch.Tensor] = None,
                   chunk_size: int = 64, allow_neg_eigval: bool = False
                   ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Channel-wise KDA with both gates fused into the chunk kernels.

    ``f`` is the decay projection output (B, L, H, D) in q's dtype (bf16), ``A_log`` (H,)
    and ``dt_bias`` (H*D,) are float32 parameters, ``b`` is the write-gate projection
    output (B, L, H).  Equivalent to ``cuda_kda(q, k, v, g, beta, state)`` with
    g = -exp(A_log) softplus(f + dt_bias) and beta = (2 if allow_neg_eigval else 1) sigmoid(b)
    (nope_gdn_mlx.py:802-816), without materialising g or beta.  bf16 q/k/v/f only.
    """
    q, k, v, f, A_log, dt_bias, b, state = _canonical_gated(q, k, v, f, A_log, dt_bias, b, state)
    need_grad = torch.is_grad_enabled() and any(
        x is not None and x.requires_grad for x in (q, k, v, f, A_log, dt_bias, b, state))
    if need_grad:
        return CudaKdaGatedFunction.apply(q, k, v, f, A_log, dt_bias, b, state, chunk_size,
                                          allow_neg_eigval)
    o, S_T, _ = kda_forward_gated(q, k, v, f, A_log, dt_bias, b, state, chunk_size,
                                  allow_neg_eigval)
    return o, S_T
