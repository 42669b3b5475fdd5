/*
 * kda_b200.h -- C ABI of libkda_b200.so, the B200 (sm_100a) chunkwise KDA recurrence.
 *
 * KDA (Kimi Delta Attention) is Gated DeltaNet with a per-channel log-decay g <= 0.  Per
 * (batch b, head h) with state S in R^{Dv x Dk} (rows = value dim, decay acts on columns):
 *     S_t = (S_{t-1} diag(exp g_t)) (I - beta_t k_t k_t^T) + beta_t v_t k_t^T,   o_t = S_t q_t
 * computed chunkwise (WY/UT form).  There is no scale inside the op (the caller pre-scales q).
 *
 * These entry points replace the reference's per-path compute methods and the MSL kernels
 * they launch through mx.fast.metal_kernel (HananKibria/MLX_VIT, nope_gdn_mlx.py):
 *   kda_fwd  <- GatedDeltaLayer._chunkwise_kda_forward (nope_gdn_mlx.py:2318-2456) and
 *               _chunkwise_kda_with_traj (:2484-2571): one call does the whole layer
 *               recurrence (preamble :549-582, M/M_oq kernel :1301-1469, IA build :585-597,
 *               per-chunk solve+finalize kernels :1519-2055); with saved != NULL it also
 *               saves what the backward needs per chunk (the U_traj / S_traj of :2565-2567).
 *   kda_bwd  <- the vjp of _get_chunkwise_kda_recurrence_fn (:2746-2809) and
 *               _chunkwise_kda_backward (:2579-2720), including the triangular-solve and
 *               M-backward kernels (:1209-1286, :2080-2295).
 * Semantics (outputs, final state, all gradients) follow the reference's `compiled` path
 * _loop_compiled_kda (:890-917) and MLX autograd through it.
 *
 * Conventions
 *   - All pointers are device pointers; buffers are owned by the caller; the library keeps no
 *     allocation of its own and writes only the listed outputs (and the caller's workspace).
 *   - Layouts are row-major [B, T, H, D]:  q, k, g, dO, dq, dk, dg: [B, T, H, Dk];  v, o, dv:
 *     [B, T, H, Dv];  beta, dbeta: [B, T, H];  state0, stateT, dstateT, dstate0: [B, H, Dv, Dk]
 *     float32.  The inputs q, k, v, g, beta, dO may be strided views (KdaDesc strides, the
 *     head dimension unit-stride; the reference's (B, L, H, D) arrays are read without the head
 *     fold of nope_gdn_mlx.py:833-838); every output is dense.  `saved` is an opaque device buffer of kda_saved_bytes() bytes that kda_fwd fills
 *     and kda_bwd reads (per-chunk entry states and WY values); pass it between the two calls
 *     with the same descriptor.
 *   - dtype_qkv applies to q, k, v, o, dO, dq, dk, dv;  dtype_beta to beta and dbeta;
 *     g, dg and every state are float32 (nope_gdn_mlx.py:804, :906).
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Calls are asynchronous.
 *   - Every function returns 0 on success or a negative KDA_ERR_* status; kda_strerror()
 *     names it.  No exception crosses the ABI and no CPU fallback exists.
 */
#ifndef KDA_B200_H
#define KDA_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(_WIN32)
#define KDA_API
#else
#define KDA_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define KDA_ABI_VERSION 6

enum kda_dtype { KDA_F32 = 0, KDA_BF16 = 1, KDA_F16 = 2 };

enum kda_status {
  KDA_OK = 0,
  KDA_ERR_INVALID_ARG = -1,   /* null pointer, non-positive size, bad descriptor   */
  KDA_ERR_UNSUPPORTED = -2,   /* shape/chunk combination no kernel here implements */
  KDA_ERR_DTYPE = -3,         /* dtype code not accepted for that operand          */
  KDA_ERR_MISALIGNED = -4,    /* pointer not aligned to 16 bytes                   */
  KDA_ERR_WORKSPACE = -5,     /* workspace missing or smaller than required        */
  KDA_ERR_CUDA = -6,          /* a CUDA launch or runtime call failed              */
  KDA_ERR_TIMEOUT = -7,       /* a bounded device-side wait gave up                */
  KDA_ERR_SCRATCH_LIMIT = -8  /* kda_bwd_noalloc: problem needs more than its scratch */
};

/* Flags for KdaDesc.flags */
#define KDA_FLAG_FORCE_GENERIC 0x1  /* use the fp32 SIMT kernels even where a tensor-core
                                       kernel exists (testing / fp32-exact arithmetic) */
#define KDA_FLAG_DEBUG_WAIT_TIMEOUT 0x2  /* testing only: the tensor-core forward's state scan
                                       first waits (a few polls) on a barrier that nothing
                                       completes, so its bounded-wait failure path runs: the
                                       call returns 0, kda_device_status() then reports
                                       KDA_ERR_TIMEOUT and the output is not written */

/* Element strides of one input along batch, time and head; the last axis (D) is unit-stride.
 * All three zero means the dense layout ([B, T, H, D]: T*H*D, H*D, D; [B, T, H]: T*H, H, 1). */
typedef struct KdaStrides {
  int64_t b, t, h;
} KdaStrides;

typedef struct KdaDesc {
  int64_t B, T, H;     /* batch, sequence length, heads                          */
  int64_t Dk, Dv;      /* key/query dim and value dim (the reference has Dk==Dv) */
  int64_t chunk;       /* chunk size C (GatedDeltaLayer.chunk_size)              */
  int32_t dtype_qkv;   /* enum kda_dtype                                         */
  int32_t dtype_beta;  /* enum kda_dtype                                         */
  int32_t flags;       /* KDA_FLAG_*                                             */
  int32_t reserved;
  /* input views read in place (e.g. q, k, v as slices of one fused projection, time-major
   * [B, T, H, D] with any b / t / h strides).  The tensor-core kernels read them by TMA, which
   * needs every nonzero stride times the element size to be a multiple of 16 bytes (else
   * KDA_ERR_MISALIGNED).  With the fused gates, f takes g's strides and b beta's.  Outputs,
   * states and the saved record are always dense. */
  KdaStrides q, k, v, g, beta, dO;
} KdaDesc;

/* ABI version of the loaded library (KDA_ABI_VERSION it was built with). */
KDA_API int kda_abi_version(void);

/* Static string for a status code. */
KDA_API const char *kda_strerror(int status);

/* Validate a descriptor without touching memory: 0 if some kernel implements it. */
KDA_API int kda_check_desc(const KdaDesc *desc, int backward);

/* Workspace bytes kda_fwd (backward = 0) or kda_bwd (backward = 1) needs; 0 means the
 * call needs none and ws may be NULL.  Returns 0 on an invalid descriptor as well. */
KDA_API size_t kda_workspace_bytes(const KdaDesc *desc, int backward);

/* Bytes of the `saved` buffer kda_fwd fills for kda_bwd (the reference keeps the same data
 * as the U_traj / S_traj outputs of _chunkwise_kda_with_traj, nope_gdn_mlx.py:2484-2571).
 * Returns 0 on an invalid descriptor. */
KDA_API size_t kda_saved_bytes(const KdaDesc *desc);

/* Device-side status of the current device: KDA_ERR_TIMEOUT if a bounded wait inside a
 * kernel gave up since the last reset (the kernel then skipped its remaining work), else 0.
 * Synchronises the current device; with reset != 0 it also clears the status.
 * No reference counterpart (the reference has no device-side waits). */
KDA_API int kda_device_status(int reset);

/* Number of kernels this library has launched in this process (instrumentation; used by
 * benchmarks to count device launches inside a timed region).  No reference counterpart. */
KDA_API uint64_t kda_launch_counter(void);

/* Forward.  state0 may be NULL (zero initial state).  saved may be NULL (inference);
 * training passes a kda_saved_bytes() buffer and hands it to kda_bwd.
 * Replaces: GatedDeltaLayer._chunkwise_kda_forward / _chunkwise_kda_with_traj
 * (nope_gdn_mlx.py:2318-2456, :2484-2571); semantics of _loop_compiled_kda (:890-917). */
KDA_API int kda_fwd(const KdaDesc *desc, const void *q, const void *k, const void *v,
            const float *g, const void *beta, const float *state0,
            void *o, float *stateT, void *saved,
            void *ws, size_t ws_bytes, void *stream);

/* Backward (VJP).  state0 may be NULL (zero); dstateT may be NULL (zero cotangent);
 * dstate0 may be NULL (not wanted).  saved is the buffer kda_fwd filled.
 * Replaces: the vjp of _get_chunkwise_kda_recurrence_fn and _chunkwise_kda_backward
 * (nope_gdn_mlx.py:2746-2809, :2579-2720). */
KDA_API int kda_bwd(const KdaDesc *desc, const void *q, const void *k, const void *v,
            const float *g, const void *beta, const float *state0,
            const void *saved, const void *dO, const float *dstateT,
            void *dq, void *dk, void *dv, float *dg, void *dbeta, float *dstate0,
            void *ws, size_t ws_bytes, void *stream);

/* Token-by-token forward: the step form, exact in fp32, one launch, no chunk padding; for
 * decoding and short segments (the state carried between calls).  Dk == Dv in {16, 32, 64, 128};
 * desc->chunk is validated but unused.  No saved record (inference only).
 * Replaces: the step path _kda_step_fused looped by _loop_compiled_kda / _loop_naive_kda
 * (nope_gdn_mlx.py:616-638, :890-917, :2870-2892) and the step kernels (:2946-3036). */
KDA_API int kda_fwd_recurrent(const KdaDesc *desc, const void *q, const void *k, const void *v,
                              const float *g, const void *beta, const float *state0, void *o,
                              float *stateT, void *stream);

/* The layer's row operations around the recurrence, one fused pass each (bf16 I/O, fp32
 * arithmetic, 16-byte aligned pointers):
 *   kda_l2norm_silu_fwd:  y = l2norm(silu(x)) * scale over rows of n contiguous elements (n a
 *                         multiple of 8, at most 8192).  In the layer a row is one token's whole
 *                         H*D channel vector (q: scale = D^-1/2, k: 1), as the reference
 *                         normalises before its head reshape (nope_gdn_mlx.py:797-799, :818-821).
 *   kda_gated_rmsnorm_fwd: y = rmsnorm(o) * w * sigmoid(gate) over rows of D = 64 or 128 (one
 *                         head), w float32 [D]
 * and their VJPs (dw float32 [D], overwritten).
 * Replaces: GatedDeltaLayer.__call__'s "SiLU + L2 norm + scale" lines (nope_gdn_mlx.py:797-799,
 * l2_normalize :76-79) and its output RMSNormGated (:340-371, applied at :880-885). */
KDA_API int kda_l2norm_silu_fwd(int64_t rows, int n, const void *x, void *y, float scale, void *stream);
KDA_API int kda_l2norm_silu_bwd(int64_t rows, int n, const void *x, const void *dy, void *dx, float scale,
                                void *stream);
KDA_API int kda_gated_rmsnorm_fwd(int64_t rows, int D, const void *o, const void *gate, const float *w,
                                  void *y, float eps, void *stream);
/* The layer's short causal depthwise convolution (kernel 4) with SiLU, and for q / k the L2 norm
 * over each token's whole H*D channel row and the scale (norm != 0), in one pass: x, y [B, T, H*D]
 * bf16 (H*D a multiple of 8, at most 2048), w [H*D][4] and bias [H*D] float32.  The VJP writes dx
 * (bf16) and dw, db (float32, overwritten) and needs a float32 [B, T, H*D] scratch.
 * Replaces: ShortCausalConv1d (nope_gdn_mlx.py:400-431) applied at :793-795 and followed by the
 * SiLU / L2 norm of :797-799. */
KDA_API int kda_conv_silu_fwd(int64_t B, int64_t T, int H, int D, const void *x, const float *w,
                              const float *bias, void *y, int norm, float scale, void *stream);
KDA_API int kda_conv_silu_bwd(int64_t B, int64_t T, int H, int D, const void *x, const float *w,
                              const float *bias, const void *dy, void *dx, float *dw, float *db,
                              int norm, float scale, float *dz_scratch, void *stream);
KDA_API int kda_gated_rmsnorm_bwd(int64_t rows, int D, const void *o, const void *gate, const float *w,
                                  const void *dy, void *dout, void *dgate, float *dw, float eps,
                                  void *stream);

/* The layer's decay and write gates, fused into the kernels' load path (channel-wise KDA,
 * GatedDeltaLayer.__call__, nope_gdn_mlx.py:802-816):
 *   g    = -exp(A_log[h]) * softplus(f + dt_bias[h * Dk + d])   (softplus as :83-86)
 *   beta = sigmoid(b), times 2 when allow_neg_eigval (:814-816).
 * f is the gate projection f_proj_2(f_proj_1(x)) as [B, T, H, Dk] in dtype_qkv, b the write-
 * gate logits b_proj(x) as [B, T, H] in dtype_beta; A_log [H] and dt_bias [H * Dk] are fp32
 * (the reference keeps them fp32, :4943-4963).  Needs the tensor-core configuration
 * (Dk = Dv = 64, chunk 64, bf16 q/k/v). */
typedef struct KdaGate {
  const void *f;
  const float *A_log;
  const float *dt_bias;
  const void *b;
  int32_t allow_neg_eigval;
  int32_t reserved;
} KdaGate;

/* kda_fwd with the gates computed in-kernel from KdaGate instead of g and beta.
 * Replaces: GatedDeltaLayer.__call__'s decay / write gate lines (:802-816) followed by the
 * chunkwise path (see kda_fwd). */
KDA_API int kda_fwd_gated(const KdaDesc *desc, const void *q, const void *k, const void *v,
                          const KdaGate *gate, const float *state0, void *o, float *stateT,
                          void *saved, void *ws, size_t ws_bytes, void *stream);

/* kda_bwd through the fused gates: df (dtype_qkv, [B, T, H, Dk]) and db (dtype_beta,
 * [B, T, H]) are the cotangents of f and b; dA_log [H] and ddt_bias [H * Dk] (fp32) are
 * overwritten with the parameter gradients summed over batch and time.
 * Replaces: the VJP of the same lines (MLX autograd through :802-816) and kda_bwd. */
KDA_API int kda_bwd_gated(const KdaDesc *desc, const void *q, const void *k, const void *v,
                          const KdaGate *gate, const float *state0, const void *saved,
                          const void *dO, const float *dstateT, void *dq, void *dk, void *dv,
                          void *df, void *db, float *dA_log, float *ddt_bias, float *dstate0,
                          void *ws, size_t ws_bytes, void *stream);

/* Size of the static device scratch kda_bwd_noalloc uses (32 MiB; enough for about 4000
 * chunks of 64 tokens x heads, e.g. B=8 H=12 T=1568 needs 2400). */
#define KDA_NOALLOC_SCRATCH_BYTES (32u << 20)

/* Backward that allocates nothing and takes no workspace: the same computation and arguments
 * as kda_bwd minus ws/ws_bytes, for callers that cannot call cudaMalloc (a host that owns all
 * device memory through its own pool, or one that must not trigger the device
 * synchronisation an allocation can cause).  Its scratch is a static device array of
 * KDA_NOALLOC_SCRATCH_BYTES that every GPU loading the library holds until exit; a problem
 * that needs more returns KDA_ERR_SCRATCH_LIMIT.  The first call on a device looks up the
 * array's address, so make it before any stream capture.  All calls share the array, so
 * calls that overlap on the GPU race on it.  No counterpart in the reference. */
KDA_API int kda_bwd_noalloc(const KdaDesc *desc, const void *q, const void *k, const void *v,
                            const float *g, const void *beta, const float *state0,
                            const void *saved, const void *dO, const float *dstateT,
                            void *dq, void *dk, void *dv, float *dg, void *dbeta, float *dstate0,
                            void *stream);

#ifdef __cplusplus
}
#endif

#endif /* KDA_B200_H */
