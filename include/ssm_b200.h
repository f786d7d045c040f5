/*
 * ssm_b200.h -- C ABI of the B200 (sm_100a) SSM-scan kernels.
 *
 * Plain pointers, sizes and a stream handle; no torch types.  Every entry point
 * returns an ssm_status (0 = success) and never throws across the boundary.
 * All pointers are device pointers unless stated otherwise; all tensors are
 * dense row-major (the Python layer makes them contiguous).  Kernels are
 * enqueued on `stream` (a cudaStream_t, or NULL for the legacy default stream)
 * and the call returns without synchronising.
 *
 * The reference (dbydd/metal-kernelops 0.3.0) has no native FFI: its hot path
 * is three Python functions that launch Metal shaders through torch.mps.  Each
 * entry point below replaces the device work behind one of them; the file:line
 * citations are paths inside that project.
 */
#ifndef SSM_B200_H
#define SSM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum ssm_status {
    SSM_OK = 0,
    SSM_ERR_INVALID = 1,      /* shape / argument violates the op's contract   */
    SSM_ERR_UNSUPPORTED = 2,  /* dtype or size outside what the kernels handle */
    SSM_ERR_CUDA = 3,         /* a CUDA runtime call failed (see message)      */
    SSM_ERR_WORKSPACE = 4     /* workspace missing or smaller than required    */
} ssm_status;

typedef enum ssm_dtype {
    SSM_F32 = 0,
    SSM_BF16 = 1,
    SSM_F16 = 2
} ssm_dtype;

/* option bits shared by the three op groups */
#define SSM_HAS_D        0x01u  /* skip connection D                            */
#define SSM_HAS_Z        0x02u  /* gate: y *= silu(z)                            */
#define SSM_HAS_BIAS     0x04u  /* delta/dt bias added before the softplus      */
#define SSM_SOFTPLUS     0x08u  /* delta/dt = softplus(delta/dt + bias)          */
#define SSM_D_PER_HEAD   0x10u  /* Mamba-2: D is (nheads, headdim), not (nheads) */
#define SSM_DT_PER_ROW   0x20u  /* decode: dt is (batch, nheads, headdim)       */
#define SSM_HAS_INIT     0x40u  /* SSD: initial_states given                    */
#define SSM_HAS_DY       0x80u  /* backward: gradient of y given                */
#define SSM_HAS_DSTATE   0x100u /* backward: gradient of the state output given */
#define SSM_CUDA_CORES   0x200u /* SSD: run the CUDA-core kernels even where the tensor-core
                                   path applies (bf16/f16; headdim a multiple of 8 up to 64,
                                   128 or 256; dstate a multiple of 8 up to 128)            */
#define SSM_SCAN_PLAIN   0x2000u /* selective scan: run the plain-staging kernels even where
                                    the TMA-staged ones apply (same results bit for bit)    */
#define SSM_SCAN_LEAN    0x4000u /* selective scan: the forward saves only the state entering
                                    every 16-step chunk (4 * dstate bytes per 16 steps, no
                                    scan output); the backward recomputes the rest.  Pass the
                                    same flag to the size query, the forward and the backward */

/* Human-readable text for a status code, and the message of the last failure
 * on the calling thread (empty if none). */
const char* ssm_status_string(int status);
const char* ssm_last_error(void);

/* ------------------------------------------------------------------------- *
 * Mamba-1 selective scan.
 *
 * Replaces the device work of `metal_kernelops.selective_scan`
 * (src/metal_kernelops/scan.py:295-320): the bias add and softplus
 * (:311-314), `_Scan.forward` with its three kernels summarize / boundaries /
 * outputs (:237-255, MSL :60-127), the skip `+ u*D` (:316-317) and the gate
 * `* silu(z)` (:318-319) -- all fused into ssm_selective_scan_fwd -- and the
 * backward `_Scan.backward` (:257-280, MSL :129-232) plus the autograd of the
 * fused epilogue -- ssm_selective_scan_bwd.
 *
 *   u, delta, z, y, dout, du, ddelta, dz : (batch, dim, length), act_dtype
 *   A                                     : (dim, dstate) fp32
 *   B, C                                  : (batch, groups, dstate, length), bc_dtype
 *   D, delta_bias                         : (dim,) fp32
 *   dA (dim, dstate), dD (dim), ddelta_bias (dim): fp32, summed over the batch
 *   dB, dC                                : (batch, groups, dstate, length) fp32
 * ------------------------------------------------------------------------- */
typedef struct ssm_selective_scan_params {
    int64_t batch, dim, length, groups, dstate;
    int32_t act_dtype;          /* ssm_dtype of u, delta, z, y and their grads */
    int32_t bc_dtype;           /* ssm_dtype of B and C                        */
    uint32_t flags;             /* SSM_HAS_D | SSM_HAS_Z | SSM_HAS_BIAS | SSM_SOFTPLUS */
    /* forward inputs */
    const void* u;
    const void* delta;
    const float* A;
    const void* B;
    const void* C;
    const float* D;             /* may be NULL without SSM_HAS_D    */
    const void* z;              /* may be NULL without SSM_HAS_Z    */
    const float* delta_bias;    /* may be NULL without SSM_HAS_BIAS */
    /* forward output */
    void* y;
    /* saved for the backward (checkpoint_bytes, 16-byte aligned): the fp32
     * states entering every 4-step sub-block, then (with SSM_HAS_Z) the scan
     * output before the D skip and the gate in act_dtype; with SSM_SCAN_LEAN
     * only the states entering every 16-step chunk.  Written by the forward
     * and read by the backward (NULL in the forward = inference, nothing
     * saved) */
    float* checkpoints;
    /* backward */
    const void* dout;
    void* du;
    void* ddelta;
    void* dz;                   /* may be NULL without SSM_HAS_Z */
    float* dA;
    float* dB;
    float* dC;
    float* dD;                  /* may be NULL without SSM_HAS_D    */
    float* ddelta_bias;         /* may be NULL without SSM_HAS_BIAS */
    /* scratch: the backward's deterministic partial sums, and the segment
     * states of either pass (sizes from ssm_selective_scan_sizes /
     * ssm_selective_scan_fwd_workspace) */
    void* workspace;
    size_t workspace_bytes;
    /* optional device word (NULL: none), the same slot every op's params
     * carry: a TMA-staged kernel whose tile wait gives up (a bounded mbarrier
     * wait) writes its error code here and in the per-device flag that
     * ssm_take_kernel_error reads; the plain-staging kernels have no such
     * waits.  Start it at 0. */
    int32_t* status;
} ssm_selective_scan_params;

/* Sizes of the forward's checkpoint buffer and of the backward's workspace,
 * for exactly these params: shapes, dtypes and flags (the checkpoint buffer
 * holds the saved scan output only with SSM_HAS_Z), so query with the flags
 * the forward will be called with. */
int ssm_selective_scan_sizes(const ssm_selective_scan_params* p,
                             size_t* checkpoint_bytes, size_t* workspace_bytes);
/* Workspace the forward needs (passed in `workspace`): zero unless the problem
 * is too small to fill the GPU, in which case the forward cuts the sequence
 * into segments and keeps their states there.  No counterpart in the
 * reference (its forward always runs three chunked passes). */
int ssm_selective_scan_fwd_workspace(const ssm_selective_scan_params* p, size_t* workspace_bytes);
int ssm_selective_scan_fwd(const ssm_selective_scan_params* p, void* stream);
int ssm_selective_scan_bwd(const ssm_selective_scan_params* p, void* stream);

/* ------------------------------------------------------------------------- *
 * Mamba-2 decode state update.
 *
 * Replaces `metal_kernelops.cv.mamba2_state_update`
 * (src/metal_kernelops/cv/mamba2_state.py:759-819): the fused forward kernel
 * `state_update_$S` (:184-267, launched by `_launch` :601-637) and the
 * two-kernel deterministic backward `state_update_backward` +
 * `state_update_reduce` (:269-536, driven by `_StateUpdate.backward` :653-756).
 *
 *   state, new_state, grad_state, dnew   : (batch, nheads, headdim, dstate), state_dtype
 *   x, z, y, dy, dx, dz                  : (batch, nheads, headdim), state_dtype (fp32 grads)
 *   dt                                   : (batch, nheads) or (batch, nheads, headdim)
 *   A, dt_bias                           : (nheads,) fp32
 *   B, C                                 : (batch, ngroups, dstate)
 *   D                                    : (nheads,) or (nheads, headdim) fp32
 * new_state may alias state (in-place update, `out_state` of the reference).
 * The backward computes in fp32: its inputs other than A/D/dt_bias are fp32
 * (the wrapper widens them, as the reference's `_wide` does, :554-558) and
 * all its outputs are fp32.
 * ------------------------------------------------------------------------- */
typedef struct ssm_state_update_params {
    int64_t batch, nheads, headdim, dstate, ngroups;
    int32_t dtype;              /* ssm_dtype of state, x, dt, B, C, z, y (forward) */
    uint32_t flags;             /* SSM_HAS_D | SSM_D_PER_HEAD | SSM_HAS_Z | SSM_HAS_BIAS |
                                   SSM_SOFTPLUS | SSM_DT_PER_ROW | SSM_HAS_DY | SSM_HAS_DSTATE */
    const void* state;
    const void* x;
    const void* dt;
    const float* A;
    const void* B;
    const void* C;
    const float* D;
    const void* z;
    const float* dt_bias;
    void* new_state;            /* forward output; may equal `state` */
    void* y;                    /* forward output */
    /* backward (all fp32) */
    const float* dy;            /* may be NULL without SSM_HAS_DY     */
    const float* dnew;          /* may be NULL without SSM_HAS_DSTATE */
    float* grad_state;          /* gradient of the entering state */
    float* dx;
    float* ddt;                 /* shaped like dt */
    float* dA;
    float* dB;
    float* dC;
    float* dD;
    float* dz;
    float* ddt_bias;
    void* workspace;
    size_t workspace_bytes;
    /* forward only: with SSM_IO_DTYPE in flags, x, B, C and z are stored in
     * io_dtype (an ssm_dtype) instead of `dtype` -- e.g. bf16 activations
     * against an fp32 state, read without a widening copy; state, dt and y
     * stay in `dtype`. */
    int32_t io_dtype;
    /* optional device word (NULL: none), the same slot every op's params
     * carry; this op's kernels have no waits that can give up and never
     * write it. */
    int32_t* status;
} ssm_state_update_params;

int ssm_state_update_sizes(const ssm_state_update_params* p, size_t* workspace_bytes);
int ssm_state_update_fwd(const ssm_state_update_params* p, void* stream);
int ssm_state_update_bwd(const ssm_state_update_params* p, void* stream);

/* The decode backward for callers that cannot allocate device memory (a
 * runtime whose device memory is pre-planned and owned elsewhere, or code that
 * must not touch the allocator where the backward runs).  No counterpart in the
 * reference.  Same params and results as ssm_state_update_bwd, but
 * `workspace`/`workspace_bytes` are ignored: the scratch is one fixed device
 * array inside the library, SSM_STATE_UPDATE_STATIC_SCRATCH_BYTES large and
 * held by every GPU that loads the library until the process exits.  Problems
 * whose scratch (ssm_state_update_sizes) exceeds it return SSM_ERR_UNSUPPORTED.
 * Allocates nothing.  The first call on each device looks up the array's
 * device address (cudaGetSymbolAddress, with that device current) and caches
 * it, so make that first call before any stream capture.  All calls share the
 * array: calls whose kernels overlap on the GPU race and must be serialised. */
#define SSM_STATE_UPDATE_STATIC_SCRATCH_BYTES ((size_t)8 << 20)
int ssm_state_update_bwd_noalloc(const ssm_state_update_params* p, void* stream);

/* ------------------------------------------------------------------------- *
 * Mamba-2 SSD chunk scan.
 *
 * Replaces `metal_kernelops.cv.mamba2_chunk_scan`
 * (src/metal_kernelops/cv/mamba2_chunk.py:617-678): `_discretize` (:447-462),
 * `_chunk_states` (:465-484), `_state_passing` (:487-505), `_chunk_outputs`
 * (:508-533) and the fused Metal output stage `mamba2_cb` / `mamba2_scan`
 * (:182-347); the backward replaces the autograd of that composition.
 *
 *   x, z, y, dy, dx, dz                  : (batch, length, nheads, headdim), dtype
 *   dt, ddt                              : (batch, length, nheads), dt_dtype / fp32
 *   A, dA, dt_bias, ddt_bias             : (nheads,) fp32
 *   B, C                                 : (batch, length, ngroups, dstate), dtype
 *   dB, dC                               : (batch, length, ngroups, dstate) fp32
 *   D, dD                                : (nheads,) or (nheads, headdim) fp32
 *   initial_states, final_state          : (batch, nheads, headdim, dstate) fp32
 * ------------------------------------------------------------------------- */
typedef struct ssm_chunk_scan_params {
    int64_t batch, length, nheads, headdim, ngroups, dstate, chunk_size;
    int32_t dtype;              /* ssm_dtype of x, B, C, z, y */
    int32_t dt_dtype;           /* ssm_dtype of dt            */
    uint32_t flags;             /* SSM_HAS_D | SSM_D_PER_HEAD | SSM_HAS_Z | SSM_HAS_BIAS |
                                   SSM_SOFTPLUS | SSM_HAS_INIT | SSM_HAS_DY | SSM_HAS_DSTATE */
    const void* x;
    const void* dt;
    const float* A;
    const void* B;
    const void* C;
    const float* D;
    const void* z;
    const float* dt_bias;
    const float* initial_states;
    void* y;
    float* final_state;
    /* backward */
    const void* dy;             /* dtype of x */
    const float* dfinal;        /* may be NULL without SSM_HAS_DSTATE */
    void* dx;                   /* dtype of x */
    float* ddt;
    float* dA;
    float* dB;
    float* dC;
    float* dD;
    void* dz;                   /* dtype of x */
    float* ddt_bias;
    float* dinitial;
    /* forward: chunk states saved for the backward (may be NULL) */
    float* saved;
    void* workspace;
    size_t workspace_bytes;
    /* Elements between consecutive tokens of x and of B / C (0: the dense
     * nheads * headdim and ngroups * dstate); heads (groups) and their
     * headdim (dstate) elements stay packed within a token, and the batch
     * stride is length tokens.  x and B / C may so be column slices of one
     * wider (batch, length, columns) buffer.  Tensor-core path only (16-byte
     * multiples); the CUDA-core path returns SSM_ERR_UNSUPPORTED for them. */
    int64_t x_token_stride, bc_token_stride;
    /* optional device word (NULL: none).  A kernel of this op that gives up
     * on a bounded wait writes its non-zero code here (the first failure
     * wins; the word is never cleared by the library), besides the per-device
     * flag that ssm_take_kernel_error reads.  Start it at 0. */
    int32_t* status;
} ssm_chunk_scan_params;

int ssm_chunk_scan_sizes(const ssm_chunk_scan_params* p, size_t* saved_bytes,
                         size_t* workspace_bytes);
/* On the tensor-core path, when batch x heads needs more than one wave of the
 * per-(row, head) state kernels, the second half of the batch runs on an
 * internal non-blocking stream of the current device, forked from `stream` and
 * joined back into it by events before these return (not while `stream` is
 * being captured): work enqueued later on `stream` runs after the whole call. */
int ssm_chunk_scan_fwd(const ssm_chunk_scan_params* p, void* stream);
int ssm_chunk_scan_bwd(const ssm_chunk_scan_params* p, void* stream);

/* ------------------------------------------------------------------------- *
 * VMamba four-path 2D selective scan (ss2d).
 *
 * Replaces `metal_kernelops.cv.ss2d_scan`
 * (src/metal_kernelops/cv/path_scan.py:546-576): the forward `_PathScan.forward`
 * (transpose_states / path_summaries / boundaries / path_scan / merge_paths)
 * and the backward `_PathScan.backward` (:495-543: stacking copies, scan.py's
 * three backward kernels, merge_paths folds).  Path k of pixel (h, w) is step
 *   0: h*W + w    1: w*H + h    2: L-1-(h*W + w)    3: L-1-(w*H + h)
 * (L = H*W); the four path outputs are added as (p0 + p2) + (p1 + p3) and
 * multiplied by `scale` (1 for merge "sum", 0.25 for "mean").
 *
 *   u, dt, y, dout, du, ddt : (batch, channels, height, width), act_dtype
 *   A                       : (channels, dstate) fp32;  dA (channels, dstate) fp32
 *   B, C                    : (batch, groups, dstate, height, width), bc_dtype
 *   dB, dC                  : (batch, groups, dstate, height, width) fp32
 * The forward writes `checkpoints` (fp32, checkpoint_bytes) that the backward
 * reads; the forward and the backward each take a workspace of the size
 * ssm_ss2d_scan_sizes returns.
 * ------------------------------------------------------------------------- */
typedef struct ssm_ss2d_scan_params {
    int64_t batch, channels, height, width, groups, dstate;
    int32_t act_dtype;          /* ssm_dtype of u, dt, y, dout, du, ddt */
    int32_t bc_dtype;           /* ssm_dtype of B and C                 */
    float scale;                /* 1 (merge "sum") or 0.25 (merge "mean") */
    const void* u;
    const void* dt;
    const float* A;
    const void* B;
    const void* C;
    void* y;
    float* checkpoints;         /* may be NULL in the forward: nothing saved */
    const void* dout;
    void* du;
    void* ddt;
    float* dA;
    float* dB;
    float* dC;
    void* workspace;
    size_t workspace_bytes;
    /* optional device word (NULL: none), the same slot every op's params
     * carry; this op's kernels have no waits that can give up and never
     * write it. */
    int32_t* status;
} ssm_ss2d_scan_params;

int ssm_ss2d_scan_sizes(const ssm_ss2d_scan_params* p, size_t* checkpoint_bytes,
                        size_t* fwd_workspace_bytes, size_t* bwd_workspace_bytes);
int ssm_ss2d_scan_fwd(const ssm_ss2d_scan_params* p, void* stream);
int ssm_ss2d_scan_bwd(const ssm_ss2d_scan_params* p, void* stream);

/* ------------------------------------------------------------------------- *
 * Causal depthwise conv1d (the convolution in front of the scan).
 *
 * Replaces `metal_kernelops.cv.causal_conv1d_fn` and `causal_conv1d_update`
 * (src/metal_kernelops/cv/causal_conv1d.py:610-690, :690-756): the forward
 * kernel `causal_conv1d_fwd` (:73-150), the fused backward
 * `causal_conv1d_bwd` + `causal_conv1d_dwfinal` (:152-340, driven by
 * `_CausalConv1d.backward` :540-607) and the decode kernel
 * `causal_conv1d_update` (:342-385).
 *
 *   x, out, dout, dx                 : (batch, channels, length), dtype
 *   weight (channels, width), bias (channels): fp32 (the wrapper converts)
 *   initial_state, final_state, dinitial : (batch, channels, width - 1), dtype
 *   dweight (channels, width), dbias (channels): fp32
 * width (K) is 1..8.  Flags: SSM_HAS_BIAS, SSM_HAS_INIT, SSM_CONV_SILU.
 * final_state may be NULL (not written).  The backward takes a workspace of
 * ssm_causal_conv1d_sizes bytes; dweight/dbias may be NULL (not written).
 * ------------------------------------------------------------------------- */
#define SSM_CONV_SILU    0x400u /* conv1d: act = SiLU */
#define SSM_IO_DTYPE     0x800u /* decode forward: x, B, C, z in io_dtype       */
#define SSM_CHANNEL_LAST 0x1000u /* conv1d: x, out, dout, dx stored (batch, length, channels) */

typedef struct ssm_causal_conv1d_params {
    int64_t batch, channels, length, width;
    int32_t dtype;              /* ssm_dtype of x, out, states and their gradients */
    uint32_t flags;
    const void* x;
    const float* weight;
    const float* bias;
    const void* initial_state;
    void* out;
    void* final_state;
    const void* dout;
    void* dx;
    float* dweight;
    float* dbias;
    void* dinitial;
    void* workspace;
    size_t workspace_bytes;
    /* With SSM_CHANNEL_LAST: x, out, dout and dx are stored (batch, length,
     * channels) -- element (b, c, t) at (b * length + t) * row_stride + c --
     * with x_row_stride / dout_row_stride elements between rows of x / dout
     * (0: channels) and out / dx dense.  Rows and the base pointers 8-byte
     * aligned, channels a multiple of 8 bytes' worth of elements; no initial
     * or final state. */
    int64_t x_row_stride, dout_row_stride;
    /* optional device word (NULL: none).  A kernel of this op that gives up
     * on a bounded wait writes its non-zero code here (the first failure
     * wins; the word is never cleared by the library), besides the per-device
     * flag that ssm_take_kernel_error reads.  Start it at 0. */
    int32_t* status;
} ssm_causal_conv1d_params;

int ssm_causal_conv1d_sizes(const ssm_causal_conv1d_params* p, size_t* workspace_bytes);
int ssm_causal_conv1d_fwd(const ssm_causal_conv1d_params* p, void* stream);
int ssm_causal_conv1d_bwd(const ssm_causal_conv1d_params* p, void* stream);

/* Decode: `length` (q) new tokens per (batch, channel) row against a rolling
 * state of state_len >= width - 1 columns, updated in place to
 * cat(state, x)[..., -state_len:].  The state is addressed through its batch
 * and channel strides (elements; the last stride is 1), so it may be a slice
 * of a larger cache.  x and out are contiguous (batch, channels, length); the
 * state has the same dtype. */
typedef struct ssm_causal_conv1d_update_params {
    int64_t batch, channels, length, width, state_len;
    int64_t state_stride_batch, state_stride_channel;
    int32_t dtype;
    uint32_t flags;             /* SSM_HAS_BIAS | SSM_CONV_SILU */
    void* state;
    const void* x;
    const float* weight;
    const float* bias;
    void* out;
    /* optional device word (NULL: none), the same slot every op's params
     * carry; this op's kernels have no waits that can give up and never
     * write it. */
    int32_t* status;
} ssm_causal_conv1d_update_params;

int ssm_causal_conv1d_update(const ssm_causal_conv1d_update_params* p, void* stream);

/* ------------------------------------------------------------------------- *
 * Gated RMSNorm (mamba's rms_norm_ref): the normalisation after the SSD scan.
 *
 * Replaces `metal_kernelops.cv.rmsnorm_gated`
 * (src/metal_kernelops/cv/gated_norm.py:647-686): the fused forward and the
 * analytic backward of `_GatedRMSNorm` (:563-644).
 *
 *   x, z, out, dy, dx, dz : (rows, features), dtype (z may be NULL: no gate)
 *   weight, bias, dweight, dbias : (features,) fp32 (bias may be NULL)
 *   rstd : (rows, features / group_size) fp32, written by the forward (may be
 *          NULL there) and read by the backward
 * gate: 0 none, 1 silu(z) multiplies x before the norm (norm_before_gate =
 * False), 2 silu(z) multiplies the output (norm_before_gate = True).  Flags:
 * SSM_HAS_BIAS.  The backward takes a workspace of ssm_gated_rmsnorm_sizes
 * bytes; dweight/dbias may be NULL (not written).
 * ------------------------------------------------------------------------- */
typedef struct ssm_gated_rmsnorm_params {
    int64_t rows, features, group_size;
    int32_t dtype;
    int32_t gate;
    uint32_t flags;
    float eps;
    const void* x;
    const void* z;
    const float* weight;
    const float* bias;
    void* out;
    float* rstd;
    const void* dy;
    void* dx;
    void* dz;
    float* dweight;
    float* dbias;
    void* workspace;
    size_t workspace_bytes;
    /* elements between consecutive rows of x and of z (0: `features`, the
     * contiguous layout); features are contiguous within a row.  Lets z (and
     * x) be column slices of a wider projection output.  out, dy, dx and dz
     * are contiguous. */
    int64_t x_row_stride, z_row_stride;
    /* optional device word (NULL: none), the same slot every op's params
     * carry; this op's kernels have no waits that can give up and never
     * write it. */
    int32_t* status;
} ssm_gated_rmsnorm_params;

int ssm_gated_rmsnorm_sizes(const ssm_gated_rmsnorm_params* p, size_t* workspace_bytes);
int ssm_gated_rmsnorm_fwd(const ssm_gated_rmsnorm_params* p, void* stream);
int ssm_gated_rmsnorm_bwd(const ssm_gated_rmsnorm_params* p, void* stream);

/* Kernels that wait on an mbarrier give up after a bounded number of polls,
 * record a non-zero code in a per-device flag (and in the call's `status`
 * word, when given) and return.  This reads the flag of the current device
 * (synchronising with it) and clears it; 0 means no kernel gave up.
 * Reference: none (the Metal kernels have no such waits). */
int ssm_take_kernel_error(void);

/* Self-test of the failure path: one CTA waits, with the library's bounded
 * wait limited to `polls` polls, on a shared-memory mbarrier that nothing
 * arrives at (no copy is in flight), gives up, writes SSM_KERR_SELFTEST into
 * *status and returns.  The per-device flag is left alone.  Lets a caller (and
 * the tests) check that a wait which runs out surfaces as a status instead of
 * a hang, and that the context stays usable.  Reference: none. */
#define SSM_KERR_SELFTEST 99
int ssm_selftest_bounded_wait(int32_t* status, uint32_t polls, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SSM_B200_H */
