/*
 * omniwave_b200 -- C ABI of the B200-native BiGEMM operator.
 *
 * BiGEMM (OmniWeave's structured two-sided tiled GEMM) maps an NHWC activation
 * x[B,H,W,C] to a residual delta of the same shape.  For every spatial tile q_s
 * (16 tokens chosen by a route plan) and channel group q_c (d channels):
 *
 *     T = x[b, tok_idx[q_s,:], ch_idx[q_c,:]]                 (16 x d)
 *     U = A_u T B_u[q_c],  V = A_v T B_v[q_c]                (16 x rd)
 *     Z = silu(U) * V
 *     delta = (A_o Z B_o[q_c]) * mask * gamma[ch]            (16 x d)
 *
 * and delta is scattered back to the positions it was gathered from.  This is
 * the computation of the reference's ``bigemm_delta_reference``
 * (omniweave/ops/reference.py:120-173) with ``pack_tiles`` (:16-64) and
 * ``unpack_tiles`` (:67-117) folded into the kernels' loads and stores.
 *
 * Conventions
 *  - All tensor pointers are device pointers owned by the caller; the library
 *    only borrows them for the duration of the call.  It keeps no state
 *    between calls except immutable per-device kernel attributes, the
 *    per-device fault word (ow_device_fault) and, for
 *    ow_bigemm_fwd_noalloc only, that entry point's fixed scratch array and
 *    its cached device address (see its comment).
 *  - ``stream`` is a ``cudaStream_t`` passed as ``void*``.  Calls are
 *    asynchronous on that stream and never synchronise the device.
 *  - Every entry point returns OW_OK (0) or an error code; no C++ exception
 *    crosses the ABI.  ``ow_last_error()`` returns a thread-local message for
 *    the last failing call made by the calling thread.
 *  - Functions are reentrant: concurrent calls on different streams are safe
 *    as long as their workspaces do not overlap.  The exception is
 *    ow_bigemm_fwd_noalloc, whose calls share one scratch array and must not
 *    overlap on the GPU (see its comment).
 */
#ifndef OMNIWAVE_B200_H
#define OMNIWAVE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OW_ABI_VERSION 5

#if defined(__GNUC__)
#define OW_API __attribute__((visibility("default")))
#else
#define OW_API
#endif

/* Element types. */
enum {
  OW_DTYPE_F32 = 0,
  OW_DTYPE_F64 = 1,
  OW_DTYPE_BF16 = 2,
  OW_DTYPE_F16 = 3
};

/* Status codes. */
enum {
  OW_OK = 0,
  OW_ERR_INVALID = 1,      /* bad argument: null pointer, shape mismatch, ... */
  OW_ERR_UNSUPPORTED = 2,  /* valid but not supported (dtype, tile size, device) */
  OW_ERR_CUDA = 3,         /* a CUDA runtime call or kernel launch failed */
  OW_ERR_WORKSPACE = 4     /* workspace missing or smaller than required */
};

/*
 * Route description of one BiGEMM call.  Mirrors the reference ``RoutePlan``
 * (omniweave/models/routing.py:17-33): ``tok_idx`` is
 * ``plan.token_indices`` and ``ch_idx`` is ``plan.channel_indices``, both as
 * int32 device arrays, with pad index H*W for tokens and C for channels.
 * Pad entries are exactly the masked-off entries of the reference's masks.
 * Valid (non-pad) token indices must be distinct, and so must valid channel
 * indices (every plan the reference builds satisfies this).
 */
typedef struct ow_route_t {
  int32_t batch, height, width, channels; /* B, H, W, C of the NHWC activation */
  int32_t q_s, q_c;                       /* number of spatial tiles / channel groups */
  int32_t g, d, rd;                       /* tile tokens (16), channel tile, expanded tile */
  const int32_t* tok_idx;                 /* [q_s * g] */
  const int32_t* ch_idx;                  /* [q_c * d] */
  /* Channel-layout hint: 0 = unknown (any table); S >= 1 = the caller
   * states that channel group q is ch_idx[q*d + k] = c0(q) + S*k for every
   * k (S == 1: one run of d consecutive channels starting on a multiple of 8;
   * the radix routes at levels 1 and 2 give S = q_c).  The hint only selects
   * a kernel: with S == 1 the forward gathers the group's rows with TMA
   * straight from x.  The kernels verify it against the table; a group that
   * does not match is not computed and the device fault word reports code 2
   * (ow_device_fault). */
  int32_t ch_stride;
} ow_route_t;

/*
 * Inputs of a forward (and of the matching backward).
 *
 * Operator mode (``rstd == NULL``, ``residual == 0``) computes exactly the
 * reference ``bigemm(x=..., plan=..., ...)`` delta.  Block mode
 * (``rstd != NULL``, ``residual == 1``) fuses ``OmniWeaveBlock.forward``
 * (omniweave/models/block.py:80-108): the tile loads apply RMSNorm
 * ``x * rstd[token] * norm_w[c]`` and the stores write ``x + scale[b]*delta``.
 */
typedef struct ow_bigemm_args_t {
  ow_route_t route;
  const void* x;            /* [B,H,W,C] contiguous, dtype x_dtype */
  int32_t x_dtype;
  int32_t compute_dtype;    /* F64/F32: exact CUDA-core path; BF16/F16: tensor-core path */
  const void* rstd;         /* [B*H*W], F64 when compute is F64 else F32; NULL in operator mode */
  const void* norm_w;       /* [C] RMSNorm weight (block mode only) */
  const void* a_u;          /* [g,g] */
  const void* a_v;          /* [g,g] */
  const void* a_o;          /* [g,g] */
  const void* b_u;          /* [q_c,d,rd] */
  const void* b_v;          /* [q_c,d,rd] */
  const void* b_o;          /* [q_c,rd,d] */
  const void* gamma;        /* [C] LayerScale */
  int32_t w_dtype;          /* dtype of norm_w, a_*, b_*, gamma as stored */
  const float* sample_scale;/* [B] per-sample drop-path scale, or NULL */
  int32_t residual;         /* 1: out = x + delta (block mode) */
  void* out;                /* [B,H,W,C], dtype out_dtype (forward only) */
  int32_t out_dtype;
  void* workspace;          /* device scratch, >= ow_bigemm_workspace_size() bytes */
  size_t workspace_bytes;
} ow_bigemm_args_t;

/* Gradients written by ow_bigemm_bwd (all outputs overwrite, never accumulate). */
typedef struct ow_bigemm_grads_t {
  const void* dout;   /* [B,H,W,C] gradient of the forward's out, dtype out_dtype */
  void* dx;           /* [B,H,W,C] dtype x_dtype (block mode: includes the residual path) */
  void* da_u;         /* [g,g]     dtype w_dtype */
  void* da_v;
  void* da_o;
  void* db_u;         /* [q_c,d,rd] */
  void* db_v;
  void* db_o;         /* [q_c,rd,d] */
  void* dgamma;       /* [C] */
  void* dnorm_w;      /* [C] block mode only, else ignored */
} ow_bigemm_grads_t;

/*
 * Number of kernels this library has launched in this process (all devices,
 * all threads).  Lets a caller check that work really ran on the GPU.
 */
OW_API uint64_t ow_launch_count(void);

/*
 * Kernel timing for measurement tools.  While set, every call in this
 * process (any host thread) records the caller's CUDA events (cudaEvent_t
 * cast to void*) on the call's stream immediately before and after one of
 * its kernels:
 *   OW_PROF_FWD   the tensor-core forward kernel,
 *   OW_PROF_PACK  the backward pack kernel (operand images),
 *   OW_PROF_BWD   the backward role kernel,
 *   OW_PROF_FPACK the forward pack kernel (P_u | P_v images).
 * Passing NULL for both events stops recording for that kernel.  Returns
 * OW_ERR_INVALID for an unknown ``kernel``.  No counterpart in the reference
 * (it is a measurement aid, not part of the operator).
 */
#define OW_PROF_FWD 0
#define OW_PROF_PACK 1
#define OW_PROF_BWD 2
#define OW_PROF_FPACK 3
OW_API int ow_profile_events(int kernel, void* start, void* stop);

/* ABI version compiled into the library (OW_ABI_VERSION). */
OW_API int ow_abi_version(void);

/* Message of the last failing call on this thread ("" if none). */
OW_API const char* ow_last_error(void);

/*
 * Returns 1 if ``device`` can run this library's kernels (sm_100a), else 0.
 * Does not change the current device.
 */
OW_API int ow_device_supported(int device);

/*
 * Fault word of this library's kernels on ``device``: 0 when no kernel ever
 * gave up on a bounded wait (every wait on the GPU is bounded at 2 s), else a
 * nonzero code (1: a wait ran out; 2: a channel group did not match the
 * route's ch_stride hint; the outputs of that call are undefined).
 * One word per device is shared by every kernel of the library.  Calls are
 * asynchronous, so a fault surfaces here, not in the failing call's status:
 * this function synchronises the device first.  ``reset`` != 0 clears the
 * word after reading it.  Returns -1 if the device cannot be queried.
 */
OW_API int ow_device_fault(int device, int reset);

/*
 * Wait-timeout self-check, a test aid with no counterpart in the reference.
 * While ``probe_ns`` is nonzero (at most 1e9), every mbarrier-pipelined
 * kernel launched afterwards first waits ``probe_ns`` nanoseconds on a
 * barrier that nothing arrives on, before it issues any copy or MMA; the
 * wait runs out, the kernel skips its work and records code 1 in the fault
 * word.  Outputs of calls made while it is set are undefined.  Pass 0 to
 * turn it off.  Returns OW_ERR_INVALID above the limit.
 */
OW_API int ow_debug_wait_probe(uint32_t probe_ns);

/*
 * Bytes of workspace a forward (``for_backward == 0``) or backward
 * (``for_backward == 1``) call with these arguments needs.  Only the shape
 * and dtype fields of ``args`` are read.
 */
OW_API size_t ow_bigemm_workspace_size(const ow_bigemm_args_t* args, int for_backward);

/*
 * Per-token reciprocal RMS for the fused block: ``rstd[r] = 1/sqrt(mean_c
 * x[r,c]^2 + eps)``, the mean taken in float32 as the reference does
 * (omniweave/models/block.py:83-84).  ``rstd`` is F64 when compute_dtype is
 * F64, else F32.
 */
OW_API int ow_rmsnorm_rstd(const void* x, int32_t x_dtype, int32_t compute_dtype,
                    int64_t rows, int32_t channels, double eps, void* rstd, void* stream);

/*
 * Forward.  Replaces the reference's ``bigemm(...)`` dispatch target
 * (omniweave/ops/bigemm.py:24-73) for backend "cuda", and in block mode the
 * body of ``OmniWeaveBlock.forward`` (omniweave/models/block.py:80-108).
 */
OW_API int ow_bigemm_fwd(const ow_bigemm_args_t* args, void* stream);

/*
 * Allocation-free variant of ow_bigemm_fwd, for callers that cannot allocate
 * device memory when they run the operator (plugin hosts that pass only input
 * and output buffers, code that must not enter the process's allocator).  It
 * has no counterpart in the reference.  Same arguments as ow_bigemm_fwd except
 * that ``workspace``/``workspace_bytes`` are ignored: scratch comes from a
 * fixed array of ow_noalloc_scratch_limit() bytes (4 MiB) in the library's
 * device memory, which every GPU that loads the library holds until exit.
 * Shapes needing more scratch are rejected with OW_ERR_WORKSPACE.  The first
 * call on a device (with that device current) looks up the array's device
 * address; make it before any stream capture.  All calls share the array, so
 * calls that overlap on the GPU race; no scratch contents need to start at
 * zero.  Allocates nothing (no cudaMalloc/cudaFree).
 */
OW_API int ow_bigemm_fwd_noalloc(const ow_bigemm_args_t* args, void* stream);

/* Scratch bytes available to ow_bigemm_fwd_noalloc (no reference counterpart). */
OW_API size_t ow_noalloc_scratch_limit(void);

/*
 * Backward of ow_bigemm_fwd with the same ``args`` (``out`` is ignored).
 * Replaces the autograd backward the reference takes through
 * ``bigemm_delta_reference`` (and, in block mode, through RMSNorm and the
 * residual add).  Weight gradients are reduced in a fixed order, so results
 * are bitwise reproducible run to run.
 */
OW_API int ow_bigemm_bwd(const ow_bigemm_args_t* args, const ow_bigemm_grads_t* grads, void* stream);

/*
 * Space-to-depth + Linear, the OmniWeave-T stem and downsamples
 * (omniweave/models/backbone.py:14-27 ``space_to_depth_nhwc`` followed by the
 * bias-free ``nn.Linear`` of :121 and :128-132, as called at :176-187), as one
 * tensor-core GEMM that reads the rearranged rows straight from x:
 *
 *   out[b, i, j, n] = sum_{dy, dx, c} s(b, i, j, dy, dx, c) * weight[n, (dy f + dx) C + c]
 *   s = x[b, f i + dy, f j + dx, c]    layout OW_LAYOUT_NHWC (downsample)
 *   s = x[b, c, f i + dy, f j + dx]    layout OW_LAYOUT_NCHW (stem: the image
 *                                      batch before its NHWC permute, :173)
 *
 * ``out`` is NHWC [batch, height/factor, width/factor, out_features] in
 * ``out_dtype`` (bf16 or f16), which is also the dtype the products are
 * taken in (f32 accumulation), as under the reference's autocast.  weight is
 * [out_features, factor^2 channels] row-major (f32 or out_dtype; f32 is
 * rounded).  Supported: NHWC with x_dtype == out_dtype, channels % 64 == 0,
 * width/factor <= 128 and out_features % 256 == 0; NCHW with channels == 3,
 * factor == 4, x f32 or out_dtype and out_features a multiple of 128 up to
 * 512.  x and out 16-byte aligned.  Anything else returns OW_ERR_UNSUPPORTED.
 */
#define OW_LAYOUT_NHWC 0
#define OW_LAYOUT_NCHW 1
typedef struct ow_s2d_linear_t {
  const void* x;
  int32_t x_dtype;
  int32_t layout;          /* OW_LAYOUT_NHWC or OW_LAYOUT_NCHW */
  int32_t batch, height, width, channels, factor;
  const void* weight;
  int32_t w_dtype;
  int32_t out_features;
  void* out;
  int32_t out_dtype;
  void* workspace;         /* ow_s2d_linear_workspace_size() bytes */
  size_t workspace_bytes;
} ow_s2d_linear_t;

/* Workspace bytes ow_s2d_linear_fwd needs (0 if the arguments are unsupported). */
OW_API size_t ow_s2d_linear_workspace_size(const ow_s2d_linear_t* args);
OW_API int ow_s2d_linear_fwd(const ow_s2d_linear_t* args, void* stream);

/*
 * Linear followed by depth-to-space, the input gradient of the downsample
 * above: the autograd of ``Linear(space_to_depth_nhwc(x, f))``
 * (omniweave/models/backbone.py:14-27, :128-132) with respect to x, without
 * the rearranged intermediate:
 *
 *   out[b, f i + dy, f j + dx, c] = sum_n y[b, i, j, n] * weight[n, (dy f + dx) C + c]
 *
 * y is NHWC [batch, height/factor, width/factor, in_features] (bf16 or f16,
 * the compute type: products in it, f32 accumulation); weight
 * [in_features, factor^2 channels] row-major (f32 or y's dtype; the folded
 * anchor weight W_a W_d where there is one); out NHWC
 * [batch, height, width, channels] in out_dtype: y's dtype, or f32 holding
 * the values rounded to y's dtype (as autocast's backward casts the 16-bit
 * input gradient to an f32 input's dtype).
 * Supported: channels and in_features multiples of 64, factor^2 channels a
 * multiple of 256, width/factor <= 128; y and out 16-byte aligned.  Anything
 * else returns OW_ERR_UNSUPPORTED.
 */
typedef struct ow_d2s_linear_t {
  const void* y;
  int32_t y_dtype;
  int32_t batch, height, width, channels, factor;   /* of the output image */
  int32_t in_features;
  const void* weight;
  int32_t w_dtype;
  void* out;
  int32_t out_dtype;
  void* workspace;         /* ow_d2s_linear_workspace_size() bytes */
  size_t workspace_bytes;
} ow_d2s_linear_t;

/* Workspace bytes ow_d2s_linear_fwd needs (0 if the arguments are unsupported). */
OW_API size_t ow_d2s_linear_workspace_size(const ow_d2s_linear_t* args);
OW_API int ow_d2s_linear_fwd(const ow_d2s_linear_t* args, void* stream);

/*
 * Global average pool + classifier head, the backbone's tail
 * (omniweave/models/backbone.py:193-197: ``pooled = stage4.mean(dim=(1, 2))``
 * then ``self.head(pooled)``, an ``nn.Linear`` with bias), as one kernel in
 * which the pooled matrix feeds the tensor-core GEMM from shared memory:
 *
 *   pooled[b, c] = round(sum_t x[b, t, c] / tokens)                 (f32 sum)
 *   out[b, n]    = round(bias[n] + sum_c weight[n, c] pooled[b, c])  (f32 acc)
 *
 * round() is to ``compute_dtype`` (bf16 or f16), which is also the dtype of
 * ``out`` [batch, classes] and of ``pooled`` [batch, channels] (written only
 * when non-NULL; the head's backward needs it), as under the reference's
 * autocast, where the f32 mean, weight and bias are cast before the GEMM.
 * x is [batch, tokens, channels] (the NHWC stage-4 map, f32 or compute_dtype);
 * weight [classes, channels] f32 or compute_dtype; bias [classes] (f32, bf16
 * or f16; rounded to compute_dtype) or NULL.  Supported: channels a multiple
 * of 512 up to 2048 and classes up to 1024; x, weight and pooled 16-byte
 * aligned.  Anything else returns OW_ERR_UNSUPPORTED.  Results are bitwise
 * reproducible (fixed summation order).
 */
typedef struct ow_pool_head_t {
  const void* x;
  int32_t x_dtype;
  int32_t batch, tokens, channels;
  const void* weight;
  int32_t w_dtype;
  const void* bias;
  int32_t bias_dtype;
  int32_t classes;
  int32_t compute_dtype;
  void* out;
  void* pooled;
  void* workspace;         /* ow_pool_head_workspace_size() bytes */
  size_t workspace_bytes;
} ow_pool_head_t;

/* Workspace bytes ow_pool_head_fwd needs (0 if the arguments are
 * unsupported): 256, plus room for the converted weight when weight is f32. */
OW_API size_t ow_pool_head_workspace_size(const ow_pool_head_t* args);
OW_API int ow_pool_head_fwd(const ow_pool_head_t* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* OMNIWAVE_B200_H */
