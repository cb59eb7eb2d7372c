/*
 * ssm_b200.h — C ABI of the B200 (sm_100a) selective-scan library (libssm_b200.so).
 *
 * The library replaces the GPU path of the reference's selective scan:
 *   kernels/triton_scan.py  (TritonSelectiveScanFn / selective_scan_triton, lines 275-329)
 * and the inline single-token decode step of
 *   models/mamba.py:113-118,123  (h = a*h0 + b; y = <h, C>; state.ssm.copy_(h)).
 *
 * Conventions shared by every entry point
 *   - All pointers are CUDA device pointers; nothing here touches host memory or
 *     allocates device memory. Every call only enqueues kernels on `stream`
 *     (a cudaStream_t passed as void*, NULL = legacy default stream) and returns.
 *   - Shapes: B = batch, L = sequence length, D = channels (d_inner), N = d_state.
 *     N must be one of 4, 8, 16, 32, 64 (a power of two, like the reference's
 *     Triton path, kernels/triton_scan.py:326-328).
 *   - Activations (B, L, D) and the selective projections B, C (B, L, N) are given
 *     as ssm_view: a base pointer, an element dtype and two element strides
 *     (batch, row). The innermost (channel / state) stride is always 1, so a
 *     channel shard or the x half of in_proj's output can be passed as a view.
 *   - A (D, N), Dskip (D), h0 / last / dlast / dh0 (B, D, N) and chunk_states
 *     (B, ceil(L/16), D, N) are dense row-major float32.
 *   - Within one call all ssm_view tensors must share one dtype (SSM_F32 or
 *     SSM_BF16); the Python layer upcasts mixed inputs to float32 exactly as
 *     models/scan.py:288-291 does. State, A, Dskip and all accumulation are float32.
 *   - method: SSM_ZOH (default of the reference), SSM_EULER, SSM_BILINEAR
 *     (models/scan.py:39-55).
 *   - Return value: SSM_OK or an SSM_ERR_* code; ssm_last_error_message() gives
 *     a one-line description of the most recent failure on the calling thread.
 */
#ifndef SSM_B200_H_
#define SSM_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SSM_B200_ABI_VERSION 5

#if defined(__GNUC__)
#define SSM_API __attribute__((visibility("default")))
#else
#define SSM_API
#endif

typedef enum {
  SSM_OK = 0,
  SSM_ERR_INVALID = 1,     /* bad shape, method, N or NULL required pointer  */
  SSM_ERR_DTYPE = 2,       /* unsupported or mixed dtypes                    */
  SSM_ERR_WORKSPACE = 3,   /* workspace missing or smaller than required     */
  SSM_ERR_CUDA = 4,        /* a CUDA launch or driver call failed            */
  SSM_ERR_UNSUPPORTED = 5  /* valid request this build does not implement    */
} ssm_status;

typedef enum { SSM_F32 = 0, SSM_BF16 = 1 } ssm_dtype;
typedef enum { SSM_ZOH = 0, SSM_EULER = 1, SSM_BILINEAR = 2 } ssm_method;

/* A strided (B, rows, cols) tensor with unit stride along cols. ptr == NULL means
 * "absent" for optional operands. Strides are in elements, not bytes. */
typedef struct {
  const void* ptr;
  int32_t dtype;          /* ssm_dtype */
  int32_t reserved;
  int64_t batch_stride;
  int64_t row_stride;
} ssm_view;

/* ---------------------------------------------------------------------------------
 * Forward scan.  Replaces TritonSelectiveScanFn.forward + _launch_fwd + _fwd_kernel
 * (kernels/triton_scan.py:27-74, 253-286) and SelectiveScanFn.forward
 * (models/scan.py:202-217).
 *
 *   h_t = a_t * h_{t-1} + b_t   (per b, d, n; a, b from discretize, models/scan.py:39-55)
 *   y_t = sum_n C_t[n] h_t[n]
 *   out_t = (y_t + Dskip * u_t) * silu(z_t)       when Dskip / z are given
 *           (the Mamba mixer's D-skip and gate, models/mamba.py:124)
 *
 * u, delta, z: (B, L, D); Bm, Cm: (B, L, N); A: (D, N); Dskip: (D) or NULL;
 * z.ptr may be NULL; h0: (B, D, N) or NULL (zeros).
 * out y: (B, L, D) view, same dtype as u (models/scan.py:299 returns y.to(x.dtype)).
 * out ygate: (B, L, D) view or NULL: the gate's input y + Dskip*u before the SiLU(z)
 *   product.  A training caller passes it when z is given; ssm_scan_bwd needs it to form dz
 *   without recomputing y (it is the one activation the backward cannot rebuild cheaply).
 * out last: (B, D, N) float32 or NULL (the reference's h_last).
 * out chunk_states: (B, ceil(L/16), D, N) float32 or NULL. When given, the state
 *   entering every 16-step chunk is saved for ssm_scan_bwd (the backward then
 *   recomputes states from these checkpoints instead of the reference's full
 *   (B, L, D_tile, N) hbuf, kernels/triton_scan.py:305-309).
 * workspace: device scratch of at least ssm_scan_fwd_workspace_size() bytes
 *   (needed only when the sequence is split across thread blocks; may be NULL
 *   when that size is 0).
 * ------------------------------------------------------------------------------- */
SSM_API int ssm_scan_fwd_workspace_size(int64_t B, int64_t L, int64_t D, int64_t N, size_t* bytes);

SSM_API int ssm_scan_fwd(int64_t B, int64_t L, int64_t D, int64_t N, int32_t method,
                 ssm_view u, ssm_view delta, const float* A, ssm_view Bm, ssm_view Cm,
                 const float* Dskip, ssm_view z, const float* h0,
                 ssm_view y, ssm_view ygate, float* last, float* chunk_states,
                 void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------
 * Backward scan.  Replaces TritonSelectiveScanFn.backward + _bwd_kernel
 * (kernels/triton_scan.py:143-226, 288-319) and SelectiveScanFn.backward
 * (models/scan.py:219-255).
 *
 * Inputs as in ssm_scan_fwd, plus chunk_states and ygate written by the forward call on
 * the same inputs (ygate required iff z.ptr != NULL), dy (B, L, D) = gradient of the
 * forward output, dlast (B, D, N) or NULL (zeros; kernels/triton_scan.py:294).
 * Outputs (all required unless noted):
 *   du, ddelta: (B, L, D) views, dtype of u;  dBm, dCm: (B, L, N) views, dtype of u;
 *   dA: (D, N) float32 (summed over batch, kernels/triton_scan.py:319);
 *   dDskip: (D) float32, required iff Dskip != NULL;
 *   dz: (B, L, D) view, required iff z.ptr != NULL;
 *   dh0: (B, D, N) float32, required iff h0 != NULL.
 * dB and dC are reduced over channels in a fixed order: the result is bitwise
 * reproducible run to run (the reference needs torch.use_deterministic_algorithms
 * for that, kernels/triton_scan.py:298-302).
 * workspace: at least ssm_scan_bwd_workspace_size() bytes.
 * A long sequence over few (batch, 32-channel) tiles is split into segments that run at the
 * same time (ssm_scan_bwd_plan); the workspace size covers the split.
 * ------------------------------------------------------------------------------- */
SSM_API int ssm_scan_bwd_workspace_size(int64_t B, int64_t L, int64_t D, int64_t N, size_t* bytes);

/* Composition of W shard summaries in shard order, float32: shard r's (B, D, N) block of decay and
 * of end starts r * shard_stride elements after decay / end (0: B*D*N, packed; both arrays may be
 * interleaved blocks of one all-gathered buffer); out is (W, B, D, N) packed.
 *   out[r] = carry;  carry = decay[r] * carry + end[r]   (r = 0..W-1; reverse != 0: r = W-1..0)
 * from carry = start (B, D, N) or zeros; last (B, D, N, or NULL) gets the final carry.  Forward:
 * decay/end = the shards' ssm_scan_fwd_summary outputs, out = the state entering every shard,
 * last = the sequence's final state.  Backward (reverse): decay/end = the ssm_scan_bwd_summary
 * outputs, start = dlast, out = the adjoint entering every shard, last = dh0.  Replaces the chunk-end
 * combine of models/scan.py:160-164 across GPUs (the reference runs on one GPU). */
SSM_API int ssm_compose_shards(int32_t W, int64_t B, int64_t D, int64_t N, const float* decay, const float* end,
                               int64_t shard_stride, const float* start, int32_t reverse, float* out, float* last,
                               void* stream);

/* The backward's sequence split for a shape on the current device: *nseg segments of *seg_len
 * steps (a multiple of 16; *nseg = 1: no split).  The reference's backward runs one program per
 * (batch, channel block) over the whole sequence (kernels/triton_scan.py:288-319); this query has
 * no reference counterpart.  dtype: SSM_F32 or SSM_BF16. */
SSM_API int ssm_scan_bwd_plan(int64_t B, int64_t L, int64_t D, int64_t N, int32_t dtype, int32_t* nseg,
                              int32_t* seg_len);

SSM_API int ssm_scan_bwd(int64_t B, int64_t L, int64_t D, int64_t N, int32_t method,
                 ssm_view u, ssm_view delta, const float* A, ssm_view Bm, ssm_view Cm,
                 const float* Dskip, ssm_view z, const float* h0,
                 const float* chunk_states, ssm_view ygate, ssm_view dy, const float* dlast,
                 ssm_view du, ssm_view ddelta, float* dA, ssm_view dBm, ssm_view dCm,
                 float* dDskip, ssm_view dz, float* dh0,
                 void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------
 * Backward scan without a caller workspace.  No counterpart in the reference: it exists
 * for callers that cannot allocate device memory when they run the backward — a process
 * whose memory pool is fixed after start-up and forbids cudaMalloc on the hot path, or a
 * plugin whose host application owns all device memory and gives it no allocator.
 *
 * Same arguments and results as ssm_scan_bwd, minus the workspace: the scratch lives in a
 * fixed device array inside the library, SSM_NOALLOC_SCRATCH_BYTES (32 MiB) per GPU that
 * loads the library, held until the process exits.  Shapes whose backward needs more
 * scratch than that (ssm_scan_bwd_workspace_size) are rejected with SSM_ERR_WORKSPACE and
 * a message naming both sizes.  The call allocates nothing.
 *   - Every call looks up the array's device address on the current device
 *     (cudaGetSymbolAddress); the first call on a device may load the library's module
 *     there, so make that first call before any stream capture.
 *   - Every call shares the one array and leaves its contents behind (the backward
 *     overwrites everything it reads, so nothing needs clearing).  Calls that overlap on
 *     the GPU — concurrent streams, or several host threads — race on it: serialise them.
 * ------------------------------------------------------------------------------- */
#define SSM_NOALLOC_SCRATCH_BYTES (32u << 20)

SSM_API int ssm_scan_bwd_noalloc(int64_t B, int64_t L, int64_t D, int64_t N, int32_t method,
                         ssm_view u, ssm_view delta, const float* A, ssm_view Bm, ssm_view Cm,
                         const float* Dskip, ssm_view z, const float* h0,
                         const float* chunk_states, ssm_view ygate, ssm_view dy, const float* dlast,
                         ssm_view du, ssm_view ddelta, float* dA, ssm_view dBm, ssm_view dCm,
                         float* dDskip, ssm_view dz, float* dh0, void* stream);

/* ---------------------------------------------------------------------------------
 * Sequence-parallel forward in two phases (one sequence split over ranks or streams).
 * Phase 1 scans this shard from a zero state and returns its affine summary:
 *   decay (B, D, N) = prod_t a_t over the shard,  hend (B, D, N) = shard's end state
 *   from zero.  Composition of shard summaries is the chunk combine of the
 *   reference's two-level scan (models/scan.py:142-165, step (2)).
 * Phase 2 runs the shard again from the carried-in state h_in (B, D, N) and writes
 * y / ygate / last / chunk_states exactly like ssm_scan_fwd with h0 = h_in.
 * Both phases take the same workspace (ssm_scan_fwd_workspace_size bytes); phase 2
 * reuses the per-block summaries phase 1 left there, so the two calls must use the
 * same workspace and inputs, in order, on the same stream.
 * ------------------------------------------------------------------------------- */
SSM_API int ssm_scan_fwd_summary(int64_t B, int64_t L, int64_t D, int64_t N, int32_t method,
                         ssm_view u, ssm_view delta, const float* A, ssm_view Bm,
                         float* decay, float* hend,
                         void* workspace, size_t workspace_bytes, void* stream);

SSM_API int ssm_scan_fwd_finish(int64_t B, int64_t L, int64_t D, int64_t N, int32_t method,
                        ssm_view u, ssm_view delta, const float* A, ssm_view Bm, ssm_view Cm,
                        const float* Dskip, ssm_view z, const float* h_in,
                        ssm_view y, ssm_view ygate, float* last, float* chunk_states,
                        void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------
 * Sequence-parallel backward, phase 1: the adjoint summary of this shard.  The
 * backward of a sequence split over shards needs, on every shard, the adjoint dlast
 * entering it from the right; that is the gradient with respect to the next shard's
 * initial state, which is affine in the next shard's own dlast:
 *   dstart(dlast) = dstart(0) + decay * dlast      (elementwise over (B, D, N))
 * This call returns dstart(0) -- the reverse adjoint dh_{t-1} = a_t (dh_t + C_t dys_t),
 * dys = dy * silu(z) (dy when z is NULL), run over the shard from a zero adjoint at its
 * end -- and decay = prod_t a_t over the shard.  Composing the shards' summaries from
 * the last shard to the first gives each shard's dlast; ssm_scan_bwd with that dlast
 * and h0 = the shard's carried-in state finishes the shard.  The reverse adjoint is
 * models/scan.py:239-240 (kernels/triton_scan.py:187, 223); the split across shards is
 * the reverse counterpart of the two-level scan's chunk combine (models/scan.py:160-164).
 * delta, z, dy: (B, L, D); Cm: (B, L, N); A: (D, N) fp32; decay, dstart: (B, D, N) fp32
 * outputs.  Workspace: ssm_scan_fwd_workspace_size bytes.
 * ------------------------------------------------------------------------------- */
SSM_API int ssm_scan_bwd_summary(int64_t B, int64_t L, int64_t D, int64_t N, int32_t method,
                         ssm_view delta, const float* A, ssm_view Cm, ssm_view z, ssm_view dy,
                         float* decay, float* dstart,
                         void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------
 * Single-token state update (decode).  The reference has no function for this; its
 * definition is the inline branch of Mamba.forward for L == 1 with a state
 * (models/mamba.py:113-118, 123-124), driven by LM.generate (models/lm.py:130-146).
 *
 *   a = exp(delta*A) etc. (same discretisation as the scan);  state <- a*state + b
 *   y = (sum_n C[n] state[n] + Dskip*x) * silu(z)
 *
 * state: (B, D, N) float32, updated in place.  x, delta, z: (B, D) given as ssm_view
 * with rows = 1 (row_stride ignored); Bm, Cm: (B, N) likewise; z.ptr may be NULL.
 * out y: (B, D) view in x's dtype.  Capturable in a CUDA graph (no allocation,
 * no synchronisation).
 * ------------------------------------------------------------------------------- */
SSM_API int ssm_state_update(int64_t B, int64_t D, int64_t N, int32_t method,
                     float* state, ssm_view x, ssm_view delta, const float* A,
                     ssm_view Bm, ssm_view Cm, const float* Dskip, ssm_view z,
                     ssm_view y, void* stream);

/* ---------------------------------------------------------------------------------
 * Step-size activation inside the scan.  The mixer computes
 *   delta = softplus(dt_proj(dt)) = softplus(dt @ W^T + bias)       (models/mamba.py:77)
 * With opts->softplus != 0 the _ex entry points take the raw dt @ W^T as `delta` and
 * apply softplus(delta + bias) in registers (torch's threshold: x > 20 gives x); the
 * backward then writes ddelta as the gradient w.r.t. that raw input and, when
 * opts->dbias is given, d loss / d bias (D) fp32, summed in a fixed order.  bias (D)
 * fp32 may be NULL (zero).  opts == NULL or softplus == 0: plain ssm_scan_fwd/_bwd.
 * ------------------------------------------------------------------------------- */
typedef struct ssm_delta_opts {
  const float* bias;
  int32_t softplus;
  int32_t reserved;
  float* dbias;
} ssm_delta_opts;

SSM_API int ssm_scan_fwd_ex(int64_t B, int64_t L, int64_t D, int64_t N, int32_t method,
                    ssm_view u, ssm_view delta, const float* A, ssm_view Bm, ssm_view Cm,
                    const float* Dskip, ssm_view z, const float* h0,
                    ssm_view y, ssm_view ygate, float* last, float* chunk_states,
                    const ssm_delta_opts* opts,
                    void* workspace, size_t workspace_bytes, void* stream);
SSM_API int ssm_scan_bwd_ex(int64_t B, int64_t L, int64_t D, int64_t N, int32_t method,
                    ssm_view u, ssm_view delta, const float* A, ssm_view Bm, ssm_view Cm,
                    const float* Dskip, ssm_view z, const float* h0,
                    const float* chunk_states, ssm_view ygate, ssm_view dy, const float* dlast,
                    ssm_view du, ssm_view ddelta, float* dA, ssm_view dBm, ssm_view dCm,
                    float* dDskip, ssm_view dz, float* dh0,
                    const ssm_delta_opts* opts,
                    void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------
 * The three core entry points under the names the reference's Python API uses for
 * this path (selective_scan_triton's forward/backward, kernels/triton_scan.py:322;
 * the decode step of models/mamba.py:113-118 as selective_state_update), for FFI
 * users who bind by those names.  Same signatures and behaviour as ssm_scan_fwd,
 * ssm_scan_bwd and ssm_state_update.
 * ------------------------------------------------------------------------------- */
SSM_API int selective_scan_fwd(int64_t B, int64_t L, int64_t D, int64_t N, int32_t method,
                       ssm_view u, ssm_view delta, const float* A, ssm_view Bm, ssm_view Cm,
                       const float* Dskip, ssm_view z, const float* h0,
                       ssm_view y, ssm_view ygate, float* last, float* chunk_states,
                       void* workspace, size_t workspace_bytes, void* stream);
SSM_API int selective_scan_bwd(int64_t B, int64_t L, int64_t D, int64_t N, int32_t method,
                       ssm_view u, ssm_view delta, const float* A, ssm_view Bm, ssm_view Cm,
                       const float* Dskip, ssm_view z, const float* h0,
                       const float* chunk_states, ssm_view ygate, ssm_view dy, const float* dlast,
                       ssm_view du, ssm_view ddelta, float* dA, ssm_view dBm, ssm_view dCm,
                       float* dDskip, ssm_view dz, float* dh0,
                       void* workspace, size_t workspace_bytes, void* stream);
SSM_API int selective_state_update(int64_t B, int64_t D, int64_t N, int32_t method,
                           float* state, ssm_view x, ssm_view delta, const float* A,
                           ssm_view Bm, ssm_view Cm, const float* Dskip, ssm_view z,
                           ssm_view y, void* stream);

/* ---------------------------------------------------------------------------------
 * Diagnostics.
 * ------------------------------------------------------------------------------- */
/* ---------------------------------------------------------------------------------
 * Causal depthwise conv1d (+ SiLU): the step in front of the scan in the Mamba mixer,
 * models/mamba.py:100-107 (x transposed to (B, D, L), left-padded with K - 1 zeros or
 * prefixed with the decode state, nn.Conv1d(D, D, K, groups=D), SiLU, transposed back).
 * Computed in the (B, L, D) layout directly:
 *   out[b, t, d] = act(bias[d] + sum_k weight[d, k] x[b, t - (K - 1) + k, d])
 * with x[b, t < 0, d] = conv_state[b, d, K - 1 + t] (zeros when conv_state is NULL) and
 * act = SiLU when silu != 0 (identity otherwise).  x, out: (B, L, D) views in fp32 or bf16
 * (x may be strided, e.g. half of in_proj's output); weight (D, K) and bias (D) fp32;
 * K in 1..4.  conv_state / new_conv_state: (B, D, K - 1) in x's dtype, optional;
 * new_conv_state receives the last K - 1 inputs of cat(conv_state, x) (the decode state
 * update of models/mamba.py:104-105); it may alias conv_state only when the sequence
 * is one time tile (always for L <= 4, e.g. a decode step; otherwise SSM_ERR_INVALID).
 * ------------------------------------------------------------------------------- */
SSM_API int ssm_conv1d_fwd(int64_t B, int64_t L, int64_t D, int64_t K, ssm_view x,
                   const float* weight, const float* bias, const void* conv_state, int32_t silu,
                   ssm_view out, void* new_conv_state, void* stream);

/* Backward of ssm_conv1d_fwd without a state (training): dx (B, L, D) in x's dtype,
 * dweight (D, K) and dbias (D, may be NULL) fp32, summed in a fixed order (deterministic).
 * Workspace: ssm_conv1d_bwd_workspace_size bytes. */
SSM_API int ssm_conv1d_bwd_workspace_size(int64_t B, int64_t L, int64_t D, int64_t K, size_t* bytes);
SSM_API int ssm_conv1d_bwd(int64_t B, int64_t L, int64_t D, int64_t K, ssm_view x,
                   const float* weight, const float* bias, int32_t silu, ssm_view dout,
                   ssm_view dx, float* dweight, float* dbias,
                   void* workspace, size_t workspace_bytes, void* stream);

/* ABI version of the loaded library (SSM_B200_ABI_VERSION). */
SSM_API int ssm_abi_version(void);
/* Message for the most recent non-OK status returned on this thread. */
SSM_API const char* ssm_last_error_message(void);
/* Reads and clears the device-side error word of the current device: nonzero when a
 * kernel gave up on a bounded wait (a TMA copy that never landed).  Synchronises
 * the device; intended for tests and debugging, not for the hot path. */
SSM_API int ssm_read_device_error(int32_t* flags);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* SSM_B200_H_ */
