/*
 * dora_b200.h -- C ABI of the B200-native DoRA hot path.
 *
 * One shared library, libdora_b200.so, built for sm_100a.  Every entry point
 * takes plain device pointers, sizes, dtype codes and a CUDA stream handle
 * (a cudaStream_t passed as void*; NULL is the legacy default stream), queues
 * its kernels on that stream and returns a dora_status_t without waiting for
 * them.  No entry point allocates device memory: scratch space is passed in
 * by the caller, sized by the matching *_workspace_size query.
 *
 * The dora_peer_buffer_* functions are the exception: they allocate and map
 * the peer-writable output buffers of the row-sharded layer.
 *
 * Each entry point names the reference interface it replaces, as
 * file:line inside sockeye44/dorafactors, where "dora.py" and "dora_fused.py"
 * are code/peft_patched/src/peft/tuners/lora/{dora,dora_fused}.py.
 *
 * Layout conventions.  Activations are row-major [rows x cols] (cols = the
 * layer's out_features, rows = every leading dim flattened), contiguous.  The
 * per-column scale g ("mag_norm_scale") is a contiguous vector of cols
 * elements.  Weights are row-major and contiguous: W0 [out x in], A [r x in],
 * B [out x r].
 */
#ifndef DORA_B200_H_
#define DORA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types.  Values are part of the ABI. */
typedef enum {
  DORA_DTYPE_F32 = 0,
  DORA_DTYPE_F16 = 1,
  DORA_DTYPE_BF16 = 2
} dora_dtype_t;

/* Status codes.  Values are part of the ABI. */
typedef enum {
  DORA_OK = 0,
  DORA_ERR_INVALID_ARGUMENT = 1, /* bad size, dtype, null pointer or alias */
  DORA_ERR_UNSUPPORTED = 2,      /* valid request this library cannot serve */
  DORA_ERR_WORKSPACE = 3,        /* workspace missing or too small */
  DORA_ERR_CUDA = 4,             /* a CUDA runtime/driver call failed */
  DORA_ERR_DEVICE_TIMEOUT = 5    /* a bounded device-side wait gave up */
} dora_status_t;

/* Library version as 10000*major + 100*minor + patch. */
int dora_version(void);

/* Human-readable text of a status code (static storage). */
const char* dora_status_string(int status);

/* Text of the last CUDA error seen by this thread inside the library. */
const char* dora_last_cuda_error(void);

/* Number of kernels this library has launched in this process (all devices). */
unsigned long long dora_launch_count(void);

/*
 * Device-side error word of the current device: 0 when no kernel has
 * recorded a failure, else a DORA_ERR_* code set by a kernel whose bounded
 * wait expired.  Synchronises the current device.  With reset != 0 the word
 * is cleared after reading.  Returns DORA_ERR_CUDA if the read itself fails
 * (*out untouched).
 */
int dora_device_error(int reset, int* out);

/*
 * Self-test of the bounded device-side waits (no counterpart in the reference,
 * whose Triton kernels have no cross-warp waits): launches one thread that
 * waits, with a limit of `limit_cycles` SM cycles (1 .. about 2^31), on an
 * mbarrier phase that never completes.  It must give up, set
 * DORA_ERR_DEVICE_TIMEOUT in the device error word (read it with
 * dora_device_error) and return; *gave_up is 1 then.  Synchronises `stream`.
 */
int dora_selftest_bounded_wait(long long limit_cycles, int* gave_up, void* stream);

/*
 * Fused compose forward.
 *   out[i,j]   = (g[j] - 1) * base[i,j] + g[j] * (scale * lora[i,j])
 *   inner[i,j] = scale * lora[i,j] + base[i,j]            (only if inner != NULL)
 * Arithmetic in fp32, one rounding into act_dtype per output.  out may alias
 * lora (in-place compose); inner must not alias any input.  g_dtype is
 * act_dtype or DORA_DTYPE_F32 (fp32 magnitude with half activations).
 * rows * cols == 0 is a no-op.
 *
 * Replaces fused_dora_compose (dora_fused.py:539-671, kernels 367-459) and
 * fused_dora_forward_and_inner (dora_fused.py:674-772, kernel 461-514).
 */
int dora_compose_fwd(const void* lora, const void* base, const void* g, int g_dtype, double scale,
                     void* out, void* inner, int64_t rows, int64_t cols, int act_dtype, void* stream);

/*
 * Bytes of workspace dora_compose_bwd needs to produce d_g for this shape on
 * the current device (0 for an empty tensor).  The workspace must be 256-byte
 * aligned.  It starts with a region of completion counters that must be zero
 * before the first call; every successful call leaves them zero again, so a
 * zero-filled workspace may be reused by later calls on the same stream
 * without clearing.  Calls that overlap on the GPU need separate workspaces.
 */
size_t dora_compose_bwd_workspace_size(int64_t rows, int64_t cols, int act_dtype);

/*
 * Fused compose backward, one pass over d_out (and inner):
 *   d_lora[i,j] = (g[j] * scale) * d_out[i,j]             (if d_lora != NULL)
 *   d_base[i,j] = (g[j] - 1) * d_out[i,j]                 (if d_base != NULL)
 *   d_g[j]      = sum_i inner[i,j] * d_out[i,j]           (if d_g != NULL)
 * d_lora / d_base are in act_dtype, d_g in g_dtype.  The column sum runs in
 * fp32 in a fixed order (per-thread, then CTA tree, then per-CTA partials
 * folded by the last CTA of each column tile), so results are deterministic.
 * inner is required iff d_g != NULL and rows * cols > 0.  With rows == 0 the
 * activation pointers may be NULL and d_g (if given) is set to zero.
 *
 * Replaces FusedDoRAComposeFunction.backward / _fused_backward_triton
 * (dora_fused.py:1137-1206, 1264-1344, kernel 1010-1062), including the
 * PyTorch d_mag reduction of dora_fused.py:1330-1342.
 */
int dora_compose_bwd(const void* d_out, const void* inner, const void* g, int g_dtype, double scale,
                     void* d_lora, void* d_base, void* d_g, void* workspace, size_t workspace_bytes,
                     int64_t rows, int64_t cols, int act_dtype, void* stream);

/*
 * Compose forward with the base output added in the same pass (the layer
 * output the PEFT variant forms as result + delta):
 *   base[i,j]  = result[i,j] - bias[j]                  (bias may be NULL)
 *   y[i,j]     = result[i,j] + ((g[j] - 1) * base[i,j] + g[j] * (scale * lora[i,j]))
 *   inner[i,j] = scale * lora[i,j] + base[i,j]           (only if inner != NULL)
 * fp32 arithmetic in that op order, one rounding per output (fp32 results equal
 * the reference's result + delta bit for bit).  bias has act_dtype.  y may not
 * alias result; y may alias lora only when inner is NULL.
 *
 * Replaces the compose of DoraLinearLayer.forward (dora.py:1443-1468) plus the
 * result + delta / result.add_(delta) glue of DoraLinearVariant.forward
 * (variants.py:244-283), one activation pass instead of three.
 */
int dora_linear_output_fwd(const void* lora, const void* result, const void* bias, const void* g, int g_dtype,
                           double scale, void* y, void* inner, int64_t rows, int64_t cols, int act_dtype,
                           void* stream);

/*
 * Backward of dora_linear_output_fwd, one pass over d_y (and inner):
 *   d_lora[i,j]   = (g[j] * scale) * d_y[i,j]
 *   d_result[i,j] = g[j] * d_y[i,j]      (both paths from y to result: 1 + (g - 1))
 *   d_g[j]        = sum_i inner[i,j] * d_y[i,j]
 * Same workspace rules as dora_compose_bwd (dora_compose_bwd_workspace_size).
 *
 * Replaces FusedDoRAComposeFunction.backward (dora_fused.py:1137-1206) plus
 * autograd's accumulation of d_y and d_base into the base output's gradient.
 */
int dora_linear_output_bwd(const void* d_y, const void* inner, const void* g, int g_dtype, double scale,
                           void* d_lora, void* d_result, void* d_g, void* workspace, size_t workspace_bytes,
                           int64_t rows, int64_t cols, int act_dtype, void* stream);

/*
 * Gradient of dora_linear_output_fwd's bias (the bias enters y only through
 * base = result - bias):
 *   d_bias[j] = (1 - g[j]) * sum_i d_y[i,j]
 * fp32 column sums in a fixed order (deterministic), one rounding into
 * act_dtype; no workspace.  rows == 0 sets d_bias to zero.
 *
 * Replaces the autograd of `base_result - bias` in DoraLinearLayer.forward
 * (dora.py:1443-1459), which sums the d_base tensor over the rows.
 */
int dora_linear_output_bias_grad(const void* d_y, const void* g, int g_dtype, void* d_bias, int64_t rows,
                                 int64_t cols, int act_dtype, void* stream);

/*
 * dora_linear_output_bwd with d_y read as a column slice of a wider gradient:
 * row i of d_y starts ld_dy elements after row i-1 (ld_dy >= cols); inner,
 * d_lora, d_result stay dense [rows x cols].  Same results and workspace rules
 * as dora_linear_output_bwd.
 *
 * Replaces, for out-feature row sharding, the slice copy of the gathered
 * output's gradient before the shard's backward; the reference has no tensor
 * parallelism, so the arithmetic replaced is that of dora_linear_output_bwd
 * (FusedDoRAComposeFunction.backward, dora_fused.py:1137-1206).
 */
int dora_linear_output_bwd_strided(const void* d_y, int64_t ld_dy, const void* inner, const void* g, int g_dtype,
                                   double scale, void* d_lora, void* d_result, void* d_g, void* workspace,
                                   size_t workspace_bytes, int64_t rows, int64_t cols, int act_dtype, void* stream);

/*
 * Row-sharded layer output with the output all-gather fused in.  This rank
 * owns output columns [col_offset, col_offset + cols) of a layer whose full
 * output y is [rows x ld] on every one of n_ranks ranks (1 .. 8).  It computes
 * its columns of y = result + delta exactly as dora_linear_output_fwd (lora,
 * result, inner and g are this rank's [rows x cols] / [cols] arrays) and
 * stores each value into all n_ranks output buffers at its final position:
 *   y_ranks[p][i * ld + col_offset + j] = y[i, j]     for every p.
 * y_ranks is a host array of n_ranks device pointers valid in this process:
 * y_ranks[rank] is this rank's own buffer, the others are peers' buffers
 * mapped into this process (dora_peer_buffer_open, over NVLink).  No
 * collective library call is made.  Ordering is the caller's: every rank must
 * have finished reading the buffers before any rank calls this, and no rank
 * may read them until every rank's call has completed (a cross-rank barrier
 * on the stream before and after).
 *
 * Replaces, for out-feature row sharding of the adapted linear, the layer
 * output compose (dora.py:1443-1468 with the result + delta of
 * variants.py:244-283) followed by an NCCL all-gather of the shards and the
 * permute that puts them in column order.  The reference has no tensor
 * parallelism; the split rests on the row independence of its factored norm
 * (dora.py:1024-1153) and of the compose (one g per output column).
 */
int dora_linear_output_fwd_allgather(const void* lora, const void* result, const void* bias, const void* g,
                                     int g_dtype, double scale, void* const* y_ranks, int n_ranks, int rank,
                                     int64_t col_offset, int64_t ld, void* inner, int64_t rows, int64_t cols,
                                     int act_dtype, void* stream);

/*
 * Peer-writable output buffers for dora_linear_output_fwd_allgather (plain
 * CUDA IPC, no multicast).  These have no counterpart in the reference, which
 * has no tensor parallelism.
 *
 * dora_peer_buffer_alloc: cudaMalloc `bytes` on the current device and export
 *   its IPC handle (DORA_PEER_HANDLE_BYTES bytes written to `handle`).
 * dora_peer_buffer_open: map another process's exported buffer into this one
 *   (peer access enabled on demand); *ptr is valid for kernels on the
 *   current device.
 * dora_peer_buffer_close: unmap a buffer opened with dora_peer_buffer_open.
 * dora_peer_buffer_free: free a buffer from dora_peer_buffer_alloc; every
 *   process that opened it must have closed it first.
 */
#define DORA_PEER_HANDLE_BYTES 64
int dora_peer_buffer_alloc(size_t bytes, void** ptr, unsigned char* handle);
int dora_peer_buffer_open(const unsigned char* handle, void** ptr);
int dora_peer_buffer_close(void* ptr);
int dora_peer_buffer_free(void* ptr);

/*
 * Compose forward for convolution outputs: activations [batch, channels,
 * spatial] contiguous (spatial = the product of the spatial dims), g[channels]
 * broadcast along the channel dimension.  out = (g-1)*base + g*(scale*lora)
 * and, if inner is non-NULL, inner = scale*lora + base, per element exactly as
 * dora_compose_fwd.  Out of place (out may not alias lora or base).
 * Replaces the compose of _DoraConvNdLayer.forward
 * (code/peft_patched/src/peft/tuners/lora/dora.py:1670-1715), which the
 * reference evaluates on its eager path (g is not on the last dimension,
 * dora_fused.py:563-574; eager formula dora.py:1331-1334).
 */
int dora_compose_fwd_channels(const void* lora, const void* base, const void* g, int g_dtype, double scale,
                              void* out, void* inner, int64_t batch, int64_t channels, int64_t spatial,
                              int act_dtype, void* stream);

/* Workspace bytes of dora_compose_bwd_channels (per channel: a completion
 * counter and one fp32 partial per batch split); zero it once before first use. */
size_t dora_compose_bwd_channels_workspace_size(int64_t batch, int64_t channels, int64_t spatial, int act_dtype);

/*
 * Compose backward for convolution outputs (layout as above): d_lora =
 * (g*scale)*d_out, d_base = (g-1)*d_out, d_g[c] = sum over batch and spatial
 * of inner*d_out (deterministic), any subset.  Replaces the eager autograd of
 * the conv compose (dora.py:1331-1334 under autograd).
 */
int dora_compose_bwd_channels(const void* d_out, const void* inner, const void* g, int g_dtype, double scale,
                              void* d_lora, void* d_base, void* d_g, void* workspace, size_t workspace_bytes,
                              int64_t batch, int64_t channels, int64_t spatial, int act_dtype, void* stream);

/*
 * Size of the fixed device scratch array behind dora_compose_bwd_noalloc:
 * 4 MiB, held once on every GPU that loads the library.
 */
#define DORA_NOALLOC_SCRATCH_BYTES (4u << 20)

/*
 * dora_compose_bwd without a caller workspace.  This entry point has no
 * counterpart in the reference.
 *
 * It is for callers that cannot allocate device memory for the column-sum
 * scratch: a C or FFI host that embeds this library with no device allocator
 * of its own, or code that must not call cudaMalloc here because cudaMalloc
 * synchronizes the device.  Same arguments and results as dora_compose_bwd,
 * minus the workspace; no cudaMalloc, cudaFree or other allocating call is
 * made.  The scratch is a fixed DORA_NOALLOC_SCRATCH_BYTES array inside the
 * library's device image.  The backward's grid is the one dora_compose_bwd
 * uses when its dora_compose_bwd_workspace_size() fits the array, else a
 * shallower one (fewer column partials; d_g then differs from
 * dora_compose_bwd's in fp32 summation order only); a shape whose partials fit
 * neither is rejected with DORA_ERR_WORKSPACE before anything is queued.  The
 * sizes depend on the current device's SM count (the backward's grid), so the
 * largest accepted shape does too.  Argument errors are reported before the
 * array is touched.
 *
 * The first call on each device looks up the array's device address (with
 * that device current) and caches it; make that first call before any stream
 * capture.  Every call shares the one array per device and it keeps the last
 * call's contents: each call clears its completion counters on the given
 * stream first.  Calls that overlap on the GPU (different streams, or
 * different host threads without ordering) race on the array and give wrong
 * d_g; order them on one stream or use dora_compose_bwd with separate
 * workspaces instead.  The cached address does not survive cudaDeviceReset:
 * do not call this entry point on a device after resetting it.
 */
int dora_compose_bwd_noalloc(const void* d_out, const void* inner, const void* g, int g_dtype, double scale,
                             void* d_lora, void* d_base, void* d_g, int64_t rows, int64_t cols, int act_dtype,
                             void* stream);

/*
 * Norm assembly: norm[i] = sqrt(max(w[i] + (2s)*c[i] + (s*s)*b[i], 0)) in
 * fp32, four separately rounded ops in that order, NaN kept by the clamp,
 * IEEE square root.
 *
 * Replaces fused_norm_assembly (dora_fused.py:873-988, kernel 789-861).
 */
int dora_norm_assembly(const float* w_norm_sq, const float* cross, const float* ba, double scale,
                       float* norm_out, int64_t n, void* stream);

/* Bytes of workspace dora_weight_norm needs for this problem. */
size_t dora_weight_norm_workspace_size(int64_t out_features, int64_t in_features, int64_t rank,
                                       int w_dtype, int a_dtype, int b_dtype);

/*
 * Factored row norm of W0 + scale * B @ A without forming B @ A:
 *   norm[j]^2 = ||W0[j,:]||^2 + 2 s <B[j,:], (W0 A^T)[j,:]> + s^2 B[j,:] (A A^T) B[j,:]^T
 * then the assembly of dora_norm_assembly and a cast to w_dtype (norm_out has
 * w_dtype).  When parts != NULL it receives 3*out floats: ||W0||^2, the cross
 * term and the B G B^T term, each [out] in fp32.  scale == 0 computes
 * sqrt(||W0||^2) only.  bf16 and fp16 weights run on the tcgen05 tensor cores,
 * with adapters of the weight dtype or fp32 (fp32 adapters are first rounded
 * into the weight dtype in the workspace, an error below the norm's own
 * rounding into that dtype); fp32 weights run an fp32 CUDA-core path.
 *
 * Replaces DoraLinearLayer._get_weight_norm_linear (dora.py:1024-1153) with
 * its fused_norm_assembly call (dora.py:1136-1148).
 */
int dora_weight_norm(const void* W, const void* A, const void* B, int64_t out_features,
                     int64_t in_features, int64_t rank, int w_dtype, int a_dtype, int b_dtype,
                     double scale, void* norm_out, float* parts, void* workspace,
                     size_t workspace_bytes, void* stream);

/*
 * Dense row norm: norm[j] = || W[j,:] + scale * L[j,:] || in fp32 (scale * L
 * rounded first, then the sum, then a fp32 sum of squares and an IEEE square
 * root), cast to w_dtype.  L is the dense [out x in] LoRA weight.
 *
 * Replaces DoraLinearLayer.get_weight_norm (dora.py:1012-1022), which the
 * merge / unmerge paths use (variants.py:164-212).
 */
int dora_weight_norm_dense(const void* W, const void* L, int64_t out_features, int64_t in_features, int w_dtype,
                           int l_dtype, double scale, void* norm_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DORA_B200_H_ */
