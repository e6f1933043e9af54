/*
 * mamba_b200.h -- C-ABI of the B200 (sm_100a) selective-scan / conv1d / decode-step library.
 *
 * The library is libmamba_b200.so (built from mamba_metal_b200/csrc/). Every entry point takes a
 * plain argument struct of device pointers, element strides and sizes, plus a CUDA stream handle,
 * and returns MM_OK (0) or a negative MM_ERR_* code. No entry point aborts or allocates device memory,
 * and none keeps hidden mutable state except the fixed scratch buffer of mm_selective_scan_fwd_noalloc:
 * the caller owns every other buffer (outputs and workspace), and all work is ordered on the given
 * stream. Integer fields are int64_t so the struct layout is the same for
 * every FFI (ctypes, cgo, JNI) without padding surprises.
 *
 * Reference interface being replaced (createcentury/mamba-metal):
 *   - mamba_metal/selective_scan.py:12-20 builds an mx.fast.metal_kernel over
 *     kernels/selective_scan_chunked.metal, and selective_scan.py:62-76 calls it with
 *     inputs=[u, delta, A, B, C, D, z, batch, dim, dstate, seqlen, apply_softplus, use_D, use_z],
 *     output_shapes=[u.shape, (batch, dim, dstate)], output_dtypes=[u.dtype, float32].
 *     -> mm_selective_scan_fwd (+ mm_selective_scan_workspace_size, mm_selective_scan_status).
 *   - mamba_metal/mamba_block.py:45-52 / :129-130 (MLX nn.Conv1d, groups=d_inner, padding=d_conv-1,
 *     output sliced to [:, :L], then nn.silu) and the conv-state capture at mamba_block.py:118-127.
 *     -> mm_causal_conv1d_fwd.
 *   - mamba_metal/mamba_block.py:171-177 (decode: window shift, dot with the conv weight, + bias, SiLU).
 *     -> mm_causal_conv1d_step.
 *   - mamba_metal/mamba_block.py:183-195 (decode: softplus(dt), h = exp(dt*A)*h + dt*x*B,
 *     y = sum(h*C) + D*x, y *= silu(z)), and optionally the dt projection at :181.
 *     -> mm_ssm_decode_step.
 *   - mamba_metal/mamba_model.py:49-58 and :40,:69 (pre-RMSNorm + residual around each mixer).
 *     -> mm_add_rmsnorm.
 */
#ifndef MAMBA_B200_H
#define MAMBA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t, passed opaquely so that this header does not need the CUDA headers. NULL = legacy
 * default stream. */
typedef void* mm_stream_t;

/* Element types of activation tensors (u, delta, z, B, C, x, y). A, D, conv weights and all
 * recurrent state are always fp32. */
enum { MM_F32 = 0, MM_F16 = 1, MM_BF16 = 2 };

enum {
  MM_OK = 0,
  MM_ERR_ARG = -1,       /* NULL pointer where one is required, or a negative size */
  MM_ERR_SHAPE = -2,     /* size outside the supported range (e.g. dstate > 64, width != 4) */
  MM_ERR_DTYPE = -3,     /* unknown dtype code */
  MM_ERR_WORKSPACE = -4, /* workspace missing, too small or not 256-byte aligned */
  MM_ERR_LAUNCH = -5,    /* the CUDA launch (or the workspace clear) failed */
  MM_ERR_TIMEOUT = -6,   /* a carry hand-off between warps waited past its limit (status only) */
  MM_ERR_TOO_LARGE = -7  /* the call needs more scratch than the fixed buffer of the no-allocation entry */
};

/* Largest dstate the scan and the decode step accept (same limit as the reference,
 * mamba_metal/selective_scan.py:9 MAX_DSTATE = 64). */
#define MM_MAX_DSTATE 64

/* ---------------------------------------------------------------------------------------------
 * Selective scan forward.
 *   delta' = softplus(delta + delta_bias[d]) if delta_softplus else delta + delta_bias[d]
 *            (softplus uses the >20 cutoff; delta_bias is optional, 0 when NULL)
 *   h[t,n] = exp(delta'[t] * A[d,n]) * h[t-1,n] + delta'[t] * u[t] * B[n,t],   h[-1] = 0
 *   y[t]   = (sum_n h[t,n] * C[n,t] + D[d] * u[t]) * silu(z[t])   (D and z optional)
 *   state_out[b,d,n] = h[seqlen-1, n]
 * Shapes (element strides given per tensor, any layout):
 *   u, delta, z, y : (batch, dim, seqlen)   strides (b, d, t)
 *   B, C           : (batch, dstate, seqlen) strides (b, n, t)
 *   A              : (dim, dstate) fp32      strides (d, n)
 *   D              : (dim,) fp32 contiguous, or NULL
 *   state_out      : (batch, dim, dstate) fp32 contiguous, or NULL
 * Replaces mamba_metal/selective_scan.py:62-76 (the mx.fast.metal_kernel call). y has dtype
 * `dtype` (= u.dtype in the reference, selective_scan.py:73-74); the state is fp32.
 * The workspace (size from mm_selective_scan_workspace_size, 256-byte aligned) carries the
 * recurrent state between the warps that own consecutive pieces of one sequence; the call clears
 * the part that must start at zero itself (one cudaMemsetAsync on `stream`). Two calls that share
 * one workspace must not overlap in time on the GPU.
 * ------------------------------------------------------------------------------------------- */
typedef struct MMScanArgs {
  const void* u;
  const void* delta;
  const float* A;
  const void* B;
  const void* C;
  const float* D;   /* may be NULL */
  const void* z;    /* may be NULL */
  void* y;
  float* state_out; /* may be NULL */
  int64_t dtype;
  int64_t batch, dim, dstate, seqlen;
  int64_t u_stride[3];
  int64_t delta_stride[3];
  int64_t z_stride[3];
  int64_t y_stride[3];
  int64_t B_stride[3];
  int64_t C_stride[3];
  int64_t A_stride[2];
  int64_t delta_softplus; /* 0 / 1 */
  int64_t piece_tiles;    /* timestep tiles per warp; 0 = chosen by the library */
  int64_t options;        /* bit 0: stage tiles with cp.async / plain loads instead of TMA */
  const float* delta_bias; /* (dim,) fp32 added to delta before softplus, or NULL. No counterpart in the
                              reference's kernel: the dt_proj bias of a Mamba block (mamba_block.py:85),
                              applied here so that dt_proj's GEMM needs no separate bias pass */
} MMScanArgs;

int mm_selective_scan_workspace_size(const MMScanArgs* args, size_t* bytes);
int mm_selective_scan_fwd(const MMScanArgs* args, void* workspace, size_t workspace_bytes,
                          mm_stream_t stream);
/* Allocation-free variant of mm_selective_scan_fwd, for callers that cannot allocate device memory:
 * for example a host that runs inside a fixed memory budget carved out up front by another allocator,
 * or an FFI host (JNI, cgo, a real-time serving loop) whose policy forbids device allocation after
 * start-up. Instead of a caller-provided workspace it uses a scratch buffer of
 * MM_SCAN_NOALLOC_SCRATCH_BYTES that is a static __device__ array of this library: every GPU that loads
 * the library holds it until the process exits. The caller still provides every input and output.
 * With piece_tiles == 0 the library lengthens the per-warp pieces until the workspace fits the buffer;
 * calls that cannot fit even so (or whose explicit piece_tiles does not fit) return MM_ERR_TOO_LARGE
 * without launching anything. The first call on a device (and the first after a device reset, which
 * reloads the module) looks up the buffer's device address with cudaGetSymbolAddress; make that first
 * call before any stream capture. All calls share the one buffer, so calls that overlap in time on the
 * GPU (other streams, other host threads) race and must be serialised by the caller; each call clears
 * the part of the buffer that must start at zero. A carry wait that reaches its time limit cannot be
 * observed for these calls (mm_selective_scan_status needs the workspace address, which stays private).
 * No counterpart exists in the reference (its Metal kernel needs no workspace). */
#define MM_SCAN_NOALLOC_SCRATCH_BYTES (16u << 20)
int mm_selective_scan_fwd_noalloc(const MMScanArgs* args, mm_stream_t stream);
/* Synchronises `stream` and reports MM_OK or MM_ERR_TIMEOUT for the last scan that used
 * `workspace`. Diagnostics only; the scan itself never blocks the host. */
int mm_selective_scan_status(const void* workspace, mm_stream_t stream);
/* Synchronises `stream` and copies four counters of the last scan that used `workspace` into
 * out4: carry-wait spin iterations, look-back hops, timesteps recomputed after the carry arrived,
 * and pieces processed. Diagnostics only. */
int mm_selective_scan_stats(const void* workspace, unsigned long long* out4, mm_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Causal depthwise conv1d (prefill):
 *   out[b,d,t] = act(bias[d] + sum_{k<width} weight[d,k] * x[b,d,t-width+1+k]),  x[.,.,<0] = 0
 *   act = SiLU if silu else identity.
 * x, out: (batch, dim, seqlen) with element strides (b, d, t) -- channel-first (t contiguous) and
 * channels-last (d contiguous) both run on vectorised paths. weight: (dim, width) fp32 contiguous
 * (the PyTorch / HF (dim, 1, width) layout), bias: (dim,) fp32 or NULL.
 * conv_state (optional, fp32 (batch, dim, width) contiguous) receives the last `width` pre-conv
 * inputs x[b,d,seqlen-width .. seqlen-1], zero-filled on the left when seqlen < width: the
 * prefill -> decode hand-off of mamba_metal/mamba_block.py:118-127.
 * Replaces MLX nn.Conv1d at mamba_metal/mamba_block.py:45-52, :129-130. width must be 4.
 * ------------------------------------------------------------------------------------------- */
typedef struct MMConvArgs {
  const void* x;
  const float* weight;
  const float* bias; /* may be NULL */
  void* out;
  float* conv_state; /* may be NULL */
  int64_t dtype;
  int64_t batch, dim, seqlen, width;
  int64_t x_stride[3];
  int64_t out_stride[3];
  int64_t silu; /* 0 / 1 */
} MMConvArgs;

int mm_causal_conv1d_fwd(const MMConvArgs* args, mm_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Conv decode step (one token), in place on conv_state:
 *   conv_state[b,d,:] <- [conv_state[b,d,1:], x[b,d]]
 *   out[b,d] = act(bias[d] + sum_k weight[d,k] * conv_state[b,d,k])
 * x, out: (batch, dim) with row strides; conv_state: fp32 (batch, dim, width) contiguous.
 * batch <= 65535. Replaces mamba_metal/mamba_block.py:171-177.
 * ------------------------------------------------------------------------------------------- */
typedef struct MMConvStepArgs {
  const void* x;
  float* conv_state;
  const float* weight;
  const float* bias; /* may be NULL */
  void* out;
  int64_t dtype;
  int64_t batch, dim, width;
  int64_t x_stride_b, out_stride_b;
  int64_t silu;
  int64_t early_state; /* 1: conv_state was not written by the kernel just before this call on `stream`, so
                          the call may start (and load the state) while that kernel finishes; everything
                          else is read after it completes (programmatic dependent launch). 0: plain
                          stream order */
} MMConvStepArgs;

int mm_causal_conv1d_step(const MMConvStepArgs* args, mm_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * SSM decode step (one token), in place on ssm_state:
 *   dt' = softplus(dt) if dt_softplus else dt
 *   h[b,d,n] <- exp(dt'*A[d,n]) * h[b,d,n] + dt' * x[b,d] * B[b,n]
 *   y[b,d]   = (sum_n h[b,d,n] * C[b,n] + D[d] * x[b,d]) * silu(z[b,d])      (D, z optional)
 * x, dt, z, y: (batch, dim) with row strides; B, C: (batch, dstate) with row strides (the
 * x_proj output slices); A: (dim, dstate) fp32 contiguous; ssm_state: fp32 (batch, dim, dstate)
 * contiguous. Replaces mamba_metal/mamba_block.py:183-195.
 * ------------------------------------------------------------------------------------------- */
typedef struct MMSSMStepArgs {
  const void* x;
  const void* dt;
  const void* z; /* may be NULL */
  const void* B;
  const void* C;
  const float* A;
  const float* D; /* may be NULL */
  float* ssm_state;
  void* y;
  int64_t dtype;
  int64_t batch, dim, dstate;
  int64_t x_stride_b, dt_stride_b, z_stride_b, B_stride_b, C_stride_b, y_stride_b;
  int64_t dt_softplus; /* 0 / 1 */
  int64_t early_state; /* 1: ssm_state was not written by the kernel just before this call on `stream`, so
                          the call may start (and stream the state in) while that kernel finishes; every
                          other input is read after it completes (programmatic dependent launch) */
  /* Optional fused dt projection (mamba_block.py:181, dt_proj(x_dbl[:, :dt_rank])): when dt_w != NULL
     the call computes dt[b,d] = sum_k dt_in[b,k] * dt_w[d,k] + dt_bias[d] in fp32 (not rounded to
     `dtype`) and does not read dt / dt_stride_b. dt_in: (batch, dt_rank) of `dtype`, unit inner stride,
     row stride dt_in_stride_b (x_proj's first dt_rank output columns); dt_w: (dim, dt_rank) of `dtype`,
     row stride dt_w_stride (dt_proj.weight); dt_bias: (dim,) fp32, may be NULL. Under early_state dt_w and
     dt_bias are read before the preceding kernel completes (they must not be its outputs). */
  const void* dt_in;
  const void* dt_w;
  const float* dt_bias;
  int64_t dt_rank, dt_in_stride_b, dt_w_stride;
} MMSSMStepArgs;

int mm_ssm_decode_step(const MMSSMStepArgs* args, mm_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Residual add + RMSNorm over the last dimension (rows of length `dim`):
 *   if delta != NULL: residual[r,:] += delta[r,:]          (residual is fp32, updated in place)
 *   out[r,:] = residual[r,:] * rsqrt(mean(residual[r,:]^2) + eps) * weight[:]
 * residual: fp32 (rows, dim) contiguous; delta, out: dtype `dtype`, rows contiguous with row
 * strides; weight: fp32 (dim,). Replaces the pre-norm residual wrapper of
 * mamba_metal/mamba_model.py:49-58 (nn.RMSNorm at :40, eps at :32) and norm_f at :69, :76.
 * ------------------------------------------------------------------------------------------- */
typedef struct MMAddNormArgs {
  float* residual;
  const void* delta; /* may be NULL */
  const float* weight;
  void* out;
  int64_t dtype;
  int64_t rows, dim;
  int64_t delta_stride_r, out_stride_r;
  double eps;
} MMAddNormArgs;

int mm_add_rmsnorm(const MMAddNormArgs* args, mm_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * One-shot all-reduce over peer memory, for the tensor-parallel decode step (a B200 addition: the
 * reference has no multi-device code). Every rank owns a receive area of `world` regions, `stride`
 * elements apart, in memory that all ranks map (symmetric memory); slots[r] is rank r's area as mapped
 * in this process. Before the call each rank has written its n-element partial at the start of region
 * `rank` of its own area. Two protocols:
 *   MM_PEER_FLAGS: CTA c stores slice c of the partial into region `rank` of every peer's area (posted
 *     NVLink stores), then tells each peer "slice c of call e has arrived" through the signal pads
 *     (epoch e from counters[c]); it waits for every peer's word, then sums slice c of the `world`
 *     partials from local memory into `out`. Signal pads: MM_PEER_MAX_BLOCKS * MM_MAX_TP words each.
 *   MM_PEER_LL (low latency, small n): the partial travels as 16-byte lines of two data words, each
 *     beside the call's epoch in the same 8-byte half; receivers poll the lines themselves (no fence,
 *     no signal pad). Needs stride * element size >= 2 * (n * element size rounded up to 8 bytes).
 * Sums are in fp32 in rank order; every wait gives up after 2 s and sets the error word. counters:
 * MM_PEER_MAX_BLOCKS + 3 words of local device memory, zero-initialised (flag epochs, the error word,
 * the LL epoch and a ticket); areas and pads zero-initialised. All ranks must make the same sequence of
 * calls with the same n, protocol and nblocks; peers rewrite an area as soon as they have passed the
 * previous call, so consecutive calls must use different areas.
 * ------------------------------------------------------------------------------------------- */
#define MM_MAX_TP 8
#define MM_PEER_MAX_BLOCKS 64
#define MM_PEER_FLAGS 0
#define MM_PEER_LL 1
typedef struct MMPeerReduceArgs {
  void* slots[MM_MAX_TP];
  unsigned* signals[MM_MAX_TP];
  unsigned* counters;
  void* out;
  int64_t dtype, n, stride, world, rank, nblocks, protocol;
} MMPeerReduceArgs;

int mm_peer_allreduce(const MMPeerReduceArgs* args, mm_stream_t stream);

/* The low-latency all-reduce of a (rows, dim) partial fused with the residual add + RMSNorm that
 * follows the out_proj reduction in a tensor-parallel decode step (mamba_model.py:49-58 with
 * nn.RMSNorm): per row, s = sum over ranks (fp32, rank order) rounded to `dtype`;
 * residual += s (fp32, in place); out = residual * rsqrt(mean(residual^2) + eps) * weight.
 * reduce.protocol must be MM_PEER_LL, reduce.n = rows * dim, reduce.out is unused; dim * element size
 * a multiple of 8 bytes and at most 16 KiB; residual (rows, dim) fp32 contiguous, 16-byte aligned;
 * weight (dim,) fp32; out (rows, dim) of `dtype` with row stride out_stride_r. One CTA per row
 * (reduce.nblocks only has to be in range); it shares the LL epoch counter with mm_peer_allreduce (one
 * sequence of calls). */
typedef struct MMPeerAddNormArgs {
  MMPeerReduceArgs reduce;
  float* residual;
  const float* weight;
  void* out;
  int64_t rows, dim, out_stride_r;
  double eps;
} MMPeerAddNormArgs;

int mm_peer_allreduce_add_rmsnorm(const MMPeerAddNormArgs* args, mm_stream_t stream);

/* Self-check of the kernels' device math: y_poly[i] = 2^x[i] from the FMA-pipe polynomial the scan uses for
 * part of its exponentials with general A, y_mufu[i] = the hardware ex2.approx of x[i]; n floats each,
 * device pointers. Test and diagnostics use only; no counterpart in the reference. */
int mm_exp2_check(const float* x, float* y_poly, float* y_mufu, int64_t n, mm_stream_t stream);

/* Library version string (static storage). */
/* ---------------------------------------------------------------------------------------------
 * Dense projection of the decode step: y = x @ w^T (+ bias), bf16 inputs, fp32 accumulation.
 *   x: (M, K) bf16, row stride ldx;  w: (N, K) bf16, row stride ldw (the nn.Linear weight layout);
 *   bias: (N,) fp32 or NULL;  y: (M, N) of y_dtype (MM_F32 or MM_BF16), row stride ldy.
 * Replaces the nn.Linear calls of the decode step, mamba_metal/mamba_block.py:167 (in_proj), :179
 * (x_proj), :181 (dt_proj) and :197 (out_proj); the same shapes serve any small-M product. Base
 * pointers and row strides of x and w must be 16-byte aligned (TMA). splits = 0 lets the library split
 * K over CTAs so that every SM streams weights; split partials are added into an fp32 tile of the
 * workspace in arrival order, so with splits > 1 results can differ in the last bits between calls.
 * The workspace (size from
 * mm_linear_workspace_size, 256-byte aligned) must be zero-filled before its first use; every call
 * leaves it zeroed again. Calls sharing a workspace must not overlap on the GPU.
 * ------------------------------------------------------------------------------------------- */
typedef struct MMLinearArgs {
  const void* x;
  const void* w;
  const float* bias; /* may be NULL */
  void* y;
  int64_t ldx, ldw, ldy;
  int64_t y_dtype;
  int64_t M, N, K;
  int64_t splits; /* 0 = chosen by the library */
} MMLinearArgs;

int mm_linear_workspace_size(const MMLinearArgs* args, size_t* bytes);
int mm_linear_fwd(const MMLinearArgs* args, void* workspace, size_t workspace_bytes, mm_stream_t stream);
/* Synchronises `stream`; MM_ERR_TIMEOUT if a pipeline wait of a call on `workspace` ran out. */
int mm_linear_status(const void* workspace, mm_stream_t stream);

const char* mm_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MAMBA_B200_H */
