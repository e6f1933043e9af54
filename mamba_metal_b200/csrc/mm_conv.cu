// Causal depthwise conv1d (width 4) for sm_100a: prefill over a sequence and the one-token decode step.
//
// Semantics: MLX nn.Conv1d with groups = channels, padding = width - 1 and the output sliced to the
// first seqlen positions (mamba_metal/mamba_block.py:45-52, :129-130), i.e.
//   out[t] = act(bias + sum_k w[k] * x[t - (width-1) + k]),  x[<0] = 0,
// which is the same window that the decode step forms by shifting its state (mamba_block.py:171-177).
// Both are HBM-bound elementwise stencils: every input element is read once with 16-byte vector loads,
// the three-element causal halo comes from the neighbouring lane (channel-first) or from a rolling
// register window (channels-last), and bias + SiLU are fused into the store.
#include "mm_common.cuh"

namespace mm {
namespace conv {

constexpr int kW = 4;   // conv width (d_conv)
constexpr int kE = 8;   // elements per thread per step

template <typename T> MM_DEV void load8(const T* p, float (&v)[kE]);
template <> MM_DEV void load8<float>(const float* p, float (&v)[kE]) {
  const uint4 a = __ldcs(reinterpret_cast<const uint4*>(p));
  const uint4 b = __ldcs(reinterpret_cast<const uint4*>(p) + 1);
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const float2 pa = vec_pair<float>(a, k), pb = vec_pair<float>(b, k);
    v[2 * k] = pa.x;
    v[2 * k + 1] = pa.y;
    v[2 * k + 4] = pb.x;
    v[2 * k + 5] = pb.y;
  }
}
template <typename T> MM_DEV void load8_16(const T* p, float (&v)[kE]) {
  const uint4 a = __ldcs(reinterpret_cast<const uint4*>(p));
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 pr = vec_pair<T>(a, k);
    v[2 * k] = pr.x;
    v[2 * k + 1] = pr.y;
  }
}
template <> MM_DEV void load8<__half>(const __half* p, float (&v)[kE]) { load8_16<__half>(p, v); }
template <> MM_DEV void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[kE]) { load8_16<__nv_bfloat16>(p, v); }

template <typename T> MM_DEV void store8(T* p, const float (&v)[kE]);
template <> MM_DEV void store8<float>(float* p, const float (&v)[kE]) {
  uint4 a, b;
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    vec_set_pair<float>(a, k, v[2 * k], v[2 * k + 1]);
    vec_set_pair<float>(b, k, v[2 * k + 4], v[2 * k + 5]);
  }
  __stcs(reinterpret_cast<uint4*>(p), a);
  __stcs(reinterpret_cast<uint4*>(p) + 1, b);
}
template <typename T> MM_DEV void store8_16(T* p, const float (&v)[kE]) {
  uint4 a;
#pragma unroll
  for (int k = 0; k < 4; ++k) vec_set_pair<T>(a, k, v[2 * k], v[2 * k + 1]);
  __stcs(reinterpret_cast<uint4*>(p), a);
}
template <> MM_DEV void store8<__half>(__half* p, const float (&v)[kE]) { store8_16<__half>(p, v); }
template <> MM_DEV void store8<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[kE]) { store8_16<__nv_bfloat16>(p, v); }

MM_DEV float act(float v, bool use_silu) { return use_silu ? silu(v) : v; }

struct Params {
  const void* x;
  const float* w;
  const float* bias;
  void* out;
  float* conv_state;
  long long xs[3], os[3];
  int batch, dim, seqlen;
  int silu;
};

// Channel-first (t contiguous). A warp covers kCPT * 32 consecutive 8-element chunks of one (b, d) row:
// lane l owns chunks l, l + 32, l + 64, ... so every load and store instruction of the warp is one
// contiguous 512-byte (fp16) access, and all kCPT loads are in flight before the first is used. The
// three-element causal halo of a chunk is the end of the previous chunk: the neighbouring lane's, lane 31's
// previous chunk for lane 0, or memory for the warp's first chunk.
constexpr int kCPT = 4;

#ifndef MM_CONV_MIN_BLOCKS
#define MM_CONV_MIN_BLOCKS 4  // resident 256-thread CTAs per SM the channel-first kernel is compiled for: 4 (64
                              // registers) measured ~5% faster than no bound (77 registers); 5 slower
#endif

template <typename T, bool VEC>
__global__ void __launch_bounds__(256, MM_CONV_MIN_BLOCKS) conv_tfirst_kernel(const Params p, int chunks_per_row, int warps_per_row) {
  const int lane = threadIdx.x & 31;
  const long long gw = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const long long rows = (long long)p.batch * p.dim;
  if (gw >= rows * warps_per_row) return;
  const long long row = gw / warps_per_row;
  const int cbase = (int)(gw % warps_per_row) * 32 * kCPT;
  const int b = (int)(row / p.dim), d = (int)(row % p.dim);
  const T* xr = static_cast<const T*>(p.x) + b * p.xs[0] + d * p.xs[1];
  T* orow = static_cast<T*>(p.out) + b * p.os[0] + d * p.os[1];
  float v[kCPT][kE];
#pragma unroll
  for (int j = 0; j < kCPT; ++j) {
    const int t0 = (cbase + j * 32 + lane) * kE;
    if (VEC && t0 + kE <= p.seqlen) {
      load8<T>(xr + t0, v[j]);
    } else {
#pragma unroll
      for (int k = 0; k < kE; ++k) v[j][k] = (t0 + k < p.seqlen) ? ld_f32(xr + (long long)(t0 + k) * p.xs[2]) : 0.f;
    }
  }
  const float w0 = p.w[d * kW + 0], w1 = p.w[d * kW + 1], w2 = p.w[d * kW + 2], w3 = p.w[d * kW + 3];
  const float bb = p.bias ? p.bias[d] : 0.f;
#pragma unroll
  for (int j = 0; j < kCPT; ++j) {
    const int chunk = cbase + j * 32 + lane;
    const int t0 = chunk * kE;
    // halo x[t0-3 .. t0-1]
    float h0 = __shfl_up_sync(0xffffffffu, v[j][5], 1);
    float h1 = __shfl_up_sync(0xffffffffu, v[j][6], 1);
    float h2 = __shfl_up_sync(0xffffffffu, v[j][7], 1);
    if (j > 0) {
      const float p0 = __shfl_sync(0xffffffffu, v[j - 1][5], 31);
      const float p1 = __shfl_sync(0xffffffffu, v[j - 1][6], 31);
      const float p2 = __shfl_sync(0xffffffffu, v[j - 1][7], 31);
      if (lane == 0) { h0 = p0; h1 = p1; h2 = p2; }
    } else if (lane == 0) {
      h0 = t0 - 3 >= 0 ? ld_f32(xr + (long long)(t0 - 3) * p.xs[2]) : 0.f;
      h1 = t0 - 2 >= 0 ? ld_f32(xr + (long long)(t0 - 2) * p.xs[2]) : 0.f;
      h2 = t0 - 1 >= 0 ? ld_f32(xr + (long long)(t0 - 1) * p.xs[2]) : 0.f;
    }
    if (chunk >= chunks_per_row) continue;
    float win[kE + 3] = {h0, h1, h2};
#pragma unroll
    for (int k = 0; k < kE; ++k) win[k + 3] = v[j][k];
    float o[kE];
#pragma unroll
    for (int k = 0; k < kE; ++k) {
      float sacc = bb;
      sacc = fmaf(w0, win[k], sacc);
      sacc = fmaf(w1, win[k + 1], sacc);
      sacc = fmaf(w2, win[k + 2], sacc);
      sacc = fmaf(w3, win[k + 3], sacc);
      o[k] = act(sacc, p.silu);
    }
    if (VEC && t0 + kE <= p.seqlen) {
      store8<T>(orow + t0, o);
    } else {
#pragma unroll
      for (int k = 0; k < kE; ++k)
        if (t0 + k < p.seqlen) st_f32(orow + (long long)(t0 + k) * p.os[2], o[k]);
    }
    // conv-state hand-off: the last kW inputs of the row, taken by the chunk that holds t = seqlen - 1
    if (p.conv_state && t0 <= p.seqlen - 1 && p.seqlen - 1 < t0 + kE) {
      const int last = p.seqlen - 1 - t0;  // index of t = seqlen-1 in this chunk
      float* cs = p.conv_state + ((long long)b * p.dim + d) * kW;
      // win[last + k] through a select over the kE possible positions: a run-time index would put the
      // whole window in local memory for every chunk
      float sel[kW];
#pragma unroll
      for (int k = 0; k < kW; ++k) sel[k] = 0.f;
#pragma unroll
      for (int m = 0; m < kE; ++m)
        if (m == last) {
#pragma unroll
          for (int k = 0; k < kW; ++k) sel[k] = win[m + k];
        }
#pragma unroll
      for (int k = 0; k < kW; ++k) {
        const int t = p.seqlen - kW + k;
        cs[k] = t >= 0 ? sel[k] : 0.f;
      }
    }
  }
}

// Channels-last (d contiguous). A thread owns 8 consecutive channels and walks `run` timesteps with a
// rolling window; a warp covers 256 channels, so each row of a step is one coalesced 512-byte access
// (fp16/bf16).
template <typename T, bool VEC>
__global__ void __launch_bounds__(256) conv_dlast_kernel(const Params p, int run, int runs_per_seq) {
  const long long gt = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int cgroups = (p.dim + kE - 1) / kE;
  const long long total = (long long)p.batch * runs_per_seq * cgroups;
  if (gt >= total) return;
  const int cg = (int)(gt % cgroups);
  const long long rest = gt / cgroups;
  const int r = (int)(rest % runs_per_seq);
  const int b = (int)(rest / runs_per_seq);
  const int d0 = cg * kE;
  const int t_begin = r * run;
  const int t_end = min(p.seqlen, t_begin + run);
  const T* xb = static_cast<const T*>(p.x) + b * p.xs[0];
  T* ob = static_cast<T*>(p.out) + b * p.os[0];
  const bool vec = VEC && d0 + kE <= p.dim;
  float w[kW][kE], bb[kE];
#pragma unroll
  for (int c = 0; c < kE; ++c) {
    const int d = min(d0 + c, p.dim - 1);
#pragma unroll
    for (int k = 0; k < kW; ++k) w[k][c] = p.w[d * kW + k];
    bb[c] = p.bias ? p.bias[d] : 0.f;
  }
  auto load_row = [&](int t, float (&v)[kE]) {
    if (t < 0) {
#pragma unroll
      for (int c = 0; c < kE; ++c) v[c] = 0.f;
    } else if (vec) {
      load8<T>(xb + (long long)t * p.xs[2] + d0, v);
    } else {
#pragma unroll
      for (int c = 0; c < kE; ++c)
        v[c] = d0 + c < p.dim ? ld_f32(xb + (long long)t * p.xs[2] + (long long)(d0 + c) * p.xs[1]) : 0.f;
    }
  };
  float x0[kE], x1[kE], x2[kE], x3[kE];
  load_row(t_begin - 3, x0);
  load_row(t_begin - 2, x1);
  load_row(t_begin - 1, x2);
#pragma unroll 4
  for (int t = t_begin; t < t_end; ++t) {
    load_row(t, x3);
    float o[kE];
#pragma unroll
    for (int c = 0; c < kE; ++c) {
      float s = bb[c];
      s = fmaf(w[0][c], x0[c], s);
      s = fmaf(w[1][c], x1[c], s);
      s = fmaf(w[2][c], x2[c], s);
      s = fmaf(w[3][c], x3[c], s);
      o[c] = act(s, p.silu);
    }
    if (vec) {
      store8<T>(ob + (long long)t * p.os[2] + d0, o);
    } else {
#pragma unroll
      for (int c = 0; c < kE; ++c)
        if (d0 + c < p.dim) st_f32(ob + (long long)t * p.os[2] + (long long)(d0 + c) * p.os[1], o[c]);
    }
#pragma unroll
    for (int c = 0; c < kE; ++c) {
      x0[c] = x1[c];
      x1[c] = x2[c];
      x2[c] = x3[c];
    }
  }
  if (p.conv_state && t_end == p.seqlen && t_begin < t_end) {
    // After the last shift x0..x2 hold x[seqlen-3 .. seqlen-1]; x[seqlen-4] is reloaded.
    float xm[kE];
    load_row(p.seqlen - 4, xm);
#pragma unroll
    for (int c = 0; c < kE; ++c) {
      if (d0 + c < p.dim) {
        float* cs = p.conv_state + ((long long)b * p.dim + d0 + c) * kW;
        cs[0] = xm[c];
        cs[1] = x0[c];
        cs[2] = x1[c];
        cs[3] = x2[c];
      }
    }
  }
}

// Any layout: one thread per output element.
template <typename T>
__global__ void __launch_bounds__(256) conv_generic_kernel(const Params p) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long n = (long long)p.batch * p.dim * p.seqlen;
  if (i >= n) return;
  const int t = (int)(i % p.seqlen);
  const long long row = i / p.seqlen;
  const int d = (int)(row % p.dim), b = (int)(row / p.dim);
  const T* xr = static_cast<const T*>(p.x) + b * p.xs[0] + d * p.xs[1];
  float s = p.bias ? p.bias[d] : 0.f;
#pragma unroll
  for (int k = 0; k < kW; ++k) {
    const int tt = t - (kW - 1) + k;
    if (tt >= 0) s = fmaf(p.w[d * kW + k], ld_f32(xr + (long long)tt * p.xs[2]), s);
  }
  T* orow = static_cast<T*>(p.out) + b * p.os[0] + d * p.os[1];
  st_f32(orow + (long long)t * p.os[2], act(s, p.silu));
  if (p.conv_state && t == p.seqlen - 1) {
    float* cs = p.conv_state + ((long long)b * p.dim + d) * kW;
#pragma unroll
    for (int k = 0; k < kW; ++k) {
      const int tt = p.seqlen - kW + k;
      cs[k] = tt >= 0 ? ld_f32(xr + (long long)tt * p.xs[2]) : 0.f;
    }
  }
}

template <typename T>
static cudaError_t launch_fwd(const Params& p, cudaStream_t s) {
  const int es = sizeof(T);
  const int epv = 16 / es;
  const bool xt = p.xs[2] == 1, ot = p.os[2] == 1;
  const bool xd = p.xs[1] == 1, od = p.os[1] == 1;
  if (xt && ot) {
    const bool vec = aligned16(p.x) && aligned16(p.out) && p.xs[0] % epv == 0 && p.xs[1] % epv == 0 &&
                     p.os[0] % epv == 0 && p.os[1] % epv == 0;
    const int cpr = (p.seqlen + kE - 1) / kE;
    const int wpr = (cpr + 32 * kCPT - 1) / (32 * kCPT);
    const long long warps = (long long)p.batch * p.dim * wpr;
    const long long blocks = (warps + 7) / 8;
    if (vec) conv_tfirst_kernel<T, true><<<(unsigned)blocks, 256, 0, s>>>(p, cpr, wpr);
    else conv_tfirst_kernel<T, false><<<(unsigned)blocks, 256, 0, s>>>(p, cpr, wpr);
  } else if (xd && od) {
    const bool vec = aligned16(p.x) && aligned16(p.out) && p.xs[0] % epv == 0 && p.xs[2] % epv == 0 &&
                     p.os[0] % epv == 0 && p.os[2] % epv == 0;
    const int cgroups = (p.dim + kE - 1) / kE;
    // enough threads to fill the GPU: runs of >= 64 steps, split further while threads are scarce
    long long base = (long long)p.batch * cgroups;
    int runs = 1;
    while (base * runs < 148LL * 2048 && p.seqlen / (runs * 2) >= 64) runs *= 2;
    const int run = (p.seqlen + runs - 1) / runs;
    const int rps = (p.seqlen + run - 1) / run;
    const long long threads = base * rps;
    const long long blocks = (threads + 255) / 256;
    if (vec) conv_dlast_kernel<T, true><<<(unsigned)blocks, 256, 0, s>>>(p, run, rps);
    else conv_dlast_kernel<T, false><<<(unsigned)blocks, 256, 0, s>>>(p, run, rps);
  } else {
    const long long n = (long long)p.batch * p.dim * p.seqlen;
    conv_generic_kernel<T><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(p);
  }
  return cudaGetLastError();
}

// ---- decode step -------------------------------------------------------------------------------
struct StepParams {
  const void* x;
  float* state;
  const float* w;
  const float* bias;
  void* out;
  long long xsb, osb;
  int batch, dim;
  int silu;
};

#ifndef MM_CONV_STEP_ROWS
#define MM_CONV_STEP_ROWS 2  // batch rows per thread in the conv decode step (the weights are reused across them)
#endif
constexpr int kStepRows = MM_CONV_STEP_ROWS;

template <typename T>
__global__ void __launch_bounds__(256) conv_step_kernel(const StepParams p) {
  // grid (channel blocks, batch / kStepRows): no per-thread division
  const int d = blockIdx.x * blockDim.x + threadIdx.x, b0 = blockIdx.y * kStepRows;
  if (d >= p.dim) return;
  // the window states first (with an early-state launch they load while the kernel before this one
  // finishes); everything else after grid_dep_wait
  float4 s[kStepRows];
#pragma unroll
  for (int r = 0; r < kStepRows; ++r)
    if (b0 + r < p.batch) s[r] = *reinterpret_cast<const float4*>(p.state + ((long long)(b0 + r) * p.dim + d) * kW);
  grid_dep_wait();
  const float4 w = *reinterpret_cast<const float4*>(p.w + d * kW);
  const float bias = p.bias ? p.bias[d] : 0.f;
  float xn[kStepRows];
#pragma unroll
  for (int r = 0; r < kStepRows; ++r)
    xn[r] = b0 + r < p.batch ? ld_f32(static_cast<const T*>(p.x) + (long long)(b0 + r) * p.xsb + d) : 0.f;
#pragma unroll
  for (int r = 0; r < kStepRows; ++r) {
    if (b0 + r >= p.batch) break;
    float v = bias;
    v = fmaf(w.x, s[r].y, v);
    v = fmaf(w.y, s[r].z, v);
    v = fmaf(w.z, s[r].w, v);
    v = fmaf(w.w, xn[r], v);
    *reinterpret_cast<float4*>(p.state + ((long long)(b0 + r) * p.dim + d) * kW) = make_float4(s[r].y, s[r].z, s[r].w, xn[r]);
    st_f32(static_cast<T*>(p.out) + (long long)(b0 + r) * p.osb + d, act(v, p.silu));
  }
}

}  // namespace conv
}  // namespace mm

using namespace mm;

extern "C" int mm_causal_conv1d_fwd(const MMConvArgs* a, mm_stream_t stream) {
  if (!a) return MM_ERR_ARG;
  if (dtype_size(a->dtype) == 0) return MM_ERR_DTYPE;
  if (a->width != conv::kW) return MM_ERR_SHAPE;
  if (a->batch < 0 || a->dim < 0 || a->seqlen < 0) return MM_ERR_SHAPE;
  if (a->batch > (1 << 30) || a->dim > (1 << 30) || a->seqlen > (1 << 30)) return MM_ERR_SHAPE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a->batch == 0 || a->dim == 0) return MM_OK;
  if (a->seqlen == 0) {
    if (a->conv_state &&
        cudaMemsetAsync(a->conv_state, 0, sizeof(float) * a->batch * a->dim * conv::kW, s) != cudaSuccess)
      return MM_ERR_LAUNCH;
    return MM_OK;
  }
  if (!a->x || !a->weight || !a->out) return MM_ERR_ARG;
  conv::Params p;
  p.x = a->x; p.w = a->weight; p.bias = a->bias; p.out = a->out; p.conv_state = a->conv_state;
  for (int i = 0; i < 3; ++i) { p.xs[i] = a->x_stride[i]; p.os[i] = a->out_stride[i]; }
  p.batch = (int)a->batch; p.dim = (int)a->dim; p.seqlen = (int)a->seqlen; p.silu = a->silu != 0;
  cudaError_t e;
  if (a->dtype == MM_F32) e = conv::launch_fwd<float>(p, s);
  else if (a->dtype == MM_F16) e = conv::launch_fwd<__half>(p, s);
  else e = conv::launch_fwd<__nv_bfloat16>(p, s);
  return e == cudaSuccess ? MM_OK : MM_ERR_LAUNCH;
}

extern "C" int mm_causal_conv1d_step(const MMConvStepArgs* a, mm_stream_t stream) {
  if (!a) return MM_ERR_ARG;
  if (dtype_size(a->dtype) == 0) return MM_ERR_DTYPE;
  if (a->width != conv::kW) return MM_ERR_SHAPE;
  if (a->batch < 0 || a->dim < 0) return MM_ERR_SHAPE;
  if (a->batch == 0 || a->dim == 0) return MM_OK;
  if (!a->x || !a->conv_state || !a->weight || !a->out) return MM_ERR_ARG;
  if (!aligned16(a->conv_state) || !aligned16(a->weight)) return MM_ERR_ARG;
  conv::StepParams p;
  p.x = a->x; p.state = a->conv_state; p.w = a->weight; p.bias = a->bias; p.out = a->out;
  p.xsb = a->x_stride_b; p.osb = a->out_stride_b; p.batch = (int)a->batch; p.dim = (int)a->dim;
  p.silu = a->silu != 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a->batch > 65535 || a->dim > (1 << 30)) return MM_ERR_SHAPE;  // grid.y = batch
  const dim3 blocks((unsigned)((p.dim + 255) / 256), (unsigned)((p.batch + conv::kStepRows - 1) / conv::kStepRows));
  cudaError_t e;
  if (a->dtype == MM_F32) e = launch_maybe_early(conv::conv_step_kernel<float>, blocks, 256, s, a->early_state, p);
  else if (a->dtype == MM_F16) e = launch_maybe_early(conv::conv_step_kernel<__half>, blocks, 256, s, a->early_state, p);
  else e = launch_maybe_early(conv::conv_step_kernel<__nv_bfloat16>, blocks, 256, s, a->early_state, p);
  return e == cudaSuccess ? MM_OK : MM_ERR_LAUNCH;
}
