// One-token SSM decode step and the fused residual-add + RMSNorm, for sm_100a.
//
// mm_ssm_decode_step restates mamba_metal/mamba_block.py:183-195: dt = softplus(dt_proj(.)),
// h = exp(dt*A)*h + (dt*x)*B, y = sum_n h*C + D*x, y *= silu(z). One thread owns one (batch, channel)
// with its dstate states in registers; the fp32 state row (64 bytes for dstate 16) is read and written
// once with 16-byte vectors, so the step is bound by the state traffic, and A / B / C rows are shared
// through L1.
//
// mm_add_rmsnorm restates the pre-norm residual wrapper of mamba_metal/mamba_model.py:49-58 with
// nn.RMSNorm (x * rsqrt(mean(x^2) + eps) * weight, eps from :32): residual += delta, then normalise.
#include "mm_common.cuh"

namespace mm {
namespace step {

struct SSMParams {
  const void* x;
  const void* dt;
  const void* z;
  const void* B;
  const void* C;
  const float* A;
  const float* D;
  float* state;
  void* y;
  long long xsb, dtsb, zsb, Bsb, Csb, ysb;
  int batch, dim, nstate;
  int softplus;
  int vec;  // state and A rows 16-byte aligned and dstate == NM: float4 path
};

template <typename T, int NM>
__global__ void __launch_bounds__(128) ssm_step_kernel(const SSMParams p) {
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.y;
  if (d >= p.dim) return;
  const T* xb = static_cast<const T*>(p.x) + b * p.xsb;
  const float xv = ld_f32(xb + d);
  const float dr = ld_f32(static_cast<const T*>(p.dt) + b * p.dtsb + d);
  const float d2 = p.softplus ? softplus_log2(dr) : dr * kLog2e;  // delta * log2(e)
  const float du = d2 * kLn2 * xv;                               // delta * x
  const T* Bb = static_cast<const T*>(p.B) + b * p.Bsb;
  const T* Cb = static_cast<const T*>(p.C) + b * p.Csb;
  const float* Ar = p.A + (long long)d * p.nstate;
  float* hs = p.state + ((long long)b * p.dim + d) * p.nstate;
  float y = 0.f;
  if (p.vec && p.nstate == NM) {
    float4* h4 = reinterpret_cast<float4*>(hs);
    const float4* a4 = reinterpret_cast<const float4*>(Ar);
#pragma unroll
    for (int q = 0; q < NM / 4; ++q) {
      float4 h = h4[q];
      const float4 a = __ldg(a4 + q);
      const int n = 4 * q;
      h.x = fmaf(ex2(d2 * a.x), h.x, du * ld_f32(Bb + n + 0));
      h.y = fmaf(ex2(d2 * a.y), h.y, du * ld_f32(Bb + n + 1));
      h.z = fmaf(ex2(d2 * a.z), h.z, du * ld_f32(Bb + n + 2));
      h.w = fmaf(ex2(d2 * a.w), h.w, du * ld_f32(Bb + n + 3));
      y = fmaf(h.x, ld_f32(Cb + n + 0), y);
      y = fmaf(h.y, ld_f32(Cb + n + 1), y);
      y = fmaf(h.z, ld_f32(Cb + n + 2), y);
      y = fmaf(h.w, ld_f32(Cb + n + 3), y);
      h4[q] = h;
    }
  } else {
    for (int n = 0; n < p.nstate; ++n) {
      const float h = fmaf(ex2(d2 * Ar[n]), hs[n], du * ld_f32(Bb + n));
      hs[n] = h;
      y = fmaf(h, ld_f32(Cb + n), y);
    }
  }
  if (p.D) y = fmaf(p.D[d], xv, y);
  if (p.z) y *= silu(ld_f32(static_cast<const T*>(p.z) + b * p.zsb + d));
  st_f32(static_cast<T*>(p.y) + b * p.ysb + d, y);
}

struct NormParams {
  float* res;
  const void* delta;
  const float* w;
  void* out;
  long long dsr, osr;
  int rows, dim;
  float eps;
};

// One CTA per row; the row is kept in registers between the sum-of-squares and the scaling pass.
template <typename T, int PER>
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(const NormParams p) {
  const int r = blockIdx.x;
  float* res = p.res + (long long)r * p.dim;
  const T* dl = p.delta ? static_cast<const T*>(p.delta) + (long long)r * p.dsr : nullptr;
  float v[PER];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    float x = 0.f;
    if (c < p.dim) {
      x = res[c];
      if (dl) {
        x += ld_f32(dl + c);
        res[c] = x;
      }
    }
    v[i] = x;
    ss = fmaf(x, x, ss);
  }
  __shared__ float red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)p.dim + p.eps);
  T* out = static_cast<T*>(p.out) + (long long)r * p.osr;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < p.dim) st_f32(out + c, v[i] * inv * p.w[c]);
  }
}

template <typename T>
static cudaError_t launch_norm(const NormParams& p, cudaStream_t s) {
  const int per = (p.dim + 255) / 256;
  if (per <= 2) add_rmsnorm_kernel<T, 2><<<p.rows, 256, 0, s>>>(p);
  else if (per <= 4) add_rmsnorm_kernel<T, 4><<<p.rows, 256, 0, s>>>(p);
  else if (per <= 8) add_rmsnorm_kernel<T, 8><<<p.rows, 256, 0, s>>>(p);
  else if (per <= 16) add_rmsnorm_kernel<T, 16><<<p.rows, 256, 0, s>>>(p);
  else if (per <= 32) add_rmsnorm_kernel<T, 32><<<p.rows, 256, 0, s>>>(p);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace step
}  // namespace mm

using namespace mm;

extern "C" int mm_ssm_decode_step(const MMSSMStepArgs* a, mm_stream_t stream) {
  if (!a) return MM_ERR_ARG;
  if (dtype_size(a->dtype) == 0) return MM_ERR_DTYPE;
  if (a->batch < 0 || a->dim < 0 || a->dstate < 1 || a->dstate > MM_MAX_DSTATE) return MM_ERR_SHAPE;
  if (a->batch > 65535 || a->dim > (1 << 30)) return MM_ERR_SHAPE;
  if (a->batch == 0 || a->dim == 0) return MM_OK;
  if (!a->x || !a->dt || !a->B || !a->C || !a->A || !a->ssm_state || !a->y) return MM_ERR_ARG;
  step::SSMParams p;
  p.x = a->x; p.dt = a->dt; p.z = a->z; p.B = a->B; p.C = a->C; p.A = a->A; p.D = a->D;
  p.state = a->ssm_state; p.y = a->y;
  p.xsb = a->x_stride_b; p.dtsb = a->dt_stride_b; p.zsb = a->z_stride_b; p.Bsb = a->B_stride_b;
  p.Csb = a->C_stride_b; p.ysb = a->y_stride_b;
  p.batch = (int)a->batch; p.dim = (int)a->dim; p.nstate = (int)a->dstate; p.softplus = a->dt_softplus != 0;
  p.vec = aligned16(a->ssm_state) && aligned16(a->A) && a->dstate == 16;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid((p.dim + 127) / 128, p.batch);
  // the NM = 16 instantiation handles any dstate through its scalar branch when not vectorisable
  if (a->dtype == MM_F32) step::ssm_step_kernel<float, 16><<<grid, 128, 0, s>>>(p);
  else if (a->dtype == MM_F16) step::ssm_step_kernel<__half, 16><<<grid, 128, 0, s>>>(p);
  else step::ssm_step_kernel<__nv_bfloat16, 16><<<grid, 128, 0, s>>>(p);
  return cudaGetLastError() == cudaSuccess ? MM_OK : MM_ERR_LAUNCH;
}

extern "C" int mm_add_rmsnorm(const MMAddNormArgs* a, mm_stream_t stream) {
  if (!a) return MM_ERR_ARG;
  if (dtype_size(a->dtype) == 0) return MM_ERR_DTYPE;
  if (a->rows < 0 || a->dim < 1 || a->dim > 32 * 256) return MM_ERR_SHAPE;
  if (a->rows > (1LL << 31) - 1) return MM_ERR_SHAPE;
  if (a->rows == 0) return MM_OK;
  if (!a->residual || !a->weight || !a->out) return MM_ERR_ARG;
  step::NormParams p;
  p.res = a->residual; p.delta = a->delta; p.w = a->weight; p.out = a->out;
  p.dsr = a->delta_stride_r; p.osr = a->out_stride_r; p.rows = (int)a->rows; p.dim = (int)a->dim;
  p.eps = (float)a->eps;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (a->dtype == MM_F32) e = step::launch_norm<float>(p, s);
  else if (a->dtype == MM_F16) e = step::launch_norm<__half>(p, s);
  else e = step::launch_norm<__nv_bfloat16>(p, s);
  return e == cudaSuccess ? MM_OK : MM_ERR_LAUNCH;
}

extern "C" const char* mm_version(void) { return "mamba_b200 0.1 (sm_100a)"; }
