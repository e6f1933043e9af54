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

// One CTA per row, ceil(dim / 8) threads, 8 consecutive elements per thread: the residual (fp32, two
// 16-byte loads) and the delta (one 16-byte load for 16-bit types) are all in flight before the single
// block reduction; the row stays in registers for the scaling pass.
constexpr int kNormE = 8;

template <typename T, bool VEC>
__global__ void __launch_bounds__(1024) add_rmsnorm_kernel(const NormParams p) {
  const int r = blockIdx.x;
  float* res = p.res + (long long)r * p.dim;
  const T* dl = p.delta ? static_cast<const T*>(p.delta) + (long long)r * p.dsr : nullptr;
  const int c0 = threadIdx.x * kNormE;
  float v[kNormE];
  if (VEC && c0 + kNormE <= p.dim) {
    const float4 a = *reinterpret_cast<const float4*>(res + c0);
    const float4 b = *reinterpret_cast<const float4*>(res + c0 + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    if (dl) {
      float d8[kNormE];
      if (sizeof(T) == 2) {
        const uint4 q = *reinterpret_cast<const uint4*>(dl + c0);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 e = vec_pair<T>(q, k);
          d8[2 * k] = e.x;
          d8[2 * k + 1] = e.y;
        }
      } else {
#pragma unroll
        for (int k = 0; k < kNormE; ++k) d8[k] = ld_f32(dl + c0 + k);
      }
#pragma unroll
      for (int k = 0; k < kNormE; ++k) v[k] += d8[k];
      *reinterpret_cast<float4*>(res + c0) = make_float4(v[0], v[1], v[2], v[3]);
      *reinterpret_cast<float4*>(res + c0 + 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
  } else {
#pragma unroll
    for (int k = 0; k < kNormE; ++k) {
      const int c = c0 + k;
      float x = 0.f;
      if (c < p.dim) {
        x = res[c];
        if (dl) {
          x += ld_f32(dl + c);
          res[c] = x;
        }
      }
      v[k] = x;
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kNormE; ++k) ss = fmaf(v[k], v[k], ss);
  __shared__ float red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const int nw = (blockDim.x + 31) >> 5;
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < nw ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)p.dim + p.eps);
  T* out = static_cast<T*>(p.out) + (long long)r * p.osr;
  if (VEC && c0 + kNormE <= p.dim) {
    const float4 wa = *reinterpret_cast<const float4*>(p.w + c0);
    const float4 wb = *reinterpret_cast<const float4*>(p.w + c0 + 4);
    const float w8[kNormE] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
    if (sizeof(T) == 2) {
      uint4 q;
#pragma unroll
      for (int k = 0; k < 4; ++k) vec_set_pair<T>(q, k, v[2 * k] * inv * w8[2 * k], v[2 * k + 1] * inv * w8[2 * k + 1]);
      *reinterpret_cast<uint4*>(out + c0) = q;
    } else {
#pragma unroll
      for (int k = 0; k < kNormE; ++k) st_f32(out + c0 + k, v[k] * inv * w8[k]);
    }
  } else {
#pragma unroll
    for (int k = 0; k < kNormE; ++k) {
      const int c = c0 + k;
      if (c < p.dim) st_f32(out + c, v[k] * inv * p.w[c]);
    }
  }
}

template <typename T>
static cudaError_t launch_norm(const NormParams& p, bool vec, cudaStream_t s) {
  const int threads = ((p.dim + kNormE - 1) / kNormE + 31) / 32 * 32;
  if (threads > 1024) return cudaErrorInvalidValue;
  if (vec) add_rmsnorm_kernel<T, true><<<p.rows, threads, 0, s>>>(p);
  else add_rmsnorm_kernel<T, false><<<p.rows, threads, 0, s>>>(p);
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
  if (a->rows < 0 || a->dim < 1 || a->dim > 1024 * 8) return MM_ERR_SHAPE;
  if (a->rows > (1LL << 31) - 1) return MM_ERR_SHAPE;
  if (a->rows == 0) return MM_OK;
  if (!a->residual || !a->weight || !a->out) return MM_ERR_ARG;
  step::NormParams p;
  p.res = a->residual; p.delta = a->delta; p.w = a->weight; p.out = a->out;
  p.dsr = a->delta_stride_r; p.osr = a->out_stride_r; p.rows = (int)a->rows; p.dim = (int)a->dim;
  p.eps = (float)a->eps;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // 16-byte vectors when every row start is aligned (dim, row strides multiples of 8 elements)
  const bool vec = a->dim % 8 == 0 && aligned16(a->residual) && aligned16(a->weight) && aligned16(a->out) &&
                   a->out_stride_r % 8 == 0 && (!a->delta || (aligned16(a->delta) && a->delta_stride_r % 8 == 0));
  cudaError_t e;
  if (a->dtype == MM_F32) e = step::launch_norm<float>(p, vec, s);
  else if (a->dtype == MM_F16) e = step::launch_norm<__half>(p, vec, s);
  else e = step::launch_norm<__nv_bfloat16>(p, vec, s);
  return e == cudaSuccess ? MM_OK : MM_ERR_LAUNCH;
}

extern "C" const char* mm_version(void) { return "mamba_b200 0.1 (sm_100a)"; }
