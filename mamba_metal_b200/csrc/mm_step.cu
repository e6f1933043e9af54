// One-token SSM decode step and the fused residual-add + RMSNorm, for sm_100a.
//
// mm_ssm_decode_step restates mamba_metal/mamba_block.py:183-195: dt = softplus(dt_proj(.)),
// h = exp(dt*A)*h + (dt*x)*B, y = sum_n h*C + D*x, y *= silu(z). The step is bound by the fp32 state
// traffic (64 bytes read and written per (batch, channel) at dstate 16). Main kernel (dstate 16, aligned
// rows): four threads per channel, 16-byte state pieces contiguous across a warp, state and per-row
// scalars staged by cp.async in two row groups. Other shapes: one thread per (batch, channel) with its
// dstate states in registers.
//
// mm_add_rmsnorm restates the pre-norm residual wrapper of mamba_metal/mamba_model.py:49-58 with
// nn.RMSNorm (x * rsqrt(mean(x^2) + eps) * weight, eps from :32): residual += delta, then normalise.
#include <type_traits>

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
  // fused dt projection (dt_w != null): dt[b,d] = sum_k dt_in[b,k] * dt_w[d,k] + dt_bias[d], in fp32
  const void* dt_in;
  const void* dt_w;
  const float* dt_bias;
  long long xsb, dtsb, zsb, Bsb, Csb, ysb, dtin_sb, dtw_s;
  int batch, dim, nstate, dt_rank;
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
  float dr;
  if (p.dt_w) {
    const T* xi = static_cast<const T*>(p.dt_in) + b * p.dtin_sb;
    const T* wr = static_cast<const T*>(p.dt_w) + (long long)d * p.dtw_s;
    float acc = p.dt_bias ? p.dt_bias[d] : 0.f;
    for (int k = 0; k < p.dt_rank; ++k) acc = fmaf(ld_f32(xi + k), ld_f32(wr + k), acc);
    dr = acc;
  } else {
    dr = ld_f32(static_cast<const T*>(p.dt) + b * p.dtsb + d);
  }
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

// dstate 16, dim a multiple of 8, 16-byte aligned rows: CTA = 32 channels x kQdGroups groups of kQdRows
// batch rows, 128 threads; thread (dl, q) owns states 4q..4q+3 of channel d0 + dl, so a warp's
// 16-byte state accesses are contiguous. At entry the CTA starts cp.async copies of both groups' state
// rows (one commit group), then of each group's dt / x / z row slices (one commit group each; nothing held in
// registers), loads B | C with plain loads, then computes group 0 while group 1 is still in flight.
#ifndef MM_SSM_ROWS
#define MM_SSM_ROWS 2  // batch rows per group in the dstate-16 decode step. At the 2.8b decode shape (batch 64,
                       // 5120 channels, CUDA graph, states beyond L2) rows x groups measured: 2 x 2 8.7 us,
                       // 4 x 1 8.7, 1 x 4 9.2, 4 x 2 9.7, 8 x 1 9.7, 4 x 4 12.0 us
#endif
#ifndef MM_SSM_GROUPS
#define MM_SSM_GROUPS 2  // row groups per CTA (copies of later groups overlap earlier groups' compute)
#endif
constexpr int kQdCh = 32, kQdRows = MM_SSM_ROWS, kQdGroups = MM_SSM_GROUPS, kQdThreads = 128;
static_assert((kQdRows * kQdGroups) % (kQdThreads / 32) == 0, "B | C rows are staged four warps at a time");
// Fused dt projection in the dstate-16 kernel (16-bit types, dt_rank a multiple of 16, at most kDtMaxRank;
// other cases take the one-thread-per-channel kernel). The CTA's dt tile (its <= 8 batch rows x 32
// channels x dt_rank) is a tensor-core product: warp w computes the 8-channel column block that its own
// threads own with one m16n8k16 MMA per 16 of dt_rank (batch rows in the M dimension, dt_in rows as the A
// operand; dt_w rows -- K-contiguous, the "col" B layout -- as B), fp32 accumulation; each thread then
// takes its (row, channel) value from the accumulator fragment with a shuffle. The CTA's dt_w rows (a
// contiguous block of dt_proj.weight) arrive by coalesced cp.async with the state, before the wait on the
// preceding kernel; both operands sit in shared memory at a pitch of kDtPitch elements (84 words: the
// fragment reads of 8 rows x 4 words hit 32 distinct banks). At this size (<= 8 x 32 x 160 per CTA) a
// tcgen05 MMA would spend more on its tensor-memory allocation and commit than the whole product.
constexpr int kDtMaxRank = 160, kDtKSteps = kDtMaxRank / 16, kDtPitch = kDtMaxRank + 8;

template <typename T, bool FDT>
struct QuadSmem {
  float4 h[kQdGroups][kQdRows][kQdThreads];
  T dxz[kQdGroups][3][kQdRows][kQdCh];  // dt (unused with FDT), x, z row slices
  float bc[kQdGroups][kQdRows][32];
  __align__(16) T wdt[FDT ? kQdCh : 1][FDT ? kDtPitch : 16 / sizeof(T)];                   // dt_w rows
  __align__(16) T dtin[FDT ? kQdGroups * kQdRows : 1][FDT ? kDtPitch : 16 / sizeof(T)];  // dt_in rows
};

// D += A * B for one m16n8k16 tile, 16-bit inputs, fp32 accumulators (fragment layouts of the PTX ISA)
template <typename T>
MM_DEV void mma_16816(float (&c)[4], unsigned a0, unsigned a1, unsigned a2, unsigned a3, unsigned b0, unsigned b1) {
  if constexpr (std::is_same<T, __half>::value) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};\n"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};\n"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

template <typename T, bool FDT>
__global__ void __launch_bounds__(kQdThreads) ssm_step_quad_kernel(const SSMParams p) {
  __shared__ __align__(16) QuadSmem<T, FDT> sm;
  constexpr int VE = 16 / sizeof(T);
  constexpr int kChunks = kQdCh / VE;  // 16-byte chunks per row slice
  const int tid = threadIdx.x, dl = tid >> 2, q = tid & 3;
  const int d0 = blockIdx.x * kQdCh, d = d0 + dl;
  const bool dok = d < p.dim;
  // State rows first: with an early-state launch (programmatic dependent launch) they stream in while the
  // kernel before this one is still finishing; everything that kernel may have produced (dt, x, z, B, C,
  // dt_in) is read only after grid_dep_wait.
#pragma unroll
  for (int g = 0; g < kQdGroups; ++g) {
    const int b0 = ((int)blockIdx.y * kQdGroups + g) * kQdRows;
    const int nrows = max(0, min(kQdRows, p.batch - b0));
#pragma unroll
    for (int r = 0; r < kQdRows; ++r)
      if (dok && r < nrows)
        cp_async16(&sm.h[g][r][tid], p.state + ((long long)(b0 + r) * p.dim + d) * 16 + 4 * q);
  }
  // dt_proj's weights and bias are parameters, not outputs of the preceding kernel: loaded before the wait
  static_assert(!FDT || (kQdGroups * kQdRows <= 8 && sizeof(T) == 2), "fused dt: <= 8 rows, 16-bit types");
  const int ksteps = FDT ? p.dt_rank / 16 : 0;
  float dbias = 0.f;
  if (FDT) {
    const int dt_chunks = p.dt_rank / VE;  // 16-byte chunks per row
    for (int i = tid; i < kQdCh * dt_chunks; i += kQdThreads) {
      const int r = i / dt_chunks, c = i - r * dt_chunks;
      if (d0 + r < p.dim)
        cp_async16(&sm.wdt[r][c * VE], static_cast<const T*>(p.dt_w) + (long long)(d0 + r) * p.dtw_s + c * VE);
    }
    if (dok && p.dt_bias) dbias = __ldg(p.dt_bias + d);
  }
  cp_async_commit();
  grid_dep_wait();
  const int row0 = (int)blockIdx.y * kQdGroups * kQdRows;  // the CTA's first batch row
  const int rows_cta = max(0, min(kQdGroups * kQdRows, p.batch - row0));
  if (FDT) {  // dt_in rows of the whole CTA: their own commit group, ahead of the x / z slices
    const int dt_chunks = p.dt_rank / VE;
    for (int i = tid; i < rows_cta * dt_chunks; i += kQdThreads) {
      const int r = i / dt_chunks, c = i - r * dt_chunks;
      cp_async16(&sm.dtin[r][c * VE], static_cast<const T*>(p.dt_in) + (long long)(row0 + r) * p.dtin_sb + c * VE);
    }
    cp_async_commit();
  }
  const float4 a = dok ? *reinterpret_cast<const float4*>(p.A + (long long)d * 16 + 4 * q) : make_float4(0, 0, 0, 0);
  const float Dd = (dok && p.D) ? p.D[d] : 0.f;
#pragma unroll
  for (int g = 0; g < kQdGroups; ++g) {
    const int b0 = ((int)blockIdx.y * kQdGroups + g) * kQdRows;
    const int nrows = max(0, min(kQdRows, p.batch - b0));
    for (int i = FDT ? tid + kQdRows * kChunks : tid; i < 3 * kQdRows * kChunks; i += kQdThreads) {
      const int a = i / (kQdRows * kChunks), rem = i - a * kQdRows * kChunks;
      const int r = rem / kChunks, c = (rem - r * kChunks) * VE;
      const T* src = static_cast<const T*>(a == 0 ? p.dt : a == 1 ? p.x : p.z);
      const long long st = a == 0 ? p.dtsb : a == 1 ? p.xsb : p.zsb;
      if (r < nrows && d0 + c < p.dim && src) cp_async16(&sm.dxz[g][a][r][c], src + (long long)(b0 + r) * st + d0 + c);
    }
    cp_async_commit();
  }
  // B | C rows of both groups: row (g, r) by warp (g*8 + r) % 4 ... four warps, sixteen rows
#pragma unroll
  for (int j = 0; j < kQdGroups * kQdRows / 4; ++j) {
    const int gr = j * 4 + (tid >> 5), g = gr / kQdRows, r = gr - g * kQdRows, lane = tid & 31;
    const int b = ((int)blockIdx.y * kQdGroups + g) * kQdRows + r;
    float v = 0.f;
    if (b < p.batch)
      v = lane < 16 ? ld_f32(static_cast<const T*>(p.B) + (long long)b * p.Bsb + lane)
                    : ld_f32(static_cast<const T*>(p.C) + (long long)b * p.Csb + (lane - 16));
    sm.bc[g][r][lane] = v;
  }
  // fused dt: the MMA's accumulator fragment (batch rows lane / 4, channels 2 * (lane % 4) + {0, 1})
  float dacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int g = 0; g < kQdGroups; ++g) {
    if (g == 0) cp_async_wait<kQdGroups - 1>();  // the state group, dt_in rows and group 0's row slices
    else cp_async_wait<0>();
    __syncthreads();
    if (FDT && g == 0) {
      // A fragments: batch row lane / 4 (rows 8..15 of the tile are empty); B fragments: this warp's channel
      // lane / 4 (this thread's own); k = 16 * ks + 2 * (lane % 4) + {0, 1}, and + 8
      const int lane = tid & 31, row = lane >> 2;
      const T* wrow = &sm.wdt[(tid >> 5) * 8 + row][2 * q];
      const T* arow = &sm.dtin[row][2 * q];
#pragma unroll
      for (int ks = 0; ks < kDtKSteps; ++ks) {
        if (ks < ksteps) {
          unsigned a0 = 0u, a2 = 0u;
          if (row < rows_cta) {
            a0 = *reinterpret_cast<const unsigned*>(arow + 16 * ks);
            a2 = *reinterpret_cast<const unsigned*>(arow + 16 * ks + 8);
          }
          const unsigned b0 = *reinterpret_cast<const unsigned*>(wrow + 16 * ks);
          const unsigned b1 = *reinterpret_cast<const unsigned*>(wrow + 16 * ks + 8);
          mma_16816<T>(dacc, a0, 0u, a2, 0u, b0, b1);
        }
      }
    }
    const int b0 = ((int)blockIdx.y * kQdGroups + g) * kQdRows;
    const int nrows = max(0, min(kQdRows, p.batch - b0));
    if (!dok) continue;  // whole warps only (dim % 8 == 0, 8 channels per warp); no barrier follows
#pragma unroll
    for (int r = 0; r < kQdRows; ++r) {
      if (r >= nrows) continue;  // uniform over the CTA
      const long long b = b0 + r;
      float dtv;
      if (FDT) {
        // (row g * kQdRows + r, this warp's channel lane / 4) sits in lane 4 * row + (lane / 4) / 2
        const int lane = tid & 31, src = 4 * (g * kQdRows + r) + (lane >> 3);
        const float v0 = __shfl_sync(0xffffffffu, dacc[0], src), v1 = __shfl_sync(0xffffffffu, dacc[1], src);
        dtv = ((lane >> 2) & 1 ? v1 : v0) + dbias;
      } else {
        dtv = ElemTraits<T>::to_f32(sm.dxz[g][0][r][dl]);
      }
      const float xv = ElemTraits<T>::to_f32(sm.dxz[g][1][r][dl]);
      const float d2 = p.softplus ? softplus_log2(dtv) : dtv * kLog2e;
      const float du = d2 * kLn2 * xv;
      const float4 Bv = *reinterpret_cast<const float4*>(&sm.bc[g][r][4 * q]);
      const float4 Cv = *reinterpret_cast<const float4*>(&sm.bc[g][r][16 + 4 * q]);
      const float4 h = sm.h[g][r][tid];
      const f2_t dd = f2_pack(d2, d2), uu = f2_pack(du, du);
      const float2 e01 = f2_unpack(f2_mul(dd, f2_pack(a.x, a.y))), e23 = f2_unpack(f2_mul(dd, f2_pack(a.z, a.w)));
      const f2_t h01 = f2_fma(f2_pack(ex2(e01.x), ex2(e01.y)), f2_pack(h.x, h.y), f2_mul(uu, f2_pack(Bv.x, Bv.y)));
      const f2_t h23 = f2_fma(f2_pack(ex2(e23.x), ex2(e23.y)), f2_pack(h.z, h.w), f2_mul(uu, f2_pack(Bv.z, Bv.w)));
      const float2 n01 = f2_unpack(h01), n23 = f2_unpack(h23);
      *reinterpret_cast<float4*>(p.state + (b * p.dim + d) * 16 + 4 * q) = make_float4(n01.x, n01.y, n23.x, n23.y);
      const float2 yy = f2_unpack(f2_fma(h23, f2_pack(Cv.z, Cv.w), f2_mul(h01, f2_pack(Cv.x, Cv.y))));
      float y = yy.x + yy.y;
      y += __shfl_xor_sync(0xffffffffu, y, 1);
      y += __shfl_xor_sync(0xffffffffu, y, 2);
      if (q == 0) {
        y = fmaf(Dd, xv, y);
        if (p.z) y *= silu(ElemTraits<T>::to_f32(sm.dxz[g][2][r][dl]));
        st_f32(static_cast<T*>(p.y) + b * p.ysb + d, y);
      }
    }
  }
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
  // the weights are loaded with the row, so that no load follows the block reduction
  float4 wa = make_float4(0.f, 0.f, 0.f, 0.f), wb = wa;
  if (VEC && c0 + kNormE <= p.dim) {
    wa = *reinterpret_cast<const float4*>(p.w + c0);
    wb = *reinterpret_cast<const float4*>(p.w + c0 + 4);
  }
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

static cudaError_t launch_ssm_quad(int64_t dtype, bool fdt, const dim3& grid, cudaStream_t s, int64_t early,
                                   const step::SSMParams& p) {
  const int nt = step::kQdThreads;
  if (fdt)  // 16-bit types only (tensor-core dt tile)
    return dtype == MM_F16 ? launch_maybe_early(step::ssm_step_quad_kernel<__half, true>, grid, nt, s, early, p)
                           : launch_maybe_early(step::ssm_step_quad_kernel<__nv_bfloat16, true>, grid, nt, s, early, p);
  if (dtype == MM_F32) return launch_maybe_early(step::ssm_step_quad_kernel<float, false>, grid, nt, s, early, p);
  if (dtype == MM_F16) return launch_maybe_early(step::ssm_step_quad_kernel<__half, false>, grid, nt, s, early, p);
  return launch_maybe_early(step::ssm_step_quad_kernel<__nv_bfloat16, false>, grid, nt, s, early, p);
}

extern "C" int mm_ssm_decode_step(const MMSSMStepArgs* a, mm_stream_t stream) {
  if (!a) return MM_ERR_ARG;
  if (dtype_size(a->dtype) == 0) return MM_ERR_DTYPE;
  if (a->batch < 0 || a->dim < 0 || a->dstate < 1 || a->dstate > MM_MAX_DSTATE) return MM_ERR_SHAPE;
  if (a->batch > 65535 || a->dim > (1 << 30)) return MM_ERR_SHAPE;
  const bool fdt = a->dt_w != nullptr;
  if (fdt && (a->dt_rank < 1 || a->dt_rank > (1 << 20))) return MM_ERR_SHAPE;
  if (a->batch == 0 || a->dim == 0) return MM_OK;
  if (!a->x || !a->B || !a->C || !a->A || !a->ssm_state || !a->y) return MM_ERR_ARG;
  if (fdt ? !a->dt_in : !a->dt) return MM_ERR_ARG;
  step::SSMParams p;
  p.x = a->x; p.dt = fdt ? nullptr : a->dt; p.z = a->z; p.B = a->B; p.C = a->C; p.A = a->A; p.D = a->D;
  p.state = a->ssm_state; p.y = a->y;
  p.dt_in = fdt ? a->dt_in : nullptr; p.dt_w = a->dt_w; p.dt_bias = fdt ? a->dt_bias : nullptr;
  p.xsb = a->x_stride_b; p.dtsb = a->dt_stride_b; p.zsb = a->z_stride_b; p.Bsb = a->B_stride_b;
  p.Csb = a->C_stride_b; p.ysb = a->y_stride_b; p.dtin_sb = a->dt_in_stride_b; p.dtw_s = a->dt_w_stride;
  p.batch = (int)a->batch; p.dim = (int)a->dim; p.nstate = (int)a->dstate; p.softplus = a->dt_softplus != 0;
  p.dt_rank = fdt ? (int)a->dt_rank : 0;
  p.vec = aligned16(a->ssm_state) && aligned16(a->A) && a->dstate == 16;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t es = (int64_t)dtype_size(a->dtype);
  const bool rows16 = aligned16(a->x) && (!a->z || aligned16(a->z)) && (a->x_stride_b * es) % 16 == 0 &&
                      (!a->z || (a->z_stride_b * es) % 16 == 0) &&
                      (fdt || (aligned16(a->dt) && (a->dt_stride_b * es) % 16 == 0));
  // fused dt in the dstate-16 kernel: 16-bit types, dt_rank a multiple of 16 up to kDtMaxRank, aligned rows
  const bool dt16 = !fdt || (es == 2 && a->dt_rank % 16 == 0 && a->dt_rank <= step::kDtMaxRank &&
                             aligned16(a->dt_in) && aligned16(a->dt_w) && (a->dt_in_stride_b * es) % 16 == 0 &&
                             (a->dt_w_stride * es) % 16 == 0);
  if (p.vec && p.dim % 8 == 0 && rows16 && dt16) {
    const int rows_per_cta = step::kQdRows * step::kQdGroups;
    const dim3 qgrid((p.dim + step::kQdCh - 1) / step::kQdCh, (p.batch + rows_per_cta - 1) / rows_per_cta);
    const cudaError_t e = launch_ssm_quad(a->dtype, fdt, qgrid, s, a->early_state, p);
    return e == cudaSuccess ? MM_OK : MM_ERR_LAUNCH;
  }
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
