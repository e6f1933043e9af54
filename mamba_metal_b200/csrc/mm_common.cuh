// Shared device helpers for the sm_100a kernels of libmamba_b200.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mamba_b200.h"

#define MM_DEV __device__ __forceinline__

namespace mm {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// ---- MUFU approximations (hardware ex2/lg2/rcp; relative error ~2^-22) ------------------------
MM_DEV float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
MM_DEV float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
MM_DEV float rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---- Packed fp32 pairs (Blackwell f32x2 ALU ops: one issue slot for two lanes of math) ---------
// With MM_F2_SCALAR defined the same helpers are plain scalar C++ (two independent float operations),
// leaving instruction selection and scheduling entirely to the compiler.
#ifdef MM_F2_SCALAR
struct f2_t {
  float x, y;
};
MM_DEV f2_t f2_pack(float lo, float hi) { return f2_t{lo, hi}; }
MM_DEV float2 f2_unpack(f2_t v) { return make_float2(v.x, v.y); }
MM_DEV f2_t f2_fma(f2_t a, f2_t b, f2_t c) { return f2_t{fmaf(a.x, b.x, c.x), fmaf(a.y, b.y, c.y)}; }
MM_DEV f2_t f2_mul(f2_t a, f2_t b) { return f2_t{a.x * b.x, a.y * b.y}; }
MM_DEV f2_t f2_add(f2_t a, f2_t b) { return f2_t{a.x + b.x, a.y + b.y}; }
MM_DEV f2_t f2_sub(f2_t a, f2_t b) { return f2_t{a.x - b.x, a.y - b.y}; }
#else
typedef unsigned long long f2_t;

MM_DEV f2_t f2_pack(float lo, float hi) {
  f2_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
MM_DEV float2 f2_unpack(f2_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
MM_DEV f2_t f2_fma(f2_t a, f2_t b, f2_t c) {
  f2_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
MM_DEV f2_t f2_mul(f2_t a, f2_t b) {
  f2_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
MM_DEV f2_t f2_add(f2_t a, f2_t b) {
  f2_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
MM_DEV f2_t f2_sub(f2_t a, f2_t b) {
  f2_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
#endif

// ---- 2^x on the FMA pipe, for a pair of arguments ----------------------------------------------
// Cody-Waite style range reduction x = j + f with j = rint(x) and |f| <= 1/2 (j from the "add 1.5 * 2^23"
// rounding trick: the low bits of t = x + 1.5 * 2^23 hold j, and (t - 1.5 * 2^23) is j exactly), then
// 2^f from a degree-5 polynomial whose coefficients are the minimax (Remez exchange, relative error) fit
// of 2^f on [-1/2, 1/2], rounded to float (csrc/exp2_poly.py reproduces them), and 2^j applied by adding
// j to the exponent field. Relative error below 2.2e-7 (1.8 ulp) for x in [-125, 126]; arguments are
// clamped to that range (2^-125 stands in for smaller results). Used to move part of the scan's
// exponentials off the MUFU pipe, which runs at an eighth of the FMA pipe's rate.
MM_DEV f2_t exp2_poly2(f2_t x2) {
  const float2 xs = f2_unpack(x2);
  const f2_t x = f2_pack(fminf(fmaxf(xs.x, -125.0f), 126.0f), fminf(fmaxf(xs.y, -125.0f), 126.0f));
  const float kShift = 12582912.0f;  // 1.5 * 2^23
  const f2_t t = f2_add(x, f2_pack(kShift, kShift));
  const f2_t f = f2_sub(x, f2_sub(t, f2_pack(kShift, kShift)));
  f2_t p = f2_pack(1.3276472e-3f, 1.3276472e-3f);
  p = f2_fma(p, f, f2_pack(9.6755410e-3f, 9.6755410e-3f));
  p = f2_fma(p, f, f2_pack(5.5507131e-2f, 5.5507131e-2f));
  p = f2_fma(p, f, f2_pack(2.4022120e-1f, 2.4022120e-1f));
  p = f2_fma(p, f, f2_pack(6.9314694e-1f, 6.9314694e-1f));
  p = f2_fma(p, f, f2_pack(1.0000001f, 1.0000001f));
  const float2 ts = f2_unpack(t);
  const float2 ps = f2_unpack(p);
  return f2_pack(__int_as_float(__float_as_int(ps.x) + (__float_as_int(ts.x) << 23)),
                 __int_as_float(__float_as_int(ps.y) + (__float_as_int(ts.y) << 23)));
}

// ---- Softplus in the log2 domain --------------------------------------------------------------
// Returns softplus(x) * log2(e) = log2(1 + e) with e = 2^(x*log2e), and the reference's cutoff
// (mamba_metal/kernels/selective_scan_chunked.metal:60-65: x > 20 -> x). For e < 2^-6, 1 + e would lose
// e's low bits, so log2(1 + e) comes from the series e*log2e*(1 - e/2 + e^2/3) instead (relative error
// below 1e-6 there); above it the MUFU lg2 of 1 + e is within ~4e-6 relative.
MM_DEV float softplus_log2(float x) {
  const float y = x * kLog2e;
  const float e = ex2(y);
  const float l = lg2(1.0f + e);
  const float ser = e * kLog2e * fmaf(e, fmaf(e, 0.33333334f, -0.5f), 1.0f);
  const float r = (e < 0.015625f) ? ser : l;
  return (x <= 20.0f) ? r : y;
}

// softplus_log2 of a pair of arguments, with the float arithmetic in packed f32x2 operations.
MM_DEV f2_t softplus_log2_2(f2_t x2) {
  const f2_t y = f2_mul(x2, f2_pack(kLog2e, kLog2e));
  const float2 ys = f2_unpack(y);
  const f2_t e = f2_pack(ex2(ys.x), ex2(ys.y));
  const float2 ope = f2_unpack(f2_add(e, f2_pack(1.0f, 1.0f)));
  const f2_t ser = f2_mul(f2_mul(e, f2_pack(kLog2e, kLog2e)),
                          f2_fma(e, f2_fma(e, f2_pack(0.33333334f, 0.33333334f), f2_pack(-0.5f, -0.5f)),
                                 f2_pack(1.0f, 1.0f)));
  const float2 es = f2_unpack(e), ss = f2_unpack(ser), xs = f2_unpack(x2);
  const float r0 = (es.x < 0.015625f) ? ss.x : lg2(ope.x);
  const float r1 = (es.y < 0.015625f) ? ss.y : lg2(ope.y);
  return f2_pack((xs.x <= 20.0f) ? r0 : ys.x, (xs.y <= 20.0f) ? r1 : ys.y);
}

// SiLU(z) = z / (1 + exp(-z)) (reference formula, selective_scan_chunked.metal:141-144).
MM_DEV float silu(float z) { return z * rcp(1.0f + ex2(-z * kLog2e)); }

// ---- Element types ------------------------------------------------------------------------------
template <typename T> struct ElemTraits;
template <> struct ElemTraits<float> {
  MM_DEV static float to_f32(float v) { return v; }
  MM_DEV static float from_f32(float v) { return v; }
};
template <> struct ElemTraits<__half> {
  MM_DEV static float to_f32(__half v) { return __half2float(v); }
  MM_DEV static __half from_f32(float v) { return __float2half_rn(v); }
};
template <> struct ElemTraits<__nv_bfloat16> {
  MM_DEV static float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
  MM_DEV static __nv_bfloat16 from_f32(float v) { return __float2bfloat16_rn(v); }
};

template <typename T> MM_DEV float ld_f32(const T* p) { return ElemTraits<T>::to_f32(*p); }
template <typename T> MM_DEV void st_f32(T* p, float v) { *p = ElemTraits<T>::from_f32(v); }

// Elements of a 16-byte register block holding 16/sizeof(T) values of T, handled in pairs so that
// 16-bit types convert with one paired instruction. Indices must be compile-time constants after
// unrolling; the block is never addressed through memory, so it stays in registers.
MM_DEV unsigned u4_word(const uint4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }
MM_DEV void u4_set_word(uint4& v, int i, unsigned w) {
  if (i == 0) v.x = w;
  else if (i == 1) v.y = w;
  else if (i == 2) v.z = w;
  else v.w = w;
}
// pair i = elements (2i, 2i+1)
template <typename T> MM_DEV float2 vec_pair(const uint4& v, int i);
template <> MM_DEV float2 vec_pair<float>(const uint4& v, int i) {
  return make_float2(__uint_as_float(u4_word(v, 2 * i)), __uint_as_float(u4_word(v, 2 * i + 1)));
}
template <> MM_DEV float2 vec_pair<__half>(const uint4& v, int i) {
  const unsigned w = u4_word(v, i);
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}
template <> MM_DEV float2 vec_pair<__nv_bfloat16>(const uint4& v, int i) {
  const unsigned w = u4_word(v, i);
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <typename T> MM_DEV void vec_set_pair(uint4& v, int i, float a, float b);
template <> MM_DEV void vec_set_pair<float>(uint4& v, int i, float a, float b) {
  u4_set_word(v, 2 * i, __float_as_uint(a));
  u4_set_word(v, 2 * i + 1, __float_as_uint(b));
}
template <> MM_DEV void vec_set_pair<__half>(uint4& v, int i, float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  u4_set_word(v, i, *reinterpret_cast<const unsigned*>(&h));
}
template <> MM_DEV void vec_set_pair<__nv_bfloat16>(uint4& v, int i, float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  u4_set_word(v, i, *reinterpret_cast<const unsigned*>(&h));
}
template <typename T> MM_DEV float vec_elem(const uint4& v, int k) {
  const float2 p = vec_pair<T>(v, k >> 1);
  return (k & 1) ? p.y : p.x;
}
template <typename T> MM_DEV void vec_set(uint4& v, int k, float x);
template <> MM_DEV void vec_set<float>(uint4& v, int k, float x) { u4_set_word(v, k, __float_as_uint(x)); }
template <> MM_DEV void vec_set<__half>(uint4& v, int k, float x) {
  const unsigned h = __half_as_ushort(__float2half_rn(x));
  const unsigned w = u4_word(v, k >> 1);
  u4_set_word(v, k >> 1, (k & 1) ? ((w & 0xffffu) | (h << 16)) : ((w & 0xffff0000u) | h));
}
template <> MM_DEV void vec_set<__nv_bfloat16>(uint4& v, int k, float x) {
  const unsigned h = __bfloat16_as_ushort(__float2bfloat16_rn(x));
  const unsigned w = u4_word(v, k >> 1);
  u4_set_word(v, k >> 1, (k & 1) ? ((w & 0xffffu) | (h << 16)) : ((w & 0xffff0000u) | h));
}

// ---- cp.async (LDGSTS) staging --------------------------------------------------------------------
MM_DEV unsigned smem_u32(const void* p) { return static_cast<unsigned>(__cvta_generic_to_shared(p)); }
MM_DEV void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
MM_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> MM_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// ---- TMA tile loads and mbarriers (no cluster multicast anywhere) --------------------------------
MM_DEV void mbar_init(unsigned long long* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// makes barrier initialisation visible to the async proxy (TMA) before first use
MM_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
MM_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
MM_DEV void mbar_arrive_expect_tx(unsigned long long* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
MM_DEV bool mbar_try_wait_parity(unsigned long long* bar, unsigned parity) {
  unsigned done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
MM_DEV unsigned long long globaltimer_ns();
// Waits for the barrier phase with the given parity; gives up (returns false) after limit_ns.
MM_DEV bool mbar_wait_parity_bounded(unsigned long long* bar, unsigned parity, unsigned long long limit_ns) {
  if (mbar_try_wait_parity(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait_parity(bar, parity)) {
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
  return true;
}
// 3-D tiled TMA load (coordinates in elements, innermost first) into shared memory, completing on bar.
MM_DEV void tma_load_3d(void* smem_dst, const CUtensorMap* tm, int x, int y, int z, unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(smem_u32(smem_dst)), "l"(tm), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// ---- Programmatic dependent launch -------------------------------------------------------------
// Waits until the grid this launch depends on (the previous kernel in the stream, when launched with
// programmatic stream serialization) has completed and its memory is visible; a no-op otherwise.
MM_DEV void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the dependent launch of this grid start its own prologue.
MM_DEV void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- Memory-model helpers for carry hand-off ----------------------------------------------------
MM_DEV unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
MM_DEV unsigned ld_relaxed(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
MM_DEV void fence_acq_rel() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
MM_DEV void st_release(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
MM_DEV unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Launches kernel<<<grid, block, 0, s>>>(params); with early != 0 as a programmatic dependent launch (the
// kernel may start while the previous kernel in the stream finishes; it calls grid_dep_wait before
// reading anything that kernel produced).
template <typename K, typename P>
inline cudaError_t launch_maybe_early(K kernel, dim3 grid, dim3 block, cudaStream_t s, int64_t early, const P& params) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = early ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, params);
}

inline int dtype_size(int64_t dtype) {
  return dtype == MM_F32 ? 4 : (dtype == MM_F16 || dtype == MM_BF16) ? 2 : 0;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace mm
