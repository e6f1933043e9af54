// Dense projections of the decode step (in_proj, x_proj, dt_proj, out_proj) for sm_100a: a tcgen05 GEMM
// shaped for a small batch of tokens against a large weight.
//
// The decode step of mamba_metal/mamba_block.py:155-198 multiplies a (batch, K) activation by four weight
// matrices (nn.Linear, y = x @ W^T). At batch 64 these products read every weight byte once and are bound
// by HBM bandwidth, so the kernel is built around streaming W:
//   - the tile is swapped: the MMA's M side is 128 output features (rows of W), its N side the batch
//     (64 tokens), so one tcgen05.mma.cta_group::1.kind::f16 (M 128, N 64, K 16, bf16 in, fp32 out)
//     consumes a 128 x 16 slab of W and the whole batch;
//   - W and x tiles arrive by TMA (128-byte swizzled rows, no multicast) into a 4-stage ring (96 KB, two
//     CTAs per SM, at most one wave of CTAs); one elected thread issues the TMA copies, another the MMAs;
//     accumulators live in TMEM (64 columns);
//   - the K range is split over CTAs so that every SM streams weight bytes even when N / 128 is small
//     (out_proj: 2560 / 128 = 20 tiles); each split adds its partial into an fp32 tile of the workspace
//     with vector reductions (red.global.add.v4.f32), and the last CTA of the tile to arrive (a per-tile
//     counter) reads the sum once, adds the bias, writes fp32 or bf16 and zeroes the tile again. The order
//     of the fp32 additions follows arrival, so split results can differ in the last bits between calls;
//   - the launch is a programmatic dependent launch: a CTA initialises its barriers and TMEM, prefetches
//     its tensor maps and starts the copies of its first weight stages (weights are constants of the
//     step) while the kernel before it in the stream is still finishing, and waits for that kernel
//     (griddepcontrol.wait) only before its first activation copy.
// Every mbarrier wait is bounded (1 s); a wait that runs out sets the error word of the workspace
// (read by mm_linear_status) and the CTA skips the rest of its work, frees its TMEM and returns.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>

#include "mm_common.cuh"

namespace mm {
namespace gemm {

constexpr int BM = 128;  // output features per CTA (MMA M)
constexpr int BN = 64;   // tokens per CTA (MMA N)
constexpr int BK = 64;   // K elements per stage: one 128-byte swizzle row of bf16
constexpr int kStages = 4;
constexpr int kThreads = 128;
constexpr unsigned long long kWaitLimitNs = 1000000000ull;
constexpr unsigned kTmemCols = 64;  // BN fp32 accumulator columns
constexpr int kMaxTiles = 4096;     // output tiles with a split counter (larger calls run unsplit)
constexpr int kMaxSplits = 16;
constexpr int kCtasPerSm = 2;      // resident CTAs per SM (shared memory: 4 stages x 24 KB)
// Instruction descriptor of tcgen05.mma kind::f16: D fp32 (bits 4-5 = 1), A and B bf16 (bits 7-9 and
// 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 at bits 17-22, M >> 4 at bits 24-28.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

struct Params {
  CUtensorMap tm_w;  // W: (N, K) bf16, box (BK, BM), 128-byte swizzle
  CUtensorMap tm_x;  // x: (M, K) bf16, box (BK, BN), 128-byte swizzle
  void* y;
  long long ldy;
  const float* bias;
  int y_f32;
  int M, N, K;
  int n_tiles, m_tiles, splits, kb_per_split, kb_total;
  float* partial;      // [m_tiles * n_tiles][BN / 4][BM][4] fp32 sums of the splits, zero between calls
  unsigned* counters;  // [m_tiles * n_tiles], zero between calls
  unsigned* err;
};

struct __align__(1024) Smem {
  uint8_t w[kStages][BM * BK * 2];  // 16 KB per stage, 1024-byte aligned (swizzle atom)
  uint8_t x[kStages][BN * BK * 2];  // 8 KB per stage
  unsigned long long full[kStages];
  unsigned long long empty[kStages];
  unsigned long long done;
  unsigned tmem_base;
  unsigned flag;  // 1: this CTA reduces its tile; 2: a wait ran out
};

MM_DEV void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y, unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(tm), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile written by TMA with 128-byte swizzling:
// start address >> 4 (bits 0-13), leading offset 1 (unused for swizzled K-major), stride offset between
// 8-row groups 1024 B >> 4 (bits 32-45), descriptor version 1 (bits 46-47), swizzle mode 2 = 128 B
// (bits 61-63). Advancing K by 16 bf16 elements inside the 128-byte row adds 32 B to the start address.
MM_DEV uint64_t sw128_desc(const void* p) {
  const uint32_t a = smem_u32(p);
  return (uint64_t)((a >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
         ((uint64_t)2 << 61);
}

// Adds tx bytes that the current phase of `bar` waits for, without arriving.
MM_DEV void mbar_expect_tx(unsigned long long* bar, unsigned bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// Waits for the phase of `bar` with the given parity: a short burst of polls, then polls bounded by time.
MM_DEV bool wait_phase(unsigned long long* bar, unsigned parity) {
#pragma unroll 1
  for (int i = 0; i < 64; ++i)
    if (mbar_try_wait_parity(bar, parity)) return true;
  return mbar_wait_parity_bounded(bar, parity, kWaitLimitNs);
}

MM_DEV void red_add_v4(float* p, float4 v) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

MM_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
MM_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

MM_DEV void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once every MMA this thread issued so far has completed.
MM_DEV void tc_commit(unsigned long long* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive fp32 columns: thread t of the warp receives row (lane base + t).
MM_DEV void tc_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
MM_DEV void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__global__ void __launch_bounds__(kThreads, kCtasPerSm) linear_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x, split = blockIdx.y, m_tile = blockIdx.z;
  const int kb0 = split * p.kb_per_split;
  const int nkb = min(kb0 + p.kb_per_split, p.kb_total) - kb0;  // >= 1 (the host sizes the split)

  if (threadIdx.x == 32) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(&p.tm_w) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&p.tm_x) : "memory");
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    mbar_init(&s.done, 1);
    s.flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == 0 && lane == 0) {
    // TMA producer. The weight copies of the first stages go out before the wait for the previous kernel
    // (weights do not depend on it); every activation copy comes after it. Stage i % kStages is free once
    // the MMAs of iteration i - kStages have completed.
    const int pre = min(nkb, kStages);
    for (int i = 0; i < pre; ++i) {
      mbar_expect_tx(&s.full[i], (unsigned)(BM * BK * 2));
      tma_load_2d(s.w[i], &p.tm_w, (kb0 + i) * BK, n_tile * BM, &s.full[i]);
    }
    grid_dep_wait();
    // Only now (the kernel before this one has completed) may the next kernel start its prologue: a
    // dependent that reads its own inputs early then never overtakes a kernel two launches back.
    grid_dep_launch();
    for (int i = 0; i < nkb; ++i) {
      const int st = i % kStages;
      if (i >= kStages && !wait_phase(&s.empty[st], ((i / kStages) & 1) ^ 1)) {
        atomicOr(p.err, 1u);
        s.flag = 2;
        break;
      }
      const int k = (kb0 + i) * BK;
      if (i >= pre) {
        mbar_arrive_expect_tx(&s.full[st], (unsigned)((BM + BN) * BK * 2));
        tma_load_2d(s.w[st], &p.tm_w, k, n_tile * BM, &s.full[st]);
      } else {
        mbar_arrive_expect_tx(&s.full[st], (unsigned)(BN * BK * 2));
      }
      tma_load_2d(s.x[st], &p.tm_x, k, m_tile * BN, &s.full[st]);
    }
  } else if (warp == 1 && lane == 0) {
    // MMA issuer: four K=16 MMAs per stage into the TMEM accumulator; each stage is released by a commit.
    bool ok = true;
    for (int i = 0; i < nkb; ++i) {
      const int st = i % kStages;
      if (!wait_phase(&s.full[st], (i / kStages) & 1)) {
        atomicOr(p.err, 2u);
        s.flag = 2;
        ok = false;
        break;
      }
      tc_fence_after();
      const uint64_t ad = sw128_desc(s.w[st]);
      const uint64_t bd = sw128_desc(s.x[st]);
#pragma unroll
      for (int k = 0; k < BK / 16; ++k) tc_mma(tmem, ad + 2 * k, bd + 2 * k, kIdesc, (i > 0 || k > 0) ? 1u : 0u);
      tc_commit(&s.empty[st]);
    }
    if (ok) tc_commit(&s.done);
  }
  __syncwarp();

  // Epilogue: thread (warp w, lane l) owns output feature n_tile * 128 + 32 w + l for the 64 tokens.
  const bool got = wait_phase(&s.done, 0);
  tc_fence_after();
  const int nl = warp * 32 + lane;
  const int n = n_tile * BM + nl;
  float acc[BN];
  if (got) {
#pragma unroll
    for (int c = 0; c < BN / 32; ++c) {
      float v[32];
      tc_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(c * 32), v);
      tc_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[c * 32 + i] = v[i];
    }
  } else {
    if (lane == 0) atomicOr(p.err, 4u);
#pragma unroll
    for (int i = 0; i < BN; ++i) acc[i] = 0.f;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
  if (!got || s.flag == 2) return;

  const int tile = m_tile * p.n_tiles + n_tile;
  if (p.splits > 1) {
    // Add this split's partial into the tile's fp32 sum ([BN / 4][BM][4]: a warp's 16-byte reductions are
    // contiguous), then count arrivals; the last CTA of the tile reads the sum, and zeroes it for the next call.
    float* sum = p.partial + (long long)tile * BM * BN;
#pragma unroll
    for (int q = 0; q < BN / 4; ++q)
      red_add_v4(sum + (q * BM + nl) * 4, make_float4(acc[4 * q], acc[4 * q + 1], acc[4 * q + 2], acc[4 * q + 3]));
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned prev = atomicAdd(p.counters + tile, 1u);
      s.flag = (prev == (unsigned)p.splits - 1) ? 1u : 0u;
    }
    __syncthreads();
    if (s.flag != 1) return;
    __threadfence();
    float4* s4 = reinterpret_cast<float4*>(sum);
#pragma unroll
    for (int q = 0; q < BN / 4; ++q) {
      const float4 v = __ldcg(s4 + q * BM + nl);
      acc[4 * q] = v.x;
      acc[4 * q + 1] = v.y;
      acc[4 * q + 2] = v.z;
      acc[4 * q + 3] = v.w;
    }
#pragma unroll
    for (int q = 0; q < BN / 4; ++q) __stcg(s4 + q * BM + nl, make_float4(0.f, 0.f, 0.f, 0.f));
    if (threadIdx.x == 0) p.counters[tile] = 0u;  // ready for the next call
  }
  if (n >= p.N) return;
  const float bv = p.bias ? p.bias[n] : 0.f;
  const int m0 = m_tile * BN;
  const int mcount = min(BN, p.M - m0);
  if (p.y_f32) {
    float* y = static_cast<float*>(p.y) + (long long)m0 * p.ldy + n;
#pragma unroll
    for (int i = 0; i < BN; ++i)
      if (i < mcount) y[(long long)i * p.ldy] = acc[i] + bv;
  } else {
    __nv_bfloat16* y = static_cast<__nv_bfloat16*>(p.y) + (long long)m0 * p.ldy + n;
#pragma unroll
    for (int i = 0; i < BN; ++i)
      if (i < mcount) y[(long long)i * p.ldy] = __float2bfloat16_rn(acc[i] + bv);
  }
}

// ---- host side ------------------------------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }();
  return fn;
}

// 2-D bf16 map of a (rows, K) row-major matrix with row stride ld elements, boxes of (BK, box_rows),
// 128-byte swizzle; elements outside (rows, K) read as zero.
static bool encode_rows(CUtensorMap* m, const void* base, long long rows, long long K, long long ld, int box_rows) {
  auto enc = encoder();
  if (!enc || !base || (reinterpret_cast<uintptr_t>(base) & 15u) || (ld * 2) % 16 != 0 || ld < K) return false;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct Plan {
  int n_tiles, m_tiles, kb_total, splits, kb_per_split;
  size_t ws_bytes, partial_off;
};

// SM count of the current device, cached per device in atomics: concurrent first calls may both query it,
// and both store the same value.
static int sm_count() {
  static std::atomic<int> cached[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int v = cached[dev].load(std::memory_order_relaxed);
  if (v > 0) return v;
  v = 148;
  cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
  cached[dev].store(v, std::memory_order_relaxed);
  return v;
}

static int make_plan(const MMLinearArgs* a, Plan* pl) {
  if (!a) return MM_ERR_ARG;
  if (a->M < 1 || a->N < 1 || a->K < 1) return MM_ERR_SHAPE;
  if (a->M > (1 << 24) || a->N > (1 << 24) || a->K > (1 << 24)) return MM_ERR_SHAPE;
  if (a->y_dtype != MM_F32 && a->y_dtype != MM_BF16) return MM_ERR_DTYPE;
  pl->n_tiles = (int)((a->N + BM - 1) / BM);
  pl->m_tiles = (int)((a->M + BN - 1) / BN);
  pl->kb_total = (int)((a->K + BK - 1) / BK);
  int splits = (int)a->splits;
  if (splits <= 0) {
    // one wave of CTAs (kCtasPerSm per SM), each streaming at least two K-blocks; at most kMaxSplits
    const int ctas = pl->n_tiles * pl->m_tiles;
    const int wave = kCtasPerSm * sm_count();
    splits = ctas >= wave ? 1 : std::min({wave / ctas, pl->kb_total / 2, kMaxSplits});
    splits = std::max(1, splits);
  }
  splits = std::min(splits, pl->kb_total);
  pl->kb_per_split = (pl->kb_total + splits - 1) / splits;
  pl->splits = (pl->kb_total + pl->kb_per_split - 1) / pl->kb_per_split;  // no empty split
  const size_t tiles = (size_t)pl->n_tiles * pl->m_tiles;
  if (tiles > (size_t)kMaxTiles) pl->splits = 1, pl->kb_per_split = pl->kb_total;  // no counter slot: no split
  // workspace: [err, pad] | counters[kMaxTiles] | partials. The counter region has a fixed size so that
  // calls of different shapes sharing one workspace never overlap one call's counters with another's
  // partials (the counters must stay zero between calls).
  size_t off = 256 + kMaxTiles * sizeof(unsigned);
  pl->partial_off = off;
  if (pl->splits > 1) off += tiles * BM * BN * sizeof(float);
  pl->ws_bytes = off;
  return MM_OK;
}

}  // namespace gemm
}  // namespace mm

using namespace mm;
using namespace mm::gemm;

extern "C" int mm_linear_workspace_size(const MMLinearArgs* a, size_t* bytes) {
  if (!bytes) return MM_ERR_ARG;
  Plan pl;
  const int rc = make_plan(a, &pl);
  if (rc != MM_OK) return rc;
  *bytes = pl.ws_bytes;
  return MM_OK;
}

extern "C" int mm_linear_fwd(const MMLinearArgs* a, void* ws, size_t ws_bytes, mm_stream_t stream) {
  Plan pl;
  const int rc = make_plan(a, &pl);
  if (rc != MM_OK) return rc;
  if (!a->x || !a->w || !a->y) return MM_ERR_ARG;
  if (!ws || ws_bytes < pl.ws_bytes || (reinterpret_cast<uintptr_t>(ws) & 255u)) return MM_ERR_WORKSPACE;
  Params p;
  if (!encode_rows(&p.tm_w, a->w, a->N, a->K, a->ldw, BM) || !encode_rows(&p.tm_x, a->x, a->M, a->K, a->ldx, BN))
    return MM_ERR_SHAPE;  // TMA rules: 16-byte aligned base and row stride
  p.y = a->y;
  p.ldy = a->ldy;
  p.bias = a->bias;
  p.y_f32 = a->y_dtype == MM_F32;
  p.M = (int)a->M;
  p.N = (int)a->N;
  p.K = (int)a->K;
  p.n_tiles = pl.n_tiles;
  p.m_tiles = pl.m_tiles;
  p.splits = pl.splits;
  p.kb_per_split = pl.kb_per_split;
  p.kb_total = pl.kb_total;
  char* w = static_cast<char*>(ws);
  p.err = reinterpret_cast<unsigned*>(w);
  p.counters = reinterpret_cast<unsigned*>(w + 256);
  p.partial = reinterpret_cast<float*>(w + pl.partial_off);
  const size_t smem = sizeof(Smem) + 1024;
  // opt-in above the default dynamic shared-memory limit (per device; idempotent)
  if (cudaFuncSetAttribute(linear_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return MM_ERR_LAUNCH;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.n_tiles, pl.splits, pl.m_tiles);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // may overlap the previous kernel's tail
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, linear_kernel, p) == cudaSuccess ? MM_OK : MM_ERR_LAUNCH;
}

extern "C" int mm_linear_status(const void* ws, mm_stream_t stream) {
  if (!ws) return MM_ERR_ARG;
  unsigned err = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(&err, ws, sizeof(unsigned), cudaMemcpyDeviceToHost, s) != cudaSuccess) return MM_ERR_LAUNCH;
  if (cudaStreamSynchronize(s) != cudaSuccess) return MM_ERR_LAUNCH;
  return err ? MM_ERR_TIMEOUT : MM_OK;
}
