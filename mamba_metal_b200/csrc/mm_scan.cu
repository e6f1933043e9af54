// Host side of the selective-scan forward: work plan, workspace layout and the C-ABI entry points.
// The device code is in mm_scan.cuh; its instantiations live in mm_scan_{f32,f16,bf16}.cu.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "mm_scan.cuh"

namespace mm {
namespace scan {


struct Plan {
  int NM, TT;
  int groups_per_batch, tiles_per_row;
  long long total_tiles;
  int tiles_per_warp, n_warps;
  size_t ws_bytes;
  size_t flags_off, agg_off, pre_off;
};

// Resident warps of the dstate <= 16 kernels on the current device. The SM count is cached per device in
// atomics: concurrent first calls may both query it, and both store the same value.
static int resident_warps() {
  static std::atomic<int> cached[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148 * MM_SCAN_MIN_BLOCKS * kWarpsPerCta;
  const bool cacheable = dev >= 0 && dev < 64;
  if (cacheable) {
    const int c = cached[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int v = sms * MM_SCAN_MIN_BLOCKS * kWarpsPerCta;
  if (cacheable) cached[dev].store(v, std::memory_order_relaxed);
  return v;
}

static inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
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

// 3-D map over a (n2, n1, n0) tensor with unit stride along n0 and element strides s1 (along n1) and s2
// (along n2), tiled in boxes of (1, box1, box0). Fails (-> plain-load path) when TMA's rules are not met.
static bool encode_3d(CUtensorMap* m, const void* base, int64_t dtype, long long n0, long long n1, long long n2,
                      long long s1, long long s2, int box0, int box1) {
  auto enc = tensor_map_encoder();
  if (!enc || !base || !aligned16(base)) return false;
  const int es = dtype_size(dtype);
  if (n1 == 1) s1 = ((n0 * es + 15) / 16) * 16 / es;  // unused dimension: any legal stride
  if (n2 == 1) s2 = s1 * n1;
  if (s1 <= 0 || s2 <= 0 || (s1 * es) % 16 != 0 || (s2 * es) % 16 != 0) return false;
  if ((s1 * es) >= (1LL << 40) || (s2 * es) >= (1LL << 40)) return false;
  const CUtensorMapDataType dt = dtype == MM_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == MM_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  cuuint64_t dims[3] = {(cuuint64_t)n0, (cuuint64_t)n1, (cuuint64_t)n2};
  cuuint64_t strides[2] = {(cuuint64_t)(s1 * es), (cuuint64_t)(s2 * es)};
  cuuint32_t box[3] = {(cuuint32_t)box0, (cuuint32_t)box1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int make_plan(const MMScanArgs* a, Plan* pl) {
  if (!a) return MM_ERR_ARG;
  const int es = dtype_size(a->dtype);
  if (es == 0) return MM_ERR_DTYPE;
  if (a->batch < 0 || a->dim < 0 || a->seqlen < 0 || a->dstate < 1) return MM_ERR_SHAPE;
  if (a->dstate > MM_MAX_DSTATE) return MM_ERR_SHAPE;
  if (a->batch > (1 << 30) || a->dim > (1 << 30) || a->seqlen > (1 << 30)) return MM_ERR_SHAPE;
  pl->NM = a->dstate <= 16 ? 16 : 64;
  pl->TT = 32 / es;
  pl->groups_per_batch = (int)((a->dim + 31) / 32);
  pl->tiles_per_row = (int)((a->seqlen + pl->TT - 1) / pl->TT);
  pl->total_tiles = (long long)a->batch * pl->groups_per_batch * pl->tiles_per_row;
  long long tpw;
  if (a->piece_tiles > 0) {
    tpw = a->piece_tiles;
  } else {
    // Fill the resident warp slots. A piece that starts mid-sequence recomputes at least its head
    // (kHeadSteps) once the carry arrives, so its time is about P + min(P, R) steps for piece length P
    // and decay length R; with the slots full, a longer P only adds time, so pieces are as short as the
    // slots allow, down to two heads (below that the look-back and ring fill per piece dominate).
    const long long min_tiles = std::max<long long>(1, (2 * kHeadSteps) / pl->TT);
    const long long want = resident_warps();
    tpw = std::max<long long>(min_tiles, (pl->total_tiles + want - 1) / want);
    // With at least as many (batch, channel group) rows as warp slots, whole rows per warp need no carry
    // hand-off at all (no look-back, no recompute, whose length grows as the decay slows); take them when
    // the longest warp's work grows by at most 1/8 over the split plan.
    const long long rows = (long long)a->batch * pl->groups_per_batch;
    if (rows >= want) {
      const long long whole = ((rows + want - 1) / want) * pl->tiles_per_row;
      if (8 * whole <= 9 * tpw) tpw = whole;
    }
  }
  tpw = std::max<long long>(1, std::min<long long>(tpw, std::max<long long>(1, pl->total_tiles)));
  pl->tiles_per_warp = (int)tpw;
  pl->n_warps = pl->total_tiles > 0 ? (int)((pl->total_tiles + tpw - 1) / tpw) : 0;
  // workspace: [ticket, err, pad, stats[4]] | flags[n_warps] (one 128-byte line each) | agg | pre
  size_t off = 256;
  pl->flags_off = off;
  off = align256(off + sizeof(unsigned) * kFlagStride * (size_t)std::max(pl->n_warps, 1));
  pl->agg_off = off;
  off = align256(off + sizeof(float) * (size_t)pl->n_warps * (pl->NM + 1) * 32);
  pl->pre_off = off;
  off = align256(off + sizeof(float) * (size_t)pl->n_warps * pl->NM * 32);
  pl->ws_bytes = off;
  return MM_OK;
}

static bool row_vec_ok(const void* base, const int64_t* st, int es, bool require) {
  if (!require) return true;
  if (base == nullptr) return true;
  if (st[2] != 1) return false;
  if (!aligned16(base)) return false;
  const int64_t epv = 16 / es;
  return (st[0] % epv == 0) && (st[1] % epv == 0);
}

}  // namespace scan
}  // namespace mm

using namespace mm;
using namespace mm::scan;

extern "C" int mm_selective_scan_workspace_size(const MMScanArgs* a, size_t* bytes) {
  if (!bytes) return MM_ERR_ARG;
  Plan pl;
  const int rc = make_plan(a, &pl);
  if (rc != MM_OK) return rc;
  *bytes = pl.ws_bytes;
  return MM_OK;
}

extern "C" int mm_selective_scan_fwd(const MMScanArgs* a, void* ws, size_t ws_bytes, mm_stream_t stream) {
  Plan pl;
  int rc = make_plan(a, &pl);
  if (rc != MM_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (pl.total_tiles == 0 || a->dim == 0 || a->batch == 0) {
    // empty sequence: the final state is the zero initial state
    if (a->state_out && a->batch > 0 && a->dim > 0) {
      if (cudaMemsetAsync(a->state_out, 0, sizeof(float) * a->batch * a->dim * a->dstate, s) != cudaSuccess)
        return MM_ERR_LAUNCH;
    }
    return MM_OK;
  }
  if (!a->u || !a->delta || !a->A || !a->B || !a->C || !a->y) return MM_ERR_ARG;
  if (!ws || ws_bytes < pl.ws_bytes || (reinterpret_cast<uintptr_t>(ws) & 255u)) return MM_ERR_WORKSPACE;
  const int es = dtype_size(a->dtype);
  Params p;
  p.u = a->u; p.delta = a->delta; p.z = a->z; p.y = a->y; p.Bm = a->B; p.Cm = a->C;
  p.A = a->A; p.D = a->D; p.dbias = a->delta_bias; p.state_out = a->state_out;
  for (int i = 0; i < 3; ++i) {
    p.us[i] = a->u_stride[i]; p.ds[i] = a->delta_stride[i]; p.zs[i] = a->z_stride[i];
    p.ys[i] = a->y_stride[i]; p.Bs[i] = a->B_stride[i]; p.Cs[i] = a->C_stride[i];
  }
  p.As[0] = a->A_stride[0]; p.As[1] = a->A_stride[1];
  p.batch = (int)a->batch; p.dim = (int)a->dim; p.nstate = (int)a->dstate; p.seqlen = (int)a->seqlen;
  p.groups_per_batch = pl.groups_per_batch; p.tiles_per_row = pl.tiles_per_row;
  p.total_tiles = pl.total_tiles; p.tiles_per_warp = pl.tiles_per_warp; p.n_warps = pl.n_warps;
  p.head_tiles = (kHeadSteps + pl.TT - 1) / pl.TT;
  p.vec_io = row_vec_ok(a->u, a->u_stride, es, true) && row_vec_ok(a->delta, a->delta_stride, es, true) &&
             row_vec_ok(a->y, a->y_stride, es, true) && row_vec_ok(a->z, a->z_stride, es, a->z != nullptr);
  p.vec_bc = row_vec_ok(a->B, a->B_stride, es, true) && row_vec_ok(a->C, a->C_stride, es, true);
  p.has_D = a->D != nullptr;
  p.has_z = a->z != nullptr;
  {
    // TMA path: every tile-fed tensor t-contiguous with 16-byte aligned rows
    const long long L = a->seqlen, nb = a->batch, nd = a->dim, nn = a->dstate;
    bool ok = a->u_stride[2] == 1 && a->delta_stride[2] == 1 && a->B_stride[2] == 1 && a->C_stride[2] == 1 &&
              (!a->z || a->z_stride[2] == 1);
    ok = ok && encode_3d(&p.tm_u, a->u, a->dtype, L, nd, nb, a->u_stride[1], a->u_stride[0], pl.TT, 32);
    ok = ok && encode_3d(&p.tm_d, a->delta, a->dtype, L, nd, nb, a->delta_stride[1], a->delta_stride[0], pl.TT, 32);
    ok = ok && (!a->z || encode_3d(&p.tm_z, a->z, a->dtype, L, nd, nb, a->z_stride[1], a->z_stride[0], pl.TT, 32));
    ok = ok && encode_3d(&p.tm_B, a->B, a->dtype, L, nn, nb, a->B_stride[1], a->B_stride[0], pl.TT, pl.NM);
    ok = ok && encode_3d(&p.tm_C, a->C, a->dtype, L, nn, nb, a->C_stride[1], a->C_stride[0], pl.TT, pl.NM);
    p.use_tma = ok && !(a->options & 1);
  }
  char* w = static_cast<char*>(ws);
  p.ticket = reinterpret_cast<unsigned*>(w);
  p.err = reinterpret_cast<unsigned*>(w) + 1;
  p.stats = reinterpret_cast<unsigned long long*>(w + 8);
  p.flags = reinterpret_cast<unsigned*>(w + pl.flags_off);
  p.agg = reinterpret_cast<float*>(w + pl.agg_off);
  p.pre = reinterpret_cast<float*>(w + pl.pre_off);
  // ticket, err and the flags must start at zero; the data arrays are written before being read
  if (cudaMemsetAsync(ws, 0, pl.agg_off, s) != cudaSuccess) return MM_ERR_LAUNCH;
  const int blocks = (pl.n_warps + kWarpsPerCta - 1) / kWarpsPerCta;
  const bool sp = a->delta_softplus != 0;
  cudaError_t e;
  if (a->dtype == MM_F32) e = launch_f32(p, pl.NM, sp, blocks, s);
  else if (a->dtype == MM_F16) e = launch_f16(p, pl.NM, sp, blocks, s);
  else e = launch_bf16(p, pl.NM, sp, blocks, s);
  return e == cudaSuccess ? MM_OK : MM_ERR_LAUNCH;
}

extern "C" int mm_selective_scan_stats(const void* ws, unsigned long long* out4, mm_stream_t stream) {
  if (!ws || !out4) return MM_ERR_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(out4, static_cast<const char*>(ws) + 8, 4 * sizeof(unsigned long long),
                      cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return MM_ERR_LAUNCH;
  return cudaStreamSynchronize(s) == cudaSuccess ? MM_OK : MM_ERR_LAUNCH;
}

extern "C" int mm_selective_scan_status(const void* ws, mm_stream_t stream) {
  if (!ws) return MM_ERR_ARG;
  unsigned err = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(&err, static_cast<const unsigned*>(ws) + 1, sizeof(unsigned), cudaMemcpyDeviceToHost, s) !=
      cudaSuccess)
    return MM_ERR_LAUNCH;
  if (cudaStreamSynchronize(s) != cudaSuccess) return MM_ERR_LAUNCH;
  return err ? MM_ERR_TIMEOUT : MM_OK;
}

// ------------------------------------------------------------------------------------------------
// Allocation-free entry point: the workspace is a fixed static __device__ array of this library.

namespace {
__device__ __align__(256) unsigned char g_scan_scratch[MM_SCAN_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
struct ScratchSlot {
  CUcontext ctx;  // context the address below belongs to
  void* ptr;
};
ScratchSlot g_scratch[kMaxDevices] = {};

// cuCtxGetCurrent through the runtime's driver entry point (no link against libcuda).
PFN_cuCtxGetCurrent_v4000 ctx_getter() {
  static const PFN_cuCtxGetCurrent_v4000 fn = []() -> PFN_cuCtxGetCurrent_v4000 {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(f);
  }();
  return fn;
}

// Device address of g_scan_scratch on the current device. The symbol's name in host code is only a
// host-side handle; kernels must be given this address. It is looked up once per device and context:
// after a device reset the runtime creates a new primary context with the module loaded anew, so the
// address is looked up again when the current context differs from the cached one.
int scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return MM_ERR_LAUNCH;
  auto get_ctx = ctx_getter();
  if (!get_ctx) return MM_ERR_LAUNCH;
  // Null until the runtime has made the device's primary context current on this thread.
  CUcontext ctx = nullptr;
  if (get_ctx(&ctx) != CUDA_SUCCESS) return MM_ERR_LAUNCH;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  ScratchSlot& slot = g_scratch[dev];
  if (slot.ptr == nullptr || ctx == nullptr || slot.ctx != ctx) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_scan_scratch) != cudaSuccess || p == nullptr) return MM_ERR_LAUNCH;
    if (get_ctx(&ctx) != CUDA_SUCCESS || ctx == nullptr) return MM_ERR_LAUNCH;
    slot.ptr = p;
    slot.ctx = ctx;
  }
  *out = slot.ptr;
  return MM_OK;
}

// Work plan whose workspace fits the fixed scratch buffer. With piece_tiles == 0 (library's choice) the
// default plan targets one piece per resident warp; when its workspace (one flag line and two state
// blocks per warp) does not fit, pieces are lengthened until it does. An explicit piece_tiles is kept.
int plan_within_scratch(const MMScanArgs* a, MMScanArgs* fitted, size_t* need) {
  *fitted = *a;
  int rc = mm_selective_scan_workspace_size(fitted, need);
  if (rc != MM_OK || *need <= MM_SCAN_NOALLOC_SCRATCH_BYTES || a->piece_tiles > 0) return rc;
  Plan pl;
  rc = make_plan(a, &pl);
  if (rc != MM_OK) return rc;
  const size_t per_warp = sizeof(unsigned) * kFlagStride + sizeof(float) * (size_t)(2 * pl.NM + 1) * 32;
  const size_t fixed = 256 + 3 * 256;  // header + alignment slack of the three per-warp arrays
  const long long max_warps = (long long)((MM_SCAN_NOALLOC_SCRATCH_BYTES - fixed) / per_warp);
  if (max_warps < 1) return MM_ERR_TOO_LARGE;
  fitted->piece_tiles = (pl.total_tiles + max_warps - 1) / max_warps;
  return mm_selective_scan_workspace_size(fitted, need);
}
}  // namespace

extern "C" int mm_selective_scan_fwd_noalloc(const MMScanArgs* a, mm_stream_t stream) {
  if (!a) return MM_ERR_ARG;
  MMScanArgs fitted;
  size_t need = 0;
  const int rc = plan_within_scratch(a, &fitted, &need);
  if (rc != MM_OK) return rc;
  if (need > MM_SCAN_NOALLOC_SCRATCH_BYTES) return MM_ERR_TOO_LARGE;
  void* ws = nullptr;
  const int rs = scratch_for_current_device(&ws);
  if (rs != MM_OK) return rs;
  return mm_selective_scan_fwd(&fitted, ws, MM_SCAN_NOALLOC_SCRATCH_BYTES, stream);
}
