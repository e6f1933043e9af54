// Host side of the selective-scan forward: work plan, workspace layout and the C-ABI entry points.
// The device code is in mm_scan.cuh; its instantiations live in mm_scan_{f32,f16,bf16}.cu.
#include <algorithm>

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

static int resident_warps() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148 * 16;
  if (dev >= 0 && dev < 64 && cached[dev] > 0) return cached[dev];
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int v = sms * MM_SCAN_MIN_BLOCKS * kWarpsPerCta;  // resident warps of the dstate <= 16 kernels
  if (dev >= 0 && dev < 64) cached[dev] = v;
  return v;
}

static inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

static int make_plan(const MMScanArgs* a, Plan* pl) {
  if (!a) return MM_ERR_ARG;
  const int es = dtype_size(a->dtype);
  if (es == 0) return MM_ERR_DTYPE;
  if (a->batch < 0 || a->dim < 0 || a->seqlen < 0 || a->dstate < 1) return MM_ERR_SHAPE;
  if (a->dstate > MM_MAX_DSTATE) return MM_ERR_SHAPE;
  if (a->batch > (1 << 30) || a->dim > (1 << 30) || a->seqlen > (1 << 30)) return MM_ERR_SHAPE;
  pl->NM = a->dstate <= 16 ? 16 : 64;
  pl->TT = 16 / es;
  pl->groups_per_batch = (int)((a->dim + 31) / 32);
  pl->tiles_per_row = (int)((a->seqlen + pl->TT - 1) / pl->TT);
  pl->total_tiles = (long long)a->batch * pl->groups_per_batch * pl->tiles_per_row;
  long long tpw;
  if (a->piece_tiles > 0) {
    tpw = a->piece_tiles;
  } else {
    // Fill the resident warp slots, but keep pieces long enough that the recomputed head
    // (kHeadSteps) stays a small fraction of the work.
    const long long min_tiles = std::max<long long>(1, (8 * kHeadSteps) / pl->TT);
    const long long want = resident_warps();
    tpw = std::max<long long>(min_tiles, (pl->total_tiles + want - 1) / want);
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
  p.A = a->A; p.D = a->D; p.state_out = a->state_out;
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
