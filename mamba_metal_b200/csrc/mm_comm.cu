// One-shot all-reduce over peer memory (NVLink / NVSwitch) for the tensor-parallel decode step.
//
// Every rank has written its partial into its own slot of a buffer that all ranks map (symmetric memory).
// CTA c of each rank owns element slice c: it tells every peer "slice c of call e is ready" by storing the
// call's epoch e into the peer's signal pad, waits (bounded) until every peer has done the same for it,
// then reads slice c of every rank's slot with plain peer loads, sums in fp32 and writes the result
// locally. Epochs come from a per-CTA counter in local device memory, so the same launch can be replayed
// from a CUDA graph. No TMA and no multicast: peer memory is read with ordinary loads only.
#include "mm_common.cuh"

namespace mm {
namespace comm {

constexpr unsigned long long kWaitLimitNs = 2000000000ull;

MM_DEV void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
MM_DEV unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct Params {
  const void* bufs[MM_MAX_TP];
  unsigned* signals[MM_MAX_TP];
  unsigned* counters;  // [nblocks] epochs, then the error word
  void* out;
  long long n;
  int world, rank, nblocks;
};

template <typename T>
__global__ void __launch_bounds__(256) peer_allreduce_kernel(const Params p) {
  const int c = blockIdx.x;
  __shared__ unsigned s_epoch;
  if (threadIdx.x == 0) s_epoch = p.counters[c] + 1u;
  __syncthreads();
  const unsigned e = s_epoch;
  if (threadIdx.x < p.world) {
    const int peer = threadIdx.x;
    __threadfence_system();  // this rank's slot (written by earlier kernels) before the signal
    st_release_sys(p.signals[peer] + c * MM_MAX_TP + p.rank, e);
  }
  if (threadIdx.x < p.world) {
    const unsigned* flag = p.signals[p.rank] + c * MM_MAX_TP + threadIdx.x;
    if (ld_acquire_sys(flag) < e) {
      const unsigned long long t0 = globaltimer_ns();
      while (ld_acquire_sys(flag) < e) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          atomicOr(p.counters + p.nblocks, 1u);  // a peer never arrived: report, do not hang
          break;
        }
        __nanosleep(32);
      }
    }
  }
  __syncthreads();
  // slice c of n, in 16-byte vectors where possible
  constexpr int V = 16 / sizeof(T);
  const long long per = ((p.n + p.nblocks - 1) / p.nblocks + V - 1) / V * V;
  const long long lo = (long long)c * per, hi = min(p.n, lo + per);
  T* out = static_cast<T*>(p.out);
  for (long long i = lo + (long long)threadIdx.x * V; i < hi; i += (long long)blockDim.x * V) {
    float acc[V];
#pragma unroll
    for (int k = 0; k < V; ++k) acc[k] = 0.f;
    if (i + V <= hi) {
      for (int r = 0; r < p.world; ++r) {
        const uint4 v = __ldcv(reinterpret_cast<const uint4*>(static_cast<const T*>(p.bufs[r]) + i));
#pragma unroll
        for (int k = 0; k < V / 2; ++k) {
          const float2 f = vec_pair<T>(v, k);
          acc[2 * k] += f.x;
          acc[2 * k + 1] += f.y;
        }
      }
      uint4 o;
#pragma unroll
      for (int k = 0; k < V / 2; ++k) vec_set_pair<T>(o, k, acc[2 * k], acc[2 * k + 1]);
      *reinterpret_cast<uint4*>(out + i) = o;
    } else {
      for (long long j = i; j < hi; ++j) {
        float a = 0.f;
        for (int r = 0; r < p.world; ++r) a += ld_f32(static_cast<const T*>(p.bufs[r]) + j);
        st_f32(out + j, a);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) p.counters[c] = e;
}

}  // namespace comm
}  // namespace mm

using namespace mm;

extern "C" int mm_peer_allreduce(const MMPeerReduceArgs* a, mm_stream_t stream) {
  if (!a) return MM_ERR_ARG;
  if (dtype_size(a->dtype) == 0) return MM_ERR_DTYPE;
  if (a->world < 1 || a->world > MM_MAX_TP || a->rank < 0 || a->rank >= a->world) return MM_ERR_SHAPE;
  if (a->nblocks < 1 || a->nblocks > MM_PEER_MAX_BLOCKS || a->n < 0) return MM_ERR_SHAPE;
  if (!a->counters || !a->out) return MM_ERR_ARG;
  comm::Params p;
  for (int r = 0; r < MM_MAX_TP; ++r) {
    p.bufs[r] = r < a->world ? a->bufs[r] : nullptr;
    p.signals[r] = r < a->world ? a->signals[r] : nullptr;
    if (r < a->world && (!a->bufs[r] || !a->signals[r] || !aligned16(a->bufs[r]))) return MM_ERR_ARG;
  }
  if (!aligned16(a->out)) return MM_ERR_ARG;
  p.counters = a->counters;
  p.out = a->out;
  p.n = a->n;
  p.world = (int)a->world;
  p.rank = (int)a->rank;
  p.nblocks = (int)a->nblocks;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a->dtype == MM_F32) comm::peer_allreduce_kernel<float><<<p.nblocks, 256, 0, s>>>(p);
  else if (a->dtype == MM_F16) comm::peer_allreduce_kernel<__half><<<p.nblocks, 256, 0, s>>>(p);
  else comm::peer_allreduce_kernel<__nv_bfloat16><<<p.nblocks, 256, 0, s>>>(p);
  return cudaGetLastError() == cudaSuccess ? MM_OK : MM_ERR_LAUNCH;
}
