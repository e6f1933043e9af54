// One-shot all-reduce over peer memory (NVLink / NVSwitch) for the tensor-parallel decode step.
//
// Push design: every rank owns a receive area of `world` partials in memory that all ranks map
// (symmetric memory). CTA c of each rank stores slice c of its own partial into every peer's area with
// plain stores (posted over NVLink: no round trip per access), releases "slice c of call e is here" to
// each peer, waits (bounded) until every peer has done the same for it, and then sums slice c of the
// `world` partials from its own HBM. A call costs one store sweep, one fence round trip and one flag
// hop, instead of a round trip per remote load.
//
// Low-latency protocol (for small partials): every 16-byte line stored to a peer holds two data words,
// each beside the call's epoch in the same naturally aligned 8-byte half (a unit NVLink delivers whole),
// so the receiver polls the data itself: no fence, no separate flag, one one-way trip per call, at twice
// the bytes. Epochs come from counters in local device memory, so the same launch can be replayed from a
// CUDA graph. No TMA and no multicast.
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
  void* slots[MM_MAX_TP];    // rank r's receive area (world partials, `stride` elements apart)
  unsigned* signals[MM_MAX_TP];
  unsigned* counters;        // [MM_PEER_MAX_BLOCKS] epochs, error word, LL epoch, LL ticket
  void* out;
  long long n, stride;
  int world, rank, nblocks;
};

constexpr int kThreads = 256;
constexpr int kErrWord = MM_PEER_MAX_BLOCKS, kLLEpoch = MM_PEER_MAX_BLOCKS + 1, kLLTicket = MM_PEER_MAX_BLOCKS + 2;

MM_DEV void st_volatile_v4(uint4* p, const uint4& v) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w) : "memory");
}
MM_DEV uint4 ld_volatile_v4(const uint4* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p) : "memory");
  return v;
}

// the elements of one 32-bit word of a T buffer, widened (fp32: one element, 16-bit types: two)
template <typename T> MM_DEV float2 word_f2(unsigned w);
template <> MM_DEV float2 word_f2<float>(unsigned w) { return make_float2(__uint_as_float(w), 0.f); }
template <> MM_DEV float2 word_f2<__half>(unsigned w) { return __half22float2(*reinterpret_cast<const __half2*>(&w)); }
template <> MM_DEV float2 word_f2<__nv_bfloat16>(unsigned w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <typename T> MM_DEV unsigned f2_word(float a, float b);
template <> MM_DEV unsigned f2_word<float>(float a, float) { return __float_as_uint(a); }
template <> MM_DEV unsigned f2_word<__half>(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const unsigned*>(&h);
}
template <> MM_DEV unsigned f2_word<__nv_bfloat16>(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const unsigned*>(&h);
}

// Low-latency protocol. Line j carries words 2j and 2j+1 of the partial (8 data bytes); rank r's lines
// land in area r of each peer. The epoch is one counter per rank, advanced once per call by the last
// CTA to finish (every CTA has read it by then; the next launch on the stream sees the new value).
template <typename T>
__global__ void __launch_bounds__(kThreads) peer_allreduce_ll_kernel(const Params p) {
  constexpr int E = 4 / sizeof(T);  // elements per word
  const int c = blockIdx.x, tid = threadIdx.x;
  const long long nwords = (p.n * (long long)sizeof(T) + 3) / 4, nlines = (nwords + 1) / 2;
  const long long per = (nlines + p.nblocks - 1) / p.nblocks;
  const long long lo = (long long)c * per, hi = min(nlines, lo + per);
  const long long own = (long long)p.rank * p.stride;
  const uint2* mine = reinterpret_cast<const uint2*>(static_cast<const T*>(p.slots[p.rank]) + own);
  const unsigned e = *reinterpret_cast<volatile unsigned*>(p.counters + kLLEpoch) + 1u;
  for (long long j = lo + tid; j < hi; j += kThreads) {
    const uint2 w = mine[j];
    const uint4 line = make_uint4(w.x, e, w.y, e);
    for (int r = 0; r < p.world; ++r)
      if (r != p.rank) st_volatile_v4(reinterpret_cast<uint4*>(static_cast<T*>(p.slots[r]) + own) + j, line);
  }
  const uint4* area = reinterpret_cast<const uint4*>(p.slots[p.rank]);
  T* out = static_cast<T*>(p.out);
  bool gave_up = false;
  for (long long j = lo + tid; j < hi; j += kThreads) {
    float acc[2 * E];
#pragma unroll
    for (int k = 0; k < 2 * E; ++k) acc[k] = 0.f;
    for (int r = 0; r < p.world; ++r) {
      uint2 w;
      if (r == p.rank) {
        w = mine[j];
      } else {
        const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(area) + (long long)r * p.stride) + j;
        uint4 v = ld_volatile_v4(src);
        if ((v.y != e || v.w != e) && !gave_up) {
          const unsigned long long t0 = globaltimer_ns();
          do {
            __nanosleep(20);
            v = ld_volatile_v4(src);
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
              atomicOr(p.counters + kErrWord, 1u);  // a peer never arrived: report, do not hang
              gave_up = true;
              break;
            }
          } while (v.y != e || v.w != e);
        }
        w = make_uint2(v.x, v.z);
      }
      const float2 a = word_f2<T>(w.x), b = word_f2<T>(w.y);
      acc[0] += a.x;
      acc[E] += b.x;
      if (E == 2) {
        acc[1] += a.y;
        acc[E + 1] += b.y;
      }
    }
    const long long e0 = j * 2 * E;  // first element of line j
    if (e0 + 2 * E <= p.n) {
      reinterpret_cast<uint2*>(out)[j] = make_uint2(f2_word<T>(acc[0], acc[E == 2 ? 1 : 0]),
                                                     f2_word<T>(acc[E], acc[E == 2 ? E + 1 : E]));
    } else {
      for (int k = 0; k < 2 * E && e0 + k < p.n; ++k) st_f32(out + e0 + k, acc[k]);
    }
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(p.counters + kLLTicket, 1u) == (unsigned)p.nblocks - 1u) {
      p.counters[kLLTicket] = 0u;
      p.counters[kLLEpoch] = e;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) peer_allreduce_kernel(const Params p) {
  constexpr int V = 16 / sizeof(T);
  const int c = blockIdx.x, tid = threadIdx.x;
  const long long per = ((p.n + p.nblocks - 1) / p.nblocks + V - 1) / V * V;
  const long long lo = (long long)c * per, hi = min(p.n, lo + per);
  const long long own = (long long)p.rank * p.stride;
  const T* mine = static_cast<const T*>(p.slots[p.rank]) + own;

  // 1. this rank's slice c into every peer's receive area
  for (long long i = lo + (long long)tid * V; i < hi; i += (long long)kThreads * V) {
    if (i + V <= hi) {
      const uint4 v = *reinterpret_cast<const uint4*>(mine + i);
      for (int r = 0; r < p.world; ++r)
        if (r != p.rank) *reinterpret_cast<uint4*>(static_cast<T*>(p.slots[r]) + own + i) = v;
    } else {
      for (long long j = i; j < hi; ++j) {
        const T v = mine[j];
        for (int r = 0; r < p.world; ++r)
          if (r != p.rank) static_cast<T*>(p.slots[r])[own + j] = v;
      }
    }
  }
  __shared__ unsigned s_epoch;
  if (tid == 0) s_epoch = p.counters[c] + 1u;
  __syncthreads();
  const unsigned e = s_epoch;
  // 2. release the slice to each peer, then wait for every peer's slice (bounded)
  if (tid < p.world && tid != p.rank) {
    __threadfence_system();
    st_release_sys(p.signals[tid] + c * MM_MAX_TP + p.rank, e);
    const unsigned* flag = p.signals[p.rank] + c * MM_MAX_TP + tid;
    if (ld_acquire_sys(flag) < e) {
      const unsigned long long t0 = globaltimer_ns();
      while (ld_acquire_sys(flag) < e) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          atomicOr(p.counters + kErrWord, 1u);  // a peer never arrived: report, do not hang
          break;
        }
        __nanosleep(20);
      }
    }
  }
  __syncthreads();
  // 3. sum the world partials of slice c from local memory (L2 reads: peers wrote them)
  const T* area = static_cast<const T*>(p.slots[p.rank]);
  T* out = static_cast<T*>(p.out);
  for (long long i = lo + (long long)tid * V; i < hi; i += (long long)kThreads * V) {
    if (i + V <= hi) {
      float acc[V];
#pragma unroll
      for (int k = 0; k < V; ++k) acc[k] = 0.f;
      for (int r = 0; r < p.world; ++r) {
        const uint4 v = __ldcg(reinterpret_cast<const uint4*>(area + (long long)r * p.stride + i));
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
        for (int r = 0; r < p.world; ++r) a += ld_f32(area + (long long)r * p.stride + j);
        st_f32(out + j, a);
      }
    }
  }
  if (tid == 0) p.counters[c] = e;
}


// Low-latency all-reduce fused with the residual add + RMSNorm that follows it (the out_proj reduction
// of a tensor-parallel decode step feeding the next pre-norm, mamba_model.py:49-58). CTA r owns row r:
// it pushes the row's lines, sums every rank's lines in rank order, rounds the sum to T (as the unfused
// all-reduce output would be), adds it into the fp32 residual, and writes the normalised row. Epochs as
// in peer_allreduce_ll_kernel (the two kernels share the counter: one sequence of LL calls).
constexpr int kNormMaxLines = 8;  // per thread: rows up to 8 x 256 lines

struct NormArgs {
  float* res;
  const float* w;
  void* out;
  long long osr;
  int dim;
  float eps;
};

template <typename T>
__global__ void __launch_bounds__(kThreads) peer_ll_addnorm_kernel(const Params p, const NormArgs q) {
  constexpr int E = 4 / sizeof(T);  // elements per word
  constexpr int LE = 2 * E;         // elements per line
  const int row = blockIdx.x, tid = threadIdx.x;
  const int lines = q.dim / LE;
  const long long l0 = (long long)row * lines;
  const long long own = (long long)p.rank * p.stride;
  const uint2* mine = reinterpret_cast<const uint2*>(static_cast<const T*>(p.slots[p.rank]) + own);
  const unsigned e = *reinterpret_cast<volatile unsigned*>(p.counters + kLLEpoch) + 1u;
  for (int j = tid; j < lines; j += kThreads) {
    const uint2 w = mine[l0 + j];
    const uint4 line = make_uint4(w.x, e, w.y, e);
    for (int r = 0; r < p.world; ++r)
      if (r != p.rank) st_volatile_v4(reinterpret_cast<uint4*>(static_cast<T*>(p.slots[r]) + own) + l0 + j, line);
  }
  const T* area = static_cast<const T*>(p.slots[p.rank]);
  float* res = q.res + (long long)row * q.dim;
  float v[kNormMaxLines][LE];
  float ss = 0.f;
  bool gave_up = false;
#pragma unroll
  for (int i = 0; i < kNormMaxLines; ++i) {
    const int j = tid + i * kThreads;
    if (j >= lines) break;
    float acc[LE];
#pragma unroll
    for (int k = 0; k < LE; ++k) acc[k] = 0.f;
    for (int r = 0; r < p.world; ++r) {
      uint2 w;
      if (r == p.rank) {
        w = mine[l0 + j];
      } else {
        const uint4* src = reinterpret_cast<const uint4*>(area + (long long)r * p.stride) + l0 + j;
        uint4 x = ld_volatile_v4(src);
        if ((x.y != e || x.w != e) && !gave_up) {
          const unsigned long long t0 = globaltimer_ns();
          do {
            __nanosleep(20);
            x = ld_volatile_v4(src);
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
              atomicOr(p.counters + kErrWord, 1u);  // a peer never arrived: report, do not hang
              gave_up = true;
              break;
            }
          } while (x.y != e || x.w != e);
        }
        w = make_uint2(x.x, x.z);
      }
      const float2 a = word_f2<T>(w.x), b = word_f2<T>(w.y);
      acc[0] += a.x;
      acc[E] += b.x;
      if (E == 2) {
        acc[1] += a.y;
        acc[E + 1] += b.y;
      }
    }
    float* rp = res + j * LE;
    float rv[LE];
    if (LE == 4) {
      const float4 r4 = *reinterpret_cast<const float4*>(rp);
      rv[0] = r4.x; rv[1] = r4.y; rv[LE > 2 ? 2 : 0] = r4.z; rv[LE > 3 ? 3 : 0] = r4.w;
    } else {
      const float2 r2 = *reinterpret_cast<const float2*>(rp);
      rv[0] = r2.x; rv[1] = r2.y;
    }
#pragma unroll
    for (int k = 0; k < LE; ++k) {
      v[i][k] = rv[k] + ElemTraits<T>::to_f32(ElemTraits<T>::from_f32(acc[k]));
      ss = fmaf(v[i][k], v[i][k], ss);
    }
    if (LE == 4) *reinterpret_cast<float4*>(rp) = make_float4(v[i][0], v[i][1], v[i][LE > 2 ? 2 : 0], v[i][LE > 3 ? 3 : 0]);
    else *reinterpret_cast<float2*>(rp) = make_float2(v[i][0], v[i][1]);
  }
  // block sum of squares
  __shared__ float red[kThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  if (tid < 32) {
    float t = tid < kThreads / 32 ? red[tid] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (tid == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)q.dim + q.eps);
  T* out = static_cast<T*>(q.out) + (long long)row * q.osr;
#pragma unroll
  for (int i = 0; i < kNormMaxLines; ++i) {
    const int j = tid + i * kThreads;
    if (j >= lines) break;
#pragma unroll
    for (int k = 0; k < LE; ++k) st_f32(out + j * LE + k, v[i][k] * inv * q.w[j * LE + k]);
  }
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(p.counters + kLLTicket, 1u) == gridDim.x - 1u) {
      p.counters[kLLTicket] = 0u;
      p.counters[kLLEpoch] = e;
    }
  }
}

}  // namespace comm
}  // namespace mm

using namespace mm;

static int fill_params(const MMPeerReduceArgs* a, comm::Params& p) {
  if (!a) return MM_ERR_ARG;
  const size_t es = dtype_size(a->dtype);
  if (es == 0) return MM_ERR_DTYPE;
  if (a->world < 1 || a->world > MM_MAX_TP || a->rank < 0 || a->rank >= a->world) return MM_ERR_SHAPE;
  if (a->nblocks < 1 || a->nblocks > MM_PEER_MAX_BLOCKS || a->n < 0 || a->stride < a->n) return MM_ERR_SHAPE;
  if ((a->stride * (int64_t)es) % 16 != 0) return MM_ERR_SHAPE;
  if (a->protocol != MM_PEER_FLAGS && a->protocol != MM_PEER_LL) return MM_ERR_ARG;
  // an LL area holds 16 bytes per 8 data bytes
  if (a->protocol == MM_PEER_LL && (a->n * (int64_t)es + 7) / 8 * 16 > a->stride * (int64_t)es) return MM_ERR_SHAPE;
  if (!a->counters) return MM_ERR_ARG;
  for (int r = 0; r < MM_MAX_TP; ++r) {
    p.slots[r] = r < a->world ? a->slots[r] : nullptr;
    p.signals[r] = r < a->world ? a->signals[r] : nullptr;
    if (r < a->world && (!a->slots[r] || !a->signals[r] || !aligned16(a->slots[r]))) return MM_ERR_ARG;
  }
  p.counters = a->counters;
  p.out = a->out;
  p.n = a->n;
  p.stride = a->stride;
  p.world = (int)a->world;
  p.rank = (int)a->rank;
  p.nblocks = (int)a->nblocks;
  return MM_OK;
}

extern "C" int mm_peer_allreduce(const MMPeerReduceArgs* a, mm_stream_t stream) {
  comm::Params p;
  const int rc = fill_params(a, p);
  if (rc != MM_OK) return rc;
  if (!a->out || !aligned16(a->out)) return MM_ERR_ARG;
  if (a->n == 0) return MM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a->protocol == MM_PEER_LL) {
    if (a->dtype == MM_F32) comm::peer_allreduce_ll_kernel<float><<<p.nblocks, comm::kThreads, 0, s>>>(p);
    else if (a->dtype == MM_F16) comm::peer_allreduce_ll_kernel<__half><<<p.nblocks, comm::kThreads, 0, s>>>(p);
    else comm::peer_allreduce_ll_kernel<__nv_bfloat16><<<p.nblocks, comm::kThreads, 0, s>>>(p);
  } else if (a->dtype == MM_F32) {
    comm::peer_allreduce_kernel<float><<<p.nblocks, comm::kThreads, 0, s>>>(p);
  } else if (a->dtype == MM_F16) {
    comm::peer_allreduce_kernel<__half><<<p.nblocks, comm::kThreads, 0, s>>>(p);
  } else {
    comm::peer_allreduce_kernel<__nv_bfloat16><<<p.nblocks, comm::kThreads, 0, s>>>(p);
  }
  return cudaGetLastError() == cudaSuccess ? MM_OK : MM_ERR_LAUNCH;
}

extern "C" int mm_peer_allreduce_add_rmsnorm(const MMPeerAddNormArgs* a, mm_stream_t stream) {
  if (!a) return MM_ERR_ARG;
  comm::Params p;
  const int rc = fill_params(&a->reduce, p);
  if (rc != MM_OK) return rc;
  const int64_t es = (int64_t)dtype_size(a->reduce.dtype);
  const int64_t le = 8 / es;  // elements per low-latency line
  if (a->reduce.protocol != MM_PEER_LL) return MM_ERR_ARG;
  if (a->rows < 0 || a->dim < 1 || a->dim % le != 0 || a->dim / le > comm::kNormMaxLines * comm::kThreads)
    return MM_ERR_SHAPE;
  if (a->reduce.n != a->rows * a->dim || a->rows > (1LL << 31) - 1) return MM_ERR_SHAPE;
  if (!a->residual || !a->weight || !a->out) return MM_ERR_ARG;
  if (!aligned16(a->residual)) return MM_ERR_ARG;
  if (a->rows == 0) return MM_OK;
  p.nblocks = (int)a->rows;
  comm::NormArgs q;
  q.res = a->residual;
  q.w = a->weight;
  q.out = a->out;
  q.osr = a->out_stride_r;
  q.dim = (int)a->dim;
  q.eps = (float)a->eps;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned grid = (unsigned)a->rows;
  if (a->reduce.dtype == MM_F32) comm::peer_ll_addnorm_kernel<float><<<grid, comm::kThreads, 0, s>>>(p, q);
  else if (a->reduce.dtype == MM_F16) comm::peer_ll_addnorm_kernel<__half><<<grid, comm::kThreads, 0, s>>>(p, q);
  else comm::peer_ll_addnorm_kernel<__nv_bfloat16><<<grid, comm::kThreads, 0, s>>>(p, q);
  return cudaGetLastError() == cudaSuccess ? MM_OK : MM_ERR_LAUNCH;
}
