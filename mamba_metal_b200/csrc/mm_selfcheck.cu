// Self-check entry point: evaluates the device math helpers the kernels use on caller-given arguments,
// so that tests can compare them with exact values and with the hardware approximations.
#include "mm_common.cuh"

namespace mm {
namespace {

__global__ void exp2_check_kernel(const float* __restrict__ x, float* __restrict__ y_poly,
                                  float* __restrict__ y_mufu, long long n) {
  const long long i = 2 * ((long long)blockIdx.x * blockDim.x + threadIdx.x);
  if (i >= n) return;
  const float a = x[i];
  const float b = i + 1 < n ? x[i + 1] : 0.f;
  const float2 p = f2_unpack(exp2_poly2(f2_pack(a, b)));
  y_poly[i] = p.x;
  y_mufu[i] = ex2(a);
  if (i + 1 < n) {
    y_poly[i + 1] = p.y;
    y_mufu[i + 1] = ex2(b);
  }
}

}  // namespace
}  // namespace mm

extern "C" int mm_exp2_check(const float* x, float* y_poly, float* y_mufu, int64_t n, mm_stream_t stream) {
  if (n < 0 || (n > 0 && (!x || !y_poly || !y_mufu))) return MM_ERR_ARG;
  if (n == 0) return MM_OK;
  const long long pairs = (n + 1) / 2;
  const int threads = 256;
  const long long blocks = (pairs + threads - 1) / threads;
  if (blocks > 0x7fffffffLL) return MM_ERR_SHAPE;
  mm::exp2_check_kernel<<<(unsigned)blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(x, y_poly, y_mufu, n);
  return cudaGetLastError() == cudaSuccess ? MM_OK : MM_ERR_LAUNCH;
}
