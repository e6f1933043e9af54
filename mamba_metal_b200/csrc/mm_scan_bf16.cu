// Selective-scan kernel instantiations for __nv_bfloat16 activations.
#include "mm_scan.cuh"

namespace mm {
namespace scan {
cudaError_t launch_bf16(const Params& p, int nm, bool sp, int blocks, cudaStream_t s) {
  return launch_typed<__nv_bfloat16>(p, nm, sp, blocks, s);
}
}  // namespace scan
}  // namespace mm
