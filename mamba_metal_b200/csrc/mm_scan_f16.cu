// Selective-scan kernel instantiations for __half activations.
#include "mm_scan.cuh"

namespace mm {
namespace scan {
cudaError_t launch_f16(const Params& p, int nm, bool sp, int blocks, cudaStream_t s) {
  return launch_typed<__half>(p, nm, sp, blocks, s);
}
}  // namespace scan
}  // namespace mm
