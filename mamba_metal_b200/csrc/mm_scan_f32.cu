// Selective-scan kernel instantiations for float activations.
#include "mm_scan.cuh"

namespace mm {
namespace scan {
cudaError_t launch_f32(const Params& p, int nm, bool sp, int blocks, cudaStream_t s) {
  return launch_typed<float>(p, nm, sp, blocks, s);
}
}  // namespace scan
}  // namespace mm
