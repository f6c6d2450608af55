// tf32-precision instantiations of the envelope-pooled token attention
// kernels (pooled_attn.cuh).
#include "pooled_attn.cuh"

namespace cg {
namespace pooled {

int launch_tf32(int which, const PParams& P, int dp, cudaStream_t stream) {
  return launch_prec<false>(which, P, dp, stream);
}

}  // namespace pooled
}  // namespace cg
