// tf32-precision instantiations of the tensor-core edge-attention kernels
// (attn_tc.cuh): one rounded tf32 product per mma tile.
#include "attn_tc.cuh"

namespace cg {
namespace attn_tc {

int launch_tf32(int which, const Params& P, int dp, cudaStream_t stream) {
  return launch_prec<false>(which, P, dp, stream);
}

}  // namespace attn_tc
}  // namespace cg
