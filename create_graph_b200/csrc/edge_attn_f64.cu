// float64 instantiations of the edge-attention kernels (padded head dims 4..16).
#include "edge_attn.cuh"

namespace cg {
namespace attn {

int dispatch_f64(Which w, const Params& P, int dp, cudaStream_t stream) {
  switch (dp) {
    case 4: return launch_typed<double, 4>(w, P, stream);
    case 8: return launch_typed<double, 8>(w, P, stream);
    case 16: return launch_typed<double, 16>(w, P, stream);
  }
  set_error("edge_attn: unsupported padded head dim %d", dp);
  return kUnsupported;
}

}  // namespace attn
}  // namespace cg
