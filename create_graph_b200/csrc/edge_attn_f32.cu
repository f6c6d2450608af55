// float32 instantiations of the edge-attention kernels (padded head dims 8..64).
#include "edge_attn.cuh"

namespace cg {
namespace attn {

int dispatch_f32(Which w, const Params& P, int dp, cudaStream_t stream) {
  switch (dp) {
    case 8: return launch_typed<float, 8>(w, P, stream);
    case 16: return launch_typed<float, 16>(w, P, stream);
    case 32: return launch_typed<float, 32>(w, P, stream);
    case 64: return launch_typed<float, 64>(w, P, stream);
  }
  set_error("edge_attn: unsupported padded head dim %d", dp);
  return kUnsupported;
}

}  // namespace attn
}  // namespace cg
