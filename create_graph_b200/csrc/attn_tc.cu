// Launchers of the tensor-core edge-attention kernels (attn_tc.cuh): the
// float32 path of cg_edge_attn_fwd1 / bwd1 / bwd2, fp32-precision
// instantiations and the precision dispatch.
#include "attn_tc.cuh"

namespace cg {
namespace attn_tc {

// Sum the per-slice partial dbias over the broadcast n and/or h dimensions in
// a fixed order (deterministic), one thread per dbias element.
__global__ void dbias_reduce_tc(const Params P, int64_t outs) {
  const cg_edge_attn_args& a = P.a;
  const int64_t per = (int64_t)P.ki * P.kj;
  const bool bn = a.bias.sn == 0, bh = a.bias.sh == 0;
  const int64_t hh = bh ? 1 : a.h;
  for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < outs; o += (int64_t)gridDim.x * blockDim.x) {
    const int64_t f = o % per, nh = o / per;
    const int64_t n0 = nh / hh, h0 = nh % hh;
    const float* part = reinterpret_cast<const float*>(a.scratch);
    float v = 0.0f;
    for (int64_t n = bn ? 0 : n0; n < (bn ? a.n : n0 + 1); ++n)
      for (int64_t h = bh ? 0 : h0; h < (bh ? a.h : h0 + 1); ++h) v += part[(n * a.h + h) * per + f];
    const int i = (int)(f / P.kj), j = (int)(f % P.kj);
    const cg_bias& db = a.dbias;
    reinterpret_cast<float*>(db.ptr)[n0 * db.sn + h0 * db.sh + (int64_t)i * db.si + (int64_t)j * db.sj] = v;
  }
}

int reduce_dbias(const Params& P, cudaStream_t stream) {
  const bool bn = P.a.bias.sn == 0, bh = P.a.bias.sh == 0;
  const int64_t outs = (bn ? 1 : P.a.n) * (bh ? 1 : P.a.h) * (int64_t)P.ki * P.kj;
  const int64_t blocks = ceil_div<int64_t>(outs, 256);
  dbias_reduce_tc<<<(int)(blocks < 4096 ? blocks : 4096), 256, 0, stream>>>(P, outs);
  CG_LAUNCHED("edge_attn_tc dbias reduction");
  return kOk;
}

int launch_fp32(int which, const Params& P, int dp, cudaStream_t stream) {
  return launch_prec<true>(which, P, dp, stream);
}

// How a bias tile is staged: one key row when it broadcasts over queries
// (si == 0); 16-byte copies when its rows are contiguous, 16-byte aligned and
// k is a multiple of 4 (a copy never crosses the row's end); else scalars.
static int bias_mode(const cg_bias& b, int k) {
  if (b.ptr == nullptr) return kBiasNone;
  if (b.si == 0) return kBiasKeyRow;
  const bool vec = b.sj == 1 && k % 4 == 0 && (reinterpret_cast<uintptr_t>(b.ptr) & 15) == 0 && b.si % 4 == 0 &&
                   b.sh % 4 == 0 && b.sn % 4 == 0;
  return vec ? kBiasVec : kBiasScalar;
}

int launch(int which, const cg_edge_attn_args& a, int dbias_mode, int ki, int kj, int vec_ok, int dp,
           cudaStream_t stream) {
  Params P;
  P.a = a;
  P.dbias_mode = dbias_mode;
  P.ki = ki;
  P.kj = kj;
  // 16-byte operand loads need rows of exactly the padded width
  P.vec_ok = vec_ok && a.d == dp;
  {
    // the operands this kernel reads (null ones excepted) share their strides
    const cg_mat* mats[7] = {&a.q, &a.k_, &a.v, &a.grad_out, &a.hq, &a.hk, &a.hv};
    const int used = which == 0 ? 3 : which == 1 ? 4 : 7;
    bool same = P.vec_ok && a.token_index == nullptr;
    for (int i = 1; i < used && same; ++i)
      same = mats[i]->ptr != nullptr && mats[i]->sn == a.q.sn && mats[i]->sh == a.q.sh && mats[i]->sr == a.q.sr;
    P.same = same ? 1 : 0;
  }
  P.bias_mode = bias_mode(a.bias, a.k);
  P.hb_mode = bias_mode(a.hb, a.k);
  // full-tile dbias in 16-byte stores: contiguous aligned rows (dbias, or the
  // scratch partials of k x k per slice), k a multiple of 4
  const bool db_rows = dbias_mode == 1
                           ? a.dbias.sj == 1 && a.dbias.si % 4 == 0 && a.dbias.sh % 4 == 0 && a.dbias.sn % 4 == 0 &&
                                 (reinterpret_cast<uintptr_t>(a.dbias.ptr) & 15) == 0
                           : (reinterpret_cast<uintptr_t>(a.scratch) & 15) == 0;
  P.dbias_vec = dbias_mode != 0 && ki == a.k && kj == a.k && a.k % 4 == 0 && db_rows;
  return a.precision == CG_ATTN_TF32 ? launch_tf32(which, P, dp, stream) : launch_fp32(which, P, dp, stream);
}

}  // namespace attn_tc
}  // namespace cg
