// Masked edge attention: argument checks and the C entry points. float32 runs
// the tensor-core kernels (attn_tc.cuh); float64 the CUDA-core kernels of
// edge_attn.cuh (edge_attn_f64.cu), kept for 1e-10 parity with the reference.
#include "edge_attn.cuh"

namespace cg {
namespace attn_tc {
int launch(int which, const cg_edge_attn_args& a, int dbias_mode, int ki, int kj, int vec_ok, int dp,
           cudaStream_t stream);
}
namespace attn {

static int run(Which w, const cg_edge_attn_args* args, void* stream) {
  CG_REQUIRE(args != nullptr, "edge_attn: args is NULL");
  const cg_edge_attn_args& a = *args;
  CG_REQUIRE(a.dtype == CG_F32 || a.dtype == CG_F64, "edge_attn: dtype must be CG_F32 or CG_F64");
  CG_REQUIRE(a.n >= 0 && a.h >= 0, "edge_attn: negative slice grid");
  CG_REQUIRE(a.k >= 1 && a.k <= KMAX, "edge_attn: k = %d outside [1, %d]", a.k, KMAX);
  const int dp = padded_d(a.d, a.dtype);
  CG_REQUIRE(a.d >= 1 && dp > 0, "edge_attn: d = %d outside [1, %d]", a.d,
             a.dtype == CG_F32 ? 64 : 16);
  if (a.n * a.h == 0) return kOk;
  int rc;
  if ((rc = check_mat(a.q, "q", true)) || (rc = check_mat(a.k_, "k", true)) ||
      (rc = check_mat(a.v, "v", true)))
    return rc;
  CG_REQUIRE(a.lse != nullptr, "edge_attn: lse is NULL");
  if (w == kFwd1) {
    if ((rc = check_mat(a.out, "out", true))) return rc;
  } else {
    if ((rc = check_mat(a.grad_out, "grad_out", true)) || (rc = check_mat(a.dq, "dq", true)) ||
        (rc = check_mat(a.dk, "dk", true)) || (rc = check_mat(a.dv, "dv", true)))
      return rc;
  }
  if (w == kBwd2) {
    if ((rc = check_mat(a.hq, "hq", true)) || (rc = check_mat(a.hk, "hk", true)) ||
        (rc = check_mat(a.hv, "hv", true)) || (rc = check_mat(a.dgrad_out, "dgrad_out", true)))
      return rc;
  }
  CG_REQUIRE(a.token_index == nullptr || a.dtype == CG_F32, "edge_attn: token_index needs float32");
  CG_REQUIRE(a.precision == CG_ATTN_FP32 || a.precision == CG_ATTN_TF32,
             "edge_attn: precision = %d is neither CG_ATTN_FP32 nor CG_ATTN_TF32", a.precision);
  Params P;
  P.a = a;
  const int es = a.dtype == CG_F32 ? 4 : 8;
  bool vec = mat_vec_ok(a.q, es, a.d, dp) && mat_vec_ok(a.k_, es, a.d, dp) &&
             mat_vec_ok(a.v, es, a.d, dp) && mat_vec_ok(a.out, es, a.d, dp) &&
             mat_vec_ok(a.grad_out, es, a.d, dp) && mat_vec_ok(a.hq, es, a.d, dp) &&
             mat_vec_ok(a.hk, es, a.d, dp) && mat_vec_ok(a.hv, es, a.d, dp) &&
             mat_vec_ok(a.dq, es, a.d, dp) && mat_vec_ok(a.dk, es, a.d, dp) &&
             mat_vec_ok(a.dv, es, a.d, dp) && mat_vec_ok(a.dgrad_out, es, a.d, dp);
  P.vec_ok = vec ? 1 : 0;
  P.dbias_mode = kNoDbias;
  P.ki = P.kj = 1;
  if (w != kFwd1 && a.bias.ptr != nullptr && a.dbias.ptr != nullptr) {
    dbias_shape(a, &P.ki, &P.kj);
    if (dbias_cross_slice(a)) {
      CG_REQUIRE(a.scratch != nullptr,
                 "edge_attn: dbias broadcasts over n or h and needs scratch "
                 "(cg_edge_attn_scratch_bytes)");
      P.dbias_mode = kDbiasScratch;
    } else {
      P.dbias_mode = kDbiasDirect;
    }
  }
  if (a.dtype == CG_F32) {
    // float32: tensor-core kernels (3-term tf32 split, fp32-level accuracy)
    const int which = w == kFwd1 ? 0 : w == kBwd1 ? 1 : 2;
    return attn_tc::launch(which, a, P.dbias_mode, P.ki, P.kj, P.vec_ok, dp, as_stream(stream));
  }
  return dispatch_f64(w, P, dp, as_stream(stream));
}

}  // namespace attn
}  // namespace cg

extern "C" {

int cg_edge_attn_fwd1(const cg_edge_attn_args* a, void* stream) {
  return cg::attn::run(cg::attn::kFwd1, a, stream);
}

int cg_edge_attn_bwd1(const cg_edge_attn_args* a, void* stream) {
  return cg::attn::run(cg::attn::kBwd1, a, stream);
}

int cg_edge_attn_bwd2(const cg_edge_attn_args* a, void* stream) {
  return cg::attn::run(cg::attn::kBwd2, a, stream);
}

int64_t cg_edge_attn_scratch_bytes(const cg_edge_attn_args* a) {
  if (a == nullptr || !cg::attn::dbias_cross_slice(*a) || a->dbias.ptr == nullptr) return 0;
  int ki, kj;
  cg::attn::dbias_shape(*a, &ki, &kj);
  const int64_t es = a->dtype == CG_F32 ? 4 : 8;
  return a->n * a->h * (int64_t)ki * kj * es;
}

}  // extern "C"
