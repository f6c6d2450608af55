// Envelope-pooled token attention: argument checks, the C entry points and
// the fp32-precision instantiations (pooled_attn.cuh).
#include "pooled_attn.cuh"

namespace cg {
namespace pooled {

int launch_fp32(int which, const PParams& P, int dp, cudaStream_t stream) {
  return launch_prec<true>(which, P, dp, stream);
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Whether the per-atom row kernels (one warp per atom over all heads, 16-byte
// column groups) apply: d % 4 == 0, h*d a multiple of 128 and at most
// 128 * kOutRowsQMax, 16-byte aligned qkv rows.
static bool rows_eligible(const cg_pooled_attn_args& a) {
  const int64_t C = (int64_t)a.h * a.d;
  return a.d % 4 == 0 && C % 128 == 0 && C / 128 <= kOutRowsQMax && a.ld_qkv % 4 == 0 && al16(a.qkv);
}

static unsigned rows_grid(int64_t n) {
  const int64_t blocks = (n + kOutRowsWarps - 1) / kOutRowsWarps;
  const int64_t cap = (int64_t)sm_count() * 8;
  return (unsigned)(blocks < cap ? blocks : cap);
}

// out[n, :] = sum_j w_j v_j for every head, from the weights w.
static int launch_out(const cg_pooled_attn_args& a, cudaStream_t s) {
  if (rows_eligible(a) && al16(a.out)) {
    const size_t smem = (size_t)kOutRowsWarps * a.h * a.k * sizeof(float);
    CG_REQUIRE(smem <= 48 * 1024, "pooled_attn_out: h * k too large (%d x %d)", a.h, a.k);
    pooled_out_rows_kernel<<<rows_grid(a.n), 32 * kOutRowsWarps, smem, s>>>(a);
  } else {
    const int64_t warps = a.n * a.h;
    const int64_t blocks = (warps * 32 + 255) / 256;
    const int64_t cap = (int64_t)sm_count() * 16;
    pooled_out_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, s>>>(a);
  }
  CG_LAUNCHED("pooled_attn_out");
  return kOk;
}

static int run(int which, const cg_pooled_attn_args* args, void* stream) {
  CG_REQUIRE(args != nullptr, "pooled_attn: args is NULL");
  const cg_pooled_attn_args& a = *args;
  CG_REQUIRE(a.n >= 0, "pooled_attn: negative atom count");
  CG_REQUIRE(a.h >= 1, "pooled_attn: h = %d must be positive", a.h);
  CG_REQUIRE(a.k >= 1 && a.k <= attn_tc::KP, "pooled_attn: k = %d outside [1, %d]", a.k, attn_tc::KP);
  CG_REQUIRE(a.d >= 1 && a.d <= 64, "pooled_attn: d = %d outside [1, 64]", a.d);
  CG_REQUIRE(a.precision == CG_ATTN_FP32 || a.precision == CG_ATTN_TF32,
             "pooled_attn: precision = %d is neither CG_ATTN_FP32 nor CG_ATTN_TF32", a.precision);
  if (a.n == 0) return kOk;
  const int64_t C = (int64_t)a.h * a.d;
  CG_REQUIRE(a.token_index && a.key_count && a.qkv && a.env && a.lse && a.w,
             "pooled_attn: token_index, key_count, qkv, env, lse and w are required");
  CG_REQUIRE(a.ld_qkv >= 3 * C, "pooled_attn: ld_qkv = %lld below 3*h*d = %lld", (long long)a.ld_qkv,
             (long long)(3 * C));
  if (which == 0) {
    CG_REQUIRE(a.out != nullptr, "pooled_attn: out is NULL");
  } else {
    CG_REQUIRE(a.dout && a.dqk && a.wv, "pooled_attn: dout, dqk and wv are required");
    CG_REQUIRE(a.ld_dqk >= 2 * C, "pooled_attn: ld_dqk = %lld below 2*h*d", (long long)a.ld_dqk);
  }
  if (which == 2) CG_REQUIRE(a.hqkv && a.ddout, "pooled_attn: hqkv and ddout are required");
  CG_REQUIRE(a.ld_bias == 0 || a.ld_bias >= a.h, "pooled_attn: ld_bias = %lld below h", (long long)a.ld_bias);
  CG_REQUIRE(a.ld_hbias == 0 || a.ld_hbias >= a.h, "pooled_attn: ld_hbias = %lld below h", (long long)a.ld_hbias);
  const int dp = a.d <= 16 ? 16 : a.d <= 32 ? 32 : 64;
  PParams P;
  P.a = a;
  if (P.a.ld_bias == 0) P.a.ld_bias = a.h;
  if (P.a.ld_hbias == 0) P.a.ld_hbias = a.h;
  bool vec = a.d == dp && a.ld_qkv % 4 == 0 && al16(a.qkv);
  if (which == 2) vec = vec && al16(a.hqkv);
  if (which != 0) vec = vec && a.ld_dqk % 4 == 0 && al16(a.dqk) && al16(a.dout);
  P.vec = vec ? 1 : 0;
  const cudaStream_t s = as_stream(stream);
  const int rc = a.precision == CG_ATTN_TF32 ? launch_tf32(which, P, dp, s) : launch_fp32(which, P, dp, s);
  if (rc != kOk || which != 0) return rc;
  return launch_out(a, s);
}

}  // namespace pooled
}  // namespace cg

extern "C" {

int cg_pooled_attn_fwd(const cg_pooled_attn_args* a, void* stream) { return cg::pooled::run(0, a, stream); }

int cg_pooled_attn_out(const cg_pooled_attn_args* a, void* stream) {
  CG_REQUIRE(a != nullptr, "pooled_attn_out: args is NULL");
  CG_REQUIRE(a->n >= 0 && a->h >= 1 && a->k >= 1 && a->k <= cg::attn_tc::KP && a->d >= 1 && a->d <= 64,
             "pooled_attn_out: bad sizes (n %lld, h %d, k %d, d %d)", (long long)a->n, a->h, a->k, a->d);
  if (a->n == 0) return cg::kOk;
  CG_REQUIRE(a->token_index && a->key_count && a->qkv && a->w && a->out,
             "pooled_attn_out: token_index, key_count, qkv, w and out are required");
  CG_REQUIRE(a->ld_qkv >= 3 * (int64_t)a->h * a->d, "pooled_attn_out: ld_qkv below 3*h*d");
  return cg::pooled::launch_out(*a, cg::as_stream(stream));
}

int cg_pooled_attn_bwd1(const cg_pooled_attn_args* a, void* stream) { return cg::pooled::run(1, a, stream); }

int cg_pooled_attn_bwd2(const cg_pooled_attn_args* a, void* stream) { return cg::pooled::run(2, a, stream); }

}  // extern "C"
