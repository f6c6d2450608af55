// Envelope-pooled token attention (cg_pooled_attn_fwd / bwd1 / bwd2) on the
// tensor cores: the energy network's attention among the k <= 32 edge tokens
// of an atom followed by the envelope-weighted sum over tokens, fused so that
// neither the (n, k, h*d) token outputs nor their cotangents exist.
//
// One CTA of two warps owns an atom and walks its heads; per head the slice
// machinery of attn_tc.cuh applies (warp w holds query rows [16w, 16w + 16)
// as mma fragments, operands gathered through the staged token index into
// swizzled shared memory, tf32 or three-term products). What pooling changes:
// - forward: w_j = sum_i env_i P_ij is a column sum of the fragments (quad
//   shuffles over g, then the two bands in a fixed order); the forward kernel
//   writes lse and w, and out = sum_j w_j v_j follows in the output kernel
//   (one pass over each token's v row for all heads); the P v product and the
//   staging of v disappear;
// - backward1: the token cotangent is env_i dm, so grad_probs = env_i u_j
//   with u = V dm, dv_j = w_j dm is rank one (left to cg_segment_sum_scaled
//   as the weight w) and only S, dq and dk are products;
// - backward2: 7 products instead of 11 (S, the two halves of d_logits, dq
//   and dk twice), the rest row or column sums and a per-column FMA loop for
//   d(dm).
// v and hv enter only through matrix-vector products (u = V dm, t = HV dm,
// d(dm) = V^T du + HV^T w): fp32 FMA loops read them straight from the
// per-atom rows (L2) while the q / k copies are in flight, so they are never
// staged in shared memory.
// The envelope gradient, a sum over heads, accumulates in registers across
// the head loop and leaves once per atom.
//
// Padded query rows (past k) get lse = +inf in the backward kernels, hence
// zero probabilities; their envelope weights and cotangents are zero as well.
#pragma once

#include "attn_tc.cuh"

namespace cg {
namespace pooled {

using attn_tc::band_mma;
using attn_tc::band_mma2;
using attn_tc::band_mma_reg;
using attn_tc::band_softmax;
using attn_tc::cp_async_commit;
using attn_tc::cp_async_wait;
using attn_tc::kk;
using attn_tc::KP;
using attn_tc::kThreads;
using attn_tc::ld2;
using attn_tc::Layout;
using attn_tc::put_band;
using attn_tc::quad_sum;
using attn_tc::store_band;
using attn_tc::zero;

struct PParams {
  cg_pooled_attn_args a;
  int vec;  // 16-byte operand rows and 8-byte output pairs (d equal to the padded width)
};

// per-token [dq | dk] rows (n*k, ld): part 0 dq, part 1 dk
__device__ __forceinline__ cg_mat token_mat(float* dqk, int part, int64_t C, int k, int d, int64_t ld) {
  cg_mat m;
  m.ptr = dqk + part * C;
  m.sn = (int64_t)k * ld;
  m.sh = d;
  m.sr = ld;
  return m;
}

// Column sums over the band's 16 rows of a k x k fragment matrix (rows g
// and g + 8 first, then a butterfly over g): lanes 0..3 write the 32
// column sums of the band to dst.
__device__ __forceinline__ void band_colsum(float* dst, const float (&v)[4][4], int g, int t) {
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int e1 = 0; e1 < 2; ++e1) {
      float x = v[nt][e1] + v[nt][2 + e1];
      x += __shfl_xor_sync(0xffffffffu, x, 4);
      x += __shfl_xor_sync(0xffffffffu, x, 8);
      x += __shfl_xor_sync(0xffffffffu, x, 16);
      if (g == 0) dst[nt * 8 + 2 * t + e1] = x;
    }
}

// Sum over rows of one column of a k x k matrix in shared memory (fixed order).
__device__ __forceinline__ float smem_colsum(const float* M, int j) {
  float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int i = 0; i < KP; i += 4)
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] += M[kk(i + q, j)];
  return (v[0] + v[1]) + (v[2] + v[3]);
}

__device__ __forceinline__ int key_count(const cg_pooled_attn_args& a, int64_t n) {
  const int c = a.key_count[n];
  return c < 0 ? 0 : (c > a.k ? a.k : c);
}

// per-token vector of the atom (env, henv) into shared memory, zeros past k
__device__ __forceinline__ void load_tokens(float* s, const float* src, int64_t n, int k) {
  if (threadIdx.x < KP) s[threadIdx.x] = (src != nullptr && (int)threadIdx.x < k) ? src[n * k + threadIdx.x] : 0.0f;
}

// key row of a per-key (n*k, h) matrix (row pitch ld) for head hh, zeros past
// k (or all zeros)
__device__ __forceinline__ void load_key_row(float* s, const float* src, int64_t n, int hh, int k, int64_t ld) {
  if (threadIdx.x < KP)
    s[threadIdx.x] = (src != nullptr && (int)threadIdx.x < k) ? src[(n * k + threadIdx.x) * ld + hh] : 0.0f;
}

// Float offsets of the atom's token rows in the per-atom row matrices
// (token_index * ld, -1 for padding and past k), staged once per atom and
// shared by every operand and head.
__device__ __forceinline__ void stage_rows(int64_t* srow, const int32_t* token_index, int64_t n, int k, int64_t ld) {
  if (threadIdx.x < KP) {
    const int32_t j = (int)threadIdx.x < k ? token_index[n * k + threadIdx.x] : -1;
    srow[threadIdx.x] = j < 0 ? -1 : (int64_t)j * ld;
  }
}

// k x d operand gathered from base + srow[r] (base = rows + part*C + h*d) into
// shared memory: 16-byte cp.async copies (vec) or scalar loads; zero rows and
// columns past d.
template <int DP>
__device__ __forceinline__ void load_rows_async(float* s, const float* base, const int64_t* srow, int d, bool vec) {
  using L = Layout<DP>;
  if (vec) {
    constexpr int VPR = DP / 4;
    for (int f = threadIdx.x; f < KP * VPR; f += kThreads) {
      const int r = f / VPR, c = (f % VPR) * 4;
      const int64_t off = srow[r];
      attn_tc::cp_async16(s + L::op(r, c), off >= 0 ? base + off + c : base, off >= 0 ? 16 : 0);
    }
  } else {
    for (int f = threadIdx.x; f < KP * DP; f += kThreads) {
      const int r = f / DP, c = f % DP;
      const int64_t off = srow[r];
      s[L::op(r, c)] = (off >= 0 && c < d) ? base[off + c] : 0.0f;
    }
  }
}

// Two operands with the same rows (q and k, or hq and hk) in one pass: the
// row offset, the swizzled destination and the predicate of a 16-byte chunk
// serve both copies.
template <int DP>
__device__ __forceinline__ void load_rows2_async(float* s1, const float* b1, float* s2, const float* b2,
                                                 const int64_t* srow, int d, bool vec) {
  using L = Layout<DP>;
  if (!vec) {
    load_rows_async<DP>(s1, b1, srow, d, false);
    load_rows_async<DP>(s2, b2, srow, d, false);
    return;
  }
  constexpr int VPR = DP / 4;
  for (int f = threadIdx.x; f < KP * VPR; f += kThreads) {
    const int r = f / VPR, c = (f % VPR) * 4;
    const int64_t off = srow[r];
    const int so = L::op(r, c);
    const bool ok = off >= 0;
    attn_tc::cp_async16(s1 + so, ok ? b1 + off + c : b1, ok ? 16 : 0);
    attn_tc::cp_async16(s2 + so, ok ? b2 + off + c : b2, ok ? 16 : 0);
  }
}

// u_j = row_j . x for the atom's tokens, read straight from the per-atom rows
// (L2) while the operand copies are in flight: two threads per token j =
// tid / 2 (alternate 4-column chunks, then one shuffle), zero for padding
// and past k. vec: 16-byte rows and x, d == DP; its loop has a compile-time
// trip count and is unrolled, so a thread's loads are in flight together.
template <int DP>
__device__ __forceinline__ void token_dots(float* out, const float* base, const int64_t* srow, const float* x, int d,
                                           bool vec) {
  const int j = threadIdx.x >> 1, half = threadIdx.x & 1;
  const int64_t off = srow[j];
  float acc = 0.0f;
  if (off >= 0) {
    const float* row = base + off;
    if (vec) {
#pragma unroll
      for (int q = half; q < DP / 4; q += 2) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(row) + q);
        const float4 m = __ldg(reinterpret_cast<const float4*>(x) + q);
        acc += v.x * m.x + v.y * m.y + v.z * m.z + v.w * m.w;
      }
    } else {
      for (int c = half; c < d; c += 2) acc += __ldg(row + c) * __ldg(x + c);
    }
  }
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  if (half == 0) out[j] = acc;
}

#define CG_A_ROWS(X) [&](int m, int c) { return ld2(X, L::op(band * 16 + m, c)); }
#define CG_B_ROWS(X) [&](int c, int j) { return ld2(X, L::op(j, c)); }
#define CG_B_COLS(X) [&](int j, int c) { return make_float2(X[L::op(j, c)], X[L::op(j + 1, c)]); }
#define CG_A_KKT(M) [&](int m, int i) { return make_float2(M[kk(i, band * 16 + m)], M[kk(i + 1, band * 16 + m)]); }

// ---------------------------------------------------------------------------

template <int DP, bool X3>
// 12 CTAs per SM (the shared-memory limit): registers capped at 85, no spills
__global__ void __launch_bounds__(kThreads, 12) pooled_fwd(const PParams P) {
  using L = Layout<DP>;
  extern __shared__ __align__(16) float smem[];
  float* sQ = smem;
  float* sK = sQ + L::OP;
  float* sB = sK + L::OP;  // key bias row
  float* sE = sB + KP;     // env of the atom's tokens
  float* sW = sE + KP;     // band partials of w: [2][KP], then w in the first row
  int64_t* sRow = reinterpret_cast<int64_t*>(sW + 2 * KP);
  const cg_pooled_attn_args& a = P.a;
  const int k = a.k, d = a.d, H = a.h;
  const int64_t C = (int64_t)H * d;
  const float scale = (float)a.scale;
  const bool vec = P.vec;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int band = warp;
  for (int64_t n = blockIdx.x; n < a.n; n += gridDim.x) {
    __syncthreads();
    stage_rows(sRow, a.token_index, n, k, a.ld_qkv);
    load_tokens(sE, a.env, n, k);
    __syncthreads();
    const int kc = key_count(a, n);
    for (int hh = 0; hh < H; ++hh) {
      if (hh > 0) __syncthreads();  // the previous head is done with shared memory
      load_rows2_async<DP>(sQ, a.qkv + (int64_t)hh * d, sK, a.qkv + C + (int64_t)hh * d, sRow, d, vec);
      load_key_row(sB, a.bias, n, hh, k, a.ld_bias);
      cp_async_commit();
      cp_async_wait<0>();
      __syncthreads();
      float S[4][4], p[4][4], lse[2];
      zero(S);
      band_mma<X3, 4, DP / 8, true>(S, CG_A_ROWS(sQ), CG_B_ROWS(sK), g, t);
      band_softmax<!X3>(p, S, sB, 0, band, g, t, scale, kc, nullptr, lse);
      const float e0 = sE[band * 16 + g], e1 = sE[band * 16 + g + 8];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) S[nt][e] = p[nt][e] * (e < 2 ? e0 : e1);  // env_i P_ij
      band_colsum(sW + band * KP, S, g, t);
      if (t == 0) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int r = band * 16 + g + 8 * half;
          if (r < k) a.lse[(n * H + hh) * k + r] = lse[half];
        }
      }
      __syncthreads();  // both bands' partials of w visible
      if (threadIdx.x < KP) {
        const float wj = sW[threadIdx.x] + sW[KP + threadIdx.x];
        if ((int)threadIdx.x < k) a.w[(n * H + hh) * k + threadIdx.x] = wj;
      }
      // out = sum_j w_j v_j is formed afterwards from w (pooled_out_*_kernel),
      // one pass over each token's whole v row for all heads
    }
  }
}

template <int DP, bool X3>
// 10 CTAs per SM: registers capped at 96 (no spills), shared memory 21 KB per CTA
__global__ void __launch_bounds__(kThreads, 10) pooled_bwd1(const PParams P) {
  using L = Layout<DP>;
  extern __shared__ __align__(16) float smem[];
  float* sQ = smem;
  float* sK = sQ + L::OP;
  float* sGL = sK + L::OP;   // grad_logits
  float* sB = sGL + L::KK;   // key bias row
  float* sE = sB + KP;       // env
  float* sU = sE + KP;       // u = V dm
  float* sW = sU + KP;       // w
  float* sLse = sW + KP;     // lse (+inf past k)
  int64_t* sRow = reinterpret_cast<int64_t*>(sLse + KP);
  const cg_pooled_attn_args& a = P.a;
  const int k = a.k, d = a.d, H = a.h;
  const int64_t C = (int64_t)H * d;
  const float scale = (float)a.scale;
  const bool vec = P.vec;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int band = warp;
  const cg_mat tq = token_mat(a.dqk, 0, C, k, d, a.ld_dqk), tk = token_mat(a.dqk, 1, C, k, d, a.ld_dqk);
  for (int64_t n = blockIdx.x; n < a.n; n += gridDim.x) {
    __syncthreads();
    stage_rows(sRow, a.token_index, n, k, a.ld_qkv);
    load_tokens(sE, a.env, n, k);
    __syncthreads();
    const int kc = key_count(a, n);
    float denv[2] = {0.0f, 0.0f};
    for (int hh = 0; hh < H; ++hh) {
      if (hh > 0) __syncthreads();
      const float* hq = a.qkv + (int64_t)hh * d;
      load_rows2_async<DP>(sQ, hq, sK, hq + C, sRow, d, vec);
      cp_async_commit();
      load_key_row(sB, a.bias, n, hh, k, a.ld_bias);
      if (threadIdx.x < KP) {
        const int i = threadIdx.x;
        sLse[i] = i < k ? a.lse[(n * H + hh) * k + i] : INFINITY;
        sW[i] = i < k ? a.w[(n * H + hh) * k + i] : 0.0f;
      }
      token_dots<DP>(sU, hq + 2 * C, sRow, a.dout + n * C + (int64_t)hh * d, d, vec);  // u = V dm
      cp_async_wait<0>();
      __syncthreads();
      float S[4][4], p[4][4], lse[2];
      zero(S);
      band_mma<X3, 4, DP / 8, true>(S, CG_A_ROWS(sQ), CG_B_ROWS(sK), g, t);
      band_softmax<!X3>(p, S, sB, 0, band, g, t, scale, kc, sLse, lse);
      float uc[4][2];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const float2 u2 = ld2(sU, nt * 8 + 2 * t);
        uc[nt][0] = u2.x;
        uc[nt][1] = u2.y;
      }
      const float er[2] = {sE[band * 16 + g], sE[band * 16 + g + 8]};
      float ubar[2];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float s = 0.0f;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) s += p[nt][2 * half] * uc[nt][0] + p[nt][2 * half + 1] * uc[nt][1];
        ubar[half] = quad_sum(s);
        denv[half] += ubar[half];
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) S[nt][e] = er[e >> 1] * p[nt][e] * (uc[nt][e & 1] - ubar[e >> 1]);  // dL
      float O[DP / 8][4];
      zero(O);  // dq = scale dL k
      band_mma_reg<X3, DP / 8>(O, S, CG_B_COLS(sK), g, t);
      store_band<DP / 8>(tq, n, hh, band, k, d, O, g, t, scale, vec);
      put_band(sGL, S, band, g, t);
      __syncthreads();
      zero(O);  // dk = scale dL^T q
      band_mma<X3, DP / 8, 4, true>(O, CG_A_KKT(sGL), CG_B_COLS(sQ), g, t);
      store_band<DP / 8>(tk, n, hh, band, k, d, O, g, t, scale, vec);
      if (warp == 0) {
        if (a.dbias != nullptr) {
          const float db = smem_colsum(sGL, lane);
          if (lane < k) a.dbias[(n * k + lane) * H + hh] = db;
        }
      } else if (lane < k) {
        a.wv[(n * k + lane) * H + hh] = sW[lane];
      }
    }
    if (t == 0 && a.denv != nullptr) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int r = band * 16 + g + 8 * half;
        if (r < k) a.denv[n * k + r] = denv[half];
      }
    }
  }
}

template <int DP, bool X3>
__global__ void __launch_bounds__(kThreads) pooled_bwd2(const PParams P) {
  using L = Layout<DP>;
  extern __shared__ __align__(16) float smem[];
  // grad_logits and d_scores take the places of k and hk, dead once dq is
  // done; those two slots hold the larger of a k x d operand and a k x k matrix
  constexpr int SLOT = L::OP > L::KK ? L::OP : L::KK;
  float* sQ = smem;
  float* sK = sQ + L::OP;
  float* sHQ = sK + SLOT;
  float* sHK = sHQ + L::OP;
  float* sGL = sK;           // grad_logits dL
  float* sDS = sHK;          // d_scores
  float* sB = sHK + SLOT;    // key bias row
  float* sHB = sB + KP;      // key row of the dbias cotangent
  float* sE = sHB + KP;      // env
  float* sHE = sE + KP;      // denv cotangent
  float* sU = sHE + KP;      // u = V dm
  float* sT = sU + KP;       // t = HV dm
  float* sW = sT + KP;       // w
  float* sLse = sW + KP;     // lse (+inf past k)
  float* sDu = sLse + KP;    // band partials of du: [2][KP]
  int64_t* sRow = reinterpret_cast<int64_t*>(sDu + 2 * KP);
  const cg_pooled_attn_args& a = P.a;
  const int k = a.k, d = a.d, H = a.h;
  const int64_t C = (int64_t)H * d;
  const float scale = (float)a.scale;
  const bool vec = P.vec;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int band = warp;
  const cg_mat tq = token_mat(a.dqk, 0, C, k, d, a.ld_dqk), tk = token_mat(a.dqk, 1, C, k, d, a.ld_dqk);
  for (int64_t n = blockIdx.x; n < a.n; n += gridDim.x) {
    __syncthreads();
    stage_rows(sRow, a.token_index, n, k, a.ld_qkv);
    load_tokens(sE, a.env, n, k);
    load_tokens(sHE, a.henv, n, k);
    __syncthreads();
    const int kc = key_count(a, n);
    float denv[2] = {0.0f, 0.0f};
    for (int hh = 0; hh < H; ++hh) {
      if (hh > 0) __syncthreads();
      const float* hq = a.qkv + (int64_t)hh * d;
      const float* nq = a.hqkv + (int64_t)hh * d;
      load_rows2_async<DP>(sQ, hq, sK, hq + C, sRow, d, vec);
      load_rows2_async<DP>(sHQ, nq, sHK, nq + C, sRow, d, vec);
      cp_async_commit();
      load_key_row(sB, a.bias, n, hh, k, a.ld_bias);
      load_key_row(sHB, a.hbias, n, hh, k, a.ld_hbias);
      if (threadIdx.x < KP) {
        const int i = threadIdx.x;
        sLse[i] = i < k ? a.lse[(n * H + hh) * k + i] : INFINITY;
        sW[i] = i < k ? a.w[(n * H + hh) * k + i] : 0.0f;
      }
      const float* dm = a.dout + n * C + (int64_t)hh * d;
      token_dots<DP>(sU, hq + 2 * C, sRow, dm, d, vec);  // u = V dm
      token_dots<DP>(sT, nq + 2 * C, sRow, dm, d, vec);  // t = HV dm
      cp_async_wait<0>();
      __syncthreads();
      float S[4][4], A[4][4], p[4][4], lse[2];
      zero(S);  // scores
      zero(A);  // d_logits = scale (hq k^T + q hk^T) + hb
      band_mma2<X3, 4, DP / 8>(S, CG_A_ROWS(sQ), CG_B_ROWS(sK), A, CG_A_ROWS(sHQ), CG_B_ROWS(sK), g, t);
      band_mma<X3, 4, DP / 8>(A, CG_A_ROWS(sQ), CG_B_ROWS(sHK), g, t);
      band_softmax<!X3>(p, S, sB, 0, band, g, t, scale, kc, sLse, lse);
      float uc[4][2], tc[4][2];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const float2 u2 = ld2(sU, nt * 8 + 2 * t), t2 = ld2(sT, nt * 8 + 2 * t), b2 = ld2(sHB, nt * 8 + 2 * t);
        uc[nt][0] = u2.x;
        uc[nt][1] = u2.y;
        tc[nt][0] = t2.x;
        tc[nt][1] = t2.y;
        A[nt][0] = scale * A[nt][0] + b2.x;
        A[nt][1] = scale * A[nt][1] + b2.y;
        A[nt][2] = scale * A[nt][2] + b2.x;
        A[nt][3] = scale * A[nt][3] + b2.y;
      }
      const float er[2] = {sE[band * 16 + g], sE[band * 16 + g + 8]};
      const float hr[2] = {sHE[band * 16 + g], sHE[band * 16 + g + 8]};
      float ubar[2], abar[2];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float su = 0.0f, sa = 0.0f;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
          for (int e1 = 0; e1 < 2; ++e1) {
            su += p[nt][2 * half + e1] * uc[nt][e1];
            sa += p[nt][2 * half + e1] * A[nt][2 * half + e1];
          }
        ubar[half] = quad_sum(su);
        abar[half] = quad_sum(sa);
      }
      // dL (into S), X = P (env (A - abar) + henv), G_P (into A), and the
      // envelope row sums de_i = sum_j P ((u - ubar) A + t)
      float X[4][4], dep[2] = {0.0f, 0.0f};
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = e >> 1;
          const float u = uc[nt][e & 1], tt = tc[nt][e & 1], pv = p[nt][e], av = A[nt][e];
          const float du = u - ubar[r];
          S[nt][e] = er[r] * pv * du;
          X[nt][e] = pv * (er[r] * (av - abar[r]) + hr[r]);
          dep[r] += pv * (du * av + tt);
          A[nt][e] = er[r] * (du * av + tt - abar[r] * u) + hr[r] * u;
        }
      float gbar[2];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float sg = 0.0f;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
          for (int e1 = 0; e1 < 2; ++e1) sg += p[nt][2 * half + e1] * A[nt][2 * half + e1];
        gbar[half] = quad_sum(sg);
        denv[half] += quad_sum(dep[half]);
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) A[nt][e] = p[nt][e] * (A[nt][e] - gbar[e >> 1]);  // d_scores
      band_colsum(sDu + band * KP, X, g, t);
      float O[DP / 8][4];
      zero(O);  // dq = scale (dL hk + d_scores k)
      band_mma_reg<X3, DP / 8>(O, S, CG_B_COLS(sHK), g, t);
      band_mma_reg<X3, DP / 8>(O, A, CG_B_COLS(sK), g, t);
      store_band<DP / 8>(tq, n, hh, band, k, d, O, g, t, scale, vec);
      __syncthreads();  // both warps are done with k and hk
      put_band(sGL, S, band, g, t);
      put_band(sDS, A, band, g, t);
      __syncthreads();
      zero(O);  // dk = scale (dL^T hq + d_scores^T q)
      band_mma<X3, DP / 8, 4>(O, CG_A_KKT(sGL), CG_B_COLS(sHQ), g, t);
      band_mma<X3, DP / 8, 4>(O, CG_A_KKT(sDS), CG_B_COLS(sQ), g, t);
      store_band<DP / 8>(tk, n, hh, band, k, d, O, g, t, scale, vec);
      if (warp == 0) {
        if (a.dbias != nullptr) {
          const float db = smem_colsum(sDS, lane);
          if (lane < k) a.dbias[(n * k + lane) * H + hh] = db;
        }
      } else if (lane < k) {
        a.wv[(n * k + lane) * H + hh] = sDu[lane] + sDu[KP + lane];
      }
      // d(dm)_c = sum_j du_j v_jc + w_j hv_jc over the valid keys (du_j = w_j = 0
      // past kc), v and hv read straight from the atom rows (coalesced over c)
      const float* vb = hq + 2 * C;
      const float* hvb = nq + 2 * C;
      for (int c = threadIdx.x; c < d; c += kThreads) {
        float acc = 0.0f;
#pragma unroll 4
        for (int j = 0; j < kc; ++j) {
          const int64_t off = sRow[j];
          if (off >= 0) acc += (sDu[j] + sDu[KP + j]) * __ldg(vb + off + c) + sW[j] * __ldg(hvb + off + c);
        }
        a.ddout[n * C + (int64_t)hh * d + c] = acc;
      }
    }
    if (t == 0 && a.denv != nullptr) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int r = band * 16 + g + 8 * half;
        if (r < k) a.denv[n * k + r] = denv[half];
      }
    }
  }
}

// out[n, h*d + c] = sum_{j < kc} w[n, h, j] v_j[h*d + c] over the atom's valid
// keys, v_j read from the per-atom rows through the token index: the forward's
// output for known weights w (a checkpoint recompute of the same inputs reuses
// the first forward's w and lse). One warp per (atom, head), lanes over the
// columns; the sum runs in the forward kernel's order with its arithmetic, so
// the result equals the forward's output bit for bit.
static __global__ void pooled_out_kernel(const cg_pooled_attn_args a) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int k = a.k, d = a.d, H = a.h;
  const int64_t C = (int64_t)H * d;
  // d = 64 on 16-byte aligned rows: each lane owns two adjacent columns
  const bool pairs = d == 64 && (a.ld_qkv & 1) == 0 && (reinterpret_cast<uintptr_t>(a.qkv) & 7) == 0 &&
                     (reinterpret_cast<uintptr_t>(a.out) & 7) == 0;
  for (int64_t task = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; task < a.n * H; task += warps) {
    const int64_t n = task / H;
    const int hh = (int)(task % H);
    const int kc = key_count(a, n);
    // the atom's token rows and this head's weights, one per lane, then broadcast
    const int32_t my_t = lane < k ? a.token_index[n * k + lane] : -1;
    const float my_w = lane < k ? a.w[(n * H + hh) * k + lane] : 0.0f;
    const float* vbase = a.qkv + 2 * C + (int64_t)hh * d;
    float* dst = a.out + n * C + (int64_t)hh * d;
    if (pairs) {
      float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll 8
      for (int j = 0; j < kc; ++j) {
        const int32_t t = __shfl_sync(0xffffffffu, my_t, j);
        const float wj = __shfl_sync(0xffffffffu, my_w, j);
        if (t >= 0) {
          const float2 v = __ldg(reinterpret_cast<const float2*>(vbase + (int64_t)t * a.ld_qkv) + lane);
          acc0 += wj * v.x;
          acc1 += wj * v.y;
        }
      }
      reinterpret_cast<float2*>(dst)[lane] = make_float2(acc0, acc1);
    } else {
      for (int c0 = 0; c0 < d; c0 += 32) {
        const int c = c0 + lane;
        float acc = 0.0f;
        for (int j = 0; j < kc; ++j) {
          const int32_t t = __shfl_sync(0xffffffffu, my_t, j);
          const float wj = __shfl_sync(0xffffffffu, my_w, j);
          if (t >= 0 && c < d) acc += wj * __ldg(vbase + (int64_t)t * a.ld_qkv + c);
        }
        if (c < d) dst[c] = acc;
      }
    }
  }
}

// The same output for all heads at once when every head's columns split into
// 16-byte groups (d % 4 == 0, h*d a multiple of 128, aligned rows): one warp
// per atom reads each valid token's whole v row (h*d contiguous floats) once
// with coalesced 16-byte loads, lane l owning column groups l, l + 32, ...
// (QMAX at most), with the atom's weights w[n, :, :] staged in shared memory.
// Per column the sum runs over j ascending with the forward kernel's
// arithmetic, so the result equals the forward's output bit for bit.
constexpr int kOutRowsWarps = 8;
constexpr int kOutRowsQMax = 8;  // h*d <= 1024

static __global__ void __launch_bounds__(32 * kOutRowsWarps) pooled_out_rows_kernel(const cg_pooled_attn_args a) {
  extern __shared__ float sw_all[];  // kOutRowsWarps x (h*k)
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int k = a.k, d = a.d, H = a.h;
  const int64_t C = (int64_t)H * d;
  const int q_count = (int)(C / 128);
  float* sw = sw_all + wid * H * k;
  int hk[kOutRowsQMax];
#pragma unroll
  for (int q = 0; q < kOutRowsQMax; ++q) hk[q] = q < q_count ? (4 * (lane + 32 * q)) / d * k : 0;
  const int64_t warps = (int64_t)gridDim.x * kOutRowsWarps;
  for (int64_t n = blockIdx.x * (int64_t)kOutRowsWarps + wid; n < a.n; n += warps) {
    const int kc = key_count(a, n);
    const int32_t my_t = lane < k ? a.token_index[n * k + lane] : -1;
    __syncwarp();  // the previous atom's weights are no longer read
    for (int i = lane; i < H * k; i += 32) sw[i] = a.w[n * H * k + i];
    __syncwarp();
    float4 acc[kOutRowsQMax];
#pragma unroll
    for (int q = 0; q < kOutRowsQMax; ++q) acc[q] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const float4* vbase = reinterpret_cast<const float4*>(a.qkv + 2 * C);
    for (int j = 0; j < kc; ++j) {
      const int32_t t = __shfl_sync(0xffffffffu, my_t, j);
      if (t < 0) continue;
      const float4* vrow = vbase + (int64_t)t * (a.ld_qkv / 4);
#pragma unroll
      for (int q = 0; q < kOutRowsQMax; ++q) {
        if (q < q_count) {
          const float wj = sw[hk[q] + j];
          const float4 v = __ldg(vrow + lane + 32 * q);
          acc[q].x += wj * v.x;
          acc[q].y += wj * v.y;
          acc[q].z += wj * v.z;
          acc[q].w += wj * v.w;
        }
      }
    }
    float4* dst = reinterpret_cast<float4*>(a.out + n * C);
#pragma unroll
    for (int q = 0; q < kOutRowsQMax; ++q)
      if (q < q_count) dst[lane + 32 * q] = acc[q];
  }
}

#undef CG_A_ROWS
#undef CG_B_ROWS
#undef CG_B_COLS
#undef CG_A_KKT

// shared memory per CTA (bytes); which: 0 fwd, 1 bwd1, 2 bwd2
template <int DP>
inline int smem_bytes(int which) {
  using L = Layout<DP>;
  switch (which) {
    case 0: return (2 * L::OP + 4 * KP + 2 * KP) * 4;
    case 1: return (2 * L::OP + L::KK + 5 * KP + 2 * KP) * 4;
    default: return (2 * L::OP + 2 * (L::OP > L::KK ? L::OP : L::KK) + 10 * KP + 2 * KP) * 4;
  }
}

// A persistent grid of as many CTAs as fit per SM, atoms strided over it.
template <int DP, bool X3>
int launch_dp(int which, const PParams& P, cudaStream_t stream) {
  const int smem = smem_bytes<DP>(which);
  void (*kernel)(const PParams) =
      which == 0 ? pooled_fwd<DP, X3> : which == 1 ? pooled_bwd1<DP, X3> : pooled_bwd2<DP, X3>;
  CG_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  int per_sm = (228 * 1024) / (smem + 1024);
  if (per_sm < 1) per_sm = 1;
  if (per_sm > 16) per_sm = 16;
  const int64_t cap = (int64_t)sm_count() * per_sm;
  const int grid = (int)(P.a.n < cap ? P.a.n : cap);
  kernel<<<grid, kThreads, smem, stream>>>(P);
  CG_LAUNCHED("pooled_attn");
  return kOk;
}

template <bool X3>
int launch_prec(int which, const PParams& P, int dp, cudaStream_t stream) {
  switch (dp) {
    case 16: return launch_dp<16, X3>(which, P, stream);
    case 32: return launch_dp<32, X3>(which, P, stream);
    case 64: return launch_dp<64, X3>(which, P, stream);
  }
  set_error("pooled_attn: no variant for padded head dim %d", dp);
  return kUnsupported;
}

int launch_fp32(int which, const PParams& P, int dp, cudaStream_t stream);  // pooled_attn.cu
int launch_tf32(int which, const PParams& P, int dp, cudaStream_t stream);  // pooled_attn_tf32.cu

}  // namespace pooled
}  // namespace cg
