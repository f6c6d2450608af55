// Masked edge attention: forward1 / backward1 / backward2 as fused kernels.
//
// Restates kernels/edge_attn/ops.py (reference): _scores (:26-34),
// _reduce (:37-44), _first (:47-54), forward1 (:64-68), backward1 (:75-76)
// and backward2 (:79-104). One warp owns one slice (n, h) of k <= 32 tokens:
// lane i holds query row i of every k x k matrix in registers, the k x d
// operands sit in shared memory (rows padded by 16 bytes, so a lane reading
// its own row and all lanes reading one row are both conflict-free), and the
// transposed products (dk, dv) are done by lane j over k x k matrices stored
// with a 33-element row pitch. The logits, probabilities and their
// derivatives never leave the SM: per slice the kernels read and write only
// the algorithmic bytes (each operand once).
#include <float.h>
#include <math.h>

#pragma once
#include "common.cuh"
#include "../../include/cg_b200.h"

namespace cg {
namespace attn {

constexpr int KMAX = 32;
constexpr int KLD = 33;  // row pitch of k x k matrices in shared memory

template <typename T> struct V16;
template <> struct V16<float> {
  using type = float4;
  static constexpr int n = 4;
  __device__ static inline float get(const float4& v, int c) {
    return c == 0 ? v.x : c == 1 ? v.y : c == 2 ? v.z : v.w;
  }
};
template <> struct V16<double> {
  using type = double2;
  static constexpr int n = 2;
  __device__ static inline double get(const double2& v, int c) { return c == 0 ? v.x : v.y; }
};

template <typename T> __device__ inline T exp_(T x);
template <> __device__ inline float exp_(float x) { return expf(x); }
template <> __device__ inline double exp_(double x) { return exp(x); }
template <typename T> __device__ inline T log_(T x);
template <> __device__ inline float log_(float x) { return logf(x); }
template <> __device__ inline double log_(double x) { return log(x); }
template <typename T> __device__ inline bool finite_(T x);
template <> __device__ inline bool finite_(float x) { return isfinite(x); }
template <> __device__ inline bool finite_(double x) { return isfinite(x); }
template <typename T> __device__ inline T neg_inf();
template <> __device__ inline float neg_inf() { return -INFINITY; }
template <> __device__ inline double neg_inf() { return -INFINITY; }

// How dbias is produced from the per-slice d_scores.
enum DbiasMode : int { kNoDbias = 0, kDbiasDirect = 1, kDbiasScratch = 2 };

struct Params {
  cg_edge_attn_args a;
  int dbias_mode;
  int ki, kj;          // per-slice reduced dbias shape (k or 1)
  int vec_ok;          // all k x d operands 16-byte aligned, d == padded d
};

template <typename T>
__device__ inline const T* row_ptr(const cg_mat& m, int64_t n, int64_t h, int r) {
  return reinterpret_cast<const T*>(m.ptr) + n * m.sn + h * m.sh + (int64_t)r * m.sr;
}
template <typename T>
__device__ inline T* out_row(const cg_mat& m, int64_t n, int64_t h, int r) {
  return reinterpret_cast<T*>(m.ptr) + n * m.sn + h * m.sh + (int64_t)r * m.sr;
}

// Load rows [0, k) x cols [0, d) of a slice operand into shared memory (pitch
// LD); columns [d, DP) are zero so the unguarded d-loops add nothing.
template <typename T, int DP, int LD>
__device__ inline void load_mat(T* s, const cg_mat& m, int64_t n, int64_t h, int k, int d,
                                bool vec, int lane) {
  using V = V16<T>;
  if (vec) {
    constexpr int VPR = DP / V::n;  // vectors per row
    for (int f = lane; f < k * VPR; f += 32) {
      const int r = f / VPR, c = (f % VPR) * V::n;
      *reinterpret_cast<typename V::type*>(s + r * LD + c) =
          __ldg(reinterpret_cast<const typename V::type*>(row_ptr<T>(m, n, h, r) + c));
    }
  } else {
    for (int f = lane; f < k * DP; f += 32) {
      const int r = f / DP, c = f % DP;
      s[r * LD + c] = c < d ? row_ptr<T>(m, n, h, r)[c] : T(0);
    }
  }
}

// Row r of output m for slice (n, h): computed 16 bytes at a time by `chunk`
// (a functor filling acc[0..V::n) for columns [c, c + V::n)) and stored at
// once, so no d-wide accumulator array lives in registers.
template <typename T, int DP, typename Chunk>
__device__ inline void emit_row(const cg_mat& m, int64_t n, int64_t h, int r, int d, bool vec,
                                Chunk chunk) {
  using V = V16<T>;
  T* dst = out_row<T>(m, n, h, r);
#pragma unroll 1
  for (int c = 0; c < DP; c += V::n) {
    T acc[V::n];
    chunk(c, acc);
    if (vec) {
      typename V::type v;
      if constexpr (V::n == 4) {
        v.x = acc[0]; v.y = acc[1]; v.z = acc[2]; v.w = acc[3];
      } else {
        v.x = acc[0]; v.y = acc[1];
      }
      *reinterpret_cast<typename V::type*>(dst + c) = v;
    } else {
#pragma unroll
      for (int e = 0; e < V::n; ++e)
        if (c + e < d) dst[c + e] = acc[e];
    }
  }
}

// acc[e] += sum_j w[j] * s[j][c + e] over j < k (broadcast reads of s rows).
template <typename T, int LD>
__device__ inline void combine(T* acc, const T (&w)[KMAX], const T* s, int c, int k) {
  using V = V16<T>;
#pragma unroll
  for (int j = 0; j < KMAX; ++j) {
    if (j < k) {
      const typename V::type sv = *reinterpret_cast<const typename V::type*>(s + j * LD + c);
#pragma unroll
      for (int e = 0; e < V::n; ++e) acc[e] = fma(w[j], V::get(sv, e), acc[e]);
    }
  }
}

// dots[j] = <own row x (pitch LD), row j of s> for j < k (broadcast reads of s).
template <typename T, int DP, int LD>
__device__ inline void row_dots(T (&dots)[KMAX], const T* x, const T* s, int k) {
  using V = V16<T>;
#pragma unroll
  for (int j = 0; j < KMAX; ++j) dots[j] = T(0);
#pragma unroll 1
  for (int c = 0; c < DP; c += V::n) {
    const typename V::type xv = *reinterpret_cast<const typename V::type*>(x + c);
#pragma unroll
    for (int j = 0; j < KMAX; ++j) {
      if (j < k) {
        const typename V::type sv = *reinterpret_cast<const typename V::type*>(s + j * LD + c);
#pragma unroll
        for (int e = 0; e < V::n; ++e) dots[j] = fma(V::get(xv, e), V::get(sv, e), dots[j]);
      }
    }
  }
}

// w[i] = M[i][col] for i < k (a column of a k x k matrix of pitch KLD), else 0.
template <typename T>
__device__ inline void load_col(T (&w)[KMAX], const T* M, int col, int k) {
#pragma unroll
  for (int i = 0; i < KMAX; ++i) w[i] = i < k ? M[i * KLD + col] : T(0);
}

// w[j] = M[row][j] for j < k, else 0.
template <typename T>
__device__ inline void load_row(T (&w)[KMAX], const T* M, int row, int k) {
#pragma unroll
  for (int j = 0; j < KMAX; ++j) w[j] = j < k ? M[row * KLD + j] : T(0);
}

// Bias row i of slice (n, h) into b[0..k) (0 where there is no bias).
template <typename T>
__device__ inline void bias_row(T (&b)[KMAX], const cg_bias& bias, int64_t n, int64_t h, int i,
                                int k) {
  if (bias.ptr == nullptr) {
#pragma unroll
    for (int j = 0; j < KMAX; ++j) b[j] = T(0);
    return;
  }
  const T* p = reinterpret_cast<const T*>(bias.ptr) + n * bias.sn + h * bias.sh + (int64_t)i * bias.si;
#pragma unroll
  for (int j = 0; j < KMAX; ++j) b[j] = j < k ? p[(int64_t)j * bias.sj] : T(0);
}

// logits -> probabilities of row i. With lse_in != nullptr the row's
// logsumexp is taken from it (backward kernels); otherwise computed and
// returned. Non-finite logits and keys j >= kc are masked; an all-masked
// row gets lse = -inf and zero probabilities.
template <typename T>
__device__ inline T softmax_row(T (&p)[KMAX], const T (&logit)[KMAX], int k, int kc,
                                const T* lse_in) {
  bool ok[KMAX];
  T m = neg_inf<T>();
#pragma unroll
  for (int j = 0; j < KMAX; ++j) {
    ok[j] = j < kc && finite_(logit[j]);
    if (ok[j]) m = fmax(m, logit[j]);
  }
  T lse;
  if (lse_in != nullptr) {
    lse = *lse_in;
  } else if (m == neg_inf<T>()) {
    lse = neg_inf<T>();
  } else {
    T sum = T(0);
#pragma unroll
    for (int j = 0; j < KMAX; ++j)
      if (ok[j]) sum += exp_(logit[j] - m);
    lse = m + log_(sum);
  }
  const bool row_ok = finite_(lse);
#pragma unroll
  for (int j = 0; j < KMAX; ++j) p[j] = (ok[j] && row_ok) ? exp_(logit[j] - lse) : T(0);
  return lse;
}

template <typename T>
__device__ inline void make_logits(T (&logit)[KMAX], const T (&dots)[KMAX], const T (&b)[KMAX],
                                   T scale) {
#pragma unroll
  for (int j = 0; j < KMAX; ++j) logit[j] = dots[j] * scale + b[j];
}

template <typename T>
__device__ inline int valid_keys(const Params& P, int64_t n) {
  const int k = P.a.k;
  if (P.a.key_count == nullptr) return k;
  const int c = P.a.key_count[n];
  return c < 0 ? 0 : (c > k ? k : c);
}

// Per-slice dbias (matrix M = d_scores in shared memory, pitch KLD): reduced
// over i and/or j when the bias broadcasts them, written to dbias or scratch.
template <typename T>
__device__ inline void write_dbias(const Params& P, const T* M, int64_t n, int64_t h,
                                   int64_t slice, int lane) {
  if (P.dbias_mode == kNoDbias) return;
  const int k = P.a.k;
  const int ki = P.ki, kj = P.kj;
  for (int f = lane; f < ki * kj; f += 32) {
    const int i = f / kj, j = f % kj;
    T v = T(0);
    if (ki == k && kj == k) {
      v = M[i * KLD + j];
    } else if (ki == 1 && kj == k) {
      for (int r = 0; r < k; ++r) v += M[r * KLD + j];
    } else if (ki == k && kj == 1) {
      for (int c = 0; c < k; ++c) v += M[i * KLD + c];
    } else {
      for (int r = 0; r < k; ++r)
        for (int c = 0; c < k; ++c) v += M[r * KLD + c];
    }
    if (P.dbias_mode == kDbiasDirect) {
      const cg_bias& db = P.a.dbias;
      T* dst = reinterpret_cast<T*>(db.ptr) + n * db.sn + h * db.sh + (int64_t)i * db.si +
               (int64_t)j * db.sj;
      *dst = v;
    } else {
      reinterpret_cast<T*>(P.a.scratch)[slice * (ki * kj) + f] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// forward1
// ---------------------------------------------------------------------------
template <typename T, int DP>
__global__ void __launch_bounds__(128) fwd1_kernel(const Params P) {
  constexpr int LD = DP + 16 / sizeof(T);
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  T* sQ = reinterpret_cast<T*>(smem_raw) + warp * (3 * KMAX * LD);
  T* sK = sQ + KMAX * LD;
  T* sV = sK + KMAX * LD;
  const cg_edge_attn_args& a = P.a;
  const int k = a.k, d = a.d;
  const T scale = T(a.scale);
  const int64_t slices = a.n * a.h;
  for (int64_t s = (int64_t)blockIdx.x * nw + warp; s < slices; s += (int64_t)gridDim.x * nw) {
    const int64_t n = s / a.h, h = s % a.h;
    __syncwarp();
    load_mat<T, DP, LD>(sQ, a.q, n, h, k, d, P.vec_ok, lane);
    load_mat<T, DP, LD>(sK, a.k_, n, h, k, d, P.vec_ok, lane);
    load_mat<T, DP, LD>(sV, a.v, n, h, k, d, P.vec_ok, lane);
    __syncwarp();
    const int kc = valid_keys<T>(P, n);
    const int i = lane < k ? lane : 0;
    T p[KMAX];
    T lse;
    {
      T dots[KMAX], b[KMAX];
      row_dots<T, DP, LD>(dots, sQ + i * LD, sK, k);
      bias_row<T>(b, a.bias, n, h, i, k);
#pragma unroll
      for (int j = 0; j < KMAX; ++j) dots[j] = dots[j] * scale + b[j];
      lse = softmax_row<T>(p, dots, k, kc, nullptr);
    }
    if (lane < k) {
      emit_row<T, DP>(a.out, n, h, lane, d, P.vec_ok, [&](int c, T* acc) {
#pragma unroll
        for (int e = 0; e < V16<T>::n; ++e) acc[e] = T(0);
        combine<T, LD>(acc, p, sV, c, k);
      });
      reinterpret_cast<T*>(a.lse)[s * k + lane] = lse;
    }
  }
}

// ---------------------------------------------------------------------------
// backward1
// ---------------------------------------------------------------------------
template <typename T, int DP>
__global__ void __launch_bounds__(128) bwd1_kernel(const Params P) {
  constexpr int LD = DP + 16 / sizeof(T);
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  T* sQ = reinterpret_cast<T*>(smem_raw) + warp * (4 * KMAX * LD + 2 * KMAX * KLD);
  T* sK = sQ + KMAX * LD;
  T* sV = sK + KMAX * LD;
  T* sG = sV + KMAX * LD;
  T* sP = sG + KMAX * LD;      // probs, pitch KLD
  T* sD = sP + KMAX * KLD;     // grad_logits, pitch KLD
  const cg_edge_attn_args& a = P.a;
  const int k = a.k, d = a.d;
  const T scale = T(a.scale);
  const int64_t slices = a.n * a.h;
  for (int64_t s = (int64_t)blockIdx.x * nw + warp; s < slices; s += (int64_t)gridDim.x * nw) {
    const int64_t n = s / a.h, h = s % a.h;
    __syncwarp();
    load_mat<T, DP, LD>(sQ, a.q, n, h, k, d, P.vec_ok, lane);
    load_mat<T, DP, LD>(sK, a.k_, n, h, k, d, P.vec_ok, lane);
    load_mat<T, DP, LD>(sV, a.v, n, h, k, d, P.vec_ok, lane);
    load_mat<T, DP, LD>(sG, a.grad_out, n, h, k, d, P.vec_ok, lane);
    __syncwarp();
    const int kc = valid_keys<T>(P, n);
    const int i = lane < k ? lane : 0;
    {
      T p[KMAX], gl[KMAX];
      {
        T dots[KMAX], b[KMAX];
        row_dots<T, DP, LD>(dots, sQ + i * LD, sK, k);
        bias_row<T>(b, a.bias, n, h, i, k);
#pragma unroll
        for (int j = 0; j < KMAX; ++j) dots[j] = dots[j] * scale + b[j];
        const T* lse_in = reinterpret_cast<const T*>(a.lse) + s * k + i;
        softmax_row<T>(p, dots, k, kc, lse_in);
        row_dots<T, DP, LD>(gl, sG + i * LD, sV, k);  // grad_probs = grad_out v^T
        T rs = T(0);
#pragma unroll
        for (int j = 0; j < KMAX; ++j) rs = fma(p[j], gl[j], rs);
#pragma unroll
        for (int j = 0; j < KMAX; ++j) gl[j] = p[j] * (gl[j] - rs);  // grad_logits
      }
      if (lane < k) {
        // grad_q = scale * grad_logits k
        emit_row<T, DP>(a.dq, n, h, lane, d, P.vec_ok, [&](int c, T* acc) {
#pragma unroll
          for (int e = 0; e < V16<T>::n; ++e) acc[e] = T(0);
          combine<T, LD>(acc, gl, sK, c, k);
#pragma unroll
          for (int e = 0; e < V16<T>::n; ++e) acc[e] *= scale;
        });
#pragma unroll
        for (int j = 0; j < KMAX; ++j) {
          sP[lane * KLD + j] = p[j];
          sD[lane * KLD + j] = gl[j];
        }
      }
    }
    __syncwarp();
    if (lane < k) {
      T w[KMAX];
      load_col<T>(w, sP, lane, k);  // grad_v = probs^T grad_out
      emit_row<T, DP>(a.dv, n, h, lane, d, P.vec_ok, [&](int c, T* acc) {
#pragma unroll
        for (int e = 0; e < V16<T>::n; ++e) acc[e] = T(0);
        combine<T, LD>(acc, w, sG, c, k);
      });
      load_col<T>(w, sD, lane, k);  // grad_k = scale * grad_logits^T q
      emit_row<T, DP>(a.dk, n, h, lane, d, P.vec_ok, [&](int c, T* acc) {
#pragma unroll
        for (int e = 0; e < V16<T>::n; ++e) acc[e] = T(0);
        combine<T, LD>(acc, w, sQ, c, k);
#pragma unroll
        for (int e = 0; e < V16<T>::n; ++e) acc[e] *= scale;
      });
    }
    write_dbias<T>(P, sD, n, h, s, lane);
  }
}

// ---------------------------------------------------------------------------
// backward2
// ---------------------------------------------------------------------------
template <typename T, int DP>
__global__ void __launch_bounds__(128) bwd2_kernel(const Params P) {
  constexpr int LD = DP + 16 / sizeof(T);
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  T* sQ = reinterpret_cast<T*>(smem_raw) + warp * (7 * KMAX * LD + 3 * KMAX * KLD);
  T* sK = sQ + KMAX * LD;
  T* sV = sK + KMAX * LD;
  T* sG = sV + KMAX * LD;
  T* sHQ = sG + KMAX * LD;
  T* sHK = sHQ + KMAX * LD;
  T* sHV = sHK + KMAX * LD;
  T* sGL = sHV + KMAX * LD;    // grad_logits (first order), pitch KLD
  T* sDS = sGL + KMAX * KLD;   // d_scores, pitch KLD
  T* sDG = sDS + KMAX * KLD;   // d_grad_probs, pitch KLD
  const cg_edge_attn_args& a = P.a;
  const int k = a.k, d = a.d;
  const T scale = T(a.scale);
  const int64_t slices = a.n * a.h;
  for (int64_t s = (int64_t)blockIdx.x * nw + warp; s < slices; s += (int64_t)gridDim.x * nw) {
    const int64_t n = s / a.h, h = s % a.h;
    __syncwarp();
    load_mat<T, DP, LD>(sQ, a.q, n, h, k, d, P.vec_ok, lane);
    load_mat<T, DP, LD>(sK, a.k_, n, h, k, d, P.vec_ok, lane);
    load_mat<T, DP, LD>(sV, a.v, n, h, k, d, P.vec_ok, lane);
    load_mat<T, DP, LD>(sG, a.grad_out, n, h, k, d, P.vec_ok, lane);
    load_mat<T, DP, LD>(sHQ, a.hq, n, h, k, d, P.vec_ok, lane);
    load_mat<T, DP, LD>(sHK, a.hk, n, h, k, d, P.vec_ok, lane);
    load_mat<T, DP, LD>(sHV, a.hv, n, h, k, d, P.vec_ok, lane);
    __syncwarp();
    const int kc = valid_keys<T>(P, n);
    const int i = lane < k ? lane : 0;
    T p[KMAX];
    {
      T x[KMAX], y[KMAX], b[KMAX];
      // probabilities from the saved row logsumexp
      row_dots<T, DP, LD>(x, sQ + i * LD, sK, k);
      bias_row<T>(b, a.bias, n, h, i, k);
#pragma unroll
      for (int j = 0; j < KMAX; ++j) y[j] = x[j] * scale + b[j];
      const T* lse_in = reinterpret_cast<const T*>(a.lse) + s * k + i;
      softmax_row<T>(p, y, k, kc, lse_in);
      // centered grad_probs: cen = gp - rowsum(p * gp)
      T cen[KMAX];
      row_dots<T, DP, LD>(cen, sG + i * LD, sV, k);
      T rs = T(0);
#pragma unroll
      for (int j = 0; j < KMAX; ++j) rs = fma(p[j], cen[j], rs);
#pragma unroll
      for (int j = 0; j < KMAX; ++j) cen[j] = cen[j] - rs;
      // d_logits = scale * (hq k^T + q hk^T) + hb
      row_dots<T, DP, LD>(x, sHQ + i * LD, sK, k);
      row_dots<T, DP, LD>(y, sQ + i * LD, sHK, k);
      bias_row<T>(b, a.hb, n, h, i, k);
#pragma unroll
      for (int j = 0; j < KMAX; ++j) b[j] = scale * (x[j] + y[j]) + b[j];  // d_logits
      // d_rowsum = -sum(d_logits * probs)
      T drs = T(0);
#pragma unroll
      for (int j = 0; j < KMAX; ++j) drs = fma(b[j], p[j], drs);
      drs = -drs;
      // d_probs = d_logits*cen + d_rowsum*gp + grad_out hv^T; d_gp = (d_logits + d_rowsum)*p
      row_dots<T, DP, LD>(x, sG + i * LD, sHV, k);
#pragma unroll
      for (int j = 0; j < KMAX; ++j) {
        const T gp = cen[j] + rs;
        y[j] = b[j] * cen[j] + drs * gp + x[j];       // d_probs
        x[j] = b[j] * p[j] + drs * p[j];              // d_grad_probs
      }
      T rs2 = T(0);
#pragma unroll
      for (int j = 0; j < KMAX; ++j) rs2 = fma(p[j], y[j], rs2);
      if (lane < k) {
#pragma unroll
        for (int j = 0; j < KMAX; ++j) {
          sGL[lane * KLD + j] = p[j] * cen[j];             // grad_logits
          sDS[lane * KLD + j] = p[j] * (y[j] - rs2);       // d_scores
          sDG[lane * KLD + j] = x[j];                      // d_grad_probs
        }
      }
    }
    __syncwarp();
    if (lane < k) {
      T w1[KMAX], w2[KMAX];
      // grad_q = scale * (grad_logits hk + d_scores k)
      load_row<T>(w1, sGL, lane, k);
      load_row<T>(w2, sDS, lane, k);
      emit_row<T, DP>(a.dq, n, h, lane, d, P.vec_ok, [&](int c, T* acc) {
#pragma unroll
        for (int e = 0; e < V16<T>::n; ++e) acc[e] = T(0);
        combine<T, LD>(acc, w1, sHK, c, k);
        combine<T, LD>(acc, w2, sK, c, k);
#pragma unroll
        for (int e = 0; e < V16<T>::n; ++e) acc[e] *= scale;
      });
      // grad_out cotangent = d_grad_probs v + probs hv
      load_row<T>(w1, sDG, lane, k);
      emit_row<T, DP>(a.dgrad_out, n, h, lane, d, P.vec_ok, [&](int c, T* acc) {
#pragma unroll
        for (int e = 0; e < V16<T>::n; ++e) acc[e] = T(0);
        combine<T, LD>(acc, w1, sV, c, k);
        combine<T, LD>(acc, p, sHV, c, k);
      });
      // grad_k = scale * (grad_logits^T hq + d_scores^T q)
      load_col<T>(w1, sGL, lane, k);
      load_col<T>(w2, sDS, lane, k);
      emit_row<T, DP>(a.dk, n, h, lane, d, P.vec_ok, [&](int c, T* acc) {
#pragma unroll
        for (int e = 0; e < V16<T>::n; ++e) acc[e] = T(0);
        combine<T, LD>(acc, w1, sHQ, c, k);
        combine<T, LD>(acc, w2, sQ, c, k);
#pragma unroll
        for (int e = 0; e < V16<T>::n; ++e) acc[e] *= scale;
      });
      // grad_v = d_grad_probs^T grad_out
      load_col<T>(w1, sDG, lane, k);
      emit_row<T, DP>(a.dv, n, h, lane, d, P.vec_ok, [&](int c, T* acc) {
#pragma unroll
        for (int e = 0; e < V16<T>::n; ++e) acc[e] = T(0);
        combine<T, LD>(acc, w1, sG, c, k);
      });
    }
    write_dbias<T>(P, sDS, n, h, s, lane);
  }
}

// Sum the per-slice partial dbias over the broadcast n and/or h dimensions in
// a fixed order (deterministic), one thread per dbias element.
template <typename T>
__global__ void dbias_reduce_kernel(const Params P, int64_t outs) {
  const cg_edge_attn_args& a = P.a;
  const int ki = P.ki, kj = P.kj;
  const int64_t per = (int64_t)ki * kj;
  const bool bn = a.bias.sn == 0, bh = a.bias.sh == 0;
  const int64_t nn = bn ? 1 : a.n, hh = bh ? 1 : a.h;
  for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < outs;
       o += (int64_t)gridDim.x * blockDim.x) {
    const int64_t f = o % per;
    const int64_t nh = o / per;
    const int64_t n0 = nh / hh, h0 = nh % hh;
    const T* part = reinterpret_cast<const T*>(a.scratch);
    T v = T(0);
    for (int64_t n = bn ? 0 : n0; n < (bn ? a.n : n0 + 1); ++n)
      for (int64_t h = bh ? 0 : h0; h < (bh ? a.h : h0 + 1); ++h) v += part[(n * a.h + h) * per + f];
    const int i = (int)(f / kj), j = (int)(f % kj);
    const cg_bias& db = a.dbias;
    T* dst = reinterpret_cast<T*>(db.ptr) + n0 * db.sn + h0 * db.sh + (int64_t)i * db.si +
             (int64_t)j * db.sj;
    *dst = v;
    (void)nn;
  }
}

enum Which { kFwd1, kBwd1, kBwd2 };

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

inline bool mat_vec_ok(const cg_mat& m, int esize, int d, int dp) {
  if (m.ptr == nullptr) return true;
  const int per = 16 / esize;
  return d == dp && aligned16(m.ptr) && m.sn % per == 0 && m.sh % per == 0 && m.sr % per == 0;
}

inline int padded_d(int d, int dtype) {
  // head dims are padded (with zero columns) to the instantiated widths
  const int steps32[] = {8, 16, 32, 64};
  const int steps64[] = {4, 8, 16};
  const int* steps = dtype == CG_F32 ? steps32 : steps64;
  const int count = dtype == CG_F32 ? 4 : 3;
  for (int i = 0; i < count; ++i)
    if (d <= steps[i]) return steps[i];
  return -1;
}

inline int smem_floats_per_warp(Which w, int ld) {
  switch (w) {
    case kFwd1: return 3 * KMAX * ld;
    case kBwd1: return 4 * KMAX * ld + 2 * KMAX * KLD;
    default: return 7 * KMAX * ld + 3 * KMAX * KLD;
  }
}

inline int check_mat(const cg_mat& m, const char* name, bool needed) {
  CG_REQUIRE(!needed || m.ptr != nullptr, "edge_attn: %s is NULL", name);
  return kOk;
}

inline void dbias_shape(const cg_edge_attn_args& a, int* ki, int* kj) {
  *ki = a.bias.si == 0 ? 1 : a.k;
  *kj = a.bias.sj == 0 ? 1 : a.k;
}

inline bool dbias_cross_slice(const cg_edge_attn_args& a) {
  return a.bias.ptr != nullptr && ((a.bias.sn == 0 && a.n > 1) || (a.bias.sh == 0 && a.h > 1));
}

template <typename T, int DP>
inline int launch_typed(Which w, const Params& P, cudaStream_t stream) {
  constexpr int LD = DP + 16 / sizeof(T);
  const int per_warp = smem_floats_per_warp(w, LD) * (int)sizeof(T);
  int warps = 4;
  while (warps > 1 && warps * per_warp > 220 * 1024) warps >>= 1;
  CG_REQUIRE(per_warp <= 227 * 1024, "edge_attn: head dim too large for shared memory");
  const size_t smem = (size_t)warps * per_warp;
  const int64_t slices = P.a.n * P.a.h;
  const int64_t want = ceil_div<int64_t>(slices, warps);
  int dev_blocks = sm_count() * 8;
  const int grid = (int)(want < dev_blocks ? want : dev_blocks);
  void (*kernel)(const Params) = w == kFwd1 ? fwd1_kernel<T, DP>
                                 : w == kBwd1 ? bwd1_kernel<T, DP>
                                              : bwd2_kernel<T, DP>;
  CG_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  kernel<<<grid, warps * 32, smem, stream>>>(P);
  CG_LAUNCHED("edge_attn");
  if (w != kFwd1 && P.dbias_mode == kDbiasScratch) {
    const bool bn = P.a.bias.sn == 0, bh = P.a.bias.sh == 0;
    const int64_t outs = (bn ? 1 : P.a.n) * (bh ? 1 : P.a.h) * (int64_t)P.ki * P.kj;
    const int threads = 256;
    const int64_t blocks = ceil_div<int64_t>(outs, threads);
    const int g = (int)(blocks < 4096 ? blocks : 4096);
    dbias_reduce_kernel<T><<<g, threads, 0, stream>>>(P, outs);
    CG_LAUNCHED("edge_attn dbias reduction");
  }
  return kOk;
}

int dispatch_f64(Which w, const Params& P, int dp, cudaStream_t stream);

}  // namespace attn
}  // namespace cg
