// Masked edge attention (float32) on the tensor cores.
//
// Same arithmetic as the CUDA-core kernels in edge_attn.cuh (the reference's
// kernels/edge_attn/ops.py:26-104), organised for mma.sync m16n8k8 tf32 in
// one of two precisions (cg_edge_attn_args.precision):
// - CG_ATTN_FP32: a three-term split of every operand (x = hi + lo, hi = x
//   truncated to tf32, lo = tf32(x - hi); a*b ~ hi*hi + hi*lo + lo*hi), which
//   keeps fp32-level accuracy (~1e-6 relative) at three products per tile;
// - CG_ATTN_TF32: one product of round-to-nearest tf32 operands per tile
//   (operand rounding 2^-11 relative, fp32 accumulation), the precision of the
//   tcgen05 projections.
// Softmax, row reductions and all elementwise work are fp32 in both.
//
// One CTA of two warps owns one slice (n, h) of k <= 32 tokens: warp w holds
// query rows [16w, 16w + 16) of every k x k matrix as mma accumulator
// fragments, so row reductions of the softmax are quad shuffles. The k x d
// operands sit in shared memory. The k x k intermediates (probs,
// grad_logits, d_scores, d_grad_probs) feed the row products (out, dq,
// grad_out) straight from their accumulator fragments, and are written to
// shared memory once for the key products (dk, dv), which read them
// transposed after a CTA barrier. Rows past k and columns past d are zero in
// shared memory.
//
// Fragment loads. The mma's k-slot t holds logical k0 + 2t and slot t + 4
// holds k0 + 2t + 1 (a reduction does not care which slot carries which k, as
// long as A and B agree), so a lane's two k values of one row are adjacent
// and come in one 64-bit shared load. Rows of 32 floats are XOR-swizzled in
// 8-float groups, element (r, c) at column c ^ 8 f(r), f(r) = (r & 3) ^
// ((r >> 2) & 1): the row-by-g 64-bit loads (rows g of a band, columns 2t)
// and the transposed row-by-t 32-bit loads (rows k0 + 2t (+1), columns g) of
// one warp then both hit 32 distinct banks, with no padding.
#pragma once

#include <math.h>
#include <stdint.h>

#include "common.cuh"
#include "../../include/cg_b200.h"

namespace cg {
namespace attn_tc {

constexpr int KP = 32;  // padded tokens per slice
constexpr int kThreads = 64;

// shared-memory bias tiles: none, one key row broadcast over queries, a full
// k x k tile by 16-byte copies, a full tile by scalar loads
enum BiasMode { kBiasNone = 0, kBiasKeyRow = 1, kBiasVec = 2, kBiasScalar = 3 };

struct Params {
  cg_edge_attn_args a;
  int dbias_mode;  // 0 none, 1 direct, 2 per-slice partials into scratch
  int ki, kj;
  int vec_ok;
  int bias_mode, hb_mode;
  int dbias_vec;  // full-tile dbias rows leave in 16-byte stores
  int same;       // 16-byte rows, no token index, and every k x d operand with the same strides
};

// per-slice dbias partials -> dbias, when the bias broadcasts over n or h
int reduce_dbias(const Params& P, cudaStream_t stream);

// ---- shared layout ------------------------------------------------------------

__device__ __forceinline__ int swz(int r) { return ((r & 3) ^ ((r >> 2) & 1)) << 3; }
// element (r, c) of a k x k matrix
__device__ __forceinline__ int kk(int r, int c) { return r * KP + (c ^ swz(r)); }

template <int DP>
struct Layout {
  // widths of 32 and 64 are swizzled in place; narrower ones padded by 4
  static constexpr bool kSwz = DP >= 32;
  static constexpr int LD = kSwz ? DP : DP + 4;
  static constexpr int OP = KP * LD;  // floats per k x d operand
  static constexpr int KK = KP * KP;  // floats per k x k matrix
  __device__ static __forceinline__ int op(int r, int c) { return r * LD + (kSwz ? (c ^ swz(r)) : c); }
};

__device__ __forceinline__ float2 ld2(const float* s, int i) { return *reinterpret_cast<const float2*>(s + i); }

// ---- mma.sync tf32 ---------------------------------------------------------------

struct Split {
  uint32_t hi, lo;
};

// The tensor cores read a tf32 operand from the top 19 bits of its register
// and ignore the low 13. Single-term products (tf32 mode) pass x with half an
// ulp added to its bit pattern, which rounds it to nearest. The three-term
// split (fp32 mode): hi = x truncated to tf32 (low bits cleared, so that the
// remainder x - hi is exact), lo = the remainder rounded the same way.
// Integer and FADD work only: no conversions.
__device__ __forceinline__ uint32_t tf32_rn(float x) { return __float_as_uint(x) + 0x1000u; }

__device__ __forceinline__ Split split(float x) {
  const uint32_t hi = __float_as_uint(x) & 0xffffe000u;
  return {hi, tf32_rn(x - __uint_as_float(hi))};
}

__device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// One 8-deep k step of acc[nt] += A(16 x 8) * B(8 x 8*NT) for one 16-row
// band, k = k0 .. k0 + 7. la(m, k) returns {A(m, k), A(m, k + 1)} and
// lb(k, n) returns {B(k, n), B(k + 1, n)} for even k. m16n8k8 fragments: A a0
// (g, slot t) a1 (g+8, t) a2 (g, t+4) a3 (g+8, t+4); B b0 (t, g) b1 (t+4, g);
// C c0 (g, 2t) c1 (g, 2t+1) c2 (g+8, 2t) c3 (g+8, 2t+1).
template <bool X3, int NT, class LB>
__device__ __forceinline__ void kstep_a(float (&acc)[NT][4], float x0, float x1, float x2, float x3, LB lb, int k0,
                                        int g, int t) {
  if constexpr (X3) {
    const Split a0 = split(x0), a1 = split(x1), a2 = split(x2), a3 = split(x3);
    const uint32_t ahi[4] = {a0.hi, a1.hi, a2.hi, a3.hi};
    const uint32_t alo[4] = {a0.lo, a1.lo, a2.lo, a3.lo};
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const float2 b = lb(k0 + 2 * t, nt * 8 + g);
      const Split b0 = split(b.x), b1 = split(b.y);
      const uint32_t bhi[2] = {b0.hi, b1.hi};
      const uint32_t blo[2] = {b0.lo, b1.lo};
      mma(acc[nt], alo, bhi);
      mma(acc[nt], ahi, blo);
      mma(acc[nt], ahi, bhi);
    }
  } else {
    const uint32_t a[4] = {tf32_rn(x0), tf32_rn(x1), tf32_rn(x2), tf32_rn(x3)};
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const float2 b = lb(k0 + 2 * t, nt * 8 + g);
      const uint32_t bb[2] = {tf32_rn(b.x), tf32_rn(b.y)};
      mma(acc[nt], a, bb);
    }
  }
}

template <bool X3, int NT, class LA, class LB>
__device__ __forceinline__ void kstep(float (&acc)[NT][4], LA la, LB lb, int k0, int g, int t) {
  const float2 r0 = la(g, k0 + 2 * t), r1 = la(g + 8, k0 + 2 * t);
  kstep_a<X3>(acc, r0.x, r1.x, r0.y, r1.y, lb, k0, g, t);
}

// acc += A(16 x 8*KT) * B(8*KT x 8*NT); the tf32 loop is unrolled, the
// three-term one (three times the code per step) only where FULL asks for it
// (kernels whose register budget holds it: the unrolled steps pipeline their
// fragment loads and splits across k).
template <bool X3, int NT, int KT, bool FULL = !X3, class LA, class LB>
__device__ __forceinline__ void band_mma(float (&acc)[NT][4], LA la, LB lb, int g, int t) {
  constexpr int U = FULL ? KT : 1;
#pragma unroll U
  for (int kt = 0; kt < KT; ++kt) kstep<X3>(acc, la, lb, kt * 8, g, t);
}

// Two independent products in one k loop: twice the accumulator chains in
// flight per warp.
template <bool X3, int NT, int KT, bool FULL = !X3, class LA1, class LB1, class LA2, class LB2>
__device__ __forceinline__ void band_mma2(float (&acc1)[NT][4], LA1 la1, LB1 lb1, float (&acc2)[NT][4], LA2 la2,
                                          LB2 lb2, int g, int t) {
  constexpr int U = FULL ? KT : 1;
#pragma unroll U
  for (int kt = 0; kt < KT; ++kt) {
    kstep<X3>(acc1, la1, lb1, kt * 8, g, t);
    kstep<X3>(acc2, la2, lb2, kt * 8, g, t);
  }
}

// acc += A(16 x 32) * B(32 x 8*NT) with A a 16 x 32 band held as C fragments
// of four m16n8 tiles (c[kt] covers columns 8kt .. 8kt + 7). With the k-slot
// mapping above, tile kt's C fragment {c0, c1, c2, c3} = {(g, 2t), (g, 2t+1),
// (g+8, 2t), (g+8, 2t+1)} is the A fragment of k step kt in the order
// {a0, a2, a1, a3}: no shared-memory round trip. Always unrolled (register
// arrays take constant indices only).
template <bool X3, int NT, class LB>
__device__ __forceinline__ void band_mma_reg(float (&acc)[NT][4], const float (&c)[4][4], LB lb, int g, int t) {
#pragma unroll
  for (int kt = 0; kt < 4; ++kt) kstep_a<X3>(acc, c[kt][0], c[kt][2], c[kt][1], c[kt][3], lb, kt * 8, g, t);
}

template <bool X3, int NT, class LB1, class LB2>
__device__ __forceinline__ void band_mma_reg2(float (&acc1)[NT][4], const float (&c1)[4][4], LB1 lb1,
                                              float (&acc2)[NT][4], const float (&c2)[4][4], LB2 lb2, int g, int t) {
#pragma unroll
  for (int kt = 0; kt < 4; ++kt) {
    kstep_a<X3>(acc1, c1[kt][0], c1[kt][2], c1[kt][1], c1[kt][3], lb1, kt * 8, g, t);
    kstep_a<X3>(acc2, c2[kt][0], c2[kt][2], c2[kt][1], c2[kt][3], lb2, kt * 8, g, t);
  }
}

template <int NT>
__device__ __forceinline__ void zero(float (&acc)[NT][4]) {
#pragma unroll
  for (int i = 0; i < NT; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[i][e] = 0.0f;
}

// Sum over the quad (the four lanes sharing g): a full row of a k x k band.
__device__ __forceinline__ float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  return v;
}
__device__ __forceinline__ float quad_max(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
  return v;
}

// ---- operand staging -------------------------------------------------------------
// Row r of a slice operand, or null for a zero row: plain rows
// ptr + n*sn + h*sh + r*sr, or, with the slice's token index staged in shared
// memory (sidx[r] = token_index[n*k + r]), the gathered row
// ptr + sidx[r]*sr + h*sh (negative index: zero row).
__device__ __forceinline__ const float* op_row(const cg_mat& m, const int32_t* sidx, int64_t n, int64_t h, int r,
                                               int k) {
  if (r >= k) return nullptr;
  const float* base = reinterpret_cast<const float*>(m.ptr) + h * m.sh;
  if (sidx == nullptr) return base + n * m.sn + (int64_t)r * m.sr;
  const int32_t j = sidx[r];
  return j < 0 ? nullptr : base + (int64_t)j * m.sr;
}

// Stage the slice's token index in shared memory (all threads; a barrier
// follows before use). Returns the pointer the loads take, or null.
__device__ __forceinline__ const int32_t* stage_index(int32_t* sidx, const int32_t* token_index, int64_t n, int k) {
  if (token_index == nullptr) return nullptr;
  if (threadIdx.x < KP) sidx[threadIdx.x] = threadIdx.x < k ? token_index[n * k + threadIdx.x] : -1;
  __syncthreads();
  return sidx;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// k x d operand into shared memory. Aligned layouts (vec): 16-byte cp.async
// copies (rows past k zero-filled by a source size of 0), completed by
// cp_async_wait<N>() + __syncthreads() before use; otherwise scalar loads
// (zeros past k and d).
template <int DP>
__device__ __forceinline__ void load_op_async(float* s, const cg_mat& m, int64_t n, int64_t h, int k, int d,
                                              bool vec, const int32_t* idx = nullptr) {
  using L = Layout<DP>;
  const float* ptr = reinterpret_cast<const float*>(m.ptr);
  if (vec) {
    constexpr int VPR = DP / 4;
    for (int f = threadIdx.x; f < KP * VPR; f += kThreads) {
      const int r = f / VPR, c = (f % VPR) * 4;
      const float* row = op_row(m, idx, n, h, r, k);
      cp_async16(s + L::op(r, c), row ? row + c : ptr, row ? 16 : 0);
    }
  } else {
    for (int f = threadIdx.x; f < KP * DP; f += kThreads) {
      const int r = f / DP, c = f % DP;
      const float* row = op_row(m, idx, n, h, r, k);
      s[L::op(r, c)] = (row && c < d) ? row[c] : 0.0f;
    }
  }
}

// Several k x d operands with the same strides (and no token index) in one
// pass: the row offset, destination and predicate of a 16-byte chunk are
// computed once for all of them.
template <int DP, int NOPS>
__device__ __forceinline__ void load_same_async(float* const (&s)[NOPS], const cg_mat (&m)[NOPS], int64_t n,
                                                int64_t h, int k) {
  using L = Layout<DP>;
  constexpr int VPR = DP / 4;
  const int64_t slice = n * m[0].sn + h * m[0].sh;
  for (int f = threadIdx.x; f < KP * VPR; f += kThreads) {
    const int r = f / VPR, c = (f % VPR) * 4;
    const bool ok = r < k;
    const int64_t off = slice + (int64_t)r * m[0].sr + c;
    const int so = L::op(r, c);
#pragma unroll
    for (int i = 0; i < NOPS; ++i) {
      const float* base = reinterpret_cast<const float*>(m[i].ptr);
      cp_async16(s[i] + so, ok ? base + off : base, ok ? 16 : 0);
    }
  }
}

// Bias tile of the slice into shared memory (zeros outside [0,k)^2; the
// 16-byte copies join the caller's next cp.async group). Returns the row mask
// its readers apply to the query row (0: one key row broadcast over queries).
__device__ __forceinline__ int load_bias(float* s, const cg_bias& b, int mode, int64_t n, int64_t h, int k) {
  const float* base = reinterpret_cast<const float*>(b.ptr);
  switch (mode) {
    case kBiasNone:
      if (threadIdx.x < KP) s[threadIdx.x] = 0.0f;
      return 0;
    case kBiasKeyRow:
      if (threadIdx.x < KP) {
        const int j = threadIdx.x;
        s[j] = j < k ? base[n * b.sn + h * b.sh + (int64_t)j * b.sj] : 0.0f;
      }
      return 0;
    case kBiasVec:
      for (int f = threadIdx.x; f < KP * (KP / 4); f += kThreads) {
        const int i = f / (KP / 4), j = (f % (KP / 4)) * 4;
        const bool ok = i < k && j < k;
        const float* src = ok ? base + n * b.sn + h * b.sh + (int64_t)i * b.si + j : base;
        cp_async16(s + kk(i, j), src, ok ? 16 : 0);
      }
      return ~0;
    default:
      for (int f = threadIdx.x; f < KP * KP; f += kThreads) {
        const int i = f / KP, j = f % KP;
        float v = 0.0f;
        if (i < k && j < k) v = base[n * b.sn + h * b.sh + (int64_t)i * b.si + (int64_t)j * b.sj];
        s[kk(i, j)] = v;
      }
      return ~0;
  }
}

// Store a 16 x 8*NT band (rows 16*band + ...) of a k x d output, times scale.
template <int NT>
__device__ __forceinline__ void store_band(const cg_mat& m, int64_t n, int64_t h, int band, int k, int d,
                                           const float (&acc)[NT][4], int g, int t, float scale, bool vec) {
  float* base = reinterpret_cast<float*>(m.ptr) + n * m.sn + h * m.sh;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = band * 16 + g + 8 * half;
      const int c = nt * 8 + 2 * t;
      if (r < k) {
        float* dst = base + (int64_t)r * m.sr + c;
        const float x = acc[nt][2 * half] * scale, y = acc[nt][2 * half + 1] * scale;
        if (vec) {
          *reinterpret_cast<float2*>(dst) = make_float2(x, y);
        } else if (c + 1 < d) {
          dst[0] = x;
          dst[1] = y;
        } else if (c < d) {
          dst[0] = x;
        }
      }
    }
  }
}

__device__ __forceinline__ int valid_keys(const Params& P, int64_t n) {
  const int k = P.a.k;
  if (P.a.key_count == nullptr) return k;
  const int c = P.a.key_count[n];
  return c < 0 ? 0 : (c > k ? k : c);
}

// Per-slice dbias from a k x k matrix M in shared memory, reduced over i
// and/or j when the bias broadcasts them; to dbias (mode 1) or to the slice's
// ki x kj partial in scratch (mode 2). Reductions run in a fixed order.
__device__ __forceinline__ void write_dbias(const Params& P, const float* M, int64_t n, int64_t h, int64_t slice) {
  if (P.dbias_mode == 0) return;
  const int k = P.a.k, ki = P.ki, kj = P.kj;
  float* dst;
  int64_t si, sj;
  if (P.dbias_mode == 1) {
    const cg_bias& db = P.a.dbias;
    dst = reinterpret_cast<float*>(db.ptr) + n * db.sn + h * db.sh;
    si = db.si;
    sj = db.sj;
  } else {
    dst = reinterpret_cast<float*>(P.a.scratch) + slice * (int64_t)(ki * kj);
    si = kj;
    sj = 1;
  }
  if (ki == k && kj == k) {
    if (P.dbias_vec) {
      for (int f = threadIdx.x; f < KP * (KP / 4); f += kThreads) {
        const int i = f >> 3, j = (f & 7) * 4;
        if (i < k && j < k)
          *reinterpret_cast<float4*>(dst + i * si + j) = *reinterpret_cast<const float4*>(M + kk(i, j));
      }
    } else {
      for (int f = threadIdx.x; f < KP * KP; f += kThreads) {
        const int i = f >> 5, j = f & 31;
        if (i < k && j < k) dst[i * si + j * sj] = M[kk(i, j)];
      }
    }
  } else if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    if (ki == 1 && kj == k) {  // column sums: lane j, four partial sums over rows
      float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 2
      for (int r = 0; r < KP; r += 4)
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] += r + q < k ? M[kk(r + q, lane)] : 0.0f;
      if (lane < k) dst[lane * sj] = (v[0] + v[1]) + (v[2] + v[3]);
    } else {  // row sums (ki == k), or the total (ki == 1): lane i
      float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 2
      for (int c = 0; c < KP; c += 4)
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] += c + q < k && lane < k ? M[kk(lane, c + q)] : 0.0f;
      float row = (v[0] + v[1]) + (v[2] + v[3]);
      if (ki == k) {
        if (lane < k) dst[lane * si] = row;
      } else {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) row += __shfl_xor_sync(0xffffffffu, row, off);
        if (lane == 0) dst[0] = row;
      }
    }
  }
}

// exp for the softmax: the accurate expf, or (FAST, tf32 precision) the
// hardware-approximated __expf, whose relative error (~1e-6 over the range
// used) is far below the tf32 operand rounding.
template <bool FAST>
__device__ __forceinline__ float sm_exp(float x) {
  if constexpr (FAST) return __expf(x);
  else return expf(x);
}

// Logits of the band from the S accumulator: scale * S + bias (bias row
// r & brow), masked to -inf for keys past kc and non-finite values. Returns
// probabilities in `p` (exp(l - lse)) and, when lse_in is null, computes the
// row lse.
template <bool FAST>
__device__ __forceinline__ void band_softmax(float (&p)[4][4], const float (&s)[4][4], const float* sbias,
                                             int brow, int band, int g, int t, float scale, int kc,
                                             const float* lse_in, float (&lse)[2]) {
  float l[4][4];
  bool ok[4][4];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = band * 16 + g + 8 * half, c = nt * 8 + 2 * t;
      const float2 b = ld2(sbias, kk(r & brow, c));
#pragma unroll
      for (int e2 = 0; e2 < 2; ++e2) {
        const float v = s[nt][2 * half + e2] * scale + (e2 ? b.y : b.x);
        l[nt][2 * half + e2] = v;
        ok[nt][2 * half + e2] = c + e2 < kc && isfinite(v);
      }
    }
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    if (lse_in != nullptr) {
      lse[half] = lse_in[band * 16 + g + 8 * half];
    } else {
      float m = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e2 = 0; e2 < 2; ++e2)
          if (ok[nt][2 * half + e2]) m = fmaxf(m, l[nt][2 * half + e2]);
      m = quad_max(m);
      float sum = 0.0f;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e2 = 0; e2 < 2; ++e2)
          if (ok[nt][2 * half + e2]) sum += sm_exp<FAST>(l[nt][2 * half + e2] - m);
      sum = quad_sum(sum);
      lse[half] = m == -INFINITY ? -INFINITY : m + logf(sum);
    }
  }
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float ls = lse[e >> 1];
      p[nt][e] = (ok[nt][e] && isfinite(ls)) ? sm_exp<FAST>(l[nt][e] - ls) : 0.0f;
    }
}

// Write a band of a k x k fragment matrix to shared memory (64-bit stores).
__device__ __forceinline__ void put_band(float* M, const float (&v)[4][4], int band, int g, int t) {
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int half = 0; half < 2; ++half)
      *reinterpret_cast<float2*>(M + kk(band * 16 + g + 8 * half, nt * 8 + 2 * t)) =
          make_float2(v[nt][2 * half], v[nt][2 * half + 1]);
}

// row sums of a band (both halves) of a product of two fragment matrices
__device__ __forceinline__ void row_dot(float (&out)[2], const float (&a)[4][4], const float (&b)[4][4]) {
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    float s = 0.0f;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) s += a[nt][2 * half] * b[nt][2 * half] + a[nt][2 * half + 1] * b[nt][2 * half + 1];
    out[half] = quad_sum(s);
  }
}

// ---- fragment loaders ---------------------------------------------------------------
// k x d operand X as A, rows from the band (reduction over d).
#define CG_A_ROWS(X) [&](int m, int c) { return ld2(X, L::op(band * 16 + m, c)); }
// X as the B of X^T (n = token row, reduction over d).
#define CG_B_ROWS(X) [&](int c, int j) { return ld2(X, L::op(j, c)); }
// X as B with the reduction over tokens (k = token row, n = column).
#define CG_B_COLS(X) [&](int j, int c) { return make_float2(X[L::op(j, c)], X[L::op(j + 1, c)]); }
// k x k matrix M as A, transposed (rows of A = columns of M from the band).
#define CG_A_KKT(M) [&](int m, int i) { return make_float2(M[kk(i, band * 16 + m)], M[kk(i + 1, band * 16 + m)]); }

// ---------------------------------------------------------------------------

template <int DP, bool X3>
__global__ void __launch_bounds__(kThreads) fwd1_tc(const Params P) {
  using L = Layout<DP>;
  extern __shared__ __align__(16) float smem[];
  float* sQ = smem;
  float* sK = sQ + L::OP;
  float* sV = sK + L::OP;
  float* sP = sV + L::OP;  // bias tile
  int32_t* sIdx = reinterpret_cast<int32_t*>(sP + L::KK);
  const cg_edge_attn_args& a = P.a;
  const int k = a.k, d = a.d;
  const float scale = (float)a.scale;
  const bool vec = P.vec_ok;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int band = warp;
  for (int64_t s = blockIdx.x; s < a.n * a.h; s += gridDim.x) {
    const int64_t n = s / a.h, h = s % a.h;
    __syncthreads();
    const int32_t* tix = stage_index(sIdx, a.token_index, n, k);
    if (P.same) {
      load_same_async<DP, 2>({sQ, sK}, {a.q, a.k_}, n, h, k);
    } else {
      load_op_async<DP>(sQ, a.q, n, h, k, d, vec, tix);
      load_op_async<DP>(sK, a.k_, n, h, k, d, vec, tix);
    }
    const int brow = load_bias(sP, a.bias, P.bias_mode, n, h, k);
    cp_async_commit();
    load_op_async<DP>(sV, a.v, n, h, k, d, vec, tix);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const int kc = valid_keys(P, n);
    float S[4][4], p[4][4], lse[2];
    zero(S);
    band_mma<X3, 4, DP / 8, true>(S, CG_A_ROWS(sQ), CG_B_ROWS(sK), g, t);
    band_softmax<!X3>(p, S, sP, brow, band, g, t, scale, kc, nullptr, lse);
    cp_async_wait<0>();
    __syncthreads();  // V landed
    float O[DP / 8][4];
    zero(O);  // out = probs v, probs straight from the fragments
    band_mma_reg<X3, DP / 8>(O, p, CG_B_COLS(sV), g, t);
    store_band<DP / 8>(a.out, n, h, band, k, d, O, g, t, 1.0f, vec);
    if (t == 0) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int r = band * 16 + g + 8 * half;
        if (r < k) reinterpret_cast<float*>(a.lse)[s * k + r] = lse[half];
      }
    }
  }
}

template <int DP, bool X3>
__global__ void __launch_bounds__(kThreads) bwd1_tc(const Params P) {
  using L = Layout<DP>;
  extern __shared__ __align__(16) float smem[];
  float* sQ = smem;
  float* sK = sQ + L::OP;
  float* sV = sK + L::OP;
  float* sG = sV + L::OP;
  float* sP = sG + L::OP;
  float* sGL = sP + L::KK;  // bias tile, then grad_logits
  float* sLse = sGL + L::KK;
  int32_t* sIdx = reinterpret_cast<int32_t*>(sLse + KP);
  const cg_edge_attn_args& a = P.a;
  const int k = a.k, d = a.d;
  const float scale = (float)a.scale;
  const bool vec = P.vec_ok;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int band = warp;
  for (int64_t s = blockIdx.x; s < a.n * a.h; s += gridDim.x) {
    const int64_t n = s / a.h, h = s % a.h;
    __syncthreads();
    const int32_t* tix = stage_index(sIdx, a.token_index, n, k);
    if (P.same) {
      load_same_async<DP, 4>({sQ, sK, sV, sG}, {a.q, a.k_, a.v, a.grad_out}, n, h, k);
    } else {
      load_op_async<DP>(sQ, a.q, n, h, k, d, vec, tix);
      load_op_async<DP>(sK, a.k_, n, h, k, d, vec, tix);
      load_op_async<DP>(sV, a.v, n, h, k, d, vec, tix);
      load_op_async<DP>(sG, a.grad_out, n, h, k, d, vec);
    }
    const int brow = load_bias(sGL, a.bias, P.bias_mode, n, h, k);
    cp_async_commit();
    if (threadIdx.x < KP)
      sLse[threadIdx.x] = threadIdx.x < k ? reinterpret_cast<const float*>(a.lse)[s * k + threadIdx.x] : 0.0f;
    cp_async_wait<0>();
    __syncthreads();
    const int kc = valid_keys(P, n);
    {
      float S[4][4], GP[4][4], p[4][4], lse[2];
      zero(S);   // scores
      zero(GP);  // grad_probs = grad_out v^T
      band_mma2<X3, 4, DP / 8>(S, CG_A_ROWS(sQ), CG_B_ROWS(sK), GP, CG_A_ROWS(sG), CG_B_ROWS(sV), g, t);
      band_softmax<!X3>(p, S, sGL, brow, band, g, t, scale, kc, sLse, lse);
      float rs[2];
      row_dot(rs, p, GP);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) GP[nt][e] = p[nt][e] * (GP[nt][e] - rs[e >> 1]);  // grad_logits
      float O[DP / 8][4];
      zero(O);  // grad_q = scale * grad_logits k, grad_logits straight from the fragments
      band_mma_reg<X3, DP / 8>(O, GP, CG_B_COLS(sK), g, t);
      store_band<DP / 8>(a.dq, n, h, band, k, d, O, g, t, scale, vec);
      __syncthreads();  // every warp is done with the bias tile
      put_band(sP, p, band, g, t);
      put_band(sGL, GP, band, g, t);
    }
    __syncthreads();
    {
      float DV[DP / 8][4], DK[DP / 8][4];
      zero(DV);  // grad_v = probs^T grad_out (rows: keys of this band)
      zero(DK);  // grad_k = scale * grad_logits^T q
      band_mma2<X3, DP / 8, 4>(DV, CG_A_KKT(sP), CG_B_COLS(sG), DK, CG_A_KKT(sGL), CG_B_COLS(sQ), g, t);
      store_band<DP / 8>(a.dv, n, h, band, k, d, DV, g, t, 1.0f, vec);
      store_band<DP / 8>(a.dk, n, h, band, k, d, DK, g, t, scale, vec);
    }
    write_dbias(P, sGL, n, h, s);
  }
}

template <int DP, bool X3>
__global__ void __launch_bounds__(kThreads) bwd2_tc(const Params P) {
  using L = Layout<DP>;
  extern __shared__ __align__(16) float smem[];
  // grad_logits, d_grad_probs and d_scores, which only the key products
  // need, take the slots of k, v and hk, dead after the row products; those
  // slots hold the larger of a k x d operand and a k x k matrix
  constexpr int SLOT = L::OP > L::KK ? L::OP : L::KK;
  float* sQ = smem;
  float* sK = sQ + L::OP;
  float* sV = sK + SLOT;
  float* sG = sV + SLOT;
  float* sHQ = sG + L::OP;
  float* sHK = sHQ + L::OP;
  float* sHV = sHK + SLOT;
  float* sBias = sHV + L::OP;  // bias tile
  float* sHb = sBias + L::KK;  // hb tile
  float* sLse = sHb + L::KK;
  int32_t* sIdx = reinterpret_cast<int32_t*>(sLse + KP);
  float* sGL = sK;
  float* sDG = sV;
  float* sDS = sHK;
  const cg_edge_attn_args& a = P.a;
  const int k = a.k, d = a.d;
  const float scale = (float)a.scale;
  const bool vec = P.vec_ok;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int band = warp;
  for (int64_t s = blockIdx.x; s < a.n * a.h; s += gridDim.x) {
    const int64_t n = s / a.h, h = s % a.h;
    __syncthreads();
    const int32_t* tix = stage_index(sIdx, a.token_index, n, k);
    // operands in the order the products need them, two cp.async groups
    if (P.same) {
      load_same_async<DP, 4>({sQ, sK, sG, sV}, {a.q, a.k_, a.grad_out, a.v}, n, h, k);
    } else {
      load_op_async<DP>(sQ, a.q, n, h, k, d, vec, tix);
      load_op_async<DP>(sK, a.k_, n, h, k, d, vec, tix);
      load_op_async<DP>(sG, a.grad_out, n, h, k, d, vec);
      load_op_async<DP>(sV, a.v, n, h, k, d, vec, tix);
    }
    const int brow = load_bias(sBias, a.bias, P.bias_mode, n, h, k);
    cp_async_commit();
    if (P.same) {
      load_same_async<DP, 3>({sHQ, sHK, sHV}, {a.hq, a.hk, a.hv}, n, h, k);
    } else {
      load_op_async<DP>(sHQ, a.hq, n, h, k, d, vec, tix);
      load_op_async<DP>(sHK, a.hk, n, h, k, d, vec, tix);
      load_op_async<DP>(sHV, a.hv, n, h, k, d, vec, tix);
    }
    const int hrow = load_bias(sHb, a.hb, P.hb_mode, n, h, k);
    cp_async_commit();
    if (threadIdx.x < KP)
      sLse[threadIdx.x] = threadIdx.x < k ? reinterpret_cast<const float*>(a.lse)[s * k + threadIdx.x] : 0.0f;
    cp_async_wait<1>();
    __syncthreads();
    const int kc = valid_keys(P, n);
    {
      float p[4][4], lse[2], A[4][4], B[4][4];
      zero(A);  // scores
      zero(B);  // grad_probs = grad_out v^T
      band_mma2<X3, 4, DP / 8, true>(A, CG_A_ROWS(sQ), CG_B_ROWS(sK), B, CG_A_ROWS(sG), CG_B_ROWS(sV), g, t);
      band_softmax<!X3>(p, A, sBias, brow, band, g, t, scale, kc, sLse, lse);
      float rs[2];
      row_dot(rs, p, B);
      float cen[4][4];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) cen[nt][e] = B[nt][e] - rs[e >> 1];
      cp_async_wait<0>();
      __syncthreads();
      zero(A);  // d_logits = scale * (hq k^T + q hk^T) + hb
      zero(B);  // grad_out hv^T
      band_mma2<X3, 4, DP / 8, true>(A, CG_A_ROWS(sHQ), CG_B_ROWS(sK), B, CG_A_ROWS(sG), CG_B_ROWS(sHV), g, t);
      band_mma<X3, 4, DP / 8, true>(A, CG_A_ROWS(sQ), CG_B_ROWS(sHK), g, t);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const float2 hb = ld2(sHb, kk((band * 16 + g + 8 * half) & hrow, nt * 8 + 2 * t));
          A[nt][2 * half] = scale * A[nt][2 * half] + hb.x;
          A[nt][2 * half + 1] = scale * A[nt][2 * half + 1] + hb.y;
        }
      float drs[2];
      row_dot(drs, A, p);
      float dg[4][4];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float dr = -drs[e >> 1];
          const float gp = cen[nt][e] + rs[e >> 1];
          B[nt][e] = A[nt][e] * cen[nt][e] + dr * gp + B[nt][e];  // d_probs
          dg[nt][e] = (A[nt][e] + dr) * p[nt][e];                  // d_grad_probs
        }
      float rs2[2];
      row_dot(rs2, p, B);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          A[nt][e] = p[nt][e] * (B[nt][e] - rs2[e >> 1]);  // d_scores
          cen[nt][e] = p[nt][e] * cen[nt][e];              // grad_logits
        }
      // row products with A straight from the fragments
      float DQ[DP / 8][4], DGO[DP / 8][4];
      zero(DQ);   // grad_q = scale * (grad_logits hk + d_scores k)
      zero(DGO);  // grad_out cotangent = d_grad_probs v + probs hv
      band_mma_reg2<X3, DP / 8>(DQ, cen, CG_B_COLS(sHK), DGO, dg, CG_B_COLS(sV), g, t);
      band_mma_reg2<X3, DP / 8>(DQ, A, CG_B_COLS(sK), DGO, p, CG_B_COLS(sHV), g, t);
      store_band<DP / 8>(a.dq, n, h, band, k, d, DQ, g, t, scale, vec);
      store_band<DP / 8>(a.dgrad_out, n, h, band, k, d, DGO, g, t, 1.0f, vec);
      __syncthreads();  // both warps are done with k, v and hk
      put_band(sDG, dg, band, g, t);
      put_band(sGL, cen, band, g, t);
      put_band(sDS, A, band, g, t);
    }
    __syncthreads();
    {
      float DK[DP / 8][4], DV[DP / 8][4];
      zero(DK);  // grad_k = scale * (grad_logits^T hq + d_scores^T q)
      zero(DV);  // grad_v = d_grad_probs^T grad_out
      band_mma2<X3, DP / 8, 4, true>(DK, CG_A_KKT(sGL), CG_B_COLS(sHQ), DV, CG_A_KKT(sDG), CG_B_COLS(sG), g, t);
      band_mma<X3, DP / 8, 4, true>(DK, CG_A_KKT(sDS), CG_B_COLS(sQ), g, t);
      store_band<DP / 8>(a.dk, n, h, band, k, d, DK, g, t, scale, vec);
      store_band<DP / 8>(a.dv, n, h, band, k, d, DV, g, t, 1.0f, vec);
    }
    write_dbias(P, sDS, n, h, s);
  }
}

#undef CG_A_ROWS
#undef CG_B_ROWS
#undef CG_B_COLS
#undef CG_A_KKT

// shared memory per CTA (bytes)
template <int DP>
inline int smem_bytes(int which) {
  using L = Layout<DP>;
  switch (which) {
    case 0: return (3 * L::OP + L::KK + KP) * 4;
    case 1: return (4 * L::OP + 2 * L::KK + 2 * KP) * 4;
    default: return (4 * L::OP + 3 * (L::OP > L::KK ? L::OP : L::KK) + 2 * L::KK + 2 * KP) * 4;
  }
}

// One launch of kernel `which` (0 fwd1, 1 bwd1, 2 bwd2): a persistent grid of
// as many CTAs as fit per SM (shared memory bound), slices strided over it.
template <int DP, bool X3>
int launch_dp(int which, const Params& P, cudaStream_t stream) {
  const int smem = smem_bytes<DP>(which);
  void (*kernel)(const Params) = which == 0 ? fwd1_tc<DP, X3> : which == 1 ? bwd1_tc<DP, X3> : bwd2_tc<DP, X3>;
  CG_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int64_t slices = P.a.n * P.a.h;
  // 228 KB of shared memory per SM, 1 KB of it reserved per resident CTA
  int per_sm = (228 * 1024) / (smem + 1024);
  if (per_sm < 1) per_sm = 1;
  if (per_sm > 16) per_sm = 16;
  const int64_t cap = (int64_t)sm_count() * per_sm;
  const int grid = (int)(slices < cap ? slices : cap);
  kernel<<<grid, kThreads, smem, stream>>>(P);
  CG_LAUNCHED("edge_attn_tc");
  if (which != 0 && P.dbias_mode == 2) return reduce_dbias(P, stream);
  return kOk;
}

template <bool X3>
int launch_prec(int which, const Params& P, int dp, cudaStream_t stream) {
  switch (dp) {
    case 8: return launch_dp<8, X3>(which, P, stream);
    case 16: return launch_dp<16, X3>(which, P, stream);
    case 32: return launch_dp<32, X3>(which, P, stream);
    case 64: return launch_dp<64, X3>(which, P, stream);
  }
  set_error("edge_attn: no tensor-core variant for padded head dim %d", dp);
  return kUnsupported;
}

// the two precisions live in separate translation units (parallel builds)
int launch_fp32(int which, const Params& P, int dp, cudaStream_t stream);  // attn_tc.cu
int launch_tf32(int which, const Params& P, int dp, cudaStream_t stream);  // attn_tc_tf32.cu

}  // namespace attn_tc
}  // namespace cg
