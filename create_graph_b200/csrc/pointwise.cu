// Elementwise and per-row kernels of the energy network: the SiLU derivative
// family, column scale/shift (LayerNorm's affine part), column dot products,
// the row normalisation of LayerNorm with its first and second derivatives,
// and the envelope pooling family (pool / outer / dot).
//
// Row kernels put one warp on one row (lanes over the columns), so every row
// reduction is a fixed-order warp tree: deterministic.
#include <math.h>

#include <initializer_list>

#include "common.cuh"
#include "../../include/cg_b200.h"

namespace cg {
namespace pw {

// logistic sigmoid with the hardware-approximated exp and division (relative
// error ~1e-6), as in the GEMM's SiLU epilogue; exp(-z) = inf gives 0
__device__ inline float sigm(float z) { return __fdividef(1.0f, 1.0f + __expf(-z)); }
// silu(z) = z s, silu' = s (1 + z (1 - s)), silu'' = s (1 - s) (2 + z (1 - 2 s))
__device__ inline float silu_d1(float z) {
  const float s = sigm(z);
  return s * (1.0f + z * (1.0f - s));
}
__device__ inline float silu_d2(float z) {
  const float s = sigm(z);
  return s * (1.0f - s) * (2.0f + z * (1.0f - 2.0f * s));
}
// silu itself, written exactly as the GEMM epilogue writes it, so that an
// activation rebuilt here equals the one the GEMM produced bit for bit
__device__ inline float silu_value(float z) { return __fdividef(z, 1.0f + __expf(-z)); }

__device__ inline float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// 16-byte column vectors: both row-major operands aligned and cols % 4 == 0
inline bool vec_ok(const float* a, const float* b, int64_t cols) {
  return (cols & 3) == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0 && (reinterpret_cast<uintptr_t>(b) & 15) == 0;
}

inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

inline int blocks_for(int64_t n, int threads) {
  const int64_t b = ceil_div<int64_t>(n, threads);
  const int64_t cap = (int64_t)sm_count() * 32;
  return (int)(b < 1 ? 1 : (b < cap ? b : cap));
}

// mode 0: out = a * silu'(z); mode 1: out = a * b * silu''(z); mode 2: out = silu(z)
__global__ void silu_grad_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                 const float* __restrict__ z, float* __restrict__ out, int64_t n,
                                 int mode) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    out[i] = mode == 2 ? silu_value(z[i]) : mode == 0 ? a[i] * silu_d1(z[i]) : a[i] * b[i] * silu_d2(z[i]);
  }
}

// float4 version of silu_grad_kernel (n4 = n / 4 groups, 16-byte aligned)
__global__ void silu_grad4_kernel(const float4* __restrict__ a, const float4* __restrict__ b,
                                  const float4* __restrict__ z, float4* __restrict__ out, int64_t n4, int mode) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 zz = __ldg(z + i);
    if (mode == 2) {
      out[i] = make_float4(silu_value(zz.x), silu_value(zz.y), silu_value(zz.z), silu_value(zz.w));
      continue;
    }
    const float4 x = __ldg(a + i);
    float4 y;
    if (mode == 0) {
      y = make_float4(x.x * silu_d1(zz.x), x.y * silu_d1(zz.y), x.z * silu_d1(zz.z), x.w * silu_d1(zz.w));
    } else {
      const float4 bb = __ldg(b + i);
      y = make_float4(x.x * bb.x * silu_d2(zz.x), x.y * bb.y * silu_d2(zz.y), x.z * bb.z * silu_d2(zz.z),
                      x.w * bb.w * silu_d2(zz.w));
    }
    out[i] = y;
  }
}

// float4 version of scale_shift_kernel: blocks walk rows, threads the row's
// 16-byte column groups (no per-element index division)
__global__ void scale_shift4_kernel(const float4* __restrict__ x, const float4* __restrict__ gamma,
                                    const float4* __restrict__ beta, float4* __restrict__ out, int64_t rows,
                                    int cols4) {
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x)
    for (int c = threadIdx.x; c < cols4; c += blockDim.x) {
      float4 v = __ldg(x + r * cols4 + c);
      if (gamma) {
        const float4 g = __ldg(gamma + c);
        v.x *= g.x; v.y *= g.y; v.z *= g.z; v.w *= g.w;
      }
      if (beta) {
        const float4 b = __ldg(beta + c);
        v.x += b.x; v.y += b.y; v.z += b.z; v.w += b.w;
      }
      out[r * cols4 + c] = v;
    }
}

// out[r, c] = x[r, c] * (gamma ? gamma[c] : 1) + (beta ? beta[c] : 0)
__global__ void scale_shift_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                                   const float* __restrict__ beta, float* __restrict__ out,
                                   int64_t rows, int64_t cols) {
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = i % cols;
    float v = x[i];
    if (gamma) v *= gamma[c];
    if (beta) v += beta[c];
    out[i] = v;
  }
}

// partial[chunk, c] = sum over the chunk's rows of a[r, c] * b[r, c]
__global__ void coldot_partial_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                      int64_t rows, int64_t cols, int64_t rows_per,
                                      float* __restrict__ partial) {
  __shared__ float red[8][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t c = blockIdx.x * 32ll + tx;
  const int64_t r0 = blockIdx.y * rows_per;
  const int64_t r1 = r0 + rows_per < rows ? r0 + rows_per : rows;
  float acc = 0.0f;
  if (c < cols)
    for (int64_t r = r0 + ty; r < r1; r += 8) acc += a[r * cols + c] * b[r * cols + c];
  red[ty][tx] = acc;
  __syncthreads();
  if (ty == 0 && c < cols) {
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += red[i][tx];
    partial[blockIdx.y * cols + c] = s;
  }
}

__global__ void partial_final_kernel(const float* __restrict__ partial, int64_t chunks, int64_t cols,
                                    float* __restrict__ out, bool accumulate) {
  // block: 32 columns x 8 warps; warp w adds chunks w, w + 8, ... of its
  // column, then the 8 warp sums are added in warp order (fixed order)
  __shared__ float red[8][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t c = blockIdx.x * 32ll + tx;
  float s = 0.0f;
  if (c < cols)
    for (int64_t k = ty; k < chunks; k += 8) s += partial[k * cols + c];
  red[ty][tx] = s;
  __syncthreads();
  if (ty == 0 && c < cols) {
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w][tx];
    out[c] = accumulate ? out[c] + t : t;
  }
}

// ---- row normalisation: xhat = (x - mean) / sqrt(var + eps) -----------------
// Per row stats: mean, rstd. One warp per row.
__global__ void rownorm_fwd_kernel(const float* __restrict__ x, int64_t rows, int cols, float eps,
                                   float* __restrict__ xhat, float* __restrict__ rstd_out) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp; r < rows; r += warps) {
    const float* xr = x + r * cols;
    float s = 0.0f;
    for (int c = lane; c < cols; c += 32) s += xr[c];
    const float mean = warp_sum(s) / cols;
    float v = 0.0f;
    for (int c = lane; c < cols; c += 32) {
      const float d = xr[c] - mean;
      v += d * d;
    }
    const float rstd = rsqrtf(warp_sum(v) / cols + eps);
    for (int c = lane; c < cols; c += 32) xhat[r * cols + c] = (xr[c] - mean) * rstd;
    if (lane == 0 && rstd_out) rstd_out[r] = rstd;
  }
}

// gx = rstd * (g - mean(g) - xhat * mean(g * xhat))
// With h (second-order mode), also d_g = rstd * (h - mean(h) - xhat mean(h xhat)) and
// d_x = -xhat (mean(h g) - mean(g) mean(h)) rstd^2 - rstd (c gx' + b hx') + b c xhat rstd^2
// where b = mean(g xhat), c = mean(h xhat), gx' = rstd (g - mean g - xhat b),
// hx' = rstd (h - mean h - xhat c).
__global__ void rownorm_bwd_kernel(const float* __restrict__ x, const float* __restrict__ g,
                                   const float* __restrict__ h, const float* __restrict__ add, int64_t rows,
                                   int cols, float eps, float* __restrict__ out_a, float* __restrict__ out_b) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp; r < rows; r += warps) {
    const float* xr = x + r * cols;
    const float* gr = g + r * cols;
    float s = 0.0f;
    for (int c = lane; c < cols; c += 32) s += xr[c];
    const float mean = warp_sum(s) / cols;
    float v = 0.0f;
    for (int c = lane; c < cols; c += 32) {
      const float d = xr[c] - mean;
      v += d * d;
    }
    const float rstd = rsqrtf(warp_sum(v) / cols + eps);
    float sg = 0.0f, sgx = 0.0f;
    for (int c = lane; c < cols; c += 32) {
      const float xh = (xr[c] - mean) * rstd;
      sg += gr[c];
      sgx += gr[c] * xh;
    }
    const float a = warp_sum(sg) / cols, b = warp_sum(sgx) / cols;
    if (h == nullptr) {
      for (int c = lane; c < cols; c += 32) {
        const float xh = (xr[c] - mean) * rstd;
        out_a[r * cols + c] = rstd * (gr[c] - a - xh * b) + (add != nullptr ? add[r * cols + c] : 0.0f);
      }
      continue;
    }
    const float* hr = h + r * cols;
    float sh = 0.0f, shx = 0.0f, shg = 0.0f;
    for (int c = lane; c < cols; c += 32) {
      const float xh = (xr[c] - mean) * rstd;
      sh += hr[c];
      shx += hr[c] * xh;
      shg += hr[c] * gr[c];
    }
    const float mh = warp_sum(sh) / cols, cc = warp_sum(shx) / cols, mhg = warp_sum(shg) / cols;
    const float r2 = rstd * rstd;
    for (int c = lane; c < cols; c += 32) {
      const float xh = (xr[c] - mean) * rstd;
      const float gx = rstd * (gr[c] - a - xh * b);
      const float hx = rstd * (hr[c] - mh - xh * cc);
      out_b[r * cols + c] = hx;  // d_g
      out_a[r * cols + c] = -xh * (mhg - a * mh) * r2 - (cc * gx + b * hx) * rstd + b * cc * xh * r2;
    }
  }
}

// Row-resident variants for cols = 128 V (V <= 8, 16-byte aligned rows): the
// lanes hold the row in registers as V float4 (column 4 (lane + 32 v)), so x,
// g and h are read from memory once and every statistic is a sum over the
// registers followed by one warp tree. `add` (bwd1 only, may be null) is
// added to gx: the gradient of a residual branch point x -> (x, rownorm(x))
// in the same pass.
template <int V>
__device__ __forceinline__ void load_row(float (&v)[4 * V], const float* row, int lane) {
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const float4 t = reinterpret_cast<const float4*>(row)[lane + 32 * i];
    v[4 * i] = t.x;
    v[4 * i + 1] = t.y;
    v[4 * i + 2] = t.z;
    v[4 * i + 3] = t.w;
  }
}

template <int V>
__device__ __forceinline__ void store_row(float* row, const float (&v)[4 * V], int lane) {
#pragma unroll
  for (int i = 0; i < V; ++i)
    reinterpret_cast<float4*>(row)[lane + 32 * i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

template <int V>
__device__ __forceinline__ void row_stats(const float (&x)[4 * V], int cols, float eps, float& mean, float& rstd) {
  float s = 0.0f;
#pragma unroll
  for (int e = 0; e < 4 * V; ++e) s += x[e];
  mean = warp_sum(s) / cols;
  float q = 0.0f;
#pragma unroll
  for (int e = 0; e < 4 * V; ++e) q += (x[e] - mean) * (x[e] - mean);
  rstd = rsqrtf(warp_sum(q) / cols + eps);
}

template <int V>
__global__ void rownorm_fwd_rows_kernel(const float* __restrict__ x, int64_t rows, int cols, float eps,
                                        float* __restrict__ xhat, float* __restrict__ rstd_out) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp; r < rows; r += warps) {
    float v[4 * V];
    load_row<V>(v, x + r * cols, lane);
    float mean, rstd;
    row_stats<V>(v, cols, eps, mean, rstd);
#pragma unroll
    for (int e = 0; e < 4 * V; ++e) v[e] = (v[e] - mean) * rstd;
    store_row<V>(xhat + r * cols, v, lane);
    if (lane == 0 && rstd_out) rstd_out[r] = rstd;
  }
}

// SECOND = false: out_a = J^T g (+ add); true: out_a = d_x, out_b = d_g of
// <h, J^T g> (no add). Separate instantiations keep the first-order kernel at
// two row arrays of registers (higher residency).
template <int V, bool SECOND>
__global__ void rownorm_bwd_rows_kernel(const float* __restrict__ x, const float* __restrict__ g,
                                        const float* __restrict__ h, const float* __restrict__ add, int64_t rows,
                                        int cols, float eps, float* __restrict__ out_a, float* __restrict__ out_b) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp; r < rows; r += warps) {
    float xh[4 * V], gv[4 * V];
    load_row<V>(xh, x + r * cols, lane);
    load_row<V>(gv, g + r * cols, lane);
    float mean, rstd;
    row_stats<V>(xh, cols, eps, mean, rstd);
    float sg = 0.0f, sgx = 0.0f;
#pragma unroll
    for (int e = 0; e < 4 * V; ++e) {
      xh[e] = (xh[e] - mean) * rstd;
      sg += gv[e];
      sgx += gv[e] * xh[e];
    }
    const float a = warp_sum(sg) / cols, b = warp_sum(sgx) / cols;
    if constexpr (!SECOND) {
#pragma unroll
      for (int e = 0; e < 4 * V; ++e) gv[e] = rstd * (gv[e] - a - xh[e] * b);
      if (add != nullptr) {
        load_row<V>(xh, add + r * cols, lane);  // xh is dead: reuse it for the residual row
#pragma unroll
        for (int e = 0; e < 4 * V; ++e) gv[e] += xh[e];
      }
      store_row<V>(out_a + r * cols, gv, lane);
    } else {
      float hv[4 * V];
      load_row<V>(hv, h + r * cols, lane);
      float sh = 0.0f, shx = 0.0f, shg = 0.0f;
#pragma unroll
      for (int e = 0; e < 4 * V; ++e) {
        sh += hv[e];
        shx += hv[e] * xh[e];
        shg += hv[e] * gv[e];
      }
      const float mh = warp_sum(sh) / cols, cc = warp_sum(shx) / cols, mhg = warp_sum(shg) / cols;
      const float r2 = rstd * rstd;
#pragma unroll
      for (int e = 0; e < 4 * V; ++e) {
        const float gx = rstd * (gv[e] - a - xh[e] * b);
        const float hx = rstd * (hv[e] - mh - xh[e] * cc);
        hv[e] = hx;  // d_g
        gv[e] = -xh[e] * (mhg - a * mh) * r2 - (cc * gx + b * hx) * rstd + b * cc * xh[e] * r2;  // d_x
      }
      store_row<V>(out_b + r * cols, hv, lane);
      store_row<V>(out_a + r * cols, gv, lane);
    }
  }
}

template <int V>
constexpr auto rownorm_bwd1_rows = rownorm_bwd_rows_kernel<V, false>;
template <int V>
constexpr auto rownorm_bwd2_rows = rownorm_bwd_rows_kernel<V, true>;

// V = cols / 128 when the row-resident kernels apply (every pointer 16-byte
// aligned), else 0
inline int rows_v(int64_t cols, std::initializer_list<const void*> ptrs) {
  if (cols % 128 != 0 || cols > 1024) return 0;
  for (const void* p : ptrs)
    if (p != nullptr && !al16(p)) return 0;
  return (int)(cols / 128);
}

#define CG_ROWS_SWITCH(V, KERNEL, GRID, ...)                  \
  switch (V) {                                                 \
    case 1: KERNEL<1><<<GRID, 256, 0, s>>>(__VA_ARGS__); break; \
    case 2: KERNEL<2><<<GRID, 256, 0, s>>>(__VA_ARGS__); break; \
    case 3: KERNEL<3><<<GRID, 256, 0, s>>>(__VA_ARGS__); break; \
    case 4: KERNEL<4><<<GRID, 256, 0, s>>>(__VA_ARGS__); break; \
    case 5: KERNEL<5><<<GRID, 256, 0, s>>>(__VA_ARGS__); break; \
    case 6: KERNEL<6><<<GRID, 256, 0, s>>>(__VA_ARGS__); break; \
    case 7: KERNEL<7><<<GRID, 256, 0, s>>>(__VA_ARGS__); break; \
    default: KERNEL<8><<<GRID, 256, 0, s>>>(__VA_ARGS__); break; \
  }

// ---- AdamW step over flat parameter / gradient / moment buffers -----------------
// torch.optim.AdamW (amsgrad off): p *= 1 - lr wd; m = lerp(m, g, 1 - b1);
// v = b2 v + (1 - b2) g^2; p -= step_size m / (sqrt(v) / sqrt_bc2 + eps), with
// step_size = lr / (1 - b1^t) and sqrt_bc2 = sqrt(1 - b2^t) from the host.
struct AdamW {
  float lr, b1, b2, eps, wd, step_size, sqrt_bc2;
  __device__ __forceinline__ void update(float& p, float g, float& m, float& v) const {
    p *= 1.0f - lr * wd;
    m = fmaf(1.0f - b1, g - m, m);
    v = fmaf(1.0f - b2, g * g, b2 * v);
    p -= step_size * (m / (sqrtf(v) / sqrt_bc2 + eps));
  }
};

// Device-resident step count and bias corrections (cg_adamw_step_counted):
// advanced by one single-thread kernel before each update, so a captured CUDA
// graph replays the right step number every time.
struct AdamWState {
  int64_t step;
  float step_size, sqrt_bc2;
};

__global__ void adamw_advance_kernel(AdamWState* st, float lr, float b1, float b2) {
  const int64_t t = st->step + 1;
  st->step = t;
  st->step_size = (float)((double)lr / (1.0 - pow((double)b1, (double)t)));
  st->sqrt_bc2 = (float)sqrt(1.0 - pow((double)b2, (double)t));
}

__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, int64_t n, AdamW a, bool vec, const AdamWState* st = nullptr) {
  if (st != nullptr) {
    a.step_size = st->step_size;
    a.sqrt_bc2 = st->sqrt_bc2;
  }
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t i0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (vec) {
    for (int64_t i = i0; i < n / 4; i += stride) {
      float4 pp = reinterpret_cast<float4*>(p)[i], mm = reinterpret_cast<float4*>(m)[i],
             vv = reinterpret_cast<float4*>(v)[i];
      const float4 gg = reinterpret_cast<const float4*>(g)[i];
      a.update(pp.x, gg.x, mm.x, vv.x);
      a.update(pp.y, gg.y, mm.y, vv.y);
      a.update(pp.z, gg.z, mm.z, vv.z);
      a.update(pp.w, gg.w, mm.w, vv.w);
      reinterpret_cast<float4*>(p)[i] = pp;
      reinterpret_cast<float4*>(m)[i] = mm;
      reinterpret_cast<float4*>(v)[i] = vv;
    }
    for (int64_t i = n / 4 * 4 + i0; i < n; i += stride) a.update(p[i], g[i], m[i], v[i]);
  } else {
    for (int64_t i = i0; i < n; i += stride) a.update(p[i], g[i], m[i], v[i]);
  }
}

// ---- MSE loss on energies and forces (F = -grad) --------------------------------
// loss = sum_b (E_b - Et_b)^2 / n_e + sum_i (g_i + Ft_i)^2 / n_f, g = dE/dpos.
// One block: each thread sums a fixed strided subset, then a fixed-shape tree
// over the block, so the value is bitwise reproducible.
constexpr int kLossThreads = 1024;

__global__ void __launch_bounds__(kLossThreads) mse_ef_kernel(const float* __restrict__ e, const float* __restrict__ et,
                                                             int64_t n_e, const float* __restrict__ g,
                                                             const float* __restrict__ ft, int64_t n_f,
                                                             float* __restrict__ loss) {
  __shared__ float part[kLossThreads / 32][2];
  float se = 0.0f, sf = 0.0f;
  for (int64_t i = threadIdx.x; i < n_e; i += kLossThreads) {
    const float r = e[i] - et[i];
    se = fmaf(r, r, se);
  }
  for (int64_t i = threadIdx.x; i < n_f; i += kLossThreads) {
    const float r = g[i] + ft[i];
    sf = fmaf(r, r, sf);
  }
  se = warp_sum(se);
  sf = warp_sum(sf);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    part[warp][0] = se;
    part[warp][1] = sf;
  }
  __syncthreads();
  if (warp == 0) {
    se = warp_sum(part[lane][0]);
    sf = warp_sum(part[lane][1]);
    if (lane == 0) *loss = (n_e > 0 ? se / (float)n_e : 0.0f) + (n_f > 0 ? sf / (float)n_f : 0.0f);
  }
}

// dE = 2 (E - Et) / n_e * gl, dg = 2 (g + Ft) / n_f * gl, gl = *grad_loss
__global__ void mse_ef_bwd_kernel(const float* __restrict__ e, const float* __restrict__ et, int64_t n_e,
                                  const float* __restrict__ g, const float* __restrict__ ft, int64_t n_f,
                                  const float* __restrict__ grad_loss, float* __restrict__ de,
                                  float* __restrict__ dg) {
  const float gl = *grad_loss;
  const float ce = n_e > 0 ? 2.0f * gl / (float)n_e : 0.0f, cf = n_f > 0 ? 2.0f * gl / (float)n_f : 0.0f;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_e + n_f; i += stride) {
    if (i < n_e) {
      de[i] = ce * (e[i] - et[i]);
    } else {
      const int64_t j = i - n_e;
      dg[j] = cf * (g[j] + ft[j]);
    }
  }
}

// ---- envelope pooling over the k tokens of each n ------------------------------
// pool:  out[n, c]    = sum_s w[n, s] x[n, s, c]
// outer: out[n, s, c] = w[n, s] g[n, c]
// dot:   out[n, s]    = sum_c g[n, c] x[n, s, c]
// One warp per row n (pool, outer) or per (n, s) pair (dot); lanes walk the
// columns in 16-byte vectors when cols % 4 == 0, with no per-element division.
__global__ void pool_kernel(const float* __restrict__ x, const float* __restrict__ w, int64_t n, int k,
                            int64_t cols, float* __restrict__ out, bool vec) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp; r < n; r += warps) {
    const float* xr = x + r * k * cols;
    const float* wr = w + r * k;
    float* dst = out + r * cols;
    if (vec) {
      for (int64_t c = lane * 4; c < cols; c += 128) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s = 0; s < k; ++s) {
          const float ws = __ldg(wr + s);
          const float4 v = __ldg(reinterpret_cast<const float4*>(xr + (int64_t)s * cols + c));
          acc.x += ws * v.x; acc.y += ws * v.y; acc.z += ws * v.z; acc.w += ws * v.w;
        }
        *reinterpret_cast<float4*>(dst + c) = acc;
      }
    } else {
      for (int64_t c = lane; c < cols; c += 32) {
        float acc = 0.0f;
        for (int s = 0; s < k; ++s) acc += wr[s] * xr[(int64_t)s * cols + c];
        dst[c] = acc;
      }
    }
  }
}

__global__ void outer_kernel(const float* __restrict__ w, const float* __restrict__ g, int64_t n, int k,
                             int64_t cols, float* __restrict__ out, bool vec) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp; r < n; r += warps) {
    const float* gr = g + r * cols;
    for (int s = 0; s < k; ++s) {
      const float ws = __ldg(w + r * k + s);
      float* dst = out + (r * k + s) * cols;
      if (vec) {
        for (int64_t c = lane * 4; c < cols; c += 128) {
          const float4 v = __ldg(reinterpret_cast<const float4*>(gr + c));
          *reinterpret_cast<float4*>(dst + c) = make_float4(ws * v.x, ws * v.y, ws * v.z, ws * v.w);
        }
      } else {
        for (int64_t c = lane; c < cols; c += 32) dst[c] = ws * gr[c];
      }
    }
  }
}

__global__ void dot_kernel(const float* __restrict__ g, const float* __restrict__ x, int64_t n, int k,
                           int64_t cols, float* __restrict__ out, bool vec) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp; r < n; r += warps) {
    const float* gr = g + r * cols;
    for (int s = 0; s < k; ++s) {
      const float* xr = x + (r * k + s) * cols;
      float acc = 0.0f;
      if (vec) {
        for (int64_t c = lane * 4; c < cols; c += 128) {
          const float4 a = __ldg(reinterpret_cast<const float4*>(gr + c));
          const float4 b = __ldg(reinterpret_cast<const float4*>(xr + c));
          acc += a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
        }
      } else {
        for (int64_t c = lane; c < cols; c += 32) acc += gr[c] * xr[c];
      }
      acc = warp_sum(acc);
      if (lane == 0) out[r * k + s] = acc;
    }
  }
}

}  // namespace pw
}  // namespace cg

extern "C" {

using namespace cg;

int cg_silu_grad(const float* a, const float* z, float* out, int64_t n, void* stream) {
  CG_REQUIRE(n >= 0, "silu_grad: negative size");
  if (n == 0) return kOk;
  if (n % 4 == 0 && pw::al16(a) && pw::al16(z) && pw::al16(out))
    pw::silu_grad4_kernel<<<pw::blocks_for(n / 4, 256), 256, 0, as_stream(stream)>>>(
        reinterpret_cast<const float4*>(a), nullptr, reinterpret_cast<const float4*>(z),
        reinterpret_cast<float4*>(out), n / 4, 0);
  else
    pw::silu_grad_kernel<<<pw::blocks_for(n, 256), 256, 0, as_stream(stream)>>>(a, nullptr, z, out, n, 0);
  CG_LAUNCHED("silu_grad");
  return kOk;
}

int cg_silu(const float* z, float* out, int64_t n, void* stream) {
  CG_REQUIRE(n >= 0, "silu: negative size");
  if (n == 0) return kOk;
  if (n % 4 == 0 && pw::al16(z) && pw::al16(out))
    pw::silu_grad4_kernel<<<pw::blocks_for(n / 4, 256), 256, 0, as_stream(stream)>>>(
        nullptr, nullptr, reinterpret_cast<const float4*>(z), reinterpret_cast<float4*>(out), n / 4, 2);
  else
    pw::silu_grad_kernel<<<pw::blocks_for(n, 256), 256, 0, as_stream(stream)>>>(nullptr, nullptr, z, out, n, 2);
  CG_LAUNCHED("silu");
  return kOk;
}

int cg_silu_grad2(const float* a, const float* b, const float* z, float* out, int64_t n, void* stream) {
  CG_REQUIRE(n >= 0, "silu_grad2: negative size");
  if (n == 0) return kOk;
  if (n % 4 == 0 && pw::al16(a) && pw::al16(b) && pw::al16(z) && pw::al16(out))
    pw::silu_grad4_kernel<<<pw::blocks_for(n / 4, 256), 256, 0, as_stream(stream)>>>(
        reinterpret_cast<const float4*>(a), reinterpret_cast<const float4*>(b), reinterpret_cast<const float4*>(z),
        reinterpret_cast<float4*>(out), n / 4, 1);
  else
    pw::silu_grad_kernel<<<pw::blocks_for(n, 256), 256, 0, as_stream(stream)>>>(a, b, z, out, n, 1);
  CG_LAUNCHED("silu_grad2");
  return kOk;
}

int cg_scale_shift(const float* x, const float* gamma, const float* beta, float* out, int64_t rows,
                   int64_t cols, void* stream) {
  CG_REQUIRE(rows >= 0 && cols >= 0, "scale_shift: negative size");
  if (rows * cols == 0) return kOk;
  if (cols % 4 == 0 && pw::al16(x) && pw::al16(out) && (gamma == nullptr || pw::al16(gamma)) &&
      (beta == nullptr || pw::al16(beta))) {
    const int64_t blocks = rows < (int64_t)sm_count() * 16 ? rows : (int64_t)sm_count() * 16;
    pw::scale_shift4_kernel<<<(unsigned)blocks, 128, 0, as_stream(stream)>>>(
        reinterpret_cast<const float4*>(x), reinterpret_cast<const float4*>(gamma),
        reinterpret_cast<const float4*>(beta), reinterpret_cast<float4*>(out), rows, (int)(cols / 4));
  } else {
    pw::scale_shift_kernel<<<pw::blocks_for(rows * cols, 256), 256, 0, as_stream(stream)>>>(x, gamma, beta, out,
                                                                                            rows, cols);
  }
  CG_LAUNCHED("scale_shift");
  return kOk;
}

int64_t cg_coldot_scratch_bytes(int64_t rows, int64_t cols) { return cg_colsum_scratch_bytes(rows, cols); }

int cg_coldot(const float* a, const float* b, int64_t rows, int64_t cols, float* out, int accumulate,
              float* scratch, void* stream) {
  CG_REQUIRE(rows >= 0 && cols >= 0, "coldot: negative size");
  if (cols == 0) return kOk;
  if (rows == 0) {
    if (!accumulate) CG_CUDA(cudaMemsetAsync(out, 0, cols * sizeof(float), as_stream(stream)));
    return kOk;
  }
  CG_REQUIRE(a && b && out && scratch, "coldot: null pointer");
  int64_t chunks, per;
  cg::seg::colsum_plan(rows, cols, &chunks, &per);
  if (!cg::seg::colsum4_launch(a, b, rows, cols, chunks, per, scratch, as_stream(stream))) {
    dim3 grid((unsigned)ceil_div<int64_t>(cols, 32), (unsigned)chunks);
    pw::coldot_partial_kernel<<<grid, 256, 0, as_stream(stream)>>>(a, b, rows, cols, per, scratch);
  }
  CG_LAUNCHED("coldot_partial");
  pw::partial_final_kernel<<<(unsigned)ceil_div<int64_t>(cols, 32), 256, 0, as_stream(stream)>>>(
      scratch, chunks, cols, out, accumulate != 0);
  CG_LAUNCHED("coldot_final");
  return kOk;
}

int cg_rownorm_fwd(const float* x, int64_t rows, int64_t cols, float eps, float* xhat, float* rstd,
                   void* stream) {
  CG_REQUIRE(rows >= 0 && cols >= 1 && cols < (1 << 30), "rownorm: bad size");
  if (rows == 0) return kOk;
  const cudaStream_t s = as_stream(stream);
  const int grid = pw::blocks_for(rows * 32, 256);
  if (const int v = pw::rows_v(cols, {x, xhat})) {
    CG_ROWS_SWITCH(v, pw::rownorm_fwd_rows_kernel, grid, x, rows, (int)cols, eps, xhat, rstd)
  } else {
    pw::rownorm_fwd_kernel<<<grid, 256, 0, s>>>(x, rows, (int)cols, eps, xhat, rstd);
  }
  CG_LAUNCHED("rownorm_fwd");
  return kOk;
}

int cg_rownorm_bwd1_add(const float* x, const float* g, const float* add, int64_t rows, int64_t cols, float eps,
                        float* gx, void* stream) {
  CG_REQUIRE(rows >= 0 && cols >= 1 && cols < (1 << 30), "rownorm: bad size");
  if (rows == 0) return kOk;
  const cudaStream_t s = as_stream(stream);
  const int grid = pw::blocks_for(rows * 32, 256);
  if (const int v = pw::rows_v(cols, {x, g, add, gx})) {
    CG_ROWS_SWITCH(v, pw::rownorm_bwd1_rows, grid, x, g, nullptr, add, rows, (int)cols, eps, gx, nullptr)
  } else {
    pw::rownorm_bwd_kernel<<<grid, 256, 0, s>>>(x, g, nullptr, add, rows, (int)cols, eps, gx, nullptr);
  }
  CG_LAUNCHED("rownorm_bwd1");
  return kOk;
}

int cg_rownorm_bwd1(const float* x, const float* g, int64_t rows, int64_t cols, float eps, float* gx,
                    void* stream) {
  return cg_rownorm_bwd1_add(x, g, nullptr, rows, cols, eps, gx, stream);
}

int cg_rownorm_bwd2(const float* x, const float* g, const float* h, int64_t rows, int64_t cols, float eps,
                    float* d_x, float* d_g, void* stream) {
  CG_REQUIRE(rows >= 0 && cols >= 1 && cols < (1 << 30), "rownorm: bad size");
  if (rows == 0) return kOk;
  CG_REQUIRE(h != nullptr, "rownorm_bwd2: h is NULL");
  const cudaStream_t s = as_stream(stream);
  const int grid = pw::blocks_for(rows * 32, 256);
  if (const int v = pw::rows_v(cols, {x, g, h, d_x, d_g})) {
    CG_ROWS_SWITCH(v, pw::rownorm_bwd2_rows, grid, x, g, h, nullptr, rows, (int)cols, eps, d_x, d_g)
  } else {
    pw::rownorm_bwd_kernel<<<grid, 256, 0, s>>>(x, g, h, nullptr, rows, (int)cols, eps, d_x, d_g);
  }
  CG_LAUNCHED("rownorm_bwd2");
  return kOk;
}

int cg_adamw_step(float* param, const float* grad, float* exp_avg, float* exp_avg_sq, int64_t n, float lr,
                  float beta1, float beta2, float eps, float weight_decay, int64_t step, void* stream) {
  CG_REQUIRE(n >= 0, "adamw: negative size");
  CG_REQUIRE(step >= 1, "adamw: step = %lld, the first step is 1", (long long)step);
  CG_REQUIRE(beta1 >= 0.0f && beta1 < 1.0f && beta2 >= 0.0f && beta2 < 1.0f, "adamw: betas outside [0, 1)");
  if (n == 0) return kOk;
  CG_REQUIRE(param && grad && exp_avg && exp_avg_sq, "adamw: null buffer");
  pw::AdamW a;
  a.lr = lr;
  a.b1 = beta1;
  a.b2 = beta2;
  a.eps = eps;
  a.wd = weight_decay;
  a.step_size = (float)((double)lr / (1.0 - pow((double)beta1, (double)step)));
  a.sqrt_bc2 = (float)sqrt(1.0 - pow((double)beta2, (double)step));
  const bool vec = pw::al16(param) && pw::al16(grad) && pw::al16(exp_avg) && pw::al16(exp_avg_sq);
  pw::adamw_kernel<<<pw::blocks_for(vec ? (n + 3) / 4 : n, 256), 256, 0, as_stream(stream)>>>(
      param, grad, exp_avg, exp_avg_sq, n, a, vec);
  CG_LAUNCHED("adamw");
  return kOk;
}

int cg_adamw_step_counted(float* param, const float* grad, float* exp_avg, float* exp_avg_sq, int64_t n, float lr,
                          float beta1, float beta2, float eps, float weight_decay, void* state, void* stream) {
  CG_REQUIRE(n >= 0, "adamw: negative size");
  CG_REQUIRE(beta1 >= 0.0f && beta1 < 1.0f && beta2 >= 0.0f && beta2 < 1.0f, "adamw: betas outside [0, 1)");
  CG_REQUIRE(state != nullptr, "adamw: state is NULL");
  CG_REQUIRE((reinterpret_cast<uintptr_t>(state) & 7) == 0, "adamw: state must be 8-byte aligned");
  if (n == 0) return kOk;
  CG_REQUIRE(param && grad && exp_avg && exp_avg_sq, "adamw: null buffer");
  pw::AdamW a;
  a.lr = lr;
  a.b1 = beta1;
  a.b2 = beta2;
  a.eps = eps;
  a.wd = weight_decay;
  a.step_size = 0.0f;
  a.sqrt_bc2 = 1.0f;
  auto* st = static_cast<pw::AdamWState*>(state);
  pw::adamw_advance_kernel<<<1, 1, 0, as_stream(stream)>>>(st, lr, beta1, beta2);
  CG_LAUNCHED("adamw counter");
  const bool vec = pw::al16(param) && pw::al16(grad) && pw::al16(exp_avg) && pw::al16(exp_avg_sq);
  pw::adamw_kernel<<<pw::blocks_for(vec ? (n + 3) / 4 : n, 256), 256, 0, as_stream(stream)>>>(
      param, grad, exp_avg, exp_avg_sq, n, a, vec, st);
  CG_LAUNCHED("adamw");
  return kOk;
}

int cg_mse_energy_force(const float* energy, const float* energy_target, int64_t n_energy, const float* grad_pos,
                        const float* force_target, int64_t n_force, float* loss, void* stream) {
  CG_REQUIRE(n_energy >= 0 && n_force >= 0, "mse_energy_force: negative size");
  CG_REQUIRE(loss != nullptr && (n_energy == 0 || (energy && energy_target)) &&
                 (n_force == 0 || (grad_pos && force_target)),
             "mse_energy_force: null buffer");
  pw::mse_ef_kernel<<<1, pw::kLossThreads, 0, as_stream(stream)>>>(energy, energy_target, n_energy, grad_pos,
                                                                  force_target, n_force, loss);
  CG_LAUNCHED("mse_energy_force");
  return kOk;
}

int cg_mse_energy_force_bwd(const float* energy, const float* energy_target, int64_t n_energy, const float* grad_pos,
                            const float* force_target, int64_t n_force, const float* grad_loss, float* d_energy,
                            float* d_grad_pos, void* stream) {
  CG_REQUIRE(n_energy >= 0 && n_force >= 0, "mse_energy_force_bwd: negative size");
  CG_REQUIRE(grad_loss != nullptr, "mse_energy_force_bwd: grad_loss is NULL");
  if (n_energy + n_force == 0) return kOk;
  CG_REQUIRE((n_energy == 0 || (energy && energy_target && d_energy)) &&
                 (n_force == 0 || (grad_pos && force_target && d_grad_pos)),
             "mse_energy_force_bwd: null buffer");
  pw::mse_ef_bwd_kernel<<<pw::blocks_for(n_energy + n_force, 256), 256, 0, as_stream(stream)>>>(
      energy, energy_target, n_energy, grad_pos, force_target, n_force, grad_loss, d_energy, d_grad_pos);
  CG_LAUNCHED("mse_energy_force_bwd");
  return kOk;
}

int cg_pool(const float* x, const float* w, int64_t n, int64_t k, int64_t cols, float* out, void* stream) {
  CG_REQUIRE(n >= 0 && k >= 0 && cols >= 0 && k < (1 << 30), "pool: bad size");
  if (n * cols == 0) return kOk;
  pw::pool_kernel<<<pw::blocks_for(n * 32, 256), 256, 0, as_stream(stream)>>>(x, w, n, (int)k, cols, out,
                                                                                     pw::vec_ok(x, out, cols));
  CG_LAUNCHED("pool");
  return kOk;
}

int cg_pool_outer(const float* w, const float* g, int64_t n, int64_t k, int64_t cols, float* out,
                  void* stream) {
  CG_REQUIRE(n >= 0 && k >= 0 && cols >= 0 && k < (1 << 30), "pool_outer: bad size");
  if (n * k * cols == 0) return kOk;
  pw::outer_kernel<<<pw::blocks_for(n * 32, 256), 256, 0, as_stream(stream)>>>(w, g, n, (int)k, cols, out,
                                                                                      pw::vec_ok(g, out, cols));
  CG_LAUNCHED("pool_outer");
  return kOk;
}

int cg_pool_dot(const float* g, const float* x, int64_t n, int64_t k, int64_t cols, float* out,
                void* stream) {
  CG_REQUIRE(n >= 0 && k >= 0 && cols >= 0 && k < (1 << 30), "pool_dot: bad size");
  if (n * k == 0) return kOk;
  pw::dot_kernel<<<pw::blocks_for(n * 32, 256), 256, 0, as_stream(stream)>>>(g, x, n, (int)k, cols, out,
                                                                                    pw::vec_ok(g, x, cols));
  CG_LAUNCHED("pool_dot");
  return kOk;
}

}  // extern "C"
