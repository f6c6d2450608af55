// Deterministic segment sums over a sorted CSR layout, their transpose (row
// gathers), and column sums.
//
// The reference's models reduce edges to atoms and atoms to systems with
// index_add (tests/test_semantics.py:68-69 there), which on a GPU is an
// atomic scatter whose summation order changes from run to run. Here every
// reduction reads its terms in a fixed order: one warp owns one output row
// and walks its CSR segment sequentially, lanes spread over the columns with
// 16-byte accesses, so results are bitwise reproducible.
#include "common.cuh"
#include "../../include/cg_b200.h"

namespace cg {
namespace seg {

// out[e, :] = index[e] >= 0 ? src[index[e], :] : 0
__global__ void gather_rows_kernel(const float* __restrict__ src, int64_t ld_src,
                                   const int32_t* __restrict__ index, int64_t n_out, int64_t cols,
                                   float* __restrict__ out, int64_t ld_out, bool vec) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t e = warp; e < n_out; e += warps) {
    const int32_t r = index[e];
    float* dst = out + e * ld_out;
    if (vec) {
      const float4* s4 = reinterpret_cast<const float4*>(src + (int64_t)(r < 0 ? 0 : r) * ld_src);
      float4* d4 = reinterpret_cast<float4*>(dst);
      for (int64_t c = lane; c < cols / 4; c += 32) d4[c] = r >= 0 ? __ldg(s4 + c) : make_float4(0, 0, 0, 0);
    } else {
      for (int64_t c = lane; c < cols; c += 32) dst[c] = r >= 0 ? src[(int64_t)r * ld_src + c] : 0.0f;
    }
  }
}

// out[r, :] (+)= sum over e in [row_ptr[r], row_ptr[r+1]) of src[perm ? perm[e] : e, :],
// in increasing e.
__global__ void segment_sum_kernel(const float* __restrict__ src, int64_t ld_src,
                                   const int32_t* __restrict__ row_ptr,
                                   const int32_t* __restrict__ perm, int64_t n_rows, int64_t cols,
                                   float* __restrict__ out, int64_t ld_out, bool accumulate, bool vec) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp; r < n_rows; r += warps) {
    const int32_t e0 = row_ptr[r], e1 = row_ptr[r + 1];
    float* dst = out + r * ld_out;
    if (vec) {
      float4* d4 = reinterpret_cast<float4*>(dst);
      for (int64_t c = lane; c < cols / 4; c += 32) {
        float4 acc = accumulate ? d4[c] : make_float4(0, 0, 0, 0);
        for (int32_t e = e0; e < e1; ++e) {
          const int64_t s = perm ? perm[e] : e;
          const float4 v = __ldg(reinterpret_cast<const float4*>(src + s * ld_src) + c);
          acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
        }
        d4[c] = acc;
      }
    } else {
      for (int64_t c = lane; c < cols; c += 32) {
        float acc = accumulate ? dst[c] : 0.0f;
        for (int32_t e = e0; e < e1; ++e) {
          const int64_t s = perm ? perm[e] : e;
          acc += src[s * ld_src + c];
        }
        dst[c] = acc;
      }
    }
  }
}

// 16-byte variant of segment_sum_kernel with one warp per (row, block of 128
// columns): a lane owns one float4 column chunk and walks the segment in
// increasing e, loads unrolled ahead of the ordered adds; rows x blocks warps
// keep enough loads in flight for HBM.
__global__ void segment_sum_blocks_kernel(const float* __restrict__ src, int64_t ld_src,
                                          const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ perm,
                                          int64_t n_rows, int cols4, float* __restrict__ out, int64_t ld_out,
                                          bool accumulate) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int nblk = (cols4 + 31) / 32;
  for (int64_t task = warp; task < n_rows * nblk; task += warps) {
    const int64_t r = task / nblk;
    const int c = (int)(task % nblk) * 32 + lane;
    if (c >= cols4) continue;
    const int32_t e0 = row_ptr[r], e1 = row_ptr[r + 1];
    float4* dst = reinterpret_cast<float4*>(out + r * ld_out) + c;
    float4 acc = accumulate ? *dst : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll 8
    for (int32_t e = e0; e < e1; ++e) {
      const int64_t s = perm ? perm[e] : e;
      const float4 v = __ldg(reinterpret_cast<const float4*>(src + s * ld_src) + c);
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    *dst = acc;
  }
}

// The rank-one version, the same way (d a multiple of 4).
__global__ void segment_sum_scaled_blocks_kernel(const float* __restrict__ w, const float* __restrict__ src,
                                                 int64_t ld_src, int group, int heads, int d,
                                                 const int32_t* __restrict__ row_ptr,
                                                 const int32_t* __restrict__ perm, int64_t n_rows,
                                                 float* __restrict__ out, int64_t ld_out, bool accumulate) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int cols4 = heads * d / 4;
  const int nblk = (cols4 + 31) / 32;
  for (int64_t task = warp; task < n_rows * nblk; task += warps) {
    const int64_t r = task / nblk;
    const int c = (int)(task % nblk) * 32 + lane;
    if (c >= cols4) continue;
    const int hh = 4 * c / d;
    const int32_t e0 = row_ptr[r], e1 = row_ptr[r + 1];
    float4* dst = reinterpret_cast<float4*>(out + r * ld_out) + c;
    float4 acc = accumulate ? *dst : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll 8
    for (int32_t e = e0; e < e1; ++e) {
      const int32_t s = perm ? perm[e] : e;
      const float wt = __ldg(w + (int64_t)s * heads + hh);
      const float4 v = __ldg(reinterpret_cast<const float4*>(src + (int64_t)(s / group) * ld_src) + c);
      acc.x += wt * v.x; acc.y += wt * v.y; acc.z += wt * v.z; acc.w += wt * v.w;
    }
    *dst = acc;
  }
}

// out[r, h*d + c] (+)= sum over e in [row_ptr[r], row_ptr[r+1]) of
// w[s*heads + h] * src[(s / group)*ld_src + h*d + c], s = perm ? perm[e] : e,
// in increasing e: one warp per output row, lanes over 4-column chunks (vec:
// d a multiple of 4, so a chunk never straddles two heads).
__global__ void segment_sum_scaled_kernel(const float* __restrict__ w, const float* __restrict__ src,
                                          int64_t ld_src, int group, int heads, int d,
                                          const int32_t* __restrict__ row_ptr,
                                          const int32_t* __restrict__ perm, int64_t n_rows,
                                          float* __restrict__ out, int64_t ld_out, bool accumulate,
                                          bool vec) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int cols = heads * d;
  for (int64_t r = warp; r < n_rows; r += warps) {
    const int32_t e0 = row_ptr[r], e1 = row_ptr[r + 1];
    float* dst = out + r * ld_out;
    if (vec) {
      for (int c = lane * 4; c < cols; c += 128) {
        const int hh = c / d;
        float4 acc = accumulate ? *reinterpret_cast<const float4*>(dst + c) : make_float4(0, 0, 0, 0);
        for (int32_t e = e0; e < e1; ++e) {
          const int32_t s = perm ? perm[e] : e;
          const float wt = __ldg(w + (int64_t)s * heads + hh);
          const float4 v = __ldg(reinterpret_cast<const float4*>(src + (int64_t)(s / group) * ld_src + c));
          acc.x += wt * v.x; acc.y += wt * v.y; acc.z += wt * v.z; acc.w += wt * v.w;
        }
        *reinterpret_cast<float4*>(dst + c) = acc;
      }
    } else {
      for (int c = lane; c < cols; c += 32) {
        const int hh = c / d;
        float acc = accumulate ? dst[c] : 0.0f;
        for (int32_t e = e0; e < e1; ++e) {
          const int32_t s = perm ? perm[e] : e;
          acc += w[(int64_t)s * heads + hh] * src[(int64_t)(s / group) * ld_src + c];
        }
        dst[c] = acc;
      }
    }
  }
}

// Column sums in two fixed-order passes: block (cb, chunk) sums rows
// [chunk*rows_per, (chunk+1)*rows_per) of 32 columns into partial[chunk, :];
// then one thread per column adds the partials in chunk order.
constexpr int kColTile = 32;

__global__ void colsum_partial_kernel(const float* __restrict__ src, int64_t ld, int64_t rows,
                                      int64_t cols, int64_t rows_per, float* __restrict__ partial) {
  __shared__ float red[8][kColTile + 1];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
  const int64_t c = blockIdx.x * (int64_t)kColTile + tx;
  const int64_t r0 = blockIdx.y * rows_per;
  const int64_t r1 = r0 + rows_per < rows ? r0 + rows_per : rows;
  float acc = 0.0f;
  if (c < cols)
    for (int64_t r = r0 + ty; r < r1; r += 8) acc += src[r * ld + c];
  red[ty][tx] = acc;
  __syncthreads();
  if (ty == 0 && c < cols) {
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += red[i][tx];
    partial[blockIdx.y * cols + c] = s;
  }
}

// Column sums (b == null) or column dot products (sum_r a[r, c] b[r, c]) of
// 16-byte rows over one chunk of rows: partial[chunk, c]. A lane owns four
// columns; the 8 warps of a block take interleaved rows, four rows in flight
// per thread; matrices narrower than 128 columns pack 32 / (cols / 4) rows into
// one warp step. The block's lanes are then summed in a fixed order (warp,
// packed row), so results are reproducible.
__global__ void colsum4_partial_kernel(const float* __restrict__ a, const float* __restrict__ b, int64_t lda,
                                       int64_t ldb, int64_t rows, int cols4, int64_t rows_per,
                                       float* __restrict__ partial) {
  __shared__ float4 red[8][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int span = cols4 < 32 ? cols4 : 32;  // float4 columns a warp covers per row
  const int pack = 32 / span;                // rows per warp step
  const int rr = lane / span, c4 = blockIdx.x * 32 + lane % span;
  const bool active = rr < pack && c4 < cols4;
  const int64_t r0 = blockIdx.y * rows_per;
  const int64_t r1 = r0 + rows_per < rows ? r0 + rows_per : rows;
  const int64_t step = 8 * (int64_t)pack;
  float4 acc[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) acc[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  if (active) {
    int64_t r = r0 + w * pack + rr;
    for (; r + 3 * step < r1; r += 4 * step) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float4 x = __ldg(reinterpret_cast<const float4*>(a + (r + u * step) * lda) + c4);
        if (b != nullptr) {
          const float4 y = __ldg(reinterpret_cast<const float4*>(b + (r + u * step) * ldb) + c4);
          x.x *= y.x; x.y *= y.y; x.z *= y.z; x.w *= y.w;
        }
        acc[u].x += x.x; acc[u].y += x.y; acc[u].z += x.z; acc[u].w += x.w;
      }
    }
    for (; r < r1; r += step) {
      float4 x = __ldg(reinterpret_cast<const float4*>(a + r * lda) + c4);
      if (b != nullptr) {
        const float4 y = __ldg(reinterpret_cast<const float4*>(b + r * ldb) + c4);
        x.x *= y.x; x.y *= y.y; x.z *= y.z; x.w *= y.w;
      }
      acc[0].x += x.x; acc[0].y += x.y; acc[0].z += x.z; acc[0].w += x.w;
    }
  }
  float4 tot;
  tot.x = (acc[0].x + acc[1].x) + (acc[2].x + acc[3].x);
  tot.y = (acc[0].y + acc[1].y) + (acc[2].y + acc[3].y);
  tot.z = (acc[0].z + acc[1].z) + (acc[2].z + acc[3].z);
  tot.w = (acc[0].w + acc[1].w) + (acc[2].w + acc[3].w);
  red[w][lane] = tot;
  __syncthreads();
  if ((int)threadIdx.x < span) {
    const int cc = blockIdx.x * 32 + threadIdx.x;
    if (cc < cols4) {
      float4 sum = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      for (int ww = 0; ww < 8; ++ww)
        for (int q = 0; q < pack; ++q) {
          const float4 v = red[ww][q * span + threadIdx.x];
          sum.x += v.x; sum.y += v.y; sum.z += v.z; sum.w += v.w;
        }
      reinterpret_cast<float4*>(partial + blockIdx.y * (int64_t)cols4 * 4)[cc] = sum;
    }
  }
}

__global__ void colsum_final_kernel(const float* __restrict__ partial, int64_t chunks, int64_t cols,
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

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static int grid_for_warps(int64_t items) {
  const int64_t blocks = ceil_div<int64_t>(items, 8);  // 8 warps per 256-thread block
  const int64_t cap = (int64_t)sm_count() * 16;
  return (int)(blocks < 1 ? 1 : (blocks < cap ? blocks : cap));
}

void colsum_plan(int64_t rows, int64_t cols, int64_t* chunks, int64_t* rows_per) {
  // enough row chunks of 128-column blocks for ~16 blocks per SM, each chunk
  // at least 64 rows, at most 512 chunks (the final pass reads them all)
  const int64_t col_blocks = ceil_div<int64_t>(cols, 128);
  int64_t want = ceil_div<int64_t>((int64_t)sm_count() * 16, col_blocks);
  if (want > 512) want = 512;
  int64_t per = ceil_div<int64_t>(rows, want < 1 ? 1 : want);
  if (per < 64) per = 64;
  *rows_per = per;
  *chunks = ceil_div<int64_t>(rows, per);
}

bool colsum4_launch(const float* a, const float* b, int64_t rows, int64_t cols, int64_t chunks, int64_t rows_per,
                    float* partial, cudaStream_t s) {
  if (cols % 4 != 0 || !aligned16(a) || (b != nullptr && !aligned16(b)) || !aligned16(partial)) return false;
  const int cols4 = (int)(cols / 4);
  dim3 grid((unsigned)(cols4 < 32 ? 1 : ceil_div<int64_t>(cols4, 32)), (unsigned)chunks);
  colsum4_partial_kernel<<<grid, 256, 0, s>>>(a, b, cols, cols, rows, cols4, rows_per, partial);
  return true;
}

int colsum_launch(const float* src, int64_t ld, int64_t rows, int64_t cols, float* out, int accumulate,
                  float* partial, cudaStream_t s) {
  int64_t chunks, per;
  colsum_plan(rows, cols, &chunks, &per);
  if (cols % 4 == 0 && ld % 4 == 0 && aligned16(src) && aligned16(partial)) {
    const int cols4 = (int)(cols / 4);
    dim3 grid((unsigned)(cols4 < 32 ? 1 : ceil_div<int64_t>(cols4, 32)), (unsigned)chunks);
    colsum4_partial_kernel<<<grid, 256, 0, s>>>(src, nullptr, ld, 0, rows, cols4, per, partial);
  } else {
    dim3 grid((unsigned)ceil_div<int64_t>(cols, kColTile), (unsigned)chunks);
    colsum_partial_kernel<<<grid, 256, 0, s>>>(src, ld, rows, cols, per, partial);
  }
  CG_LAUNCHED("colsum_partial");
  colsum_final_kernel<<<(unsigned)ceil_div<int64_t>(cols, 32), 256, 0, s>>>(partial, chunks, cols, out,
                                                                               accumulate != 0);
  CG_LAUNCHED("colsum_final");
  return kOk;
}


// ---- CSR of a small many-to-one map (species and similar) -----------------------
// One block of 1024 threads, rows <= kCsrMaxRows: counts per row (shared
// atomics on integers: exact), an exclusive scan into row_ptr, then a stable
// placement pass over 1024-element chunks in which each element's rank among
// the chunk's elements of its row is its in-warp rank (match + popc) plus the
// counts of the earlier warps, so perm lists every row's elements in
// ascending order. No host synchronisation: sizes are known up front.
constexpr int kCsrMaxRows = 256;
constexpr int kCsrThreads = 1024;

__global__ void __launch_bounds__(kCsrThreads) csr_small_kernel(const int32_t* __restrict__ index, int64_t n, int rows,
                                                               int32_t* __restrict__ row_ptr,
                                                               int32_t* __restrict__ perm) {
  __shared__ int count[kCsrMaxRows];
  __shared__ int start[kCsrMaxRows];
  __shared__ int warp_count[kCsrThreads / 32][kCsrMaxRows];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int r = tid; r < rows; r += kCsrThreads) count[r] = 0;
  __syncthreads();
  for (int64_t e = tid; e < n; e += kCsrThreads) {
    const int r = index[e];
    if (r >= 0 && r < rows) atomicAdd(&count[r], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int r = 0; r < rows; ++r) {
      start[r] = acc;
      row_ptr[r] = acc;
      acc += count[r];
    }
    row_ptr[rows] = acc;
  }
  __syncthreads();
  for (int64_t base = 0; base < n; base += kCsrThreads) {
    const int64_t e = base + tid;
    const int r = e < n ? index[e] : -1;
    const bool ok = r >= 0 && r < rows;
    for (int i = tid; i < (kCsrThreads / 32) * rows; i += kCsrThreads) warp_count[i / rows][i % rows] = 0;
    __syncthreads();
    const unsigned peers = __match_any_sync(0xffffffffu, ok ? r : -1);
    const int in_warp = __popc(peers & ((1u << lane) - 1u));
    if (ok && in_warp == 0) warp_count[warp][r] = __popc(peers);
    __syncthreads();
    if (ok) {
      int before = 0;
      for (int w = 0; w < warp; ++w) before += warp_count[w][r];
      // in [0, n) by construction (counts of distinct elements); kept as a guard
      const int64_t slot = (int64_t)start[r] + before + in_warp;
      if (slot >= 0 && slot < n) perm[slot] = (int32_t)e;
    }
    __syncthreads();
    // advance each row's start by this chunk's elements of it
    for (int rr = tid; rr < rows; rr += kCsrThreads) {
      int add = 0;
      for (int w = 0; w < kCsrThreads / 32; ++w) add += warp_count[w][rr];
      start[rr] += add;
    }
    __syncthreads();
  }
  // slots past the mapped elements (index outside [0, rows)) hold -1
  for (int64_t e = (int64_t)row_ptr[rows] + tid; e < n; e += kCsrThreads) perm[e] = -1;
}

// CSR of any many-to-one map over the whole input: element e goes to row
// index[e] (outside [0, rows): nowhere). Counts per row with integer
// atomics into row_ptr, an inclusive scan, each element placed at
// atomicSub(end of its row) - 1 (which leaves row_ptr[r] at the row's start),
// then every row sorted by element index, which fixes the order: perm lists
// each row's elements in ascending order on every run.
__global__ void count_rows_kernel(const int32_t* __restrict__ index, int64_t n, int64_t rows,
                                  int32_t* __restrict__ cnt) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int32_t r = index[e];
    if (r >= 0 && r < rows) atomicAdd(&cnt[r], 1);
  }
}

// In place inclusive scan of x[0, n) by one block of kScanThreads threads
// (a contiguous chunk each, then a scan of the chunk totals); x[n] = total.
constexpr int kScanThreads = 1024;
__global__ void __launch_bounds__(kScanThreads) scan_inclusive_kernel(int32_t* __restrict__ x, int64_t n) {
  __shared__ int32_t part[kScanThreads];
  const int t = threadIdx.x;
  const int64_t per = (n + kScanThreads - 1) / kScanThreads;
  const int64_t b0 = t * per < n ? t * per : n, b1 = b0 + per < n ? b0 + per : n;
  int32_t sum = 0;
  for (int64_t e = b0; e < b1; ++e) sum += x[e];
  part[t] = sum;
  __syncthreads();
  for (int off = 1; off < kScanThreads; off <<= 1) {  // Hillis-Steele over the chunk totals
    const int32_t v = t >= off ? part[t - off] : 0;
    __syncthreads();
    part[t] += v;
    __syncthreads();
  }
  int32_t run = t > 0 ? part[t - 1] : 0;
  for (int64_t e = b0; e < b1; ++e) {
    run += x[e];
    x[e] = run;
  }
  if (t == kScanThreads - 1) x[n] = part[t];
}

__global__ void place_rows_kernel(const int32_t* __restrict__ index, int64_t n, int64_t rows,
                                  int32_t* __restrict__ end, int32_t* __restrict__ perm) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int32_t r = index[e];
    if (r >= 0 && r < rows) perm[atomicSub(&end[r], 1) - 1] = (int32_t)e;
  }
}

// Insertion sort of each row's segment of perm.
__global__ void sort_rows_kernel(const int32_t* __restrict__ row_ptr, int64_t rows, int32_t* __restrict__ perm) {
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < rows; j += (int64_t)gridDim.x * blockDim.x) {
    const int32_t s0 = row_ptr[j], s1 = row_ptr[j + 1];
    for (int32_t a = s0 + 1; a < s1; ++a) {
      const int32_t v = perm[a];
      int32_t b = a;
      while (b > s0 && perm[b - 1] > v) {
        perm[b] = perm[b - 1];
        --b;
      }
      perm[b] = v;
    }
  }
}

int csr_build_launch(const int32_t* index, int64_t n, int64_t rows, int32_t* row_ptr, int32_t* perm,
                     cudaStream_t s) {
  CG_CUDA(cudaMemsetAsync(row_ptr, 0, (rows + 1) * sizeof(int32_t), s));
  if (n == 0) return kOk;
  CG_CUDA(cudaMemsetAsync(perm, 0xff, n * sizeof(int32_t), s));  // -1 past the mapped elements
  const int64_t cap = (int64_t)sm_count() * 8;
  auto grid = [&](int64_t items) {
    const int64_t b = (items + 255) / 256;
    return (unsigned)(b < 1 ? 1 : (b < cap ? b : cap));
  };
  count_rows_kernel<<<grid(n), 256, 0, s>>>(index, n, rows, row_ptr);
  CG_LAUNCHED("csr count");
  scan_inclusive_kernel<<<1, kScanThreads, 0, s>>>(row_ptr, rows);
  CG_LAUNCHED("csr scan");
  place_rows_kernel<<<grid(n), 256, 0, s>>>(index, n, rows, row_ptr, perm);
  CG_LAUNCHED("csr place");
  sort_rows_kernel<<<grid(rows), 256, 0, s>>>(row_ptr, rows, perm);
  CG_LAUNCHED("csr sort");
  return kOk;
}

}  // namespace seg
}  // namespace cg

extern "C" {

int cg_csr_from_index(const int32_t* index, int64_t n, int64_t rows, int32_t* row_ptr, int32_t* perm, void* stream) {
  CG_REQUIRE(n >= 0 && n < (1ll << 31), "csr_from_index: n = %lld outside [0, 2^31)", (long long)n);
  CG_REQUIRE(rows >= 0 && rows < (1ll << 31), "csr_from_index: rows = %lld outside [0, 2^31)", (long long)rows);
  CG_REQUIRE(row_ptr != nullptr && (n == 0 || (index != nullptr && perm != nullptr)),
             "csr_from_index: null buffer");
  if (rows > cg::seg::kCsrMaxRows) return cg::seg::csr_build_launch(index, n, rows, row_ptr, perm, cg::as_stream(stream));
  cg::seg::csr_small_kernel<<<1, cg::seg::kCsrThreads, 0, cg::as_stream(stream)>>>(index, n, (int)rows, row_ptr, perm);
  CG_LAUNCHED("csr_from_index");
  return cg::kOk;
}

int cg_gather_rows(const float* src, int64_t ld_src, const int32_t* index, int64_t n_out, int64_t cols,
                   float* out, int64_t ld_out, void* stream) {
  using namespace cg;
  CG_REQUIRE(n_out >= 0 && cols >= 0, "gather_rows: negative size");
  if (n_out == 0 || cols == 0) return kOk;
  CG_REQUIRE(src && index && out, "gather_rows: null pointer");
  const bool vec = cols % 4 == 0 && ld_src % 4 == 0 && ld_out % 4 == 0 && seg::aligned16(src) &&
                   seg::aligned16(out);
  seg::gather_rows_kernel<<<seg::grid_for_warps(n_out), 256, 0, as_stream(stream)>>>(
      src, ld_src, index, n_out, cols, out, ld_out, vec);
  CG_LAUNCHED("gather_rows");
  return kOk;
}

int cg_segment_sum(const float* src, int64_t ld_src, const int32_t* row_ptr, const int32_t* perm,
                   int64_t n_rows, int64_t cols, float* out, int64_t ld_out, int accumulate,
                   void* stream) {
  using namespace cg;
  CG_REQUIRE(n_rows >= 0 && cols >= 0, "segment_sum: negative size");
  if (n_rows == 0 || cols == 0) return kOk;
  CG_REQUIRE(src && row_ptr && out, "segment_sum: null pointer");
  const bool vec = cols % 4 == 0 && ld_src % 4 == 0 && ld_out % 4 == 0 && seg::aligned16(src) &&
                   seg::aligned16(out);
  if (vec) {
    const int64_t tasks = n_rows * ceil_div<int64_t>(cols / 4, 32);
    seg::segment_sum_blocks_kernel<<<seg::grid_for_warps(tasks), 256, 0, as_stream(stream)>>>(
        src, ld_src, row_ptr, perm, n_rows, (int)(cols / 4), out, ld_out, accumulate != 0);
  } else {
    seg::segment_sum_kernel<<<seg::grid_for_warps(n_rows), 256, 0, as_stream(stream)>>>(
        src, ld_src, row_ptr, perm, n_rows, cols, out, ld_out, accumulate != 0, vec);
  }
  CG_LAUNCHED("segment_sum");
  return kOk;
}

int cg_segment_sum_scaled(const float* w, const float* src, int64_t ld_src, int64_t group, int32_t heads,
                          int32_t d, const int32_t* row_ptr, const int32_t* perm, int64_t n_rows, float* out,
                          int64_t ld_out, int accumulate, void* stream) {
  using namespace cg;
  CG_REQUIRE(n_rows >= 0 && heads >= 0 && d >= 0, "segment_sum_scaled: negative size");
  if (n_rows == 0 || heads == 0 || d == 0) return kOk;
  CG_REQUIRE(w && src && row_ptr && out, "segment_sum_scaled: null pointer");
  CG_REQUIRE(group >= 1 && group <= (1 << 30), "segment_sum_scaled: group = %lld outside [1, 2^30]",
             (long long)group);
  const bool vec = d % 4 == 0 && ld_src % 4 == 0 && ld_out % 4 == 0 && seg::aligned16(src) && seg::aligned16(out);
  if (vec) {
    const int64_t tasks = n_rows * ceil_div<int64_t>((int64_t)heads * d / 4, 32);
    seg::segment_sum_scaled_blocks_kernel<<<seg::grid_for_warps(tasks), 256, 0, as_stream(stream)>>>(
        w, src, ld_src, (int)group, heads, d, row_ptr, perm, n_rows, out, ld_out, accumulate != 0);
  } else {
    seg::segment_sum_scaled_kernel<<<seg::grid_for_warps(n_rows), 256, 0, as_stream(stream)>>>(
        w, src, ld_src, (int)group, heads, d, row_ptr, perm, n_rows, out, ld_out, accumulate != 0, vec);
  }
  CG_LAUNCHED("segment_sum_scaled");
  return kOk;
}

int64_t cg_colsum_scratch_bytes(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  int64_t chunks, per;
  cg::seg::colsum_plan(rows, cols, &chunks, &per);
  return chunks * cols * (int64_t)sizeof(float);
}

int cg_colsum(const float* src, int64_t ld, int64_t rows, int64_t cols, float* out, int accumulate,
              float* scratch, void* stream) {
  using namespace cg;
  CG_REQUIRE(rows >= 0 && cols >= 0, "colsum: negative size");
  if (cols == 0) return kOk;
  if (rows == 0) {
    if (!accumulate) CG_CUDA(cudaMemsetAsync(out, 0, cols * sizeof(float), as_stream(stream)));
    return kOk;
  }
  CG_REQUIRE(src && out && scratch, "colsum: null pointer (scratch: cg_colsum_scratch_bytes bytes)");
  return seg::colsum_launch(src, ld, rows, cols, out, accumulate, scratch, as_stream(stream));
}

}  // extern "C"
