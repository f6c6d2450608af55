// Dense projections on the 5th-generation tensor cores: C = epilogue(A . B^T)
// with kind::tf32 UMMA (fp32 in, fp32 accumulate in TMEM).
//
// Persistent: one CTA per SM walks the BM x BN output tiles (BM = 128,
// BN in {16, 32, 64, 128, 192, 256}) and k-splits:
//   warp 0        TMA producer: A and B k-slices of 32 fp32 (128 B, 128B
//                 swizzle) into a ring of STAGES shared-memory stages;
//   warp 1        allocates TMEM (two accumulators); one thread issues 4 UMMAs
//                 (K = 8) per stage and commits each stage back to the producer
//                 and each finished accumulator to the epilogue;
//   warps 2..5    epilogue: tcgen05.ld of the accumulator (one TMEM lane =
//                 one output row per thread), a shared-memory transpose,
//                 bias / SiLU / SiLU-derivative / accumulate and coalesced
//                 stores, overlapping the next tile's UMMAs.
// A and B are each either K-major (rows contiguous along K) or MN-major
// (contiguous along M / N), so the forward (x W^T), the data gradient (g W)
// and the weight gradient (g^T x) all read their operands in place.
// Precision: CG_GEMM_TF32 makes one tf32 product per k-slice. CG_GEMM_FP32
// adds a converter warpgroup (warps 2 + EPI ..): once a stage lands it
// rewrites every operand x in place as hi = x truncated to tf32 and writes
// lo = x - hi (exact) beside it; the issuer then accumulates A_lo B_hi +
// A_hi B_lo + A_hi B_hi, which keeps fp32-level accuracy (the dropped
// A_lo B_lo term and lo's own tf32 rounding are ~2^-21 relative).
// Every mbarrier wait is bounded: on timeout the kernel records an error in
// the device error word and unwinds, freeing its TMEM.
#include <cudaTypedefs.h>
#include <math.h>

#include <atomic>

#include "common.cuh"
#include "sm100.cuh"
#include "../../include/cg_b200.h"

namespace cg {
namespace gemm {

// device error word of this translation unit's kernels
__device__ int g_gemm_error = 0;

using namespace cg::sm100;

constexpr int BM = 128;
constexpr int BK = 32;  // fp32 elements per k-slice: one 128-byte swizzle row
// warp 0 TMA producer, warp 1 UMMA issuer, then EPI epilogue warps (4, or 8 for
// GEMMs whose epilogue streams extra operands: two warps per TMEM lane quarter),
// then, in the three-term split mode, CONV converter warps
constexpr int CONV = 4;
__host__ __device__ constexpr int threads_of(int epi, bool split = false) { return 32 * (2 + epi + (split ? CONV : 0)); }
// floats per staged epilogue row (a 32 x 32 block per warp); the row's eight
// 16-byte chunks are XOR-swizzled by (row & 7), so both the row-per-lane
// writes and the 4-rows-per-instruction reads are free of bank conflicts
// without padding
constexpr int kStagePitch = 32;
__device__ __forceinline__ int stage_idx(int r, int c) {
  return r * kStagePitch + ((((c >> 2) ^ (r & 7)) << 2) | (c & 3));
}

struct Epilogue {
  float* c;
  int64_t ldc;
  const float* bias;    // (N,) or null
  const float* aux_in;  // (M, N) SiLU pre-activation (SILU_GRAD) or residual (ADD), ld = ld_aux
  float* aux_out;       // (M, N) pre-activation written by the SiLU forward, ld = ld_aux
  int64_t ld_aux;
  int act;              // CG_ACT_*
  int accumulate;       // C += result
  float alpha;
  int vec;              // 16-byte column groups: N, ldc, ld_aux multiples of 4, pointers aligned
};

// SiLU and its derivative in the epilogue, with the hardware-approximated
// exp and division (relative error ~1e-6, far below the tf32 rounding of the
// products): the epilogue warps apply them to every output element, and with
// the accurate expf and IEEE division they, not the tensor cores, bound the
// SiLU GEMMs. exp(-z) overflowing to inf gives silu = 0 and silu' = 0.
__device__ inline float silu(float z) { return __fdividef(z, 1.0f + __expf(-z)); }
__device__ inline float silu_grad(float z) {
  const float s = __fdividef(1.0f, 1.0f + __expf(-z));
  return s * (1.0f + z * (1.0f - s));
}

// x = hi + lo with hi = x truncated to tf32 (the low 13 mantissa bits
// cleared: exactly representable, so the tensor core's own tf32 conversion
// leaves it alone) and lo = x - hi (exact in fp32). A non-finite operand makes
// its products NaN in this mode (inf - inf, or inf times a zero lo term).
__device__ inline void split_tf32(float x, float& hi, float& lo) {
  hi = __uint_as_float(__float_as_uint(x) & 0xffffe000u);
  lo = x - hi;
}

template <int BN, int STAGES, int EPI = 4, bool SPLIT = false>
struct Smem {
  static constexpr int kA = BM * BK * 4;
  static constexpr int kB = BN * BK * 4;
  static constexpr int kLoad = kA + kB;                      // bytes TMA brings per stage
  static constexpr int kStage = SPLIT ? 2 * kLoad : kLoad;   // + the lo copies of A and B
  static_assert(kLoad % 1024 == 0, "lo tiles keep the 1024-byte swizzle alignment");
  static constexpr int kTiles = STAGES * kStage;
  static constexpr int kStaging = EPI * 32 * kStagePitch * 4;  // epilogue transpose, one 32 x 32 block per warp
  static constexpr int kBytes = kTiles + kStaging + 1024 /*alignment*/ + 256 /*barriers*/;
  static_assert(kBytes <= 227 * 1024, "shared memory budget");
};

// Epilogue of one output element x = alpha * acc at (row, col).
__device__ inline void epilogue_store(const Epilogue& ep, int64_t row, int col, float x) {
  x *= ep.alpha;
  if (ep.bias) x += ep.bias[col];
  if (ep.act == CG_ACT_SILU) {
    if (ep.aux_out) ep.aux_out[row * ep.ld_aux + col] = x;
    x = silu(x);
  } else if (ep.act == CG_ACT_SILU_GRAD) {
    if (ep.aux_out) ep.aux_out[row * ep.ld_aux + col] = x;
    x *= silu_grad(ep.aux_in[row * ep.ld_aux + col]);
  } else if (ep.act == CG_ACT_ADD) {
    x += ep.aux_in[row * ep.ld_aux + col];
  }
  float* c = ep.c + row * ep.ldc + col;
  if (ep.accumulate) x += *c;
  *c = x;
}

// Whether the epilogue reads aux_in (the SiLU pre-activation or the residual).
__device__ inline bool reads_aux(const Epilogue& ep) { return ep.act == CG_ACT_SILU_GRAD || ep.act == CG_ACT_ADD; }

__device__ inline float4 load_aux4(const Epilogue& ep, int64_t row, int col) {
  return *reinterpret_cast<const float4*>(ep.aux_in + row * ep.ld_aux + col);
}

// Epilogue of four consecutive columns (col % 4 == 0, all in range); aux =
// aux_in[row, col .. col + 3] when reads_aux(ep), loaded ahead by the caller.
__device__ inline void epilogue_store4(const Epilogue& ep, int64_t row, int col, float4 x, float4 bias, float4 aux) {
  float v[4] = {x.x * ep.alpha + bias.x, x.y * ep.alpha + bias.y, x.z * ep.alpha + bias.z, x.w * ep.alpha + bias.w};
  if (ep.act == CG_ACT_SILU) {
    if (ep.aux_out) *reinterpret_cast<float4*>(ep.aux_out + row * ep.ld_aux + col) = make_float4(v[0], v[1], v[2], v[3]);
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = silu(v[e]);
  } else if (ep.act == CG_ACT_SILU_GRAD) {
    if (ep.aux_out) *reinterpret_cast<float4*>(ep.aux_out + row * ep.ld_aux + col) = make_float4(v[0], v[1], v[2], v[3]);
    v[0] *= silu_grad(aux.x);
    v[1] *= silu_grad(aux.y);
    v[2] *= silu_grad(aux.z);
    v[3] *= silu_grad(aux.w);
  } else if (ep.act == CG_ACT_ADD) {
    v[0] += aux.x;
    v[1] += aux.y;
    v[2] += aux.z;
    v[3] += aux.w;
  }
  float4* c = reinterpret_cast<float4*>(ep.c + row * ep.ldc + col);
  if (ep.accumulate) {
    const float4 old = *c;
    v[0] += old.x;
    v[1] += old.y;
    v[2] += old.z;
    v[3] += old.w;
  }
  *c = make_float4(v[0], v[1], v[2], v[3]);
}

// Persistent kernel: CTA b processes work items b, b + gridDim.x, ... where an
// item is (m-tile, n-tile, k-split z). Split z accumulates k-tiles
// [z * kt_per, (z+1) * kt_per) and, when `partial` is set, stores its raw fp32
// tile to partial[z] (M x N); the reduction pass adds the splits in z order.
// Two TMEM accumulators (2 * BN columns) let the epilogue of item j overlap
// the UMMAs of item j + 1.
template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI, bool SPLIT>
__global__ void __launch_bounds__(threads_of(EPI, SPLIT), 1)
    gemm_tf32_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                     int M, int N, int K, int kt_per, int splits, float* partial, Epilogue ep) {
  static_assert(EPI == 4 || EPI == 8, "four or eight epilogue warps");
  using S = Smem<BN, STAGES, EPI, SPLIT>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // tiles need 1024-byte alignment for the 128B swizzle pattern
  unsigned char* tiles = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* staging = reinterpret_cast<float*>(tiles + S::kTiles);
  uint64_t* full = reinterpret_cast<uint64_t*>(tiles + S::kTiles + S::kStaging);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* split_done = acc_empty + 2;  // SPLIT: stage s converted (one arrival per converter warp)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(split_done + (SPLIT ? STAGES : 0));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (M + BM - 1) / BM, n_tiles = (N + BN - 1) / BN;
  const int ktiles_all = (K + BK - 1) / BK;
  const int items = m_tiles * n_tiles * splits;
  // tcgen05.alloc takes a power of two of at least 32 columns
  constexpr uint32_t kTmemCols = 2 * BN <= 32 ? 32 : 2 * BN <= 64 ? 64 : 2 * BN <= 128 ? 128 : 2 * BN <= 256 ? 256 : 512;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      if (SPLIT) mbar_init(&split_done[s], CONV);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], EPI);  // one arrival per epilogue warp
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto item_coords = [&](int w, int& m0, int& n0, int& kt0, int& kt1) {
    const int mn = m_tiles * n_tiles;
    const int z = w / mn, t = w % mn;
    m0 = (t % m_tiles) * BM;
    n0 = (t / m_tiles) * BN;
    kt0 = z * kt_per;
    kt1 = kt0 + kt_per < ktiles_all ? kt0 + kt_per : ktiles_all;
  };

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    prefetch_tmap(&map_a);
    prefetch_tmap(&map_b);
    bool ok = true;
    uint32_t it = 0;
    for (int w = blockIdx.x; w < items && ok; w += gridDim.x) {
      int m0, n0, kt0, kt1;
      item_coords(w, m0, n0, kt0, kt1);
      for (int kt = kt0; kt < kt1; ++kt, ++it) {
        const int s = it % STAGES;
        const uint32_t round = it / STAGES;
        if (it >= STAGES && !(ok = mbar_wait(&empty[s], (round - 1) & 1, &g_gemm_error))) break;
        unsigned char* sa = tiles + s * S::kStage;
        unsigned char* sb = sa + S::kA;
        mbar_arrive_expect_tx(&full[s], S::kLoad);
        const int k0 = kt * BK;
        if (!A_MN) {
          tma_load_2d(sa, &map_a, &full[s], k0, m0);
        } else {
#pragma unroll
          for (int c = 0; c < BM / 32; ++c) tma_load_2d(sa + c * (BK * 128), &map_a, &full[s], m0 + 32 * c, k0);
        }
        if (!B_MN) {
          tma_load_2d(sb, &map_b, &full[s], k0, n0);
        } else {
#pragma unroll
          for (int c = 0; c < BN / 32; ++c) tma_load_2d(sb + c * (BK * 128), &map_b, &full[s], n0 + 32 * c, k0);
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- UMMA issuer ----------------
    constexpr uint32_t idesc = idesc_tf32(BM, BN, A_MN, B_MN);
    bool ok = true;
    uint32_t it = 0;
    int j = 0;
    for (int w = blockIdx.x; w < items && ok; w += gridDim.x, ++j) {
      int m0, n0, kt0, kt1;
      item_coords(w, m0, n0, kt0, kt1);
      const int b = j & 1, use = j >> 1;
      if (use > 0 && !(ok = mbar_wait(&acc_empty[b], (use - 1) & 1, &g_gemm_error))) break;
      tc_fence_after();
      const uint32_t acc = tmem + b * BN;
      for (int kt = kt0; kt < kt1; ++kt, ++it) {
        const int s = it % STAGES;
        if (!(ok = mbar_wait(SPLIT ? &split_done[s] : &full[s], (it / STAGES) & 1, &g_gemm_error))) break;
        tc_fence_after();
        const uint32_t sa = smem_u32(tiles + s * S::kStage);
        const uint32_t sb = sa + S::kA;
        // K-major (128B swizzle, 8-row groups at 1024 B): advance 32 bytes
        // along the row. MN-major (128B swizzle with 32 B granules, 4-row K
        // groups at 512 B, 32-wide MN groups at BK * 128 B): advance 8 rows.
        auto desc_a = [](uint32_t base, int kk) {
          return A_MN ? smem_desc(base + kk * 1024, BK * 128, 512, kSwizzle128BBase32B)
                      : smem_desc(base + kk * 32, 16, 1024, kSwizzle128B);
        };
        auto desc_b = [](uint32_t base, int kk) {
          return B_MN ? smem_desc(base + kk * 1024, BK * 128, 512, kSwizzle128BBase32B)
                      : smem_desc(base + kk * 32, 16, 1024, kSwizzle128B);
        };
#pragma unroll
        for (int kk = 0; kk < BK / 8; ++kk) {
          const bool acc_on = kt > kt0 || kk > 0;
          if (SPLIT) {
            // the small cross terms first, then the hi product
            umma_tf32(acc, desc_a(sa + S::kLoad, kk), desc_b(sb, kk), idesc, acc_on);
            umma_tf32(acc, desc_a(sa, kk), desc_b(sb + S::kLoad, kk), idesc, true);
            umma_tf32(acc, desc_a(sa, kk), desc_b(sb, kk), idesc, true);
          } else {
            umma_tf32(acc, desc_a(sa, kk), desc_b(sb, kk), idesc, acc_on);
          }
        }
        umma_commit(&empty[s]);
      }
      umma_commit(&acc_full[b]);
    }
  } else if (SPLIT && warp >= 2 + EPI) {
    // ---------------- three-term split converter ----------------
    // Stage s holds A then B as TMA wrote them (kLoad bytes, swizzled); the
    // same bytes at +kLoad receive the lo parts. The transform is elementwise,
    // so the swizzle carries over unchanged.
    const int ct = threadIdx.x - 32 * (2 + EPI);
    bool ok = true;
    uint32_t it = 0;
    for (int w = blockIdx.x; w < items && ok; w += gridDim.x) {
      int m0, n0, kt0, kt1;
      item_coords(w, m0, n0, kt0, kt1);
      for (int kt = kt0; kt < kt1; ++kt, ++it) {
        const int s = it % STAGES;
        if (!(ok = mbar_wait(&full[s], (it / STAGES) & 1, &g_gemm_error))) break;
        float4* hi = reinterpret_cast<float4*>(tiles + s * S::kStage);
        float4* lo = reinterpret_cast<float4*>(tiles + s * S::kStage + S::kLoad);
#pragma unroll 4
        for (int i = ct; i < S::kLoad / 16; i += 32 * CONV) {
          const float4 x = hi[i];
          float4 h, l;
          split_tf32(x.x, h.x, l.x);
          split_tf32(x.y, h.y, l.y);
          split_tf32(x.z, h.z, l.z);
          split_tf32(x.w, h.w, l.w);
          hi[i] = h;
          lo[i] = l;
        }
        // make this thread's generic-proxy writes visible to the tensor core
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) mbar_arrive(&split_done[s]);
      }
    }
  } else if (warp >= 2) {
    // ---------------- epilogue ----------------
    // Each warp owns 32 accumulator rows (its TMEM lane quarter). Per 32-column
    // chunk: tcgen05.ld (thread = row), transpose through shared memory, then
    // store row by row with the lanes along the columns: every store is one
    // coalesced 128-byte line.
    // with eight warps the two warps of a quarter take alternate 32-column chunks
    const int quarter = warp & 3, e = warp - 2, first = 32 * (e >> 2), chunk_step = 32 * (EPI / 4);
    float* stage = staging + e * 32 * kStagePitch;
    const int64_t mn = (int64_t)M * N;
    int j = 0;
    for (int w = blockIdx.x; w < items; w += gridDim.x, ++j) {
      int m0, n0, kt0, kt1;
      item_coords(w, m0, n0, kt0, kt1);
      const int z = w / (m_tiles * n_tiles);
      const int b = j & 1, use = j >> 1;
      // aux_in rows of a 32-column chunk (SiLU gradient, residual), loaded two
      // chunks ahead so that their latency hides behind the accumulator wait
      // and the previous chunks' stores (the four epilogue warps alone must
      // keep enough loads in flight); lane (l & 7) holds columns
      // 4 (l & 7) .. +3 of rows (l >> 3) + 4 i
      const int cl = (lane & 7) * 4;
      const bool prefetch = ep.vec && partial == nullptr && reads_aux(ep);
      auto fetch_aux = [&](float4 (&dst)[8], int c0) {
        const int col = n0 + c0 + cl;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int row = m0 + quarter * 32 + (lane >> 3) + 4 * i;
          dst[i] = (prefetch && c0 < BN && c0 + cl < BN && col < N && row < M) ? load_aux4(ep, row, col)
                                                                                : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      };
      float4 aux[8], aux1[8];
      if (prefetch) {
        fetch_aux(aux, first);
        fetch_aux(aux1, first + chunk_step);
      }
      if (!mbar_wait(&acc_full[b], use & 1, &g_gemm_error)) break;
      tc_fence_after();
#pragma unroll 1
      for (int c0 = first; c0 < BN; c0 += chunk_step) {
        float v[32];
        tmem_load_32(tmem + b * BN + ((uint32_t)(quarter * 32) << 16) + c0, v);
        // row `lane` of the warp's 32 x 32 block, as 8 16-byte stores
#pragma unroll
        for (int q = 0; q < 8; ++q)
          *reinterpret_cast<float4*>(stage + stage_idx(lane, 4 * q)) =
              make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        __syncwarp();
        float4 aux2[8];
        if (prefetch) fetch_aux(aux2, c0 + 2 * chunk_step);
        // each store instruction writes 4 full rows of 32 columns (8 lanes x 16 B per row)
        const int col = n0 + c0 + cl;
        if (ep.vec && c0 + cl < BN && col < N) {
          const float4 bias = ep.bias ? *reinterpret_cast<const float4*>(ep.bias + col) : make_float4(0, 0, 0, 0);
          if (prefetch) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int r = (lane >> 3) + 4 * i;
              const int row = m0 + quarter * 32 + r;
              if (row >= M) break;
              const float4 x = *reinterpret_cast<const float4*>(stage + stage_idx(r, cl));
              epilogue_store4(ep, row, col, x, bias, aux[i]);
            }
          } else {
            const float4 none = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 2
            for (int r = lane >> 3; r < 32; r += 4) {
              const int row = m0 + quarter * 32 + r;
              if (row >= M) break;
              const float4 x = *reinterpret_cast<const float4*>(stage + stage_idx(r, cl));
              if (partial) {
                *reinterpret_cast<float4*>(partial + z * mn + (int64_t)row * N + col) = x;
              } else {
                epilogue_store4(ep, row, col, x, bias, none);
              }
            }
          }
        } else if (!ep.vec) {
          // unaligned or ragged outputs: one column per lane, one row per step
          const int colc = n0 + c0 + lane;
          const bool ok_c = c0 + lane < BN && colc < N;
          for (int r = 0; r < 32; ++r) {
            const int row = m0 + quarter * 32 + r;
            if (!ok_c || row >= M) continue;
            const float x = stage[stage_idx(r, lane)];
            if (partial) {
              partial[z * mn + (int64_t)row * N + colc] = x;
            } else {
              epilogue_store(ep, row, colc, x);
            }
          }
        }
        __syncwarp();
        if (prefetch) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            aux[i] = aux1[i];
            aux1[i] = aux2[i];
          }
        }
      }
      // the accumulator may be overwritten once every epilogue warp has read it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// C = epi(alpha * sum_z partial[z]) in z order; one thread per element.
__global__ void splitk_reduce_kernel(const float* __restrict__ partial, int splits, int M, int N, Epilogue ep) {
  const int64_t mn = (int64_t)M * N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < mn; i += (int64_t)gridDim.x * blockDim.x) {
    float x = 0.0f;
    for (int z = 0; z < splits; ++z) x += partial[z * mn + i];
    epilogue_store(ep, i / N, (int)(i % N), x);
  }
}

// The same on 16-byte column groups (ep.vec): blocks walk rows, threads the
// row's groups, splits added in z order.
__global__ void splitk_reduce4_kernel(const float* __restrict__ partial, int splits, int M, int N, Epilogue ep) {
  const int64_t mn = (int64_t)M * N;
  const int n4 = N / 4;
  for (int64_t r = blockIdx.x; r < M; r += gridDim.x)
    for (int c4 = threadIdx.x; c4 < n4; c4 += blockDim.x) {
      float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      for (int z = 0; z < splits; ++z) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(partial + z * mn + r * N) + c4);
        x.x += v.x; x.y += v.y; x.z += v.z; x.w += v.w;
      }
      const float4 bias =
          ep.bias ? __ldg(reinterpret_cast<const float4*>(ep.bias) + c4) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      const float4 aux = reads_aux(ep) ? load_aux4(ep, r, 4 * c4) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      epilogue_store4(ep, r, 4 * c4, x, bias, aux);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2D fp32 tensor map over `rows` x `cols` (cols contiguous, row pitch `ld`),
// box = box_cols x box_rows, 128-byte swizzle with 16-byte granules
// (K-major tiles) or 32-byte granules (MN-major tiles).
static int make_map(CUtensorMap* map, const float* ptr, int64_t rows, int64_t cols, int64_t ld,
                    int box_cols, int box_rows, bool mn_major) {
  auto fn = encode_fn();
  CG_REQUIRE(fn != nullptr, "gemm: cuTensorMapEncodeTiled is unavailable");
  // the driver call needs a current context; threads such as autograd's
  // backward workers may not have bound the runtime's primary context yet
  int dev = 0;
  CG_CUDA(cudaGetDevice(&dev));
  CG_CUDA(cudaSetDevice(dev));
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 4)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  CG_REQUIRE(r == CUDA_SUCCESS, "gemm: cuTensorMapEncodeTiled failed (%d): rows %lld cols %lld ld %lld",
             (int)r, (long long)rows, (long long)cols, (long long)ld);
  return kOk;
}

struct Plan {
  int bn;
  int splits;
  int kt_per;
  bool split3;  // CG_GEMM_FP32: three-term tf32 split
};

// Tile width and split-K factor of a problem. Wide (128 x 256) tiles halve
// the operand bytes per flop against 128 x 128 ones, which L2 cannot feed at
// the tensor-core rate: they are used whenever N allows and either fill the
// SMs by themselves or K is long enough to split. Short-output, long-K
// problems split K into as many parts as fit one wave (floor(SMs / tiles)),
// each of at least 4 k-tiles.
static Plan plan_of(const cg_gemm_args& g) {
  Plan p;
  const int64_t mt = ceil_div<int64_t>(g.m, BM);
  const int64_t ktiles = ceil_div<int64_t>(g.k, BK);
  const int64_t sms = sm_count();
  if (g.n <= 16 && !g.b_mn_major) p.bn = 16;
  else if (g.n <= 32) p.bn = 32;
  else if (g.n <= 64) p.bn = 64;
  else if (g.n >= 256 && mt * ceil_div<int64_t>(g.n, 256) < sms && ktiles >= 32) {
    // K is split below: the width whose split fills the SMs for the least
    // time per wave (waves x width x k-tiles per split, 192 weighted for its
    // lower flops per operand byte)
    const int widths[2] = {256, 192};
    const double weight[2] = {1.0, 1.05};
    double best = 0.0;
    for (int i = 0; i < 2; ++i) {
      const int64_t tiles = mt * ceil_div<int64_t>(g.n, widths[i]);
      int64_t splits = tiles < sms ? sms / tiles : 1;
      if (splits > ktiles / 4) splits = ktiles / 4;
      if (splits < 1) splits = 1;
      const int64_t waves = ceil_div<int64_t>(tiles * splits, sms);
      const double cost = (double)waves * widths[i] * (double)ceil_div<int64_t>(ktiles, splits) * weight[i];
      if (best == 0.0 || cost < best) {
        best = cost;
        p.bn = widths[i];
      }
    }
  }
  else if (g.n >= 192) {
    // the width whose waves of tiles take the least time: waves x width,
    // narrower tiles weighted for their lower flops per operand byte
    const int widths[3] = {256, 192, 128};
    const double weight[3] = {1.0, 1.05, 1.15};
    double best = 0.0;
    for (int i = 0; i < 3; ++i) {
      if (g.n < widths[i]) continue;
      const int64_t waves = ceil_div<int64_t>(mt * ceil_div<int64_t>(g.n, widths[i]), sms);
      const double cost = (double)waves * widths[i] * weight[i];
      if (best == 0.0 || cost < best) {
        best = cost;
        p.bn = widths[i];
      }
    }
  } else p.bn = 128;
  // the split mode keeps a lo copy of every stage: tiles up to 128 wide
  p.split3 = g.precision == CG_GEMM_FP32;
  if (p.split3 && p.bn > 128) p.bn = 128;
  const int64_t tiles = mt * ceil_div<int64_t>(g.n, p.bn);
  int64_t splits = 1;
  if (tiles < sms && ktiles >= 8) {
    splits = sms / tiles;
    const int64_t cap = ktiles / 4;
    if (splits > cap) splits = cap;
    if (splits < 1) splits = 1;
  }
  p.kt_per = (int)ceil_div<int64_t>(ktiles, splits);
  p.splits = (int)ceil_div<int64_t>(ktiles, p.kt_per);
  return p;
}

static int64_t workspace_bytes(const cg_gemm_args& g) {
  const Plan p = plan_of(g);
  return p.splits > 1 ? (int64_t)p.splits * g.m * g.n * (int64_t)sizeof(float) : 0;
}

template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI = 4, bool SPLIT = false>
static int launch(const cg_gemm_args& g, const Plan& p, cudaStream_t stream) {
  CUtensorMap ma, mb;
  int rc;
  // A as stored: K-major (M rows x K cols) or MN-major (K rows x M cols)
  if ((rc = A_MN ? make_map(&ma, g.a, g.k, g.m, g.lda, 32, BK, true)
                 : make_map(&ma, g.a, g.m, g.k, g.lda, BK, BM, false)))
    return rc;
  if ((rc = B_MN ? make_map(&mb, g.b, g.k, g.n, g.ldb, 32, BK, true)
                 : make_map(&mb, g.b, g.n, g.k, g.ldb, BK, BN, false)))
    return rc;
  Epilogue ep;
  ep.c = g.c;
  ep.ldc = g.ldc;
  ep.bias = g.bias;
  ep.aux_in = g.aux_in;
  ep.aux_out = g.aux_out;
  ep.ld_aux = g.ld_aux;
  ep.act = g.act;
  ep.accumulate = g.accumulate;
  ep.alpha = g.alpha;
  {
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    const bool aux = g.aux_in != nullptr || g.aux_out != nullptr;
    ep.vec = g.n % 4 == 0 && g.ldc % 4 == 0 && al(g.c) && (g.bias == nullptr || al(g.bias)) &&
             (!aux || (g.ld_aux % 4 == 0 && al(g.aux_in) && al(g.aux_out)));
  }
  float* partial = nullptr;
  if (p.splits > 1) {
    CG_REQUIRE(g.workspace != nullptr && g.workspace_bytes >= workspace_bytes(g),
               "gemm: this shape splits K %d ways and needs %lld workspace bytes (cg_gemm_workspace_bytes)",
               p.splits, (long long)workspace_bytes(g));
    partial = g.workspace;
  }
  using S = Smem<BN, STAGES, EPI, SPLIT>;
  auto kernel = gemm_tf32_kernel<BN, STAGES, A_MN, B_MN, EPI, SPLIT>;
  CG_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBytes));
  const int64_t items = ceil_div<int64_t>(g.m, BM) * ceil_div<int64_t>(g.n, BN) * p.splits;
  CG_REQUIRE(items < (1ll << 31), "gemm: too many tiles");
  const int grid = (int)(items < sm_count() ? items : sm_count());
  kernel<<<grid, threads_of(EPI, SPLIT), S::kBytes, stream>>>(ma, mb, (int)g.m, (int)g.n, (int)g.k, p.kt_per,
                                                             p.splits, partial, ep);
  CG_LAUNCHED("gemm_tf32");
  if (p.splits > 1) {
    if (ep.vec) {
      const int64_t blocks = g.m < (int64_t)sm_count() * 16 ? g.m : (int64_t)sm_count() * 16;
      splitk_reduce4_kernel<<<(unsigned)blocks, 128, 0, stream>>>(partial, p.splits, (int)g.m, (int)g.n, ep);
    } else {
      const int64_t mn = g.m * g.n;
      const int64_t blocks = ceil_div<int64_t>(mn, 256);
      splitk_reduce_kernel<<<(unsigned)(blocks < 8192 ? blocks : 8192), 256, 0, stream>>>(partial, p.splits,
                                                                                          (int)g.m, (int)g.n, ep);
    }
    CG_LAUNCHED("gemm_tf32 split-K reduction");
  }
  return kOk;
}

template <int BN, int STAGES, int EPI = 4, bool SPLIT = false>
static int launch_majors(const cg_gemm_args& g, const Plan& p, cudaStream_t s) {
  if (!g.a_mn_major && !g.b_mn_major) return launch<BN, STAGES, false, false, EPI, SPLIT>(g, p, s);
  if (!g.a_mn_major && g.b_mn_major) return launch<BN, STAGES, false, true, EPI, SPLIT>(g, p, s);
  if (g.a_mn_major && !g.b_mn_major) return launch<BN, STAGES, true, false, EPI, SPLIT>(g, p, s);
  return launch<BN, STAGES, true, true, EPI, SPLIT>(g, p, s);
}

// Three-term split GEMMs (CG_GEMM_FP32): each stage is twice as large, so
// fewer stages fit.
static int run_split3(const cg_gemm_args& g, const Plan& p, cudaStream_t s) {
  switch (p.bn) {
    case 16:
      return g.a_mn_major ? launch<16, 5, true, false, 4, true>(g, p, s) : launch<16, 5, false, false, 4, true>(g, p, s);
    case 32: return launch_majors<32, 5, 4, true>(g, p, s);
    case 64: return launch_majors<64, 4, 4, true>(g, p, s);
    default: return launch_majors<128, 3, 4, true>(g, p, s);
  }
}

// Unsplit wide-tile GEMMs with a short main loop (K <= 1024) and K-major A
// run on eight epilogue warps: their epilogue, the output plus any residual
// or SiLU stream, bounds a tile, and four warps keep too few stores and loads
// in flight. (The 192-wide tile gives up a stage for the extra staging
// blocks; with long K the deeper pipeline wins.)
static bool heavy_epilogue(const cg_gemm_args& g, const Plan& p) {
  return p.splits == 1 && !g.a_mn_major && (p.bn == 256 || p.bn == 192) && g.k <= 1024;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static int run(const cg_gemm_args* args, void* stream) {
  CG_REQUIRE(args != nullptr, "gemm: args is NULL");
  const cg_gemm_args& g = *args;
  CG_REQUIRE(g.m >= 0 && g.n >= 0 && g.k >= 0, "gemm: negative size");
  if (g.m == 0 || g.n == 0) return kOk;
  CG_REQUIRE(g.k >= 1, "gemm: k must be >= 1 (use a fill for k = 0)");
  CG_REQUIRE(g.m < (1ll << 31) && g.n < (1ll << 31) && g.k < (1ll << 31), "gemm: size too large");
  CG_REQUIRE(g.a && g.b && g.c, "gemm: a, b and c must be non-null");
  CG_REQUIRE(aligned16(g.a) && aligned16(g.b), "gemm: a and b must be 16-byte aligned");
  CG_REQUIRE(g.lda % 4 == 0 && g.ldb % 4 == 0, "gemm: lda and ldb must be multiples of 4 floats");
  CG_REQUIRE(g.lda >= (g.a_mn_major ? g.m : g.k) && g.ldb >= (g.b_mn_major ? g.n : g.k),
             "gemm: leading dimension smaller than the contiguous extent");
  CG_REQUIRE(g.act == CG_ACT_NONE || g.act == CG_ACT_SILU || g.act == CG_ACT_SILU_GRAD || g.act == CG_ACT_ADD,
             "gemm: bad act");
  CG_REQUIRE((g.act != CG_ACT_SILU_GRAD && g.act != CG_ACT_ADD) || g.aux_in != nullptr,
             "gemm: the SiLU gradient and the residual add need aux_in");
  CG_REQUIRE(g.precision == CG_GEMM_TF32 || g.precision == CG_GEMM_FP32, "gemm: bad precision %d", g.precision);
  cudaStream_t s = as_stream(stream);
  const Plan p = plan_of(g);
  if (p.split3) return run_split3(g, p, s);
  switch (p.bn) {
    case 16: return g.a_mn_major ? launch<16, 10, true, false>(g, p, s) : launch<16, 10, false, false>(g, p, s);
    case 32: return launch_majors<32, 9>(g, p, s);
    case 64: return launch_majors<64, 8>(g, p, s);
    case 128: return launch_majors<128, 6>(g, p, s);
    case 192:
      if (heavy_epilogue(g, p))
        return g.b_mn_major ? launch<192, 4, false, true, 8>(g, p, s) : launch<192, 4, false, false, 8>(g, p, s);
      return launch_majors<192, 5>(g, p, s);
    default:
      if (heavy_epilogue(g, p))
        return g.b_mn_major ? launch<256, 4, false, true, 8>(g, p, s) : launch<256, 4, false, false, 8>(g, p, s);
      return launch_majors<256, 4>(g, p, s);
  }
}

// ---------------------------------------------------------------------------
// The allocation-free variant (cg_gemm_tf32_noalloc). Its split-K partial
// tiles live in this file-scope device array instead of a caller workspace.
// Every GPU that loads the library keeps the array for the life of the
// process. Host code must not pass the symbol itself to a kernel (on the host
// it is only a stand-in); the device address comes from cudaGetSymbolAddress.
// ---------------------------------------------------------------------------
constexpr int64_t kNoAllocScratchFloats = 2 * 1024 * 1024;  // 8 MiB per device
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

// Device address of the array on the current device, looked up once per device
// (the first call on a device therefore runs a runtime query; make it before
// any stream capture). Concurrent first calls from several host threads may
// each look the address up; they find the same value, and the slots are atomic.
// A cudaDeviceReset while the library is in use leaves a stale address: the
// cache is not refreshed.
static int noalloc_scratch(float** out) {
  static std::atomic<float*> cached[64];
  int dev = -1;
  CG_CUDA(cudaGetDevice(&dev));
  CG_REQUIRE(dev >= 0 && dev < 64, "gemm_noalloc: device index %d out of range", dev);
  float* p = cached[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    void* found = nullptr;
    CG_CUDA(cudaGetSymbolAddress(&found, g_noalloc_scratch));
    p = static_cast<float*>(found);
    cached[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return kOk;
}

static int run_noalloc(const cg_gemm_args* args, void* stream) {
  CG_REQUIRE(args != nullptr, "gemm_noalloc: args is NULL");
  cg_gemm_args local = *args;
  local.workspace = nullptr;
  local.workspace_bytes = 0;
  if (local.m > 0 && local.n > 0 && local.k > 0) {
    const int64_t need = workspace_bytes(local);
    const int64_t have = kNoAllocScratchFloats * (int64_t)sizeof(float);
    CG_REQUIRE(need <= have,
               "gemm_noalloc: this shape splits K and needs %lld bytes of scratch, more than the %lld-byte "
               "static buffer; call cg_gemm_tf32 with a workspace instead",
               (long long)need, (long long)have);
    if (need > 0) {
      int rc = noalloc_scratch(&local.workspace);
      if (rc) return rc;
      local.workspace_bytes = have;
    }
  }
  return run(&local, stream);
}

}  // namespace gemm
}  // namespace cg

extern "C" {

int cg_gemm_tf32_noalloc(const cg_gemm_args* args, void* stream) { return cg::gemm::run_noalloc(args, stream); }

int cg_gemm_tf32(const cg_gemm_args* args, void* stream) { return cg::gemm::run(args, stream); }

int64_t cg_gemm_workspace_bytes(const cg_gemm_args* args) {
  if (args == nullptr || args->m <= 0 || args->n <= 0 || args->k <= 0) return 0;
  return cg::gemm::workspace_bytes(*args);
}

int cg_device_error(int* out, int reset) {
  int v = 0;
  CG_CUDA(cudaMemcpyFromSymbol(&v, cg::gemm::g_gemm_error, sizeof(int)));
  if (reset) {
    const int zero = 0;
    CG_CUDA(cudaMemcpyToSymbol(cg::gemm::g_gemm_error, &zero, sizeof(int)));
  }
  if (out) *out = v;
  return cg::kOk;
}

}  // extern "C"
