// Neighbour lists of a batch of non-periodic systems, bit-exact.
//
// Atoms are sorted by system (sys_ptr). For atom i the candidates are the
// other atoms j of its system with d2 < cutoff^2, where
//   d2 = (dx*dx + dy*dy) + dz*dz,  dx = pos[j].x - pos[i].x, ...
// is evaluated with round-to-nearest single operations (no FMA contraction),
// so a CPU evaluating the same expression gets the same bits. The k nearest
// by (d2, j) are kept in that order. The reverse CSR (slots grouped by
// neighbour, slots ascending) lists every segment in ascending slot order.
// Integer atomics only count or place entries whose final order is fixed
// afterwards: the output is identical on every run.
//
// Systems of up to 256 atoms (the batches of small molecules the models
// train on) run per system in shared memory; larger ones (up to 12000
// atoms) run over the whole batch with the candidates read from L2.
//
// The reference leaves neighbour lists to model code before its region
// (README.md:28 there); this is the GPU builder of the padded layout the
// geometry, attention and segment kernels use.
#include "common.cuh"
#include "../../include/cg_b200.h"

namespace cg {
namespace nbl {

constexpr int KMAX = 64;

__device__ inline float d2_exact(float xi, float yi, float zi, float xj, float yj, float zj) {
  const float dx = __fsub_rn(xj, xi), dy = __fsub_rn(yj, yi), dz = __fsub_rn(zj, zi);
  return __fadd_rn(__fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy)), __fmul_rn(dz, dz));
}

// Ascending bitonic sort of the warp's 256 keys, element p = 8 lane + r in
// key[r]: strides below 8 inside a lane, the others across lanes by shuffles.
__device__ __forceinline__ void warp_sort256(unsigned long long (&key)[8], int lane) {
#pragma unroll
  for (int size = 2; size <= 256; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (stride >= 8) {
        const int other_lane = lane ^ (stride >> 3);
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const unsigned long long o = __shfl_xor_sync(0xffffffffu, key[r], stride >> 3);
          const bool up = ((8 * lane + r) & size) == 0;
          const bool keep_min = (lane < other_lane) == up;
          key[r] = keep_min ? (o < key[r] ? o : key[r]) : (o > key[r] ? o : key[r]);
        }
      } else {
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const int q = r ^ stride;
          if (q > r) {
            const bool up = ((8 * lane + r) & size) == 0;
            const unsigned long long lo = key[r] < key[q] ? key[r] : key[q];
            const unsigned long long hi = key[r] < key[q] ? key[q] : key[r];
            key[r] = up ? lo : hi;
            key[q] = up ? hi : lo;
          }
        }
      }
    }
  }
}

// Key of candidate j for atom i: bits of d2 << 32 | j (d2 >= 0, so the
// integer order is the (d2, j) order), or the largest key when j is not a
// candidate (j == i, or d2 not below the cutoff).
__device__ __forceinline__ unsigned long long cand_key(float xi, float yi, float zi, float xj, float yj, float zj,
                                                       int i, int j, float cutoff2) {
  if (j == i) return ~0ull;
  const float d = d2_exact(xi, yi, zi, xj, yj, zj);
  return d < cutoff2 ? ((unsigned long long)__float_as_uint(d) << 32) | (unsigned)j : ~0ull;
}

// Writes the first k sorted keys (lanes 0..7 hold positions 0..63) as atom
// i's neighbour row; returns the number kept (on every lane).
__device__ __forceinline__ int write_row(const unsigned long long (&key)[8], int lane, int64_t i, int k,
                                         int32_t* __restrict__ nbr) {
  int kept = 0;
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const int p = 8 * lane + r;
    const bool valid = key[r] != ~0ull;
    if (p < k) {
      nbr[i * k + p] = valid ? (int32_t)(key[r] & 0xffffffffull) : -1;
      kept += valid;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) kept += __shfl_xor_sync(0xffffffffu, kept, off);
  return kept;
}

// Systems of at most kSmallSystem atoms: one block per system, one warp per
// atom. The system's positions are staged in shared memory; lane l scores
// candidates l, l + 32, ... (8 per lane) and the warp sorts the 256 keys; the
// first k are the kept neighbours in (d2, j) order.
constexpr int kSmallSystem = 256;
constexpr int kSelectWarps = 4;

__global__ void __launch_bounds__(32 * kSelectWarps) select_small_kernel(
    const float* __restrict__ pos, const int32_t* __restrict__ sys_ptr, int k, float cutoff2,
    int32_t* __restrict__ nbr, int32_t* __restrict__ counts, int32_t* __restrict__ sys_edges) {
  __shared__ float sp[3 * kSmallSystem];
  __shared__ int total;
  const int b = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int a0 = sys_ptr[b], n = sys_ptr[b + 1] - a0;
  if (threadIdx.x == 0) total = 0;
  for (int e = threadIdx.x; e < 3 * n; e += 32 * kSelectWarps) sp[e] = pos[3 * (int64_t)a0 + e];
  __syncthreads();
  int mine = 0;
  for (int li = warp; li < n; li += kSelectWarps) {
    const float xi = sp[3 * li], yi = sp[3 * li + 1], zi = sp[3 * li + 2];
    unsigned long long key[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int c = lane + 32 * r;
      key[r] = c < n ? cand_key(xi, yi, zi, sp[3 * c], sp[3 * c + 1], sp[3 * c + 2], li, c, cutoff2) : ~0ull;
      if (key[r] != ~0ull) key[r] += (unsigned)a0;  // local to global atom index (no carry: c + a0 < 2^31)
    }
    warp_sort256(key, lane);
    const int kept = write_row(key, lane, a0 + li, k, nbr);
    if (lane == 0) counts[a0 + li] = kept;
    mine += lane == 0 ? kept : 0;
  }
  if (lane == 0) atomicAdd(&total, mine);  // integer count: order does not matter
  __syncthreads();
  if (threadIdx.x == 0) sys_edges[b] = total;
}

// Any system size: one warp per atom of the batch (its system found by a
// binary search of sys_ptr), candidates read from L2. The first chunk is 256
// candidates; each later chunk brings 192 more into lanes 8..31 while lanes
// 0..7 keep the 64 smallest keys so far, and the warp re-sorts. k <= 64.
__global__ void __launch_bounds__(32 * kSelectWarps) select_chunked_kernel(
    const float* __restrict__ pos, const int32_t* __restrict__ sys_ptr, int n_sys, int64_t n_atoms, int k,
    float cutoff2, int32_t* __restrict__ nbr, int32_t* __restrict__ counts) {
  const int lane = threadIdx.x & 31;
  const int64_t i = (int64_t)blockIdx.x * kSelectWarps + (threadIdx.x >> 5);
  if (i >= n_atoms) return;
  int lo = 0, hi = n_sys;  // the system b with sys_ptr[b] <= i < sys_ptr[b + 1]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (sys_ptr[mid] <= i) lo = mid;
    else hi = mid;
  }
  const int a0 = sys_ptr[lo], n = sys_ptr[lo + 1] - a0, li = (int)(i - a0);
  const float xi = pos[3 * i], yi = pos[3 * i + 1], zi = pos[3 * i + 2];
  auto key_of = [&](int c) {
    if (c >= n) return ~0ull;
    const int64_t j = a0 + c;
    const unsigned long long kk = cand_key(xi, yi, zi, pos[3 * j], pos[3 * j + 1], pos[3 * j + 2], li, c, cutoff2);
    return kk == ~0ull ? kk : kk + (unsigned)a0;
  };
  unsigned long long key[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) key[r] = key_of(lane + 32 * r);
  warp_sort256(key, lane);
  for (int base = 256; base < n; base += 192) {
    if (lane >= 8) {
#pragma unroll
      for (int r = 0; r < 8; ++r) key[r] = key_of(base + (lane - 8) + 24 * r);
    }
    warp_sort256(key, lane);
  }
  const int kept = write_row(key, lane, i, k, nbr);
  if (lane == 0) counts[i] = kept;
}

// Exclusive scan of the per-system slot totals (one thread: a few hundred systems).
__global__ void scan_systems_kernel(const int32_t* __restrict__ sys_edges, int n_sys,
                                    int32_t* __restrict__ sys_offset) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  int32_t run = 0;
  for (int b = 0; b < n_sys; ++b) {
    sys_offset[b] = run;
    run += sys_edges[b];
  }
  sys_offset[n_sys] = run;
}

// Systems of at most kSmallSystem atoms: the same reverse CSR by a stable
// counting sort in O(slots) per system (the kernel above walks all slots
// once per target). Integer shared atomics count slots per target; an
// exclusive scan gives each target's start; slots are then placed in
// chunks of the block's width in ascending order, a slot's rank among the
// chunk's slots of its target being its rank within its warp (match + popc)
// plus the counts of that target in the chunk's earlier warps. Placement
// depends only on slot order: identical output on every run, equal to the
// kernel above.
constexpr int kReverseThreads = 128;

__global__ void __launch_bounds__(kReverseThreads) reverse_small_kernel(
    const int32_t* __restrict__ sys_ptr, const int32_t* __restrict__ sys_offset, const int32_t* __restrict__ nbr,
    int k, int n_atoms, int32_t* __restrict__ rev_ptr, int32_t* __restrict__ rev_idx) {
  constexpr int W = kReverseThreads / 32;
  __shared__ int32_t start[kSmallSystem];
  __shared__ int32_t wcount[W][kSmallSystem];
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int a0 = sys_ptr[b], n = sys_ptr[b + 1] - a0;
  const int slots = n * k;
  const int32_t* src = nbr + (int64_t)a0 * k;
  for (int t = tid; t < n; t += kReverseThreads) start[t] = 0;
  __syncthreads();
  for (int e = tid; e < slots; e += kReverseThreads) {
    const int32_t j = src[e];
    if (j >= 0) atomicAdd(&start[j - a0], 1);  // integer counts: order does not matter
  }
  __syncthreads();
  if (tid == 0) {
    int32_t run = sys_offset[b];
    for (int t = 0; t < n; ++t) {
      const int32_t c = start[t];
      start[t] = run;
      run += c;
    }
  }
  __syncthreads();
  for (int t = tid; t < n; t += kReverseThreads) rev_ptr[a0 + t] = start[t];
  const uint32_t lower_lanes = (1u << lane) - 1u;
  for (int c0 = 0; c0 < slots; c0 += kReverseThreads) {
    const int e = c0 + tid;
    const int32_t j = e < slots ? src[e] : -1;
    const int t = j >= 0 ? j - a0 : -1;
    const uint32_t same = __match_any_sync(0xffffffffu, t);
    const int rank = __popc(same & lower_lanes);
    for (int i = tid; i < W * kSmallSystem; i += kReverseThreads) (&wcount[0][0])[i] = 0;
    __syncthreads();
    if (t >= 0 && rank == 0) wcount[warp][t] = __popc(same);
    __syncthreads();
    if (t >= 0) {
      int32_t before = 0;
      for (int w = 0; w < warp; ++w) before += wcount[w][t];
      rev_idx[start[t] + before + rank] = (int32_t)((int64_t)a0 * k + e);
    }
    __syncthreads();
    if (t >= 0 && rank == 0) atomicAdd(&start[t], __popc(same));  // integer: exact
    __syncthreads();
  }
  if (b == gridDim.x - 1 && tid == 0) rev_ptr[n_atoms] = sys_offset[gridDim.x];
}

}  // namespace nbl
}  // namespace cg

extern "C" {

int cg_neighbor_list_workspace(int64_t n_systems) { return (int)(2 * n_systems + 1); }

int cg_neighbor_list(const float* pos, const int32_t* sys_ptr, int64_t n_systems, int64_t n_atoms,
                     int64_t max_atoms_per_system, float cutoff, int32_t k, int32_t* nbr, int32_t* counts,
                     int32_t* rev_ptr, int32_t* rev_idx, int32_t* workspace, void* stream) {
  using namespace cg;
  CG_REQUIRE(n_systems >= 0 && n_atoms >= 0, "neighbor_list: negative size");
  CG_REQUIRE(k >= 1 && k <= nbl::KMAX, "neighbor_list: k = %d outside [1, %d]", k, nbl::KMAX);
  CG_REQUIRE(cutoff > 0.0f, "neighbor_list: cutoff must be positive");
  CG_REQUIRE(max_atoms_per_system >= 0 && max_atoms_per_system <= 12000,
             "neighbor_list: systems of up to 12000 atoms (O(n^2) distances per system)");
  CG_REQUIRE(n_atoms * (int64_t)k < (1ll << 31), "neighbor_list: n_atoms * k must stay below 2^31 slots");
  if (n_systems == 0) {
    if (n_atoms == 0) CG_CUDA(cudaMemsetAsync(rev_ptr, 0, sizeof(int32_t), as_stream(stream)));
    return kOk;
  }
  CG_REQUIRE(pos && sys_ptr && nbr && counts && rev_ptr && rev_idx && workspace, "neighbor_list: null pointer");
  int32_t* sys_edges = workspace;
  int32_t* sys_offset = workspace + n_systems;
  const float cutoff2 = cutoff * cutoff;
  cudaStream_t s = as_stream(stream);
  if (max_atoms_per_system <= nbl::kSmallSystem) {
    nbl::select_small_kernel<<<(unsigned)n_systems, 32 * nbl::kSelectWarps, 0, s>>>(pos, sys_ptr, k, cutoff2, nbr,
                                                                                   counts, sys_edges);
    CG_LAUNCHED("neighbor_list select");
    nbl::scan_systems_kernel<<<1, 32, 0, s>>>(sys_edges, (int)n_systems, sys_offset);
    CG_LAUNCHED("neighbor_list scan");
    nbl::reverse_small_kernel<<<(unsigned)n_systems, nbl::kReverseThreads, 0, s>>>(sys_ptr, sys_offset, nbr, k,
                                                                                  (int)n_atoms, rev_ptr, rev_idx);
    CG_LAUNCHED("neighbor_list reverse");
    return kOk;
  }
  const int64_t slots = n_atoms * k;
  const unsigned sel_blocks = (unsigned)((n_atoms + nbl::kSelectWarps - 1) / nbl::kSelectWarps);
  nbl::select_chunked_kernel<<<sel_blocks, 32 * nbl::kSelectWarps, 0, s>>>(pos, sys_ptr, (int)n_systems, n_atoms,
                                                                          k, cutoff2, nbr, counts);
  CG_LAUNCHED("neighbor_list select");
  // the reverse CSR over the whole batch: row j = the slots whose neighbour is j
  const int rc = seg::csr_build_launch(nbr, slots, n_atoms, rev_ptr, rev_idx, s);
  if (rc != kOk) return rc;
  CG_LAUNCHED("neighbor_list reverse");
  return kOk;
}

}  // extern "C"
