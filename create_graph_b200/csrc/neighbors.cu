// Neighbour lists of a batch of non-periodic systems, bit-exact.
//
// Atoms are sorted by system (sys_ptr). For atom i the candidates are the
// other atoms j of its system with d2 < cutoff^2, where
//   d2 = (dx*dx + dy*dy) + dz*dz,  dx = pos[j].x - pos[i].x, ...
// is evaluated with round-to-nearest single operations (no FMA contraction),
// so a CPU evaluating the same expression gets the same bits. The k nearest
// by (d2, j) are kept in that order. The reverse CSR (slots grouped by
// neighbour, slots ascending) is filled in a fixed order. Nothing is atomic:
// the output is identical on every run.
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

__device__ inline bool before(float da, int ja, float db, int jb) {
  return da < db || (da == db && ja < jb);
}

// One block per system: the k nearest neighbours of every atom, and the
// number of kept slots of the system.
__global__ void select_kernel(const float* __restrict__ pos, const int32_t* __restrict__ sys_ptr, int k,
                              float cutoff2, int32_t* __restrict__ nbr, int32_t* __restrict__ counts,
                              int32_t* __restrict__ sys_edges) {
  const int b = blockIdx.x;
  const int a0 = sys_ptr[b], a1 = sys_ptr[b + 1];
  __shared__ int total;
  if (threadIdx.x == 0) total = 0;
  __syncthreads();
  int mine = 0;
  for (int i = a0 + threadIdx.x; i < a1; i += blockDim.x) {
    float bd[KMAX];
    int bj[KMAX];
    int n = 0;
    const float xi = pos[3 * i], yi = pos[3 * i + 1], zi = pos[3 * i + 2];
    for (int j = a0; j < a1; ++j) {
      if (j == i) continue;
      const float d = d2_exact(xi, yi, zi, pos[3 * j], pos[3 * j + 1], pos[3 * j + 2]);
      if (!(d < cutoff2)) continue;
      if (n == k && !before(d, j, bd[k - 1], bj[k - 1])) continue;
      int p = n < k ? n : k - 1;  // insertion position from the end
      while (p > 0 && before(d, j, bd[p - 1], bj[p - 1])) {
        bd[p] = bd[p - 1];
        bj[p] = bj[p - 1];
        --p;
      }
      bd[p] = d;
      bj[p] = j;
      if (n < k) ++n;
    }
    for (int s = 0; s < k; ++s) nbr[(int64_t)i * k + s] = s < n ? bj[s] : -1;
    counts[i] = n;
    mine += n;
  }
  atomicAdd(&total, mine);  // integer count: order does not matter
  __syncthreads();
  if (threadIdx.x == 0) sys_edges[b] = total;
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

// One block per system: reverse CSR of its slots. Thread t owns targets
// j = a0 + t, a0 + t + blockDim, ...; each walks the system's slots in
// ascending order, so every segment is sorted.
__global__ void reverse_kernel(const int32_t* __restrict__ sys_ptr, const int32_t* __restrict__ sys_offset,
                               const int32_t* __restrict__ nbr, const int32_t* __restrict__ counts, int k,
                               int n_atoms, int32_t* __restrict__ rev_ptr, int32_t* __restrict__ rev_idx) {
  const int b = blockIdx.x;
  const int a0 = sys_ptr[b], a1 = sys_ptr[b + 1];
  extern __shared__ int32_t scan[];  // per-target counts, then offsets
  const int n = a1 - a0;
  for (int t = threadIdx.x; t < n; t += blockDim.x) {
    const int j = a0 + t;
    int c = 0;
    for (int i = a0; i < a1; ++i)
      for (int s = 0; s < counts[i]; ++s) c += nbr[(int64_t)i * k + s] == j;
    scan[t] = c;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int32_t run = sys_offset[b];
    for (int t = 0; t < n; ++t) {
      const int32_t c = scan[t];
      scan[t] = run;
      run += c;
    }
  }
  __syncthreads();
  for (int t = threadIdx.x; t < n; t += blockDim.x) {
    const int j = a0 + t;
    int32_t w = scan[t];
    rev_ptr[j] = w;
    for (int i = a0; i < a1; ++i)
      for (int s = 0; s < counts[i]; ++s)
        if (nbr[(int64_t)i * k + s] == j) rev_idx[w++] = (int32_t)((int64_t)i * k + s);
  }
  if (b == gridDim.x - 1 && threadIdx.x == 0) rev_ptr[n_atoms] = sys_offset[gridDim.x];
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
             "neighbor_list: systems of up to 12000 atoms (shared-memory scan)");
  if (n_systems == 0) {
    if (n_atoms == 0) CG_CUDA(cudaMemsetAsync(rev_ptr, 0, sizeof(int32_t), as_stream(stream)));
    return kOk;
  }
  CG_REQUIRE(pos && sys_ptr && nbr && counts && rev_ptr && rev_idx && workspace, "neighbor_list: null pointer");
  int32_t* sys_edges = workspace;
  int32_t* sys_offset = workspace + n_systems;
  const float cutoff2 = cutoff * cutoff;
  cudaStream_t s = as_stream(stream);
  nbl::select_kernel<<<(unsigned)n_systems, 128, 0, s>>>(pos, sys_ptr, k, cutoff2, nbr, counts, sys_edges);
  CG_LAUNCHED("neighbor_list select");
  nbl::scan_systems_kernel<<<1, 32, 0, s>>>(sys_edges, (int)n_systems, sys_offset);
  CG_LAUNCHED("neighbor_list scan");
  const size_t smem = (size_t)(max_atoms_per_system > 0 ? max_atoms_per_system : 1) * sizeof(int32_t);
  nbl::reverse_kernel<<<(unsigned)n_systems, 128, smem, s>>>(sys_ptr, sys_offset, nbr, counts, k, (int)n_atoms,
                                                             rev_ptr, rev_idx);
  CG_LAUNCHED("neighbor_list reverse");
  return kOk;
}

}  // extern "C"
