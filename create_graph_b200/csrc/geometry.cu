// Edge geometry of the neighbour layout and its first and second derivatives.
//
// Edges live in a padded (n_atoms, k) slot layout: slot e = i*k + s holds the
// neighbour nbr[e] of centre atom i (or -1). Per edge:
//   vec = pos[nbr] - pos[i],  d = |vec|,
//   rbf[e, r] = exp(-gamma (d - mu_r)^2),  mu_r = r * cutoff / (n_rbf - 1),
//   env[e]    = (cos(pi d / cutoff) + 1) / 2 for d < cutoff, else 0.
// The reference keeps this geometry as eager model code before its region
// (README.md:28, tests/test_semantics.py:46-48 there); here it is one fused
// op whose backward1 (the force pass) and backward2 (the parameter backward
// through the force) are kernels too. Atom gradients are gathered per atom
// from a reverse CSR sorted by (neighbour, slot): deterministic, no atomics.
#include <math.h>

#include "common.cuh"
#include "../../include/cg_b200.h"

namespace cg {
namespace geom {

constexpr float kPi = 3.14159265358979323846f;

struct Edge {
  bool valid;
  float vx, vy, vz, d;
};

__device__ inline Edge edge_of(const float* pos, const int32_t* nbr, int64_t e, int k) {
  Edge g;
  const int32_t j = nbr[e];
  g.valid = j >= 0;
  if (!g.valid) {
    g.vx = g.vy = g.vz = g.d = 0.0f;
    return g;
  }
  const int64_t i = e / k;
  g.vx = pos[3 * (int64_t)j] - pos[3 * i];
  g.vy = pos[3 * (int64_t)j + 1] - pos[3 * i + 1];
  g.vz = pos[3 * (int64_t)j + 2] - pos[3 * i + 2];
  g.d = sqrtf(g.vx * g.vx + g.vy * g.vy + g.vz * g.vz);
  return g;
}

struct Basis {
  float gamma, cutoff, step;  // step = cutoff / (n_rbf - 1)
  int n_rbf;
};

__device__ inline float env_f(float d, float rc) {
  return d < rc ? 0.5f * (cospif(d / rc) + 1.0f) : 0.0f;
}
__device__ inline float env_d1(float d, float rc) {
  return d < rc ? -0.5f * (kPi / rc) * sinpif(d / rc) : 0.0f;
}
__device__ inline float env_d2(float d, float rc) {
  const float w = kPi / rc;
  return d < rc ? -0.5f * w * w * cospif(d / rc) : 0.0f;
}

// One warp per edge, lanes over the radial functions.
__global__ void fwd_kernel(const float* __restrict__ pos, const int32_t* __restrict__ nbr, int64_t n_edges,
                           int k, Basis b, float* __restrict__ rbf, float* __restrict__ env) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t e = warp; e < n_edges; e += warps) {
    const Edge g = edge_of(pos, nbr, e, k);
    for (int r = lane; r < b.n_rbf; r += 32) {
      const float t = g.d - r * b.step;
      rbf[e * b.n_rbf + r] = g.valid ? expf(-b.gamma * t * t) : 0.0f;
    }
    if (lane == 0) env[e] = g.valid ? env_f(g.d, b.cutoff) : 0.0f;
  }
}

// backward1: gvec[e] = (sum_r g_rbf rbf'(d) + g_env env'(d)) * vec / d.
// backward2 (h != null): with dvec = h[nbr] - h[i], t = u . dvec (u = vec / d):
//   d_g_rbf[e, r] = rbf_r'(d) t,  d_g_env[e] = env'(d) t,
//   gvec[e] = gd'(d) t u + gd (dvec - t u) / d      (the edge part of d_pos).
__global__ void bwd_kernel(const float* __restrict__ pos, const int32_t* __restrict__ nbr, int64_t n_edges,
                           int k, Basis b, const float* __restrict__ g_rbf, const float* __restrict__ g_env,
                           const float* __restrict__ h, float* __restrict__ gvec,
                           float* __restrict__ d_g_rbf, float* __restrict__ d_g_env) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t e = warp; e < n_edges; e += warps) {
    const Edge g = edge_of(pos, nbr, e, k);
    if (!g.valid || g.d == 0.0f) {
      if (lane < 3) gvec[e * 3 + lane] = 0.0f;
      if (h) {
        for (int r = lane; r < b.n_rbf; r += 32) d_g_rbf[e * b.n_rbf + r] = 0.0f;
        if (lane == 0) d_g_env[e] = 0.0f;
      }
      continue;
    }
    const float ux = g.vx / g.d, uy = g.vy / g.d, uz = g.vz / g.d;
    float t = 0.0f, dx = 0.0f, dy = 0.0f, dz = 0.0f;
    if (h) {
      const int32_t j = nbr[e];
      const int64_t i = e / k;
      dx = h[3 * (int64_t)j] - h[3 * i];
      dy = h[3 * (int64_t)j + 1] - h[3 * i + 1];
      dz = h[3 * (int64_t)j + 2] - h[3 * i + 2];
      t = ux * dx + uy * dy + uz * dz;
    }
    float gd = 0.0f, gdd = 0.0f;
    for (int r = lane; r < b.n_rbf; r += 32) {
      const float m = g.d - r * b.step;
      const float f = expf(-b.gamma * m * m);
      const float f1 = -2.0f * b.gamma * m * f;
      const float gr = g_rbf[e * b.n_rbf + r];
      gd += gr * f1;
      if (h) {
        gdd += gr * (4.0f * b.gamma * b.gamma * m * m - 2.0f * b.gamma) * f;
        d_g_rbf[e * b.n_rbf + r] = f1 * t;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      gd += __shfl_xor_sync(0xffffffffu, gd, o);
      gdd += __shfl_xor_sync(0xffffffffu, gdd, o);
    }
    const float ge = g_env ? g_env[e] : 0.0f;
    gd += ge * env_d1(g.d, b.cutoff);
    if (!h) {
      if (lane == 0) {
        gvec[e * 3] = gd * ux;
        gvec[e * 3 + 1] = gd * uy;
        gvec[e * 3 + 2] = gd * uz;
      }
      continue;
    }
    gdd += ge * env_d2(g.d, b.cutoff);
    if (lane == 0) {
      d_g_env[e] = env_d1(g.d, b.cutoff) * t;
      const float inv = gd / g.d;
      gvec[e * 3] = gdd * t * ux + inv * (dx - t * ux);
      gvec[e * 3 + 1] = gdd * t * uy + inv * (dy - t * uy);
      gvec[e * 3 + 2] = gdd * t * uz + inv * (dz - t * uz);
    }
  }
}

// out[a] = sum over edges e with nbr[e] == a (reverse CSR, fixed order) of gvec[e]
//          - sum over a's own slots s of gvec[a*k + s]
__global__ void scatter_kernel(const float* __restrict__ gvec, const int32_t* __restrict__ rev_ptr,
                               const int32_t* __restrict__ rev_idx, int64_t n_atoms, int k,
                               float* __restrict__ out) {
  for (int64_t a = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; a < n_atoms;
       a += (int64_t)gridDim.x * blockDim.x) {
    float x = 0.0f, y = 0.0f, z = 0.0f;
    for (int32_t p = rev_ptr[a]; p < rev_ptr[a + 1]; ++p) {
      const int64_t e = rev_idx[p];
      x += gvec[3 * e];
      y += gvec[3 * e + 1];
      z += gvec[3 * e + 2];
    }
    for (int s = 0; s < k; ++s) {
      const int64_t e = a * k + s;
      x -= gvec[3 * e];
      y -= gvec[3 * e + 1];
      z -= gvec[3 * e + 2];
    }
    out[3 * a] = x;
    out[3 * a + 1] = y;
    out[3 * a + 2] = z;
  }
}

static int warp_grid(int64_t items) {
  const int64_t b = ceil_div<int64_t>(items, 8);
  const int64_t cap = (int64_t)sm_count() * 16;
  return (int)(b < 1 ? 1 : (b < cap ? b : cap));
}

static int check(const cg_geom_args* a) {
  CG_REQUIRE(a != nullptr, "edge_geom: args is NULL");
  CG_REQUIRE(a->n_atoms >= 0 && a->k >= 1 && a->n_rbf >= 2 && a->n_rbf <= 4096,
             "edge_geom: bad sizes (k >= 1, 2 <= n_rbf <= 4096)");
  CG_REQUIRE(a->cutoff > 0.0f && a->gamma > 0.0f, "edge_geom: cutoff and gamma must be positive");
  CG_REQUIRE(a->pos && a->nbr, "edge_geom: pos and nbr must be non-null");
  return kOk;
}

static Basis basis_of(const cg_geom_args* a) {
  Basis b;
  b.gamma = a->gamma;
  b.cutoff = a->cutoff;
  b.n_rbf = a->n_rbf;
  b.step = a->cutoff / (a->n_rbf - 1);
  return b;
}

}  // namespace geom
}  // namespace cg

extern "C" {

using namespace cg;

int cg_edge_geom_fwd(const cg_geom_args* a, float* rbf, float* env, void* stream) {
  int rc = geom::check(a);
  if (rc) return rc;
  const int64_t e = a->n_atoms * a->k;
  if (e == 0) return kOk;
  CG_REQUIRE(rbf && env, "edge_geom_fwd: outputs must be non-null");
  geom::fwd_kernel<<<geom::warp_grid(e), 256, 0, as_stream(stream)>>>(a->pos, a->nbr, e, a->k,
                                                                      geom::basis_of(a), rbf, env);
  CG_LAUNCHED("edge_geom_fwd");
  return kOk;
}

int cg_edge_geom_bwd1(const cg_geom_args* a, const float* g_rbf, const float* g_env, float* gvec,
                      float* g_pos, void* stream) {
  int rc = geom::check(a);
  if (rc) return rc;
  const int64_t e = a->n_atoms * a->k;
  if (a->n_atoms == 0) return kOk;
  CG_REQUIRE(g_rbf && gvec && g_pos && a->rev_ptr && a->rev_idx, "edge_geom_bwd1: null pointer");
  geom::bwd_kernel<<<geom::warp_grid(e), 256, 0, as_stream(stream)>>>(
      a->pos, a->nbr, e, a->k, geom::basis_of(a), g_rbf, g_env, nullptr, gvec, nullptr, nullptr);
  CG_LAUNCHED("edge_geom_bwd1");
  geom::scatter_kernel<<<(unsigned)ceil_div<int64_t>(a->n_atoms, 128), 128, 0, as_stream(stream)>>>(
      gvec, a->rev_ptr, a->rev_idx, a->n_atoms, a->k, g_pos);
  CG_LAUNCHED("edge_geom_scatter");
  return kOk;
}

int cg_edge_geom_bwd2(const cg_geom_args* a, const float* g_rbf, const float* g_env, const float* h_pos,
                      float* gvec, float* d_pos, float* d_g_rbf, float* d_g_env, void* stream) {
  int rc = geom::check(a);
  if (rc) return rc;
  const int64_t e = a->n_atoms * a->k;
  if (a->n_atoms == 0) return kOk;
  CG_REQUIRE(g_rbf && h_pos && gvec && d_pos && d_g_rbf && d_g_env && a->rev_ptr && a->rev_idx,
             "edge_geom_bwd2: null pointer");
  geom::bwd_kernel<<<geom::warp_grid(e), 256, 0, as_stream(stream)>>>(
      a->pos, a->nbr, e, a->k, geom::basis_of(a), g_rbf, g_env, h_pos, gvec, d_g_rbf, d_g_env);
  CG_LAUNCHED("edge_geom_bwd2");
  geom::scatter_kernel<<<(unsigned)ceil_div<int64_t>(a->n_atoms, 128), 128, 0, as_stream(stream)>>>(
      gvec, a->rev_ptr, a->rev_idx, a->n_atoms, a->k, d_pos);
  CG_LAUNCHED("edge_geom_scatter");
  return kOk;
}

}  // extern "C"
