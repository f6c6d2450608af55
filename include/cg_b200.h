/*
 * cg_b200.h -- C ABI of the create_graph_b200 sm_100a library (libcg_b200.so).
 *
 * Every entry point takes plain device pointers, sizes and strides (in
 * elements, not bytes) and a cudaStream_t passed as void*; it launches on that
 * stream and returns 0, or a non-zero status whose text cg_last_error() gives.
 * Nothing here allocates device memory: callers pass every output and, where a
 * *_scratch_bytes() query says so, a scratch buffer.
 *
 * The reference (create_graph) is pure Python: its fused-op boundary is
 * `cg.custom_op` (src/create_graph/ops.py:82-212), whose forward1 / backward1 /
 * backward2 bodies for the masked edge attention are the PyTorch code of
 * kernels/edge_attn/ops.py. Each function below names the reference code it
 * replaces. The Python package calls these through ctypes
 * (create_graph_b200/native.py); other hosts bind the same symbols.
 */
#ifndef CG_B200_H
#define CG_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CG_B200_ABI_VERSION 1

/* dtype codes */
#define CG_F32 0
#define CG_F64 1

/* Text of the last error raised on the calling thread ("" if none). */
const char* cg_last_error(void);
/* CG_B200_ABI_VERSION of the loaded library. */
int cg_version(void);
/* Kernels this library has launched in this process (all threads). No
 * reference counterpart: it lets a benchmark report its own launches. */
int64_t cg_launch_count(void);

/* ------------------------------------------------------------------------
 * Masked edge attention, per slice (n, h) of k tokens with head dim d:
 *   logits = q k^T * scale + bias,  keys j >= key_count[n] masked (-inf);
 *   probs  = softmax over finite logits (all-masked rows give zeros);
 *   out    = probs v,  lse = row logsumexp (-inf for all-masked rows).
 * A matrix operand's row r of slice (n, h) starts at
 *   ptr + n*sn + h*sh + r*sr   (elements; columns contiguous).
 * bias / hb / dbias use (sn, sh, si, sj); a stride of 0 broadcasts that
 * dimension, and dbias is then summed over it (deterministically).
 * Limits: 1 <= k <= 32, 1 <= d <= 64 (d <= 16 for float64).
 * ---------------------------------------------------------------------- */
typedef struct cg_mat {
  void* ptr;
  int64_t sn, sh, sr;
} cg_mat;

typedef struct cg_bias {
  void* ptr;
  int64_t sn, sh, si, sj;
} cg_bias;

/* Precision of the float32 attention products (the float64 kernels ignore it):
 * CG_ATTN_FP32 three-term tf32 split on the tensor cores, fp32-level accuracy
 * (~1e-6 relative); CG_ATTN_TF32 one tf32 product (operands rounded to
 * nearest tf32, 2^-11 relative; fp32 accumulation), the precision of the
 * projections. Softmax and elementwise work are fp32 in both. */
#define CG_ATTN_FP32 0
#define CG_ATTN_TF32 1

typedef struct cg_edge_attn_args {
  int64_t n, h;           /* slice grid */
  int32_t k, d;           /* tokens per slice, head dim */
  int32_t dtype;          /* CG_F32 or CG_F64 */
  int32_t precision;      /* float32 products: CG_ATTN_FP32 (0) or CG_ATTN_TF32 */
  double scale;
  const int32_t* key_count; /* optional (n,): valid keys per n; NULL = all k */
  /* inputs */
  cg_mat q, k_, v;
  cg_bias bias;           /* ptr may be NULL: no bias */
  void* lse;              /* (n, h, k) contiguous: output of fwd1, input of bwd1/bwd2 */
  cg_mat grad_out;        /* bwd1, bwd2 */
  cg_mat hq, hk, hv;      /* bwd2: cotangents of dq, dk, dv */
  cg_bias hb;             /* bwd2: cotangent of dbias (bias's broadcast shape), may be NULL */
  /* outputs */
  cg_mat out;             /* fwd1 */
  cg_mat dq, dk, dv;      /* bwd1, bwd2 */
  cg_bias dbias;          /* bwd1, bwd2; strides of broadcast dims ignored; NULL = skip */
  cg_mat dgrad_out;       /* bwd2 */
  void* scratch;          /* cg_edge_attn_scratch_bytes() bytes, or NULL if that is 0 */
  /* optional (n, k) token index (float32 only): when set, row r of q, k, v,
   * hq, hk, hv for slice (n, h) is read at ptr + token_index[n*k + r]*sr + h*sh
   * (sn unused; index < 0 reads zeros): the kernels gather the edge tokens
   * from per-atom rows instead of a materialised (n*k, ...) token tensor. */
  const int32_t* token_index;
} cg_edge_attn_args;

/* Replaces EdgeAttention.forward1 (kernels/edge_attn/ops.py:64-68, with
 * _scores at :26-34): writes out and lse. */
int cg_edge_attn_fwd1(const cg_edge_attn_args* a, void* stream);

/* Replaces EdgeAttention.backward1 (kernels/edge_attn/ops.py:75-76 via _first
 * at :47-54, bias reduction _reduce at :37-44): rebuilds probs from lse,
 * writes dq, dk, dv and dbias. */
int cg_edge_attn_bwd1(const cg_edge_attn_args* a, void* stream);

/* Replaces EdgeAttention.backward2 (kernels/edge_attn/ops.py:79-104): the
 * gradients of <hq,dq>+<hk,dk>+<hv,dv>+<hb,dbias> w.r.t. q, k, v, bias and
 * grad_out; writes dq, dk, dv, dbias and dgrad_out. */
int cg_edge_attn_bwd2(const cg_edge_attn_args* a, void* stream);

/* Scratch bytes bwd1 / bwd2 need for a dbias broadcast over n or h (the
 * per-slice partial sums reduced in a fixed order); 0 otherwise. Replaces the
 * cross-batch part of _reduce (kernels/edge_attn/ops.py:37-44). */
int64_t cg_edge_attn_scratch_bytes(const cg_edge_attn_args* a);

/* ------------------------------------------------------------------------
 * Envelope-pooled token attention of the energy network: for atom n and
 * head h, over the atom's k <= 32 edge tokens (token (n, r) reads row
 * token_index[n*k + r] of qkv; < 0 reads zeros),
 *   L_ij = scale q_i.k_j + bias[n*k + j, h]   (keys j >= key_count[n] masked)
 *   P    = softmax_j(L)                        (rows without a key: zeros)
 *   w_j  = sum_i env[n, i] P_ij,   out[n, h] = sum_j w_j v_j.
 * This is the reference model's attention over neighbour tokens followed by
 * the envelope-weighted sum over tokens (the masked edge attention of
 * kernels/edge_attn/ops.py:26-34, 64-68, then a pooling), fused so that the
 * (n, k, h*d) token outputs and their cotangents never exist. No counterpart
 * entry point in the reference (its model composes the two ops).
 * Backward1 (given dout = dm): u_j = v_j.dm, ubar_i = sum_j P_ij u_j,
 *   dL_ij = env_i P_ij (u_j - ubar_i), dq_i = scale sum_j dL_ij k_j,
 *   dk_j = scale sum_i dL_ij q_i, dbias_j = sum_i dL_ij, dv_j = w_j dm,
 *   denv_i = sum_h ubar_i.
 * Backward2: the gradients of <hq,dq> + <hk,dk> + <hv,dv> + <hb,dbias> +
 * <he,denv> w.r.t. qkv, bias, env and dm (cotangents hq, hk, hv read through
 * token_index from hqkv). dv of a token is rank one, wv[n*k + j, h] * dm[n, h]:
 * the kernels write the weight wv and cg_segment_sum_scaled reduces it to
 * atoms; dq and dk leave per token in dqk for cg_segment_sum.
 * ---------------------------------------------------------------------- */
typedef struct cg_pooled_attn_args {
  int64_t n;                  /* atoms */
  int32_t h, k, d;            /* heads, tokens per atom (<= 32), head dim (<= 64) */
  int32_t precision;          /* CG_ATTN_FP32 or CG_ATTN_TF32 */
  double scale;
  const int32_t* token_index; /* (n*k,) row of qkv / hqkv of token (n, r), < 0: zero row */
  const int32_t* key_count;   /* (n,) keys j >= key_count[n] are masked */
  const float* qkv;           /* (rows, ld_qkv): [q | k | v], heads contiguous, h*d each */
  const float* hqkv;          /* bwd2: cotangent of the q/k/v gradient, same layout */
  int64_t ld_qkv;
  const float* bias;          /* (n*k, h) additive bias of key (n, j), row pitch ld_bias; NULL = none */
  const float* env;           /* (n, k) pooling weight of query token (n, i) */
  float* lse;                 /* (n, h, k): written by fwd, read by bwd1 / bwd2 */
  float* w;                   /* (n, h, k): w_j, written by fwd, read by bwd1 / bwd2 */
  float* out;                 /* fwd: (n, h*d) */
  const float* dout;          /* bwd1 / bwd2: (n, h*d) cotangent of out */
  const float* hbias;         /* bwd2: (n*k, h) cotangent of dbias, row pitch ld_hbias; NULL = 0 */
  const float* henv;          /* bwd2: (n, k) cotangent of denv; NULL = 0 */
  float* dqk;                 /* bwd1 / bwd2: (n*k, ld_dqk) per-token [dq | dk], 2*h*d columns */
  int64_t ld_dqk;
  float* wv;                  /* bwd1 / bwd2: (n*k, h) v gradient of token j is wv[j, h] * dout[n, h] */
  float* dbias;               /* bwd1 / bwd2: (n*k, h); NULL = skip */
  float* denv;                /* bwd1 / bwd2: (n, k), summed over heads; NULL = skip */
  float* ddout;               /* bwd2: (n, h*d) gradient w.r.t. dout */
  int64_t ld_bias, ld_hbias;  /* row pitch (floats, >= h) of bias and hbias; 0 = h */
} cg_pooled_attn_args;

int cg_pooled_attn_fwd(const cg_pooled_attn_args* a, void* stream);
int cg_pooled_attn_bwd1(const cg_pooled_attn_args* a, void* stream);
int cg_pooled_attn_bwd2(const cg_pooled_attn_args* a, void* stream);
/* The forward's output for known weights: out[n, h] = sum_j w[n, h, j] v_j over
 * the valid keys (qkv, token_index, key_count, w, out used); cg_pooled_attn_fwd
 * forms its out with this same kernel after writing lse and w, so the two are
 * equal bit for bit. A
 * checkpoint recompute of a block on the same inputs reuses the first
 * forward's w and lse through it instead of recomputing the softmax. No
 * counterpart in the reference (its recompute reruns the whole forward). */
int cg_pooled_attn_out(const cg_pooled_attn_args* a, void* stream);

/* ------------------------------------------------------------------------
 * Dense projections on the tcgen05 tensor cores (kind::tf32, fp32
 * accumulation in TMEM; `precision` picks one tf32 product or the
 * three-term split of fp32 accuracy):
 *   C[m, n] = epi( alpha * sum_k A(m, k) B(n, k) )
 * A(m, k) is a[m*lda + k] (K-major) or a[k*lda + m] (a_mn_major);
 * B(n, k) is b[n*ldb + k] (K-major) or b[k*ldb + n] (b_mn_major).
 * epi adds bias[n], then per act:
 *   CG_ACT_NONE       nothing;
 *   CG_ACT_SILU       aux_out[m, n] = x (pre-activation), x = silu(x);
 *   CG_ACT_SILU_GRAD  aux_out[m, n] = x when aux_out is set, x *= silu'(aux_in[m, n]);
 *   CG_ACT_ADD        x += aux_in[m, n] (a residual: y = h + x W^T + b);
 * then C = x, or C += x with accumulate. a, b 16-byte aligned; lda, ldb
 * multiples of 4. Replaces the nn.Linear (+ activation) GEMMs Inductor
 * generates inside a compiled region (src/create_graph/region.py:191-198).
 * ---------------------------------------------------------------------- */
#define CG_ACT_NONE 0
#define CG_ACT_SILU 1
#define CG_ACT_SILU_GRAD 2
#define CG_ACT_ADD 3
/* product precision (cg_gemm_args.precision) */
#define CG_GEMM_TF32 0 /* one product of tf32-rounded operands, fp32 accumulation */
#define CG_GEMM_FP32 1 /* three-term tf32 split x = hi + lo: A_lo B_hi + A_hi B_lo + A_hi B_hi,
                          fp32-level accuracy (<= 1e-5 relative) at a third of the tf32 rate */

typedef struct cg_gemm_args {
  int64_t m, n, k;
  const float* a;
  int64_t lda;
  const float* b;
  int64_t ldb;
  float* c;
  int64_t ldc;
  const float* bias;     /* (n,) or NULL */
  const float* aux_in;   /* CG_ACT_SILU_GRAD: pre-activation; CG_ACT_ADD: residual; pitch ld_aux */
  float* aux_out;        /* CG_ACT_SILU / CG_ACT_SILU_GRAD: x before the activation, pitch ld_aux; may be NULL */
  int64_t ld_aux;
  int32_t a_mn_major, b_mn_major;
  int32_t act, accumulate;
  float alpha;
  int32_t precision;     /* CG_GEMM_TF32 (0) or CG_GEMM_FP32 (1) */
  float* workspace;         /* split-K partial tiles; cg_gemm_workspace_bytes() bytes */
  int64_t workspace_bytes;
} cg_gemm_args;

/* When the output tiles cannot fill the GPU and K is long (the weight
 * gradients, K = atoms or edges), K is split across CTAs; their partial tiles
 * go to `workspace` and are added in a fixed order (deterministic). */
int cg_gemm_tf32(const cg_gemm_args* args, void* stream);
/* Workspace bytes cg_gemm_tf32 needs for these args (0: no split). */
int64_t cg_gemm_workspace_bytes(const cg_gemm_args* args);
/* cg_gemm_tf32 for callers that cannot allocate device memory: hosts whose
 * device memory belongs to another allocator (a framework's caching pool, or
 * a Go / JVM / Node service that hands its libraries fixed buffers) and that
 * forbid cudaMalloc, which synchronises the device and can fail under memory
 * pressure. The split-K partial tiles of the weight-gradient shapes go to one
 * static 8 MiB device buffer inside the library instead of args->workspace
 * (ignored); every GPU that loads the library holds that buffer until exit.
 * Shapes needing more scratch are rejected with an error before any launch.
 * The call allocates nothing; its first call on a device looks up the
 * buffer's address (make it before any stream capture) and caches it for the
 * process (host threads may make first calls concurrently; a cudaDeviceReset
 * while the library is in use leaves the cached address stale). All calls
 * share the buffer, so calls that overlap on the GPU (other streams, other
 * threads) race; each call writes every scratch element it later reads, so
 * nothing needs clearing between calls. No counterpart in the reference. */
int cg_gemm_tf32_noalloc(const cg_gemm_args* args, void* stream);

/* ------------------------------------------------------------------------
 * Segment sums over a sorted CSR, their transpose, column reductions.
 * The reference's models reduce with index_add (tests/test_semantics.py:68-69
 * there), an atomic scatter on GPUs; these read every segment in a fixed
 * order, so results are bitwise reproducible.
 * ---------------------------------------------------------------------- */
/* out[e, :] = index[e] >= 0 ? src[index[e], :] : 0 (the transpose of
 * cg_segment_sum); replaces the tensor indexing pos[src] / h[index]. */
int cg_gather_rows(const float* src, int64_t ld_src, const int32_t* index, int64_t n_out, int64_t cols,
                   float* out, int64_t ld_out, void* stream);
/* out[r, :] (+)= sum_{e in [row_ptr[r], row_ptr[r+1])} src[perm ? perm[e] : e, :],
 * in increasing e; replaces index_add (tests/test_semantics.py:68-69 there). */
/* CSR of a many-to-one map: element e goes to row index[e] (outside
 * [0, rows): nowhere). row_ptr (rows + 1) and perm (n; each row's elements in
 * ascending order, then -1 for the unmapped ones), without host
 * synchronisation: one single-block kernel for rows <= 256, else a count /
 * scan / place / sort-rows sequence (integer atomics, order fixed by the
 * final sort: deterministic). Builds the species map of a batch (torch
 * argsort + bincount there would read sizes back to the host). */
int cg_csr_from_index(const int32_t* index, int64_t n, int64_t rows, int32_t* row_ptr, int32_t* perm, void* stream);
int cg_segment_sum(const float* src, int64_t ld_src, const int32_t* row_ptr, const int32_t* perm,
                   int64_t n_rows, int64_t cols, float* out, int64_t ld_out, int accumulate,
                   void* stream);
/* The segment sum of rank-one rows: for s = perm ? perm[e] : e,
 * out[r, h*d + c] (+)= sum_{e in [row_ptr[r], row_ptr[r+1])} w[s*heads + h] * src[(s / group)*ld_src + h*d + c],
 * in increasing e (c < d, h < heads). Reduces the per-token v gradient
 * w[token, h] * dm[atom of token, h] of the pooled attention to atoms without
 * materialising it; no reference counterpart. */
int cg_segment_sum_scaled(const float* w, const float* src, int64_t ld_src, int64_t group, int32_t heads,
                          int32_t d, const int32_t* row_ptr, const int32_t* perm, int64_t n_rows, float* out,
                          int64_t ld_out, int accumulate, void* stream);
/* out[c] (+)= sum_r src[r*ld + c], two fixed-order passes through `scratch`
 * (cg_colsum_scratch_bytes bytes); the bias gradients of nn.Linear. */
int64_t cg_colsum_scratch_bytes(int64_t rows, int64_t cols);
int cg_colsum(const float* src, int64_t ld, int64_t rows, int64_t cols, float* out, int accumulate,
              float* scratch, void* stream);
/* out[c] (+)= sum_r a[r, c] b[r, c] (contiguous rows), as cg_colsum. */
int64_t cg_coldot_scratch_bytes(int64_t rows, int64_t cols);
int cg_coldot(const float* a, const float* b, int64_t rows, int64_t cols, float* out, int accumulate,
              float* scratch, void* stream);

/* ------------------------------------------------------------------------
 * Pointwise and per-row kernels of the energy network (nn.SiLU, nn.LayerNorm
 * of the reference's test models, tests/test_semantics.py:51-69 there).
 * ---------------------------------------------------------------------- */
/* out = silu(z) = z / (1 + exp(-z)), the same arithmetic as the GEMM's SiLU
 * epilogue (a rebuilt activation equals the GEMM's bit for bit); rebuilds
 * activations a memory budget below 1 did not keep. */
int cg_silu(const float* z, float* out, int64_t n, void* stream);
/* out = a * silu'(z) */
int cg_silu_grad(const float* a, const float* z, float* out, int64_t n, void* stream);
/* out = a * b * silu''(z) */
int cg_silu_grad2(const float* a, const float* b, const float* z, float* out, int64_t n, void* stream);
/* out[r, c] = x[r, c] * gamma[c] + beta[c] (either may be NULL) */
int cg_scale_shift(const float* x, const float* gamma, const float* beta, float* out, int64_t rows,
                   int64_t cols, void* stream);
/* xhat = (x - mean) / sqrt(var + eps) per row (rstd may be NULL) */
int cg_rownorm_fwd(const float* x, int64_t rows, int64_t cols, float eps, float* xhat, float* rstd,
                   void* stream);
/* gx = d xhat / dx applied to g */
int cg_rownorm_bwd1(const float* x, const float* g, int64_t rows, int64_t cols, float eps, float* gx,
                    void* stream);
/* gx = d xhat / dx applied to g, plus add (may be NULL): the gradient at a
 * residual branch point x -> (x, rownorm(x)) in one pass (no reference
 * counterpart: autograd adds the two branch gradients there). */
int cg_rownorm_bwd1_add(const float* x, const float* g, const float* add, int64_t rows, int64_t cols, float eps,
                        float* gx, void* stream);
/* gradients of <h, gx(x, g)> w.r.t. x (d_x) and g (d_g) */
int cg_rownorm_bwd2(const float* x, const float* g, const float* h, int64_t rows, int64_t cols, float eps,
                    float* d_x, float* d_g, void* stream);
/* One AdamW step (torch.optim.AdamW, amsgrad off) over n contiguous fp32
 * parameters with their gradients and moment buffers, in place; step counts
 * from 1. The optimizer update after loss.backward() in the training step:
 * the reference leaves it to the user's torch optimizer. */
int cg_adamw_step(float* param, const float* grad, float* exp_avg, float* exp_avg_sq, int64_t n, float lr,
                  float beta1, float beta2, float eps, float weight_decay, int64_t step, void* stream);
/* The same update with the step count kept on the device: `state` (16 bytes,
 * 8-byte aligned, zeroed before the first step) holds the step count and its
 * bias corrections; each call advances it on the stream before updating, so
 * the call can sit in a captured CUDA graph and every replay is the next step. */
int cg_adamw_step_counted(float* param, const float* grad, float* exp_avg, float* exp_avg_sq, int64_t n, float lr,
                          float beta1, float beta2, float eps, float weight_decay, void* state, void* stream);
/* Envelope pooling of k tokens per row n (x contiguous (n, k, cols)):
 * pool: out[n, c] = sum_s w[n, s] x[n, s, c];  outer: out[n, s, c] = w[n, s] g[n, c];
 * dot: out[n, s] = sum_c g[n, c] x[n, s, c]. A family closed under differentiation. */
/* The training loss on energies and forces, F = -dE/dpos:
 *   loss = mean_b (E_b - Et_b)^2 + mean_i (F_i - Ft_i)^2,
 * given grad_pos = dE/dpos (the sign is folded in). One block, fixed
 * reduction order (bitwise reproducible). Replaces the MSE losses the
 * reference's training steps build from torch ops (tests/test_semantics.py,
 * examples/mlp.py there). */
int cg_mse_energy_force(const float* energy, const float* energy_target, int64_t n_energy, const float* grad_pos,
                        const float* force_target, int64_t n_force, float* loss, void* stream);
/* Its gradient: d_energy = 2 (E - Et) / n_energy * g, d_grad_pos = 2 (grad_pos +
 * Ft) / n_force * g, with g = *grad_loss read on the device. */
int cg_mse_energy_force_bwd(const float* energy, const float* energy_target, int64_t n_energy, const float* grad_pos,
                            const float* force_target, int64_t n_force, const float* grad_loss, float* d_energy,
                            float* d_grad_pos, void* stream);
int cg_pool(const float* x, const float* w, int64_t n, int64_t k, int64_t cols, float* out, void* stream);
int cg_pool_outer(const float* w, const float* g, int64_t n, int64_t k, int64_t cols, float* out,
                  void* stream);
int cg_pool_dot(const float* g, const float* x, int64_t n, int64_t k, int64_t cols, float* out,
                void* stream);

/* ------------------------------------------------------------------------
 * Edge geometry of the padded (n_atoms, k) neighbour layout: slot e = i*k + s
 * holds neighbour nbr[e] of centre i (or -1). vec = pos[nbr] - pos[i],
 * d = |vec|, rbf[e, r] = exp(-gamma (d - r*cutoff/(n_rbf-1))^2),
 * env[e] = (cos(pi d / cutoff) + 1) / 2 inside the cutoff. rev_ptr/rev_idx:
 * reverse CSR (slots grouped by neighbour, ascending). Replaces the eager
 * geometry before the reference's region (README.md:28,
 * tests/test_semantics.py:46-48 there) and its autograd double backward.
 * ---------------------------------------------------------------------- */
typedef struct cg_geom_args {
  const float* pos;        /* (n_atoms, 3) */
  const int32_t* nbr;      /* (n_atoms, k) */
  const int32_t* rev_ptr;  /* (n_atoms + 1) */
  const int32_t* rev_idx;  /* (valid slots) */
  int64_t n_atoms;
  int32_t k, n_rbf;
  float cutoff, gamma;
} cg_geom_args;

int cg_edge_geom_fwd(const cg_geom_args* a, float* rbf, float* env, void* stream);
/* g_pos from (g_rbf, g_env); gvec: (n_atoms*k, 3) scratch */
int cg_edge_geom_bwd1(const cg_geom_args* a, const float* g_rbf, const float* g_env, float* gvec,
                      float* g_pos, void* stream);
/* gradients of <h_pos, g_pos(pos, g_rbf, g_env)> w.r.t. pos, g_rbf, g_env */
int cg_edge_geom_bwd2(const cg_geom_args* a, const float* g_rbf, const float* g_env, const float* h_pos,
                      float* gvec, float* d_pos, float* d_g_rbf, float* d_g_env, void* stream);

/* ------------------------------------------------------------------------
 * Neighbour lists of a batch of non-periodic systems (atoms sorted by system,
 * system b = atoms [sys_ptr[b], sys_ptr[b+1])). For atom i: the other atoms
 * of its system with d2 < cutoff^2, d2 = (dx*dx + dy*dy) + dz*dz in
 * round-to-nearest single operations (no FMA), the k nearest by (d2, j) in
 * that order; nbr (n_atoms, k) padded with -1, counts (n_atoms). rev_ptr
 * (n_atoms + 1) / rev_idx (sum of counts) is the reverse CSR, slots grouped by
 * neighbour in ascending slot order. workspace: cg_neighbor_list_workspace()
 * int32s. Bit-exact and deterministic. Limits: k <= 64, systems of up to
 * 12000 atoms (max_atoms_per_system must bound every system), n_atoms * k
 * below 2^31; the distance work is O(n^2) per system. The reference leaves
 * neighbour lists to model code before its region (README.md:28 there).
 * ---------------------------------------------------------------------- */
int cg_neighbor_list_workspace(int64_t n_systems);
int cg_neighbor_list(const float* pos, const int32_t* sys_ptr, int64_t n_systems, int64_t n_atoms,
                     int64_t max_atoms_per_system, float cutoff, int32_t k, int32_t* nbr, int32_t* counts,
                     int32_t* rev_ptr, int32_t* rev_idx, int32_t* workspace, void* stream);

/* The device error word kernels set when a bounded wait gave up (0: none);
 * reset != 0 clears it. Synchronises with the device. No reference
 * counterpart: the reference's kernels are generated by Inductor and have no
 * waits. */
int cg_device_error(int* out, int reset);

#ifdef __cplusplus
}
#endif

#endif /* CG_B200_H */
