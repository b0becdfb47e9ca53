/*
 * sparsepr_b200 — C ABI of the B200-native SparsePR attention hot path.
 *
 * Every entry point is stream-ordered on `stream` (a cudaStream_t passed as
 * void*), performs no host<->device synchronisation and allocates no memory:
 * outputs and scratch ("workspace") belong to the caller, who sizes scratch
 * with the matching *_workspace_bytes query.  All pointers are device
 * pointers unless stated.  Tensors are dense, row-major, last dimension
 * contiguous; "bh" is batch*heads.
 *
 * Return value: SPR_OK (0) or a negative SPR_ERR_* status; the message of the
 * last failure on the calling host thread is available from spr_last_error().
 *
 * Each declaration cites the reference interface it replaces (paths relative
 * to the SparsePR project root).
 */
#ifndef SPARSEPR_B200_H
#define SPARSEPR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  SPR_OK = 0,
  SPR_ERR_SHAPE = -1,
  SPR_ERR_DTYPE = -2,
  SPR_ERR_ALIGN = -3,
  SPR_ERR_LAUNCH = -4,
  SPR_ERR_TIMEOUT = -5,
  SPR_ERR_UNIMPLEMENTED = -6,
  SPR_ERR_WORKSPACE = -7,
  SPR_ERR_ARG = -8
};

/* Element type codes for `*_dtype` arguments. */
enum { SPR_F32 = 0, SPR_BF16 = 1, SPR_F16 = 2 };

/* Distance precision of the k-means assignment GEMM: TF32 tensor-core dot
 * products (the reference's GPU behaviour), or 3xTF32 split products that
 * reproduce fp32 dot products (d <= 64). */
enum { SPR_KMEANS_TF32 = 0, SPR_KMEANS_FP32 = 1 };

/* Library version (major*10000 + minor*100 + patch). */
int spr_version(void);
/* Message of the last failed call on this host thread ("" if none). */
const char* spr_last_error(void);

/* ---------------------------------------------------------------- k-means */

/* Scratch bytes needed by spr_kmeans_lloyd / spr_kmeans_assign / spr_label_sort.
 * The first int32 of the workspace holds the device status of the last call
 * (0 = ok, else a bounded wait inside a kernel gave up). */
size_t spr_kmeans_workspace_bytes(int64_t bh, int64_t n, int d, int k);

/*
 * Batched Lloyd k-means, `iters` iterations with an on-device stop when the
 * max L2 centroid shift falls below `tol` (later iterations become no-ops).
 * x [bh,n,d] (x_dtype), centroids_inout [bh,k,d] fp32 (initial in, final out).
 * Outputs (for the last assignment): labels [bh,n] i32, sizes [bh,k] i32,
 * offsets [bh,k+1] i32 (exclusive prefix of sizes), order [bh,n] i32 (token
 * ids sorted by label, ties by token id), iters_done [1] i32.
 * centroid_round_dtype: SPR_F32, or x_dtype to round updated centroids to the
 * storage type each iteration like the standalone flash_kmeans path.
 * precision: SPR_KMEANS_TF32 or SPR_KMEANS_FP32 (see above).
 * Replaces: src/sparsepr/kmeans_utils.py:1504-1580 batch_kmeans_Euclid(backend="flash")
 *   -> 1281-1465 (assign kmeans_utils.py:775-893 / flash_kmeans/assign_euclid_triton.py:803-1412,
 *   update flash_kmeans/centroid_update_triton.py:316-386, sizes kmeans_utils.py:1110-1157),
 *   and flash_kmeans/kmeans_triton_impl.py:55-115.
 */
int spr_kmeans_lloyd(const void* x, int x_dtype, int64_t bh, int64_t n, int d, int k,
                     int iters, float tol, int centroid_round_dtype, int precision,
                     float* centroids_inout, int32_t* labels, int32_t* sizes,
                     int32_t* offsets, int32_t* order, int32_t* iters_done,
                     void* workspace, size_t workspace_bytes, void* stream);

/*
 * One assignment step: labels[b,i] = argmin_j max(|x|^2+|c_j|^2-2 x.c_j, 0),
 * ties to the lowest j.  Replaces flash_kmeans/assign_euclid_triton.py:1238-1412
 * euclid_assign_triton.
 */
int spr_kmeans_assign(const void* x, int x_dtype, int64_t bh, int64_t n, int d, int k,
                      const float* centroids, int precision, int32_t* labels, void* workspace,
                      size_t workspace_bytes, void* stream);

/*
 * Stable counting sort of labels: sizes [bh,k], offsets [bh,k+1], order [bh,n].
 * Replaces the torch.argsort(labels) of src/sparsepr/models/common/n8_v6.py:905 and
 * src/sparsepr/adapters/wan22.py:2031 plus _cluster_sizes_from_labels (kmeans_utils.py:1110-1157).
 */
int spr_label_sort(const int32_t* labels, int64_t bh, int64_t n, int k, int32_t* sizes,
                   int32_t* offsets, int32_t* order, void* workspace, size_t workspace_bytes,
                   void* stream);

/*
 * Segmented mean over the label-sorted order, fused with the permute:
 * means[b,c,:] = mean of x[b, order[b, offsets[b,c]:offsets[b,c+1]], :] in fp32,
 * empty clusters take fallback[b,c,:] (or 0 when fallback is NULL);
 * when x_perm != NULL also writes x_perm[b,s,:] = x[b,order[b,s],:].
 * Replaces models/cosmos3/operator_kmeans.py:609-679 (original_centroids,
 * joint_original_centroids -> kernels/triton/centroid_reduction.py:138-196) and
 * kernels/triton/permute.py:126-172 permute_tensor_by_labels_triton.
 */
int spr_centroid_means(const void* x, int x_dtype, const int32_t* order, const int32_t* offsets,
                       int64_t bh, int64_t n, int d, int k, const float* fallback, float* means,
                       void* x_perm, void* stream);

/*
 * Row permute of [bh,n,d] elements of elem_bytes each: inverse==0 gathers
 * y[b,s]=x[b,idx[b,s]]; inverse==1 scatters y[b,idx[b,s]]=x[b,s].
 * Replaces kernels/triton/permute.py:126-172 and 235-274 (apply_inverse_permutation_triton).
 */
int spr_permute_rows(const void* x, const int32_t* idx, void* y, int64_t bh, int64_t n, int d,
                     int elem_bytes, int inverse, void* stream);

/* ---------------------------------------------------------------- routing */

/*
 * Wan producer step: full-channel RMSNorm of Q and K (mean of squares over all
 * C = heads*head_dim channels of a token, fp32), times the norm weight, rounded
 * to the model dtype; complex RoPE on channel pairs (2i, 2i+1) of each head
 * with freq_real/freq_imag [tokens, head_dim/2] fp32; rounded again; written as
 * [batch, heads, tokens, head_dim].  V is only re-laid out.  q, k, v
 * [batch, tokens, C] and the weights [C] share `dtype` (SPR_BF16, SPR_F16 or
 * SPR_F32); head_dim even and a multiple of 8 (16-bit) / 4 (fp32).
 * Replaces wan_qkv_norm_rope_layout (src/sparsepr/kernels/n8_ext/csrc/n8_ops.cu:357-411,
 * kernel 16-105; Python entry kernels/n8_extension.py).
 */
int spr_wan_qkv_norm_rope_layout(const void* q, const void* k, const void* v, const void* q_weight,
                                 const void* k_weight, const float* freq_real, const float* freq_imag, int dtype,
                                 int64_t batch, int64_t tokens, int channels, int heads, float epsilon, void* q_out,
                                 void* k_out, void* v_out, void* stream);

/*
 * Attention-mass selector scores: scores[b,q,c] = log sum_{t in cluster c}
 * exp(qc[b,q].k_sorted[b,t] / sqrt(d)), -inf for empty clusters.
 * q_centroids [bh,cq,d] fp32, k_sorted [bh,n,d] bf16, k_offsets [bh,ck+1] i32;
 * d = 128.  Tensor cores: each centroid as three bf16 parts, fp32 accumulation.
 * Replaces kernels/triton/svg_ear.py:372-450 attention_mass_scores_triton (kernel 7-92).
 */
int spr_attention_mass_scores(const float* q_centroids, const void* k_sorted, const int32_t* k_offsets,
                              int64_t bh, int cq, int ck, int64_t n, int d, float* scores, void* stream);

/*
 * SVG-EAR value-error selector scores: for query centroid c and key cluster j
 * with tokens t (sorted order), a = exp(qc.kbar_j/sqrt(d)), b_t = exp(qc.k_t/sqrt(d)),
 *   scores[b,c,j] = log( (1/n_j) sum_t |a vbar_j - b_t v_t|^2 ),
 * -inf for an empty cluster.  k_sorted, v_sorted [bh,n,d] bf16; q_centroids
 * [bh,cq,d], k_centroids, v_centroids [bh,ck,d] fp32; d = 128.  Workspace from
 * spr_svg_ear_value_scores_workspace_bytes.
 * Replaces svg_ear_value_error_scores_triton (src/sparsepr/kernels/triton/svg_ear.py:453-531,
 * kernel 95-193) as the route calls it (no Jensen term, n8_v6.py:984-998).
 */
size_t spr_svg_ear_value_scores_workspace_bytes(int64_t bh, int cq, int ck, int64_t n);
int spr_svg_ear_value_scores(const float* q_centroids, const void* k_sorted, const void* v_sorted,
                             const float* k_centroids, const float* v_centroids, const int32_t* k_offsets, int64_t bh,
                             int cq, int ck, int64_t n, int d, float* scores, void* workspace, size_t workspace_bytes,
                             void* stream);

/*
 * Role-equal probe representatives: best[b,c] = the token of cluster c nearest
 * (squared distance, ties to the lowest token) to the mean of the cluster's
 * role features, n for an empty cluster.  feat fp32 [bh,n,r] (r <= 64), order
 * int32 [bh,n] (tokens sorted by cluster, ascending within a cluster), offsets
 * int32 [bh,k+1]; best int32 [bh,k].  Replaces the token pass of
 * select_role_equal_probes_vectorized (src/sparsepr/models/cosmos3/residual_repair.py:118-208).
 */
int spr_probe_representatives(const float* feat, const int32_t* order, const int32_t* offsets, int64_t bh, int64_t n,
                              int r, int k, int32_t* best, void* stream);

/*
 * Role projection of the route (tensor cores): out[b,t,:] = x[b,t,:] F[b] / rms,
 * x bf16 [bh,n,d] (d = 128), F fp32 [bh,d,r] (r = 16, 32, 48 or 64), out fp32
 * [bh,n,r].  mode 0: one RMS over all n*r features of a head (clamped at
 * 1e-8), written to scale[bh]; mode 1: one RMS per row (clamped at 1e-6),
 * scale unused.  Workspace from spr_role_projection_workspace_bytes.
 * Replaces the K-role projection + normalize_feature_scale and the Q-role
 * role_projection_rms_triton (src/sparsepr/models/common/n8_v6.py:141-178,
 * 659-806; src/sparsepr/kernels/triton/role_projection.py:58-103).
 */
size_t spr_role_projection_workspace_bytes(int64_t bh, int64_t n, int r);
int spr_role_projection(const void* x, const float* factor, int64_t bh, int64_t n, int d, int r, int mode, float* out,
                        float* scale, void* workspace, size_t workspace_bytes, void* stream);
/* Status of the last spr_role_projection launch (synchronous copy; 0 = ok). */
int spr_role_projection_status(int* out);
/* Stream-ordered copy of the same status word into device memory at dst (one
 * int32), so a caller can collect it without synchronising. */
int spr_role_projection_status_async(int32_t* dst, void* stream);

/*
 * Status of the last spr_attention_mass_scores launch (synchronous copy):
 * *out = 0, or the code of a device-side bounded wait that gave up.
 */
int spr_attention_mass_scores_status(int* out);
/* Stream-ordered copy of the same status word into device memory at dst (one
 * int32), so a caller can collect it without synchronising. */
int spr_attention_mass_scores_status_async(int32_t* dst, void* stream);

/*
 * Budgeted cluster selection per (b, q): descending score (ties -> lower
 * cluster id), keep the positive-size prefix within budgets[b,q], plus the
 * first crossing cluster.  routed [bh,cq+1,ck+1] u8 (nullable; header row/col
 * as the reference), sel_ids [bh,cq,ck] i32 ascending selected cluster ids
 * (-1 padded), sel_counts [bh,cq] i32.  ck <= 2048.
 * Replaces kernels/triton/selector_budget.py:131-171 exact_budget_dynamic_map_triton and
 * kernels/n8_ext/csrc/n8_ops.cu:271-355 (svg_ear_select_budget_schedule, compact_selected_clusters).
 */
int spr_select_budget(const float* scores, const int32_t* k_sizes, const int32_t* budgets,
                      int64_t bh, int cq, int ck, uint8_t* routed, int32_t* sel_ids,
                      int32_t* sel_counts, void* stream);

/* ---------------------------------------------------------------- attention */

/*
 * Reduced-rank residual repair state of one call (all device pointers, fp32
 * unless noted; per problem b): x_mean, x_scale, y_mean [bh][d]; left, basis
 * [bh][d][rank] (rank == 16); alpha the repair strength; probe_rows [bh][m]
 * the probe token ids in ascending order and probe_dense [bh][m][d] bf16 their
 * exact rows (m <= 128).  Mirrors the state N8V6Core.repair fits
 * (src/sparsepr/models/cosmos3/residual_repair.py:263-465) and the arguments
 * of the fused apply + overwrite kernel it launches
 * (src/sparsepr/kernels/triton/residual_repair.py:565-653).
 */
typedef struct SprRepairState {
  const float* x_mean;
  const float* x_scale;
  const float* y_mean;
  const float* left;
  const float* basis;
  int rank;
  float alpha;
  const int32_t* probe_rows;
  const void* probe_dense;
  int m;
} SprRepairState;

/*
 * Block-sparse attention over kept cluster pairs, bf16 in, fp32 accumulate:
 * for query row s of q-cluster c (rows q_offsets[b,c]..q_offsets[b,c+1] of
 * q_perm), softmax(q.K^T/sqrt(d)) V over the key rows of the clusters
 * sel_ids[b,c,0:sel_counts[b,c]] (runs k_offsets[b,j]..k_offsets[b,j+1] of
 * k_perm/v_perm).  Rows with no keys output 0.  q_perm [bh,nq,d],
 * k_perm/v_perm [bh,nk,d] bf16, d == 128.  When q_order != NULL the row is
 * stored at out[b, q_order[b,s]] (fused inverse permute), else at out[b,s].
 * repair (nullable): the repair is applied in the epilogue, each row v (the
 * bf16-rounded attention row) stored as bf16(v + alpha*((((v - x_mean)/x_scale)
 * left) basis^T + y_mean)), and the rows of the probe tokens are stored as
 * their dense rows instead (needs ck <= 1024; tokens are the stored row
 * indices, i.e. q_order[b,s] when q_order is given).
 * Replaces src/sparsepr/kmeans_utils.py:2164-2350 dynamic_block_sparse_fwd_flashinfer
 * (+ its plan() index build), kernels/triton/permute.py:235-274 and, with a
 * repair state, kernels/triton/residual_repair.py:158-254 / 565-653 (fused
 * apply + probe overwrite).
 */
int spr_block_sparse_attn(const void* q_perm, const void* k_perm, const void* v_perm,
                          const int32_t* q_offsets, const int32_t* k_offsets,
                          const int32_t* sel_ids, const int32_t* sel_counts,
                          int64_t bh, int64_t nq, int64_t nk, int d, int cq, int ck,
                          const int32_t* q_order, const SprRepairState* repair, void* out,
                          void* workspace, size_t workspace_bytes, void* stream);
size_t spr_block_sparse_attn_workspace_bytes(int64_t bh, int64_t nq, int cq);

/*
 * Probe pre-pass of the fused repair: for the m probe rows of each problem
 * (rows [bh][m] token ids into the original-order q [bh][n][d] bf16, and
 * row_cluster [bh][m] their query clusters), attention against every key of
 * the cluster-sorted k_perm/v_perm [bh][nk][d] in one pass: out_dense [bh][m][d]
 * the exact dense rows (src/sparsepr/models/common/n8_v6.py:1234-1243) and
 * out_base [bh][m][d] the rows restricted to the key clusters their query
 * cluster keeps in routed [bh][cq+1][ck+1] (header row/column first), i.e.
 * the sparse attention output at those rows, which the repair fit regresses
 * from (n8_v6.py:1244-1262).  m <= 128, d == 128; the keys are split over
 * several CTAs per problem and merged in a fixed order; workspace of
 * spr_probe_rows_attn_workspace_bytes(bh, nk, m) bytes (its first int32 is the
 * status).
 */
size_t spr_probe_rows_attn_workspace_bytes(int64_t bh, int64_t nk, int m);
int spr_probe_rows_attn(const void* q, const void* k_perm, const void* v_perm, const int32_t* k_offsets,
                        const uint8_t* routed, const int32_t* rows, const int32_t* row_cluster,
                        int64_t bh, int64_t n, int64_t nk, int d, int cq, int ck, int m,
                        void* out_dense, void* out_base, void* workspace, size_t workspace_bytes,
                        void* stream);

/*
 * spr_block_sparse_attn without a workspace, for callers that cannot allocate
 * device memory (a host that owns all of HBM through its own pool, or a loop
 * that must not call cudaMalloc and has no buffer to lend).  Same arguments and
 * result as spr_block_sparse_attn minus the workspace.  Its scratch is a fixed
 * library-owned device array of 65,536 tile-table entries: every GPU that loads
 * the library keeps 256 KiB for it until the process exits, and calls with
 * bh*(cq+1) > 65,536 are rejected with SPR_ERR_SHAPE.  Every call looks up
 * the array's device address on the current device (cudaGetSymbolAddress).
 * All calls share the array: calls that overlap on the GPU (other streams,
 * other host threads) race; the array keeps the last call's contents and each
 * call rewrites what it reads.  No counterpart in the reference.
 */
int spr_block_sparse_attn_noalloc(const void* q_perm, const void* k_perm, const void* v_perm,
                                  const int32_t* q_offsets, const int32_t* k_offsets,
                                  const int32_t* sel_ids, const int32_t* sel_counts,
                                  int64_t bh, int64_t nq, int64_t nk, int d, int cq, int ck,
                                  const int32_t* q_order, void* out, void* stream);

/*
 * Device status word of the last spr_block_sparse_attn_noalloc call on the
 * current device (0 = ok, else the code of the bounded wait that gave up, in
 * which case that call's output is incomplete).  Synchronous copy.  No
 * counterpart in the reference (its kernels trap instead of reporting).
 */
int spr_block_sparse_attn_noalloc_status(int* out);

/*
 * Self-test of the bounded device wait used by every pipelined kernel here:
 * one thread waits on an mbarrier that nothing completes, gives up after
 * limit_ns (at most 0.1 s), writes `code` into the device int *err (if it is
 * still 0) and the kernel returns; the context stays usable.  No counterpart
 * in the reference (its kernels have no bounded waits).
 */
int spr_selftest_bounded_wait(int* err, int code, int64_t limit_ns, void* stream);

/* ---------------------------------------------------------------- small linear algebra */

/*
 * Batched symmetric eigendecomposition (one CTA per matrix; n = 64, 128:
 * Householder tridiagonalisation, multisection and twisted-factorisation
 * eigenvectors, Jacobi for matrices with repeated eigenvalues; other n:
 * cyclic two-sided Jacobi): a [batch,n,n] fp32 (symmetrised on load), n even <= 128.  Outputs
 * evals [batch,n] ascending and evecs [batch,n,n] with eigenvectors in the
 * columns, the torch.linalg.eigh convention.  Replaces the torch.linalg.eigh calls of
 * src/sparsepr/models/cosmos3/operator_kmeans.py:94-151 (metric_factor) and
 * src/sparsepr/models/cosmos3/residual_repair.py:468-491 (reduced_rank_output_basis).
 */
int spr_sym_eig(const float* a, int64_t batch, int n, int max_sweeps, float* evals, float* evecs,
                void* stream);

/*
 * The same decomposition when only the `top` largest eigenpairs are used:
 * evals [batch,n] all eigenvalues ascending; evecs [batch,n,n] holds the
 * eigenvectors of the `top` largest eigenvalues in its last `top` columns and
 * zeros elsewhere (n = 64 and 128; other n return all eigenvectors).  The
 * callers of the reference take the top columns of a full torch.linalg.eigh
 * (src/sparsepr/models/cosmos3/operator_kmeans.py:94-151, metric_factor;
 * src/sparsepr/models/cosmos3/residual_repair.py:468-491), so the unused
 * vectors are not formed.  1 <= top <= n, else SPR_ERR_ARG.
 */
int spr_sym_eig_top(const float* a, int64_t batch, int n, int top, int max_sweeps, float* evals, float* evecs,
                    void* stream);

/*
 * Batched Cholesky solve A x = b of symmetric positive definite systems:
 * a [batch,m,m] fp32 (m <= 128), b and x [batch,m,nrhs] fp32 (x must not alias b).
 * A system that is not positive definite yields non-finite x (no error, no trap).
 * Replaces the torch.linalg.cholesky_ex + cholesky_solve dual ridge solve of
 * src/sparsepr/models/cosmos3/residual_repair.py:389-404.
 */
int spr_chol_solve(const float* a, const float* b, int64_t batch, int m, int nrhs, float* x, void* stream);

/*
 * Cholesky-QR of x [batch][n][r] (n, r <= 128): columns normalised to unit
 * length, G = X^T X + mean(diag G)*relative_ridge*I = L L^T, out = X L^{-T}.
 * When G is not positive definite: out = the normalised X and failed[b] = 1.
 * Replaces the cholesky_qr step of warm_subspace_metric_factor
 * (src/sparsepr/models/cosmos3/operator_kmeans.py:332-364).
 */
int spr_cholesky_qr(const float* x, int64_t batch, int n, int r, float relative_ridge, float* out, int32_t* failed,
                    void* stream);

/*
 * Batched lower Cholesky factor l [batch][m][m] of a + scale[b]*relative_ridge*I,
 * falling back to scale[b]*fallback_ridge; when both fail, l = I and failed[b] = 1.
 * Replaces cholesky_with_device_fallback (operator_kmeans.py:154-218).
 */
int spr_ridge_cholesky(const float* a, const float* scale, int64_t batch, int m, float relative_ridge,
                       float fallback_ridge, float* l, int32_t* failed, void* stream);

/* ---------------------------------------------------------------- repair */

/*
 * Apply the reduced-rank residual repair and overwrite probe rows:
 * out[b,i] = base[b,i] + alpha*((((base[b,i]-x_mean)/x_scale) L) B^T + y_mean),
 * then out[b, rows[b,m]] = dense[b,m].  base/out [bh,n,d] bf16 (may alias),
 * x_mean/x_scale/y_mean [bh,d] fp32, left/basis [bh,d,r] fp32, rows [bh,m] i32,
 * dense [bh,m,d] bf16.  Replaces kernels/triton/residual_repair.py:388-562
 * n8_repair_apply_output_triton and 656-700 n8_exact_probe_scatter_triton.
 */
int spr_repair_apply(const void* base, const float* x_mean, const float* x_scale, const float* y_mean,
                     const float* left, const float* basis, int64_t bh, int64_t n, int d, int r,
                     float alpha, const int32_t* rows, const void* dense, int m, void* out,
                     void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPARSEPR_B200_H */
