/*
 * e2a.h -- C ABI of the B200 (sm_100a) E2Former-V2 sparse equivariant attention library.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream (as void*; NULL = legacy
 * default stream), returns an int status (E2A_OK = 0) and never allocates device memory: the caller
 * owns all outputs and passes scratch as a workspace whose size it queries first.  Device code never
 * traps; bad arguments return E2A_ERR_ARG and CUDA failures E2A_ERR_CUDA (the cudaError_t is kept in
 * e2a_last_cuda_error()).  All reductions are CSR-ordered (no float atomics): results are bitwise
 * reproducible run to run.
 *
 * Reference interfaces replaced (paths inside IQuestLab/UBio-MolFM, e2f = src/molfm/models/e2former):
 *   e2a_csr_*            prepare_sparse_qk_edge_index_metadata   e2f/triton_dr/triton_sparse_qk_autograd.py:635-652
 *   e2a_pbc_expand       CellExpander.expand_includeself         e2f/module_utils.py:1065-1275
 *   e2a_radius_graph_*   construct_radius_neighbor               e2f/module_utils.py:3119-3242
 *   e2a_sparse_qk_fwd    sparse_qk_edge_index_triton (forward)   e2f/triton_dr/triton_sparse_qk_autograd.py:839-871, 52-98
 *   e2a_grouped_reduce   _edge_grouped_reduce_triton (dQ, dK)    e2f/triton_dr/triton_sparse_qk_autograd.py:654-673, 388-435
 *   e2a_alpha_sum_*      sparse_alpha_sum_edge_index_triton      e2f/triton_dr/sparse_alpha_sum_edge_index_autograd.py:207-213
 *   e2a_v_agg_*          sparse_v_agg_edge_index_triton_cblocked e2f/triton_dr/sparse_v_agg_edge_index_cblocked_bench.py:428-449
 *   e2a_edge_outer_*     edge_degree_outer_triton                e2f/triton_dr/edge_degree_outer_autograd.py:348-375
 *   e2a_attn_fwd         E2AttentionArbOrder_sparse.forward, QK logits -> segmented softmax ->
 *                        alpha/r -> value aggregation            e2f/e2former.py:311-364, 393-422;
 *                                                                e2f/wigner6j/so2_tensor_product.py:370-377
 *   e2a_attn_bwd_query / e2a_attn_bwd_key
 *                        the first-order backward of the same span (what autograd runs for forces)
 */
#ifndef E2A_H
#define E2A_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define E2A_OK 0
#define E2A_ERR_ARG 1
#define E2A_ERR_CUDA 2
#define E2A_ERR_WORKSPACE 3
#define E2A_ERR_UNSUPPORTED 4

/* Library version (major*10000 + minor*100 + patch). */
int e2a_version(void);
/* Human-readable name of a status code. */
const char* e2a_status_string(int status);
/* cudaError_t of the most recent E2A_ERR_CUDA on this host thread (0 if none). */
int e2a_last_cuda_error(void);
/* Number of kernels this library has launched in this process (all host threads). */
uint64_t e2a_launch_count(void);

/* ------------------------------------------------------------------------------------------ */
/* CSR metadata: prepare_sparse_qk_edge_index_metadata (triton_sparse_qk_autograd.py:635-652). */
/* query-CSR: q_row_ptr[N+1], q_col[E] (neighbour of each CSR slot), q_perm[E] (edge id of each  */
/* slot; identity when query_idx is already sorted).  key-CSR: the stable grouping by neighbour: */
/* k_row_ptr[M+1], k_col[E] (query of each slot), k_perm[E] (edge id).  int32 everywhere.        */
/* ------------------------------------------------------------------------------------------ */
size_t e2a_csr_workspace_bytes(int64_t num_edges, int64_t num_queries, int64_t num_keys);
int e2a_csr_build(const int32_t* query_idx, const int32_t* neighbor_idx, int64_t num_edges,
                  int64_t num_queries, int64_t num_keys,
                  int32_t* q_row_ptr, int32_t* q_col, int32_t* q_perm,
                  int32_t* k_row_ptr, int32_t* k_col, int32_t* k_perm,
                  void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------------ */
/* PBC image expansion: CellExpander.expand_includeself (module_utils.py:1065-1275).            */
/* offsets[n_img,3] are the fp32 lattice translations in the reference's cell order with image 0 */
/* = (0,0,0).  Image (c, a) = pos[a] + offsets[c] is kept iff some atom lies strictly within     */
/* `cutoff` of it; kept images are written cell-major, atom-ascending: exp_pos[k] its position,  */
/* image_atom[k] = c * n_atoms + a.  Both must hold n_img*n_atoms entries; *n_expanded (host)    */
/* receives the kept count (synchronises).                                                       */
/* ------------------------------------------------------------------------------------------ */
size_t e2a_pbc_expand_workspace_bytes(int64_t n_atoms, int n_img);
int e2a_pbc_expand(const float* pos, int64_t n_atoms, const float* offsets, int n_img, float cutoff,
                   float* exp_pos, int64_t* image_atom, int64_t* n_expanded,
                   void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------------ */
/* Radius graph: construct_radius_neighbor (module_utils.py:3119-3242), cell-list build.        */
/* Systems b = 0..B-1 own queries [q_ptr[b], q_ptr[b+1]) and expanded points                     */
/* [p_ptr[b], p_ptr[b+1]) (q_ptr/p_ptr are DEVICE int64 arrays).  Row i keeps the candidates j   */
/* of its system with min_dist <= |pos_i - pts_j| <= max_dist, ordered by (distance, j)          */
/* ascending and truncated to max_neighbors (<= 0: no cap).  Distances use the fp32 operation    */
/* sequence of torch.linalg.norm on CPU, so edge sets and distances are bit-exact.               */
/* Two phases sharing one workspace: _plan counts (synchronises; returns E and the candidate     */
/* total on the host), _fill writes E edges.                                                     */
/* ------------------------------------------------------------------------------------------ */
size_t e2a_radius_graph_workspace_bytes(int64_t n_queries, int64_t n_points, int64_t n_systems);
int e2a_radius_graph_plan(const float* pos, const float* pts, const int64_t* q_ptr, const int64_t* p_ptr,
                          int64_t n_queries, int64_t n_points, int64_t n_systems,
                          float max_dist, float min_dist, int64_t max_neighbors,
                          int64_t* num_edges, int64_t* num_candidates,
                          void* workspace, size_t workspace_bytes, void* stream);
size_t e2a_radius_graph_fill_workspace_bytes(int64_t num_candidates);
int e2a_radius_graph_fill(const float* pos, const float* pts, const int64_t* q_ptr, const int64_t* p_ptr,
                          int64_t n_queries, int64_t n_points, int64_t n_systems,
                          float max_dist, float min_dist, int64_t max_neighbors,
                          int64_t num_edges, int64_t num_candidates,
                          int64_t* query_idx, int64_t* neighbor_idx, int32_t* row_ptr, int32_t* col,
                          float* edge_vec, float* dist, float* poly,
                          void* workspace, size_t workspace_bytes,
                          void* fill_workspace, size_t fill_workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------------ */
/* Kernel-level sparse ops (same arithmetic as the reference's Triton kernels).                  */
/* ------------------------------------------------------------------------------------------ */
/* out[perm[p], h] = <q[i,h,:], k[col[p],h,:]> for p in row i of the query-CSR.  q:[N,H,D] k:[M,H,D] */
int e2a_sparse_qk_fwd(const float* q, const float* k, const int32_t* row_ptr, const int32_t* col,
                      const int32_t* perm, int64_t n_rows, int64_t n_edges, int H, int D,
                      float* out, void* stream);
/* out[r,h,:] = sum_{p in row r} alpha[perm[p],h] * x[col[p],h,:]   (dQ with the query-CSR and x=k, */
/* dK with the key-CSR and x=q).  alpha:[E,H]  x:[*,H,D]  out:[n_rows,H,D]                         */
int e2a_grouped_reduce(const float* alpha, const float* x, const int32_t* row_ptr, const int32_t* col,
                       const int32_t* perm, int64_t n_rows, int H, int D, float* out, void* stream);
/* out[i,h] = sum_{p in row i} alpha[perm[p],h] */
int e2a_alpha_sum_fwd(const float* alpha, const int32_t* row_ptr, const int32_t* perm, int64_t n_rows,
                      int H, float* out, void* stream);
/* grad_alpha[e,h] = grad_out[query_idx[e],h] */
int e2a_alpha_sum_bwd(const float* grad_out, const int32_t* query_idx, int64_t n_edges, int H,
                      float* grad_alpha, void* stream);
/* out[i,c,h] = sum_{p in row i} alpha[perm[p],h] * value[col[p],c,h].  value:[M,C,H] out:[N,C,H] */
int e2a_v_agg_fwd(const float* value, const float* alpha, const int32_t* row_ptr, const int32_t* col,
                  const int32_t* perm, int64_t n_rows, int C, int H, float* out, void* stream);
/* The same aggregation of bf16 value rows (value: [M,C,H] bfloat16, 8-byte aligned), widened to fp32  */
/* as they are gathered; fp32 alpha, sums and out.  E2A_ERR_UNSUPPORTED unless H divides 1024, H % 4 == 0 */
/* and C*H <= 16384 (the caller then widens value itself and calls e2a_v_agg_fwd).                       */
/* Replaces: sparse_v_agg_edge_index_triton_cblocked on bf16 values                                      */
/*           (e2f/triton_dr/sparse_v_agg_edge_index_cblocked_bench.py:428-449, 197-240).                 */
int e2a_v_agg_fwd_bf16(const void* value, const float* alpha, const int32_t* row_ptr, const int32_t* col,
                       const int32_t* perm, int64_t n_rows, int C, int H, float* out, void* stream);
/* d_alpha[perm[p],h] = sum_c dout[i,c,h] * value[col[p],c,h]  (query-CSR) */
int e2a_v_agg_bwd_alpha(const float* dout, const float* value, const int32_t* row_ptr, const int32_t* col,
                        const int32_t* perm, int64_t n_rows, int C, int H, float* d_alpha, void* stream);
/* d_value[m,c,h] = sum_{p in key row m} alpha[perm[p],h] * dout[col[p],c,h]  (key-CSR) */
int e2a_v_agg_bwd_value(const float* alpha, const float* dout, const int32_t* k_row_ptr,
                        const int32_t* k_col, const int32_t* k_perm, int64_t n_keys, int C, int H,
                        float* d_value, void* stream);
/* out[i,l,h] = sum_{p in row i} sh[perm[p],l] * fea[perm[p],h].  sh:[E,L] fea:[E,F] out:[N,L,F] */
int e2a_edge_outer_fwd(const float* sh, const float* fea, const int32_t* row_ptr, const int32_t* perm,
                       int64_t n_rows, int L, int F, float* out, void* stream);
/* d_sh[e,l] = sum_h go[q_e,l,h] fea[e,h];  d_fea[e,h] = sum_l go[q_e,l,h] sh[e,l] (either may be NULL) */
int e2a_edge_outer_bwd(const float* grad_out, const float* sh, const float* fea, const int32_t* query_idx,
                       int64_t n_edges, int L, int F, float* d_sh, float* d_fea, void* stream);

/* ------------------------------------------------------------------------------------------ */
/* Fused attention span of E2AttentionArbOrder_sparse (e2former.py:311-364, 393-422, and the    */
/* sparse aggregation inside E2TensorProductSO2_FirstOrder, so2_tensor_product.py:370-377):      */
/*   s  = <q_i, k_j>          (q already scaled by 1/sqrt(D))                                    */
/*   a  = gate * s;  m_i = max_e a;  x = exp(a - m_i) * poly;  S_i = sum_e x                      */
/*   beta = x * inputhead / (S_i + 1e-3) / max(dist, 1e-6)                                       */
/*   out[i,c,h] = sum_e beta[e,h] * value[j,c,h]                                                 */
/* Edges are in query-CSR order (row_ptr/col; edge id = CSR slot).  gate / inputhead point at    */
/* [E,H] views with row stride ld_gi (the two halves of the radial-MLP output).  row_order (may  */
/* be NULL) is a processing order of the rows (a spatially coherent order improves L2 reuse of   */
/* the gathered value rows); results do not depend on it.  Saves beta [E,H], row_max and row_sum */
/* [N,H] for the backward.  Requires D % 4 == 0, D/4 a power of two <= 32, H dividing 256,      */
/* H % 4 == 0, H*D <= 1024 and (C*H) % 4 == 0.                                                                */
/* ------------------------------------------------------------------------------------------ */
int e2a_attn_fwd(const float* q, const float* k, const float* value,
                 const float* gate, const float* inputhead, int64_t ld_gi,
                 const float* poly, const float* dist,
                 const int32_t* row_ptr, const int32_t* col, const int32_t* row_order,
                 int64_t n_rows, int64_t n_keys, int64_t n_edges, int H, int D, int C,
                 float* out, float* beta, float* row_max, float* row_sum, void* stream);
/* The same forward that also writes the q.k scores s[e,h] (before the gate) to logits [E,H], for   */
/* e2a_attn_bwd_softmax_logits (no reference counterpart: the reference recomputes them in its     */
/* backward).  logits = NULL is e2a_attn_fwd.  Only the H = 128, D = 8, ld_gi % 4 == 0 layout keeps  */
/* them; any other layout with logits != NULL returns E2A_ERR_UNSUPPORTED.                          */
int e2a_attn_fwd_logits(const float* q, const float* k, const float* value,
                        const float* gate, const float* inputhead, int64_t ld_gi,
                        const float* poly, const float* dist,
                        const int32_t* row_ptr, const int32_t* col, const int32_t* row_order,
                        int64_t n_rows, int64_t n_keys, int64_t n_edges, int H, int D, int C,
                        float* out, float* beta, float* row_max, float* row_sum, float* logits,
                        void* stream);
/* Query-side backward: given dout [N,C,H] produces d_q [N,H,D] (w.r.t. the scaled q), d_gate and */
/* d_inputhead ([E,H] views with row stride ld_dgi), d_poly [E], d_dist [E] and d_logit [E,H]     */
/* (= dL/ds, consumed by e2a_attn_bwd_key).  The gradient of the row max follows PyTorch's        */
/* scatter_reduce(amax) rule: shared equally by the tied maxima.  Scratch: a workspace of        */
/* e2a_attn_bwd_workspace_bytes(n_edges, H) bytes.                                               */
size_t e2a_attn_bwd_workspace_bytes(int64_t n_edges, int H);
int e2a_attn_bwd_query(const float* q, const float* k, const float* value,
                       const float* gate, const float* inputhead, int64_t ld_gi,
                       const float* poly, const float* dist,
                       const int32_t* row_ptr, const int32_t* col, const int32_t* row_order,
                       int64_t n_rows, int64_t n_keys, int64_t n_edges, int H, int D, int C,
                       const float* beta, const float* row_max, const float* row_sum, const float* dout,
                       float* d_q, float* d_gate, float* d_inputhead, int64_t ld_dgi,
                       float* d_poly, float* d_dist, float* d_logit,
                       void* workspace, size_t workspace_bytes, void* stream);
/* Key-side backward over the key-CSR (k_row_ptr, k_col = query of each slot, k_perm = edge id):  */
/* d_value[j,c,h] = sum_e beta[e,h] dout[i_e,c,h];  d_k[j,h,:] = sum_e d_logit[e,h] q[i_e,h,:].    */
/* key_order (may be NULL) is a processing order of the key rows, like row_order above.          */
int e2a_attn_bwd_key(const float* q, const float* dout, const float* beta, const float* d_logit,
                     const int32_t* k_row_ptr, const int32_t* k_col, const int32_t* k_perm,
                     const int32_t* key_order, int64_t n_rows, int64_t n_keys, int64_t n_edges,
                     int H, int D, int C, float* d_k, float* d_value, void* stream);

/* The backward as three stages, the first one fused (preferred; e2a_attn_bwd_query + _key remain):   */
/* 1. key side, one pass over the key CSR gathering each destination cotangent row once:               */
/*    d_value[k] = sum_e beta[e] dout[i_e] (sparse_v_agg_edge_index backward, d value) and             */
/*    d_beta[e,h] = <dout[i_e], value[k]>_h (its d alpha).  H must divide 1024 and be <= 128, else       */
/*    E2A_ERR_UNSUPPORTED.                                                                               */
int e2a_attn_bwd_value(const float* value, const float* dout, const float* beta, const int32_t* k_row_ptr,
                       const int32_t* k_col, const int32_t* k_perm, const int32_t* key_order, int64_t n_rows,
                       int64_t n_keys, int64_t n_edges, int H, int D, int C, float* d_value, float* d_beta,
                       void* stream);
/* 2. query side from d_beta: softmax backward (PyTorch amax tie rule) -> d_gate, d_inputhead, d_poly,  */
/*    d_dist, ds = d_logit, and d_q = sum_e ds k.  Workspace: e2a_attn_bwd_softmax_workspace_bytes.      */
size_t e2a_attn_bwd_softmax_workspace_bytes(int64_t n_edges, int H);
int e2a_attn_bwd_softmax(const float* q, const float* k, const float* gate, const float* inputhead, int64_t ld_gi,
                         const float* poly, const float* dist, const int32_t* row_ptr, const int32_t* col,
                         const int32_t* row_order, int64_t n_rows, int64_t n_keys, int64_t n_edges, int H, int D,
                         int C, const float* beta, const float* row_max, const float* row_sum, const float* d_beta,
                         float* d_q, float* d_gate, float* d_inputhead, int64_t ld_dgi, float* d_poly, float* d_dist,
                         float* d_logit, void* workspace, size_t workspace_bytes, void* stream);
/* 2'. stage 2 from the forward's kept logits (e2a_attn_fwd_logits): reads s[e,h] instead of gathering */
/*    k rows for q.k; needs no q and no workspace; results equal e2a_attn_bwd_softmax's bit for bit     */
/*    (same s, same arithmetic).  H = 128, D = 8, ld_gi % 4 == 0, ld_dgi % 4 == 0, else                 */
/*    E2A_ERR_UNSUPPORTED.                                                                               */
int e2a_attn_bwd_softmax_logits(const float* k, const float* gate, const float* inputhead, int64_t ld_gi,
                                const float* poly, const float* dist, const int32_t* row_ptr, const int32_t* col,
                                const int32_t* row_order, int64_t n_rows, int64_t n_keys, int64_t n_edges, int H,
                                int D, int C, const float* beta, const float* row_max, const float* row_sum,
                                const float* logits, const float* d_beta, float* d_q, float* d_gate,
                                float* d_inputhead, int64_t ld_dgi, float* d_poly, float* d_dist, float* d_logit,
                                void* stream);
/* 3. key side: d_k[k] = sum_e ds[e] q[i_e]. */
int e2a_attn_bwd_dk(const float* q, const float* d_logit, const int32_t* k_row_ptr, const int32_t* k_col,
                    const int32_t* k_perm, const int32_t* key_order, int64_t n_rows, int64_t n_keys, int64_t n_edges,
                    int H, int D, int C, float* d_k, void* stream);

/* ------------------------------------------------------------------------------------------ */
/* Dense fp32 projection on tcgen05 tensor cores: C[M,N] = A[M,K] B[N,K]^T (+bias[N]) (+C when  */
/* accumulate != 0); A, B row-major (K contiguous, leading dims lda/ldb >= K), C leading dim     */
/* ldc >= N.  passes = 3 splits every operand into tf32 hi + lo parts and accumulates           */
/* hi*hi + hi*lo + lo*hi (fp32-level accuracy); passes = 1 is plain TF32.  Replaces the         */
/* nn.Linear / einsum products of SO3_Linear_e2former (module_utils.py:2035-2052),              */
/* SO3_Linear2Scalar_e2former (2240-2274), RadialProfile (2151-2178) and forward_linear          */
/* (so2_tensor_product.py:273-290).                                                             */
/* ------------------------------------------------------------------------------------------ */
int e2a_gemm_tf32x3(const float* A, int64_t lda, const float* B, const float* B_lo, int64_t ldb, float* C,
                    int64_t ldc, const float* bias, int64_t M, int64_t N, int64_t K, int accumulate, int passes,
                    void* stream);
/* B_lo != NULL: B holds tf32(B) and B_lo tf32(B - tf32(B)) (e2a_tf32_split; worth it when B, the    */
/* weight operand, is reused); then 16-byte-aligned rows are required, else E2A_ERR_UNSUPPORTED.    */
int e2a_tf32_split(const float* B, int64_t ldb, int64_t N, int64_t K, float* B_hi, float* B_lo, int64_t ldo,
                   void* stream);
/* Pair-product epilogue for SO3_Linear2Scalar_e2former (module_utils.py:2240-2274): B's rows come */
/* interleaved (o1_j, o2_j); P[r, j] = (P[r, j] if accumulate) + o1_j * o2_j with leading dim ldp, */
/* C (may be NULL) receives the raw [M, N] values.  N even, K > 0; 16-byte-aligned A / B rows     */
/* (lda, ldb multiples of 4) required, else E2A_ERR_UNSUPPORTED.  B_lo as for e2a_gemm_tf32x3.     */
int e2a_gemm_tf32x3_pairprod(const float* A, int64_t lda, const float* B, const float* B_lo, int64_t ldb, float* C,
                             int64_t ldc, const float* bias, float* P, int64_t ldp, int64_t M, int64_t N, int64_t K,
                             int accumulate, int passes, void* stream);
/* Backward of the pair product fused into the GEMM (no reference counterpart to a fused form; it      */
/* replaces e2a_pair_grad followed by e2a_gemm_tf32x3 on D, SO3_Linear2Scalar_e2former's backward,      */
/* module_utils.py:2198-2274): C[M,N] = D[M,K] B[N,K]^T with D[r,2j] = G[r,j] O[r,2j+1] and            */
/* D[r,2j+1] = G[r,j] O[r,2j], D formed inside the GEMM from the O and G tiles (D never reaches HBM).  */
/* O rows of K floats (ld ldo), G rows of K/2 floats (ld ldg), B pre-split (B_lo required), K % 32 == 0 */
/* and 16-byte aligned rows; E2A_ERR_UNSUPPORTED otherwise.                                            */
int e2a_gemm_tf32x3_pairgrad(const float* O, int64_t ldo, const float* G, int64_t ldg, const float* B,
                             const float* B_lo, int64_t ldb, float* C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                             int passes, void* stream);
/* Backward of the pair product: D[n,m,2j] = G[n,l(m),j] O[n,m,2j+1], D[n,m,2j+1] = G[n,l(m),j] O[n,m,2j] */
/* for O, D [n_nodes, R, 2h], G [n_nodes, L1, h], l(m) the degree of row m.                      */
int e2a_pair_grad(const float* O, const float* G, int64_t n_nodes, int R, int L1, int h, float* D, void* stream);
/* Node-local map of irreps rows (both halves of the first-order SO(2) product,                   */
/* so2_tensor_product.py:363-385, with A = W_inv diag(CG |pos|) S W precomputed per node):         */
/* out[n,k,c] = sum_s A[n,k,s] h[n,s,c] - sub[n,k,c] (sub may be NULL), A [n, 20, 9]; h / sub / out */
/* rows of C floats with node strides; append_h != 0 also copies h into out rows 20..28.           */
/* Backward: dh[n,s,c] = sum_k A[n,k,s] dout[n,k,c] + dh_add[n,s,c] (dh_add may be NULL),          */
/* dsub = -dout (if dsub != NULL) and dA[n,k,s] = sum_c dout[n,k,c] h[n,s,c] (if dA != NULL).      */
int e2a_node_apply_fwd(const float* A, const float* h, int64_t h_node_stride, const float* sub,
                       int64_t sub_node_stride, int64_t n_nodes, int ko, int ki, int C, float* out,
                       int64_t out_node_stride, int append_h, void* stream);
int e2a_node_apply_bwd(const float* A, const float* h, int64_t h_node_stride, const float* dout,
                       int64_t dout_node_stride, const float* dh_add, int64_t dh_add_node_stride, int64_t n_nodes,
                       int ko, int ki, int C, float* dh, int64_t dh_node_stride, float* dsub, int64_t dsub_node_stride,
                       float* dA, void* stream);
/* Status bits of the GEMM's bounded waits (1 = a wait timed out); copies and optionally clears. */
int e2a_gemm_status(unsigned int* status, int reset, void* stream);
/* Test hook (no reference counterpart): one bounded mbarrier wait on a barrier nothing arrives at,   */
/* giving up after limit_ns (1e3..1e8 ns) and setting the timeout bit that e2a_gemm_status reports.   */
int e2a_gemm_wait_selftest(long long limit_ns, void* stream);

/* ------------------------------------------------------------------------------------------ */
/* Fused row-wise LayerNorm + SiLU of the radial MLP (RadialProfile, module_utils.py:2151-2178), */
/* one warp per row of width W (W % 128 == 0, W <= 1024):                                       */
/*   x = h (+ T[zt[r]] + S[zs[r]] when T != NULL; written to x_out if x_out != NULL),            */
/*   y = SiLU((x - mean) * rstd * gamma + beta), mean / rstd saved per row.                      */
/* The optional tables are the per-element embedding part of fc_easy's first Linear             */
/* (e2former.py:258-266) gathered per edge.  Backward: input gradient only.                      */
/* ------------------------------------------------------------------------------------------ */
int e2a_ln_silu_fwd(const float* h, const float* T, const int64_t* zt, const float* S, const int64_t* zs,
                    const float* gamma, const float* beta, int64_t rows, int W, float eps, float* x_out,
                    float* y, float* mean, float* rstd, void* stream);
int e2a_ln_silu_bwd(const float* x, const float* dy, const float* gamma, const float* beta,
                    const float* mean, const float* rstd, int64_t rows, int W, float* dx, void* stream);

/* Same as e2a_attn_bwd_query, but allocates nothing and takes no workspace.  No counterpart in  */
/* the reference: it serves callers that cannot allocate device memory when they run the        */
/* backward (an operator plugin handed only its tensors, code that must not call cudaMalloc).    */
/* Its scratch is a fixed 8 MiB array in the library's device memory, held by every GPU that     */
/* loads the library until exit; n_edges * H above 2^20 returns E2A_ERR_WORKSPACE.  The first    */
/* call on a device looks up that array's address, so make it before any stream capture.  All   */
/* calls share the array: calls that overlap on the GPU race.                                    */
int e2a_attn_bwd_query_noalloc(const float* q, const float* k, const float* value,
                               const float* gate, const float* inputhead, int64_t ld_gi,
                               const float* poly, const float* dist,
                               const int32_t* row_ptr, const int32_t* col, const int32_t* row_order,
                               int64_t n_rows, int64_t n_keys, int64_t n_edges, int H, int D, int C,
                               const float* beta, const float* row_max, const float* row_sum,
                               const float* dout, float* d_q, float* d_gate, float* d_inputhead,
                               int64_t ld_dgi, float* d_poly, float* d_dist, float* d_logit,
                               void* stream);

/* ------------------------------------------------------------------------------------------ */
/* Node-wise irreps kernels of the transformer block (one warp per node; rows = (lmax+1)^2).    */
/* Equivariant RMS norm, EquivariantRMSNormArraySphericalHarmonicsV2_BL (module_utils.py:      */
/* 1720-1772): f = x with row 0 centred over channels, rstd = (sum_r bw_r mean_c f^2 + eps)^-1/2 */
/* (bw_r = 1/((2l+1)(lmax+1))), y = f rstd w[l(r)] (+ b on row 0); stats [n, 2] = (mean0, rstd). */
/* C % 128 == 0, C <= 256, 16-byte-aligned rows, else E2A_ERR_UNSUPPORTED.                     */
int e2a_rms_norm_fwd(const float* x, int64_t n_nodes, int rows, int C, const float* weight, const float* bias,
                     float eps, float* y, float* stats, void* stream);
int e2a_rms_norm_bwd(const float* x, const float* dy, int64_t n_nodes, int rows, int C, const float* weight,
                     const float* stats, float* dx, void* stream);
/* Gate_s3 (module_utils.py:2694-2745): y[0] = cs silu(s[0]), y[r] = cv sigmoid(s[l(r)]) h[r] for  */
/* r >= 1; s [n, 3, C] is the gate linear of row 0, h / y [n, 9, C].  Backward gives ds and dh   */
/* (dh row 0 = 0).                                                                                 */
int e2a_gate_fwd(const float* s, const float* h, int64_t n_nodes, int rows, int C, float c_scalar, float c_vector,
                 float* y, void* stream);
int e2a_gate_bwd(const float* s, const float* h, const float* dy, int64_t n_nodes, int rows, int C, float c_scalar,
                 float c_vector, float* ds, float* dh, void* stream);

/* Gaussian radial basis formed by its consumer (GaussianSmearing, module_utils.py:1853-1870):     */
/* out[e,k] = exp(coeff (d_e - mu_k)^2); backward d_dist[e] = sum_k grad[e,k] out[e,k] 2 coeff (d_e - mu_k) */
/* with the basis recomputed (nothing stored).                                                      */
int e2a_rbf_fwd(const float* dist, int64_t n_edges, const float* mu, int nb, float coeff, float* out, void* stream);
int e2a_rbf_bwd(const float* dist, const float* grad, int64_t n_edges, const float* mu, int nb, float coeff,
                float* d_dist, void* stream);

/* The radial basis fused into its consumers (GaussianSmearing, module_utils.py:1853-1870; the first   */
/* layer of fc_easy / gbf_projs, e2former.py:134-138, 701-712):                                       */
/* C[M,N] = rbf(dist)[M,K] B[N,K]^T (+ bias), rbf[m,k] = exp(coeff (dist[m] - mu[k])^2) formed on chip */
/* (K <= 256; B / B_lo as in e2a_gemm_tf32x3).                                                        */
int e2a_gemm_tf32x3_rbf(const float* dist, const float* mu, float coeff, const float* B, const float* B_lo,
                        int64_t ldb, float* C, int64_t ldc, const float* bias, int64_t M, int64_t N, int64_t K,
                        int passes, void* stream);
/* The matching distance gradient without the [M, N] basis gradient: G = A[M,K] B[N,K]^T contracted in */
/* the epilogue, partial[m, j] = sum_{n in [64 j, 64 j + 64)} G[m,n] rbf[m,n] 2 coeff (dist[m] - mu[n]); */
/* d(dist)[m] = sum_j partial[m, j] (ld_partial >= ceil(N / 64)).                                     */
int e2a_gemm_tf32x3_rbf_dist_grad(const float* A, int64_t lda, const float* B, const float* B_lo, int64_t ldb,
                                  const float* dist, const float* mu, float coeff, float* partial, int64_t ld_partial,
                                  int64_t M, int64_t N, int64_t K, int passes, void* stream);

/* Per-node map of the first-order SO(2) product from the node position (fp64 inside):            */
/* A[n,k,s] = |p| sum_j Wi^T[k,j] W[sel[j],s] cg[j] with W = blockdiag(D^0, D^1, D^2),                */
/* D^l = J_l Y_l(-beta) J_l Y_l(-alpha) of the position's Euler angles (module_utils.py:182-337),     */
/* Wi = the l3_sequential ((0,1),(1,3),(2,2)) repetition of the blocks (so2_tensor_product.py:341-389); */
/* rows written in row_perm order (NULL = identity).  j1 [3x3], j2 [5x5], sel [20], cg [20],          */
/* row_perm [20] are HOST arrays.  Backward: dpos from dA (angles held constant at the poles and near */
/* the origin, as the reference detaches them).                                                       */
int e2a_node_map_fwd(const float* pos, int64_t n_nodes, const double* j1, const double* j2, const int32_t* sel,
                     const double* cg, const int32_t* row_perm, float* A, void* stream);
int e2a_node_map_bwd(const float* pos, const float* dA, int64_t n_nodes, const double* j1, const double* j2,
                     const int32_t* sel, const double* cg, const int32_t* row_perm, float* dpos, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* E2A_H */
