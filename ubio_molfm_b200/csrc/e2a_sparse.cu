// Kernel-level sparse ops with the reference's Triton-kernel semantics (used directly by callers of
// the reference's kernel API, and as building blocks by the edge-degree embedding).  Every output
// row is produced by one warp or CTA from CSR-ordered inputs: deterministic, atomic-free.
#include "e2a_common.cuh"

// fast paths (e2a_attn.cu): E2A_ERR_UNSUPPORTED outside the layouts they take
namespace e2a_fast {
int agg_ch(const float* X, const float* w, int H, int C, const int32_t* row_ptr, const int32_t* col,
           const int32_t* perm, int64_t n_rows, float* out, cudaStream_t st);
int agg_ch_bf16(const void* X, const float* w, int H, int C, const int32_t* row_ptr, const int32_t* col,
                const int32_t* perm, int64_t n_rows, float* out, cudaStream_t st);
int agg_hd(const float* X, const float* w, int H, int D, const int32_t* row_ptr, const int32_t* col,
           const int32_t* perm, int64_t n_rows, float* out, cudaStream_t st);
int dbeta(const float* value, const float* dout, int H, int C, const int32_t* row_ptr, const int32_t* col,
          const int32_t* perm, int64_t n_rows, float* d_w, cudaStream_t st);
int qk(const float* q, const float* k, int H, int D, const int32_t* row_ptr, const int32_t* col,
       const int32_t* perm, int64_t n_rows, float* out, cudaStream_t st);
}  // namespace e2a_fast

// head-sliced gathers of [H, D] rows (e2a_sliced.cu) for tables too large to stay in L2 in one piece
namespace e2a_sliced {
int agg_hd(const float* X, const float* w, int H, int D, const int32_t* row_ptr, const int32_t* col,
           const int32_t* perm, int64_t n_rows, float* out, cudaStream_t st);
int qk(const float* q, const float* k, int H, int D, const int32_t* row_ptr, const int32_t* col,
       const int32_t* perm, int64_t n_rows, float* out, cudaStream_t st);
}  // namespace e2a_sliced

namespace {

// A gathered [H, D] table larger than this (estimated from the output row count, the callers' row and
// table counts being of one size in this model) is gathered in head slices (e2a_sliced.cu).
constexpr double kSliceAboveBytes = 32.0 * 1048576.0;
bool sliced(int64_t rows, int64_t row_floats) { return (double)rows * (double)row_floats * 4.0 > kSliceAboveBytes; }

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

// out[perm[p],h] = <q[i,h,:], k[col[p],h,:]>  (one warp per CSR slot)
__global__ void k_sparse_qk(const float* __restrict__ q, const float* __restrict__ k,
                            const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col,
                            const int32_t* __restrict__ perm, int64_t n_rows, int H, int D,
                            float* __restrict__ out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t i = blockIdx.x; i < n_rows; i += gridDim.x) {
    const int rs = row_ptr[i], re = row_ptr[i + 1];
    const float* qr = q + i * (int64_t)H * D;
    for (int p = rs + warp; p < re; p += kWarps) {
      const float* kr = k + (int64_t)col[p] * H * D;
      const int64_t e = perm ? perm[p] : p;
      for (int h = lane; h < H; h += 32) {
        float s = 0.f;
        for (int d = 0; d < D; ++d) s = fmaf(qr[h * D + d], kr[h * D + d], s);
        out[e * H + h] = s;
      }
    }
  }
}

// out[r,h,d] = sum_p alpha[perm[p],h] x[col[p],h,d]   (thread per (h,d), CTA per row)
__global__ void k_grouped_reduce(const float* __restrict__ alpha, const float* __restrict__ x,
                                 const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col,
                                 const int32_t* __restrict__ perm, int64_t n_rows, int H, int D,
                                 float* __restrict__ out) {
  const int HD = H * D;
  for (int64_t r = blockIdx.x; r < n_rows; r += gridDim.x) {
    const int rs = row_ptr[r], re = row_ptr[r + 1];
    for (int t = threadIdx.x; t < HD; t += blockDim.x) {
      const int h = t / D;
      float acc = 0.f;
      for (int p = rs; p < re; ++p) {
        const int64_t e = perm ? perm[p] : p;
        acc = fmaf(alpha[e * H + h], x[(int64_t)col[p] * HD + t], acc);
      }
      out[r * HD + t] = acc;
    }
  }
}

__global__ void k_alpha_sum(const float* __restrict__ alpha, const int32_t* __restrict__ row_ptr,
                            const int32_t* __restrict__ perm, int64_t n_rows, int H, float* __restrict__ out) {
  for (int64_t r = blockIdx.x; r < n_rows; r += gridDim.x) {
    const int rs = row_ptr[r], re = row_ptr[r + 1];
    for (int h = threadIdx.x; h < H; h += blockDim.x) {
      float acc = 0.f;
      for (int p = rs; p < re; ++p) acc += alpha[(int64_t)(perm ? perm[p] : p) * H + h];
      out[r * H + h] = acc;
    }
  }
}

// ga[e, 4j..4j+4) = go[qidx[e], 4j..4j+4)  (H % 4 == 0, H / 4 a power of two, 16-byte aligned rows):
// four float4 per thread (index loads, then row loads, then stores: four independent chains in
// flight), the output streamed (evict-first stores).
__global__ void k_broadcast_rows4(const float4* __restrict__ go, const int32_t* __restrict__ qidx, int64_t n4,
                                  int sh, float4* __restrict__ ga) {
  const int64_t t0 = blockIdx.x * (int64_t)blockDim.x * 4 + threadIdx.x;
  int64_t src[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int64_t t = t0 + (int64_t)u * blockDim.x;
    const int64_t e = t >> sh;
    src[u] = t < n4 ? ((int64_t)__ldg(qidx + e) << sh) + (t - (e << sh)) : -1;
  }
  float4 v[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) v[u] = src[u] >= 0 ? __ldg(go + src[u]) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int u = 0; u < 4; ++u)
    if (src[u] >= 0) __stcs(ga + t0 + (int64_t)u * blockDim.x, v[u]);
}

__global__ void k_broadcast_rows(const float* __restrict__ go, const int32_t* __restrict__ qidx, int64_t E, int H,
                                 float* __restrict__ ga) {
  const int64_t n = E * H;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = t / H;
    const int h = (int)(t - e * H);
    ga[t] = go[(int64_t)qidx[e] * H + h];
  }
}

// out[r,c,h] = sum_p alpha[perm[p],h] v[col[p],c,h]   (CTA per row, thread per (c,h))
__global__ void k_v_agg(const float* __restrict__ v, const float* __restrict__ alpha,
                        const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col,
                        const int32_t* __restrict__ perm, int64_t n_rows, int C, int H, float* __restrict__ out) {
  const int CH = C * H;
  for (int64_t r = blockIdx.x; r < n_rows; r += gridDim.x) {
    const int rs = row_ptr[r], re = row_ptr[r + 1];
    for (int t = threadIdx.x; t < CH; t += blockDim.x) {
      const int h = t % H;
      float acc = 0.f;
      for (int p = rs; p < re; ++p) {
        const int64_t e = perm ? perm[p] : p;
        acc = fmaf(alpha[e * H + h], v[(int64_t)col[p] * CH + t], acc);
      }
      out[r * CH + t] = acc;
    }
  }
}

// d_alpha[perm[p],h] = sum_c dout[r,c,h] v[col[p],c,h]   (warp per slot)
__global__ void k_v_agg_dalpha(const float* __restrict__ dout, const float* __restrict__ v,
                               const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col,
                               const int32_t* __restrict__ perm, int64_t n_rows, int C, int H,
                               float* __restrict__ d_alpha) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int CH = C * H;
  for (int64_t r = blockIdx.x; r < n_rows; r += gridDim.x) {
    const int rs = row_ptr[r], re = row_ptr[r + 1];
    for (int p = rs + warp; p < re; p += kWarps) {
      const int64_t e = perm ? perm[p] : p;
      const float* vr = v + (int64_t)col[p] * CH;
      for (int h = lane; h < H; h += 32) {
        float acc = 0.f;
        for (int c = 0; c < C; ++c) acc = fmaf(dout[r * CH + c * H + h], vr[c * H + h], acc);
        d_alpha[e * H + h] = acc;
      }
    }
  }
}

__global__ void k_edge_outer(const float* __restrict__ sh, const float* __restrict__ fea,
                             const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ perm,
                             int64_t n_rows, int L, int F, float* __restrict__ out) {
  const int LF = L * F;
  for (int64_t r = blockIdx.x; r < n_rows; r += gridDim.x) {
    const int rs = row_ptr[r], re = row_ptr[r + 1];
    for (int t = threadIdx.x; t < LF; t += blockDim.x) {
      const int l = t / F, f = t % F;
      float acc = 0.f;
      for (int p = rs; p < re; ++p) {
        const int64_t e = perm ? perm[p] : p;
        acc = fmaf(sh[e * L + l], fea[e * F + f], acc);
      }
      out[r * LF + t] = acc;
    }
  }
}

// d_sh[e,l] = sum_f go[q_e,l,f] fea[e,f]  and  d_fea[e,f] = sum_l go[q_e,l,f] sh[e,l]   (warp per edge)
__global__ void k_edge_outer_bwd(const float* __restrict__ go, const float* __restrict__ sh,
                                 const float* __restrict__ fea, const int32_t* __restrict__ qidx, int64_t E,
                                 int L, int F, float* __restrict__ d_sh, float* __restrict__ d_fea) {
  const int lane = threadIdx.x & 31;
  int64_t e = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (; e < E; e += nw) {
    const float* g = go + (int64_t)qidx[e] * L * F;
    if (d_sh) {
      for (int l = 0; l < L; ++l) {
        float acc = 0.f;
        for (int f = lane; f < F; f += 32) acc = fmaf(g[l * F + f], fea[e * F + f], acc);
        acc = e2a_warp_sum(acc);
        if (lane == 0) d_sh[e * L + l] = acc;
      }
    }
    if (d_fea) {
      for (int f = lane; f < F; f += 32) {
        float acc = 0.f;
        for (int l = 0; l < L; ++l) acc = fmaf(g[l * F + f], sh[e * L + l], acc);
        d_fea[e * F + f] = acc;
      }
    }
  }
}

// Same products, vectorised: one warp per edge, float4 lanes over the F channels (F = 128 FV), the
// destination's L gradient rows read once for both outputs (L, FV compile-time).
template <int L, int FV>
__global__ void __launch_bounds__(256)
k_edge_outer_bwd_v(const float* __restrict__ go, const float* __restrict__ sh, const float* __restrict__ fea,
                   const int32_t* __restrict__ qidx, int64_t E, float* __restrict__ d_sh, float* __restrict__ d_fea) {
  constexpr int F = 128 * FV;
  const int lane = threadIdx.x & 31;
  int64_t e = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (; e < E; e += nw) {
    const float* g = go + (int64_t)qidx[e] * L * F;
    float s[L], ps[L];
#pragma unroll
    for (int l = 0; l < L; ++l) {
      s[l] = d_fea ? __ldg(sh + e * L + l) : 0.f;
      ps[l] = 0.f;
    }
    float4 fv[FV], dv[FV];
#pragma unroll
    for (int j = 0; j < FV; ++j) {
      fv[j] = d_sh ? __ldg(reinterpret_cast<const float4*>(fea + e * F) + lane + 32 * j) : make_float4(0.f, 0.f, 0.f, 0.f);
      dv[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int l = 0; l < L; ++l) {
#pragma unroll
      for (int j = 0; j < FV; ++j) {
        const float4 gv = __ldg(reinterpret_cast<const float4*>(g + l * F) + lane + 32 * j);
        dv[j].x = fmaf(s[l], gv.x, dv[j].x); dv[j].y = fmaf(s[l], gv.y, dv[j].y);
        dv[j].z = fmaf(s[l], gv.z, dv[j].z); dv[j].w = fmaf(s[l], gv.w, dv[j].w);
        ps[l] += (gv.x * fv[j].x + gv.y * fv[j].y) + (gv.z * fv[j].z + gv.w * fv[j].w);
      }
    }
    if (d_fea) {
#pragma unroll
      for (int j = 0; j < FV; ++j) reinterpret_cast<float4*>(d_fea + e * F)[lane + 32 * j] = dv[j];
    }
    if (d_sh) {
#pragma unroll
      for (int l = 0; l < L; ++l) ps[l] = e2a_warp_sum(ps[l]);
      if (lane < L) {
        float v = 0.f;
#pragma unroll
        for (int l = 0; l < L; ++l) v = lane == l ? ps[l] : v;
        d_sh[e * L + lane] = v;
      }
    }
  }
}

int rows_grid(int64_t n) { return (int)(n < (1 << 30) ? (n > 0 ? n : 1) : (1 << 30)); }
int flat_grid(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  if (b > 148 * 32) b = 148 * 32;
  return (int)(b > 0 ? b : 1);
}

}  // namespace

extern "C" {

int e2a_sparse_qk_fwd(const float* q, const float* k, const int32_t* row_ptr, const int32_t* col,
                      const int32_t* perm, int64_t n_rows, int64_t n_edges, int H, int D, float* out, void* stream) {
  if (n_rows < 0 || n_edges < 0 || H <= 0 || D <= 0) return E2A_ERR_ARG;
  if (n_rows == 0 || n_edges == 0) return E2A_OK;
  if (!q || !k || !row_ptr || !col || !out) return E2A_ERR_ARG;
  int rc = sliced(n_rows, (int64_t)H * D)
               ? e2a_sliced::qk(q, k, H, D, row_ptr, col, perm, n_rows, out, (cudaStream_t)stream)
               : E2A_ERR_UNSUPPORTED;
  if (rc == E2A_ERR_UNSUPPORTED) rc = e2a_fast::qk(q, k, H, D, row_ptr, col, perm, n_rows, out, (cudaStream_t)stream);
  if (rc != E2A_ERR_UNSUPPORTED) return rc;
  k_sparse_qk<<<rows_grid(n_rows), kThreads, 0, (cudaStream_t)stream>>>(q, k, row_ptr, col, perm, n_rows, H, D, out);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

int e2a_grouped_reduce(const float* alpha, const float* x, const int32_t* row_ptr, const int32_t* col,
                       const int32_t* perm, int64_t n_rows, int H, int D, float* out, void* stream) {
  if (n_rows < 0 || H <= 0 || D <= 0) return E2A_ERR_ARG;
  if (n_rows == 0) return E2A_OK;
  if (!row_ptr || !out) return E2A_ERR_ARG;
  int rc = sliced(n_rows, (int64_t)H * D)
               ? e2a_sliced::agg_hd(x, alpha, H, D, row_ptr, col, perm, n_rows, out, (cudaStream_t)stream)
               : E2A_ERR_UNSUPPORTED;
  if (rc == E2A_ERR_UNSUPPORTED)
    rc = e2a_fast::agg_hd(x, alpha, H, D, row_ptr, col, perm, n_rows, out, (cudaStream_t)stream);
  if (rc != E2A_ERR_UNSUPPORTED) return rc;
  k_grouped_reduce<<<rows_grid(n_rows), kThreads, 0, (cudaStream_t)stream>>>(alpha, x, row_ptr, col, perm, n_rows,
                                                                              H, D, out);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

int e2a_alpha_sum_fwd(const float* alpha, const int32_t* row_ptr, const int32_t* perm, int64_t n_rows, int H,
                      float* out, void* stream) {
  if (n_rows < 0 || H <= 0) return E2A_ERR_ARG;
  if (n_rows == 0) return E2A_OK;
  if (!row_ptr || !out) return E2A_ERR_ARG;
  k_alpha_sum<<<rows_grid(n_rows), 128, 0, (cudaStream_t)stream>>>(alpha, row_ptr, perm, n_rows, H, out);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

int e2a_alpha_sum_bwd(const float* grad_out, const int32_t* query_idx, int64_t n_edges, int H, float* grad_alpha,
                      void* stream) {
  if (n_edges < 0 || H <= 0) return E2A_ERR_ARG;
  if (n_edges == 0) return E2A_OK;
  if (!grad_out || !query_idx || !grad_alpha) return E2A_ERR_ARG;
  const int H4 = H / 4;
  if (H % 4 == 0 && (H4 & (H4 - 1)) == 0 && ((uintptr_t)grad_out & 15u) == 0 && ((uintptr_t)grad_alpha & 15u) == 0 &&
      (n_edges * H4 + 1023) / 1024 <= INT32_MAX) {
    int sh = 0;
    while ((1 << sh) < H4) ++sh;
    const int64_t n4 = n_edges * H4;
    k_broadcast_rows4<<<(int)((n4 + 1023) / 1024), 256, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const float4*>(grad_out), query_idx, n4, sh, reinterpret_cast<float4*>(grad_alpha));
    E2A_CHECK_LAUNCH();
    return E2A_OK;
  }
  k_broadcast_rows<<<flat_grid(n_edges * H, 256), 256, 0, (cudaStream_t)stream>>>(grad_out, query_idx, n_edges, H,
                                                                                 grad_alpha);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

int e2a_v_agg_fwd(const float* value, const float* alpha, const int32_t* row_ptr, const int32_t* col,
                  const int32_t* perm, int64_t n_rows, int C, int H, float* out, void* stream) {
  if (n_rows < 0 || C <= 0 || H <= 0) return E2A_ERR_ARG;
  if (n_rows == 0) return E2A_OK;
  if (!row_ptr || !out) return E2A_ERR_ARG;
  const int rc = e2a_fast::agg_ch(value, alpha, H, C, row_ptr, col, perm, n_rows, out, (cudaStream_t)stream);
  if (rc != E2A_ERR_UNSUPPORTED) return rc;
  k_v_agg<<<rows_grid(n_rows), kThreads, 0, (cudaStream_t)stream>>>(value, alpha, row_ptr, col, perm, n_rows, C, H,
                                                                     out);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

int e2a_v_agg_fwd_bf16(const void* value, const float* alpha, const int32_t* row_ptr, const int32_t* col,
                       const int32_t* perm, int64_t n_rows, int C, int H, float* out, void* stream) {
  if (n_rows < 0 || C <= 0 || H <= 0) return E2A_ERR_ARG;
  if (n_rows == 0) return E2A_OK;
  if (!row_ptr || !out || !value || !alpha || !col) return E2A_ERR_ARG;
  return e2a_fast::agg_ch_bf16(value, alpha, H, C, row_ptr, col, perm, n_rows, out, (cudaStream_t)stream);
}

int e2a_v_agg_bwd_alpha(const float* dout, const float* value, const int32_t* row_ptr, const int32_t* col,
                        const int32_t* perm, int64_t n_rows, int C, int H, float* d_alpha, void* stream) {
  if (n_rows < 0 || C <= 0 || H <= 0) return E2A_ERR_ARG;
  if (n_rows == 0) return E2A_OK;
  if (!row_ptr || !dout) return E2A_ERR_ARG;
  const int rc = e2a_fast::dbeta(value, dout, H, C, row_ptr, col, perm, n_rows, d_alpha, (cudaStream_t)stream);
  if (rc != E2A_ERR_UNSUPPORTED) return rc;
  k_v_agg_dalpha<<<rows_grid(n_rows), kThreads, 0, (cudaStream_t)stream>>>(dout, value, row_ptr, col, perm, n_rows,
                                                                            C, H, d_alpha);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

int e2a_v_agg_bwd_value(const float* alpha, const float* dout, const int32_t* k_row_ptr, const int32_t* k_col,
                        const int32_t* k_perm, int64_t n_keys, int C, int H, float* d_value, void* stream) {
  // same contraction as the forward with the roles of the two CSR orientations swapped
  return e2a_v_agg_fwd(dout, alpha, k_row_ptr, k_col, k_perm, n_keys, C, H, d_value, stream);
}

int e2a_edge_outer_fwd(const float* sh, const float* fea, const int32_t* row_ptr, const int32_t* perm,
                       int64_t n_rows, int L, int F, float* out, void* stream) {
  if (n_rows < 0 || L <= 0 || F <= 0) return E2A_ERR_ARG;
  if (n_rows == 0) return E2A_OK;
  if (!row_ptr || !out) return E2A_ERR_ARG;
  k_edge_outer<<<rows_grid(n_rows), kThreads, 0, (cudaStream_t)stream>>>(sh, fea, row_ptr, perm, n_rows, L, F, out);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

int e2a_edge_outer_bwd(const float* grad_out, const float* sh, const float* fea, const int32_t* query_idx,
                       int64_t n_edges, int L, int F, float* d_sh, float* d_fea, void* stream) {
  if (n_edges < 0 || L <= 0 || F <= 0) return E2A_ERR_ARG;
  if (n_edges == 0) return E2A_OK;
  if (!grad_out || !query_idx || (d_sh && !fea) || (d_fea && !sh)) return E2A_ERR_ARG;
  const bool al = ((reinterpret_cast<uintptr_t>(grad_out) | reinterpret_cast<uintptr_t>(fea) |
                    reinterpret_cast<uintptr_t>(d_fea)) & 15u) == 0;
  const int grid = flat_grid(n_edges * 32, 256);
  cudaStream_t st = (cudaStream_t)stream;
#define E2A_EO_BWD(LL, FVV) k_edge_outer_bwd_v<LL, FVV><<<grid, 256, 0, st>>>(grad_out, sh, fea, query_idx, n_edges, d_sh, d_fea)
  if (al && (F == 128 || F == 256) && (L == 1 || L == 3 || L == 5)) {
    const int fv = F / 128;
    if (L == 1) { if (fv == 1) E2A_EO_BWD(1, 1); else E2A_EO_BWD(1, 2); }
    else if (L == 3) { if (fv == 1) E2A_EO_BWD(3, 1); else E2A_EO_BWD(3, 2); }
    else { if (fv == 1) E2A_EO_BWD(5, 1); else E2A_EO_BWD(5, 2); }
  } else {
    k_edge_outer_bwd<<<grid, 256, 0, st>>>(grad_out, sh, fea, query_idx, n_edges, L, F, d_sh, d_fea);
  }
#undef E2A_EO_BWD
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

}  // extern "C"
