// Fused row-wise pieces of the edge radial MLP (RadialProfile, module_utils.py:2151-2178, used by
// fc_easy in e2former.py:134-138, 301-306):
//
//   forward   y = SiLU(LayerNorm(x)),  x = h (+ T[zt[e]] + S[zs[e]])     one warp per row
//   backward  dx = d/dx of the same map (input gradient; gamma / beta / tables treated as constants)
//
// The optional table terms are the exact decomposition of the first Linear over the concatenated
// [rbf, target_embedding(Z_i), source_embedding(Z_j)] input: the embedding parts are per-element
// tables gathered per edge instead of an [E, nb + 256] concatenation.  Each row (width W, W % 128
// == 0 and W <= 1024) is held in registers (W/32 floats per lane); mean / rstd are saved for the
// backward, which recomputes the normalised row.  LayerNorm eps and the two-pass variance match
// torch.nn.LayerNorm (biased variance, eps = 1e-5).
#include "e2a_common.cuh"

namespace {

constexpr int kWarpsPerBlock = 8;

__device__ __forceinline__ float silu(float z) { return z / (1.f + expf(-z)); }

template <int V>  // V = W / 128 float4 per lane
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
k_ln_silu_fwd(const float* __restrict__ h, const float* __restrict__ T, const int64_t* __restrict__ zt,
              const float* __restrict__ S, const int64_t* __restrict__ zs, const float* __restrict__ gamma,
              const float* __restrict__ beta, int64_t rows, int W, float eps, float* __restrict__ x_out,
              float* __restrict__ y, float* __restrict__ mean_out, float* __restrict__ rstd_out) {
  const int lane = threadIdx.x & 31;
  int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  // the next row's input is loaded before this row's reductions (one more row of loads in flight)
  float4 nxt[V];
  if (r < rows) {
#pragma unroll
    for (int i = 0; i < V; ++i) nxt[i] = ldg4(h + r * W + 4 * (lane + 32 * i));
  }
  for (; r < rows; r += nw) {
    float4 v[V];
#pragma unroll
    for (int i = 0; i < V; ++i) v[i] = nxt[i];
    if (r + nw < rows) {
#pragma unroll
      for (int i = 0; i < V; ++i) nxt[i] = ldg4(h + (r + nw) * W + 4 * (lane + 32 * i));
    }
    if (T) {
      const float* tr = T + zt[r] * W;
      const float* sr = S + zs[r] * W;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const float4 a = ldg4(tr + 4 * (lane + 32 * i)), b = ldg4(sr + 4 * (lane + 32 * i));
        v[i].x += a.x + b.x; v[i].y += a.y + b.y; v[i].z += a.z + b.z; v[i].w += a.w + b.w;
      }
      if (x_out) {
#pragma unroll
        for (int i = 0; i < V; ++i) reinterpret_cast<float4*>(x_out + r * W)[lane + 32 * i] = v[i];
      }
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    const float mean = e2a_warp_sum(s) / W;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
      q += (a * a + b * b) + (c * c + d * d);
    }
    const float rstd = rsqrtf(e2a_warp_sum(q) / W + eps);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int c = 4 * (lane + 32 * i);
      const float4 g = ldg4(gamma + c), b = ldg4(beta + c);
      float4 o;
      o.x = silu((v[i].x - mean) * rstd * g.x + b.x);
      o.y = silu((v[i].y - mean) * rstd * g.y + b.y);
      o.z = silu((v[i].z - mean) * rstd * g.z + b.z);
      o.w = silu((v[i].w - mean) * rstd * g.w + b.w);
      reinterpret_cast<float4*>(y + r * W)[lane + 32 * i] = o;
    }
    if (lane == 0) {
      mean_out[r] = mean;
      rstd_out[r] = rstd;
    }
  }
}

template <int V>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
k_ln_silu_bwd(const float* __restrict__ x, const float* __restrict__ dy, const float* __restrict__ gamma,
              const float* __restrict__ beta, const float* __restrict__ mean_in, const float* __restrict__ rstd_in,
              int64_t rows, int W, float* __restrict__ dx) {
  const int lane = threadIdx.x & 31;
  int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  // the next row's operands are loaded before this row's reductions (one more row of loads in flight)
  float4 nx[V], nd[V];
  float nmean = 0.f, nrstd = 0.f;
  if (r < rows) {
#pragma unroll
    for (int i = 0; i < V; ++i) {
      nx[i] = ldg4(x + r * W + 4 * (lane + 32 * i));
      nd[i] = ldg4(dy + r * W + 4 * (lane + 32 * i));
    }
    nmean = mean_in[r];
    nrstd = rstd_in[r];
  }
  for (; r < rows; r += nw) {
    const float mean = nmean, rstd = nrstd;
    float4 cx[V], cd[V];
#pragma unroll
    for (int i = 0; i < V; ++i) { cx[i] = nx[i]; cd[i] = nd[i]; }
    if (r + nw < rows) {
#pragma unroll
      for (int i = 0; i < V; ++i) {
        nx[i] = ldg4(x + (r + nw) * W + 4 * (lane + 32 * i));
        nd[i] = ldg4(dy + (r + nw) * W + 4 * (lane + 32 * i));
      }
      nmean = mean_in[r + nw];
      nrstd = rstd_in[r + nw];
    }
    float4 xh[V], g[V];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int c = 4 * (lane + 32 * i);
      const float4 xv = cx[i], d = cd[i];
      const float4 ga = ldg4(gamma + c), be = ldg4(beta + c);
      const float xs[4] = {xv.x, xv.y, xv.z, xv.w}, ds[4] = {d.x, d.y, d.z, d.w};
      const float gs[4] = {ga.x, ga.y, ga.z, ga.w}, bs[4] = {be.x, be.y, be.z, be.w};
      float hs[4], gg[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float xn = (xs[t] - mean) * rstd;
        const float z = xn * gs[t] + bs[t];
        const float sg = 1.f / (1.f + expf(-z));
        const float dz = ds[t] * sg * (1.f + z * (1.f - sg));  // d SiLU
        const float dxn = dz * gs[t];
        hs[t] = xn;
        gg[t] = dxn;
        s1 += dxn;
        s2 += dxn * xn;
      }
      xh[i] = make_float4(hs[0], hs[1], hs[2], hs[3]);
      g[i] = make_float4(gg[0], gg[1], gg[2], gg[3]);
    }
    s1 = e2a_warp_sum(s1) / W;
    s2 = e2a_warp_sum(s2) / W;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      float4 o;
      o.x = rstd * (g[i].x - s1 - xh[i].x * s2);
      o.y = rstd * (g[i].y - s1 - xh[i].y * s2);
      o.z = rstd * (g[i].z - s1 - xh[i].z * s2);
      o.w = rstd * (g[i].w - s1 - xh[i].w * s2);
      reinterpret_cast<float4*>(dx + r * W)[lane + 32 * i] = o;
    }
  }
}

int grid_rows(int64_t rows) {
  int64_t b = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
  if (b > 148 * 64) b = 148 * 64;
  return (int)(b > 0 ? b : 1);
}

// D[n, m, 2j] = G[n, l(m), j] * O[n, m, 2j+1];  D[n, m, 2j+1] = G[n, l(m), j] * O[n, m, 2j]
__global__ void k_pair_grad(const float* __restrict__ O, const float* __restrict__ G, int64_t n_nodes, int R,
                            int L1, int h, float* __restrict__ D) {
  const int64_t total = n_nodes * R * (int64_t)(h / 2);  // float4 units of O / D
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j2 = t % (h / 2);           // pair of pairs: j = 2*j2, 2*j2+1
    const int64_t nm = t / (h / 2);
    const int m = (int)(nm % R);
    const int64_t n = nm / R;
    int l = 0;
    while ((l + 1) * (l + 1) <= m) ++l;
    const float4 o = ldg4(O + nm * (2 * h) + 4 * j2);
    const float2 g = __ldg(reinterpret_cast<const float2*>(G + (n * L1 + l) * h + 2 * j2));
    reinterpret_cast<float4*>(D + nm * (2 * h))[j2] = make_float4(g.x * o.y, g.x * o.x, g.y * o.w, g.y * o.z);
  }
}

}  // namespace

extern "C" {

int e2a_pair_grad(const float* O, const float* G, int64_t n_nodes, int R, int L1, int h, float* D, void* stream) {
  if (n_nodes < 0 || R <= 0 || L1 <= 0 || h <= 0 || (h & 1) || R > L1 * L1) return E2A_ERR_ARG;
  if (n_nodes == 0) return E2A_OK;
  if (!O || !G || !D) return E2A_ERR_ARG;
  const int64_t total = n_nodes * R * (int64_t)(h / 2);
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  k_pair_grad<<<(int)blocks, 256, 0, (cudaStream_t)stream>>>(O, G, n_nodes, R, L1, h, D);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

int e2a_ln_silu_fwd(const float* h, const float* T, const int64_t* zt, const float* S, const int64_t* zs,
                    const float* gamma, const float* beta, int64_t rows, int W, float eps, float* x_out, float* y,
                    float* mean, float* rstd, void* stream) {
  if (rows < 0 || W <= 0 || W % 128 || W > 1024) return rows < 0 || W <= 0 ? E2A_ERR_ARG : E2A_ERR_UNSUPPORTED;
  if (rows == 0) return E2A_OK;
  if (!h || !gamma || !beta || !y || !mean || !rstd || (T && (!zt || !S || !zs))) return E2A_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const int g = grid_rows(rows), b = kWarpsPerBlock * 32;
  switch (W / 128) {
    case 1: k_ln_silu_fwd<1><<<g, b, 0, st>>>(h, T, zt, S, zs, gamma, beta, rows, W, eps, x_out, y, mean, rstd); break;
    case 2: k_ln_silu_fwd<2><<<g, b, 0, st>>>(h, T, zt, S, zs, gamma, beta, rows, W, eps, x_out, y, mean, rstd); break;
    case 4: k_ln_silu_fwd<4><<<g, b, 0, st>>>(h, T, zt, S, zs, gamma, beta, rows, W, eps, x_out, y, mean, rstd); break;
    case 8: k_ln_silu_fwd<8><<<g, b, 0, st>>>(h, T, zt, S, zs, gamma, beta, rows, W, eps, x_out, y, mean, rstd); break;
    default: return E2A_ERR_UNSUPPORTED;
  }
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

int e2a_ln_silu_bwd(const float* x, const float* dy, const float* gamma, const float* beta, const float* mean,
                    const float* rstd, int64_t rows, int W, float* dx, void* stream) {
  if (rows < 0 || W <= 0 || W % 128 || W > 1024) return rows < 0 || W <= 0 ? E2A_ERR_ARG : E2A_ERR_UNSUPPORTED;
  if (rows == 0) return E2A_OK;
  if (!x || !dy || !gamma || !beta || !mean || !rstd || !dx) return E2A_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const int g = grid_rows(rows), b = kWarpsPerBlock * 32;
  switch (W / 128) {
    case 1: k_ln_silu_bwd<1><<<g, b, 0, st>>>(x, dy, gamma, beta, mean, rstd, rows, W, dx); break;
    case 2: k_ln_silu_bwd<2><<<g, b, 0, st>>>(x, dy, gamma, beta, mean, rstd, rows, W, dx); break;
    case 4: k_ln_silu_bwd<4><<<g, b, 0, st>>>(x, dy, gamma, beta, mean, rstd, rows, W, dx); break;
    case 8: k_ln_silu_bwd<8><<<g, b, 0, st>>>(x, dy, gamma, beta, mean, rstd, rows, W, dx); break;
    default: return E2A_ERR_UNSUPPORTED;
  }
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------
// Node-local linear map of irreps rows: out[n, k, c] = sum_s A[n, k, s] h[n, s, c]  (A: [n, KO, KI]),
// used for both halves of the first-order SO(2) tensor product (so2_tensor_product.py:363-385) with
// A = W_inv diag(CG |pos|) S W.  One CTA per node, one thread per channel (coalesced rows).
// Backward: dh = A^T dout, dA[n,k,s] = sum_c dout[n,k,c] h[n,s,c].
// ------------------------------------------------------------------------------------------------
namespace {
// fixed shape of the first-order SO(2) product: 20 output rows from 9 input rows
constexpr int KO = 20, KI = 9;

__global__ void __launch_bounds__(256)
k_node_apply_fwd(const float* __restrict__ A, const float* __restrict__ h, int64_t h_node_stride,
                 const float* __restrict__ sub, int64_t sub_node_stride, int64_t n_nodes, int C,
                 float* __restrict__ out, int64_t out_node_stride, int append_h) {
  __shared__ float As[KO * KI];
  for (int64_t n = blockIdx.x; n < n_nodes; n += gridDim.x) {
    __syncthreads();
    for (int t = threadIdx.x; t < KO * KI; t += blockDim.x) As[t] = A[n * KO * KI + t];
    __syncthreads();
    const float* hn = h + n * h_node_stride;
    float* on = out + n * out_node_stride;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
      float hv[KI];
#pragma unroll
      for (int s = 0; s < KI; ++s) hv[s] = __ldg(hn + (int64_t)s * C + c);
#pragma unroll
      for (int k = 0; k < KO; ++k) {
        float acc = 0.f;
#pragma unroll
        for (int s = 0; s < KI; ++s) acc = fmaf(As[k * KI + s], hv[s], acc);
        if (sub) acc -= __ldg(sub + n * sub_node_stride + (int64_t)k * C + c);
        on[(int64_t)k * C + c] = acc;
      }
      if (append_h) {
#pragma unroll
        for (int s = 0; s < KI; ++s) on[(int64_t)(KO + s) * C + c] = hv[s];
      }
    }
  }
}

// One CTA per node: dh[s,c] = sum_k A[k,s] dout[k,c] (+ dh_add[s,c]) with one thread per channel,
// dsub = -dout, and dA[k,s] with one warp per output row k (lanes over channels, 9 warp sums per k,
// fixed order).  The node's rows are read straight from global memory (they stay in L1 across the
// two loops).
__global__ void __launch_bounds__(256)
k_node_apply_bwd(const float* __restrict__ A, const float* __restrict__ h, int64_t h_node_stride,
                 const float* __restrict__ dout, int64_t dout_node_stride, const float* __restrict__ dh_add,
                 int64_t dh_add_node_stride, int64_t n_nodes, int C, float* __restrict__ dh, int64_t dh_node_stride,
                 float* __restrict__ dsub, int64_t dsub_node_stride, float* __restrict__ dA) {
  __shared__ float As[KO * KI];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarp = blockDim.x >> 5;
  for (int64_t n = blockIdx.x; n < n_nodes; n += gridDim.x) {
    __syncthreads();
    for (int t = threadIdx.x; t < KO * KI; t += blockDim.x) As[t] = A[n * KO * KI + t];
    __syncthreads();
    const float* hn = h + n * h_node_stride;
    const float* gn = dout + n * dout_node_stride;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
      float dv[KI];
#pragma unroll
      for (int s = 0; s < KI; ++s) dv[s] = dh_add ? __ldg(dh_add + n * dh_add_node_stride + (int64_t)s * C + c) : 0.f;
#pragma unroll
      for (int k = 0; k < KO; ++k) {
        const float g = __ldg(gn + (int64_t)k * C + c);
        if (dsub) dsub[n * dsub_node_stride + (int64_t)k * C + c] = -g;
#pragma unroll
        for (int s = 0; s < KI; ++s) dv[s] = fmaf(As[k * KI + s], g, dv[s]);
      }
#pragma unroll
      for (int s = 0; s < KI; ++s) dh[n * dh_node_stride + (int64_t)s * C + c] = dv[s];
    }
    if (dA) {
      for (int k = warp; k < KO; k += nwarp) {
        float p[KI];
#pragma unroll
        for (int s = 0; s < KI; ++s) p[s] = 0.f;
        for (int c = lane; c < C; c += 32) {
          const float g = __ldg(gn + (int64_t)k * C + c);
#pragma unroll
          for (int s = 0; s < KI; ++s) p[s] = fmaf(g, __ldg(hn + (int64_t)s * C + c), p[s]);
        }
#pragma unroll
        for (int s = 0; s < KI; ++s) p[s] = e2a_warp_sum(p[s]);
        if (lane == 0) {
#pragma unroll
          for (int s = 0; s < KI; ++s) dA[n * KO * KI + k * KI + s] = p[s];
        }
      }
    }
  }
}

// Butterfly reduce-scatter of 36 per-lane partials over the warp: 37 shuffles instead of 36 x 5.
// On return lane holds in v[0..1] the full sums of the indices given by rs36_index.
__device__ __forceinline__ void rs36(float (&v)[36], int lane) {
#define E2A_RS_STEP(H, W)                                              \
  {                                                                    \
    const bool up = (lane & (W)) != 0;                                 \
    _Pragma("unroll") for (int i = 0; i < (H); ++i) {                  \
      const float send = up ? v[i] : v[i + (H)];                       \
      const float keep = up ? v[i + (H)] : v[i];                       \
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, (W));           \
    }                                                                  \
  }
  E2A_RS_STEP(18, 16)
  E2A_RS_STEP(9, 8)
  v[9] = 0.f;
  E2A_RS_STEP(5, 4)
  v[5] = 0.f;
  E2A_RS_STEP(3, 2)
  v[3] = 0.f;
  E2A_RS_STEP(2, 1)
#undef E2A_RS_STEP
}
// index (0..35) of this lane's v[j] after rs36, or -1 for a padding slot
__device__ __forceinline__ int rs36_index(int lane, int j) {
  int p = j + ((lane & 1) ? 2 : 0);
  if (p >= 3) return -1;
  p += (lane & 2) ? 3 : 0;
  if (p >= 5) return -1;
  p += (lane & 4) ? 5 : 0;
  if (p >= 9) return -1;
  p += (lane & 8) ? 9 : 0;
  return p + ((lane & 16) ? 18 : 0);
}

// Vectorised backward, one warp per node, lanes over float4 channel groups (C % 128 == 0, rows
// 16-byte aligned): dh (+ dh_add) = A^T dout with A from shared memory, dsub = -dout, and
// dA[k,s] = <dout[k,:], h[s,:]> accumulated per lane for four k rows at a time and summed across
// the warp by one reduce-scatter per group.
__global__ void __launch_bounds__(256, 2)
k_node_apply_bwd_warp(const float* __restrict__ A, const float* __restrict__ h, int64_t h_node_stride,
                      const float* __restrict__ dout, int64_t dout_node_stride, const float* __restrict__ dh_add,
                      int64_t dh_add_node_stride, int64_t n_nodes, int C, float* __restrict__ dh,
                      int64_t dh_node_stride, float* __restrict__ dsub, int64_t dsub_node_stride,
                      float* __restrict__ dA) {
  __shared__ float As[8][KO * KI];
  __shared__ float dAs[8][KO * KI];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int64_t n = (int64_t)blockIdx.x * 8 + w; n < n_nodes; n += (int64_t)gridDim.x * 8) {
    for (int t = lane; t < KO * KI; t += 32) {
      As[w][t] = A[n * KO * KI + t];
      dAs[w][t] = 0.f;
    }
    __syncwarp();
    const float* hn = h + n * h_node_stride;
    const float* gn = dout + n * dout_node_stride;
    for (int c = 4 * lane; c < C; c += 128) {
      float4 hv[KI], dv[KI];
#pragma unroll
      for (int s = 0; s < KI; ++s) {
        hv[s] = __ldg(reinterpret_cast<const float4*>(hn + (int64_t)s * C + c));
        dv[s] = dh_add ? __ldg(reinterpret_cast<const float4*>(dh_add + n * dh_add_node_stride + (int64_t)s * C + c))
                       : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll 1
      for (int kg = 0; kg < KO / 4; ++kg) {
        float p[36];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const int k = 4 * kg + kk;
          const float4 g = __ldg(reinterpret_cast<const float4*>(gn + (int64_t)k * C + c));
          if (dsub)
            *reinterpret_cast<float4*>(dsub + n * dsub_node_stride + (int64_t)k * C + c) =
                make_float4(-g.x, -g.y, -g.z, -g.w);
#pragma unroll
          for (int s = 0; s < KI; ++s) {
            const float a = As[w][k * KI + s];
            dv[s].x = fmaf(a, g.x, dv[s].x); dv[s].y = fmaf(a, g.y, dv[s].y);
            dv[s].z = fmaf(a, g.z, dv[s].z); dv[s].w = fmaf(a, g.w, dv[s].w);
            p[kk * KI + s] = g.x * hv[s].x + g.y * hv[s].y + g.z * hv[s].z + g.w * hv[s].w;
          }
        }
        if (dA) {
          rs36(p, lane);
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int idx = rs36_index(lane, j);
            if (idx >= 0) dAs[w][(4 * kg) * KI + idx] += p[j];
          }
        }
      }
#pragma unroll
      for (int s = 0; s < KI; ++s) *reinterpret_cast<float4*>(dh + n * dh_node_stride + (int64_t)s * C + c) = dv[s];
    }
    __syncwarp();
    if (dA)
      for (int t = lane; t < KO * KI; t += 32) dA[n * KO * KI + t] = dAs[w][t];
    __syncwarp();
  }
}
}  // namespace

extern "C" {

int e2a_node_apply_fwd(const float* A, const float* h, int64_t h_node_stride, const float* sub,
                       int64_t sub_node_stride, int64_t n_nodes, int ko, int ki, int C, float* out,
                       int64_t out_node_stride, int append_h, void* stream) {
  if (n_nodes < 0 || C <= 0) return E2A_ERR_ARG;
  if (ko != KO || ki != KI) return E2A_ERR_UNSUPPORTED;
  if (n_nodes == 0) return E2A_OK;
  if (!A || !h || !out || h_node_stride < (int64_t)KI * C ||
      out_node_stride < (int64_t)(append_h ? KO + KI : KO) * C || (sub && sub_node_stride < (int64_t)KO * C))
    return E2A_ERR_ARG;
  const int64_t g = n_nodes < (1 << 30) ? n_nodes : (1 << 30);
  k_node_apply_fwd<<<(int)g, 256, 0, (cudaStream_t)stream>>>(A, h, h_node_stride, sub, sub_node_stride, n_nodes, C,
                                                             out, out_node_stride, append_h ? 1 : 0);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

int e2a_node_apply_bwd(const float* A, const float* h, int64_t h_node_stride, const float* dout,
                       int64_t dout_node_stride, const float* dh_add, int64_t dh_add_node_stride, int64_t n_nodes,
                       int ko, int ki, int C, float* dh, int64_t dh_node_stride, float* dsub, int64_t dsub_node_stride,
                       float* dA, void* stream) {
  if (n_nodes < 0 || C <= 0) return E2A_ERR_ARG;
  if (ko != KO || ki != KI) return E2A_ERR_UNSUPPORTED;
  if (n_nodes == 0) return E2A_OK;
  if (!A || !h || !dout || !dh || dh_node_stride < (int64_t)KI * C || (dsub && dsub_node_stride < (int64_t)KO * C))
    return E2A_ERR_ARG;
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (C % 128 == 0 && h_node_stride % 4 == 0 && dout_node_stride % 4 == 0 && dh_node_stride % 4 == 0 &&
      (!dh_add || dh_add_node_stride % 4 == 0) && (!dsub || dsub_node_stride % 4 == 0) && al(h) && al(dout) &&
      al(dh) && al(dh_add) && al(dsub)) {
    const int64_t blocks = (n_nodes + 7) / 8 < 148 * 16 ? (n_nodes + 7) / 8 : 148 * 16;
    k_node_apply_bwd_warp<<<(int)blocks, 256, 0, (cudaStream_t)stream>>>(A, h, h_node_stride, dout, dout_node_stride,
                                                                         dh_add, dh_add_node_stride, n_nodes, C, dh,
                                                                         dh_node_stride, dsub, dsub_node_stride, dA);
    E2A_CHECK_LAUNCH();
    return E2A_OK;
  }
  const int64_t g = n_nodes < (1 << 30) ? n_nodes : (1 << 30);
  k_node_apply_bwd<<<(int)g, 256, 0, (cudaStream_t)stream>>>(A, h, h_node_stride, dout, dout_node_stride, dh_add,
                                                             dh_add_node_stride, n_nodes, C, dh, dh_node_stride,
                                                             dsub, dsub_node_stride, dA);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

}  // extern "C"
