// Node-wise irreps kernels of the E2Former-V2 block: the equivariant RMS norm and the gated
// activation of the feed-forward network, forward and backward, one warp per node with float4
// lanes over the channels (memory bound: each node's [R, C] rows are read and written once).
//
//  * e2a_rms_norm_fwd / _bwd -- EquivariantRMSNormArraySphericalHarmonicsV2_BL (module_utils.py:
//    1720-1772; component normalisation, degree-balanced, centred, affine):
//      f = x with the l=0 row centred over channels,
//      rstd = (sum_r bw_r mean_c f[r,c]^2 + eps)^-1/2,  bw_r = 1 / ((2 l(r) + 1)(lmax + 1)),
//      y[r,c] = f[r,c] rstd w[l(r),c]  (+ b[c] on r = 0).
//  * e2a_gate_fwd / _bwd -- Gate_s3 (module_utils.py:2694-2745):
//      y[0,c] = cs silu(s[c]),  y[r,c] = cv sigmoid(s[l(r) C + c]) h[r,c]  (r >= 1),
//    s = the gate linear of the l=0 row, [lmax+1, C] per node; cs, cv the normalising constants.
#include "e2a_common.cuh"

namespace {

constexpr int kNodeThreads = 256;
constexpr int kMaxRows = 9;       // lmax <= 2

__device__ __forceinline__ int degree_of_row(int r) { return r == 0 ? 0 : (r < 4 ? 1 : 2); }

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }

// CPR = float4 groups per lane per row (C = 128 * CPR)
template <int CPR>
__global__ void __launch_bounds__(kNodeThreads)
k_rms_norm_fwd(const float* __restrict__ x, int64_t n, int R, int lmax, const float* __restrict__ w,
               const float* __restrict__ b, float eps, float* __restrict__ y, float* __restrict__ stats) {
  constexpr int C = 128 * CPR;
  const int lane = threadIdx.x & 31;
  const int64_t node = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (node >= n) return;
  const float* xn = x + node * R * C;
  float4 v[kMaxRows][CPR];
#pragma unroll
  for (int r = 0; r < kMaxRows; ++r)
    if (r < R)
#pragma unroll
      for (int j = 0; j < CPR; ++j) v[r][j] = ld4(xn + r * C + 4 * (lane + 32 * j));
  float s0 = 0.f;
#pragma unroll
  for (int j = 0; j < CPR; ++j) s0 += (v[0][j].x + v[0][j].y) + (v[0][j].z + v[0][j].w);
  const float mean0 = e2a_warp_sum(s0) / C;
#pragma unroll
  for (int j = 0; j < CPR; ++j) {
    v[0][j].x -= mean0; v[0][j].y -= mean0; v[0][j].z -= mean0; v[0][j].w -= mean0;
  }
  float ss = 0.f;
#pragma unroll
  for (int r = 0; r < kMaxRows; ++r) {
    if (r >= R) continue;
    const float bw = 1.f / ((2 * degree_of_row(r) + 1) * (lmax + 1));
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < CPR; ++j)
      q += (v[r][j].x * v[r][j].x + v[r][j].y * v[r][j].y) + (v[r][j].z * v[r][j].z + v[r][j].w * v[r][j].w);
    ss += bw * q;
  }
  const float rstd = rsqrtf(e2a_warp_sum(ss) / C + eps);
  float* yn = y + node * R * C;
#pragma unroll
  for (int r = 0; r < kMaxRows; ++r) {
    if (r >= R) continue;
    const float* wl = w + degree_of_row(r) * C;
#pragma unroll
    for (int j = 0; j < CPR; ++j) {
      const int c = 4 * (lane + 32 * j);
      const float4 ww = ld4(wl + c);
      float4 o = make_float4(v[r][j].x * rstd * ww.x, v[r][j].y * rstd * ww.y, v[r][j].z * rstd * ww.z,
                             v[r][j].w * rstd * ww.w);
      if (r == 0) {
        const float4 bb = ld4(b + c);
        o.x += bb.x; o.y += bb.y; o.z += bb.z; o.w += bb.w;
      }
      st4(yn + r * C + c, o);
    }
  }
  if (lane == 0) {
    stats[2 * node] = mean0;
    stats[2 * node + 1] = rstd;
  }
}

// dx from dy: df = g w rstd - rstd^3 bw_r f S / C with S = sum g w f; the centred row subtracts its mean.
template <int CPR>
__global__ void __launch_bounds__(kNodeThreads)
k_rms_norm_bwd(const float* __restrict__ x, const float* __restrict__ dy, int64_t n, int R, int lmax,
               const float* __restrict__ w, const float* __restrict__ stats, float* __restrict__ dx) {
  constexpr int C = 128 * CPR;
  const int lane = threadIdx.x & 31;
  const int64_t node = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (node >= n) return;
  const float mean0 = stats[2 * node], rstd = stats[2 * node + 1];
  const float* xn = x + node * R * C;
  const float* gn = dy + node * R * C;
  float4 f[kMaxRows][CPR], gw[kMaxRows][CPR];
  float S = 0.f;
#pragma unroll
  for (int r = 0; r < kMaxRows; ++r) {
    if (r >= R) continue;
    const float* wl = w + degree_of_row(r) * C;
#pragma unroll
    for (int j = 0; j < CPR; ++j) {
      const int c = 4 * (lane + 32 * j);
      float4 xv = ld4(xn + r * C + c);
      if (r == 0) { xv.x -= mean0; xv.y -= mean0; xv.z -= mean0; xv.w -= mean0; }
      const float4 g = ld4(gn + r * C + c), ww = ld4(wl + c);
      f[r][j] = xv;
      gw[r][j] = make_float4(g.x * ww.x, g.y * ww.y, g.z * ww.z, g.w * ww.w);
      S += (gw[r][j].x * xv.x + gw[r][j].y * xv.y) + (gw[r][j].z * xv.z + gw[r][j].w * xv.w);
    }
  }
  S = e2a_warp_sum(S);
  const float k3 = rstd * rstd * rstd * S / C;
  float* dn = dx + node * R * C;
  float4 d0[CPR];
  float s0 = 0.f;
#pragma unroll
  for (int r = 0; r < kMaxRows; ++r) {
    if (r >= R) continue;
    const float bw = 1.f / ((2 * degree_of_row(r) + 1) * (lmax + 1));
#pragma unroll
    for (int j = 0; j < CPR; ++j) {
      const float4 d = make_float4(gw[r][j].x * rstd - k3 * bw * f[r][j].x, gw[r][j].y * rstd - k3 * bw * f[r][j].y,
                                   gw[r][j].z * rstd - k3 * bw * f[r][j].z, gw[r][j].w * rstd - k3 * bw * f[r][j].w);
      if (r == 0) {
        d0[j] = d;
        s0 += (d.x + d.y) + (d.z + d.w);
      } else {
        st4(dn + r * C + 4 * (lane + 32 * j), d);
      }
    }
  }
  const float m = e2a_warp_sum(s0) / C;
#pragma unroll
  for (int j = 0; j < CPR; ++j)
    st4(dn + 4 * (lane + 32 * j), make_float4(d0[j].x - m, d0[j].y - m, d0[j].z - m, d0[j].w - m));
}

__device__ __forceinline__ float sigm(float t) { return 1.f / (1.f + expf(-t)); }

// Gate forward: grid-stride over (node, float4 channel group).
__global__ void k_gate_fwd(const float* __restrict__ s, const float* __restrict__ h, int64_t n, int R, int C,
                           float cs, float cv, float* __restrict__ y) {
  const int C4 = C / 4;
  const int64_t total = n * C4;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t node = t / C4;
    const int c = 4 * (int)(t - node * C4);
    const float* sn = s + node * 3 * C;
    const float* hn = h + node * R * C;
    float* yn = y + node * R * C;
    const float4 s0 = ld4(sn + c);
    st4(yn + c, make_float4(cs * s0.x * sigm(s0.x), cs * s0.y * sigm(s0.y), cs * s0.z * sigm(s0.z),
                            cs * s0.w * sigm(s0.w)));
    for (int l = 1; l <= 2; ++l) {
      const float4 sl = ld4(sn + l * C + c);
      const float4 g = make_float4(cv * sigm(sl.x), cv * sigm(sl.y), cv * sigm(sl.z), cv * sigm(sl.w));
      for (int r = l * l; r < (l + 1) * (l + 1) && r < R; ++r) {
        const float4 hv = ld4(hn + r * C + c);
        st4(yn + r * C + c, make_float4(g.x * hv.x, g.y * hv.y, g.z * hv.z, g.w * hv.w));
      }
    }
  }
}

// Gate backward: ds and dh (dh row 0 is zero: that row reaches the output through s only).
__global__ void k_gate_bwd(const float* __restrict__ s, const float* __restrict__ h, const float* __restrict__ dy,
                           int64_t n, int R, int C, float cs, float cv, float* __restrict__ ds, float* __restrict__ dh) {
  const int C4 = C / 4;
  const int64_t total = n * C4;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t node = t / C4;
    const int c = 4 * (int)(t - node * C4);
    const float* sn = s + node * 3 * C;
    const float* hn = h + node * R * C;
    const float* gn = dy + node * R * C;
    float* dsn = ds + node * 3 * C;
    float* dhn = dh + node * R * C;
    {
      const float4 s0 = ld4(sn + c), g0 = ld4(gn + c);
      const float sx[4] = {s0.x, s0.y, s0.z, s0.w}, gx[4] = {g0.x, g0.y, g0.z, g0.w};
      float o[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float sg = sigm(sx[u]);
        o[u] = gx[u] * cs * sg * (1.f + sx[u] * (1.f - sg));
      }
      st4(dsn + c, make_float4(o[0], o[1], o[2], o[3]));
      st4(dhn + c, make_float4(0.f, 0.f, 0.f, 0.f));
    }
    for (int l = 1; l <= 2; ++l) {
      const float4 sl = ld4(sn + l * C + c);
      const float sx[4] = {sl.x, sl.y, sl.z, sl.w};
      float sg[4], acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int u = 0; u < 4; ++u) sg[u] = sigm(sx[u]);
      for (int r = l * l; r < (l + 1) * (l + 1) && r < R; ++r) {
        const float4 hv = ld4(hn + r * C + c), gv = ld4(gn + r * C + c);
        const float hx[4] = {hv.x, hv.y, hv.z, hv.w}, gx[4] = {gv.x, gv.y, gv.z, gv.w};
        float o[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          acc[u] += gx[u] * hx[u];
          o[u] = gx[u] * cv * sg[u];
        }
        st4(dhn + r * C + c, make_float4(o[0], o[1], o[2], o[3]));
      }
      float o[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) o[u] = acc[u] * cv * sg[u] * (1.f - sg[u]);
      st4(dsn + l * C + c, make_float4(o[0], o[1], o[2], o[3]));
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

unsigned grid_nodes(int64_t n) {
  const int64_t b = (n * 32 + kNodeThreads - 1) / kNodeThreads;
  return (unsigned)(b < 1 ? 1 : b);
}

unsigned grid_flat(int64_t total) {
  const int64_t b = (total + 255) / 256;
  return (unsigned)(b < 1 ? 1 : (b > 148 * 64 ? 148 * 64 : b));
}

}  // namespace

extern "C" {

int e2a_rms_norm_fwd(const float* x, int64_t n_nodes, int rows, int C, const float* weight, const float* bias,
                     float eps, float* y, float* stats, void* stream) {
  if (n_nodes < 0 || rows < 1 || rows > kMaxRows || (rows != 1 && rows != 4 && rows != 9)) return E2A_ERR_ARG;
  if (n_nodes == 0) return E2A_OK;
  if (!x || !weight || !bias || !y || !stats) return E2A_ERR_ARG;
  if (C % 128 || C > 256 || !aligned16(x) || !aligned16(y) || !aligned16(weight) || !aligned16(bias))
    return E2A_ERR_UNSUPPORTED;
  const int lmax = rows == 1 ? 0 : (rows == 4 ? 1 : 2);
  cudaStream_t st = (cudaStream_t)stream;
  switch (C / 128) {
    case 1: k_rms_norm_fwd<1><<<grid_nodes(n_nodes), kNodeThreads, 0, st>>>(x, n_nodes, rows, lmax, weight, bias, eps, y, stats); break;
    default: k_rms_norm_fwd<2><<<grid_nodes(n_nodes), kNodeThreads, 0, st>>>(x, n_nodes, rows, lmax, weight, bias, eps, y, stats); break;
  }
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

int e2a_rms_norm_bwd(const float* x, const float* dy, int64_t n_nodes, int rows, int C, const float* weight,
                     const float* stats, float* dx, void* stream) {
  if (n_nodes < 0 || rows < 1 || rows > kMaxRows || (rows != 1 && rows != 4 && rows != 9)) return E2A_ERR_ARG;
  if (n_nodes == 0) return E2A_OK;
  if (!x || !dy || !weight || !stats || !dx) return E2A_ERR_ARG;
  if (C % 128 || C > 256 || !aligned16(x) || !aligned16(dy) || !aligned16(dx) || !aligned16(weight))
    return E2A_ERR_UNSUPPORTED;
  const int lmax = rows == 1 ? 0 : (rows == 4 ? 1 : 2);
  cudaStream_t st = (cudaStream_t)stream;
  switch (C / 128) {
    case 1: k_rms_norm_bwd<1><<<grid_nodes(n_nodes), kNodeThreads, 0, st>>>(x, dy, n_nodes, rows, lmax, weight, stats, dx); break;
    default: k_rms_norm_bwd<2><<<grid_nodes(n_nodes), kNodeThreads, 0, st>>>(x, dy, n_nodes, rows, lmax, weight, stats, dx); break;
  }
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

int e2a_gate_fwd(const float* s, const float* h, int64_t n_nodes, int rows, int C, float c_scalar, float c_vector,
                 float* y, void* stream) {
  if (n_nodes < 0 || rows != 9 || C <= 0) return E2A_ERR_ARG;
  if (n_nodes == 0) return E2A_OK;
  if (!s || !h || !y) return E2A_ERR_ARG;
  if (C % 4 || !aligned16(s) || !aligned16(h) || !aligned16(y)) return E2A_ERR_UNSUPPORTED;
  k_gate_fwd<<<grid_flat(n_nodes * (C / 4)), 256, 0, (cudaStream_t)stream>>>(s, h, n_nodes, rows, C, c_scalar,
                                                                            c_vector, y);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

int e2a_gate_bwd(const float* s, const float* h, const float* dy, int64_t n_nodes, int rows, int C, float c_scalar,
                 float c_vector, float* ds, float* dh, void* stream) {
  if (n_nodes < 0 || rows != 9 || C <= 0) return E2A_ERR_ARG;
  if (n_nodes == 0) return E2A_OK;
  if (!s || !h || !dy || !ds || !dh) return E2A_ERR_ARG;
  if (C % 4 || !aligned16(s) || !aligned16(h) || !aligned16(dy) || !aligned16(ds) || !aligned16(dh))
    return E2A_ERR_UNSUPPORTED;
  k_gate_bwd<<<grid_flat(n_nodes * (C / 4)), 256, 0, (cudaStream_t)stream>>>(s, h, dy, n_nodes, rows, C, c_scalar,
                                                                            c_vector, ds, dh);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------
// Gaussian radial basis (GaussianSmearing, module_utils.py:1853-1870) formed where it is consumed:
//   rbf[e, k] = exp(coeff (d_e - mu_k)^2)
// and the distance gradient of a consumer's d(rbf), reduced over k without storing rbf:
//   d_d[e] = sum_k g[e, k] rbf[e, k] 2 coeff (d_e - mu_k)
// ------------------------------------------------------------------------------------------------
namespace {

__global__ void k_rbf_fwd(const float* __restrict__ d, int64_t E, const float* __restrict__ mu, int nb, float coeff,
                          float* __restrict__ out) {
  const int64_t total = E * (int64_t)nb;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = t / nb;
    const int k = (int)(t - e * nb);
    const float x = d[e] - mu[k];
    out[t] = expf(coeff * (x * x));
  }
}

// Same basis, four consecutive basis functions per thread (nb % 4 == 0): one 16-byte store each, the
// offsets staged in shared memory (nb <= 1024).
__global__ void k_rbf_fwd4(const float* __restrict__ d, int64_t E, const float* __restrict__ mu, int nb, float coeff,
                           float* __restrict__ out) {
  __shared__ float mu_s[1024];
  for (int k = threadIdx.x; k < nb; k += blockDim.x) mu_s[k] = mu[k];
  __syncthreads();
  const int nb4 = nb >> 2;
  const int64_t total = E * (int64_t)nb4;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = t / nb4;
    const int k = 4 * (int)(t - e * nb4);
    const float de = __ldg(d + e);
    const float x0 = de - mu_s[k], x1 = de - mu_s[k + 1], x2 = de - mu_s[k + 2], x3 = de - mu_s[k + 3];
    reinterpret_cast<float4*>(out)[t] =
        make_float4(expf(coeff * (x0 * x0)), expf(coeff * (x1 * x1)), expf(coeff * (x2 * x2)), expf(coeff * (x3 * x3)));
  }
}

__global__ void k_rbf_bwd(const float* __restrict__ d, const float* __restrict__ g, int64_t E,
                          const float* __restrict__ mu, int nb, float coeff, float* __restrict__ dd) {
  const int lane = threadIdx.x & 31;
  int64_t e = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (; e < E; e += nw) {
    const float de = d[e];
    float acc = 0.f;
    for (int k = lane; k < nb; k += 32) {
      const float x = de - mu[k];
      acc += g[e * nb + k] * expf(coeff * (x * x)) * (2.f * coeff * x);
    }
    acc = e2a_warp_sum(acc);
    if (lane == 0) dd[e] = acc;
  }
}

}  // namespace

extern "C" {

int e2a_rbf_fwd(const float* dist, int64_t n_edges, const float* mu, int nb, float coeff, float* out, void* stream) {
  if (n_edges < 0 || nb <= 0) return E2A_ERR_ARG;
  if (n_edges == 0) return E2A_OK;
  if (!dist || !mu || !out) return E2A_ERR_ARG;
  if (nb % 4 == 0 && nb <= 1024 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0)
    k_rbf_fwd4<<<grid_flat(n_edges * (nb / 4)), 256, 0, (cudaStream_t)stream>>>(dist, n_edges, mu, nb, coeff, out);
  else
    k_rbf_fwd<<<grid_flat(n_edges * nb), 256, 0, (cudaStream_t)stream>>>(dist, n_edges, mu, nb, coeff, out);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

int e2a_rbf_bwd(const float* dist, const float* grad, int64_t n_edges, const float* mu, int nb, float coeff,
                float* d_dist, void* stream) {
  if (n_edges < 0 || nb <= 0) return E2A_ERR_ARG;
  if (n_edges == 0) return E2A_OK;
  if (!dist || !grad || !mu || !d_dist) return E2A_ERR_ARG;
  k_rbf_bwd<<<grid_flat(n_edges * 32), 256, 0, (cudaStream_t)stream>>>(dist, grad, n_edges, mu, nb, coeff, d_dist);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------
// Per-node map of the first-order SO(2) product, straight from the node's position (fp64 inside):
//   (alpha, beta) = the Euler angles of the position (module_utils.py:182-226, eval: gamma = 0; the
//                   angles are held constant at the poles / near the origin, as the reference
//                   detaches them there),
//   D^l = J_l Y_l(-beta) J_l Y_l(-alpha)  (module_utils.py:266-337; Y_l = rotation about y),
//   W   = blockdiag(D^0, D^1, D^2),  Wi^T = blockdiag over l3_sequential of (D^l3)^T,
//   A[k, s] = |pos| sum_j Wi^T[k, j] W[sel[j], s] cg[j]       (so2_tensor_product.py:341-389),
// rows written in the order row_perm (new row k <- old row row_perm[k]).  The backward is the
// analytic derivative of A with respect to the position (through |pos| and the two angles).
// ------------------------------------------------------------------------------------------------
namespace {

struct NodeMapTables {
  double J1[9], J2[25];
  double cg[20];
  int sel[20];
  int perm[20];
};

// (row0, l) of the six Wi blocks for l3_sequential = ((0,1), (1,3), (2,2))
__device__ __forceinline__ void wi_block(int k, int& r0, int& l) {
  if (k == 0) { r0 = 0; l = 0; }
  else if (k < 10) { r0 = 1 + 3 * ((k - 1) / 3); l = 1; }
  else { r0 = 10 + 5 * ((k - 10) / 5); l = 2; }
}

template <int L>
__device__ __forceinline__ void yrot(double th, double (&Y)[2 * L + 1][2 * L + 1], double (&dY)[2 * L + 1][2 * L + 1]) {
  constexpr int M = 2 * L + 1;
#pragma unroll
  for (int i = 0; i < M; ++i)
#pragma unroll
    for (int j = 0; j < M; ++j) { Y[i][j] = 0.0; dY[i][j] = 0.0; }
#pragma unroll
  for (int i = 0; i < M; ++i) {
    const double f = (double)(L - i);
    double s, c;
    sincos(f * th, &s, &c);
    Y[i][2 * L - i] = s;
    dY[i][2 * L - i] = f * c;
    Y[i][i] = c;                  // overwrites the centre entry (f = 0): cos 0 = 1
    dY[i][i] = -f * s;
  }
}

template <int M>
__device__ __forceinline__ void matmul(const double (&A)[M][M], const double (&B)[M][M], double (&C)[M][M]) {
#pragma unroll
  for (int i = 0; i < M; ++i)
#pragma unroll
    for (int j = 0; j < M; ++j) {
      double acc = 0.0;
#pragma unroll
      for (int k = 0; k < M; ++k) acc += A[i][k] * B[k][j];
      C[i][j] = acc;
    }
}

template <int L>
__device__ __forceinline__ void load_j(const double* src, double (&J)[2 * L + 1][2 * L + 1]) {
#pragma unroll
  for (int i = 0; i < 2 * L + 1; ++i)
#pragma unroll
    for (int j = 0; j < 2 * L + 1; ++j) J[i][j] = src[i * (2 * L + 1) + j];
}

// D = J Yb J Yc and (optionally) the pieces of its angle derivatives
template <int L>
struct DBlock {
  static constexpr int M = 2 * L + 1;
  double D[M][M], JYbJ[M][M], Yc[M][M], dYc[M][M], Yb[M][M], dYb[M][M], J[M][M];
  __device__ __forceinline__ void build(const double* jsrc, double b, double c) {
    load_j<L>(jsrc, J);
    yrot<L>(b, Yb, dYb);
    yrot<L>(c, Yc, dYc);
    double T[M][M];
    matmul<M>(J, Yb, T);
    matmul<M>(T, J, JYbJ);
    matmul<M>(JYbJ, Yc, D);
  }
};

struct Geo {
  double p[3], d, xn, yn, zn;
  bool mask;
  double beta, alpha;
};

__device__ __forceinline__ Geo geometry(const float* pos, int64_t n) {
  Geo g;
  g.p[0] = pos[3 * n]; g.p[1] = pos[3 * n + 1]; g.p[2] = pos[3 * n + 2];
  g.d = sqrt(g.p[0] * g.p[0] + g.p[1] * g.p[1] + g.p[2] * g.p[2]);
  const bool small = g.d < 1e-5;
  const double dd = small ? 1.0 : g.d;
  g.xn = g.p[0] / dd; g.yn = g.p[1] / dd; g.zn = g.p[2] / dd;
  g.mask = small || fabs(fabs(g.yn) - 1.0) <= 1e-8 + 1e-5;
  g.beta = acos(fmin(1.0, fmax(-1.0, g.yn)));
  g.alpha = atan2(g.xn, g.zn);
  return g;
}

// W[row][s] for row, s in 0..8 from the blocks
__device__ __forceinline__ double wget(const DBlock<1>& b1, const DBlock<2>& b2, int r, int s) {
  if (r == 0) return s == 0 ? 1.0 : 0.0;
  if (r < 4) return (s >= 1 && s < 4) ? b1.D[r - 1][s - 1] : 0.0;
  return s >= 4 ? b2.D[r - 4][s - 4] : 0.0;
}

__device__ __forceinline__ double dget(const DBlock<1>& b1, const DBlock<2>& b2, int l, int i, int j) {
  return l == 0 ? 1.0 : (l == 1 ? b1.D[i][j] : b2.D[i][j]);
}

__global__ void __launch_bounds__(128)
k_node_map_fwd(const float* __restrict__ pos, int64_t n_nodes, NodeMapTables t, float* __restrict__ A) {
  const int64_t n = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (n >= n_nodes) return;
  const Geo g = geometry(pos, n);
  DBlock<1> b1;
  DBlock<2> b2;
  b1.build(t.J1, -g.beta, -g.alpha);
  b2.build(t.J2, -g.beta, -g.alpha);
  float* out = A + n * 180;
  for (int kn = 0; kn < 20; ++kn) {
    const int k = t.perm[kn];
    int r0, l;
    wi_block(k, r0, l);
    const int kk = k - r0;
    for (int s = 0; s < 9; ++s) {
      double acc = 0.0;
      for (int jj = 0; jj < 2 * l + 1; ++jj) {
        const int j = r0 + jj;
        acc += dget(b1, b2, l, jj, kk) * wget(b1, b2, t.sel[j], s) * t.cg[j];
      }
      out[kn * 9 + s] = (float)(g.d * acc);
    }
  }
}

__global__ void __launch_bounds__(128)
k_node_map_bwd(const float* __restrict__ pos, const float* __restrict__ dA, int64_t n_nodes, NodeMapTables t,
               float* __restrict__ dpos) {
  const int64_t n = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (n >= n_nodes) return;
  const Geo g = geometry(pos, n);
  DBlock<1> b1;
  DBlock<2> b2;
  b1.build(t.J1, -g.beta, -g.alpha);
  b2.build(t.J2, -g.beta, -g.alpha);
  double dD1[3][3] = {}, dD2[5][5] = {};
  double dW[9][9] = {};
  double dscale = 0.0;
  const float* gA = dA + n * 180;
  for (int kn = 0; kn < 20; ++kn) {
    const int k = t.perm[kn];
    int r0, l;
    wi_block(k, r0, l);
    const int kk = k - r0;
    for (int s = 0; s < 9; ++s) {
      const double ga = gA[kn * 9 + s];
      if (ga == 0.0) continue;
      double tks = 0.0;
      for (int jj = 0; jj < 2 * l + 1; ++jj) {
        const int j = r0 + jj;
        const double m = wget(b1, b2, t.sel[j], s) * t.cg[j];
        const double wi = dget(b1, b2, l, jj, kk);
        tks += wi * m;
        // A = d * sum_j Wi^T[k][j] M[j][s]:  d(D^l[jj][kk]) += ga d M[j][s];  dM[j][s] += ga d Wi^T[k][j]
        if (l == 1) dD1[jj][kk] += ga * g.d * m;
        else if (l == 2) dD2[jj][kk] += ga * g.d * m;
        dW[t.sel[j]][s] += ga * g.d * wi * t.cg[j];
      }
      dscale += ga * tks;
    }
  }
  // W blocks -> D blocks
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) dD1[i][j] += dW[1 + i][1 + j];
  for (int i = 0; i < 5; ++i)
    for (int j = 0; j < 5; ++j) dD2[i][j] += dW[4 + i][4 + j];
  double gp[3] = {0.0, 0.0, 0.0};
  if (g.d > 0.0) {
    gp[0] = dscale * g.p[0] / g.d; gp[1] = dscale * g.p[1] / g.d; gp[2] = dscale * g.p[2] / g.d;
  }
  if (!g.mask) {
    // D = (J Yb J) Yc:  dL/dc = <dD, JYbJ Yc'>;  dL/db = <dD, J Yb' J Yc>
    double dLdb = 0.0, dLdc = 0.0;
    {
      double T[3][3], U[3][3], V[3][3], X[3][3];
      matmul<3>(b1.JYbJ, b1.dYc, T);
      matmul<3>(b1.J, b1.dYb, U);
      matmul<3>(U, b1.J, V);
      matmul<3>(V, b1.Yc, X);
      for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) { dLdc += dD1[i][j] * T[i][j]; dLdb += dD1[i][j] * X[i][j]; }
    }
    {
      double T[5][5], U[5][5], V[5][5], X[5][5];
      matmul<5>(b2.JYbJ, b2.dYc, T);
      matmul<5>(b2.J, b2.dYb, U);
      matmul<5>(U, b2.J, V);
      matmul<5>(V, b2.Yc, X);
      for (int i = 0; i < 5; ++i)
        for (int j = 0; j < 5; ++j) { dLdc += dD2[i][j] * T[i][j]; dLdb += dD2[i][j] * X[i][j]; }
    }
    const double dbeta = -dLdb, dalpha = -dLdc;     // b = -beta, c = -alpha
    const double pn[3] = {g.xn, g.yn, g.zn};
    const double dbdy = -1.0 / sqrt(fmax(1e-300, 1.0 - g.yn * g.yn));
    const double rxz = g.xn * g.xn + g.zn * g.zn;
    const double dadx = g.zn / rxz, dadz = -g.xn / rxz;
    for (int i = 0; i < 3; ++i) {
      const double dyn = ((i == 1 ? 1.0 : 0.0) - g.yn * pn[i]) / g.d;
      const double dxn = ((i == 0 ? 1.0 : 0.0) - g.xn * pn[i]) / g.d;
      const double dzn = ((i == 2 ? 1.0 : 0.0) - g.zn * pn[i]) / g.d;
      gp[i] += dbeta * dbdy * dyn + dalpha * (dadx * dxn + dadz * dzn);
    }
  }
  dpos[3 * n] = (float)gp[0];
  dpos[3 * n + 1] = (float)gp[1];
  dpos[3 * n + 2] = (float)gp[2];
}

int fill_tables(NodeMapTables& t, const double* j1, const double* j2, const int32_t* sel, const double* cg,
                const int32_t* row_perm) {
  if (!j1 || !j2 || !sel || !cg) return E2A_ERR_ARG;
  for (int i = 0; i < 9; ++i) t.J1[i] = j1[i];
  for (int i = 0; i < 25; ++i) t.J2[i] = j2[i];
  uint32_t seen = 0;
  for (int i = 0; i < 20; ++i) {
    if (sel[i] < 0 || sel[i] > 8) return E2A_ERR_ARG;
    t.sel[i] = sel[i];
    t.cg[i] = cg[i];
    t.perm[i] = row_perm ? row_perm[i] : i;
    if (t.perm[i] < 0 || t.perm[i] >= 20 || (seen >> t.perm[i]) & 1u) return E2A_ERR_ARG;   // a permutation
    seen |= 1u << t.perm[i];
  }
  return E2A_OK;
}

}  // namespace

extern "C" {

int e2a_node_map_fwd(const float* pos, int64_t n_nodes, const double* j1, const double* j2, const int32_t* sel,
                     const double* cg, const int32_t* row_perm, float* A, void* stream) {
  if (n_nodes < 0) return E2A_ERR_ARG;
  if (n_nodes == 0) return E2A_OK;
  if (!pos || !A) return E2A_ERR_ARG;
  NodeMapTables t;
  const int rc = fill_tables(t, j1, j2, sel, cg, row_perm);
  if (rc) return rc;
  k_node_map_fwd<<<(unsigned)((n_nodes + 127) / 128), 128, 0, (cudaStream_t)stream>>>(pos, n_nodes, t, A);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

int e2a_node_map_bwd(const float* pos, const float* dA, int64_t n_nodes, const double* j1, const double* j2,
                     const int32_t* sel, const double* cg, const int32_t* row_perm, float* dpos, void* stream) {
  if (n_nodes < 0) return E2A_ERR_ARG;
  if (n_nodes == 0) return E2A_OK;
  if (!pos || !dA || !dpos) return E2A_ERR_ARG;
  NodeMapTables t;
  const int rc = fill_tables(t, j1, j2, sel, cg, row_perm);
  if (rc) return rc;
  k_node_map_bwd<<<(unsigned)((n_nodes + 127) / 128), 128, 0, (cudaStream_t)stream>>>(pos, dA, n_nodes, t, dpos);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

}  // extern "C"
