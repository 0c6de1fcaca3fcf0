// Fused sparse attention span of E2AttentionArbOrder_sparse (QK logits, segmented softmax with the
// reference's non-standard eps/envelope, alpha/r, value aggregation) and its first-order backward.
//
// Layout (fp32, row-major): q [N,H,D] (already scaled by 1/sqrt(D)), k [M,H,D], value [M,C,H] (the
// merged SO(2)+irreps message, head innermost), gate / inputhead [E,H] views (row stride ld_gi),
// poly/dist [E].  Edges are in query-CSR order; edge id == CSR slot.
//
// One CTA (256 threads) owns one destination row.  The dominant cost is the gather of the value row
// of every neighbour (C*H*4 bytes, 29.7 KB at the full config): each thread owns fixed float4 slots
// of the [C,H] output tile, so every gathered row is read with fully coalesced 16-byte loads and
// accumulated in registers; per-edge softmax weights are shared by the whole CTA.  All sums over
// edges run in CSR order inside one CTA: results are deterministic and need no atomics.
#include "e2a_common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr float kSoftmaxEps = 1e-3f;   // e2former.py:364
constexpr float kMinDist = 1e-6f;      // e2former.py:422 clamp_min

struct Dims {
  int H, D, C;
  int HD4;   // H*D/4 float4 per q/k row
  int CH4;   // C*H/4 float4 per value row
  int g;     // lanes per head in the q.k dot (D/4)
};

__device__ __forceinline__ int row_of(const int32_t* __restrict__ order, int64_t r) {
  return order ? order[r] : (int)r;
}

// s[e,h] = <q_i,h, k_col[e],h> for e in [rs, re), one warp per edge.  q_s holds q_i (H*D floats).
template <typename F>
__device__ __forceinline__ void edge_scores(const float* __restrict__ q_s, const float* __restrict__ k,
                                            const int32_t* __restrict__ col, int rs, int re, const Dims& dm,
                                            F&& emit) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int e = rs + warp; e < re; e += kWarps) {
    const float* kr = k + (int64_t)col[e] * dm.HD4 * 4;
    for (int f0 = 0; f0 < dm.HD4; f0 += 32) {
      const int f = f0 + lane;
      float p = 0.f;
      if (f < dm.HD4) {
        const float4 kv = ldg4(kr + 4 * f);
        const float4 qv = *reinterpret_cast<const float4*>(q_s + 4 * f);
        p = qv.x * kv.x + qv.y * kv.y + qv.z * kv.z + qv.w * kv.w;
      }
      for (int o = 1; o < dm.g; o <<= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
      if (f < dm.HD4 && (f % dm.g) == 0) emit(e, f / dm.g, p);
    }
  }
}

__device__ __forceinline__ void stage_row(float* __restrict__ dst, const float* __restrict__ src, int n4) {
  for (int f = threadIdx.x; f < n4; f += kThreads)
    reinterpret_cast<float4*>(dst)[f] = ldg4(src + 4 * f);
}

// Combine per-stripe partials red[stripe*H + h] (fixed order) -> out_s[h].
__device__ __forceinline__ void combine_stripes(float* red, float* out_s, int H, int stripes, bool is_max) {
  __syncthreads();
  for (int h = threadIdx.x; h < H; h += kThreads) {
    float v = red[h];
    for (int s = 1; s < stripes; ++s) v = is_max ? fmaxf(v, red[s * H + h]) : v + red[s * H + h];
    out_s[h] = v;
  }
  __syncthreads();
}

// ------------------------------------------------------------------------------------------------
// Forward
// ------------------------------------------------------------------------------------------------
template <int KS>
__global__ void __launch_bounds__(kThreads)
k_attn_fwd(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ value,
           const float* __restrict__ gate, const float* __restrict__ inputhead, int64_t ld_gi,
           const float* __restrict__ poly, const float* __restrict__ dist,
           const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col,
           const int32_t* __restrict__ order, int64_t n_rows, Dims dm,
           float* __restrict__ out, float* __restrict__ beta, float* __restrict__ row_max,
           float* __restrict__ row_sum) {
  extern __shared__ float4 smem4[];
  float* q_s = reinterpret_cast<float*>(smem4);      // H*D
  float* red = q_s + dm.HD4 * 4;                     // kThreads
  float* m_s = red + kThreads;                       // H
  float* sum_s = m_s + dm.H;                         // H
  const int H = dm.H;
  const int stripes = kThreads / H;
  const int hh = threadIdx.x % H, stripe = threadIdx.x / H;

  for (int64_t r = blockIdx.x; r < n_rows; r += gridDim.x) {
    const int i = row_of(order, r);
    const int rs = row_ptr[i], re = row_ptr[i + 1];
    stage_row(q_s, q + (int64_t)i * dm.HD4 * 4, dm.HD4);
    __syncthreads();
    // 1. logits a = gate * (q.k) -> beta (scratch)
    edge_scores(q_s, k, col, rs, re, dm, [&](int e, int h, float s) {
      beta[(int64_t)e * H + h] = gate[(int64_t)e * ld_gi + h] * s;
    });
    __syncthreads();
    // 2. row max per head
    float mx = -INFINITY;
    for (int e = rs + stripe; e < re; e += stripes) mx = fmaxf(mx, beta[(int64_t)e * H + hh]);
    red[threadIdx.x] = mx;
    combine_stripes(red, m_s, H, stripes, true);
    // 3. x = exp(a - m) * poly, row sum
    const float m = m_s[hh];
    float sm = 0.f;
    for (int e = rs + stripe; e < re; e += stripes) {
      const int64_t o = (int64_t)e * H + hh;
      const float x = expf(beta[o] - m) * poly[e];
      beta[o] = x;
      sm += x;
    }
    red[threadIdx.x] = sm;
    combine_stripes(red, sum_s, H, stripes, false);
    // 4. beta = x * inputhead / (S + eps) / max(dist, 1e-6)
    const float den = sum_s[hh] + kSoftmaxEps;
    for (int e = rs + stripe; e < re; e += stripes) {
      const int64_t o = (int64_t)e * H + hh;
      const float a = beta[o] * inputhead[(int64_t)e * ld_gi + hh] / den;
      beta[o] = a / fmaxf(dist[e], kMinDist);
    }
    if (stripe == 0) {
      row_max[(int64_t)i * H + hh] = m;
      row_sum[(int64_t)i * H + hh] = sum_s[hh];
    }
    __syncthreads();
    // 5. out[i,c,h] = sum_e beta[e,h] value[j,c,h]
    const int h0 = (4 * threadIdx.x) % H;
    float4 acc[KS];
#pragma unroll
    for (int s = 0; s < KS; ++s) acc[s] = f4_zero();
    int e = rs;
    for (; e + 1 < re; e += 2) {
      const float* v0 = value + (int64_t)col[e] * dm.CH4 * 4;
      const float* v1 = value + (int64_t)col[e + 1] * dm.CH4 * 4;
      const float4 b0 = *reinterpret_cast<const float4*>(beta + (int64_t)e * H + h0);
      const float4 b1 = *reinterpret_cast<const float4*>(beta + (int64_t)(e + 1) * H + h0);
      float4 x0[KS], x1[KS];
#pragma unroll
      for (int s = 0; s < KS; ++s) {
        const int f = threadIdx.x + s * kThreads;
        if (f < dm.CH4) { x0[s] = ldg4(v0 + 4 * f); x1[s] = ldg4(v1 + 4 * f); }
      }
#pragma unroll
      for (int s = 0; s < KS; ++s) {
        const int f = threadIdx.x + s * kThreads;
        if (f < dm.CH4) acc[s] = f4_fma4(b1, x1[s], f4_fma4(b0, x0[s], acc[s]));
      }
    }
    if (e < re) {
      const float* v0 = value + (int64_t)col[e] * dm.CH4 * 4;
      const float4 b0 = *reinterpret_cast<const float4*>(beta + (int64_t)e * H + h0);
#pragma unroll
      for (int s = 0; s < KS; ++s) {
        const int f = threadIdx.x + s * kThreads;
        if (f < dm.CH4) acc[s] = f4_fma4(b0, ldg4(v0 + 4 * f), acc[s]);
      }
    }
    float* orow = out + (int64_t)i * dm.CH4 * 4;
#pragma unroll
    for (int s = 0; s < KS; ++s) {
      const int f = threadIdx.x + s * kThreads;
      if (f < dm.CH4) reinterpret_cast<float4*>(orow)[f] = acc[s];
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------------------------------------
// Backward, query side
// ------------------------------------------------------------------------------------------------
constexpr int kEB = 8;  // edges per reduction batch in the d(beta) pass

template <int KS>
__global__ void __launch_bounds__(kThreads)
k_attn_bwd_query(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ value,
                 const float* __restrict__ gate, const float* __restrict__ inputhead, int64_t ld_gi,
                 const float* __restrict__ poly, const float* __restrict__ dist,
                 const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col,
                 const int32_t* __restrict__ order, int64_t n_rows, Dims dm,
                 const float* __restrict__ beta, const float* __restrict__ row_max,
                 const float* __restrict__ row_sum, const float* __restrict__ dout,
                 float* __restrict__ d_q, float* __restrict__ d_gate, float* __restrict__ d_inputhead,
                 int64_t ld_dgi, float* __restrict__ d_poly, float* __restrict__ d_dist,
                 float* __restrict__ d_logit, float* __restrict__ bufA, float* __restrict__ bufB) {
  extern __shared__ float4 smem4[];
  float4* red4 = smem4;                                         // kEB * kThreads float4
  float* q_s = reinterpret_cast<float*>(red4 + kEB * kThreads); // H*D
  float* red = q_s + dm.HD4 * 4;                                // kThreads
  float* T_s = red + kThreads;                                  // H
  float* dm_s = T_s + dm.H;                                     // H
  float* nt_s = dm_s + dm.H;                                    // H
  const int H = dm.H;
  const int H4 = H / 4;
  const int stripes = kThreads / H;
  const int hh = threadIdx.x % H, stripe = threadIdx.x / H;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

  for (int64_t r = blockIdx.x; r < n_rows; r += gridDim.x) {
    const int i = row_of(order, r);
    const int rs = row_ptr[i], re = row_ptr[i + 1];
    if (rs == re) {  // isolated query: only d_q (zero) to write
      for (int f = threadIdx.x; f < dm.HD4 * 4; f += kThreads) d_q[(int64_t)i * dm.HD4 * 4 + f] = 0.f;
      continue;
    }
    stage_row(q_s, q + (int64_t)i * dm.HD4 * 4, dm.HD4);
    // 1. d(beta)[e,h] = sum_c dout[i,c,h] value[j,c,h]  -> bufA
    {
      float4 go[KS];
      const float* gr = dout + (int64_t)i * dm.CH4 * 4;
#pragma unroll
      for (int s = 0; s < KS; ++s) {
        const int f = threadIdx.x + s * kThreads;
        go[s] = f < dm.CH4 ? ldg4(gr + 4 * f) : f4_zero();
      }
      for (int e0 = rs; e0 < re; e0 += kEB) {
        const int ne = min(kEB, re - e0);
#pragma unroll
        for (int b = 0; b < kEB; ++b) {
          float4 p = f4_zero();
          if (b < ne) {
            const float* vr = value + (int64_t)col[e0 + b] * dm.CH4 * 4;
#pragma unroll
            for (int s = 0; s < KS; ++s) {
              const int f = threadIdx.x + s * kThreads;
              if (f < dm.CH4) p = f4_fma4(go[s], ldg4(vr + 4 * f), p);
            }
          }
          red4[b * kThreads + threadIdx.x] = p;
        }
        __syncthreads();
        // thread t reduces edge b = t / H4... over all threads sharing head group t % H4
        for (int o = threadIdx.x; o < ne * H4; o += kThreads) {
          const int b = o / H4, hg = o % H4;
          float4 a = f4_zero();
          for (int t = hg; t < kThreads; t += H4) {
            const float4 v = red4[b * kThreads + t];
            a.x += v.x; a.y += v.y; a.z += v.z; a.w += v.w;
          }
          *reinterpret_cast<float4*>(bufA + (int64_t)(e0 + b) * H + 4 * hg) = a;
        }
        __syncthreads();
      }
    }
    // 2. s = q.k -> bufB
    edge_scores(q_s, k, col, rs, re, dm, [&](int e, int h, float s) { bufB[(int64_t)e * H + h] = s; });
    __syncthreads();
    const float m = row_max[(int64_t)i * H + hh];
    const float S = row_sum[(int64_t)i * H + hh];
    const float den = S + kSoftmaxEps;
    // 3. T_h = sum_e d_alpha * alpha
    {
      float T = 0.f;
      for (int e = rs + stripe; e < re; e += stripes) {
        const int64_t o = (int64_t)e * H + hh;
        const float a = gate[(int64_t)e * ld_gi + hh] * bufB[o];
        const float x = expf(a - m) * poly[e];
        const float al = x * inputhead[(int64_t)e * ld_gi + hh] / den;
        const float dal = bufA[o] / fmaxf(dist[e], kMinDist);
        T += dal * al;
      }
      red[threadIdx.x] = T;
      combine_stripes(red, T_s, H, stripes, false);
    }
    const float dS = -T_s[hh] / den;
    // 4. dz = dx * x; d_inputhead; accumulate dm and tie counts
    {
      float dmacc = 0.f, nt = 0.f;
      for (int e = rs + stripe; e < re; e += stripes) {
        const int64_t o = (int64_t)e * H + hh;
        const float a = gate[(int64_t)e * ld_gi + hh] * bufB[o];
        const float ex = expf(a - m);
        const float x = ex * poly[e];
        const float ih = inputhead[(int64_t)e * ld_gi + hh];
        const float dal = bufA[o] / fmaxf(dist[e], kMinDist);
        const float dx = dal * ih / den + dS;
        d_inputhead[(int64_t)e * ld_dgi + hh] = dal * x / den;
        const float dz = dx * x;
        d_logit[o] = dz;
        dmacc -= dz;
        nt += (a == m) ? 1.f : 0.f;
      }
      red[threadIdx.x] = dmacc;
      combine_stripes(red, dm_s, H, stripes, false);
      red[threadIdx.x] = nt;
      combine_stripes(red, nt_s, H, stripes, false);
    }
    // 5. da = dz + [a == m] dm / n_ties;  d_gate = da * s;  d_logit = ds = da * gate
    {
      const float share = nt_s[hh] > 0.f ? dm_s[hh] / nt_s[hh] : 0.f;
      for (int e = rs + stripe; e < re; e += stripes) {
        const int64_t o = (int64_t)e * H + hh;
        const float g = gate[(int64_t)e * ld_gi + hh];
        const float s = bufB[o];
        const float a = g * s;
        const float da = d_logit[o] + ((a == m) ? share : 0.f);
        d_gate[(int64_t)e * ld_dgi + hh] = da * s;
        d_logit[o] = da * g;
      }
    }
    // 6. per-edge sums over heads: d_dist = -sum_h dbeta * beta / r ; d_poly = sum_h dx * exp(a-m)
    //    (T_s and the row stats are complete; one warp per edge, fixed shuffle order)
    for (int e = rs + warp; e < re; e += kWarps) {
      const float d = dist[e];
      const float rr = fmaxf(d, kMinDist);
      const float p = poly[e];
      float sd = 0.f, sp = 0.f;
      for (int h = lane; h < H; h += 32) {
        const int64_t o = (int64_t)e * H + h;
        const float mh = row_max[(int64_t)i * H + h];
        const float denh = row_sum[(int64_t)i * H + h] + kSoftmaxEps;
        const float dSh = -T_s[h] / denh;
        const float a = gate[(int64_t)e * ld_gi + h] * bufB[o];
        const float ex = expf(a - mh);
        const float dal = bufA[o] / rr;
        const float dx = dal * inputhead[(int64_t)e * ld_gi + h] / denh + dSh;
        sd += bufA[o] * beta[o];
        sp += dx * ex;
      }
      sd = e2a_warp_sum(sd);
      sp = e2a_warp_sum(sp);
      if (lane == 0) {
        d_dist[e] = d >= kMinDist ? -sd / rr : 0.f;
        d_poly[e] = sp;
        (void)p;
      }
    }
    __syncthreads();
    // 7. d_q[i,h,:] = sum_e ds[e,h] k[j,h,:]   (warps take edges, fixed-order cross-warp sum)
    {
      constexpr int kMaxSlots = 8;  // H*D/4 <= 32 * 8 float4 per lane
      float4 acc[kMaxSlots];
#pragma unroll
      for (int s = 0; s < kMaxSlots; ++s) acc[s] = f4_zero();
      for (int e = rs + warp; e < re; e += kWarps) {
        const float* kr = k + (int64_t)col[e] * dm.HD4 * 4;
#pragma unroll
        for (int s = 0; s < kMaxSlots; ++s) {
          const int f = lane + 32 * s;
          if (f < dm.HD4) {
            const float w = d_logit[(int64_t)e * H + (4 * f) / dm.D];
            acc[s] = f4_fma(w, ldg4(kr + 4 * f), acc[s]);
          }
        }
      }
      // cross-warp reduction through red4 (kEB*kThreads float4 >= kWarps * HD4)
#pragma unroll
      for (int s = 0; s < kMaxSlots; ++s) {
        const int f = lane + 32 * s;
        if (f < dm.HD4) red4[warp * dm.HD4 + f] = acc[s];
      }
      __syncthreads();
      for (int f = threadIdx.x; f < dm.HD4; f += kThreads) {
        float4 a = red4[f];
        for (int w = 1; w < kWarps; ++w) {
          const float4 v = red4[w * dm.HD4 + f];
          a.x += v.x; a.y += v.y; a.z += v.z; a.w += v.w;
        }
        reinterpret_cast<float4*>(d_q + (int64_t)i * dm.HD4 * 4)[f] = a;
      }
      __syncthreads();
    }
  }
}

// ------------------------------------------------------------------------------------------------
// Backward, key side (key-CSR)
// ------------------------------------------------------------------------------------------------
template <int KS>
__global__ void __launch_bounds__(kThreads)
k_attn_bwd_key(const float* __restrict__ q, const float* __restrict__ dout, const float* __restrict__ beta,
               const float* __restrict__ d_logit, const int32_t* __restrict__ k_row_ptr,
               const int32_t* __restrict__ k_col, const int32_t* __restrict__ k_perm, int64_t n_keys, Dims dm,
               float* __restrict__ d_k, float* __restrict__ d_value) {
  extern __shared__ float4 smem4[];
  const int H = dm.H;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t j = blockIdx.x; j < n_keys; j += gridDim.x) {
    const int rs = k_row_ptr[j], re = k_row_ptr[j + 1];
    // d_value[j] = sum_p beta[e_p] * dout[i_p]
    const int h0 = (4 * threadIdx.x) % H;
    float4 acc[KS];
#pragma unroll
    for (int s = 0; s < KS; ++s) acc[s] = f4_zero();
    int p = rs;
    for (; p + 1 < re; p += 2) {
      const int e0 = k_perm[p], e1 = k_perm[p + 1];
      const float* g0 = dout + (int64_t)k_col[p] * dm.CH4 * 4;
      const float* g1 = dout + (int64_t)k_col[p + 1] * dm.CH4 * 4;
      const float4 b0 = ldg4(beta + (int64_t)e0 * H + h0);
      const float4 b1 = ldg4(beta + (int64_t)e1 * H + h0);
      float4 x0[KS], x1[KS];
#pragma unroll
      for (int s = 0; s < KS; ++s) {
        const int f = threadIdx.x + s * kThreads;
        if (f < dm.CH4) { x0[s] = ldg4(g0 + 4 * f); x1[s] = ldg4(g1 + 4 * f); }
      }
#pragma unroll
      for (int s = 0; s < KS; ++s) {
        const int f = threadIdx.x + s * kThreads;
        if (f < dm.CH4) acc[s] = f4_fma4(b1, x1[s], f4_fma4(b0, x0[s], acc[s]));
      }
    }
    if (p < re) {
      const int e0 = k_perm[p];
      const float* g0 = dout + (int64_t)k_col[p] * dm.CH4 * 4;
      const float4 b0 = ldg4(beta + (int64_t)e0 * H + h0);
#pragma unroll
      for (int s = 0; s < KS; ++s) {
        const int f = threadIdx.x + s * kThreads;
        if (f < dm.CH4) acc[s] = f4_fma4(b0, ldg4(g0 + 4 * f), acc[s]);
      }
    }
    float* vrow = d_value + (int64_t)j * dm.CH4 * 4;
#pragma unroll
    for (int s = 0; s < KS; ++s) {
      const int f = threadIdx.x + s * kThreads;
      if (f < dm.CH4) reinterpret_cast<float4*>(vrow)[f] = acc[s];
    }
    // d_k[j,h,:] = sum_p ds[e_p,h] q[i_p,h,:]
    constexpr int kMaxSlots = 8;
    float4 kacc[kMaxSlots];
#pragma unroll
    for (int s = 0; s < kMaxSlots; ++s) kacc[s] = f4_zero();
    for (int pp = rs + warp; pp < re; pp += kWarps) {
      const int e = k_perm[pp];
      const float* qr = q + (int64_t)k_col[pp] * dm.HD4 * 4;
#pragma unroll
      for (int s = 0; s < kMaxSlots; ++s) {
        const int f = lane + 32 * s;
        if (f < dm.HD4) kacc[s] = f4_fma(__ldg(d_logit + (int64_t)e * H + (4 * f) / dm.D), ldg4(qr + 4 * f), kacc[s]);
      }
    }
#pragma unroll
    for (int s = 0; s < kMaxSlots; ++s) {
      const int f = lane + 32 * s;
      if (f < dm.HD4) smem4[warp * dm.HD4 + f] = kacc[s];
    }
    __syncthreads();
    for (int f = threadIdx.x; f < dm.HD4; f += kThreads) {
      float4 a = smem4[f];
      for (int w = 1; w < kWarps; ++w) {
        const float4 v = smem4[w * dm.HD4 + f];
        a.x += v.x; a.y += v.y; a.z += v.z; a.w += v.w;
      }
      reinterpret_cast<float4*>(d_k + (int64_t)j * dm.HD4 * 4)[f] = a;
    }
    __syncthreads();
  }
}

int check_dims(int H, int D, int C, Dims& dm, int& ks) {
  if (H <= 0 || D <= 0 || C <= 0) return E2A_ERR_ARG;
  if (H % 4 || kThreads % H) return E2A_ERR_UNSUPPORTED;
  if (D % 4) return E2A_ERR_UNSUPPORTED;
  const int g = D / 4;
  if (g > 32 || (g & (g - 1))) return E2A_ERR_UNSUPPORTED;
  if ((C * H) % 4) return E2A_ERR_UNSUPPORTED;
  if (H * D / 4 > 32 * 8) return E2A_ERR_UNSUPPORTED;
  dm.H = H; dm.D = D; dm.C = C; dm.HD4 = H * D / 4; dm.CH4 = C * H / 4; dm.g = g;
  const int need = (dm.CH4 + kThreads - 1) / kThreads;
  if (need <= 1) ks = 1;
  else if (need <= 2) ks = 2;
  else if (need <= 4) ks = 4;
  else if (need <= 8) ks = 8;
  else if (need <= 16) ks = 16;
  else return E2A_ERR_UNSUPPORTED;
  return E2A_OK;
}

int grid_for(int64_t rows) {
  int64_t g = rows;
  if (g > (int64_t)1 << 30) g = (int64_t)1 << 30;
  return (int)(g > 0 ? g : 1);
}

template <typename Kern>
cudaError_t prep_smem(Kern kern, size_t smem) {
  if (smem > 48 * 1024) return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  return cudaSuccess;
}

}  // namespace

#define E2A_DISPATCH_KS(ks, KERN, ...)                               \
  switch (ks) {                                                      \
    case 1: { auto kf = KERN<1>; __VA_ARGS__; break; }               \
    case 2: { auto kf = KERN<2>; __VA_ARGS__; break; }               \
    case 4: { auto kf = KERN<4>; __VA_ARGS__; break; }               \
    case 8: { auto kf = KERN<8>; __VA_ARGS__; break; }               \
    default: { auto kf = KERN<16>; __VA_ARGS__; break; }             \
  }

extern "C" {

int e2a_attn_fwd(const float* q, const float* k, const float* value, const float* gate, const float* inputhead,
                 int64_t ld_gi, const float* poly, const float* dist, const int32_t* row_ptr, const int32_t* col,
                 const int32_t* row_order, int64_t n_rows, int64_t n_keys, int64_t n_edges, int H, int D, int C,
                 float* out, float* beta, float* row_max, float* row_sum, void* stream) {
  Dims dm;
  int ks;
  int rc = check_dims(H, D, C, dm, ks);
  if (rc) return rc;
  if (n_rows < 0 || n_keys < 0 || n_edges < 0 || ld_gi < H || n_edges > INT32_MAX) return E2A_ERR_ARG;
  if (n_rows == 0) return E2A_OK;
  if (!q || !row_ptr || !out || !row_max || !row_sum) return E2A_ERR_ARG;
  if (n_edges > 0 && (!k || !value || !gate || !inputhead || !poly || !dist || !col || !beta)) return E2A_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const size_t smem = (size_t)dm.HD4 * 16 + (kThreads + 2 * H) * 4;
  E2A_DISPATCH_KS(ks, k_attn_fwd, {
    E2A_CUDA(prep_smem(kf, smem));
    kf<<<grid_for(n_rows), kThreads, smem, st>>>(q, k, value, gate, inputhead, ld_gi, poly, dist, row_ptr, col,
                                                 row_order, n_rows, dm, out, beta, row_max, row_sum);
  });
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

size_t e2a_attn_bwd_workspace_bytes(int64_t n_edges, int H) {
  return 2 * e2a_align_up((size_t)(n_edges > 0 ? n_edges : 1) * H * 4, 256) + 512;
}

int e2a_attn_bwd_query(const float* q, const float* k, const float* value, const float* gate,
                       const float* inputhead, int64_t ld_gi, const float* poly, const float* dist,
                       const int32_t* row_ptr, const int32_t* col, const int32_t* row_order, int64_t n_rows,
                       int64_t n_keys, int64_t n_edges, int H, int D, int C, const float* beta, const float* row_max,
                       const float* row_sum, const float* dout, float* d_q, float* d_gate, float* d_inputhead,
                       int64_t ld_dgi, float* d_poly, float* d_dist, float* d_logit, void* workspace,
                       size_t workspace_bytes, void* stream) {
  Dims dm;
  int ks;
  int rc = check_dims(H, D, C, dm, ks);
  if (rc) return rc;
  if (n_rows < 0 || n_keys < 0 || n_edges < 0 || ld_gi < H || ld_dgi < H || n_edges > INT32_MAX) return E2A_ERR_ARG;
  if (n_rows == 0) return E2A_OK;
  if (!q || !row_ptr || !d_q) return E2A_ERR_ARG;
  if (n_edges > 0 && (!k || !value || !gate || !inputhead || !poly || !dist || !col || !beta || !dout ||
                      !d_gate || !d_inputhead || !d_poly || !d_dist || !d_logit))
    return E2A_ERR_ARG;
  if (workspace_bytes < e2a_attn_bwd_workspace_bytes(n_edges, H)) return E2A_ERR_WORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  E2aArena ar{(char*)workspace, workspace_bytes, 0};
  const size_t half = (size_t)(n_edges > 0 ? n_edges : 1) * H * 4;
  float* bufA = (float*)ar.take(half);
  float* bufB = (float*)ar.take(half);
  if (!bufA || !bufB) return E2A_ERR_WORKSPACE;
  const size_t smem = (size_t)kEB * kThreads * 16 + (size_t)dm.HD4 * 16 + (kThreads + 3 * H) * 4;
  if ((size_t)kEB * kThreads < (size_t)kWarps * dm.HD4) return E2A_ERR_UNSUPPORTED;
  E2A_DISPATCH_KS(ks, k_attn_bwd_query, {
    E2A_CUDA(prep_smem(kf, smem));
    kf<<<grid_for(n_rows), kThreads, smem, st>>>(q, k, value, gate, inputhead, ld_gi, poly, dist, row_ptr, col,
                                                 row_order, n_rows, dm, beta, row_max, row_sum, dout, d_q, d_gate,
                                                 d_inputhead, ld_dgi, d_poly, d_dist, d_logit, bufA, bufB);
  });
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

int e2a_attn_bwd_key(const float* q, const float* dout, const float* beta, const float* d_logit,
                     const int32_t* k_row_ptr, const int32_t* k_col, const int32_t* k_perm, int64_t n_rows,
                     int64_t n_keys, int64_t n_edges, int H, int D, int C, float* d_k, float* d_value,
                     void* stream) {
  Dims dm;
  int ks;
  int rc = check_dims(H, D, C, dm, ks);
  if (rc) return rc;
  if (n_rows < 0 || n_keys < 0 || n_edges < 0) return E2A_ERR_ARG;
  if (n_keys == 0) return E2A_OK;
  if (!k_row_ptr || !d_k || !d_value) return E2A_ERR_ARG;
  if (n_edges > 0 && (!q || !dout || !beta || !d_logit || !k_col || !k_perm)) return E2A_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const size_t smem = (size_t)kWarps * dm.HD4 * 16;
  E2A_DISPATCH_KS(ks, k_attn_bwd_key, {
    E2A_CUDA(prep_smem(kf, smem));
    kf<<<grid_for(n_keys), kThreads, smem, st>>>(q, dout, beta, d_logit, k_row_ptr, k_col, k_perm, n_keys, dm, d_k,
                                                 d_value);
  });
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------
// Query-side backward without any allocation (no counterpart in the reference).
//
// Some callers cannot allocate device memory at the moment they call the backward: code running
// inside a host framework whose allocator they do not own, plugins that are handed only the tensors
// of one operator, or code paths that must not call cudaMalloc (which synchronises the device).
// For them this variant keeps its scratch (two [E, H] fp32 buffers) in a fixed array in the
// library's device memory instead of a caller workspace.
//
// Limits and behaviour:
//  * the scratch holds kNoAllocScratchFloats floats (2 x 2^20 floats = 8 MiB); calls with
//    n_edges * H > 2^20 are rejected with E2A_ERR_WORKSPACE;
//  * every GPU that loads the library holds the 8 MiB array until the process exits;
//  * the first call on a device looks up the array's device address (cudaGetSymbolAddress) with
//    that device current; make that first call before any stream capture;
//  * all calls share the one array: calls whose execution overlaps on the GPU (different streams,
//    or different host threads on one device) race and corrupt each other's results.  Nothing in the
//    array needs to start at zero: every scratch element is written before it is read in a call.
// ------------------------------------------------------------------------------------------------
namespace {
constexpr size_t kNoAllocScratchFloats = (size_t)2 << 20;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];
constexpr int kMaxDevices = 64;
float* g_noalloc_ptr[kMaxDevices] = {nullptr};
}  // namespace

extern "C" int e2a_attn_bwd_query_noalloc(
    const float* q, const float* k, const float* value, const float* gate, const float* inputhead, int64_t ld_gi,
    const float* poly, const float* dist, const int32_t* row_ptr, const int32_t* col, const int32_t* row_order,
    int64_t n_rows, int64_t n_keys, int64_t n_edges, int H, int D, int C, const float* beta, const float* row_max,
    const float* row_sum, const float* dout, float* d_q, float* d_gate, float* d_inputhead, int64_t ld_dgi,
    float* d_poly, float* d_dist, float* d_logit, void* stream) {
  Dims dm;
  int ks;
  int rc = check_dims(H, D, C, dm, ks);
  if (rc) return rc;
  if (n_rows < 0 || n_keys < 0 || n_edges < 0 || ld_gi < H || ld_dgi < H || n_edges > INT32_MAX) return E2A_ERR_ARG;
  if ((size_t)n_edges * (size_t)H > kNoAllocScratchFloats / 2) return E2A_ERR_WORKSPACE;  // beyond the fixed scratch
  if (n_rows == 0) return E2A_OK;
  if (!q || !row_ptr || !d_q) return E2A_ERR_ARG;
  if (n_edges > 0 && (!k || !value || !gate || !inputhead || !poly || !dist || !col || !beta || !dout ||
                      !d_gate || !d_inputhead || !d_poly || !d_dist || !d_logit))
    return E2A_ERR_ARG;
  int dev = 0;
  E2A_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return E2A_ERR_UNSUPPORTED;
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    E2A_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  float* bufA = g_noalloc_ptr[dev];
  float* bufB = bufA + kNoAllocScratchFloats / 2;
  cudaStream_t st = (cudaStream_t)stream;
  const size_t smem = (size_t)kEB * kThreads * 16 + (size_t)dm.HD4 * 16 + (kThreads + 3 * H) * 4;
  if ((size_t)kEB * kThreads < (size_t)kWarps * dm.HD4) return E2A_ERR_UNSUPPORTED;
  E2A_DISPATCH_KS(ks, k_attn_bwd_query, {
    E2A_CUDA(prep_smem(kf, smem));
    kf<<<grid_for(n_rows), kThreads, smem, st>>>(q, k, value, gate, inputhead, ld_gi, poly, dist, row_ptr, col,
                                                 row_order, n_rows, dm, beta, row_max, row_sum, dout, d_q, d_gate,
                                                 d_inputhead, ld_dgi, d_poly, d_dist, d_logit, bufA, bufB);
  });
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}
