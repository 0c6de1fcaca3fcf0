// Sparse attention span of E2AttentionArbOrder_sparse (QK logits, segmented softmax with the
// reference's non-standard eps/envelope, alpha/r, value aggregation) and its first-order backward.
//
// Layout (fp32, row-major): q [N,H,D] (already scaled by 1/sqrt(D)), k [M,H,D], value [M,C,H] (the
// merged SO(2)+irreps message, head innermost), gate / inputhead [E,H] views (row stride ld_gi),
// poly/dist [E].  Edges are in query-CSR order; edge id == CSR slot.
//
// Each C-ABI entry point launches a short pipeline of kernels of two kinds:
//  * softmax kernels (one CTA per destination row): q.k logits with one warp per edge, then row
//    reductions with one thread per head.  Few registers, so many CTAs stay resident and the latency
//    of the row-sequential phases is hidden by occupancy.
//  * row-aggregation kernels (one CTA per output row): out[r] = sum_p w[p] * X[col[p]] where every
//    X row is a contiguous row (29.7 KB value / cotangent rows, 4 KB q / k rows).  Each thread owns
//    fixed float4 slots of the row, so every gathered row is read with fully coalesced 16-byte loads
//    and accumulated in registers; register use is bounded so that enough CTAs are resident to keep
//    the gathers in flight.  Rows run in a spatially coherent (Morton) order so that concurrently
//    running CTAs share their gathered rows in L2.
// Every sum over edges runs in CSR order inside one CTA: deterministic, no atomics.
#include <mutex>

#include "e2a_common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr float kSoftmaxEps = 1e-3f;   // e2former.py:364
constexpr float kMinDist = 1e-6f;      // e2former.py:422 clamp_min
constexpr int kEB = 8;                 // edges per cross-thread reduction batch in the d(beta) kernel

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
  for (int f = threadIdx.x; f < n4; f += kThreads) reinterpret_cast<float4*>(dst)[f] = ldg4(src + 4 * f);
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
// CSR row aggregation: out[r, :] = sum_{p in row r} w[e_p, head(f)] * X[col[p], f]
//   HEAD_INNER = true : rows are [C, H] (head = f % H, four heads per float4)
//   HEAD_INNER = false: rows are [H, D] (head = f / D, one head per float4, D % 4 == 0)
// e_p = perm[p] (or p).  One CTA per output row, launched over the rows in `order`.
// ------------------------------------------------------------------------------------------------
template <int KS, bool HEAD_INNER, int MINB = 3, typename T = float>
__global__ void __launch_bounds__(kThreads, MINB)
k_row_agg(const T* __restrict__ X, const float* __restrict__ w, int H, int D, int row_f4,
          const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col, const int32_t* __restrict__ perm,
          const int32_t* __restrict__ order, int64_t n_rows, float* __restrict__ out) {
  for (int64_t r = blockIdx.x; r < n_rows; r += gridDim.x) {
    const int i = row_of(order, r);
    const int rs = row_ptr[i], re = row_ptr[i + 1];
    float4 acc[KS];
#pragma unroll
    for (int s = 0; s < KS; ++s) acc[s] = f4_zero();
    const int h0 = HEAD_INNER ? (4 * threadIdx.x) % H : 0;
    int p = rs;
    if constexpr (!HEAD_INNER && KS == 1) {
      // one float4 per thread and edge: gather four edges at a time (more loads in flight), then
      // accumulate them in CSR order (the same sum, term by term)
      const int f = threadIdx.x;
      if (f < row_f4) {
        const int hcol = (4 * f) / D;
        for (; p + 4 <= re; p += 4) {
          float4 x[4];
          float wv[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int64_t e = perm ? perm[p + u] : p + u;
            x[u] = ld4v(X, (int64_t)col[p + u] * row_f4 * 4 + 4 * f);
            wv[u] = __ldg(w + e * H + hcol);
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) acc[0] = f4_fma(wv[u], x[u], acc[0]);
        }
      }
    }
    for (; p < re; ++p) {
      const int64_t e = perm ? perm[p] : p;
      const int64_t xr = (int64_t)col[p] * row_f4 * 4;   // row start, in values
      if (HEAD_INNER) {
        const float4 b = ldg4(w + e * H + h0);
#pragma unroll
        for (int s = 0; s < KS; ++s) {
          const int f = threadIdx.x + s * kThreads;
          if (f < row_f4) acc[s] = f4_fma4(b, ld4v(X, xr + 4 * f), acc[s]);
        }
      } else {
#pragma unroll
        for (int s = 0; s < KS; ++s) {
          const int f = threadIdx.x + s * kThreads;
          if (f < row_f4) acc[s] = f4_fma(__ldg(w + e * H + (4 * f) / D), ld4v(X, xr + 4 * f), acc[s]);
        }
      }
    }
    float* orow = out + (int64_t)i * row_f4 * 4;
#pragma unroll
    for (int s = 0; s < KS; ++s) {
      const int f = threadIdx.x + s * kThreads;
      if (f < row_f4) reinterpret_cast<float4*>(orow)[f] = acc[s];
    }
  }
}

// ------------------------------------------------------------------------------------------------
// CSR row aggregation of bf16 [C, H] rows: out[r, :] = sum_{p in row r} w[e_p, f % H] * X[col[p], f], one
// CTA per output row.  Each thread owns KS groups of eight consecutive values (one 16-byte load of eight
// bf16, widened to fp32 exactly; eight consecutive heads, H % 8 == 0), fp32 sums and output.  Edges are
// gathered two at a time (more loads in flight) and accumulated in CSR order.
// ------------------------------------------------------------------------------------------------
template <int KS>
__global__ void __launch_bounds__(kThreads, 3)
k_row_agg_bf16(const uint4* __restrict__ X, const float* __restrict__ w, int H, int row_f8,
               const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col, const int32_t* __restrict__ perm,
               int64_t n_rows, float* __restrict__ out) {
  for (int64_t r = blockIdx.x; r < n_rows; r += gridDim.x) {
    const int rs = row_ptr[r], re = row_ptr[r + 1];
    float4 acc[2 * KS];
#pragma unroll
    for (int s = 0; s < 2 * KS; ++s) acc[s] = f4_zero();
    const int h0 = (8 * threadIdx.x) % H;   // the same heads for every slot (kThreads * 8 is a multiple of H)
    int p = rs;
    for (; p + 2 <= re; p += 2) {
      uint4 x[2][KS];
      float4 b[2][2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int64_t e = perm ? perm[p + u] : p + u;
        const uint4* xr = X + (int64_t)col[p + u] * row_f8;
        b[u][0] = ldg4(w + e * H + h0);
        b[u][1] = ldg4(w + e * H + h0 + 4);
#pragma unroll
        for (int s = 0; s < KS; ++s) {
          const int f = threadIdx.x + s * kThreads;
          x[u][s] = f < row_f8 ? __ldg(xr + f) : make_uint4(0u, 0u, 0u, 0u);
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int s = 0; s < KS; ++s) {
          const uint4 v = x[u][s];
          acc[2 * s] = f4_fma4(b[u][0], make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u),
                                                    __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xFFFF0000u)),
                               acc[2 * s]);
          acc[2 * s + 1] = f4_fma4(b[u][1], make_float4(__uint_as_float(v.z << 16), __uint_as_float(v.z & 0xFFFF0000u),
                                                        __uint_as_float(v.w << 16), __uint_as_float(v.w & 0xFFFF0000u)),
                                   acc[2 * s + 1]);
        }
    }
    for (; p < re; ++p) {
      const int64_t e = perm ? perm[p] : p;
      const uint4* xr = X + (int64_t)col[p] * row_f8;
      const float4 b0 = ldg4(w + e * H + h0), b1 = ldg4(w + e * H + h0 + 4);
#pragma unroll
      for (int s = 0; s < KS; ++s) {
        const int f = threadIdx.x + s * kThreads;
        if (f < row_f8) {
          const uint4 v = __ldg(xr + f);
          acc[2 * s] = f4_fma4(b0, make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u),
                                               __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xFFFF0000u)), acc[2 * s]);
          acc[2 * s + 1] = f4_fma4(b1, make_float4(__uint_as_float(v.z << 16), __uint_as_float(v.z & 0xFFFF0000u),
                                                   __uint_as_float(v.w << 16), __uint_as_float(v.w & 0xFFFF0000u)),
                                   acc[2 * s + 1]);
        }
      }
    }
    float4* orow = reinterpret_cast<float4*>(out + r * (int64_t)row_f8 * 8);
#pragma unroll
    for (int s = 0; s < KS; ++s) {
      const int f = threadIdx.x + s * kThreads;
      if (f < row_f8) {
        orow[2 * f] = acc[2 * s];
        orow[2 * f + 1] = acc[2 * s + 1];
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------
// Key-side value backward, fused: one CTA per key row k (key CSR, spatial key order).  For every edge
// e = (i -> k) the destination cotangent row dout[i] ([C,H] layout, channel = c*H + h) is gathered
// once and serves both products:
//   d_value[k] += beta[e,h] dout[i]                       (the value aggregation's transpose)
//   d_beta[e,h] = sum_c dout[i,c,h] value[k,c,h]          (the aggregation's weight gradient)
// The key's own value row sits in shared memory (each thread owns KS float4 slots, all of the same four
// heads, and reads back only what it wrote), which keeps registers for 3 resident CTAs; d_beta partials of a batch of kVB edges are combined across the warps in shared memory.
// Requires H dividing 1024 and H <= 128 (a thread's slots share heads, every warp covers all head
// quads, one batch is one float4 per thread) and the [C,H] channel layout.
// ------------------------------------------------------------------------------------------------
template <int KS>
__global__ void __launch_bounds__(kThreads, 3)
k_value_bwd(const float* __restrict__ value, const float* __restrict__ dout, const float* __restrict__ beta, int H,
            int row_f4, const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col,
            const int32_t* __restrict__ perm, const int32_t* __restrict__ order, int64_t n_rows,
            float* __restrict__ d_value, float* __restrict__ d_beta) {
  extern __shared__ float4 smem4[];
  float4* part = smem4;                       // [kWarps][kVB = 1024 / H][H / 4]
  float4* vv = smem4 + kThreads * kWarps;     // the key's value row [row_f4]
  const int H4 = H / 4, vb = kThreads / H4;   // edges per batch
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int hq = threadIdx.x % H4;            // this thread's head quad (heads 4 hq .. 4 hq + 3)
  for (int64_t r = blockIdx.x; r < n_rows; r += gridDim.x) {
    const int kk = row_of(order, r);
    const int rs = row_ptr[kk], re = row_ptr[kk + 1];
    const float4* vr = reinterpret_cast<const float4*>(value + (int64_t)kk * row_f4 * 4);
    float4 acc[KS];
#pragma unroll
    for (int s = 0; s < KS; ++s) {   // each thread reads back only the slots it wrote: no barrier
      const int f = threadIdx.x + s * kThreads;
      if (f < row_f4) vv[f] = __ldg(vr + f);
      acc[s] = f4_zero();
    }
    for (int p0 = rs; p0 < re; p0 += vb) {
      const int nb = min(vb, re - p0);
      for (int b = 0; b < nb; ++b) {
        const int p = p0 + b;
        const int64_t e = perm[p];
        const float4* xr = reinterpret_cast<const float4*>(dout + (int64_t)col[p] * row_f4 * 4);
        const float4 bw = ldg4(beta + e * H + 4 * hq);
        float4 pt = f4_zero();
#pragma unroll
        for (int s = 0; s < KS; ++s) {
          const int f = threadIdx.x + s * kThreads;
          if (f < row_f4) {
            const float4 x = __ldg(xr + f);
            acc[s] = f4_fma4(bw, x, acc[s]);
            pt = f4_fma4(x, vv[f], pt);
          }
        }
        // lanes of one warp cover head quads (32 * warp + lane) % H4; fold the warp's duplicates
        for (int o = H4; o < 32; o <<= 1) {
          pt.x += __shfl_xor_sync(0xffffffffu, pt.x, o);
          pt.y += __shfl_xor_sync(0xffffffffu, pt.y, o);
          pt.z += __shfl_xor_sync(0xffffffffu, pt.z, o);
          pt.w += __shfl_xor_sync(0xffffffffu, pt.w, o);
        }
        if (lane < H4 || H4 >= 32) part[(warp * vb + b) * H4 + hq] = pt;
      }
      __syncthreads();
      {  // thread t finalises head quad t % H4 of batch edge t / H4 (warp partials in fixed order)
        const int b = threadIdx.x / H4;
        if (b < nb) {
          float4 sum = f4_zero();
          for (int w = 0; w < kWarps; ++w) {
            const float4 v = part[(w * vb + b) * H4 + hq];
            sum.x += v.x; sum.y += v.y; sum.z += v.z; sum.w += v.w;
          }
          *reinterpret_cast<float4*>(d_beta + (int64_t)perm[p0 + b] * H + 4 * hq) = sum;
        }
      }
      __syncthreads();
    }
    float4* orow = reinterpret_cast<float4*>(d_value + (int64_t)kk * row_f4 * 4);
#pragma unroll
    for (int s = 0; s < KS; ++s) {
      const int f = threadIdx.x + s * kThreads;
      if (f < row_f4) orow[f] = acc[s];
    }
  }
}

// ------------------------------------------------------------------------------------------------
// Forward softmax: beta[e,h] = exp(g s - m) poly ih / (S + eps) / max(d, 1e-6), plus row stats
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads)
k_softmax_fwd(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ gate,
              const float* __restrict__ inputhead, int64_t ld_gi, const float* __restrict__ poly,
              const float* __restrict__ dist, const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col,
              const int32_t* __restrict__ order, int64_t n_rows, Dims dm, float* __restrict__ beta,
              float* __restrict__ row_max, float* __restrict__ row_sum) {
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
  }
}

// ------------------------------------------------------------------------------------------------
// Backward: d(beta)[e,h] = sum_c dout[i,c,h] value[j,c,h]  (gather kernel, one CTA per row)
// ------------------------------------------------------------------------------------------------
template <int KS>
__global__ void __launch_bounds__(kThreads, 2)
k_dbeta(const float* __restrict__ value, const float* __restrict__ dout, const int32_t* __restrict__ row_ptr,
        const int32_t* __restrict__ col, const int32_t* __restrict__ order, int64_t n_rows, Dims dm,
        float* __restrict__ dbeta) {
  extern __shared__ float4 smem4[];
  float4* red4 = smem4;  // kEB * kThreads
  const int H = dm.H, H4 = H / 4;
  for (int64_t r = blockIdx.x; r < n_rows; r += gridDim.x) {
    const int i = row_of(order, r);
    const int rs = row_ptr[i], re = row_ptr[i + 1];
    float4 go[KS];
    const float* gr = dout + (int64_t)i * dm.CH4 * 4;
#pragma unroll
    for (int s = 0; s < KS; ++s) {
      const int f = threadIdx.x + s * kThreads;
      go[s] = f < dm.CH4 ? ldg4(gr + 4 * f) : f4_zero();
    }
    for (int e0 = rs; e0 < re; e0 += kEB) {
      const int ne = min(kEB, re - e0);
      for (int b = 0; b < ne; ++b) {
        float4 p = f4_zero();
        const float* vr = value + (int64_t)col[e0 + b] * dm.CH4 * 4;
#pragma unroll
        for (int s = 0; s < KS; ++s) {
          const int f = threadIdx.x + s * kThreads;
          if (f < dm.CH4) p = f4_fma4(go[s], ldg4(vr + 4 * f), p);
        }
        red4[b * kThreads + threadIdx.x] = p;
      }
      __syncthreads();
      // threads sharing head group t % H4 hold partial sums of the same four heads
      for (int o = threadIdx.x; o < ne * H4; o += kThreads) {
        const int b = o / H4, hg = o % H4;
        float4 a = f4_zero();
        for (int t = hg; t < kThreads; t += H4) {
          const float4 v = red4[b * kThreads + t];
          a.x += v.x; a.y += v.y; a.z += v.z; a.w += v.w;
        }
        *reinterpret_cast<float4*>(dbeta + (int64_t)(e0 + b) * H + 4 * hg) = a;
      }
      __syncthreads();
    }
  }
}

// Same d(beta), one warp per edge: the destination cotangent row is staged once in shared memory and
// lane l owns head group l % (H/4) of rows c = l / (H/4) (mod 32 / (H/4)): no cross-warp reduction.
// Requires H/4 to divide 32.
__global__ void __launch_bounds__(kThreads)
k_dbeta_warp(const float* __restrict__ value, const float* __restrict__ dout, const int32_t* __restrict__ row_ptr,
             const int32_t* __restrict__ col, const int32_t* __restrict__ order, int64_t n_rows, Dims dm,
             float* __restrict__ dbeta, const int32_t* __restrict__ perm = nullptr) {
  extern __shared__ float4 smem4[];
  float4* go_s = smem4;  // CH4
  const int H4 = dm.H / 4;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int hg = lane % H4, csub = lane / H4, cstep = 32 / H4;
  for (int64_t r = blockIdx.x; r < n_rows; r += gridDim.x) {
    const int i = row_of(order, r);
    const int rs = row_ptr[i], re = row_ptr[i + 1];
    stage_row(reinterpret_cast<float*>(go_s), dout + (int64_t)i * dm.CH4 * 4, dm.CH4);
    __syncthreads();
    for (int e = rs + warp; e < re; e += kWarps) {
      const float4* vr = reinterpret_cast<const float4*>(value + (int64_t)col[e] * dm.CH4 * 4);
      float4 a0 = f4_zero(), a1 = f4_zero();
      int c = csub;
#pragma unroll 4
      for (; c + cstep < dm.C; c += 2 * cstep) {
        const int f0 = c * H4 + hg, f1 = (c + cstep) * H4 + hg;
        a0 = f4_fma4(go_s[f0], __ldg(vr + f0), a0);
        a1 = f4_fma4(go_s[f1], __ldg(vr + f1), a1);
      }
      if (c < dm.C) a0 = f4_fma4(go_s[c * H4 + hg], __ldg(vr + c * H4 + hg), a0);
      a0.x += a1.x; a0.y += a1.y; a0.z += a1.z; a0.w += a1.w;
      for (int o = H4; o < 32; o <<= 1) {
        a0.x += __shfl_xor_sync(0xffffffffu, a0.x, o);
        a0.y += __shfl_xor_sync(0xffffffffu, a0.y, o);
        a0.z += __shfl_xor_sync(0xffffffffu, a0.z, o);
        a0.w += __shfl_xor_sync(0xffffffffu, a0.w, o);
      }
      if (csub == 0) *reinterpret_cast<float4*>(dbeta + (int64_t)(perm ? perm[e] : e) * dm.H + 4 * hg) = a0;
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------------------------------------
// Backward softmax: from d(beta) (bufA) to d_gate, d_inputhead, d_poly, d_dist and ds = d_logit
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads)
k_softmax_bwd(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ gate,
              const float* __restrict__ inputhead, int64_t ld_gi, const float* __restrict__ poly,
              const float* __restrict__ dist, const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col,
              const int32_t* __restrict__ order, int64_t n_rows, Dims dm, const float* __restrict__ beta,
              const float* __restrict__ row_max, const float* __restrict__ row_sum, float* __restrict__ d_gate,
              float* __restrict__ d_inputhead, int64_t ld_dgi, float* __restrict__ d_poly,
              float* __restrict__ d_dist, float* __restrict__ d_logit, const float* __restrict__ bufA,
              float* __restrict__ bufB) {
  extern __shared__ float4 smem4[];
  float* q_s = reinterpret_cast<float*>(smem4);  // H*D
  float* red = q_s + dm.HD4 * 4;                 // kThreads
  float* T_s = red + kThreads;                   // H
  float* dm_s = T_s + dm.H;                      // H
  float* nt_s = dm_s + dm.H;                     // H
  const int H = dm.H;
  const int stripes = kThreads / H;
  const int hh = threadIdx.x % H, stripe = threadIdx.x / H;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t r = blockIdx.x; r < n_rows; r += gridDim.x) {
    const int i = row_of(order, r);
    const int rs = row_ptr[i], re = row_ptr[i + 1];
    if (rs == re) continue;
    stage_row(q_s, q + (int64_t)i * dm.HD4 * 4, dm.HD4);
    __syncthreads();
    // s = q.k -> bufB
    edge_scores(q_s, k, col, rs, re, dm, [&](int e, int h, float s) { bufB[(int64_t)e * H + h] = s; });
    __syncthreads();
    const float m = row_max[(int64_t)i * H + hh];
    const float S = row_sum[(int64_t)i * H + hh];
    const float den = S + kSoftmaxEps;
    // T_h = sum_e d_alpha * alpha
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
    // dz = dx * x; d_inputhead; accumulate dm and tie counts
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
    // da = dz + [a == m] dm / n_ties (PyTorch's amax rule); d_gate = da * s; d_logit = ds = da * gate
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
    // per-edge sums over heads: d_dist = -sum_h dbeta * beta / r ; d_poly = sum_h dx * exp(a-m)
    for (int e = rs + warp; e < re; e += kWarps) {
      const float d = dist[e];
      const float rr = fmaxf(d, kMinDist);
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
      }
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------------------------------------
// Warp-per-row softmax kernels for H = 32 * HPL heads of width D (full config: HPL = 4, D = 8):
// lane l owns heads [l*HPL, (l+1)*HPL), so every per-head row statistic is lane-local and the q.k
// dot needs only the lane's own HPL*D-float slice of each k row (coalesced across the warp).
// ------------------------------------------------------------------------------------------------
template <int HPL, int D, int MINB = 1, bool KEEP_S = false>
__global__ void __launch_bounds__(kThreads, MINB)
k_softmax_fwd_warp(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ gate,
                   const float* __restrict__ inputhead, int64_t ld_gi, const float* __restrict__ poly,
                   const float* __restrict__ dist, const int32_t* __restrict__ row_ptr,
                   const int32_t* __restrict__ col, const int32_t* __restrict__ order, int64_t n_rows,
                   float* __restrict__ beta, float* __restrict__ row_max, float* __restrict__ row_sum,
                   float* __restrict__ s_out = nullptr) {
  static_assert(HPL == 4, "float4 head groups");
  constexpr int H = 32 * HPL, F4 = HPL * D / 4;  // float4 per lane slice
  const int lane = threadIdx.x & 31;
  const int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (r >= n_rows) return;
  const int i = row_of(order, r);
  const int rs = row_ptr[i], re = row_ptr[i + 1];
  float4 qv[F4];
  const float* qr = q + (int64_t)i * H * D + lane * HPL * D;
#pragma unroll
  for (int t = 0; t < F4; ++t) qv[t] = ldg4(qr + 4 * t);
  float m[HPL];
#pragma unroll
  for (int u = 0; u < HPL; ++u) m[u] = -INFINITY;
  for (int e = rs; e < re; ++e) {
    const float* kr = k + (int64_t)col[e] * H * D + lane * HPL * D;
    float sv[HPL];
#pragma unroll
    for (int u = 0; u < HPL; ++u) {
      float acc = 0.f;
#pragma unroll
      for (int t = 0; t < D / 4; ++t) {
        const float4 kv = ldg4(kr + 4 * (u * (D / 4) + t));
        const float4 qq = qv[u * (D / 4) + t];
        acc += qq.x * kv.x + qq.y * kv.y + qq.z * kv.z + qq.w * kv.w;
      }
      sv[u] = acc;
    }
    const float4 g = ldg4(gate + (int64_t)e * ld_gi + lane * HPL);
    const float4 a = make_float4(g.x * sv[0], g.y * sv[1], g.z * sv[2], g.w * sv[3]);
    *reinterpret_cast<float4*>(beta + (int64_t)e * H + lane * HPL) = a;
    if constexpr (KEEP_S) *reinterpret_cast<float4*>(s_out + (int64_t)e * H + lane * HPL) = make_float4(sv[0], sv[1], sv[2], sv[3]);
    m[0] = fmaxf(m[0], a.x); m[1] = fmaxf(m[1], a.y); m[2] = fmaxf(m[2], a.z); m[3] = fmaxf(m[3], a.w);
  }
  float S[HPL] = {0.f, 0.f, 0.f, 0.f};
  for (int e = rs; e < re; ++e) {
    float4* bp = reinterpret_cast<float4*>(beta + (int64_t)e * H + lane * HPL);
    const float4 a = *bp;
    const float p = poly[e];
    const float4 x = make_float4(expf(a.x - m[0]) * p, expf(a.y - m[1]) * p, expf(a.z - m[2]) * p, expf(a.w - m[3]) * p);
    *bp = x;
    S[0] += x.x; S[1] += x.y; S[2] += x.z; S[3] += x.w;
  }
  const float den[HPL] = {S[0] + kSoftmaxEps, S[1] + kSoftmaxEps, S[2] + kSoftmaxEps, S[3] + kSoftmaxEps};
  for (int e = rs; e < re; ++e) {
    float4* bp = reinterpret_cast<float4*>(beta + (int64_t)e * H + lane * HPL);
    const float4 x = *bp;
    const float4 ih = ldg4(inputhead + (int64_t)e * ld_gi + lane * HPL);
    const float rr = fmaxf(dist[e], kMinDist);
    *bp = make_float4(x.x * ih.x / den[0] / rr, x.y * ih.y / den[1] / rr, x.z * ih.z / den[2] / rr,
                      x.w * ih.w / den[3] / rr);
  }
  *reinterpret_cast<float4*>(row_max + (int64_t)i * H + lane * HPL) = make_float4(m[0], m[1], m[2], m[3]);
  *reinterpret_cast<float4*>(row_sum + (int64_t)i * H + lane * HPL) = make_float4(S[0], S[1], S[2], S[3]);
}

template <int HPL, int D, int MINB = 1, bool HAVE_S = false>
__global__ void __launch_bounds__(kThreads, MINB)
k_softmax_bwd_warp(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ gate,
                   const float* __restrict__ inputhead, int64_t ld_gi, const float* __restrict__ poly,
                   const float* __restrict__ dist, const int32_t* __restrict__ row_ptr,
                   const int32_t* __restrict__ col, const int32_t* __restrict__ order, int64_t n_rows,
                   const float* __restrict__ beta, const float* __restrict__ row_max,
                   const float* __restrict__ row_sum, float* __restrict__ d_gate, float* __restrict__ d_inputhead,
                   int64_t ld_dgi, float* __restrict__ d_poly, float* __restrict__ d_dist,
                   float* __restrict__ d_logit, const float* __restrict__ bufA, float* __restrict__ bufB) {
  static_assert(HPL == 4, "float4 head groups");
  constexpr int H = 32 * HPL, F4 = HPL * D / 4;
  const int lane = threadIdx.x & 31;
  const int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (r >= n_rows) return;
  const int i = row_of(order, r);
  const int rs = row_ptr[i], re = row_ptr[i + 1];
  if (rs == re) return;
  const int ho = lane * HPL;
  float4 qv[HAVE_S ? 1 : F4];
  if constexpr (!HAVE_S) {
    const float* qr = q + (int64_t)i * H * D + ho * D;
#pragma unroll
    for (int t = 0; t < F4; ++t) qv[t] = ldg4(qr + 4 * t);
  }
  const float4 mv = ldg4(row_max + (int64_t)i * H + ho), sv4 = ldg4(row_sum + (int64_t)i * H + ho);
  const float m[HPL] = {mv.x, mv.y, mv.z, mv.w};
  const float den[HPL] = {sv4.x + kSoftmaxEps, sv4.y + kSoftmaxEps, sv4.z + kSoftmaxEps, sv4.w + kSoftmaxEps};
  // pass 1: s = q.k -> bufB; T_h = sum_e d_alpha * alpha
  float T[HPL] = {0.f, 0.f, 0.f, 0.f};
  for (int e = rs; e < re; ++e) {
    float s[HPL];
    if constexpr (HAVE_S) {   // the forward's q.k scores, kept (no key-row gather)
      const float4 s4 = ldg4(bufB + (int64_t)e * H + ho);
      s[0] = s4.x; s[1] = s4.y; s[2] = s4.z; s[3] = s4.w;
    } else {
      const float* kr = k + (int64_t)col[e] * H * D + ho * D;
#pragma unroll
      for (int u = 0; u < HPL; ++u) {
        float acc = 0.f;
#pragma unroll
        for (int t = 0; t < D / 4; ++t) {
          const float4 kv = ldg4(kr + 4 * (u * (D / 4) + t));
          const float4 qq = qv[u * (D / 4) + t];
          acc += qq.x * kv.x + qq.y * kv.y + qq.z * kv.z + qq.w * kv.w;
        }
        s[u] = acc;
      }
      *reinterpret_cast<float4*>(bufB + (int64_t)e * H + ho) = make_float4(s[0], s[1], s[2], s[3]);
    }
    const float4 g4 = ldg4(gate + (int64_t)e * ld_gi + ho), ih4 = ldg4(inputhead + (int64_t)e * ld_gi + ho);
    const float4 db4 = *reinterpret_cast<const float4*>(bufA + (int64_t)e * H + ho);
    const float g[HPL] = {g4.x, g4.y, g4.z, g4.w}, ih[HPL] = {ih4.x, ih4.y, ih4.z, ih4.w};
    const float db[HPL] = {db4.x, db4.y, db4.z, db4.w};
    const float p = poly[e], rr = fmaxf(dist[e], kMinDist);
#pragma unroll
    for (int u = 0; u < HPL; ++u) {
      const float x = expf(g[u] * s[u] - m[u]) * p;
      const float al = x * ih[u] / den[u];
      T[u] += (db[u] / rr) * al;
    }
  }
  float dS[HPL];
#pragma unroll
  for (int u = 0; u < HPL; ++u) dS[u] = -T[u] / den[u];
  // pass 2: dz, d_inputhead, d_dist, d_poly, and d_gate = dz * s, ds = dz * gate (beta recomputed in
  // registers); row max gradient dm = -sum dz and tie counts
  float dmacc[HPL] = {0.f, 0.f, 0.f, 0.f}, nt[HPL] = {0.f, 0.f, 0.f, 0.f};
  int em[HPL] = {-1, -1, -1, -1};   // first edge attaining the row max, per head
  for (int e = rs; e < re; ++e) {
    const float4 s4 = *reinterpret_cast<const float4*>(bufB + (int64_t)e * H + ho);
    const float4 g4 = ldg4(gate + (int64_t)e * ld_gi + ho), ih4 = ldg4(inputhead + (int64_t)e * ld_gi + ho);
    const float4 db4 = *reinterpret_cast<const float4*>(bufA + (int64_t)e * H + ho);
    const float s[HPL] = {s4.x, s4.y, s4.z, s4.w}, g[HPL] = {g4.x, g4.y, g4.z, g4.w};
    const float ih[HPL] = {ih4.x, ih4.y, ih4.z, ih4.w}, db[HPL] = {db4.x, db4.y, db4.z, db4.w};
    const float p = poly[e], d = dist[e], rr = fmaxf(d, kMinDist);
    float dih[HPL], dg[HPL], ds[HPL], sd = 0.f, sp = 0.f;
#pragma unroll
    for (int u = 0; u < HPL; ++u) {
      const float a = g[u] * s[u];
      const float ex = expf(a - m[u]);
      const float x = ex * p;
      const float bt = x * ih[u] / den[u] / rr;   // beta, as the forward computes it
      const float dal = db[u] / rr;
      const float dx = dal * ih[u] / den[u] + dS[u];
      dih[u] = dal * x / den[u];
      const float dz = dx * x;
      dmacc[u] -= dz;
      if (a == m[u]) {
        nt[u] += 1.f;
        if (em[u] < 0) em[u] = e;
      }
      sd += db[u] * bt;
      sp += dx * ex;
      dg[u] = dz * s[u];
      ds[u] = dz * g[u];
    }
    *reinterpret_cast<float4*>(d_inputhead + (int64_t)e * ld_dgi + ho) = make_float4(dih[0], dih[1], dih[2], dih[3]);
    *reinterpret_cast<float4*>(d_gate + (int64_t)e * ld_dgi + ho) = make_float4(dg[0], dg[1], dg[2], dg[3]);
    *reinterpret_cast<float4*>(d_logit + (int64_t)e * H + ho) = make_float4(ds[0], ds[1], ds[2], ds[3]);
    sd = e2a_warp_sum(sd);
    sp = e2a_warp_sum(sp);
    if (lane == 0) {
      d_dist[e] = d >= kMinDist ? -sd / rr : 0.f;
      d_poly[e] = sp;
    }
  }
  // the row max passes dm to the edges attaining it, shared equally among ties (PyTorch's amax
  // rule): da = dz + dm / n_ties there, so d_gate += share * s and ds += share * gate.  One edge per
  // head in the common case; a tie re-walks the row for that head only.
#pragma unroll
  for (int u = 0; u < HPL; ++u) {
    if (nt[u] <= 0.f) continue;
    const float share = dmacc[u] / nt[u];
    const int h = ho + u;
    if (nt[u] == 1.f) {
      const int e = em[u];
      const float sv = bufB[(int64_t)e * H + h], gv = __ldg(gate + (int64_t)e * ld_gi + h);
      d_gate[(int64_t)e * ld_dgi + h] += share * sv;
      d_logit[(int64_t)e * H + h] += share * gv;
    } else {
      for (int e = em[u]; e < re; ++e) {
        const float sv = bufB[(int64_t)e * H + h], gv = __ldg(gate + (int64_t)e * ld_gi + h);
        if (gv * sv == m[u]) {
          d_gate[(int64_t)e * ld_dgi + h] += share * sv;
          d_logit[(int64_t)e * H + h] += share * gv;
        }
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------
// Per-edge scores alone (the reference's sparse_qk_edge_index): out[perm[p], h] = <q[i,h,:], k[col[p],h,:]>,
// one warp per query row, lane l owning heads [4l, 4l+4) (128 heads of 8): the row's q slice stays in
// registers and each key row is one coalesced 4 KB gather; two edges are gathered per iteration.
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 4)
k_qk_warp(const float* __restrict__ q, const float* __restrict__ k, const int32_t* __restrict__ row_ptr,
          const int32_t* __restrict__ col, const int32_t* __restrict__ perm, int64_t n_rows,
          float* __restrict__ out) {
  constexpr int H = 128, D = 8, F4 = 4 * D / 4;   // 8 float4 per lane slice
  const int lane = threadIdx.x & 31;
  const int64_t i = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (i >= n_rows) return;
  const int rs = row_ptr[i], re = row_ptr[i + 1];
  if (rs == re) return;
  float4 qv[F4];
  const float* qr = q + i * H * D + lane * 4 * D;
#pragma unroll
  for (int t = 0; t < F4; ++t) qv[t] = ldg4(qr + 4 * t);
  auto dot4 = [&](const float4* kv) {
    float sv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float acc = 0.f;
#pragma unroll
      for (int t = 0; t < D / 4; ++t) {
        const float4 a = qv[u * (D / 4) + t], b = kv[u * (D / 4) + t];
        acc += a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
      }
      sv[u] = acc;
    }
    return make_float4(sv[0], sv[1], sv[2], sv[3]);
  };
  int e = rs;
  for (; e + 2 <= re; e += 2) {
    float4 k0[F4], k1[F4];
    const float* kr0 = k + (int64_t)col[e] * H * D + lane * 4 * D;
    const float* kr1 = k + (int64_t)col[e + 1] * H * D + lane * 4 * D;
#pragma unroll
    for (int t = 0; t < F4; ++t) { k0[t] = ldg4(kr0 + 4 * t); k1[t] = ldg4(kr1 + 4 * t); }
    const int64_t o0 = perm ? perm[e] : e, o1 = perm ? perm[e + 1] : e + 1;
    *reinterpret_cast<float4*>(out + o0 * H + lane * 4) = dot4(k0);
    *reinterpret_cast<float4*>(out + o1 * H + lane * 4) = dot4(k1);
  }
  if (e < re) {
    float4 k0[F4];
    const float* kr0 = k + (int64_t)col[e] * H * D + lane * 4 * D;
#pragma unroll
    for (int t = 0; t < F4; ++t) k0[t] = ldg4(kr0 + 4 * t);
    *reinterpret_cast<float4*>(out + (int64_t)(perm ? perm[e] : e) * H + lane * 4) = dot4(k0);
  }
}

int check_dims(int H, int D, int C, Dims& dm, int& ks) {
  if (H <= 0 || D <= 0 || C <= 0) return E2A_ERR_ARG;
  if (H % 4 || kThreads % H) return E2A_ERR_UNSUPPORTED;
  if (D % 4) return E2A_ERR_UNSUPPORTED;
  const int g = D / 4;
  if (g > 32 || (g & (g - 1))) return E2A_ERR_UNSUPPORTED;
  if ((C * H) % 4) return E2A_ERR_UNSUPPORTED;
  if (H * D / 4 > kThreads) return E2A_ERR_UNSUPPORTED;
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

#define E2A_DISPATCH_KS(ks, KERN, ...)                               \
  switch (ks) {                                                      \
    case 1: { auto kf = KERN<1>; __VA_ARGS__; break; }               \
    case 2: { auto kf = KERN<2>; __VA_ARGS__; break; }               \
    case 4: { auto kf = KERN<4>; __VA_ARGS__; break; }               \
    case 8: { auto kf = KERN<8>; __VA_ARGS__; break; }               \
    default: { auto kf = KERN<16>; __VA_ARGS__; break; }             \
  }

template <int KS, typename T = float>
void agg_ch(const T* X, const float* w, const Dims& dm, const int32_t* row_ptr, const int32_t* col,
            const int32_t* perm, const int32_t* order, int64_t n_rows, float* out, cudaStream_t st) {
  k_row_agg<KS, true, (KS >= 16 ? 2 : 4), T><<<grid_for(n_rows), kThreads, 0, st>>>(X, w, dm.H, dm.D, dm.CH4, row_ptr,
                                                                                  col, perm, order, n_rows, out);
}

// the same aggregation of bf16 [C,H] rows (widened to fp32 as they are loaded; fp32 sums and output)
int launch_agg_ch_bf16(const e2a_bf16x4* X, const float* w, const Dims& dm, int ks, const int32_t* row_ptr,
                       const int32_t* col, const int32_t* perm, const int32_t* order, int64_t n_rows, float* out,
                       cudaStream_t st) {
  switch (ks) {
    case 1: agg_ch<1>(X, w, dm, row_ptr, col, perm, order, n_rows, out, st); break;
    case 2: agg_ch<2>(X, w, dm, row_ptr, col, perm, order, n_rows, out, st); break;
    case 4: agg_ch<4>(X, w, dm, row_ptr, col, perm, order, n_rows, out, st); break;
    case 8: agg_ch<8>(X, w, dm, row_ptr, col, perm, order, n_rows, out, st); break;
    default: agg_ch<16>(X, w, dm, row_ptr, col, perm, order, n_rows, out, st); break;
  }
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

// out rows = CSR aggregation of [C,H] rows (value / cotangent), weights w[E,H]
int launch_agg_ch(const float* X, const float* w, const Dims& dm, int ks, const int32_t* row_ptr, const int32_t* col,
                  const int32_t* perm, const int32_t* order, int64_t n_rows, float* out, cudaStream_t st) {
  switch (ks) {
    case 1: agg_ch<1>(X, w, dm, row_ptr, col, perm, order, n_rows, out, st); break;
    case 2: agg_ch<2>(X, w, dm, row_ptr, col, perm, order, n_rows, out, st); break;
    case 4: agg_ch<4>(X, w, dm, row_ptr, col, perm, order, n_rows, out, st); break;
    case 8: agg_ch<8>(X, w, dm, row_ptr, col, perm, order, n_rows, out, st); break;
    default: agg_ch<16>(X, w, dm, row_ptr, col, perm, order, n_rows, out, st); break;
  }
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

// out rows = CSR aggregation of [H,D] rows (q / k), weights w[E,H]; H*D/4 <= kThreads
int launch_agg_hd(const float* X, const float* w, const Dims& dm, const int32_t* row_ptr, const int32_t* col,
                  const int32_t* perm, const int32_t* order, int64_t n_rows, float* out, cudaStream_t st) {
  k_row_agg<1, false><<<grid_for(n_rows), kThreads, 0, st>>>(X, w, dm.H, dm.D, dm.HD4, row_ptr, col, perm, order,
                                                             n_rows, out);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

// the warp-per-row softmax path: 128 heads of width 8 (4 heads per lane), 16-byte-aligned edge rows
bool warp_softmax_ok(const Dims& dm, int64_t ld_gi) { return dm.H == 128 && dm.D == 8 && ld_gi % 4 == 0; }

size_t softmax_smem(const Dims& dm, int extra_h) { return (size_t)dm.HD4 * 16 + (kThreads + extra_h * dm.H) * 4; }

// Query-side backward with caller-provided scratch bufA/bufB ([E,H] each).
int bwd_query_launch(const float* q, const float* k, const float* value, const float* gate, const float* inputhead,
                     int64_t ld_gi, const float* poly, const float* dist, const int32_t* row_ptr, const int32_t* col,
                     const int32_t* row_order, int64_t n_rows, const Dims& dm, int ks, const float* beta,
                     const float* row_max, const float* row_sum, const float* dout, float* d_q, float* d_gate,
                     float* d_inputhead, int64_t ld_dgi, float* d_poly, float* d_dist, float* d_logit, float* bufA,
                     float* bufB, cudaStream_t st) {
  if (32 % (dm.H / 4) == 0) {
    const size_t wsm = (size_t)dm.CH4 * 16;
    E2A_CUDA(prep_smem(k_dbeta_warp, wsm));
    k_dbeta_warp<<<grid_for(n_rows), kThreads, wsm, st>>>(value, dout, row_ptr, col, row_order, n_rows, dm, bufA,
                                                          nullptr);
  } else {
    const size_t dsm = (size_t)kEB * kThreads * 16;
    E2A_DISPATCH_KS(ks, k_dbeta, {
      E2A_CUDA(prep_smem(kf, dsm));
      kf<<<grid_for(n_rows), kThreads, dsm, st>>>(value, dout, row_ptr, col, row_order, n_rows, dm, bufA);
    });
  }
  E2A_CHECK_LAUNCH();
  if (warp_softmax_ok(dm, ld_gi) && ld_dgi % 4 == 0) {
    k_softmax_bwd_warp<4, 8, 3><<<(int)((n_rows + kWarps - 1) / kWarps), kThreads, 0, st>>>(
        q, k, gate, inputhead, ld_gi, poly, dist, row_ptr, col, row_order, n_rows, beta, row_max, row_sum, d_gate,
        d_inputhead, ld_dgi, d_poly, d_dist, d_logit, bufA, bufB);
  } else {
    const size_t ssm = softmax_smem(dm, 3);
    E2A_CUDA(prep_smem(k_softmax_bwd, ssm));
    k_softmax_bwd<<<grid_for(n_rows), kThreads, ssm, st>>>(q, k, gate, inputhead, ld_gi, poly, dist, row_ptr, col,
                                                           row_order, n_rows, dm, beta, row_max, row_sum, d_gate,
                                                           d_inputhead, ld_dgi, d_poly, d_dist, d_logit, bufA, bufB);
  }
  E2A_CHECK_LAUNCH();
  // d_q[i] = sum_e ds[e] k[j]  (isolated rows get zeros from the empty sum)
  return launch_agg_hd(k, d_logit, dm, row_ptr, col, nullptr, row_order, n_rows, d_q, st);
}

// fused key-side value backward (d_value and d_beta); E2A_ERR_UNSUPPORTED outside its layout
int value_bwd_launch(const float* value, const float* dout, const float* beta, const Dims& dm, int ks,
                     const int32_t* k_row_ptr, const int32_t* k_col, const int32_t* k_perm, const int32_t* key_order,
                     int64_t n_keys, float* d_value, float* d_beta, cudaStream_t st) {
  if (1024 % dm.H != 0 || dm.H > 128) return E2A_ERR_UNSUPPORTED;  // every warp covers all head quads
  // kWarps x (1024 / H edges x H / 4 quads) float4 partials + the key's value row
  const size_t sm = (size_t)kWarps * kThreads * 16 + (size_t)dm.CH4 * 16;
  E2A_DISPATCH_KS(ks, k_value_bwd, {
    E2A_CUDA(prep_smem(kf, sm));
    kf<<<grid_for(n_keys), kThreads, sm, st>>>(value, dout, beta, dm.H, dm.CH4, k_row_ptr, k_col, k_perm, key_order,
                                               n_keys, d_value, d_beta);
  });
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

// query-side backward from a given d_beta: softmax backward + d_q; scratch bufB ([E,H])
// logits != nullptr: bufB holds the forward's q.k scores ([E,H]) and pass 1 reads them instead of
// gathering k rows (warp layout only; the caller checks)
int softmax_bwd_dq_launch(const float* q, const float* k, const float* gate, const float* inputhead, int64_t ld_gi,
                          const float* poly, const float* dist, const int32_t* row_ptr, const int32_t* col,
                          const int32_t* row_order, int64_t n_rows, const Dims& dm, const float* beta,
                          const float* row_max, const float* row_sum, const float* d_beta, float* d_q, float* d_gate,
                          float* d_inputhead, int64_t ld_dgi, float* d_poly, float* d_dist, float* d_logit,
                          float* bufB, cudaStream_t st, bool have_logits = false) {
  if (have_logits) {
    k_softmax_bwd_warp<4, 8, 4, true><<<(int)((n_rows + kWarps - 1) / kWarps), kThreads, 0, st>>>(
        q, k, gate, inputhead, ld_gi, poly, dist, row_ptr, col, row_order, n_rows, beta, row_max, row_sum, d_gate,
        d_inputhead, ld_dgi, d_poly, d_dist, d_logit, d_beta, bufB);
  } else if (warp_softmax_ok(dm, ld_gi) && ld_dgi % 4 == 0) {
    k_softmax_bwd_warp<4, 8, 3><<<(int)((n_rows + kWarps - 1) / kWarps), kThreads, 0, st>>>(
        q, k, gate, inputhead, ld_gi, poly, dist, row_ptr, col, row_order, n_rows, beta, row_max, row_sum, d_gate,
        d_inputhead, ld_dgi, d_poly, d_dist, d_logit, d_beta, bufB);
  } else {
    const size_t ssm = softmax_smem(dm, 3);
    E2A_CUDA(prep_smem(k_softmax_bwd, ssm));
    k_softmax_bwd<<<grid_for(n_rows), kThreads, ssm, st>>>(q, k, gate, inputhead, ld_gi, poly, dist, row_ptr, col,
                                                           row_order, n_rows, dm, beta, row_max, row_sum, d_gate,
                                                           d_inputhead, ld_dgi, d_poly, d_dist, d_logit, d_beta, bufB);
  }
  E2A_CHECK_LAUNCH();
  return launch_agg_hd(k, d_logit, dm, row_ptr, col, nullptr, row_order, n_rows, d_q, st);
}

}  // namespace

extern "C" {

int e2a_attn_fwd_logits(const float* q, const float* k, const float* value, const float* gate,
                        const float* inputhead, int64_t ld_gi, const float* poly, const float* dist,
                        const int32_t* row_ptr, const int32_t* col, const int32_t* row_order, int64_t n_rows,
                        int64_t n_keys, int64_t n_edges, int H, int D, int C, float* out, float* beta, float* row_max,
                        float* row_sum, float* logits, void* stream) {
  Dims dm;
  int ks;
  int rc = check_dims(H, D, C, dm, ks);
  if (rc) return rc;
  if (n_rows < 0 || n_keys < 0 || n_edges < 0 || ld_gi < H || n_edges > INT32_MAX) return E2A_ERR_ARG;
  if (logits && !warp_softmax_ok(dm, ld_gi)) return E2A_ERR_UNSUPPORTED;
  if (n_rows == 0) return E2A_OK;
  if (!q || !row_ptr || !out || !row_max || !row_sum) return E2A_ERR_ARG;
  if (n_edges > 0 && (!k || !value || !gate || !inputhead || !poly || !dist || !col || !beta)) return E2A_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  if (warp_softmax_ok(dm, ld_gi)) {
    // 64 registers: 4 CTAs (32 warps) per SM keep more k-row gathers in flight
    if (logits)
      k_softmax_fwd_warp<4, 8, 4, true><<<(int)((n_rows + kWarps - 1) / kWarps), kThreads, 0, st>>>(
          q, k, gate, inputhead, ld_gi, poly, dist, row_ptr, col, row_order, n_rows, beta, row_max, row_sum, logits);
    else
      k_softmax_fwd_warp<4, 8, 4><<<(int)((n_rows + kWarps - 1) / kWarps), kThreads, 0, st>>>(
          q, k, gate, inputhead, ld_gi, poly, dist, row_ptr, col, row_order, n_rows, beta, row_max, row_sum);
  } else {
    const size_t ssm = softmax_smem(dm, 2);
    E2A_CUDA(prep_smem(k_softmax_fwd, ssm));
    k_softmax_fwd<<<grid_for(n_rows), kThreads, ssm, st>>>(q, k, gate, inputhead, ld_gi, poly, dist, row_ptr, col,
                                                           row_order, n_rows, dm, beta, row_max, row_sum);
  }
  E2A_CHECK_LAUNCH();
  return launch_agg_ch(value, beta, dm, ks, row_ptr, col, nullptr, row_order, n_rows, out, st);
}

int e2a_attn_fwd(const float* q, const float* k, const float* value, const float* gate, const float* inputhead,
                 int64_t ld_gi, const float* poly, const float* dist, const int32_t* row_ptr, const int32_t* col,
                 const int32_t* row_order, int64_t n_rows, int64_t n_keys, int64_t n_edges, int H, int D, int C,
                 float* out, float* beta, float* row_max, float* row_sum, void* stream) {
  return e2a_attn_fwd_logits(q, k, value, gate, inputhead, ld_gi, poly, dist, row_ptr, col, row_order, n_rows, n_keys,
                             n_edges, H, D, C, out, beta, row_max, row_sum, nullptr, stream);
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
  E2aArena ar{(char*)workspace, workspace_bytes, 0};
  const size_t half = (size_t)(n_edges > 0 ? n_edges : 1) * H * 4;
  float* bufA = (float*)ar.take(half);
  float* bufB = (float*)ar.take(half);
  if (!bufA || !bufB) return E2A_ERR_WORKSPACE;
  return bwd_query_launch(q, k, value, gate, inputhead, ld_gi, poly, dist, row_ptr, col, row_order, n_rows, dm, ks,
                          beta, row_max, row_sum, dout, d_q, d_gate, d_inputhead, ld_dgi, d_poly, d_dist, d_logit,
                          bufA, bufB, (cudaStream_t)stream);
}

int e2a_attn_bwd_key(const float* q, const float* dout, const float* beta, const float* d_logit,
                     const int32_t* k_row_ptr, const int32_t* k_col, const int32_t* k_perm, const int32_t* key_order,
                     int64_t n_rows, int64_t n_keys, int64_t n_edges, int H, int D, int C, float* d_k, float* d_value,
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
  rc = launch_agg_ch(dout, beta, dm, ks, k_row_ptr, k_col, k_perm, key_order, n_keys, d_value, st);
  if (rc) return rc;
  return launch_agg_hd(q, d_logit, dm, k_row_ptr, k_col, k_perm, key_order, n_keys, d_k, st);
}


int e2a_attn_bwd_value(const float* value, const float* dout, const float* beta, const int32_t* k_row_ptr,
                       const int32_t* k_col, const int32_t* k_perm, const int32_t* key_order, int64_t n_rows,
                       int64_t n_keys, int64_t n_edges, int H, int D, int C, float* d_value, float* d_beta,
                       void* stream) {
  Dims dm;
  int ks;
  int rc = check_dims(H, D, C, dm, ks);
  if (rc) return rc;
  if (n_rows < 0 || n_keys < 0 || n_edges < 0 || n_edges > INT32_MAX) return E2A_ERR_ARG;
  if (n_keys == 0) return E2A_OK;
  if (!k_row_ptr || !d_value || !value) return E2A_ERR_ARG;
  if (n_edges > 0 && (!dout || !beta || !k_col || !k_perm || !d_beta)) return E2A_ERR_ARG;
  return value_bwd_launch(value, dout, beta, dm, ks, k_row_ptr, k_col, k_perm, key_order, n_keys, d_value, d_beta,
                          (cudaStream_t)stream);
}

size_t e2a_attn_bwd_softmax_workspace_bytes(int64_t n_edges, int H) {
  return e2a_align_up((size_t)(n_edges > 0 ? n_edges : 1) * H * 4, 256) + 256;
}

int e2a_attn_bwd_softmax(const float* q, const float* k, const float* gate, const float* inputhead, int64_t ld_gi,
                         const float* poly, const float* dist, const int32_t* row_ptr, const int32_t* col,
                         const int32_t* row_order, int64_t n_rows, int64_t n_keys, int64_t n_edges, int H, int D,
                         int C, const float* beta, const float* row_max, const float* row_sum, const float* d_beta,
                         float* d_q, float* d_gate, float* d_inputhead, int64_t ld_dgi, float* d_poly, float* d_dist,
                         float* d_logit, void* workspace, size_t workspace_bytes, void* stream) {
  Dims dm;
  int ks;
  int rc = check_dims(H, D, C, dm, ks);
  if (rc) return rc;
  if (n_rows < 0 || n_keys < 0 || n_edges < 0 || ld_gi < H || ld_dgi < H || n_edges > INT32_MAX) return E2A_ERR_ARG;
  if (n_rows == 0) return E2A_OK;
  if (!q || !row_ptr || !d_q) return E2A_ERR_ARG;
  if (n_edges > 0 && (!k || !gate || !inputhead || !poly || !dist || !col || !beta || !d_beta || !d_gate ||
                      !d_inputhead || !d_poly || !d_dist || !d_logit))
    return E2A_ERR_ARG;
  if (workspace_bytes < e2a_attn_bwd_softmax_workspace_bytes(n_edges, H)) return E2A_ERR_WORKSPACE;
  E2aArena ar{(char*)workspace, workspace_bytes, 0};
  float* bufB = (float*)ar.take((size_t)(n_edges > 0 ? n_edges : 1) * H * 4);
  if (!bufB) return E2A_ERR_WORKSPACE;
  return softmax_bwd_dq_launch(q, k, gate, inputhead, ld_gi, poly, dist, row_ptr, col, row_order, n_rows, dm, beta,
                               row_max, row_sum, d_beta, d_q, d_gate, d_inputhead, ld_dgi, d_poly, d_dist, d_logit,
                               bufB, (cudaStream_t)stream);
}

int e2a_attn_bwd_softmax_logits(const float* k, const float* gate, const float* inputhead, int64_t ld_gi,
                                const float* poly, const float* dist, const int32_t* row_ptr, const int32_t* col,
                                const int32_t* row_order, int64_t n_rows, int64_t n_keys, int64_t n_edges, int H,
                                int D, int C, const float* beta, const float* row_max, const float* row_sum,
                                const float* logits, const float* d_beta, float* d_q, float* d_gate,
                                float* d_inputhead, int64_t ld_dgi, float* d_poly, float* d_dist, float* d_logit,
                                void* stream) {
  Dims dm;
  int ks;
  int rc = check_dims(H, D, C, dm, ks);
  if (rc) return rc;
  if (n_rows < 0 || n_keys < 0 || n_edges < 0 || ld_gi < H || ld_dgi < H || n_edges > INT32_MAX) return E2A_ERR_ARG;
  if (!warp_softmax_ok(dm, ld_gi) || ld_dgi % 4) return E2A_ERR_UNSUPPORTED;
  if (n_rows == 0) return E2A_OK;
  if (!row_ptr || !d_q) return E2A_ERR_ARG;
  if (n_edges > 0 && (!k || !gate || !inputhead || !poly || !dist || !col || !beta || !logits || !d_beta ||
                      !d_gate || !d_inputhead || !d_poly || !d_dist || !d_logit))
    return E2A_ERR_ARG;
  return softmax_bwd_dq_launch(nullptr, k, gate, inputhead, ld_gi, poly, dist, row_ptr, col, row_order, n_rows, dm,
                               beta, row_max, row_sum, d_beta, d_q, d_gate, d_inputhead, ld_dgi, d_poly, d_dist,
                               d_logit, const_cast<float*>(logits), (cudaStream_t)stream, true);
}

int e2a_attn_bwd_dk(const float* q, const float* d_logit, const int32_t* k_row_ptr, const int32_t* k_col,
                    const int32_t* k_perm, const int32_t* key_order, int64_t n_rows, int64_t n_keys, int64_t n_edges,
                    int H, int D, int C, float* d_k, void* stream) {
  Dims dm;
  int ks;
  int rc = check_dims(H, D, C, dm, ks);
  if (rc) return rc;
  if (n_rows < 0 || n_keys < 0 || n_edges < 0) return E2A_ERR_ARG;
  if (n_keys == 0) return E2A_OK;
  if (!k_row_ptr || !d_k) return E2A_ERR_ARG;
  if (n_edges > 0 && (!q || !d_logit || !k_col || !k_perm)) return E2A_ERR_ARG;
  return launch_agg_hd(q, d_logit, dm, k_row_ptr, k_col, k_perm, key_order, n_keys, d_k, (cudaStream_t)stream);
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
//    that device current; make that first call before any stream capture.  The address is kept per
//    device together with the id of the CUDA context it was looked up in: when that context is
//    destroyed and a new one made (cudaDeviceReset, a framework tearing its context down), the next
//    call looks the address up again (the array's contents do not survive);
//  * all calls share the one array: calls whose execution overlaps on the GPU (different streams,
//    or different host threads on one device) race and corrupt each other's results.  Nothing in the
//    array needs to start at zero: every scratch element is written before it is read in a call.
// ------------------------------------------------------------------------------------------------
namespace {
constexpr size_t kNoAllocScratchFloats = (size_t)2 << 20;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];
constexpr int kMaxDevices = 64;
struct NoAllocSlot {
  unsigned long long ctx_id = 0;  // id of the context the address belongs to (0: none yet)
  float* ptr = nullptr;
};
NoAllocSlot g_noalloc_slot[kMaxDevices];
std::mutex g_noalloc_mutex;  // set-up may race between host threads

// Unique id of the calling thread's current CUDA context (cuCtxGetCurrent + cuCtxGetId, reached through
// the runtime's driver entry points, so the library needs no link against libcuda); 0 if unavailable.
unsigned long long current_context_id() {
  typedef int (*GetCurrentFn)(void**);
  typedef int (*GetIdFn)(void*, unsigned long long*);
  static GetCurrentFn get_current = nullptr;
  static GetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrentFn>(f);
    f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetIdFn>(f);
  });
  void* ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != 0 || !ctx || get_id(ctx, &id) != 0) return 0;
  return id;
}
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
  const unsigned long long ctx = current_context_id();
  float* bufA = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    NoAllocSlot& slot = g_noalloc_slot[dev];
    if (slot.ptr == nullptr || ctx == 0 || slot.ctx_id != ctx) {  // ctx 0: no id available, look up again
      void* p = nullptr;
      E2A_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
      slot.ptr = static_cast<float*>(p);
      slot.ctx_id = ctx;
    }
    bufA = slot.ptr;
  }
  float* bufB = bufA + kNoAllocScratchFloats / 2;
  return bwd_query_launch(q, k, value, gate, inputhead, ld_gi, poly, dist, row_ptr, col, row_order, n_rows, dm, ks,
                          beta, row_max, row_sum, dout, d_q, d_gate, d_inputhead, ld_dgi, d_poly, d_dist, d_logit,
                          bufA, bufB, (cudaStream_t)stream);
}

// ------------------------------------------------------------------------------------------------
// Fast paths of the kernel-level functions (e2a_sparse.cu's entry points call these first and use their
// generic kernels on E2A_ERR_UNSUPPORTED): the span's row-aggregation, d(beta) and score kernels on
// the layouts they take.
// ------------------------------------------------------------------------------------------------
namespace e2a_fast {

static bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

int agg_ch(const float* X, const float* w, int H, int C, const int32_t* row_ptr, const int32_t* col,
           const int32_t* perm, int64_t n_rows, float* out, cudaStream_t st) {
  if (H <= 0 || C <= 0 || H % 4 || 1024 % H || (C * H) % 4 || (C * H) / 4 > 16 * kThreads) return E2A_ERR_UNSUPPORTED;
  if (!al16(X) || !al16(w) || !al16(out)) return E2A_ERR_UNSUPPORTED;
  Dims dm{};
  dm.H = H; dm.C = C; dm.D = 4; dm.CH4 = C * H / 4; dm.HD4 = H; dm.g = 1;
  const int need = (dm.CH4 + kThreads - 1) / kThreads;
  const int ks = need <= 1 ? 1 : need <= 2 ? 2 : need <= 4 ? 4 : need <= 8 ? 8 : 16;
  return launch_agg_ch(X, w, dm, ks, row_ptr, col, perm, nullptr, n_rows, out, st);
}

int agg_ch_bf16(const void* X, const float* w, int H, int C, const int32_t* row_ptr, const int32_t* col,
                const int32_t* perm, int64_t n_rows, float* out, cudaStream_t st) {
  if (H <= 0 || C <= 0 || H % 4 || 1024 % H || (C * H) % 4 || (C * H) / 4 > 16 * kThreads) return E2A_ERR_UNSUPPORTED;
  if (((uintptr_t)X & 7u) || !al16(w) || !al16(out)) return E2A_ERR_UNSUPPORTED;
  if (H % 8 == 0 && (C * H) % 8 == 0 && al16(X) && (C * H) / 8 <= 4 * kThreads) {
    // 16-byte loads of eight values
    const int f8 = C * H / 8;
    const int need = (f8 + kThreads - 1) / kThreads;
    const uint4* x8 = reinterpret_cast<const uint4*>(X);
    const int g = grid_for(n_rows);
    if (need <= 1) k_row_agg_bf16<1><<<g, kThreads, 0, st>>>(x8, w, H, f8, row_ptr, col, perm, n_rows, out);
    else if (need <= 2) k_row_agg_bf16<2><<<g, kThreads, 0, st>>>(x8, w, H, f8, row_ptr, col, perm, n_rows, out);
    else k_row_agg_bf16<4><<<g, kThreads, 0, st>>>(x8, w, H, f8, row_ptr, col, perm, n_rows, out);
    E2A_CHECK_LAUNCH();
    return E2A_OK;
  }
  Dims dm{};
  dm.H = H; dm.C = C; dm.D = 4; dm.CH4 = C * H / 4; dm.HD4 = H; dm.g = 1;
  const int need = (dm.CH4 + kThreads - 1) / kThreads;
  const int ks = need <= 1 ? 1 : need <= 2 ? 2 : need <= 4 ? 4 : need <= 8 ? 8 : 16;
  return launch_agg_ch_bf16(reinterpret_cast<const e2a_bf16x4*>(X), w, dm, ks, row_ptr, col, perm, nullptr, n_rows,
                            out, st);
}

int agg_hd(const float* X, const float* w, int H, int D, const int32_t* row_ptr, const int32_t* col,
           const int32_t* perm, int64_t n_rows, float* out, cudaStream_t st) {
  if (H <= 0 || D <= 0 || D % 4 || H * D / 4 > kThreads) return E2A_ERR_UNSUPPORTED;
  if (!al16(X) || !al16(out)) return E2A_ERR_UNSUPPORTED;
  Dims dm{};
  dm.H = H; dm.D = D; dm.HD4 = H * D / 4; dm.g = D / 4; dm.C = 1; dm.CH4 = 1;
  return launch_agg_hd(X, w, dm, row_ptr, col, perm, nullptr, n_rows, out, st);
}

int dbeta(const float* value, const float* dout, int H, int C, const int32_t* row_ptr, const int32_t* col,
          const int32_t* perm, int64_t n_rows, float* d_w, cudaStream_t st) {
  if (H <= 0 || C <= 0 || H % 4 || 32 % (H / 4) || (C * H) % 4) return E2A_ERR_UNSUPPORTED;
  if (!al16(value) || !al16(dout) || !al16(d_w)) return E2A_ERR_UNSUPPORTED;
  Dims dm{};
  dm.H = H; dm.C = C; dm.D = 4; dm.CH4 = C * H / 4; dm.HD4 = H; dm.g = 1;
  const size_t wsm = (size_t)dm.CH4 * 16;
  if (wsm > 200 * 1024) return E2A_ERR_UNSUPPORTED;
  E2A_CUDA(prep_smem(k_dbeta_warp, wsm));
  k_dbeta_warp<<<grid_for(n_rows), kThreads, wsm, st>>>(value, dout, row_ptr, col, nullptr, n_rows, dm, d_w, perm);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

int qk(const float* q, const float* k, int H, int D, const int32_t* row_ptr, const int32_t* col,
       const int32_t* perm, int64_t n_rows, float* out, cudaStream_t st) {
  if (H != 128 || D != 8 || !al16(q) || !al16(k) || !al16(out)) return E2A_ERR_UNSUPPORTED;
  k_qk_warp<<<(int)((n_rows + kWarps - 1) / kWarps), kThreads, 0, st>>>(q, k, row_ptr, col, perm, n_rows, out);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

}  // namespace e2a_fast
