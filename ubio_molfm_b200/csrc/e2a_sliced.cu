// Head-sliced gathers of [H, D] rows for the kernel-level functions (the reference's
// sparse_qk_edge_index and its backward) when the caller gives no spatial processing order.  Without
// one, the key rows a query row gathers are spread over the whole table (a 4 KB row per key, ~0.5 GB
// at 1.2e5 keys), most gathers miss L2 and the kernel runs at DRAM speed on the gathered bytes.  Here
// a launch covers one slice of 8 heads (8 x D contiguous floats, 256 B at D = 8) for every output row
// before the next slice starts (the head group is the slow grid dimension), so the slice being
// gathered (keys x 256 B, ~31 MB) stays resident in the 126 MB L2: each table byte comes from DRAM
// about once.  The table is loaded with an evict-last L2 policy, the streamed operands with
// evict-first.
//
// Slicing [C, H] value rows the same way (8 heads = one 32-byte sector per channel) was measured
// slower than gathering whole rows (36-44 ms against 14.2 ms for the 3.2 M-edge value aggregation):
// sector-sized gathers from many lines per warp instruction bound the load path, so value rows are
// gathered whole (e2a_fast::agg_ch).
//
// The aggregation sums a row's edges in CSR order, one fused multiply-add per term: the results equal
// the generic kernel's bit for bit.
#include "e2a_common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kHG = 8;   // heads per slice

// L2 policy for the gathered table's slice (kept in preference to streamed operands)
__device__ __forceinline__ uint64_t l2_keep_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ float4 ldg4_keep(const float* ptr, uint64_t pol) {
  float4 v;
  asm volatile("ld.global.nc.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(ptr), "l"(pol));
  return v;
}

// ------------------------------------------------------------------------------------------------
// out[i, 8g..8g+8, :] = sum_{p in row i} w[e_p, h] * X[col[p], h, :]  ([H, D] rows; the slice is
// 8 x D contiguous floats, one float4 per lane, 2D lanes per row; D in {4, 8, 16}).  Grid: (row blocks, head groups).
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads)
k_agg_hd_sliced(const float* __restrict__ X, const float* __restrict__ w, int H, int D,
                const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col,
                const int32_t* __restrict__ perm, int64_t n_rows, float* __restrict__ out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tpr = 2 * D;   // (8 heads x D floats) / 4
  const int rpw = 32 / tpr;
  const int64_t i = ((int64_t)blockIdx.x * kWarps + warp) * rpw + lane / tpr;
  const int fl = lane % tpr;
  if (i >= n_rows) return;
  const int h0 = blockIdx.y * kHG;
  const int h = h0 + (4 * fl) / D;
  const int64_t HD = (int64_t)H * D, off = (int64_t)h0 * D + 4 * fl;
  const int rs = row_ptr[i], re = row_ptr[i + 1];
  const uint64_t keep = l2_keep_policy();
  float4 acc = f4_zero();
  int p = rs;
  for (; p + 4 <= re; p += 4) {
    float4 x[4];
    float wv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t e = perm ? perm[p + u] : p + u;
      x[u] = ldg4_keep(X + (int64_t)col[p + u] * HD + off, keep);
      wv[u] = __ldcs(w + e * H + h);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) acc = f4_fma(wv[u], x[u], acc);
  }
  for (; p < re; ++p) {
    const int64_t e = perm ? perm[p] : p;
    acc = f4_fma(__ldcs(w + e * H + h), ldg4_keep(X + (int64_t)col[p] * HD + off, keep), acc);
  }
  __stcs(reinterpret_cast<float4*>(out + i * HD + off), acc);
}

// ------------------------------------------------------------------------------------------------
// out[perm[p], h] = <q[i, h, :], k[col[p], h, :]> for the 8 heads of the slice: one warp per query
// row, lane = (edge e % 4, head); each lane keeps its head's q in registers and gathers D floats of a
// key row per edge.  D in {4, 8, 16}.  Grid: (row blocks, head groups).
// ------------------------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kThreads)
k_qk_sliced(const float* __restrict__ q, const float* __restrict__ k, int H, const int32_t* __restrict__ row_ptr,
            const int32_t* __restrict__ col, const int32_t* __restrict__ perm, int64_t n_rows,
            float* __restrict__ out) {
  constexpr int D4 = D / 4;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t i = (int64_t)blockIdx.x * kWarps + warp;
  if (i >= n_rows) return;
  const int es = lane >> 3, h = blockIdx.y * kHG + (lane & 7);
  const int rs = row_ptr[i], re = row_ptr[i + 1];
  const uint64_t keep = l2_keep_policy();
  float4 qv[D4];
#pragma unroll
  for (int t = 0; t < D4; ++t) qv[t] = ldg4(q + (i * H + h) * D + 4 * t);
  auto dot = [&](const float4* kv) {
    float s = 0.f;
#pragma unroll
    for (int t = 0; t < D4; ++t) {
      s = fmaf(qv[t].x, kv[t].x, s);
      s = fmaf(qv[t].y, kv[t].y, s);
      s = fmaf(qv[t].z, kv[t].z, s);
      s = fmaf(qv[t].w, kv[t].w, s);
    }
    return s;
  };
  int p = rs + es;
  for (; p + 4 < re; p += 8) {   // two edges per lane in flight
    float4 k0[D4], k1[D4];
    const float* kr0 = k + ((int64_t)col[p] * H + h) * D;
    const float* kr1 = k + ((int64_t)col[p + 4] * H + h) * D;
#pragma unroll
    for (int t = 0; t < D4; ++t) { k0[t] = ldg4_keep(kr0 + 4 * t, keep); k1[t] = ldg4_keep(kr1 + 4 * t, keep); }
    __stcs(out + (int64_t)(perm ? perm[p] : p) * H + h, dot(k0));
    __stcs(out + (int64_t)(perm ? perm[p + 4] : p + 4) * H + h, dot(k1));
  }
  if (p < re) {
    float4 k0[D4];
    const float* kr0 = k + ((int64_t)col[p] * H + h) * D;
#pragma unroll
    for (int t = 0; t < D4; ++t) k0[t] = ldg4_keep(kr0 + 4 * t, keep);
    __stcs(out + (int64_t)(perm ? perm[p] : p) * H + h, dot(k0));
  }
}

bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

int grid_rows(int64_t n_rows, int rows_per_cta) {
  const int64_t g = (n_rows + rows_per_cta - 1) / rows_per_cta;
  return (int)(g > 0 ? g : 1);
}

}  // namespace

// ------------------------------------------------------------------------------------------------
// Entry points for e2a_sparse.cu (E2A_ERR_UNSUPPORTED outside their layouts).
// ------------------------------------------------------------------------------------------------
namespace e2a_sliced {

int agg_hd(const float* X, const float* w, int H, int D, const int32_t* row_ptr, const int32_t* col,
           const int32_t* perm, int64_t n_rows, float* out, cudaStream_t st) {
  if (H <= 0 || H % kHG || (D != 4 && D != 8 && D != 16) || !al16(X) || !al16(out)) return E2A_ERR_UNSUPPORTED;
  if (H / kHG > 65535 || (n_rows + kWarps - 1) / kWarps > INT32_MAX) return E2A_ERR_UNSUPPORTED;
  const int rows_per_cta = kWarps * (32 / (2 * D));
  dim3 grid(grid_rows(n_rows, rows_per_cta), H / kHG);
  k_agg_hd_sliced<<<grid, kThreads, 0, st>>>(X, w, H, D, row_ptr, col, perm, n_rows, out);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

int qk(const float* q, const float* k, int H, int D, const int32_t* row_ptr, const int32_t* col,
       const int32_t* perm, int64_t n_rows, float* out, cudaStream_t st) {
  if (H <= 0 || H % kHG || H / kHG > 65535 || !al16(q) || !al16(k)) return E2A_ERR_UNSUPPORTED;
  if ((n_rows + kWarps - 1) / kWarps > INT32_MAX) return E2A_ERR_UNSUPPORTED;
  dim3 grid(grid_rows(n_rows, kWarps), H / kHG);
  switch (D) {
    case 4: k_qk_sliced<4><<<grid, kThreads, 0, st>>>(q, k, H, row_ptr, col, perm, n_rows, out); break;
    case 8: k_qk_sliced<8><<<grid, kThreads, 0, st>>>(q, k, H, row_ptr, col, perm, n_rows, out); break;
    case 16: k_qk_sliced<16><<<grid, kThreads, 0, st>>>(q, k, H, row_ptr, col, perm, n_rows, out); break;
    default: return E2A_ERR_UNSUPPORTED;
  }
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

}  // namespace e2a_sliced
