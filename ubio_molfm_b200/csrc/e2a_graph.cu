// Graph construction for the E2Former-V2 attention path: CSR metadata, PBC image expansion and the
// cell-list radius graph.  All of it is integer/byte work plus fp32 distance tests, so it is bound by
// HBM/L2 traffic and latency, not by arithmetic: kernels are warp-per-row with coalesced loads and
// no float atomics; grouping uses integer atomics followed by a deterministic in-segment ordering.
#include <cub/cub.cuh>
#include <stdio.h>
#include <atomic>
#include "e2a_common.cuh"

namespace {

constexpr int kWarpsPerBlock = 8;
constexpr int kSegSmem = 512;  // candidate keys kept in shared memory per warp in the fill kernel

// ------------------------------------------------------------------------------------------------
// Stable group-by: for key[e] in [0, R) produce row_ptr[R+1] and perm (edge ids, ascending inside a
// row), plus other_out[p] = other[perm[p]].
// ------------------------------------------------------------------------------------------------
__global__ void k_count_keys(const int32_t* __restrict__ key, int64_t n, int64_t R,
                             int32_t* __restrict__ counts, int* __restrict__ err) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    int32_t k = key[e];
    if (k < 0 || k >= R) { atomicOr(err, 1); continue; }
    atomicAdd(&counts[k], 1);
  }
}

__global__ void k_scatter_keys(const int32_t* __restrict__ key, int64_t n, int64_t R,
                               int32_t* __restrict__ cursor, int32_t* __restrict__ tmp) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    int32_t k = key[e];
    if (k < 0 || k >= R) continue;
    int32_t slot = atomicAdd(&cursor[k], 1);
    tmp[slot] = (int32_t)e;
  }
}

// One warp per row: place every element of the unordered segment at its rank (edge ids are unique).
__global__ void k_rank_segments(const int32_t* __restrict__ row_ptr, int64_t R,
                                const int32_t* __restrict__ tmp, const int32_t* __restrict__ other,
                                int32_t* __restrict__ perm, int32_t* __restrict__ other_out) {
  const int lane = threadIdx.x & 31;
  int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (; row < R; row += nwarps) {
    const int32_t b = row_ptr[row], n = row_ptr[row + 1] - b;
    if (n == 1) {
      if (lane == 0) { int32_t v = tmp[b]; perm[b] = v; other_out[b] = other[v]; }
      continue;
    }
    for (int t = lane; t < n; t += 32) {
      const int32_t v = tmp[b + t];
      int rank = 0;
      for (int u = 0; u < n; ++u) rank += (tmp[b + u] < v);
      perm[b + rank] = v;
      other_out[b + rank] = other[v];
    }
  }
}

template <typename T>
size_t scan_temp_bytes(int64_t n) {
  size_t bytes = 0;
  cub::DeviceScan::ExclusiveSum(nullptr, bytes, (T*)nullptr, (T*)nullptr, (int)n);
  return bytes;
}

int group_by(const int32_t* key, const int32_t* other, int64_t n, int64_t R, int32_t* row_ptr,
             int32_t* perm, int32_t* other_out, E2aArena& ar, int* d_err, cudaStream_t st) {
  int32_t* counts = (int32_t*)ar.take((R + 1) * sizeof(int32_t));
  int32_t* tmp = (int32_t*)ar.take((n > 0 ? n : 1) * sizeof(int32_t));
  size_t tb = scan_temp_bytes<int32_t>(R + 1);
  void* tstore = ar.take(tb);
  if (!counts || !tmp || !tstore) return E2A_ERR_WORKSPACE;
  E2A_CUDA(cudaMemsetAsync(counts, 0, (R + 1) * sizeof(int32_t), st));
  const int threads = 256;
  int blocks = (int)((n + threads - 1) / threads);
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  if (n > 0) {
    k_count_keys<<<blocks, threads, 0, st>>>(key, n, R, counts, d_err);
    E2A_CHECK_LAUNCH();
  }
  E2A_CUDA(cub::DeviceScan::ExclusiveSum(tstore, tb, counts, row_ptr, (int)(R + 1), st));
  if (n == 0) return E2A_OK;
  E2A_CUDA(cudaMemcpyAsync(counts, row_ptr, R * sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
  k_scatter_keys<<<blocks, threads, 0, st>>>(key, n, R, counts, tmp);
  E2A_CHECK_LAUNCH();
  int64_t wblocks = (R + kWarpsPerBlock - 1) / kWarpsPerBlock;
  if (wblocks > 148 * 32) wblocks = 148 * 32;
  k_rank_segments<<<(int)wblocks, kWarpsPerBlock * 32, 0, st>>>(row_ptr, R, tmp, other, perm, other_out);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

// ------------------------------------------------------------------------------------------------
// Uniform cell grid over a point set (one grid per system).
// ------------------------------------------------------------------------------------------------
struct GridDev {
  float* lo;        // [B,3]
  float* cs;        // [B,3] cell edge
  int* dims;        // [B,3]
  int32_t* cell_off;   // [B+1] first cell id of each system
  int32_t* cell_of;    // [P] cell of each point
  int32_t* cell_start; // [ncap+1]
  int32_t* cell_items; // [P] point ids grouped by cell
};

__global__ void k_sys_bbox(const float* __restrict__ pts, const int64_t* __restrict__ p_ptr, int64_t B,
                           float* __restrict__ lo, float* __restrict__ hi) {
  __shared__ float s[6][32];
  for (int64_t b = blockIdx.x; b < B; b += gridDim.x) {
    float mn[3] = {INFINITY, INFINITY, INFINITY}, mx[3] = {-INFINITY, -INFINITY, -INFINITY};
    for (int64_t p = p_ptr[b] + threadIdx.x; p < p_ptr[b + 1]; p += blockDim.x) {
#pragma unroll
      for (int d = 0; d < 3; ++d) {
        float v = pts[3 * p + d];
        mn[d] = fminf(mn[d], v);
        mx[d] = fmaxf(mx[d], v);
      }
    }
#pragma unroll
    for (int d = 0; d < 3; ++d) {
      for (int o = 16; o > 0; o >>= 1) {
        mn[d] = fminf(mn[d], __shfl_xor_sync(0xffffffffu, mn[d], o));
        mx[d] = fmaxf(mx[d], __shfl_xor_sync(0xffffffffu, mx[d], o));
      }
    }
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
      for (int d = 0; d < 3; ++d) { s[d][w] = mn[d]; s[3 + d][w] = mx[d]; }
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      const int nw = blockDim.x >> 5;
      for (int d = 0; d < 3; ++d) {
        float a = lane < nw ? s[d][lane] : INFINITY;
        float c = lane < nw ? s[3 + d][lane] : -INFINITY;
        for (int o = 16; o > 0; o >>= 1) {
          a = fminf(a, __shfl_xor_sync(0xffffffffu, a, o));
          c = fmaxf(c, __shfl_xor_sync(0xffffffffu, c, o));
        }
        if (lane == 0) { lo[3 * b + d] = a; hi[3 * b + d] = c; }
      }
    }
    __syncthreads();
  }
}

// Cell edge >= cell_min, at most max(1, n_pts) cells per system.
__global__ void k_sys_grid(const float* __restrict__ lo, const float* __restrict__ hi,
                           const int64_t* __restrict__ p_ptr, int64_t B, float cell_min,
                           float* __restrict__ cs, int* __restrict__ dims, int32_t* __restrict__ ncell) {
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < B; b += (int64_t)gridDim.x * blockDim.x) {
    const int64_t np = p_ptr[b + 1] - p_ptr[b];
    double ext[3];
    long long dm[3];
    for (int d = 0; d < 3; ++d) {
      ext[d] = (np > 0) ? (double)hi[3 * b + d] - (double)lo[3 * b + d] : 0.0;
      if (!(ext[d] >= 0.0)) ext[d] = 0.0;
      long long v = (long long)floor(ext[d] / (double)cell_min);
      dm[d] = v < 1 ? 1 : (v > 4096 ? 4096 : v);
    }
    const long long cap = np > 1 ? np : 1;
    while (dm[0] * dm[1] * dm[2] > cap) {
      int a = 0;
      if (dm[1] > dm[a]) a = 1;
      if (dm[2] > dm[a]) a = 2;
      dm[a] = (dm[a] + 1) / 2;
    }
    for (int d = 0; d < 3; ++d) {
      dims[3 * b + d] = (int)dm[d];
      float c = (float)(ext[d] / (double)dm[d]);
      cs[3 * b + d] = (c > cell_min) ? c : cell_min;
    }
    ncell[b] = (int32_t)(dm[0] * dm[1] * dm[2]);
  }
}

__device__ __forceinline__ int cell_coord(float p, float lo, float cs, int dim) {
  int c = (int)floorf((p - lo) / cs);
  return c < 0 ? 0 : (c >= dim ? dim - 1 : c);
}

__global__ void k_bin_points(const float* __restrict__ pts, const int64_t* __restrict__ p_ptr, int64_t B,
                             int64_t P, GridDev g, int32_t* __restrict__ counts) {
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < P; p += (int64_t)gridDim.x * blockDim.x) {
    // system of point p (binary search over p_ptr)
    int64_t lo = 0, hi = B - 1;
    while (lo < hi) {
      int64_t mid = (lo + hi + 1) >> 1;
      if (p_ptr[mid] <= p) lo = mid; else hi = mid - 1;
    }
    const int64_t b = lo;
    int c[3];
    for (int d = 0; d < 3; ++d) c[d] = cell_coord(pts[3 * p + d], g.lo[3 * b + d], g.cs[3 * b + d], g.dims[3 * b + d]);
    const int32_t cell = g.cell_off[b] + (c[0] * g.dims[3 * b + 1] + c[1]) * g.dims[3 * b + 2] + c[2];
    g.cell_of[p] = cell;
    atomicAdd(&counts[cell], 1);
  }
}

__global__ void k_fill_cells(int64_t P, const int32_t* __restrict__ cell_of, int32_t* __restrict__ cursor,
                             int32_t* __restrict__ items) {
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < P; p += (int64_t)gridDim.x * blockDim.x) {
    int32_t slot = atomicAdd(&cursor[cell_of[p]], 1);
    items[slot] = (int32_t)p;
  }
}

int build_grid(const float* pts, const int64_t* p_ptr, int64_t P, int64_t B, float cell_min, GridDev& g,
               E2aArena& ar, cudaStream_t st) {
  const int64_t ncap = P + B;
  float* hi = (float*)ar.take(B * 3 * sizeof(float));
  g.lo = (float*)ar.take(B * 3 * sizeof(float));
  g.cs = (float*)ar.take(B * 3 * sizeof(float));
  g.dims = (int*)ar.take(B * 3 * sizeof(int));
  int32_t* ncell = (int32_t*)ar.take((B + 1) * sizeof(int32_t));
  g.cell_off = (int32_t*)ar.take((B + 1) * sizeof(int32_t));
  g.cell_of = (int32_t*)ar.take((P > 0 ? P : 1) * sizeof(int32_t));
  int32_t* counts = (int32_t*)ar.take((ncap + 1) * sizeof(int32_t));
  g.cell_start = (int32_t*)ar.take((ncap + 1) * sizeof(int32_t));
  g.cell_items = (int32_t*)ar.take((P > 0 ? P : 1) * sizeof(int32_t));
  size_t tb1 = scan_temp_bytes<int32_t>(B + 1), tb2 = scan_temp_bytes<int32_t>(ncap + 1);
  size_t tb = tb1 > tb2 ? tb1 : tb2;
  void* tstore = ar.take(tb);
  if (!hi || !g.lo || !g.cs || !g.dims || !ncell || !g.cell_off || !g.cell_of || !counts || !g.cell_start ||
      !g.cell_items || !tstore)
    return E2A_ERR_WORKSPACE;
  int bb = (int)(B < 148 * 8 ? B : 148 * 8);
  k_sys_bbox<<<bb > 0 ? bb : 1, 256, 0, st>>>(pts, p_ptr, B, g.lo, hi);
  E2A_CHECK_LAUNCH();
  E2A_CUDA(cudaMemsetAsync(ncell, 0, (B + 1) * sizeof(int32_t), st));
  k_sys_grid<<<(int)((B + 127) / 128), 128, 0, st>>>(g.lo, hi, p_ptr, B, cell_min, g.cs, g.dims, ncell);
  E2A_CHECK_LAUNCH();
  E2A_CUDA(cub::DeviceScan::ExclusiveSum(tstore, tb, ncell, g.cell_off, (int)(B + 1), st));
  E2A_CUDA(cudaMemsetAsync(counts, 0, (ncap + 1) * sizeof(int32_t), st));
  int blocks = (int)((P + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (P > 0) {
    k_bin_points<<<blocks, 256, 0, st>>>(pts, p_ptr, B, P, g, counts);
    E2A_CHECK_LAUNCH();
  }
  E2A_CUDA(cub::DeviceScan::ExclusiveSum(tstore, tb, counts, g.cell_start, (int)(ncap + 1), st));
  if (P > 0) {
    E2A_CUDA(cudaMemcpyAsync(counts, g.cell_start, ncap * sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
    k_fill_cells<<<blocks, 256, 0, st>>>(P, g.cell_of, counts, g.cell_items);
    E2A_CHECK_LAUNCH();
  }
  return E2A_OK;
}

size_t grid_ws_bytes(int64_t P, int64_t B) {
  const int64_t ncap = P + B;
  size_t tb1 = scan_temp_bytes<int32_t>(B + 1), tb2 = scan_temp_bytes<int32_t>(ncap + 1);
  size_t tb = tb1 > tb2 ? tb1 : tb2;
  size_t s = 0;
  auto add = [&](size_t b) { s += e2a_align_up(b, 256) + 256; };
  add(B * 3 * 4); add(B * 3 * 4); add(B * 3 * 4); add(B * 3 * 4);
  add((B + 1) * 4); add((B + 1) * 4); add((P > 0 ? P : 1) * 4);
  add((ncap + 1) * 4); add((ncap + 1) * 4); add((P > 0 ? P : 1) * 4); add(tb);
  return s;
}

// Range of cells of system b that can hold a point within `reach` of q.
struct CellRange { int lo[3], hi[3]; };
__device__ __forceinline__ CellRange cell_range(const float q[3], const GridDev& g, int64_t b, float reach) {
  CellRange r;
  for (int d = 0; d < 3; ++d) {
    r.lo[d] = cell_coord(q[d] - reach, g.lo[3 * b + d], g.cs[3 * b + d], g.dims[3 * b + d]);
    r.hi[d] = cell_coord(q[d] + reach, g.lo[3 * b + d], g.cs[3 * b + d], g.dims[3 * b + d]);
  }
  return r;
}

// ------------------------------------------------------------------------------------------------
// PBC expansion
// ------------------------------------------------------------------------------------------------
__global__ void k_pbc_flags(const float* __restrict__ pos, int64_t n_atoms, const float* __restrict__ offsets,
                            int n_img, float cutoff, GridDev g, int32_t* __restrict__ flags) {
  const int lane = threadIdx.x & 31;
  const int64_t total = (int64_t)n_img * n_atoms;
  int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const float reach = cutoff * 1.0001f + 1e-4f;
  for (; w < total; w += nw) {
    const int c = (int)(w / n_atoms);
    const int64_t a = w - (int64_t)c * n_atoms;
    if (c == 0) {  // the home cell: every atom is at distance 0 of itself
      if (lane == 0) flags[w] = cutoff > 0.f ? 1 : 0;
      continue;
    }
    float p[3];
    for (int d = 0; d < 3; ++d) p[d] = __fadd_rn(pos[3 * a + d], offsets[3 * c + d]);
    CellRange r = cell_range(p, g, 0, reach);
    int found = 0;
    for (int cx = r.lo[0]; cx <= r.hi[0] && !found; ++cx)
      for (int cy = r.lo[1]; cy <= r.hi[1] && !found; ++cy)
        for (int cz = r.lo[2]; cz <= r.hi[2] && !found; ++cz) {
          const int32_t cell = (cx * g.dims[1] + cy) * g.dims[2] + cz;
          const int32_t s = g.cell_start[cell], e = g.cell_start[cell + 1];
          for (int32_t t = s + lane; t < e; t += 32) {
            const int32_t i = g.cell_items[t];
            const float dx = __fsub_rn(pos[3 * i], p[0]);
            const float dy = __fsub_rn(pos[3 * i + 1], p[1]);
            const float dz = __fsub_rn(pos[3 * i + 2], p[2]);
            if (e2a_norm3(dx, dy, dz) < cutoff) found = 1;
          }
          found = __any_sync(0xffffffffu, found);
        }
    if (lane == 0) flags[w] = found;
  }
}

__global__ void k_pbc_emit(const float* __restrict__ pos, int64_t n_atoms, const float* __restrict__ offsets,
                           int n_img, const int32_t* __restrict__ flags, const int32_t* __restrict__ slot,
                           float* __restrict__ exp_pos, int64_t* __restrict__ outcell) {
  const int64_t total = (int64_t)n_img * n_atoms;
  for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < total; w += (int64_t)gridDim.x * blockDim.x) {
    if (!flags[w]) continue;
    const int c = (int)(w / n_atoms);
    const int64_t a = w - (int64_t)c * n_atoms;
    const int32_t s = slot[w];
    for (int d = 0; d < 3; ++d) exp_pos[3 * (int64_t)s + d] = __fadd_rn(pos[3 * a + d], offsets[3 * c + d]);
    outcell[s] = w;
  }
}

// ------------------------------------------------------------------------------------------------
// Radius graph
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ int64_t find_sys(const int64_t* __restrict__ ptr, int64_t B, int64_t i) {
  int64_t lo = 0, hi = B - 1;
  while (lo < hi) {
    int64_t mid = (lo + hi + 1) >> 1;
    if (ptr[mid] <= i) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ bool in_shell(float d, float min_dist, float max_dist) {
  return d >= min_dist && d <= max_dist;
}

__global__ void k_rg_count(const float* __restrict__ pos, const float* __restrict__ pts,
                           const int64_t* __restrict__ q_ptr, int64_t NQ, int64_t B, GridDev g,
                           float max_dist, float min_dist, int64_t max_nb,
                           int32_t* __restrict__ cnt, int32_t* __restrict__ kept) {
  const int lane = threadIdx.x & 31;
  int64_t i = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const float reach = max_dist * 1.0001f + 1e-4f;
  for (; i < NQ; i += nw) {
    const int64_t b = find_sys(q_ptr, B, i);
    const float q[3] = {pos[3 * i], pos[3 * i + 1], pos[3 * i + 2]};
    CellRange r = cell_range(q, g, b, reach);
    int c = 0;
    const int dy = g.dims[3 * b + 1], dz = g.dims[3 * b + 2];
    const int32_t off = g.cell_off[b];
    for (int cx = r.lo[0]; cx <= r.hi[0]; ++cx)
      for (int cy = r.lo[1]; cy <= r.hi[1]; ++cy) {
        // cells (cx,cy,lo..hi) are contiguous: one span of items
        const int32_t c0 = off + (cx * dy + cy) * dz;
        const int32_t s = g.cell_start[c0 + r.lo[2]], e = g.cell_start[c0 + r.hi[2] + 1];
        for (int32_t t = s + lane; t < e; t += 32) {
          const int32_t j = g.cell_items[t];
          const float d = e2a_norm3(__fsub_rn(q[0], pts[3 * j]), __fsub_rn(q[1], pts[3 * j + 1]),
                                    __fsub_rn(q[2], pts[3 * j + 2]));
          c += in_shell(d, min_dist, max_dist);
        }
      }
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if (lane == 0) {
      cnt[i] = c;
      kept[i] = (max_nb > 0 && c > max_nb) ? (int32_t)max_nb : c;
    }
  }
}

__device__ __forceinline__ float poly_envelope(float d, float cutoff) {
  // polynomial(dist, cutoff, exponent=5): 1 + r^5 (a + r (b + c r)), zero for r >= 1
  // (module_utils.py:1946-1954) with a = -21, b = 35, c = -15.
  const float r = d / cutoff;
  const float r2 = r * r, r5 = r2 * r2 * r;
  const float v = 1.0f + r5 * (-21.0f + r * (35.0f + (-15.0f) * r));
  return r < 1.0f ? v : 0.0f;
}

__global__ void k_rg_fill(const float* __restrict__ pos, const float* __restrict__ pts,
                          const int64_t* __restrict__ q_ptr, int64_t NQ, int64_t B, GridDev g,
                          float max_dist, float min_dist,
                          const int32_t* __restrict__ cand_ptr, const int32_t* __restrict__ kept,
                          const int32_t* __restrict__ row_ptr, unsigned long long* __restrict__ cand,
                          int64_t* __restrict__ query_idx, int64_t* __restrict__ neighbor_idx,
                          int32_t* __restrict__ col, float* __restrict__ edge_vec,
                          float* __restrict__ dist, float* __restrict__ poly) {
  __shared__ unsigned long long s_keys[kWarpsPerBlock][kSegSmem];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  int64_t i = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const float reach = max_dist * 1.0001f + 1e-4f;
  for (; i < NQ; i += nw) {
    const int64_t b = find_sys(q_ptr, B, i);
    const float q[3] = {pos[3 * i], pos[3 * i + 1], pos[3 * i + 2]};
    CellRange r = cell_range(q, g, b, reach);
    const int32_t base = cand_ptr[i];
    const int32_t n = cand_ptr[i + 1] - base;
    const bool in_smem = n <= kSegSmem;
    unsigned long long* seg = in_smem ? s_keys[wib] : cand + base;
    int wr = 0;
    const int dy = g.dims[3 * b + 1], dz = g.dims[3 * b + 2];
    const int32_t off = g.cell_off[b];
    for (int cx = r.lo[0]; cx <= r.hi[0]; ++cx)
      for (int cy = r.lo[1]; cy <= r.hi[1]; ++cy) {
        const int32_t c0 = off + (cx * dy + cy) * dz;
        const int32_t s = g.cell_start[c0 + r.lo[2]], e = g.cell_start[c0 + r.hi[2] + 1];
        for (int32_t t0 = s; t0 < e; t0 += 32) {
          const int32_t t = t0 + lane;
          bool ok = false;
          unsigned long long key = 0ull;
          if (t < e) {
            const int32_t j = g.cell_items[t];
            const float d = e2a_norm3(__fsub_rn(q[0], pts[3 * j]), __fsub_rn(q[1], pts[3 * j + 1]),
                                      __fsub_rn(q[2], pts[3 * j + 2]));
            ok = in_shell(d, min_dist, max_dist);
            key = ((unsigned long long)__float_as_uint(d) << 32) | (unsigned int)j;
          }
          const unsigned m = __ballot_sync(0xffffffffu, ok);
          if (ok) {
            const int at = wr + __popc(m & ((1u << lane) - 1u));
            if (at < n) seg[at] = key;
          }
          wr += __popc(m);
        }
      }
    __syncwarp();
    // Rank every candidate by (distance, point id); keep the first kept[i].
    const int32_t k = kept[i];
    const int32_t ob = row_ptr[i];
    for (int t = lane; t < n; t += 32) {
      const unsigned long long v = seg[t];
      int rank = 0;
      for (int u = 0; u < n; ++u) rank += (seg[u] < v);
      if (rank < k) {
        const int32_t j = (int32_t)(v & 0xffffffffull);
        const float d = __uint_as_float((unsigned)(v >> 32));
        const int64_t o = (int64_t)ob + rank;
        query_idx[o] = i;
        neighbor_idx[o] = j;
        col[o] = j;
        edge_vec[3 * o] = __fsub_rn(q[0], pts[3 * j]);
        edge_vec[3 * o + 1] = __fsub_rn(q[1], pts[3 * j + 1]);
        edge_vec[3 * o + 2] = __fsub_rn(q[2], pts[3 * j + 2]);
        dist[o] = d;
        poly[o] = poly_envelope(d, max_dist);
      }
    }
    __syncwarp();
  }
}

size_t rg_ws_bytes(int64_t NQ, int64_t P, int64_t B) {
  size_t tb = scan_temp_bytes<int32_t>(NQ + 1);
  size_t s = grid_ws_bytes(P, B);
  auto add = [&](size_t b) { s += e2a_align_up(b, 256) + 256; };
  add((NQ + 1) * 4); add((NQ + 1) * 4); add((NQ + 1) * 4); add((NQ + 1) * 4); add(tb); add(16);
  return s;
}

struct RgBufs {
  GridDev g;
  int32_t *cnt, *kept, *cand_ptr, *row_ptr_tmp;
};

int rg_prepare(const float* pts, const int64_t* p_ptr, int64_t NQ, int64_t P, int64_t B, float max_dist,
               void* ws, size_t wsb, RgBufs& rb, E2aArena& ar, cudaStream_t st) {
  ar = E2aArena{(char*)ws, wsb, 0};
  int rc = build_grid(pts, p_ptr, P, B, max_dist > 0.f ? max_dist : 1.0f, rb.g, ar, st);
  if (rc) return rc;
  rb.cnt = (int32_t*)ar.take((NQ + 1) * 4);
  rb.kept = (int32_t*)ar.take((NQ + 1) * 4);
  rb.cand_ptr = (int32_t*)ar.take((NQ + 1) * 4);
  rb.row_ptr_tmp = (int32_t*)ar.take((NQ + 1) * 4);
  if (!rb.cnt || !rb.kept || !rb.cand_ptr || !rb.row_ptr_tmp) return E2A_ERR_WORKSPACE;
  return E2A_OK;
}

}  // namespace

static thread_local int g_last_cuda_error = 0;
void e2a_set_cuda_error(cudaError_t e) { g_last_cuda_error = (int)e; }
static std::atomic<unsigned long long> g_launches{0};
void e2a_note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

extern "C" {

int e2a_version(void) { return 100; }

const char* e2a_status_string(int status) {
  switch (status) {
    case E2A_OK: return "ok";
    case E2A_ERR_ARG: return "invalid argument";
    case E2A_ERR_CUDA: return "CUDA error";
    case E2A_ERR_WORKSPACE: return "workspace too small";
    case E2A_ERR_UNSUPPORTED: return "unsupported shape";
    default: return "unknown status";
  }
}

int e2a_last_cuda_error(void) { return g_last_cuda_error; }

uint64_t e2a_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

size_t e2a_csr_workspace_bytes(int64_t E, int64_t N, int64_t M) {
  int64_t R = N > M ? N : M;
  size_t s = 0;
  auto add = [&](size_t b) { s += e2a_align_up(b, 256) + 256; };
  add(16);
  for (int rep = 0; rep < 2; ++rep) {
    add((R + 1) * 4);
    add((E > 0 ? E : 1) * 4);
    add(scan_temp_bytes<int32_t>(R + 1));
  }
  return s;
}

int e2a_csr_build(const int32_t* query_idx, const int32_t* neighbor_idx, int64_t E, int64_t N, int64_t M,
                  int32_t* q_row_ptr, int32_t* q_col, int32_t* q_perm, int32_t* k_row_ptr, int32_t* k_col,
                  int32_t* k_perm, void* ws, size_t wsb, void* stream) {
  if (E < 0 || N < 0 || M < 0 || E > INT32_MAX || N >= INT32_MAX || M >= INT32_MAX) return E2A_ERR_ARG;
  if (!q_row_ptr || !k_row_ptr || (E > 0 && (!query_idx || !neighbor_idx || !q_col || !q_perm || !k_col || !k_perm)))
    return E2A_ERR_ARG;
  if (wsb < e2a_csr_workspace_bytes(E, N, M)) return E2A_ERR_WORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  E2aArena ar{(char*)ws, wsb, 0};
  int* d_err = (int*)ar.take(16);
  if (!d_err) return E2A_ERR_WORKSPACE;
  E2A_CUDA(cudaMemsetAsync(d_err, 0, sizeof(int), st));
  int rc = group_by(query_idx, neighbor_idx, E, N, q_row_ptr, q_perm, q_col, ar, d_err, st);
  if (rc) return rc;
  rc = group_by(neighbor_idx, query_idx, E, M, k_row_ptr, k_perm, k_col, ar, d_err, st);
  if (rc) return rc;
  int h_err = 0;
  E2A_CUDA(cudaMemcpyAsync(&h_err, d_err, sizeof(int), cudaMemcpyDeviceToHost, st));
  E2A_CUDA(cudaStreamSynchronize(st));
  return h_err ? E2A_ERR_ARG : E2A_OK;
}

size_t e2a_pbc_expand_workspace_bytes(int64_t n_atoms, int n_img) {
  const int64_t total = (int64_t)n_img * n_atoms;
  size_t s = grid_ws_bytes(n_atoms, 1);
  auto add = [&](size_t b) { s += e2a_align_up(b, 256) + 256; };
  add(16);                    // p_ptr
  add((total + 1) * 4);       // flags
  add((total + 1) * 4);       // slots
  add(scan_temp_bytes<int32_t>(total + 1));
  return s;
}

int e2a_pbc_expand(const float* pos, int64_t n_atoms, const float* offsets, int n_img, float cutoff,
                   float* exp_pos, int64_t* outcell, int64_t* n_expanded, void* ws, size_t wsb, void* stream) {
  if (n_atoms <= 0 || n_img <= 0 || !pos || !offsets || !exp_pos || !outcell || !n_expanded) return E2A_ERR_ARG;
  const int64_t total = (int64_t)n_img * n_atoms;
  if (total >= INT32_MAX) return E2A_ERR_ARG;
  if (wsb < e2a_pbc_expand_workspace_bytes(n_atoms, n_img)) return E2A_ERR_WORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  E2aArena ar{(char*)ws, wsb, 0};
  int64_t* p_ptr = (int64_t*)ar.take(16);
  if (!p_ptr) return E2A_ERR_WORKSPACE;
  const int64_t h_ptr[2] = {0, n_atoms};
  E2A_CUDA(cudaMemcpyAsync(p_ptr, h_ptr, sizeof(h_ptr), cudaMemcpyHostToDevice, st));
  GridDev g;
  int rc = build_grid(pos, p_ptr, n_atoms, 1, cutoff > 0.f ? cutoff : 1.0f, g, ar, st);
  if (rc) return rc;
  int32_t* flags = (int32_t*)ar.take((total + 1) * 4);
  int32_t* slots = (int32_t*)ar.take((total + 1) * 4);
  size_t tb = scan_temp_bytes<int32_t>(total + 1);
  void* tstore = ar.take(tb);
  if (!flags || !slots || !tstore) return E2A_ERR_WORKSPACE;
  E2A_CUDA(cudaMemsetAsync(flags, 0, (total + 1) * 4, st));
  int64_t wblocks = (total * 32 + 255) / 256;
  if (wblocks > 148 * 64) wblocks = 148 * 64;
  k_pbc_flags<<<(int)wblocks, 256, 0, st>>>(pos, n_atoms, offsets, n_img, cutoff, g, flags);
  E2A_CHECK_LAUNCH();
  E2A_CUDA(cub::DeviceScan::ExclusiveSum(tstore, tb, flags, slots, (int)(total + 1), st));
  int32_t h_total = 0;
  E2A_CUDA(cudaMemcpyAsync(&h_total, slots + total, 4, cudaMemcpyDeviceToHost, st));
  int64_t eblocks = (total + 255) / 256;
  if (eblocks > 148 * 16) eblocks = 148 * 16;
  k_pbc_emit<<<(int)eblocks, 256, 0, st>>>(pos, n_atoms, offsets, n_img, flags, slots, exp_pos, outcell);
  E2A_CHECK_LAUNCH();
  E2A_CUDA(cudaStreamSynchronize(st));
  *n_expanded = h_total;
  return E2A_OK;
}

size_t e2a_radius_graph_workspace_bytes(int64_t NQ, int64_t P, int64_t B) { return rg_ws_bytes(NQ, P, B); }

int e2a_radius_graph_plan(const float* pos, const float* pts, const int64_t* q_ptr, const int64_t* p_ptr,
                          int64_t NQ, int64_t P, int64_t B, float max_dist, float min_dist, int64_t max_nb,
                          int64_t* num_edges, int64_t* num_candidates, void* ws, size_t wsb, void* stream) {
  if (NQ < 0 || P < 0 || B <= 0 || !q_ptr || !p_ptr || !num_edges || !num_candidates) return E2A_ERR_ARG;
  if (NQ >= INT32_MAX || P >= INT32_MAX) return E2A_ERR_ARG;
  if (wsb < rg_ws_bytes(NQ, P, B)) return E2A_ERR_WORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  RgBufs rb;
  E2aArena ar{nullptr, 0, 0};
  int rc = rg_prepare(pts, p_ptr, NQ, P, B, max_dist, ws, wsb, rb, ar, st);
  if (rc) return rc;
  size_t tb = scan_temp_bytes<int32_t>(NQ + 1);
  void* tstore = ar.take(tb);
  if (!tstore) return E2A_ERR_WORKSPACE;
  E2A_CUDA(cudaMemsetAsync(rb.cnt, 0, (NQ + 1) * 4, st));
  E2A_CUDA(cudaMemsetAsync(rb.kept, 0, (NQ + 1) * 4, st));
  if (NQ > 0) {
    int64_t blocks = (NQ + kWarpsPerBlock - 1) / kWarpsPerBlock;
    if (blocks > 148 * 32) blocks = 148 * 32;
    k_rg_count<<<(int)blocks, kWarpsPerBlock * 32, 0, st>>>(pos, pts, q_ptr, NQ, B, rb.g, max_dist, min_dist,
                                                             max_nb, rb.cnt, rb.kept);
    E2A_CHECK_LAUNCH();
  }
  E2A_CUDA(cub::DeviceScan::ExclusiveSum(tstore, tb, rb.cnt, rb.cand_ptr, (int)(NQ + 1), st));
  E2A_CUDA(cub::DeviceScan::ExclusiveSum(tstore, tb, rb.kept, rb.row_ptr_tmp, (int)(NQ + 1), st));
  int32_t h[2] = {0, 0};
  E2A_CUDA(cudaMemcpyAsync(&h[0], rb.row_ptr_tmp + NQ, 4, cudaMemcpyDeviceToHost, st));
  E2A_CUDA(cudaMemcpyAsync(&h[1], rb.cand_ptr + NQ, 4, cudaMemcpyDeviceToHost, st));
  E2A_CUDA(cudaStreamSynchronize(st));
  *num_edges = h[0];
  *num_candidates = h[1];
  return E2A_OK;
}

size_t e2a_radius_graph_fill_workspace_bytes(int64_t num_candidates) {
  return e2a_align_up((size_t)(num_candidates > 0 ? num_candidates : 1) * 8, 256) + 256;
}

int e2a_radius_graph_fill(const float* pos, const float* pts, const int64_t* q_ptr, const int64_t* p_ptr,
                          int64_t NQ, int64_t P, int64_t B, float max_dist, float min_dist, int64_t max_nb,
                          int64_t E, int64_t C, int64_t* query_idx, int64_t* neighbor_idx, int32_t* row_ptr,
                          int32_t* col, float* edge_vec, float* dist, float* poly, void* ws, size_t wsb,
                          void* fws, size_t fwsb, void* stream) {
  if (NQ < 0 || P < 0 || B <= 0 || !row_ptr) return E2A_ERR_ARG;
  if (E > 0 && (!query_idx || !neighbor_idx || !col || !edge_vec || !dist || !poly)) return E2A_ERR_ARG;
  if (wsb < rg_ws_bytes(NQ, P, B)) return E2A_ERR_WORKSPACE;
  if (fwsb < e2a_radius_graph_fill_workspace_bytes(C)) return E2A_ERR_WORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  // The plan call left the grid and the per-row counts in the workspace; recompute the layout only.
  E2aArena ar{(char*)ws, wsb, 0};
  GridDev g;
  {
    const int64_t ncap = P + B;
    (void)ar.take(B * 3 * sizeof(float));  // hi
    g.lo = (float*)ar.take(B * 3 * sizeof(float));
    g.cs = (float*)ar.take(B * 3 * sizeof(float));
    g.dims = (int*)ar.take(B * 3 * sizeof(int));
    (void)ar.take((B + 1) * sizeof(int32_t));  // ncell
    g.cell_off = (int32_t*)ar.take((B + 1) * sizeof(int32_t));
    g.cell_of = (int32_t*)ar.take((P > 0 ? P : 1) * sizeof(int32_t));
    (void)ar.take((ncap + 1) * sizeof(int32_t));  // counts
    g.cell_start = (int32_t*)ar.take((ncap + 1) * sizeof(int32_t));
    g.cell_items = (int32_t*)ar.take((P > 0 ? P : 1) * sizeof(int32_t));
    size_t tb1 = scan_temp_bytes<int32_t>(B + 1), tb2 = scan_temp_bytes<int32_t>(ncap + 1);
    (void)ar.take(tb1 > tb2 ? tb1 : tb2);
  }
  int32_t* cnt = (int32_t*)ar.take((NQ + 1) * 4);
  int32_t* kept = (int32_t*)ar.take((NQ + 1) * 4);
  int32_t* cand_ptr = (int32_t*)ar.take((NQ + 1) * 4);
  int32_t* rp = (int32_t*)ar.take((NQ + 1) * 4);
  if (!cnt || !kept || !cand_ptr || !rp) return E2A_ERR_WORKSPACE;
  (void)cnt;
  E2A_CUDA(cudaMemcpyAsync(row_ptr, rp, (NQ + 1) * 4, cudaMemcpyDeviceToDevice, st));
  if (NQ > 0 && E > 0) {
    int64_t blocks = (NQ + kWarpsPerBlock - 1) / kWarpsPerBlock;
    if (blocks > 148 * 32) blocks = 148 * 32;
    k_rg_fill<<<(int)blocks, kWarpsPerBlock * 32, 0, st>>>(pos, pts, q_ptr, NQ, B, g, max_dist, min_dist, cand_ptr,
                                                            kept, rp, (unsigned long long*)fws, query_idx,
                                                            neighbor_idx, col, edge_vec, dist, poly);
    E2A_CHECK_LAUNCH();
  }
  return E2A_OK;
}

}  // extern "C"
