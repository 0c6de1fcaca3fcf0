/*
 * CPU oracle for the radius-graph path -- TEST INFRASTRUCTURE ONLY (loaded by tests/ and by the
 * bench's CPU-baseline leg through ctypes; never by the product library).
 *
 * Restates, in plain C, the semantics of the reference's (IQuestLab/UBio-MolFM,
 * e2f = src/molfm/models/e2former):
 *   - CellExpander.expand_includeself (e2f/module_utils.py:1065-1275): image (c, a) of atom a
 *     shifted by offsets[c] is kept iff some atom i has |pos_i - (pos_a + offsets[c])| < cutoff;
 *     kept images are listed cell-major, atom-ascending (1202-1207).
 *   - construct_radius_neighbor (e2f/module_utils.py:3119-3242): per query row, candidates of the
 *     same system with min_dist <= d <= max_dist (3166-3171), ascending distance (3172), truncated
 *     to max_neighbors (3173-3178); distances from torch.linalg.norm of pos_i - pts_j (3164-3165),
 *     whose CPU kernel evaluates sqrt(fma(z,z,fma(y,y,x*x))) in fp32.
 * Exact distance ties are ordered by candidate index (the reference's sort is unstable there).
 * Build: gcc -O2 -ffp-contract=off -fPIC -shared (see oracle/Makefile).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline float norm3(float x, float y, float z) { return sqrtf(fmaf(z, z, fmaf(y, y, x * x))); }

int64_t orc_pbc_expand(const float* pos, int64_t n, const float* off, int nimg, float cutoff, int64_t* out) {
  int64_t k = 0;
  for (int c = 0; c < nimg; ++c) {
    for (int64_t a = 0; a < n; ++a) {
      const float p0 = pos[3 * a] + off[3 * c], p1 = pos[3 * a + 1] + off[3 * c + 1], p2 = pos[3 * a + 2] + off[3 * c + 2];
      int keep = 0;
      for (int64_t i = 0; i < n && !keep; ++i) {
        if (norm3(pos[3 * i] - p0, pos[3 * i + 1] - p1, pos[3 * i + 2] - p2) < cutoff) keep = 1;
      }
      if (keep) out[k++] = (int64_t)c * n + a;
    }
  }
  return k;
}

typedef struct { float d; int32_t j; } Cand;

static int cand_cmp(const void* a, const void* b) {
  const Cand* x = (const Cand*)a;
  const Cand* y = (const Cand*)b;
  if (x->d < y->d) return -1;
  if (x->d > y->d) return 1;
  return (x->j > y->j) - (x->j < y->j);
}

/* Returns the number of edges E; writes at most `cap` of them. */
int64_t orc_radius_graph(const float* pos, const float* pts, const int64_t* q_ptr, const int64_t* p_ptr, int64_t B,
                         float max_dist, float min_dist, int64_t max_nb, int64_t cap, int64_t* qidx, int64_t* nidx,
                         float* dist) {
  int64_t E = 0;
  for (int64_t b = 0; b < B; ++b) {
    const int64_t p0 = p_ptr[b], p1 = p_ptr[b + 1], np = p1 - p0;
    if (np <= 0) continue;
    /* uniform grid over the system's points, cell edge >= max_dist */
    float lo[3] = {INFINITY, INFINITY, INFINITY}, hi[3] = {-INFINITY, -INFINITY, -INFINITY};
    for (int64_t p = p0; p < p1; ++p)
      for (int d = 0; d < 3; ++d) {
        if (pts[3 * p + d] < lo[d]) lo[d] = pts[3 * p + d];
        if (pts[3 * p + d] > hi[d]) hi[d] = pts[3 * p + d];
      }
    int dims[3];
    double cs[3];
    for (int d = 0; d < 3; ++d) {
      double ext = (double)hi[d] - (double)lo[d];
      long long v = (long long)floor(ext / (double)(max_dist > 0 ? max_dist : 1.0f));
      if (v < 1) v = 1;
      if (v > 256) v = 256;
      dims[d] = (int)v;
      cs[d] = ext / v;
      if (cs[d] < (double)max_dist) cs[d] = max_dist;
      if (cs[d] <= 0) cs[d] = 1.0;
    }
    const int64_t ncell = (int64_t)dims[0] * dims[1] * dims[2];
    int64_t* start = (int64_t*)calloc(ncell + 1, sizeof(int64_t));
    int64_t* items = (int64_t*)malloc(np * sizeof(int64_t));
    int64_t* cellof = (int64_t*)malloc(np * sizeof(int64_t));
    for (int64_t p = p0; p < p1; ++p) {
      int c[3];
      for (int d = 0; d < 3; ++d) {
        long long v = (long long)floor(((double)pts[3 * p + d] - lo[d]) / cs[d]);
        c[d] = v < 0 ? 0 : (v >= dims[d] ? dims[d] - 1 : (int)v);
      }
      cellof[p - p0] = ((int64_t)c[0] * dims[1] + c[1]) * dims[2] + c[2];
      start[cellof[p - p0] + 1]++;
    }
    for (int64_t c = 0; c < ncell; ++c) start[c + 1] += start[c];
    int64_t* fill = (int64_t*)malloc(ncell * sizeof(int64_t));
    memcpy(fill, start, ncell * sizeof(int64_t));
    for (int64_t p = p0; p < p1; ++p) items[fill[cellof[p - p0]]++] = p;
    free(fill);
    Cand* buf = (Cand*)malloc(np * sizeof(Cand));
    const double reach = (double)max_dist * 1.0001 + 1e-4;
    for (int64_t i = q_ptr[b]; i < q_ptr[b + 1]; ++i) {
      const float q0 = pos[3 * i], q1 = pos[3 * i + 1], q2 = pos[3 * i + 2];
      int clo[3], chi[3];
      const float qq[3] = {q0, q1, q2};
      for (int d = 0; d < 3; ++d) {
        long long a = (long long)floor(((double)qq[d] - reach - lo[d]) / cs[d]);
        long long z = (long long)floor(((double)qq[d] + reach - lo[d]) / cs[d]);
        clo[d] = a < 0 ? 0 : (a >= dims[d] ? dims[d] - 1 : (int)a);
        chi[d] = z < 0 ? 0 : (z >= dims[d] ? dims[d] - 1 : (int)z);
      }
      int64_t nc = 0;
      for (int x = clo[0]; x <= chi[0]; ++x)
        for (int y = clo[1]; y <= chi[1]; ++y)
          for (int z = clo[2]; z <= chi[2]; ++z) {
            const int64_t c = ((int64_t)x * dims[1] + y) * dims[2] + z;
            for (int64_t t = start[c]; t < start[c + 1]; ++t) {
              const int64_t j = items[t];
              const float d = norm3(q0 - pts[3 * j], q1 - pts[3 * j + 1], q2 - pts[3 * j + 2]);
              if (d >= min_dist && d <= max_dist) { buf[nc].d = d; buf[nc].j = (int32_t)j; nc++; }
            }
          }
      qsort(buf, nc, sizeof(Cand), cand_cmp);
      const int64_t k = (max_nb > 0 && nc > max_nb) ? max_nb : nc;
      for (int64_t t = 0; t < k; ++t) {
        if (E < cap) { qidx[E] = i; nidx[E] = buf[t].j; dist[E] = buf[t].d; }
        E++;
      }
    }
    free(buf);
    free(start);
    free(items);
    free(cellof);
  }
  return E;
}
