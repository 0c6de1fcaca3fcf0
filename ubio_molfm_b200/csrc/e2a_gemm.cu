// Dense fp32 GEMM on the 5th-generation tensor cores with fp32-level accuracy (3xTF32 split).
//
//   C[M,N] = A[M,K] * B[N,K]^T (+ bias[N]) (+ C if accumulate)       (both operands K-major)
//
// This is the node-side projection workhorse of the attention layer (the per-degree SO(3) linears,
// the Q/K scalar MLPs, the edge radial MLP): nn.Linear-shaped products y = x W^T.
//
// Design (one CTA = one 128 x 128 output tile, 256 threads):
//  * all threads stream a 128 x 32 fp32 k-slab of A and of B from global memory (coalesced 16-byte
//    loads), split every value into a tf32 "hi" part (round to nearest, low 13 bits zero) and the
//    fp32 remainder "lo", and store hi and lo into shared memory in the 128-byte-swizzled K-major
//    layout the tensor core reads (8-row atoms of 1 KB, 16-byte chunk c of row r at c ^ (r % 8));
//  * one thread issues, per 8-wide k step, tcgen05.mma kind::tf32 for hi*hi + hi*lo + lo*hi into a
//    fp32 accumulator in tensor memory (128 lanes x 128 columns), then tcgen05.commit to the stage's
//    mbarrier; the loads of slab k+1 overlap the MMAs of slab k;
//  * the tensor core's fp32 accumulation truncates, so long accumulation chains drift (measured ~7x
//    the error of an fp32 SIMT GEMM at K = 1536).  Each 32-wide k-slab therefore accumulates into a
//    fresh tensor-memory buffer (12 MMA steps per chain; two buffers alternate) and every thread adds
//    its 64 values of that buffer into fp32 registers with round-to-nearest adds;
//  * the epilogue adds bias / the previous C to the register accumulators and stores.
// The dropped lo*lo term is below fp32 resolution (|error| ~ 2^-22 relative per product).
// Every mbarrier wait is bounded in time; on a timeout the kernel records E2A_DEV_WAIT_TIMEOUT,
// still waits (bounded) for its MMAs, frees its tensor memory and returns.
#include "e2a_common.cuh"

__device__ unsigned int g_e2a_gemm_status = 0;

namespace {

constexpr int BM = 128, BN = 128, BK = 32, STAGES = 2, kThreads = 256;
constexpr int kTileBytes = BM * BK * 4;            // 16 KB per operand part
constexpr int kStageBytes = 4 * kTileBytes;        // A_hi, A_lo, B_hi, B_lo
constexpr int kSmemBytes = STAGES * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
constexpr uint32_t kTmemCols = 256;  // two 128-column accumulators

// instruction descriptor: D fp32, A/B tf32, both K-major, M = 128, N = 128
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  // K-major, 128-byte swizzle: LBO unused (1), SBO = 1024 B between 8-row atoms, version 1
  return (uint64_t)((addr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(e2a_smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ float tf32_hi(float a) {
  return __uint_as_float((__float_as_uint(a) + 0x1000u) & 0xFFFFE000u);
}

// A 128 x 32 slab (rows r0.., cols k0..) of a row-major fp32 matrix: each thread loads 4 float4
// (zero outside the matrix) into registers ...
constexpr int kF4PerThread = (BM * BK / 4) / kThreads;

template <bool VEC>
__device__ __forceinline__ void load_slab(const float* __restrict__ X, int64_t ld, int rows, int K, int r0, int k0,
                                          float4 (&v)[kF4PerThread]) {
#pragma unroll
  for (int j = 0; j < kF4PerThread; ++j) {
    const int c = threadIdx.x + j * kThreads;
    const int r = c >> 3, ch = c & 7;
    const int gr = r0 + r, gk = k0 + ch * 4;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (gr < rows) {
      const float* p = X + (int64_t)gr * ld + gk;
      if (VEC && gk + 3 < K) {
        x = __ldg(reinterpret_cast<const float4*>(p));
      } else {
        if (gk < K) x.x = __ldg(p);
        if (gk + 1 < K) x.y = __ldg(p + 1);
        if (gk + 2 < K) x.z = __ldg(p + 2);
        if (gk + 3 < K) x.w = __ldg(p + 3);
      }
    }
    v[j] = x;
  }
}

// ... then splits them into hi / lo and stores both in the swizzled K-major layout.
__device__ __forceinline__ void split_store(const float4 (&v)[kF4PerThread], uint8_t* hi, uint8_t* lo) {
#pragma unroll
  for (int j = 0; j < kF4PerThread; ++j) {
    const int c = threadIdx.x + j * kThreads;
    const int r = c >> 3, ch = c & 7;
    float4 h, l;
    h.x = tf32_hi(v[j].x); h.y = tf32_hi(v[j].y); h.z = tf32_hi(v[j].z); h.w = tf32_hi(v[j].w);
    l.x = v[j].x - h.x; l.y = v[j].y - h.y; l.z = v[j].z - h.z; l.w = v[j].w - h.w;
    const int off = r * 128 + ((ch ^ (r & 7)) << 4);
    *reinterpret_cast<float4*>(hi + off) = h;
    *reinterpret_cast<float4*>(lo + off) = l;
  }
}

template <bool VEC>
__global__ void __launch_bounds__(kThreads, 1)
k_gemm_tf32x3(const float* __restrict__ A, int64_t lda, const float* __restrict__ B, int64_t ldb, float* C,
              int64_t ldc, const float* __restrict__ bias, int M, int N, int K, int accumulate, int passes) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = e2a_smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * kStageBytes);  // STAGES barriers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + STAGES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(e2a_smem_u32(tmem_slot)), "r"(kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) e2a_mbar_init(&bars[s], 1);
    e2a_fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int nk = (K + BK - 1) / BK;
  const int q = warp & 3, half = warp >> 2;        // TMEM lane quadrant and column half of this warp
  const uint32_t lane_base = (uint32_t)(32 * q) << 16;
  float acc[BN / 2];
#pragma unroll
  for (int i = 0; i < BN / 2; ++i) acc[i] = 0.f;
  bool ok = true;
  float4 ra[kF4PerThread], rb[kF4PerThread];  // slab kb, loaded one iteration ahead
  if (nk > 0) {
    load_slab<VEC>(A, lda, M, K, m0, 0, ra);
    load_slab<VEC>(B, ldb, N, K, n0, 0, rb);
  }
  for (int kb = 0; kb < nk; ++kb) {
    const int s = kb % STAGES;
    uint8_t* st = smem + s * kStageBytes;
    // issue the loads of slab kb+1 now; they are in flight during the stores, the MMAs and the drain
    float4 na[kF4PerThread], nb[kF4PerThread];
    if (kb + 1 < nk) {
      load_slab<VEC>(A, lda, M, K, m0, (kb + 1) * BK, na);
      load_slab<VEC>(B, ldb, N, K, n0, (kb + 1) * BK, nb);
    }
    // stage s was last read by the MMAs of slab kb-2, which finished before slab kb-1 was drained
    split_store(ra, st, st + kTileBytes);
    split_store(rb, st + 2 * kTileBytes, st + 3 * kTileBytes);
    e2a_fence_proxy_async();  // make the generic-proxy stores visible to the tensor core
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) {
      tc_fence_after();
      const uint32_t d = tmem + (uint32_t)((kb & 1) * BN);
      const uint32_t a_hi = e2a_smem_u32(st), a_lo = a_hi + kTileBytes;
      const uint32_t b_hi = a_hi + 2 * kTileBytes, b_lo = a_hi + 3 * kTileBytes;
#pragma unroll
      for (int kk = 0; kk < BK / 8; ++kk) {
        const uint32_t koff = kk * 32;  // 8 tf32 = 32 bytes along the swizzled row
        mma_tf32(d, smem_desc_sw128(a_hi + koff), smem_desc_sw128(b_hi + koff), kk > 0 ? 1u : 0u);
        if (passes == 3) {
          mma_tf32(d, smem_desc_sw128(a_hi + koff), smem_desc_sw128(b_lo + koff), 1u);
          mma_tf32(d, smem_desc_sw128(a_lo + koff), smem_desc_sw128(b_hi + koff), 1u);
        }
      }
      mma_commit(&bars[s]);
    }
    // drain the previous slab's buffer into registers while slab kb runs on the tensor core
    if (kb >= 1) {
      const int pk = kb - 1;
      ok = e2a_mbar_wait_bounded(&bars[pk % STAGES], (pk / STAGES) & 1, &g_e2a_gemm_status);
      if (__syncthreads_or(!ok)) { ok = false; break; }
      tc_fence_after();
#pragma unroll
      for (int c0 = 0; c0 < BN / 2; c0 += 16) {
        float v[16];
        tmem_ld16(tmem + lane_base + (uint32_t)((pk & 1) * BN + 64 * half + c0), v);
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[c0 + i] += v[i];
      }
    }
    if (kb + 1 < nk) {
#pragma unroll
      for (int j = 0; j < kF4PerThread; ++j) { ra[j] = na[j]; rb[j] = nb[j]; }
    }
  }
  if (ok && nk > 0) {
    const int pk = nk - 1;
    ok = e2a_mbar_wait_bounded(&bars[pk % STAGES], (pk / STAGES) & 1, &g_e2a_gemm_status);
    if (!__syncthreads_or(!ok)) {
      tc_fence_after();
#pragma unroll
      for (int c0 = 0; c0 < BN / 2; c0 += 16) {
        float v[16];
        tmem_ld16(tmem + lane_base + (uint32_t)((pk & 1) * BN + 64 * half + c0), v);
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[c0 + i] += v[i];
      }
    } else {
      ok = false;
    }
  }
  const bool all_ok = !__syncthreads_or(!ok);
  if (all_ok) {
    const int row = m0 + 32 * q + lane;
    if (row < M) {
      float* crow = C + (int64_t)row * ldc + n0 + 64 * half;
#pragma unroll
      for (int i = 0; i < BN / 2; ++i) {
        const int gc = n0 + 64 * half + i;
        if (gc < N) {
          float x = acc[i];
          if (bias) x += bias[gc];
          if (accumulate) x += crow[i];
          crow[i] = x;
        }
      }
    }
  } else if (threadIdx.x == 0 && nk > 0) {
    // a wait gave up: give the issued MMAs a bounded chance to finish before the memory is freed
    for (int pk = (nk >= 2 ? nk - 2 : 0); pk < nk; ++pk)
      e2a_mbar_wait_bounded(&bars[pk % STAGES], (pk / STAGES) & 1, &g_e2a_gemm_status);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}


// ------------------------------------------------------------------------------------------------
// Pipelined kernel for 16-byte-aligned operands: raw fp32 slabs arrive by cp.async (16-byte copies,
// zero-filled past the matrix edge, destination already in the swizzled layout) several slabs ahead;
// each slab is split shared -> shared into one of two hi/lo operand buffers while the tensor core
// works on the other.  Global-memory latency is off the critical path.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// ------------------------------------------------------------------------------------------------
// v2: 16-wide k-slabs in the 64-byte-swizzled K-major layout (8-row atoms of 512 B, 16-byte chunk c
// of row r at c ^ ((r >> 1) & 3)).  112 KB of shared memory and <= 128 registers per thread, so two
// CTAs (two 256-column TMEM allocations) share an SM and overlap each other's stalls.
// ------------------------------------------------------------------------------------------------
constexpr int BK2 = 16;
constexpr int kTile2 = BM * BK2 * 4;                 // 8 KB per operand part
constexpr int kRaw2 = 2 * kTile2;                    // A and B raw slab
constexpr int kOp2 = 4 * kTile2;                     // A_hi, A_lo, B_hi, B_lo
constexpr int RAW2 = 3;
constexpr int kSmem2 = RAW2 * kRaw2 + 2 * kOp2 + 256;
constexpr int kF4PerThread2 = (BM * BK2 / 4) / kThreads;   // 2

__device__ __forceinline__ uint64_t smem_desc_sw64(uint32_t addr) {
  // K-major, 64-byte swizzle: LBO unused (1), SBO = 512 B between 8-row atoms, version 1
  return (uint64_t)((addr >> 4) & 0x3FFFu) | (1ull << 16) | (32ull << 32) | (1ull << 46) | (4ull << 61);
}

__device__ __forceinline__ void issue_slab2(const float* __restrict__ X, int64_t ld, int rows, int K, int r0, int k0,
                                            uint32_t dst) {
#pragma unroll
  for (int j = 0; j < kF4PerThread2; ++j) {
    const int c = threadIdx.x + j * kThreads;
    const int r = c >> 2, ch = c & 3;
    const int gr = r0 + r, gk = k0 + ch * 4;
    const int valid = (gr < rows && gk < K) ? min(4, K - gk) : 0;
    const float* src = valid ? X + (int64_t)gr * ld + gk : X;
    cp_async16(dst + (uint32_t)(r * 64 + ((ch ^ ((r >> 1) & 3)) << 4)), src, (uint32_t)valid * 4u);
  }
}

__device__ __forceinline__ void split_smem2(const uint8_t* raw, uint8_t* hi, uint8_t* lo) {
#pragma unroll
  for (int j = 0; j < kF4PerThread2; ++j) {
    const int off = (threadIdx.x + j * kThreads) * 16;
    const float4 v = *reinterpret_cast<const float4*>(raw + off);
    float4 h, l;
    h.x = tf32_hi(v.x); h.y = tf32_hi(v.y); h.z = tf32_hi(v.z); h.w = tf32_hi(v.w);
    l.x = v.x - h.x; l.y = v.y - h.y; l.z = v.z - h.z; l.w = v.w - h.w;
    *reinterpret_cast<float4*>(hi + off) = h;
    *reinterpret_cast<float4*>(lo + off) = l;
  }
}

__global__ void __launch_bounds__(kThreads, 2)
k_gemm_tf32x3_v2(const float* __restrict__ A, int64_t lda, const float* __restrict__ B, int64_t ldb, float* C,
                 int64_t ldc, const float* __restrict__ bias, int M, int N, int K, int accumulate, int passes,
                 float* P, int64_t ldp) {
  extern __shared__ __align__(1024) uint8_t smem2[];
  if ((e2a_smem_u32(smem2) & 1023u) != 0) {  // the descriptors assume 1 KB-aligned tiles
    if (threadIdx.x == 0) atomicOr(&g_e2a_gemm_status, 2u);
    return;
  }
  uint8_t* raw = smem2;
  uint8_t* ops = smem2 + RAW2 * kRaw2;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ops + 2 * kOp2);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(e2a_smem_u32(tmem_slot)), "r"(kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 0) {
    e2a_mbar_init(&bars[0], 1);
    e2a_mbar_init(&bars[1], 1);
    e2a_fence_mbar_init();
  }
  const int nk = (K + BK2 - 1) / BK2;
#pragma unroll
  for (int p = 0; p < RAW2 - 1; ++p) {
    if (p < nk) {
      const uint32_t d = e2a_smem_u32(raw + p * kRaw2);
      issue_slab2(A, lda, M, K, m0, p * BK2, d);
      issue_slab2(B, ldb, N, K, n0, p * BK2, d + kTile2);
    }
    cp_async_commit();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int q = warp & 3, half = warp >> 2;
  const uint32_t lane_base = (uint32_t)(32 * q) << 16;
  float acc[BN / 2];
#pragma unroll
  for (int i = 0; i < BN / 2; ++i) acc[i] = 0.f;
  bool ok = true;
  // Slabs kb = 2g, 2g+1 accumulate into TMEM buffer g & 1 (a 12-MMA chain, like a 32-wide slab);
  // group g-1 is drained into the fp32 registers while group g runs.  Every wait targets the latest
  // or the second-latest commit on its barrier, so a parity never wraps.
  auto drain = [&](int g) {
    tc_fence_after();
#pragma unroll
    for (int c0 = 0; c0 < BN / 2; c0 += 16) {
      float v[16];
      tmem_ld16(tmem + lane_base + (uint32_t)((g & 1) * BN + 64 * half + c0), v);
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[c0 + i] += v[i];
    }
  };
  for (int kb = 0; kb < nk; ++kb) {
    {
      const int p = kb + RAW2 - 1;
      if (p < nk) {
        const uint32_t d = e2a_smem_u32(raw + (p % RAW2) * kRaw2);
        issue_slab2(A, lda, M, K, m0, p * BK2, d);
        issue_slab2(B, ldb, N, K, n0, p * BK2, d + kTile2);
      }
      cp_async_commit();
    }
    // operand buffer kb & 1 was read by the MMAs of slab kb-2
    if (kb >= 2) {
      ok = e2a_mbar_wait_bounded(&bars[kb & 1], ((kb - 2) >> 1) & 1, &g_e2a_gemm_status);
      if (__syncthreads_or(!ok)) { ok = false; break; }
    }
    cp_async_wait<RAW2 - 1>();
    __syncthreads();
    const uint8_t* rs = raw + (kb % RAW2) * kRaw2;
    uint8_t* op = ops + (kb & 1) * kOp2;
    split_smem2(rs, op, op + kTile2);
    split_smem2(rs + kTile2, op + 2 * kTile2, op + 3 * kTile2);
    e2a_fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) {
      tc_fence_after();
      const uint32_t d = tmem + (uint32_t)(((kb >> 1) & 1) * BN);
      const uint32_t a_hi = e2a_smem_u32(op), a_lo = a_hi + kTile2;
      const uint32_t b_hi = a_hi + 2 * kTile2, b_lo = a_hi + 3 * kTile2;
#pragma unroll
      for (int kk = 0; kk < BK2 / 8; ++kk) {
        const uint32_t koff = kk * 32;
        const uint32_t first = ((kb & 1) == 0 && kk == 0) ? 0u : 1u;
        mma_tf32(d, smem_desc_sw64(a_hi + koff), smem_desc_sw64(b_hi + koff), first);
        if (passes == 3) {
          mma_tf32(d, smem_desc_sw64(a_hi + koff), smem_desc_sw64(b_lo + koff), 1u);
          mma_tf32(d, smem_desc_sw64(a_lo + koff), smem_desc_sw64(b_hi + koff), 1u);
        }
      }
      mma_commit(&bars[kb & 1]);
    }
    // drain group (kb >> 1) - 1 before its TMEM buffer is reused by the next group.  Its last slab,
    // kb - 2, was awaited at the top of this iteration (waiting for it again here could see the
    // barrier's parity already advanced by slab kb's commit).
    if ((kb & 1) == 1 && kb >= 3) {
      drain((kb >> 1) - 1);
      tc_fence_before();
    }
  }
  cp_async_wait<0>();
  // drain the remaining (one or two) groups
  if (ok && nk > 0) {
    const int last_group = (nk - 1) >> 1;
    const int first_left = (nk >= 4 && (((nk - 1) & 1) == 1)) ? last_group : (nk >= 3 ? last_group - 1 : 0);
    for (int g = first_left; g <= last_group && ok; ++g) {
      const int last = min(2 * g + 1, nk - 1);
      ok = e2a_mbar_wait_bounded(&bars[last & 1], (last >> 1) & 1, &g_e2a_gemm_status);
      if (__syncthreads_or(!ok)) { ok = false; break; }
      drain(g);
    }
  }
  const bool all_ok = !__syncthreads_or(!ok);
  if (all_ok) {
    constexpr int kLd = BN + 4;
    float* tile = reinterpret_cast<float*>(smem2);  // raw + operand region, idle now (67.6 KB used)
    {
      float* trow = tile + (32 * q + lane) * kLd + 64 * half;
#pragma unroll
      for (int i = 0; i < BN / 2; i += 4)
        *reinterpret_cast<float4*>(trow + i) = make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]);
    }
    __syncthreads();
    const int gc = n0 + 4 * lane;
    float4 bv = make_float4(0.f, 0.f, 0.f, 0.f);
    if (bias) {
      if (gc < N) bv.x = bias[gc];
      if (gc + 1 < N) bv.y = bias[gc + 1];
      if (gc + 2 < N) bv.z = bias[gc + 2];
      if (gc + 3 < N) bv.w = bias[gc + 3];
    }
    const bool cvec = C && ((ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(C) & 15u) == 0) && (gc + 3 < N);
    for (int r = warp; r < BM; r += kThreads / 32) {
      const int row = m0 + r;
      if (row >= M) break;
      float4 x = *reinterpret_cast<const float4*>(tile + r * kLd + 4 * lane);
      x.x += bv.x; x.y += bv.y; x.z += bv.z; x.w += bv.w;
      if (P) {
        float* pp = P + (int64_t)row * ldp + (gc >> 1);
        if (gc + 1 < N) pp[0] = (accumulate ? pp[0] : 0.f) + x.x * x.y;
        if (gc + 3 < N) pp[1] = (accumulate ? pp[1] : 0.f) + x.z * x.w;
        if (!C) continue;
        float* cp = C + (int64_t)row * ldc + gc;
        if (cvec) {
          *reinterpret_cast<float4*>(cp) = x;
        } else {
          const float xv[4] = {x.x, x.y, x.z, x.w};
          for (int t = 0; t < 4; ++t)
            if (gc + t < N) cp[t] = xv[t];
        }
        continue;
      }
      float* cp = C + (int64_t)row * ldc + gc;
      if (cvec) {
        if (accumulate) {
          const float4 o = *reinterpret_cast<const float4*>(cp);
          x.x += o.x; x.y += o.y; x.z += o.z; x.w += o.w;
        }
        *reinterpret_cast<float4*>(cp) = x;
      } else {
        const float xv[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int t = 0; t < 4; ++t)
          if (gc + t < N) cp[t] = accumulate ? cp[t] + xv[t] : xv[t];
      }
    }
  } else if (threadIdx.x == 0 && nk > 0) {
    for (int pk = (nk >= 2 ? nk - 2 : 0); pk < nk; ++pk)
      e2a_mbar_wait_bounded(&bars[pk & 1], (pk >> 1) & 1, &g_e2a_gemm_status);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

}  // namespace

extern "C" {

int e2a_gemm_tf32x3(const float* A, int64_t lda, const float* B, int64_t ldb, float* C, int64_t ldc,
                    const float* bias, int64_t M, int64_t N, int64_t K, int accumulate, int passes, void* stream) {
  if (M < 0 || N < 0 || K < 0 || (passes != 1 && passes != 3)) return E2A_ERR_ARG;
  if (M == 0 || N == 0) return E2A_OK;
  if (!C || (K > 0 && (!A || !B)) || lda < K || ldb < K || ldc < N) return E2A_ERR_ARG;
  if ((M + BM - 1) / BM > INT32_MAX || (N + BN - 1) / BN > 65535 || K > INT32_MAX) return E2A_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const bool vec = (lda % 4 == 0) && (ldb % 4 == 0) && ((reinterpret_cast<uintptr_t>(A) & 15u) == 0) &&
                   ((reinterpret_cast<uintptr_t>(B) & 15u) == 0);
  dim3 grid((unsigned)((M + BM - 1) / BM), (unsigned)((N + BN - 1) / BN));
  if (vec) {
    E2A_CUDA(cudaFuncSetAttribute(k_gemm_tf32x3_v2, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem2));
    k_gemm_tf32x3_v2<<<grid, kThreads, kSmem2, st>>>(A, lda, B, ldb, C, ldc, bias, (int)M, (int)N, (int)K,
                                                     accumulate, passes, nullptr, 0);
  } else {
    E2A_CUDA(cudaFuncSetAttribute(k_gemm_tf32x3<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    k_gemm_tf32x3<false><<<grid, kThreads, kSmemBytes, st>>>(A, lda, B, ldb, C, ldc, bias, (int)M, (int)N, (int)K,
                                                             accumulate, passes);
  }
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

int e2a_gemm_tf32x3_pairprod(const float* A, int64_t lda, const float* B, int64_t ldb, float* C, int64_t ldc,
                             const float* bias, float* P, int64_t ldp, int64_t M, int64_t N, int64_t K,
                             int accumulate, int passes, void* stream) {
  if (M < 0 || N < 0 || K < 0 || (passes != 1 && passes != 3) || (N & 1)) return E2A_ERR_ARG;
  if (M == 0 || N == 0) return E2A_OK;
  if (!P || (K > 0 && (!A || !B)) || lda < K || ldb < K || (C && ldc < N) || ldp < N / 2) return E2A_ERR_ARG;
  if ((M + BM - 1) / BM > INT32_MAX || (N + BN - 1) / BN > 65535 || K > INT32_MAX) return E2A_ERR_ARG;
  const bool vec = (lda % 4 == 0) && (ldb % 4 == 0) && ((reinterpret_cast<uintptr_t>(A) & 15u) == 0) &&
                   ((reinterpret_cast<uintptr_t>(B) & 15u) == 0);
  if (!vec) return E2A_ERR_UNSUPPORTED;
  cudaStream_t st = (cudaStream_t)stream;
  dim3 grid((unsigned)((M + BM - 1) / BM), (unsigned)((N + BN - 1) / BN));
  E2A_CUDA(cudaFuncSetAttribute(k_gemm_tf32x3_v2, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem2));
  k_gemm_tf32x3_v2<<<grid, kThreads, kSmem2, st>>>(A, lda, B, ldb, C, ldc, bias, (int)M, (int)N, (int)K,
                                                   accumulate, passes, P, ldp);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

int e2a_gemm_status(unsigned int* status, int reset, void* stream) {
  if (!status) return E2A_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  E2A_CUDA(cudaMemcpyFromSymbolAsync(status, g_e2a_gemm_status, sizeof(unsigned int), 0, cudaMemcpyDeviceToHost, st));
  E2A_CUDA(cudaStreamSynchronize(st));
  if (reset) {
    const unsigned int zero = 0;
    E2A_CUDA(cudaMemcpyToSymbolAsync(g_e2a_gemm_status, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, st));
    E2A_CUDA(cudaStreamSynchronize(st));
  }
  return E2A_OK;
}

}  // extern "C"
