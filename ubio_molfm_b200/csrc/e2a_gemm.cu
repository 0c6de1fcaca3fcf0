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
#include <cuda.h>  // CUtensorMap; the encoder is fetched from the driver at run time
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

// D (+)= A B^T with A read from tensor memory (row m in lane m, k in consecutive columns)
__device__ __forceinline__ void mma_tf32_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(kIdesc), "r"(accumulate));
}

// this warp's 32 lanes x 16 consecutive columns of tensor memory from registers
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])),
        "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
        "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
        "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
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
// Warp-specialised persistent kernel for 16-byte-aligned operands.  One CTA per SM walks 128 x 128
// output tiles (n fastest, so CTAs running together share A rows in L2).  Roles:
//  * warp 0 (one lane): TMA producer -- per k-slab one 2-D tensor copy each of raw fp32 A and of B
//    (or of B_hi and B_lo when the caller pre-split the weight operand) into a stage ring, already
//    in the swizzled K-major layout the tensor core reads;
//  * warps 2-3 (and 12-13 for 32-wide slabs): splitters -- turn each raw slab into hi = tf32(x) (in
//    place) and lo = tf32(x - hi)
//    (A only when B arrives pre-split, which measured faster: shared-memory traffic per slab is the
//    tighter resource);
//  * warp 1 (one lane): MMA issuer -- tcgen05.mma kind::tf32 hi*hi + hi*lo + lo*hi into one of four
//    128-column TMEM chain buffers (a chain = 64 k, 24 MMAs), then tcgen05.commit frees the
//    stage and, at a chain end, hands the buffer to the drain warps;
//  * warps 4-11: drain every chain into fp32 registers with round-to-nearest adds (the tensor core's
//    own accumulation truncates, so chains are kept short), then run the tile's epilogue (bias /
//    accumulate / pair product) through a per-warp staging area with coalesced row stores.
// The roles meet only at mbarriers; there is no block-wide barrier in the loop.  Every wait is
// bounded (~2 s): a timeout sets E2A_DEV_WAIT_TIMEOUT and an abort flag that ends every role, and
// the producer / issuer then wait (bounded) for their copies / MMAs in flight before TMEM is freed.
// ------------------------------------------------------------------------------------------------
template <int V>
struct IntC { static constexpr int value = V; };

// Two slab shapes: 16-wide slabs (64-byte rows and swizzle, six stages) suit K <= 256, where tiles
// turn over quickly; 32-wide slabs (128-byte rows and swizzle, three stages) move more bytes per
// TMA request and suit long K.
#ifndef E2A_WS_CHAINS16
#define E2A_WS_CHAINS16 3
#endif
#ifndef E2A_WS_CHAINS32
#define E2A_WS_CHAINS32 3
#endif
#ifndef E2A_WS_ATS16
#define E2A_WS_ATS16 4
#endif
#ifndef E2A_WS_ATS32
#define E2A_WS_ATS32 2
#endif
// k per TMEM chain: the tensor core's accumulation truncates, so a longer chain costs accuracy and a
// shorter one costs drains.  Measured (err / err of torch's fp32 SIMT product, TFLOP/s at the model's
// shapes): 32 k 0.95x worst case; 64 k 1.53x and +5..19% throughput; 128 k 2.84x and +2..5% more.
#ifndef E2A_WS_CHAINK
#define E2A_WS_CHAINK 64
#endif
template <int BK_, bool PG_ = false>
struct WsCfg {
  static constexpr int BK = BK_;
  // PG: A is formed on chip from the projections O (loaded as the A slab) and the pair gradient G (one
  // extra half-width slab per stage): A[r, 2j] = G[r, j] O[r, 2j+1], A[r, 2j+1] = G[r, j] O[r, 2j]
  static constexpr bool PG = PG_;
  static constexpr int SPC = E2A_WS_CHAINK / BK;         // slabs per TMEM chain (64 k = 24 MMAs by default)
#ifndef E2A_WS_STAGES16
#define E2A_WS_STAGES16 6   // shared memory allows up to 8 (24 KB stages)
#endif
#ifndef E2A_WS_STAGES32
#define E2A_WS_STAGES32 4   // 48 KB stages
#endif
  static constexpr int STAGES = PG ? 3 : (BK == 16 ? E2A_WS_STAGES16 : E2A_WS_STAGES32);
  static constexpr int TILE = BM * BK * 4;               // bytes per operand part
  static constexpr int GSLAB = PG ? BM * (BK / 2) * 4 : 0;   // the G slab (64-byte rows, 64-byte swizzle)
  static constexpr int STAGE = 3 * TILE + GSLAB;         // A (raw), B (split in place when not pre-split), B_lo, G
  static constexpr int CHAINS = BK == 16 ? E2A_WS_CHAINS16 : E2A_WS_CHAINS32;   // TMEM chain buffers (BN columns)
  static constexpr int ATS = BK == 16 ? E2A_WS_ATS16 : E2A_WS_ATS32;  // A hi / lo slots in TMEM (2 BK columns each)
  static constexpr uint32_t ACOL = CHAINS * 128;         // first A-slot column
  static constexpr int NBARS = 3 * STAGES + 2 * CHAINS + ATS;
  static_assert(CHAINS * 128 + ATS * 2 * BK <= 512, "chain buffers + A slots exceed the 512 TMEM columns");
  static constexpr int SPLIT = 128;                      // splitter threads (warps 2-3 and 12-13)
  static constexpr int THREADS = 384 + (SPLIT - 64);      // + 8 drain warps (4-11)
  static __device__ __forceinline__ uint64_t desc(uint32_t addr) {
    // K-major; LBO unused (1); SBO = 8 rows x row bytes; version 1; swizzle 64 B (4) or 128 B (2)
    return (uint64_t)((addr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(BK * 4 * 8 / 16) << 32) | (1ull << 46) |
           ((BK == 16 ? 4ull : 2ull) << 61);
  }
};
constexpr int WS_DRAIN = 8;                      // drain warps: 4 TMEM lane quarters x 2 column halves
constexpr int WS_DCOLS = BN / 2;                 // accumulator columns per drain warp
constexpr int WS_EH = 16;                        // epilogue staged 16 columns at a time
constexpr int WS_LD = WS_EH + 4;                 // staging row stride (floats)
constexpr int WS_EPI = WS_DRAIN * 32 * WS_LD * 4;
constexpr uint32_t kWsTmemCols = 512;
template <int BK, bool PG = false>
constexpr int ws_smem() {
  return WsCfg<BK, PG>::STAGES * WsCfg<BK, PG>::STAGE + WS_EPI + WsCfg<BK, PG>::NBARS * 8 + 16 + 1024 + 1024;
}

__device__ __forceinline__ float tf32_lo(float a, float h) { return tf32_hi(a - h); }

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(e2a_smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(e2a_smem_u32(bar)) : "memory");
}
// 2-D tensor copy global -> this CTA's shared memory (this CTA only), completion on `bar`
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(e2a_smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(e2a_smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Bounded wait that also gives up when another role has set the abort flag.
__device__ __forceinline__ bool ws_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (e2a_mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = e2a_globaltimer();
  for (uint32_t it = 0;; ++it) {
    if (e2a_mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0u) {
      if (*abort_flag) return false;
      if (e2a_globaltimer() - t0 > 2000000000ull) {
        *abort_flag = 1;
        atomicOr(&g_e2a_gemm_status, E2A_DEV_WAIT_TIMEOUT);
        return false;
      }
    }
  }
}

#ifdef E2A_GEMM_TRACE
__device__ unsigned long long g_ws_trace[8][512];
#define WS_TRACE(k, i) do { if (blockIdx.x == 0 && (i) < 512) g_ws_trace[k][i] = e2a_globaltimer(); } while (0)
#else
#define WS_TRACE(k, i) do { } while (0)
#endif

// Gaussian radial basis rbf[m, k] = exp(coeff (d[m] - mu[k])^2) (module_utils.py:1853-1870) as a GEMM
// operand or epilogue factor:
//  * gen (d set, rdot null): A is not read; the splitter warps form A's tile from d and mu on chip;
//  * rdot (rdot set): the epilogue writes no C but, per row and 64-column block of the tile,
//    rdot[m, n / 64] = sum_n acc[m, n] * rbf[m, n] * 2 coeff (d[m] - mu[n])   (d rbf / d d, contracted).
struct RbfArgs {
  const float* d;
  const float* mu;
  float coeff;
  float* rdot;
  int64_t ld_rdot;
};

template <int BK_, bool PG_ = false>
__global__ void __launch_bounds__(WsCfg<BK_, PG_>::THREADS, 1)
k_gemm_ws(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
          const __grid_constant__ CUtensorMap tmBl, const __grid_constant__ CUtensorMap tmG, int b_split, float* C,
          int64_t ldc, const float* __restrict__ bias, float* P, int64_t ldp, int M, int N, int K, int accumulate,
          int passes, const RbfArgs rb) {
  using Cfg = WsCfg<BK_, PG_>;
  const bool gen = rb.d != nullptr && rb.rdot == nullptr;   // A formed on chip
  extern __shared__ uint8_t ws_raw[];
  uint8_t* smem = ws_raw + ((1024u - (e2a_smem_u32(ws_raw) & 1023u)) & 1023u);
  uint8_t* stages = smem;
  float* epi = reinterpret_cast<float*>(smem + Cfg::STAGES * Cfg::STAGE);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::STAGES * Cfg::STAGE + WS_EPI);
  uint64_t* full = bars;                          // TMA landed            (1 arrive + tx bytes)
  uint64_t* split_done = bars + Cfg::STAGES;        // A hi / lo written     (one per splitter)
  uint64_t* empty = bars + 2 * Cfg::STAGES;         // MMAs of the slab done (tcgen05.commit)
  uint64_t* tfull = bars + 3 * Cfg::STAGES;         // chain buffer ready    (tcgen05.commit)
  uint64_t* tempty = tfull + Cfg::CHAINS;           // chain buffer drained  (256 arrives)
  uint64_t* a_empty = tempty + Cfg::CHAINS;         // A slot read by the slab's MMAs (tcgen05.commit)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Cfg::NBARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* mu_s = reinterpret_cast<float*>(tmem_slot + 4);   // gen: the basis offsets (K <= 256)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_n = (N + BN - 1) / BN;
  const int tiles = ((M + BM - 1) / BM) * tiles_n;
  const int nk = (K + Cfg::BK - 1) / Cfg::BK;
  // slabs per TMEM chain: the whole K in one chain when K <= E2A_WS_CHAINK_SMALLK, else E2A_WS_CHAINK
#ifndef E2A_WS_CHAINK_SMALLK
#define E2A_WS_CHAINK_SMALLK 0
#endif
  const int spc = (K <= E2A_WS_CHAINK_SMALLK) ? (nk > 0 ? nk : 1) : Cfg::SPC;
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(e2a_smem_u32(tmem_slot)), "r"(kWsTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 32) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      e2a_mbar_init(&full[s], 1);
      e2a_mbar_init(&split_done[s], Cfg::SPLIT);
      e2a_mbar_init(&empty[s], 1);
    }
    for (int c = 0; c < Cfg::CHAINS; ++c) {
      e2a_mbar_init(&tfull[c], 1);
      e2a_mbar_init(&tempty[c], 32 * WS_DRAIN);
    }
    for (int a = 0; a < Cfg::ATS; ++a) e2a_mbar_init(&a_empty[a], 1);
    *abort_flag = 0;
    e2a_fence_mbar_init();
  }
  if (gen)
    for (int k = threadIdx.x; k < 256; k += blockDim.x) mu_s[k] = k < K ? __ldg(rb.mu + k) : 0.f;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
      if (b_split) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmBl)) : "memory");
      if (Cfg::PG) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmG)) : "memory");
      const uint32_t bytes = (b_split ? 2 : 1) * Cfg::TILE + (gen ? 0 : Cfg::TILE) + Cfg::GSLAB;
      uint32_t n = 0;
      bool run = true;
      for (int tile = blockIdx.x; tile < tiles && run; tile += gridDim.x) {
        const int m0 = (tile / tiles_n) * BM, n0 = (tile % tiles_n) * BN;
        for (int kb = 0; kb < nk; ++kb, ++n) {
          const uint32_t s = n % Cfg::STAGES;
          if (!ws_wait(&empty[s], ((n / Cfg::STAGES) & 1) ^ 1, abort_flag)) { run = false; break; }
          WS_TRACE(0, n);
          uint8_t* st = stages + s * Cfg::STAGE;
          mbar_expect_tx(&full[s], bytes);
          if (!gen) tma_load_2d(st, &tmA, kb * Cfg::BK, m0, &full[s]);
          tma_load_2d(st + Cfg::TILE, &tmB, kb * Cfg::BK, n0, &full[s]);
          if (b_split) tma_load_2d(st + 2 * Cfg::TILE, &tmBl, kb * Cfg::BK, n0, &full[s]);
          if (Cfg::PG) tma_load_2d(st + 3 * Cfg::TILE, &tmG, kb * (Cfg::BK / 2), m0, &full[s]);
        }
      }
      if (!run) {  // copies still in flight must land before the CTA exits
        for (uint32_t j = (n >= Cfg::STAGES ? n - Cfg::STAGES : 0); j < n; ++j)
          e2a_mbar_wait_bounded(&full[j % Cfg::STAGES], (j / Cfg::STAGES) & 1, &g_e2a_gemm_status);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t n = 0, c = 0;
      int64_t last = -1;  // last slab whose MMAs were committed
      bool run = true;
      for (int tile = blockIdx.x; tile < tiles && run; tile += gridDim.x) {
        for (int kb = 0; kb < nk; ++kb, ++n) {
          const uint32_t s = n % Cfg::STAGES, cb = c % Cfg::CHAINS;
          if ((kb % spc) == 0 && !ws_wait(&tempty[cb], ((c / Cfg::CHAINS) & 1) ^ 1, abort_flag)) { run = false; break; }
          if (!ws_wait(&split_done[s], (n / Cfg::STAGES) & 1, abort_flag)) { run = false; break; }
          WS_TRACE(3, n);
          tc_fence_after();
          const uint32_t d = tmem + cb * BN;
          const uint32_t a_hi = tmem + Cfg::ACOL + (n % Cfg::ATS) * 2 * Cfg::BK, a_lo = a_hi + Cfg::BK;
          const uint32_t b_hi = e2a_smem_u32(stages + s * Cfg::STAGE) + Cfg::TILE, b_lo = b_hi + Cfg::TILE;
#pragma unroll
          for (int kk = 0; kk < Cfg::BK / 8; ++kk) {
            const uint32_t koff = kk * 32;
            mma_tf32_ta(d, a_hi + 8 * kk, Cfg::desc(b_hi + koff), ((kb % spc) == 0 && kk == 0) ? 0u : 1u);
            if (passes == 3) {
              mma_tf32_ta(d, a_hi + 8 * kk, Cfg::desc(b_lo + koff), 1u);
              mma_tf32_ta(d, a_lo + 8 * kk, Cfg::desc(b_hi + koff), 1u);
            }
          }
          mma_commit(&empty[s]);
          mma_commit(&a_empty[n % Cfg::ATS]);
          last = n;
          if ((kb % spc) == spc - 1 || kb == nk - 1) {
            mma_commit(&tfull[cb]);
            ++c;
          }
        }
      }
      if (!run && last >= 0)  // let the committed MMAs finish before the tensor memory is freed
        e2a_mbar_wait_bounded(&empty[last % Cfg::STAGES], (uint32_t)((last / Cfg::STAGES) & 1), &g_e2a_gemm_status);
    }
  } else if (warp < 4 || warp >= 12) {
    // ------------------------------------------------------------------ splitters (4 warps)
    // Warp w owns tensor-memory lane quarter w % 4 (warps 2, 3, 12, 13: quarters 2, 3, 0, 1), so lane l of
    // it owns tile row 32 (w % 4) + l: it reads that row of the raw A slab from its swizzled stage (or forms
    // it from the radial basis), splits it into tf32 hi / lo in registers and stores both into this slab's
    // A slot in tensor memory, where the MMAs read it.  Shared memory then carries only the TMA writes and
    // the MMAs' B reads.
    static_assert(Cfg::SPLIT == 128, "four splitter warps cover the four lane quarters");
    const int q = warp & 3;
    const int r = 32 * q + lane;                              // tile row of this thread
    const uint32_t lane_addr = (uint32_t)(32 * q) << 16;
    const int t = warp < 4 ? threadIdx.x - 64 : threadIdx.x - 320;   // 0 .. 127 (B split)
    const float c2 = rb.coeff * 1.44269504088896341f;         // gen: exp(a) = 2^(a log2 e)
    uint32_t n = 0;
    bool run = true;
    float dcur = 0.f, dnext = 0.f;                            // gen: this row's distance, this / next tile
    if (gen) {
      const int row = ((int)blockIdx.x / tiles_n) * BM + r;
      dnext = (int)blockIdx.x < tiles && row < M ? __ldg(rb.d + row) : 0.f;
    }
    for (int tile = blockIdx.x; tile < tiles && run; tile += gridDim.x) {
      for (int kb = 0; kb < nk; ++kb, ++n) {
        const uint32_t s = n % Cfg::STAGES;
        if (!ws_wait(&full[s], (n / Cfg::STAGES) & 1, abort_flag)) { run = false; break; }
        // the A slot must have been read by the MMAs of slab n - ATS
        if (!ws_wait(&a_empty[n % Cfg::ATS], ((n / Cfg::ATS) & 1) ^ 1, abort_flag)) { run = false; break; }
        if (t == 0) WS_TRACE(1, n);
        uint8_t* st = stages + s * Cfg::STAGE;
        if (gen && kb == 0) {   // this tile's distance (prefetched a tile ahead), then the next tile's
          dcur = dnext;
          const int row = ((tile + (int)gridDim.x) / tiles_n) * BM + r;
          dnext = tile + (int)gridDim.x < tiles && row < M ? __ldg(rb.d + row) : 0.f;
        }
        const uint32_t acol = tmem + lane_addr + Cfg::ACOL + (n % Cfg::ATS) * 2 * Cfg::BK;
#pragma unroll
        for (int h = 0; h < Cfg::BK / 16; ++h) {   // 16 columns at a time
          float v[16], hi[16], lo[16];
          if (gen) {
#pragma unroll
            for (int u = 0; u < 16; ++u) {
              const int k = kb * Cfg::BK + 16 * h + u;
              const float x = dcur - mu_s[k & 255];
              v[u] = k < K ? exp2f(c2 * (x * x)) : 0.f;
            }
          } else {
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) {
              // logical 16-byte chunk c of the row sits at chunk c ^ ((r / 2) % 4) (64-byte swizzle, 16-wide
              // slabs) or c ^ (r % 8) (128-byte swizzle, 32-wide slabs)
              const int c = 4 * h + c4;
              const int pc = Cfg::BK == 16 ? (c ^ ((r >> 1) & 3)) : (c ^ (r & 7));
              const float4 x = *reinterpret_cast<const float4*>(st + r * (Cfg::BK * 4) + 16 * pc);
              v[4 * c4] = x.x; v[4 * c4 + 1] = x.y; v[4 * c4 + 2] = x.z; v[4 * c4 + 3] = x.w;
            }
            if constexpr (Cfg::PG) {
              // G columns 8h .. 8h+7 of this row: logical 16-byte chunks 2h, 2h+1 of its 64-byte G row
              // (64-byte swizzle: chunk c at c ^ ((r / 2) % 4)); A[2i] = G[i] O[2i+1], A[2i+1] = G[i] O[2i]
              const uint8_t* gs = st + 3 * Cfg::TILE + r * (Cfg::BK / 2) * 4;
              float g[8];
#pragma unroll
              for (int c2 = 0; c2 < 2; ++c2) {
                const int pc = (2 * h + c2) ^ ((r >> 1) & 3);
                const float4 x = *reinterpret_cast<const float4*>(gs + 16 * pc);
                g[4 * c2] = x.x; g[4 * c2 + 1] = x.y; g[4 * c2 + 2] = x.z; g[4 * c2 + 3] = x.w;
              }
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const float o0 = v[2 * i], o1 = v[2 * i + 1];
                v[2 * i] = g[i] * o1;
                v[2 * i + 1] = g[i] * o0;
              }
            }
          }
#pragma unroll
          for (int u = 0; u < 16; ++u) {
            hi[u] = tf32_hi(v[u]);
            lo[u] = tf32_lo(v[u], hi[u]);
          }
          tmem_st16(acol + 16 * h, hi);
          tmem_st16(acol + Cfg::BK + 16 * h, lo);
        }
        if (!b_split) {   // B's tile split in place (hi) and into the B_lo part
#pragma unroll
          for (int j = 0; j < Cfg::TILE / 16 / Cfg::SPLIT; ++j) {
            const int off = Cfg::TILE + (t + j * Cfg::SPLIT) * 16;
            const float4 x = *reinterpret_cast<const float4*>(st + off);
            float4 hh, ll;
            hh.x = tf32_hi(x.x); hh.y = tf32_hi(x.y); hh.z = tf32_hi(x.z); hh.w = tf32_hi(x.w);
            ll.x = tf32_lo(x.x, hh.x); ll.y = tf32_lo(x.y, hh.y); ll.z = tf32_lo(x.z, hh.z); ll.w = tf32_lo(x.w, hh.w);
            *reinterpret_cast<float4*>(st + off) = hh;
            *reinterpret_cast<float4*>(st + Cfg::TILE + off) = ll;
          }
          e2a_fence_proxy_async();
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        mbar_arrive(&split_done[s]);
        if (t == 0) WS_TRACE(2, n);
      }
    }
  } else {
    // ------------------------------------------------------------------ drain + epilogue (8 warps)
    const int q = warp & 3;                        // TMEM lane quarter this warp may read
    const int half = (warp - 4) >> 2;              // column half of the tile
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    float* stg = epi + (warp - 4) * 32 * WS_LD;
    uint32_t c = 0;
    bool run = true;
    const int nch = (nk + spc - 1) / spc;
    for (int tile = blockIdx.x; tile < tiles && run; tile += gridDim.x) {
      const int m0 = (tile / tiles_n) * BM, n0 = (tile % tiles_n) * BN + WS_DCOLS * half;
      float acc[WS_DCOLS];
#pragma unroll
      for (int i = 0; i < WS_DCOLS; ++i) acc[i] = 0.f;
      for (int ch = 0; ch < nch; ++ch, ++c) {
        const uint32_t cb = c % Cfg::CHAINS;
        if (!ws_wait(&tfull[cb], (c / Cfg::CHAINS) & 1, abort_flag)) { run = false; break; }
        if (threadIdx.x == 128) WS_TRACE(4, c);
        tc_fence_after();
#pragma unroll
        for (int h = 0; h < WS_DCOLS / 32; ++h) {
          float v[32];
#pragma unroll
          for (int j = 0; j < 2; ++j)
            tmem_ld16_nowait(tmem + lane_base + cb * BN + WS_DCOLS * half + 32 * h + 16 * j, v + 16 * j);
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[32 * h + i] += v[i];
        }
        tc_fence_before();
        mbar_arrive(&tempty[cb]);
        if (threadIdx.x == 128) WS_TRACE(5, c);
      }
      if (!run) break;
      if (rb.rdot) {   // contract this warp's 64 columns with d rbf / d d; no C
        const int row = m0 + 32 * q + lane;
        if (row < M && n0 < N) {
          const float dv = __ldg(rb.d + row);
          float sum = 0.f;
#pragma unroll
          for (int j = 0; j < WS_DCOLS; ++j) {   // fully unrolled: acc stays in registers
            if (n0 + j < N) {
              const float x = dv - __ldg(rb.mu + n0 + j);
              sum += acc[j] * expf(rb.coeff * (x * x)) * (2.f * rb.coeff * x);
            }
          }
          rb.rdot[(int64_t)row * rb.ld_rdot + n0 / WS_DCOLS] = sum;
        }
        continue;
      }
      // epilogue: stage this warp's 32 rows x 64 columns 16 columns at a time, then write them row by
      // row (4 lanes per row, 8 rows per step)
#pragma unroll
      for (int hh = 0; hh < WS_DCOLS / WS_EH; ++hh) {
#pragma unroll
        for (int i = 0; i < WS_EH; i += 4)
          *reinterpret_cast<float4*>(stg + lane * WS_LD + i) =
              make_float4(acc[hh * WS_EH + i], acc[hh * WS_EH + i + 1], acc[hh * WS_EH + i + 2], acc[hh * WS_EH + i + 3]);
        __syncwarp();
        constexpr int kLanesPerRow = WS_EH / 4, kRowsPerStep = 32 / kLanesPerRow;
        const int sub = lane % kLanesPerRow, rr = lane / kLanesPerRow;
        const int gc = n0 + hh * WS_EH + 4 * sub;
        float4 bv = make_float4(0.f, 0.f, 0.f, 0.f);
        if (bias) {
          if (gc < N) bv.x = bias[gc];
          if (gc + 1 < N) bv.y = bias[gc + 1];
          if (gc + 2 < N) bv.z = bias[gc + 2];
          if (gc + 3 < N) bv.w = bias[gc + 3];
        }
        const bool cvec = C && ((ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(C) & 15u) == 0) && (gc + 3 < N);
        constexpr int kSteps = 32 / kRowsPerStep;
        // the previous values of a read-modify-write output (P with accumulate, or C with accumulate) are
        // loaded for all of this warp's row steps first, so their memory latencies overlap instead of
        // adding up one row step at a time
        float4 old[kSteps];
#pragma unroll
        for (int st2 = 0; st2 < kSteps; ++st2) {
          old[st2] = make_float4(0.f, 0.f, 0.f, 0.f);
          const int row = m0 + 32 * q + st2 * kRowsPerStep + rr;
          if (!accumulate || row >= M) continue;
          if (P) {
            const float* pp = P + (int64_t)row * ldp + (gc >> 1);
            if (gc + 1 < N) old[st2].x = pp[0];
            if (gc + 3 < N) old[st2].y = pp[1];
          } else if (cvec) {
            old[st2] = *reinterpret_cast<const float4*>(C + (int64_t)row * ldc + gc);
          }
        }
#pragma unroll
        for (int st2 = 0; st2 < kSteps; ++st2) {
          const int r = st2 * kRowsPerStep + rr;
          const int row = m0 + 32 * q + r;
          if (row >= M) continue;
          float4 x = *reinterpret_cast<const float4*>(stg + r * WS_LD + 4 * sub);
          x.x += bv.x; x.y += bv.y; x.z += bv.z; x.w += bv.w;
          if (P) {
            float* pp = P + (int64_t)row * ldp + (gc >> 1);
            if (gc + 1 < N) pp[0] = old[st2].x + x.x * x.y;
            if (gc + 3 < N) pp[1] = old[st2].y + x.z * x.w;
            if (!C) continue;
            float* cp = C + (int64_t)row * ldc + gc;
            if (cvec) {
              *reinterpret_cast<float4*>(cp) = x;
            } else {
              const float xv[4] = {x.x, x.y, x.z, x.w};
              for (int u = 0; u < 4; ++u)
                if (gc + u < N) cp[u] = xv[u];
            }
            continue;
          }
          float* cp = C + (int64_t)row * ldc + gc;
          if (cvec) {
            if (accumulate) {
              x.x += old[st2].x; x.y += old[st2].y; x.z += old[st2].z; x.w += old[st2].w;
            }
            *reinterpret_cast<float4*>(cp) = x;
          } else {
            const float xv[4] = {x.x, x.y, x.z, x.w};
            for (int u = 0; u < 4; ++u)
              if (gc + u < N) cp[u] = accumulate ? cp[u] + xv[u] : xv[u];
          }
        }
        __syncwarp();
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kWsTmemCols) : "memory");
  }
}

}  // namespace

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled from the driver through the runtime (no link against libcuda)
EncodeTiledFn tensor_map_encoder() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// [rows, cols] fp32 row-major with leading dim ld: bk x 128 boxes, (bk * 4)-byte swizzle, zero fill
bool make_map_2d(EncodeTiledFn enc, CUtensorMap* map, const float* base, int64_t rows, int64_t cols, int64_t ld,
                 int bk) {
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  const cuuint32_t box[2] = {(cuuint32_t)bk, (cuuint32_t)BM};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, bk == 16 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

__global__ void k_tf32_split(const float* __restrict__ B, int64_t ldb, int64_t N, int K, float* __restrict__ hi,
                             float* __restrict__ lo, int64_t ldo) {
  const int64_t total = N * (int64_t)K;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / K;
    const int c = (int)(i - r * K);
    const float x = B[r * ldb + c];
    const float h = tf32_hi(x);
    hi[r * ldo + c] = h;
    lo[r * ldo + c] = tf32_lo(x, h);
  }
}

}  // namespace

// Launches the warp-specialised kernel; E2A_ERR_UNSUPPORTED when the operands do not suit it.
static int launch_ws(const float* A, int64_t lda, const float* B, const float* B_lo, int64_t ldb, float* C,
                     int64_t ldc, const float* bias, float* P, int64_t ldp, int64_t M, int64_t N, int64_t K,
                     int accumulate, int passes, cudaStream_t st, RbfArgs rb = RbfArgs{nullptr, nullptr, 0.f, nullptr, 0},
                     const float* G = nullptr, int64_t ldg = 0) {
  const bool gen = rb.d != nullptr && rb.rdot == nullptr;
  if (gen) { A = B; lda = ldb; }   // the A map is never read
  const bool vec = (lda % 4 == 0) && (ldb % 4 == 0) && ((reinterpret_cast<uintptr_t>(A) & 15u) == 0) &&
                   ((reinterpret_cast<uintptr_t>(B) & 15u) == 0) && ((reinterpret_cast<uintptr_t>(B_lo) & 15u) == 0);
  if (!vec || K == 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return E2A_ERR_UNSUPPORTED;
  EncodeTiledFn enc = tensor_map_encoder();
  if (!enc) return E2A_ERR_UNSUPPORTED;
  // 32-wide slabs (four stages) from K = E2A_WS_BK32_MINK up; 16-wide for shorter K and for the on-chip basis
  // (K = 128 measured 7-17% faster with 32-wide slabs)
#ifndef E2A_WS_BK32_MINK
#define E2A_WS_BK32_MINK 128
#endif
#ifndef E2A_WS_GEN_BK32
#define E2A_WS_GEN_BK32 0
#endif
  // the pair-gradient mode always runs 32-wide slabs
  const int bk = G ? 32 : (((gen && !E2A_WS_GEN_BK32) || K < E2A_WS_BK32_MINK) ? 16 : 32);
  if (G && ((K % 32) != 0 || !B_lo || (ldg % 4) != 0 || (reinterpret_cast<uintptr_t>(G) & 15u) != 0))
    return E2A_ERR_UNSUPPORTED;
  CUtensorMap ta, tb, tbl, tg;
  if (!make_map_2d(enc, &ta, A, gen ? N : M, K, lda, bk) || !make_map_2d(enc, &tb, B, N, K, ldb, bk) ||
      !make_map_2d(enc, &tbl, B_lo ? B_lo : B, N, K, ldb, bk))
    return E2A_ERR_UNSUPPORTED;
  // the pair-gradient slab: K / 2 columns of G, 16-column boxes with the 64-byte swizzle
  if (G ? !make_map_2d(enc, &tg, G, M, K / 2, ldg, 16) : false) return E2A_ERR_UNSUPPORTED;
  if (!G) tg = ta;   // not read
  int dev = 0, sms = 0;
  E2A_CUDA(cudaGetDevice(&dev));
  E2A_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  if (tiles > INT32_MAX) return E2A_ERR_ARG;
  const int grid = (int)(tiles < sms ? tiles : sms);
  if (G) {
    E2A_CUDA(cudaFuncSetAttribute(k_gemm_ws<32, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, ws_smem<32, true>()));
    k_gemm_ws<32, true><<<grid, WsCfg<32, true>::THREADS, ws_smem<32, true>(), st>>>(
        ta, tb, tbl, tg, 1, C, ldc, bias, P, ldp, (int)M, (int)N, (int)K, accumulate, passes, rb);
  } else if (bk == 16) {
    E2A_CUDA(cudaFuncSetAttribute(k_gemm_ws<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, ws_smem<16>()));
    k_gemm_ws<16><<<grid, WsCfg<16>::THREADS, ws_smem<16>(), st>>>(ta, tb, tbl, tg, B_lo ? 1 : 0, C, ldc, bias, P, ldp,
                                                            (int)M, (int)N, (int)K, accumulate, passes, rb);
  } else {
    E2A_CUDA(cudaFuncSetAttribute(k_gemm_ws<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, ws_smem<32>()));
    k_gemm_ws<32><<<grid, WsCfg<32>::THREADS, ws_smem<32>(), st>>>(ta, tb, tbl, tg, B_lo ? 1 : 0, C, ldc, bias, P, ldp,
                                                            (int)M, (int)N, (int)K, accumulate, passes, rb);
  }
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

extern "C" {

int e2a_gemm_tf32x3(const float* A, int64_t lda, const float* B, const float* B_lo, int64_t ldb, float* C,
                    int64_t ldc, const float* bias, int64_t M, int64_t N, int64_t K, int accumulate, int passes,
                    void* stream) {
  if (M < 0 || N < 0 || K < 0 || (passes != 1 && passes != 3)) return E2A_ERR_ARG;
  if (M == 0 || N == 0) return E2A_OK;
  if (!C || (K > 0 && (!A || !B)) || lda < K || ldb < K || ldc < N) return E2A_ERR_ARG;
  if ((M + BM - 1) / BM > INT32_MAX || (N + BN - 1) / BN > 65535 || K > INT32_MAX) return E2A_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const int r = launch_ws(A, lda, B, B_lo, ldb, C, ldc, bias, nullptr, 0, M, N, K, accumulate, passes, st);
  if (r != E2A_ERR_UNSUPPORTED) return r;
  if (B_lo) return E2A_ERR_UNSUPPORTED;  // a pre-split B needs the pipelined kernel
  // general operands (unaligned rows, K = 0): the register-staged kernel
  dim3 grid((unsigned)((M + BM - 1) / BM), (unsigned)((N + BN - 1) / BN));
  E2A_CUDA(cudaFuncSetAttribute(k_gemm_tf32x3<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
  k_gemm_tf32x3<false><<<grid, kThreads, kSmemBytes, st>>>(A, lda, B, ldb, C, ldc, bias, (int)M, (int)N, (int)K,
                                                           accumulate, passes);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

int e2a_gemm_tf32x3_pairprod(const float* A, int64_t lda, const float* B, const float* B_lo, int64_t ldb, float* C,
                             int64_t ldc, const float* bias, float* P, int64_t ldp, int64_t M, int64_t N, int64_t K,
                             int accumulate, int passes, void* stream) {
  if (M < 0 || N < 0 || K < 0 || (passes != 1 && passes != 3) || (N & 1)) return E2A_ERR_ARG;
  if (M == 0 || N == 0) return E2A_OK;
  if (!P || (K > 0 && (!A || !B)) || lda < K || ldb < K || (C && ldc < N) || ldp < N / 2) return E2A_ERR_ARG;
  return launch_ws(A, lda, B, B_lo, ldb, C, ldc, bias, P, ldp, M, N, K, accumulate, passes, (cudaStream_t)stream);
}

int e2a_gemm_tf32x3_pairgrad(const float* O, int64_t ldo, const float* G, int64_t ldg, const float* B,
                             const float* B_lo, int64_t ldb, float* C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                             int passes, void* stream) {
  if (M < 0 || N < 0 || K < 0 || (passes != 1 && passes != 3) || (K & 1)) return E2A_ERR_ARG;
  if (M == 0 || N == 0) return E2A_OK;
  if (!O || !G || !B || !B_lo || !C || ldo < K || ldg < K / 2 || ldb < K || ldc < N) return E2A_ERR_ARG;
  return launch_ws(O, ldo, B, B_lo, ldb, C, ldc, nullptr, nullptr, 0, M, N, K, 0, passes, (cudaStream_t)stream,
                   RbfArgs{nullptr, nullptr, 0.f, nullptr, 0}, G, ldg);
}

int e2a_gemm_tf32x3_rbf(const float* dist, const float* mu, float coeff, const float* B, const float* B_lo,
                        int64_t ldb, float* C, int64_t ldc, const float* bias, int64_t M, int64_t N, int64_t K,
                        int passes, void* stream) {
  if (M < 0 || N < 0 || K < 0 || (passes != 1 && passes != 3)) return E2A_ERR_ARG;
  if (M == 0 || N == 0) return E2A_OK;
  if (!C || !dist || !mu || !B || K == 0 || ldb < K || ldc < N) return E2A_ERR_ARG;
  if (K > 256) return E2A_ERR_UNSUPPORTED;
  return launch_ws(nullptr, 0, B, B_lo, ldb, C, ldc, bias, nullptr, 0, M, N, K, 0, passes, (cudaStream_t)stream,
                   RbfArgs{dist, mu, coeff, nullptr, 0});
}

int e2a_gemm_tf32x3_rbf_dist_grad(const float* A, int64_t lda, const float* B, const float* B_lo, int64_t ldb,
                                  const float* dist, const float* mu, float coeff, float* partial, int64_t ld_partial,
                                  int64_t M, int64_t N, int64_t K, int passes, void* stream) {
  if (M < 0 || N < 0 || K < 0 || (passes != 1 && passes != 3)) return E2A_ERR_ARG;
  if (M == 0 || N == 0) return E2A_OK;
  if (!A || !B || !dist || !mu || !partial || K == 0 || lda < K || ldb < K || ld_partial < (N + 63) / 64)
    return E2A_ERR_ARG;
  return launch_ws(A, lda, B, B_lo, ldb, nullptr, 0, nullptr, nullptr, 0, M, N, K, 0, passes, (cudaStream_t)stream,
                   RbfArgs{dist, mu, coeff, partial, ld_partial});
}

int e2a_tf32_split(const float* B, int64_t ldb, int64_t N, int64_t K, float* B_hi, float* B_lo, int64_t ldo,
                   void* stream) {
  if (N < 0 || K < 0 || K > INT32_MAX) return E2A_ERR_ARG;
  if (N == 0 || K == 0) return E2A_OK;
  if (!B || !B_hi || !B_lo || ldb < K || ldo < K) return E2A_ERR_ARG;
  const int64_t total = N * K;
  const int64_t blocks = (total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096;
  k_tf32_split<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(B, ldb, N, (int)K, B_hi, B_lo, ldo);
  E2A_CHECK_LAUNCH();
  return E2A_OK;
}

#ifdef E2A_GEMM_TRACE
int e2a_gemm_trace(unsigned long long* out) {
  E2A_CUDA(cudaMemcpyFromSymbol(out, g_ws_trace, sizeof(g_ws_trace)));
  return E2A_OK;
}
#endif

// One thread waits, through the same bounded wait the GEMM roles use, on an mbarrier that nothing
// arrives at: the wait gives up after `limit_ns` and records E2A_DEV_WAIT_TIMEOUT in the GEMM's status
// word, so the host-side reporting path can be exercised without a stuck kernel.
__global__ void k_gemm_wait_selftest(uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  e2a_mbar_init(&bar, 1);
  e2a_fence_mbar_init();
  e2a_mbar_wait_bounded(&bar, 0, &g_e2a_gemm_status, limit_ns);
}

int e2a_gemm_wait_selftest(long long limit_ns, void* stream) {
  if (limit_ns < 1000 || limit_ns > 100000000LL) return E2A_ERR_ARG;
  k_gemm_wait_selftest<<<1, 32, 0, (cudaStream_t)stream>>>((uint64_t)limit_ns);
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
