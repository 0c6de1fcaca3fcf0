// Shared helpers for the E2Former-V2 attention kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "../../include/e2a.h"

#define E2A_CHECK_LAUNCH()                                   \
  do {                                                       \
    e2a_note_launch();                                       \
    cudaError_t _e = cudaGetLastError();                     \
    if (_e != cudaSuccess) { e2a_set_cuda_error(_e); return E2A_ERR_CUDA; } \
  } while (0)

#define E2A_CUDA(call)                                       \
  do {                                                       \
    cudaError_t _e = (call);                                 \
    if (_e != cudaSuccess) { e2a_set_cuda_error(_e); return E2A_ERR_CUDA; } \
  } while (0)

void e2a_set_cuda_error(cudaError_t e);
void e2a_note_launch();  // counts kernel launches for e2a_launch_count

static inline size_t e2a_align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Bump allocator over a caller-provided workspace.  Every sub-buffer is 256-byte aligned.
struct E2aArena {
  char* base;
  size_t cap;
  size_t used;
  __host__ void* take(size_t bytes) {
    size_t off = e2a_align_up(used, 256);
    used = off + e2a_align_up(bytes, 256);
    if (base == nullptr || used > cap) return nullptr;
    return base + off;
  }
};

__device__ __forceinline__ float e2a_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Two independent round-to-nearest fp32 fmas in one instruction (Blackwell's packed f32x2 pipe):
// the same results as two fmaf calls, half the issue slots.
__device__ __forceinline__ float2 f2_fma(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(d)
      : "l"(*reinterpret_cast<const uint64_t*>(&a)), "l"(*reinterpret_cast<const uint64_t*>(&b)),
        "l"(*reinterpret_cast<const uint64_t*>(&c)));
  return *reinterpret_cast<float2*>(&d);
}

__device__ __forceinline__ float4 f4_fma(float s, float4 v, float4 acc) {
  const float2 ss = make_float2(s, s);
  const float2 lo = f2_fma(ss, make_float2(v.x, v.y), make_float2(acc.x, acc.y));
  const float2 hi = f2_fma(ss, make_float2(v.z, v.w), make_float2(acc.z, acc.w));
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}

__device__ __forceinline__ float4 f4_fma4(float4 s, float4 v, float4 acc) {
  const float2 lo = f2_fma(make_float2(s.x, s.y), make_float2(v.x, v.y), make_float2(acc.x, acc.y));
  const float2 hi = f2_fma(make_float2(s.z, s.w), make_float2(v.z, v.w), make_float2(acc.z, acc.w));
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}

__device__ __forceinline__ float4 f4_zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// Four consecutive bf16 values (one 8-byte load) widened to fp32; bf16 -> fp32 is exact (the bf16 bits
// are the high half of the fp32 word).
struct e2a_bf16x4 { uint16_t v[4]; };
__device__ __forceinline__ float4 ldg4(const e2a_bf16x4* p) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u), __uint_as_float(u.y << 16),
                     __uint_as_float(u.y & 0xFFFF0000u));
}
// Row element offsets counted in values: float rows are addressed per value, bf16 rows per group of four.
__device__ __forceinline__ float4 ld4v(const float* base, int64_t off) { return ldg4(base + off); }
__device__ __forceinline__ float4 ld4v(const e2a_bf16x4* base, int64_t off) { return ldg4(base + (off >> 2)); }

// Euclidean norm of a 3-vector, evaluated as fma(z,z,fma(y,y,x*x)) then a correctly rounded
// sqrt: the exact fp32 operation sequence of PyTorch's CPU vector-norm kernel for a length-3
// reduction (torch.linalg.norm / torch.norm, p=2), which the reference uses for every distance
// (module_utils.py:3164, 1205).  Bit-equal distances are what makes the edge lists bit-exact.
__device__ __forceinline__ float e2a_norm3(float x, float y, float z) {
  return __fsqrt_rn(__fmaf_rn(z, z, __fmaf_rn(y, y, __fmul_rn(x, x))));
}

// ------------------------------------------------------------------------------------------------
// mbarrier / async-proxy primitives.  Every wait is bounded in time.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t e2a_smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void e2a_mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(e2a_smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void e2a_fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// orders this thread's (and, after a barrier, the block's) generic shared-memory accesses before
// later async-proxy accesses (tensor-core operand reads, bulk copies)
__device__ __forceinline__ void e2a_fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ bool e2a_mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(e2a_smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t e2a_globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

#define E2A_DEV_WAIT_TIMEOUT 1u

// Wait for phase `parity` of `bar`, giving up after `limit_ns` (~2 s by default; then sets
// E2A_DEV_WAIT_TIMEOUT in *status); returns false on timeout.
__device__ __forceinline__ bool e2a_mbar_wait_bounded(uint64_t* bar, uint32_t parity, unsigned int* status,
                                                      uint64_t limit_ns = 2000000000ull) {
  if (e2a_mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = e2a_globaltimer();
  for (uint32_t it = 0; it < (1u << 30); ++it) {
    if (e2a_mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0u && e2a_globaltimer() - t0 > limit_ns) break;
  }
  atomicOr(status, E2A_DEV_WAIT_TIMEOUT);
  return false;
}
