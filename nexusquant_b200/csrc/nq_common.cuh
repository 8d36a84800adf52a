// Shared device helpers for the NexusQuant B200 kernels (sm_100a only).
//
// Floating-point rule for every kernel in this library: each multiply and add
// is written with an explicit round-to-nearest intrinsic (__fmul_rn, __fadd_rn,
// __fsub_rn, __fmaf_rn) so that nvcc never contracts them into a fused
// multiply-add.  The lattice codes are then a deterministic function of the
// input bits, identical to the CPU oracle built with -ffp-contract=off.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "nexusquant_b200 kernels target sm_100a only"
#endif

namespace nq {

constexpr float kMagic = 12582912.0f;          // 1.5 * 2^23 : x + kMagic rounds x to an integer (RNE)
constexpr uint32_t kMagicBits = 0x4B400000u;   // bit pattern of kMagic

// fl32(1/sqrt(n)): the entry magnitude of the reference's orthonormal Sylvester
// Hadamard matrix of order n (nexusquant/core/hadamard.py:23-43).
__host__ __device__ constexpr float hadamard_entry(int n) {
  return n == 8 ? 0.35355339059327373f
       : n == 16 ? 0.25f
       : n == 32 ? 0.17677669529663687f
       : n == 64 ? 0.125f
       : n == 128 ? 0.08838834764831845f
       : 0.0625f;
}

// ------------------------------------------------- packed fp32 pairs (sm_100)
// Two IEEE-rounded fp32 results per instruction, bit-identical to scalar code.
typedef unsigned long long u64;

__device__ __forceinline__ u64 pk(float a, float b) {
  u64 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void upk(u64 p, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(p));
}
__device__ __forceinline__ u64 add2(u64 a, u64 b) {
  u64 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ u64 sub2(u64 a, u64 b) {
  u64 r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ u64 mul2(u64 a, u64 b) {
  u64 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ u64 fma2(u64 a, u64 b, u64 c) {
  u64 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ----------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}
// Bounded wait on phase `parity`.  Returns false when the iteration budget ran
// out (the caller records an error flag and carries on; nothing spins forever).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t max_iters = (1u << 26)) {
  uint32_t done = 0;
  for (uint32_t it = 0; it < max_iters; ++it) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

// 1-D bulk copy global -> shared through the TMA engine (no multicast).
// dst and src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// L2 cache policy for data read once (streamed) vs data reused across CTAs.
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void bulk_g2s_hint(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// ------------------------------------------------------------- conversions
template <typename T>
struct InTraits;
template <>
struct InTraits<__half> {
  static constexpr int kBytes = 2;
};
template <>
struct InTraits<__nv_bfloat16> {
  static constexpr int kBytes = 2;
};
template <>
struct InTraits<float> {
  static constexpr int kBytes = 4;
};

// Load 8 consecutive elements from shared memory (16-byte aligned for 2-byte
// types, 32-byte for float) and widen to fp32 (exact).
__device__ __forceinline__ void load8(const __half* p, float* o) {
  uint4 r = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __half22float2(h[i]);
    o[2 * i] = f.x;
    o[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* o) {
  uint4 r = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    o[2 * i] = f.x;
    o[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void load8(const float* p, float* o) {
  float4 a = *reinterpret_cast<const float4*>(p);
  float4 b = *reinterpret_cast<const float4*>(p + 4);
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
  o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}

// Correctly rounded y / b given r = RN(1/b): one residual correction
// (Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Dev. 34(1), 1990; also Muller et al.,
// Handbook of Floating-Point Arithmetic, the "Markstein" division iteration):
//   q = RN(y*r);  rem = y - b*q (exact through FMA);  RN(q + rem*r).
// Valid for normal b and quotients well inside the normal range, which holds
// for the quantizer (|y / b| <= L/2, b >= 1.25e-9); checked against __fdiv_rn
// by the GPU tests.
__device__ __forceinline__ float div_by(float y, float b, float r) {
  float q = __fmul_rn(y, r);
  float rem = __fmaf_rn(-q, b, y);
  return __fmaf_rn(rem, r, q);
}

}  // namespace nq
