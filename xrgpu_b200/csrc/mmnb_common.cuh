// Device helpers shared by the MatMulNBits kernels (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

#include "mmnb_internal.h"

namespace xrgpu {

// Kernels record a nonzero code in the device error word (atomicMax) when a bounded wait
// expires; the host reads it after synchronising (the reference's scratch error word,
// framework.glsl:64, checked on the host as in vulkan.cpp:115).
__device__ __forceinline__ void record_device_error(unsigned* word, unsigned code) {
  if (word) atomicMax(word, code);
}

__device__ __forceinline__ float load_f(const void* p, int f16, int64_t i) {
  return f16 ? __half2float(reinterpret_cast<const __half*>(p)[i]) : reinterpret_cast<const float*>(p)[i];
}

// Zero point of (column n, block blk) as float; 2^(bits-1) when absent (complex_kernel.glsl:80).
// Packed uint8 zero points are low-first with row stride ceil(kb*bits/8) (complex_kernel.glsl:85).
__device__ __forceinline__ float load_zero_point(const Problem& p, int64_t n, int64_t blk) {
  switch (p.zp) {
    case kZpF32: return reinterpret_cast<const float*>(p.zp_ptr)[n * p.kb + blk];
    case kZpF16: return __half2float(reinterpret_cast<const __half*>(p.zp_ptr)[n * p.kb + blk]);
    case kZpPacked: {
      const int64_t stride = (p.kb * p.bits + 7) / 8;
      const uint32_t byte = reinterpret_cast<const uint8_t*>(p.zp_ptr)[n * stride + (blk * p.bits) / 8];
      return static_cast<float>((byte >> ((blk * p.bits) % 8)) & ((1u << p.bits) - 1u));
    }
    default: return static_cast<float>(1u << (p.bits - 1));
  }
}

// (a & b) | c in one LOP3.
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// D(16x8, f32) += A(16x16, f16, row) * B(16x8, f16, col).
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 8-byte streaming load that bypasses L1 and asks L2 to fetch 256-byte lines.
__device__ __forceinline__ uint2 ldg_stream_u2(const void* ptr) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v2.u32 {%0,%1}, [%2];"
               : "=r"(v.x), "=r"(v.y)
               : "l"(ptr));
  return v;
}

}  // namespace xrgpu

namespace xrgpu {

// ------------------------------------------------------------------ mbarrier / bulk copy
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes mbarrier initialisation visible to the async proxy (bulk copies / TMA).
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity), "r"(0x989680u)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait on an mbarrier phase: gives up after `limit_ns` of device time, records
// `code` in the device error word and returns false. Never spins without bound.
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s: legitimate waits here last microseconds
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, unsigned* err, unsigned code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - start > kWaitLimitNs) {
      record_device_error(err, code);
      return false;
    }
  }
}

// 1-D bulk async copy global -> this CTA's shared memory, completing on `bar` (tx bytes).
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

}  // namespace xrgpu
