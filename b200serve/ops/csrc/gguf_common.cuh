// Shared device helpers of the GGUF block-quantised kernels (gguf_gemm.cu, gguf_gemv.cu):
// the m16n8k16 bf16 tensor-core MMA and the in-register dequantisation of the fragment-ordered
// codes (4-bit with a scale and min per 32, 8-bit with a scale per 16/32, E8 vector codes with a
// scale and offset per group).
#pragma once
#include "common.cuh"

namespace b200 {

__device__ __forceinline__ void qmma(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t bf2_sub(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bf2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

// 4-bit codes: word w holds register i's pair in nibbles (i) and (i + 4) -> bits 4i..4i+3 and 16+4i..
__device__ __forceinline__ void dequant_u4(uint32_t w, uint32_t sa, uint32_t ma, uint32_t sb, uint32_t mb,
                                           uint32_t* a) {
  const uint32_t bias = 0x43004300u;  // bf16 (128, 128)
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t q = ((w >> (4 * i)) & 0x000F000Fu) | bias;   // (128 + q_lo, 128 + q_hi)
    const uint32_t qv = bf2_sub(q, bias);
    const bool row_b = (i & 1);                                  // a1, a3: row g + 8
    a[i] = bf2_fma(qv, row_b ? sb : sa, row_b ? mb : ma);         // q * s + (-m)
  }
}

// 8-bit signed codes: two words, register i's pair = bytes (2i, 2i+1) as int8
__device__ __forceinline__ void dequant_s8(uint32_t w0, uint32_t w1, uint32_t sa, uint32_t sb, uint32_t* a) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t w = i < 2 ? w0 : w1;
    const int sh = (i & 1) * 16;
    const float lo = (float)(int8_t)((w >> sh) & 0xFF), hi = (float)(int8_t)((w >> (sh + 8)) & 0xFF);
    const uint32_t qv = pack_bf16x2(lo, hi);
    const bool row_b = (i & 1);
    a[i] = bf2_fma(qv, row_b ? sb : sa, 0u);
  }
}

// Explicit shared-memory reads (32-bit addresses) for the table lookups of the E8 and IQ4 paths.
__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint2 lds_u64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

}  // namespace b200
