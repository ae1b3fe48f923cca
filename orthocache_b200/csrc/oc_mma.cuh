// Warp-level bfloat16 tensor-core helpers (ldmatrix + mma.sync m16n8k16)
// shared by the decode attention kernels.  Inline PTX for sm_100a.
#pragma once

#include <stdint.h>

namespace oc {

// D += A B, A 16x16 row-major (4 registers), B 16x8 column-major (2
// registers), bfloat16 inputs, float32 accumulators.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Byte offset of (token t, 16-byte chunk of channels c8) in a swizzled tile of
// CH rows stored as D/64 boxes of 128-byte rows.
template <int CH>
__device__ __forceinline__ uint32_t swz(int t, int c8) {
  return (uint32_t)((c8 >> 3) * (CH * 128) + t * 128 + (((c8 & 7) ^ (t & 7)) << 4));
}

}  // namespace oc
