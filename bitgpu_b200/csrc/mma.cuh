// Warp-level tensor-core helpers shared by the decode kernels (sm_100a): ldmatrix, the
// m16n8k16 f16 MMA with f32 accumulation, movmatrix, f16 packing, the exact int8 -> f16 code
// conversion and the 128-byte swizzle address of a TMA-written tile.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace bg {

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

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_f16(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}

constexpr uint32_t kSelLo = 0x4140, kSelHi = 0x4342, kSelEven = 0x4240, kSelOdd = 0x4341;

// Biased form without the subtraction: (code + 1152) as exact f16x2, from a word already xored
// with 0x80808080.  The kernels remove the +1152 inside the MMA instead (accumulator seed for K,
// an extra MMA with a constant -1152 operand for V).
__device__ __forceinline__ uint32_t i8pair_biased(uint32_t wx, uint32_t sel) {
  return __byte_perm(wx, 0x64646464u, sel);
}
__device__ __forceinline__ uint32_t kNeg1152x2() {
  __half2 h = __half2(__float2half_rn(-1152.f), __float2half_rn(-1152.f));
  return *reinterpret_cast<uint32_t *>(&h);
}

// Shared-memory byte address of 16-byte chunk `gc` of tile row `row` (128B-swizzled column blocks
// of TP rows each, the layout TMA writes with CU_TENSOR_MAP_SWIZZLE_128B).
template <int TP>
__device__ __forceinline__ uint32_t swz(uint32_t base, int row, int gc) {
  return base + (gc >> 3) * (TP * 128) + row * 128 + (((gc & 7) ^ (row & 7)) << 4);
}

}  // namespace bg
