// Shared device helpers for the phantom-moe sm_100a kernels.
//
// Numeric conventions:
//  * packed int4 weights: one row of K elements is K/2 bytes; group g of G
//    elements (G = 32 or 64) is bytes [g*G/2, (g+1)*G/2); byte j of a group
//    holds element j in its low nibble and element j + G/2 in its high
//    nibble (GGUF Q4_0 block order, python/phantom/loader/gguf_loader.py:372-378);
//    value = (nibble - 8) * scale[row][g] with fp16 scales.
//  * activations/router weights are bf16 or fp32; all sums are fp32.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>
#include <type_traits>

#include "../../include/phmoe.h"

namespace phmoe {

constexpr int kWarp = 32;

__device__ __forceinline__ float bf16_lo_to_f32(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi_to_f32(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// Round-to-nearest-even fp32 pair -> packed bf16x2 (lo in bits 0..15).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Split fp32 pairs into a bf16 'hi' pair and the bf16 residual 'lo' pair, so
// that hi + lo carries ~16 significant bits of each value.
__device__ __forceinline__ void split_bf16x2(float a, float b, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf16x2(a, b);
  float ra = a - bf16_lo_to_f32(hi);
  float rb = b - bf16_hi_to_f32(hi);
  lo = pack_bf16x2(ra, rb);
}

// Dequantise the low/high nibbles of bytes b0,b1 (t = [b0,0,b1,0] after
// byte_perm) into bf16x2 holding (nibble - 8). 0x4300 | n is bf16 128 + n
// exactly; subtracting 136 is exact.
__device__ __forceinline__ uint32_t nib_lo_pair(uint32_t t) {
  uint32_t r;
  asm("lop3.b32 %0, %1, 0x000F000F, 0x43004300, 0xEA;" : "=r"(r) : "r"(t));
  return r;
}
__device__ __forceinline__ uint32_t nib_hi_pair(uint32_t t) {
  uint32_t r;
  asm("{\n\t.reg .b32 s;\n\tshr.u32 s, %1, 4;\n\t"
      "lop3.b32 %0, s, 0x000F000F, 0x43004300, 0xEA;\n\t}"
      : "=r"(r) : "r"(t));
  return r;
}
__device__ __forceinline__ uint32_t bf16x2_sub136(uint32_t v) {
  uint32_t r;
  const uint32_t one = 0x3F803F80u;     // (1.0, 1.0)
  const uint32_t m136 = 0xC308C308u;    // (-136.0, -136.0)
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(v), "r"(one), "r"(m136));
  return r;
}

// One 32-bit word of packed weights (bytes b0..b3) -> four bf16x2 registers:
//   lo01 = (e[b0.lo], e[b1.lo]), lo23 = (e[b2.lo], e[b3.lo]),
//   hi01 = (e[b0.hi], e[b1.hi]), hi23 = (e[b2.hi], e[b3.hi]).
__device__ __forceinline__ void dequant_word(uint32_t w, uint32_t& lo01, uint32_t& lo23,
                                             uint32_t& hi01, uint32_t& hi23) {
  uint32_t t01 = __byte_perm(w, 0u, 0x4140);
  uint32_t t23 = __byte_perm(w, 0u, 0x4342);
  lo01 = bf16x2_sub136(nib_lo_pair(t01));
  lo23 = bf16x2_sub136(nib_lo_pair(t23));
  hi01 = bf16x2_sub136(nib_hi_pair(t01));
  hi23 = bf16x2_sub136(nib_hi_pair(t23));
}

// D = A * B + C, m16n8k16, bf16 inputs, fp32 accumulate (register operands).
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1, const float (&c)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1),
        "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

__device__ __forceinline__ uint2 ldg_nc_v2(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
               : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t ldg_nc_u32(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}

__device__ __forceinline__ float silu_f32(float g) { return g / (1.0f + expf(-g)); }

}  // namespace phmoe
