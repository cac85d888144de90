// Shared device helpers for the phantom-moe sm_100a kernels.
//
// Numeric conventions:
//  * packed int4 weights: one row of K elements is K/2 bytes; every 8
//    consecutive elements e0..e7 are one little-endian 32-bit word with
//    e_{2i} in bits [4i, 4i+4) and e_{2i+1} in bits [16+4i, 16+4i+4);
//    value = (nibble - 8) * scale[row][k / G] with fp16 scales (GGUF Q4_0
//    semantics, python/phantom/loader/gguf_loader.py:372-378, group 32 or 64).
//  * activations/router weights are bf16 or fp32; all sums are fp32.
#pragma once

#include <utility>
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

constexpr uint32_t kBf16x2One = 0x3F803F80u;  // (1.0, 1.0)

// (v & 0x000F000F) | 0x43004300: the two nibbles at bits 0-3 and 16-19 as
// bf16 (128 + n) - exact, since bf16 has 7 mantissa bits above 128.
__device__ __forceinline__ uint32_t nib_pair_biased(uint32_t v) {
  uint32_t r;
  asm("lop3.b32 %0, %1, 0x000F000F, 0x43004300, 0xEA;" : "=r"(r) : "r"(v));
  return r;
}

// One packed word (8 consecutive elements e0..e7) -> p[i] = (e_{2i}, e_{2i+1})
// as bf16x2 holding 128 + nibble: 3 shifts + 4 lop3. The caller removes the
// +136 offset (128 + the format's 8) linearly, after the MMA.
__device__ __forceinline__ void unpack_word_biased(uint32_t w, uint32_t (&p)[4]) {
  p[0] = nib_pair_biased(w);
  p[1] = nib_pair_biased(w >> 4);
  p[2] = nib_pair_biased(w >> 8);
  p[3] = nib_pair_biased(w >> 12);
}

__device__ __forceinline__ uint32_t bf16x2_sub136(uint32_t v) {
  uint32_t r;
  const uint32_t m136 = 0xC308C308u;  // (-136.0, -136.0)
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(v), "r"(kBf16x2One), "r"(m136));
  return r;
}

// As unpack_word_biased, but each pair holds (nibble - 8) exactly.
__device__ __forceinline__ void unpack_word(uint32_t w, uint32_t (&p)[4]) {
  unpack_word_biased(w, p);
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = bf16x2_sub136(p[i]);
}

// One packed word -> p[i] = (e_{2i}, e_{2i+1}) as f16x2 holding nibble - 8
// exactly. The fp16 magic 1024 (0x6400) has a 10-bit mantissa, so the
// nibbles at bits 0-3 and at bits 4-7 of each 16-bit half both land inside
// it, as 1024 + n and 1024 + 16n: one shift and four lop3 give the four
// pairs, and one fma each removes the offset ((v - 1032), (v / 16 - 72)),
// every result an exactly representable integer.
__device__ __forceinline__ void unpack_word_f16(uint32_t w, uint32_t (&p)[4]) {
  const uint32_t w8 = w >> 8;
  uint32_t a, b, c, d;
  asm("lop3.b32 %0, %1, 0x000F000F, 0x64006400, 0xEA;" : "=r"(a) : "r"(w));
  asm("lop3.b32 %0, %1, 0x00F000F0, 0x64006400, 0xEA;" : "=r"(b) : "r"(w));
  asm("lop3.b32 %0, %1, 0x000F000F, 0x64006400, 0xEA;" : "=r"(c) : "r"(w8));
  asm("lop3.b32 %0, %1, 0x00F000F0, 0x64006400, 0xEA;" : "=r"(d) : "r"(w8));
  const uint32_t one = 0x3C003C00u, m1032 = 0xE408E408u;       // 1.0, -1032.0
  const uint32_t sixteenth = 0x2C002C00u, m72 = 0xD480D480u;   // 1/16, -72.0
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(p[0]) : "r"(a), "r"(one), "r"(m1032));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(p[1]) : "r"(b), "r"(sixteenth), "r"(m72));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(p[2]) : "r"(c), "r"(one), "r"(m1032));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(p[3]) : "r"(d), "r"(sixteenth), "r"(m72));
}

// D = A * B + C, m16n8k16, fp16 inputs, fp32 accumulate (register operands).
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                              const float (&c)[4]) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1),
        "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

// Programmatic dependent launch (the decode chain: router, dispatch, expert
// FFN, combine). A kernel launched with launch_pdl may be scheduled while the
// previous kernel of its stream still runs; its first statement waits for
// that kernel to finish (all blocks done, memory visible) before any global
// access, then lets the next kernel be scheduled. Both instructions are
// no-ops for an ordinary launch.
__device__ __forceinline__ void pdl_begin() {
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// D = A * B + C, m16n8k16, bf16 inputs, fp32 accumulate (register operands).
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1, const float (&c)[4]) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1),
        "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

__device__ __forceinline__ float silu_f32(float g) { return g / (1.0f + expf(-g)); }

}  // namespace phmoe
