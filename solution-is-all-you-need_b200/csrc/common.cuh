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
// The two halves of pdl_begin, for a kernel that starts work which does not
// depend on the previous kernel before it waits. Every kernel of the chain
// waits before it triggers, so a kernel scheduled early may already read
// what the kernels before its predecessor wrote: its predecessor's blocks
// triggered only after those had finished.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

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

// launch_pdl with a thread-block cluster of `cluster` CTAs (grid dimensions
// must be multiples of it).
template <typename... KArgs, typename... Args>
inline void launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, dim3 cluster, size_t smem,
                               cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster.x;
  attr[1].val.clusterDim.y = cluster.y;
  attr[1].val.clusterDim.z = cluster.z;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
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
// SiLU from the hardware exp2 approximation and a fast reciprocal (a few
// ulp; the decode FFN's h is then held to 2^-13 of its group maximum, far
// coarser). For g below ~-88, e^-g is infinite and the result is -0.
__device__ __forceinline__ float silu_fast(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// ---------------------------------------------------------------------------
// Integer tensor-core path of the decode FFN
// ---------------------------------------------------------------------------
// D = A * B + C, m16n8k32, A unsigned 8-bit (int4 nibbles 0..15), B signed
// 8-bit (the hi and lo bytes of fx rows), exact int32 accumulation.
__device__ __forceinline__ void mma_u8s8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// First step of a chain: D = A * B + C with C = (c0, c1, c0, c1) given as
// plain inputs (the constants of the pass's two token columns, or zeros),
// so no register copies are needed to seed the accumulators.
__device__ __forceinline__ void mma_u8s8_16832_first(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                                     int c0, int c1) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%10,%11};\n"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c0), "r"(c1));
}
// One packed word (elements e0..e7, packed layout above) as two registers of
// unsigned bytes: lo = (e0, e4, e1, e5), hi = (e2, e6, e3, e7). One AND and
// one shift + AND: the whole int4 -> int8 unpack of 8 weights.
__device__ __forceinline__ void nib_bytes(uint32_t w, uint32_t& lo, uint32_t& hi) {
  lo = w & 0x0F0F0F0Fu;
  hi = (w >> 4) & 0x0F0F0F0Fu;
}

// Fixed-point rows ("fx rows"): the decode FFN's activations (x) and SwiGLU
// output (h) as exact integers for the int8 tensor cores.
//  * Per row and group of G elements: an exponent e with A = rint(v * 2^-e)
//    and |A| <= kFxAmax(G) (8191 for G = 64, 16383 for G = 32; the largest
//    element of the group lands in the top two binades, so every element is
//    held to 2^-13 of the group's maximum or better).
//  * A = 256 * hi + lo with hi = (A + 128) >> 8 and lo = A - 256 * hi, both
//    signed bytes (lo in [-128, 127]; its byte is A & 255), so both planes
//    enter the MMAs as s8 (one MMA type). Each 8-element word of a row is 16
//    bytes: 8 hi bytes then 8 lo bytes, each in element order
//    (0, 4, 1, 5, 2, 6, 3, 7) - the order nib_bytes gives the weight bytes,
//    so one load per word yields matching B fragments.
//  * Per row and group, two int32 constants {C0, M}: M = the bits of the
//    float 1.5 * 2^(23 + e) and C0 = M - 8 * sum(A). For int4 nibbles n the
//    group's dot product sum((n - 8) * A) = v is exact in int32 and, since
//    |v| < 2^22, the int32 M + v read as a float is 1.5 * 2^(23 + e) + v * 2^e
//    exactly: float(M + v) - float(M) = v * 2^e with no conversion
//    instruction (I2F runs on a quarter-rate pipe).
// The dot product of one group is then: i_lo = C0 + sum(n * lo) and i_hi =
// sum(n * hi) by the tensor cores (u8 x s8), i = 256 * i_hi + i_lo (one IMAD), and
// __int_as_float(i) - __int_as_float(M) = v * 2^e.
constexpr int kFxMagic = 0x4B400000;  // float 1.5 * 2^23
constexpr int kFxMinExp = -126;       // 2^-e stays a normal float (and M + v one too)
constexpr int kFxMaxExp = 100;        // keeps M + v below 2^31
template <int G>
struct FxLimits {
  static constexpr int kAmax = G == 64 ? 8191 : 16383;  // G * 8 * kAmax < 2^22
  static constexpr int kShift = G == 64 ? 12 : 13;
  static constexpr float kLim = G == 64 ? 8191.5f : 16383.5f;
};

// floor(log2(m)) for a finite m > 0 (normal or subnormal).
__device__ __forceinline__ int ilog2_f32(float m) {
  const int b = __float_as_int(m);
  const int ex = (b >> 23) & 255;
  return ex ? ex - 127 : -149 + (31 - __clz(b));
}

// 2^-e as a float, for e in [kFxMinExp, kFxMaxExp] (a normal power of two,
// so multiplying by it is exact unless the product underflows).
__device__ __forceinline__ float fx_pow2_neg(int e) { return __int_as_float((127 - e) << 23); }

// The exponent of a group whose largest |value| is m. `bad` is set when the
// group cannot be held (m beyond 2^(kFxMaxExp + 13), infinite or NaN): its
// values are then clamped. Groups below 2^(kFxMinExp + 12) take kFxMinExp.
template <int G>
__device__ __forceinline__ int fx_exponent(float m, bool& bad) {
  bad = !(m <= 3.0e38f);  // NaN or infinite
  if (bad) return kFxMaxExp;
  if (m == 0.0f) return 0;
  int e = ilog2_f32(m) - FxLimits<G>::kShift;
  if (e < kFxMinExp) return kFxMinExp;
  if (e >= kFxMaxExp) {
    if (e > kFxMaxExp || m * fx_pow2_neg(e) >= FxLimits<G>::kLim) bad = true;
    return kFxMaxExp;
  }
  if (m * fx_pow2_neg(e) >= FxLimits<G>::kLim) ++e;
  return e;
}

template <int G>
__device__ __forceinline__ int fx_encode(float v, int e) {
  int a = __float2int_rn(v * fx_pow2_neg(e));
  return max(-FxLimits<G>::kAmax, min(FxLimits<G>::kAmax, a));
}

__device__ __forceinline__ int fx_magic(int e) { return kFxMagic + e * (1 << 23); }

// Byte slot of element p (0..7) inside its word's 8-byte plane.
__device__ __forceinline__ int fx_slot(int p) { return (p & 3) * 2 + (p >> 2); }

// The 16 bytes of one word from its 8 integers A[0..7].
__device__ __forceinline__ uint4 fx_word(const int (&a)[8]) {
  auto hb = [&](int i) { return (uint32_t)(((a[i] + 128) >> 8) & 255); };
  auto lb = [&](int i) { return (uint32_t)(a[i] & 255); };
  uint4 r;
  r.x = hb(0) | (hb(4) << 8) | (hb(1) << 16) | (hb(5) << 24);
  r.y = hb(2) | (hb(6) << 8) | (hb(3) << 16) | (hb(7) << 24);
  r.z = lb(0) | (lb(4) << 8) | (lb(1) << 16) | (lb(5) << 24);
  r.w = lb(2) | (lb(6) << 8) | (lb(3) << 16) | (lb(7) << 24);
  return r;
}

}  // namespace phmoe
