// Load-time weight utilities: the symmetric int4 group quantiser and the
// GGUF importers (Q4_0 lossless, Q4_K re-quantised).
//
// The reference has no quantiser: it reads GGUF files already quantised by
// llama.cpp and dequantises them (python/phantom/loader/gguf_loader.py:362-381).
// The quantiser produces the packed layout the FFN kernels read:
//   scale = fp16_rn(absmax(group) / 7)          (IEEE fp32 division)
//   q     = clamp(rint(w / scale), -8, 7) + 8   (0 when scale == 0)
//   every 8 consecutive elements e0..e7 form one little-endian 32-bit word:
//   bytes (e0|e2<<4, e4|e6<<4, e1|e3<<4, e5|e7<<4)
// One warp per (row, group); every operation is IEEE-rounded so the CPU
// restatement reproduces the bytes exactly.
//
// GGUF Q4_0 (llama.cpp block_q4_0, 18 bytes per 32 elements: fp16 d, then 16
// bytes whose low nibbles are elements 0-15 and high nibbles 16-31; value
// (q - 8) * d; gguf_loader.py:588-596) is the packed layout's group-32 case
// with the nibbles in another order: the importer only moves nibbles and
// copies d, so it is lossless.
//
// GGUF Q4_K (block_q4_K, 144 bytes per 256 elements: fp16 d, fp16 dmin, 12
// bytes of 6-bit sub-block scales and mins, 128 bytes of nibbles; value
// d*sc_j*q - dmin*m_j for sub-block j of 32 elements, chunk c of 32 bytes
// holding sub-block 2c in its low and 2c+1 in its high nibbles;
// gguf_loader.py:648-666, the path the loader runs at gguf_loader.py:799) is
// asymmetric, so the importer dequantises each element in fp32 exactly as the
// reference does (d*sc and dmin*m rounded to fp32, then one multiply and one
// subtract) and re-quantises the result with the symmetric rule above.
#include "common.cuh"
#include "launch.h"

namespace phmoe {

namespace {

template <typename WT>
__device__ __forceinline__ float load_w(const WT* p);
template <>
__device__ __forceinline__ float load_w<float>(const float* p) { return __ldg(p); }
template <>
__device__ __forceinline__ float load_w<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

__device__ __forceinline__ int quant_one(float w, float s) {
  if (!(s > 0.f)) return 8;
  float q = rintf(__fdiv_rn(w, s));
  q = fminf(fmaxf(q, -8.f), 7.f);
  return (int)q + 8;
}

// Quantise one group held as v[i] = element lane + 32 i of the group (one
// warp) and write its packed bytes and fp16 scale.
template <int G>
__device__ __forceinline__ void quantize_group(const float (&v)[G / 32], int lane, uint8_t* __restrict__ dst,
                                               uint16_t* __restrict__ sdst) {
  constexpr int kPer = G / 32;  // elements per lane: lane, lane+32
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < kPer; ++i) m = fmaxf(m, fabsf(v[i]));
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  const __half sh = __float2half_rn(__fdiv_rn(m, 7.0f));
  const float s = __half2float(sh);
  // Lane holds the nibbles of elements lane and (G=64) lane+32. Byte b of
  // the group belongs to 8-element word m = b/4; its low nibble is element
  // 8m + 4(b&1) + ((b&3)>>1) and its high nibble that element + 2.
  const int q0 = quant_one(v[0], s);
  const int q1 = kPer > 1 ? quant_one(v[kPer - 1], s) : 8;
  const int wm = lane >> 2, p = lane & 3;
  const int elo = 8 * wm + 4 * (p & 1) + (p >> 1), ehi = elo + 2;
  const int lo_a = __shfl_sync(0xffffffffu, q0, elo & 31), lo_b = __shfl_sync(0xffffffffu, q1, elo & 31);
  const int hi_a = __shfl_sync(0xffffffffu, q0, ehi & 31), hi_b = __shfl_sync(0xffffffffu, q1, ehi & 31);
  const int qlo = elo < 32 ? lo_a : lo_b;
  const int qhi = ehi < 32 ? hi_a : hi_b;
  if (lane < G / 2) dst[lane] = (uint8_t)(qlo | (qhi << 4));
  if (lane == 0) *sdst = __half_as_ushort(sh);
}

template <typename WT, int G>
__global__ void __launch_bounds__(256)
quantize_kernel(const WT* __restrict__ w, long long rows, int K, uint8_t* __restrict__ packed,
                uint16_t* __restrict__ scales) {
  const int lane = threadIdx.x & 31;
  const long long gid = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int ng = K / G;
  if (gid >= rows * ng) return;
  const long long row = gid / ng;
  const int g = (int)(gid - row * ng);
  const WT* src = w + row * K + (long long)g * G;
  float v[G / 32];
#pragma unroll
  for (int i = 0; i < G / 32; ++i) v[i] = load_w<WT>(src + lane + 32 * i);
  quantize_group<G>(v, lane, packed + row * (K / 2) + (long long)g * (G / 2), scales + row * ng + g);
}

__device__ __forceinline__ float f16_bits_to_f32(uint16_t b) { return __half2float(__ushort_as_half(b)); }

// One thread per Q4_0 block: 16 nibble bytes -> four packed words (element j
// of the block is byte j & 15, low nibble for j < 16, high for j >= 16).
__global__ void __launch_bounds__(256)
gguf_q4_0_kernel(const uint8_t* __restrict__ blocks, long long nblk, uint8_t* __restrict__ packed,
                 uint16_t* __restrict__ scales) {
  const long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nblk) return;
  const uint16_t* src = reinterpret_cast<const uint16_t*>(blocks + b * 18);  // 18-byte blocks: 2-byte aligned
  uint32_t qs[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) qs[i] = (uint32_t)__ldg(src + 1 + 2 * i) | ((uint32_t)__ldg(src + 2 + 2 * i) << 16);
  auto nib = [&](int j) -> uint32_t {  // nibble of block element j
    const int byte = j & 15;
    const uint32_t v = (qs[byte >> 2] >> (8 * (byte & 3))) & 0xFFu;
    return j < 16 ? (v & 0xFu) : (v >> 4);
  };
  uint4 out;
  uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
  for (int m = 0; m < 4; ++m) {  // word m: elements 8m..8m+7, e_{2i} at bit 4i, e_{2i+1} at bit 16+4i
    uint32_t w = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) w |= (nib(8 * m + 2 * i) << (4 * i)) | (nib(8 * m + 2 * i + 1) << (16 + 4 * i));
    o[m] = w;
  }
  reinterpret_cast<uint4*>(packed)[b] = out;
  scales[b] = __ldg(src);
}

// Element e (0..255) of a Q4_K super-block in fp32, as the reference computes
// it: sub-block j = e / 32 reads byte 32 * (j / 2) + e % 32, low nibble for
// even j; value = fp32(d * sc_j) * q - fp32(dmin * m_j).
__device__ __forceinline__ float q4_k_element(const uint8_t* __restrict__ sb, int e) {
  const float d = f16_bits_to_f32((uint16_t)sb[0] | ((uint16_t)sb[1] << 8));
  const float dmin = f16_bits_to_f32((uint16_t)sb[2] | ((uint16_t)sb[3] << 8));
  const uint8_t* sc = sb + 4;
  const int j = e >> 5;
  int s, m;
  if (j < 4) {
    s = sc[j] & 0x3F;
    m = sc[j + 4] & 0x3F;
  } else {
    s = (sc[j + 4] & 0x0F) | ((sc[j - 4] >> 6) << 4);
    m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
  }
  const uint8_t byte = sb[16 + 32 * (j >> 1) + (e & 31)];
  const int q = (j & 1) ? (byte >> 4) : (byte & 0x0F);
  return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)s), (float)q), __fmul_rn(dmin, (float)m));
}

// One warp per (row, output group): dequantise the group's elements from the
// row's Q4_K super-blocks, then quantise them like quantize_kernel.
template <int G>
__global__ void __launch_bounds__(256)
gguf_q4_k_kernel(const uint8_t* __restrict__ blocks, long long rows, int K, uint8_t* __restrict__ packed,
                 uint16_t* __restrict__ scales) {
  const int lane = threadIdx.x & 31;
  const long long gid = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int ng = K / G;
  if (gid >= rows * ng) return;
  const long long row = gid / ng;
  const int g = (int)(gid - row * ng);
  const uint8_t* rb = blocks + row * (long long)(K / 256) * 144;
  float v[G / 32];
#pragma unroll
  for (int i = 0; i < G / 32; ++i) {
    const int e = g * G + lane + 32 * i;  // element within the row
    v[i] = q4_k_element(rb + (long long)(e >> 8) * 144, e & 255);
  }
  quantize_group<G>(v, lane, packed + row * (K / 2) + (long long)g * (G / 2), scales + row * ng + g);
}

// Q4_K super-blocks -> fp32 (the reference's dequantised values), one thread
// per element.
__global__ void __launch_bounds__(256)
gguf_q4_k_dequant_kernel(const uint8_t* __restrict__ blocks, long long n, float* __restrict__ out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  out[i] = q4_k_element(blocks + (i >> 8) * 144, (int)(i & 255));
}

template <typename WT>
void launch_q(const void* w, long long rows, int K, int G, uint8_t* packed, uint16_t* scales,
              cudaStream_t st) {
  const long long groups = rows * (K / G);
  const long long blocks = (groups + 7) / 8;
  if (G == 64)
    quantize_kernel<WT, 64><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const WT*>(w), rows, K, packed, scales);
  else
    quantize_kernel<WT, 32><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const WT*>(w), rows, K, packed, scales);
}

}  // namespace

int launch_quantize(const void* w, int w_dtype, long long rows, int K, int G, uint8_t* packed,
                    uint16_t* scales, cudaStream_t st) {
  if (rows == 0) return PHMOE_OK;
  if (w_dtype == PHMOE_DTYPE_BF16) launch_q<__nv_bfloat16>(w, rows, K, G, packed, scales, st);
  else launch_q<float>(w, rows, K, G, packed, scales, st);
  note_launches(1);
  return PHMOE_OK;
}

int launch_gguf_q4_0(const void* blocks, long long rows, int K, uint8_t* packed, uint16_t* scales, cudaStream_t st) {
  const long long nblk = rows * (K / 32);
  if (nblk == 0) return PHMOE_OK;
  gguf_q4_0_kernel<<<(unsigned)((nblk + 255) / 256), 256, 0, st>>>(static_cast<const uint8_t*>(blocks), nblk,
                                                                    packed, scales);
  note_launches(1);
  return PHMOE_OK;
}

int launch_gguf_q4_k(const void* blocks, long long rows, int K, int G, uint8_t* packed, uint16_t* scales,
                     cudaStream_t st) {
  const long long groups = rows * (K / G);
  if (groups == 0) return PHMOE_OK;
  const unsigned grid = (unsigned)((groups + 7) / 8);
  const uint8_t* b = static_cast<const uint8_t*>(blocks);
  if (G == 64) gguf_q4_k_kernel<64><<<grid, 256, 0, st>>>(b, rows, K, packed, scales);
  else gguf_q4_k_kernel<32><<<grid, 256, 0, st>>>(b, rows, K, packed, scales);
  note_launches(1);
  return PHMOE_OK;
}

int launch_gguf_q4_k_dequant(const void* blocks, long long n, float* out, cudaStream_t st) {
  if (n == 0) return PHMOE_OK;
  gguf_q4_k_dequant_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(static_cast<const uint8_t*>(blocks), n, out);
  note_launches(1);
  return PHMOE_OK;
}

}  // namespace phmoe
