// Symmetric int4 group quantiser (load-time utility).
//
// The reference has no quantiser: it reads GGUF files already quantised by
// llama.cpp and dequantises them (python/phantom/loader/gguf_loader.py:362-381).
// This kernel produces the packed layout the FFN kernels read:
//   scale = fp16_rn(absmax(group) / 7)          (IEEE fp32 division)
//   q     = clamp(rint(w / scale), -8, 7) + 8   (0 when scale == 0)
//   every 8 consecutive elements e0..e7 form one little-endian 32-bit word:
//   bytes (e0|e2<<4, e4|e6<<4, e1|e3<<4, e5|e7<<4)
// One warp per (row, group); every operation is IEEE-rounded so the CPU
// restatement reproduces the bytes exactly.
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
  constexpr int kPer = G / 32;  // elements per lane: lane, lane+32
  float v[kPer];
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    v[i] = load_w<WT>(src + lane + 32 * i);
    m = fmaxf(m, fabsf(v[i]));
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  const __half sh = __float2half_rn(__fdiv_rn(m, 7.0f));
  const float s = __half2float(sh);
  uint8_t* dst = packed + row * (K / 2) + (long long)g * (G / 2);
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
  if (lane == 0) scales[row * ng + g] = __half_as_ushort(sh);
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

}  // namespace phmoe
