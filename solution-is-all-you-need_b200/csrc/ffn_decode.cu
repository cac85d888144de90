// Grouped SwiGLU expert FFN, decode form (few tokens per expert).
//
// Reference: Qwen3MoeExperts.forward loop body (transformers 5.5.0
// models/qwen3_moe/modeling_qwen3_moe.py:245-247):
//   gate, up = linear(x_e, gate_up_proj[e]).chunk(2); h = silu(gate) * up;
//   y_e = linear(h, down_proj[e])
// on weights dequantised as (nibble - 8) * scale (gguf_loader.py:372-378).
//
// Design. At decode sizes the layer streams ~2.5 MB of packed weights per
// expert hit and does only a few FMAs per weight, so the bound is HBM. Each
// packed weight is loaded once from HBM (8-byte coalesced loads: the four
// lanes of a quad read one 32-byte group of a row), turned into bf16
// (nibble - 8) values in registers, and fed directly as the A operand of
// mma.sync m16n8k16 - the dequantised weights never touch shared memory,
// whose bandwidth would otherwise be the limit (bf16 is 4x the bytes of
// int4). Tokens are the N=8 side of the MMA. The fp16 group scale is applied
// to the fp32 partial of each group (exact factorisation), with the scales of
// the CTA's rows staged in shared memory.
//
// The K order inside a group is permuted identically for A and B (a dot
// product does not depend on the order): for G=64 lane c of a quad holds
// elements 8c..8c+7 (low nibbles) and 32+8c..32+8c+7 (high nibbles), which
// are exactly the activations it loads with two 16-byte loads.
//
// Precision: bf16 activations enter the MMA exactly; fp32 activations and
// the intermediate h are split into bf16 hi + lo parts (two MMAs), keeping
// ~16 significant bits, so the kernel tracks the fp32 reference closely.
#include "common.cuh"
#include "launch.h"

namespace phmoe {

namespace {

constexpr int kFfnWarps = 4;
constexpr int kFfnThreads = kFfnWarps * 32;

// B fragments for one group and one 8-token chunk: for each of the MMA
// sub-steps s (2 per 32-bit weight word: low then high nibbles) the two
// b registers, for the "hi" part and (fp32 input only) the "lo" part.
template <int G>
struct GroupB {
  static constexpr int kWords = G / 32;          // 32-bit weight words per lane per row
  static constexpr int kSteps = 2 * kWords;      // MMAs per group per tile
  uint32_t hi[kSteps][2];
  uint32_t lo[kSteps][2];
};

// Load activations for one group. Step order: word 0 low, word 0 high,
// word 1 low, word 1 high. For G=64: word w low covers elements 8c+4w..+3,
// high covers 32+8c+4w..+3. For G=32: low 4c..4c+3, high 16+4c..+3.
template <int G, bool kSplit>
__device__ __forceinline__ void load_b_bf16(const __nv_bfloat16* row, int g, int c, bool ok,
                                            GroupB<G>& b) {
  if constexpr (G == 64) {
    uint4 x0 = make_uint4(0, 0, 0, 0), x1 = make_uint4(0, 0, 0, 0);
    if (ok) {
      x0 = __ldg(reinterpret_cast<const uint4*>(row + g * 64 + 8 * c));
      x1 = __ldg(reinterpret_cast<const uint4*>(row + g * 64 + 32 + 8 * c));
    }
    b.hi[0][0] = x0.x; b.hi[0][1] = x0.y;  // word0 low
    b.hi[1][0] = x1.x; b.hi[1][1] = x1.y;  // word0 high
    b.hi[2][0] = x0.z; b.hi[2][1] = x0.w;  // word1 low
    b.hi[3][0] = x1.z; b.hi[3][1] = x1.w;  // word1 high
  } else {
    uint2 x0 = make_uint2(0, 0), x1 = make_uint2(0, 0);
    if (ok) {
      x0 = __ldg(reinterpret_cast<const uint2*>(row + g * 32 + 4 * c));
      x1 = __ldg(reinterpret_cast<const uint2*>(row + g * 32 + 16 + 4 * c));
    }
    b.hi[0][0] = x0.x; b.hi[0][1] = x0.y;
    b.hi[1][0] = x1.x; b.hi[1][1] = x1.y;
  }
}

__device__ __forceinline__ void split4(const float4 v, uint32_t& h0, uint32_t& h1, uint32_t& l0,
                                       uint32_t& l1) {
  split_bf16x2(v.x, v.y, h0, l0);
  split_bf16x2(v.z, v.w, h1, l1);
}

template <int G>
__device__ __forceinline__ void load_b_f32(const float* row, int g, int c, bool ok, GroupB<G>& b) {
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  if constexpr (G == 64) {
    const float4* p0 = reinterpret_cast<const float4*>(row + g * 64 + 8 * c);
    const float4* p1 = reinterpret_cast<const float4*>(row + g * 64 + 32 + 8 * c);
    const float4 a0 = ok ? __ldg(p0) : z, a1 = ok ? __ldg(p0 + 1) : z;
    const float4 c0 = ok ? __ldg(p1) : z, c1 = ok ? __ldg(p1 + 1) : z;
    split4(a0, b.hi[0][0], b.hi[0][1], b.lo[0][0], b.lo[0][1]);
    split4(c0, b.hi[1][0], b.hi[1][1], b.lo[1][0], b.lo[1][1]);
    split4(a1, b.hi[2][0], b.hi[2][1], b.lo[2][0], b.lo[2][1]);
    split4(c1, b.hi[3][0], b.hi[3][1], b.lo[3][0], b.lo[3][1]);
  } else {
    const float4 a0 = ok ? __ldg(reinterpret_cast<const float4*>(row + g * 32 + 4 * c)) : z;
    const float4 c0 = ok ? __ldg(reinterpret_cast<const float4*>(row + g * 32 + 16 + 4 * c)) : z;
    split4(a0, b.hi[0][0], b.hi[0][1], b.lo[0][0], b.lo[0][1]);
    split4(c0, b.hi[1][0], b.hi[1][1], b.lo[1][0], b.lo[1][1]);
  }
}

// Pre-split bf16 planes of h (hi and lo), same element mapping as bf16 x.
template <int G>
__device__ __forceinline__ void load_b_split_planes(const __nv_bfloat16* hi_row,
                                                    const __nv_bfloat16* lo_row, int g, int c,
                                                    bool ok, GroupB<G>& b) {
  load_b_bf16<G, false>(hi_row, g, c, ok, b);
  GroupB<G> t;
  load_b_bf16<G, false>(lo_row, g, c, ok, t);
#pragma unroll
  for (int s = 0; s < GroupB<G>::kSteps; ++s) { b.lo[s][0] = t.hi[s][0]; b.lo[s][1] = t.hi[s][1]; }
}

// Raw packed words of one row for one group, for this lane.
template <int G>
struct RowWords {
  uint32_t w[G / 32];
};

template <int G>
__device__ __forceinline__ RowWords<G> load_row_words(const uint8_t* row, int g, int c) {
  RowWords<G> r;
  if constexpr (G == 64) {
    const uint2 v = ldg_nc_v2(row + g * 32 + 8 * c);
    r.w[0] = v.x; r.w[1] = v.y;
  } else {
    r.w[0] = ldg_nc_u32(row + g * 16 + 4 * c);
  }
  return r;
}

// tmp += A(rows r, r+8; this group) * B(chunk), over all MMA steps.
template <int G, bool kTwoParts>
__device__ __forceinline__ void mma_group(float (&tmp)[4], const RowWords<G>& r0,
                                          const RowWords<G>& r8, const GroupB<G>& b) {
#pragma unroll
  for (int w = 0; w < G / 32; ++w) {
    uint32_t lo01a, lo23a, hi01a, hi23a, lo01b, lo23b, hi01b, hi23b;
    dequant_word(r0.w[w], lo01a, lo23a, hi01a, hi23a);
    dequant_word(r8.w[w], lo01b, lo23b, hi01b, hi23b);
    const uint32_t alo[4] = {lo01a, lo01b, lo23a, lo23b};
    const uint32_t ahi[4] = {hi01a, hi01b, hi23a, hi23b};
    mma_bf16_16816(tmp, alo, b.hi[2 * w][0], b.hi[2 * w][1], tmp);
    mma_bf16_16816(tmp, ahi, b.hi[2 * w + 1][0], b.hi[2 * w + 1][1], tmp);
    if constexpr (kTwoParts) {
      mma_bf16_16816(tmp, alo, b.lo[2 * w][0], b.lo[2 * w][1], tmp);
      mma_bf16_16816(tmp, ahi, b.lo[2 * w + 1][0], b.lo[2 * w + 1][1], tmp);
    }
  }
}

// ---------------------------------------------------------------------------
// gate/up + SwiGLU. Work item = (active expert, 16 intermediate rows). The 4
// warps split K (groups g = warp, warp+4, ...) and are reduced through shared
// memory in warp order (deterministic). Output: h as bf16 hi/lo planes.
// ---------------------------------------------------------------------------
template <int G, typename XT, int NCH>
__global__ void __launch_bounds__(kFfnThreads)
ffn_gateup_kernel(const XT* __restrict__ x, const int32_t* __restrict__ row_token,
                  const int32_t* __restrict__ offsets, const int32_t* __restrict__ active,
                  const uint8_t* __restrict__ w13_q, const uint16_t* __restrict__ w13_s, int H,
                  int I, __nv_bfloat16* __restrict__ h_hi, __nv_bfloat16* __restrict__ h_lo) {
  constexpr bool kTwo = std::is_same<XT, float>::value;
  constexpr int kUnroll = 4;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int NG = H / G;
  __half* sc = reinterpret_cast<__half*>(smem_raw);                     // [32][NG]
  float* red = reinterpret_cast<float*>(smem_raw + ((32 * NG * 2 + 15) & ~15));  // [3][NCH*8][32]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, c = lane & 3;
  const int tiles = I / 16;
  const int total = active[0] * tiles;
  const size_t row_bytes = (size_t)H / 2;

  for (int item = blockIdx.x; item < total; item += gridDim.x) {
    const int slot = item / tiles, tile = item - slot * tiles;
    const int e = active[1 + slot];
    const int row0 = offsets[e];
    const int n_e = offsets[e + 1] - row0;
    const int i0 = tile * 16;
    const size_t ebase = (size_t)e * 2 * I;
    __syncthreads();
    for (int idx = threadIdx.x; idx < 32 * NG; idx += kFfnThreads) {
      const int lr = idx / NG, g = idx - lr * NG;
      const int grow = lr < 16 ? i0 + lr : I + i0 + (lr - 16);
      reinterpret_cast<uint16_t*>(sc)[idx] = w13_s[(ebase + grow) * NG + g];
    }
    __syncthreads();
    const uint8_t* wg0 = w13_q + (ebase + i0 + r) * row_bytes;
    const uint8_t* wg8 = wg0 + 8 * row_bytes;
    const uint8_t* wu0 = w13_q + (ebase + I + i0 + r) * row_bytes;
    const uint8_t* wu8 = wu0 + 8 * row_bytes;

    for (int p0 = 0; p0 < n_e; p0 += 8 * NCH) {
      float acc[NCH][2][4];
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
        for (int q = 0; q < 4; ++q) { acc[ch][0][q] = 0.f; acc[ch][1][q] = 0.f; }
      const XT* xrow[NCH];
      bool xok[NCH];
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {
        const int rr = p0 + ch * 8 + r;
        xok[ch] = rr < n_e;
        xrow[ch] = x + (size_t)(xok[ch] ? row_token[row0 + rr] : 0) * H;
      }
      for (int gb = warp; gb < NG; gb += kFfnWarps * kUnroll) {
        RowWords<G> g0[kUnroll], g8[kUnroll], u0[kUnroll], u8[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int g = gb + u * kFfnWarps;
          if (g < NG) {
            g0[u] = load_row_words<G>(wg0, g, c);
            g8[u] = load_row_words<G>(wg8, g, c);
            u0[u] = load_row_words<G>(wu0, g, c);
            u8[u] = load_row_words<G>(wu8, g, c);
          }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int g = gb + u * kFfnWarps;
          if (g >= NG) break;
          const float sg0 = __half2float(sc[r * NG + g]);
          const float sg8 = __half2float(sc[(r + 8) * NG + g]);
          const float su0 = __half2float(sc[(16 + r) * NG + g]);
          const float su8 = __half2float(sc[(24 + r) * NG + g]);
#pragma unroll
          for (int ch = 0; ch < NCH; ++ch) {
            if (p0 + ch * 8 >= n_e) break;  // warp-uniform
            GroupB<G> b;
            if constexpr (kTwo) load_b_f32<G>(reinterpret_cast<const float*>(xrow[ch]), g, c, xok[ch], b);
            else load_b_bf16<G, false>(reinterpret_cast<const __nv_bfloat16*>(xrow[ch]), g, c, xok[ch], b);
            float tg[4] = {0.f, 0.f, 0.f, 0.f}, tu[4] = {0.f, 0.f, 0.f, 0.f};
            mma_group<G, kTwo>(tg, g0[u], g8[u], b);
            mma_group<G, kTwo>(tu, u0[u], u8[u], b);
            acc[ch][0][0] = fmaf(sg0, tg[0], acc[ch][0][0]);
            acc[ch][0][1] = fmaf(sg0, tg[1], acc[ch][0][1]);
            acc[ch][0][2] = fmaf(sg8, tg[2], acc[ch][0][2]);
            acc[ch][0][3] = fmaf(sg8, tg[3], acc[ch][0][3]);
            acc[ch][1][0] = fmaf(su0, tu[0], acc[ch][1][0]);
            acc[ch][1][1] = fmaf(su0, tu[1], acc[ch][1][1]);
            acc[ch][1][2] = fmaf(su8, tu[2], acc[ch][1][2]);
            acc[ch][1][3] = fmaf(su8, tu[3], acc[ch][1][3]);
          }
        }
      }
      // Cross-warp reduction in warp order 0,1,2,3.
      if (warp > 0) {
        float* dst = red + (size_t)(warp - 1) * NCH * 8 * 32;
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            dst[(ch * 8 + q) * 32 + lane] = acc[ch][0][q];
            dst[(ch * 8 + 4 + q) * 32 + lane] = acc[ch][1][q];
          }
      }
      __syncthreads();
      if (warp == 0) {
#pragma unroll
        for (int w = 0; w < kFfnWarps - 1; ++w) {
          const float* src = red + (size_t)w * NCH * 8 * 32;
#pragma unroll
          for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              acc[ch][0][q] += src[(ch * 8 + q) * 32 + lane];
              acc[ch][1][q] += src[(ch * 8 + 4 + q) * 32 + lane];
            }
        }
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int i = i0 + r + (q >= 2 ? 8 : 0);
            const int col = 2 * c + (q & 1);
            const int rr = p0 + ch * 8 + col;
            if (rr < n_e) {
              const float hv = silu_f32(acc[ch][0][q]) * acc[ch][1][q];
              const __nv_bfloat16 hb = __float2bfloat16_rn(hv);
              const __nv_bfloat16 lb = __float2bfloat16_rn(hv - __bfloat162float(hb));
              const size_t o = (size_t)(row0 + rr) * I + i;
              h_hi[o] = hb;
              h_lo[o] = lb;
            }
          }
        }
      }
      __syncthreads();
    }
  }
}

// ---------------------------------------------------------------------------
// down projection. Work item = (active expert, 64 output rows); warp w owns
// 16 of them and runs the whole K = I. B = h (hi + lo planes, two MMAs).
// ---------------------------------------------------------------------------
template <int G, int NCH>
__global__ void __launch_bounds__(kFfnThreads)
ffn_down_kernel(const __nv_bfloat16* __restrict__ h_hi, const __nv_bfloat16* __restrict__ h_lo,
                const int32_t* __restrict__ offsets, const int32_t* __restrict__ active,
                const uint8_t* __restrict__ w2_q, const uint16_t* __restrict__ w2_s, int H, int I,
                float* __restrict__ y) {
  constexpr int kUnroll = 4;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int NG = I / G;
  __half* sc = reinterpret_cast<__half*>(smem_raw);  // [64][NG]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, c = lane & 3;
  const int tiles = H / 64;
  const int total = active[0] * tiles;
  const size_t row_bytes = (size_t)I / 2;

  for (int item = blockIdx.x; item < total; item += gridDim.x) {
    const int slot = item / tiles, tile = item - slot * tiles;
    const int e = active[1 + slot];
    const int row0 = offsets[e];
    const int n_e = offsets[e + 1] - row0;
    const size_t ebase = (size_t)e * H + tile * 64;
    __syncthreads();
    for (int idx = threadIdx.x; idx < 64 * NG; idx += kFfnThreads)
      reinterpret_cast<uint16_t*>(sc)[idx] = w2_s[ebase * NG + idx];
    __syncthreads();
    const int lr0 = warp * 16 + r;
    const uint8_t* w0 = w2_q + (ebase + lr0) * row_bytes;
    const uint8_t* w8 = w0 + 8 * row_bytes;

    for (int p0 = 0; p0 < n_e; p0 += 8 * NCH) {
      float acc[NCH][4];
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[ch][q] = 0.f;
      for (int gb = 0; gb < NG; gb += kUnroll) {
        RowWords<G> a0[kUnroll], a8[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int g = gb + u;
          if (g < NG) {
            a0[u] = load_row_words<G>(w0, g, c);
            a8[u] = load_row_words<G>(w8, g, c);
          }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int g = gb + u;
          if (g >= NG) break;
          const float s0 = __half2float(sc[lr0 * NG + g]);
          const float s8 = __half2float(sc[(lr0 + 8) * NG + g]);
#pragma unroll
          for (int ch = 0; ch < NCH; ++ch) {
            if (p0 + ch * 8 >= n_e) break;
            const int rr = p0 + ch * 8 + r;
            const bool ok = rr < n_e;
            const size_t hoff = (size_t)(row0 + (ok ? rr : 0)) * I;
            GroupB<G> b;
            load_b_split_planes<G>(h_hi + hoff, h_lo + hoff, g, c, ok, b);
            float t[4] = {0.f, 0.f, 0.f, 0.f};
            mma_group<G, true>(t, a0[u], a8[u], b);
            acc[ch][0] = fmaf(s0, t[0], acc[ch][0]);
            acc[ch][1] = fmaf(s0, t[1], acc[ch][1]);
            acc[ch][2] = fmaf(s8, t[2], acc[ch][2]);
            acc[ch][3] = fmaf(s8, t[3], acc[ch][3]);
          }
        }
      }
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int hrow = tile * 64 + lr0 + (q >= 2 ? 8 : 0);
          const int rr = p0 + ch * 8 + 2 * c + (q & 1);
          if (rr < n_e) y[(size_t)(row0 + rr) * H + hrow] = acc[ch][q];
        }
      }
    }
  }
}

template <int G, typename XT, int NCH>
void launch_gateup(const void* x, const int32_t* row_token, const int32_t* offsets,
                   const int32_t* active, const uint8_t* w13_q, const uint16_t* w13_s, int H,
                   int I, __nv_bfloat16* h_hi, __nv_bfloat16* h_lo, int grid, cudaStream_t st) {
  const int NG = H / G;
  const size_t smem = ((32 * NG * 2 + 15) & ~15) + (size_t)3 * NCH * 8 * 32 * sizeof(float);
  auto kern = ffn_gateup_kernel<G, XT, NCH>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  kern<<<grid, kFfnThreads, smem, st>>>(static_cast<const XT*>(x), row_token, offsets, active,
                                         w13_q, w13_s, H, I, h_hi, h_lo);
}

template <int G, int NCH>
void launch_down(const __nv_bfloat16* h_hi, const __nv_bfloat16* h_lo, const int32_t* offsets,
                 const int32_t* active, const uint8_t* w2_q, const uint16_t* w2_s, int H, int I,
                 float* y, int grid, cudaStream_t st) {
  const size_t smem = (size_t)64 * (I / G) * 2;
  auto kern = ffn_down_kernel<G, NCH>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  kern<<<grid, kFfnThreads, smem, st>>>(h_hi, h_lo, offsets, active, w2_q, w2_s, H, I, y);
}

template <int G, int NCH>
void launch_all(const void* x, int x_dtype, const int32_t* row_token, const int32_t* offsets,
                const int32_t* active, const uint8_t* w13_q, const uint16_t* w13_s,
                const uint8_t* w2_q, const uint16_t* w2_s, int H, int I, int max_active,
                __nv_bfloat16* h_hi, __nv_bfloat16* h_lo, float* y, cudaStream_t st,
                cudaEvent_t mid_event) {
  const int sms = device_sm_count();
  const int cap = sms * 8;
  const int g1 = std::max(1, std::min(max_active * (I / 16), cap));
  const int g2 = std::max(1, std::min(max_active * (H / 64), cap));
  if (x_dtype == PHMOE_DTYPE_BF16)
    launch_gateup<G, __nv_bfloat16, NCH>(x, row_token, offsets, active, w13_q, w13_s, H, I, h_hi, h_lo, g1, st);
  else
    launch_gateup<G, float, NCH>(x, row_token, offsets, active, w13_q, w13_s, H, I, h_hi, h_lo, g1, st);
  if (mid_event) cudaEventRecord(mid_event, st);
  launch_down<G, NCH>(h_hi, h_lo, offsets, active, w2_q, w2_s, H, I, y, g2, st);
  note_launches(2);
}

}  // namespace

int launch_ffn_decode(const void* x, int x_dtype, const int32_t* row_token,
                      const int32_t* offsets, const int32_t* active, const uint8_t* w13_q,
                      const uint16_t* w13_s, const uint8_t* w2_q, const uint16_t* w2_s, int T,
                      int H, int E, int top_k, int I, int G, float* h, float* y,
                      cudaStream_t st, cudaEvent_t mid_event) {
  const long long R = (long long)T * top_k;
  if (R == 0) return PHMOE_OK;
  const int max_active = (int)std::min<long long>(E, R);
  __nv_bfloat16* h_hi = reinterpret_cast<__nv_bfloat16*>(h);
  __nv_bfloat16* h_lo = h_hi + (size_t)R * I;
  const long long mean = (R + E - 1) / E;
  const int nch = mean <= 2 ? 1 : (mean <= 6 ? 2 : 4);
#define PHMOE_FFN_CASE(GG, NN)                                                                 \
  if (G == GG && nch == NN) {                                                                  \
    launch_all<GG, NN>(x, x_dtype, row_token, offsets, active, w13_q, w13_s, w2_q, w2_s, H, I, \
                       max_active, h_hi, h_lo, y, st, mid_event);                              \
    return PHMOE_OK;                                                                           \
  }
  PHMOE_FFN_CASE(64, 1)
  PHMOE_FFN_CASE(64, 2)
  PHMOE_FFN_CASE(64, 4)
  PHMOE_FFN_CASE(32, 1)
  PHMOE_FFN_CASE(32, 2)
  PHMOE_FFN_CASE(32, 4)
#undef PHMOE_FFN_CASE
  return PHMOE_ERR_UNSUPPORTED;
}

}  // namespace phmoe
