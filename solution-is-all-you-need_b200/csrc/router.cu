// Fused MoE router: logits GEMV (fixed fp32 reduction order), fp32 softmax
// with a bit-reproducible exp, warp-shuffle top-k (ties -> lower expert
// index) and renormalisation.
//
// Reference semantics: Qwen3MoeTopKRouter.forward (transformers 5.5.0
// models/qwen3_moe/modeling_qwen3_moe.py:263-272): linear -> softmax(fp32) ->
// topk -> divide by the sum of the picked values; PhantomTopKRouter.forward
// (tests/test_moe_routing.py:56-72) computes the same weights as
// softmax over the k largest logits.
//
// Every fp32 operation below is an explicitly rounded __fmul_rn/__fadd_rn/
// __fdiv_rn so that the CPU restatement can replay it bit for bit:
//   logit(t,e): element h goes to lane (h/8)%32; each lane adds its products
//   in increasing h; lanes are combined by an xor butterfly 16,8,4,2,1.
//   softmax: expert e on lane e%32, lane sums in increasing e, xor butterfly.
#include <cooperative_groups.h>

#include "common.cuh"
#include "launch.h"

namespace cg = cooperative_groups;

namespace phmoe {

// Error bit the fused router raises (read by phmoe_device_error): 2 when a
// value of x could not be held by the decode FFN's fixed-point rows (about
// 1e34 or beyond, infinite or NaN) and was clamped.
__device__ int g_router_error;

namespace {

__device__ __forceinline__ void fx_flag_bad() { atomicOr(&g_router_error, 2); }

constexpr int kRouterWarps = 8;     // experts per CTA (one warp each)
constexpr int kRouterTokens = 8;    // tokens per CTA
constexpr int kBlockRouterMinTokens = 256;  // from here the register-blocked kernel is used
constexpr size_t kMaxTileBytes = 232448;    // dynamic shared memory per CTA

// One lane's 8 router-weight elements in their stored form: a batch of
// loads is kept in flight unconverted, and converted one chunk at a time.
template <typename T>
struct RawW8;
template <>
struct RawW8<__nv_bfloat16> {
  uint4 u;
  __device__ __forceinline__ void load(const __nv_bfloat16* p, bool ok) {
    u = ok ? __ldg(reinterpret_cast<const uint4*>(p)) : make_uint4(0, 0, 0, 0);
  }
  __device__ __forceinline__ void to_f32(float (&v)[8]) const {
    v[0] = bf16_lo_to_f32(u.x); v[1] = bf16_hi_to_f32(u.x);
    v[2] = bf16_lo_to_f32(u.y); v[3] = bf16_hi_to_f32(u.y);
    v[4] = bf16_lo_to_f32(u.z); v[5] = bf16_hi_to_f32(u.z);
    v[6] = bf16_lo_to_f32(u.w); v[7] = bf16_hi_to_f32(u.w);
  }
};
template <>
struct RawW8<float> {
  float4 a, b;
  __device__ __forceinline__ void load(const float* p, bool ok) {
    a = ok ? __ldg(reinterpret_cast<const float4*>(p)) : make_float4(0.f, 0.f, 0.f, 0.f);
    b = ok ? __ldg(reinterpret_cast<const float4*>(p) + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __device__ __forceinline__ void to_f32(float (&v)[8]) const {
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
};
template <typename WT>
constexpr int kWBatch = std::is_same<WT, float>::value ? 4 : 8;  // 16-byte chunk loads in flight per lane

// acc + x*w as one rounded operation sequence matching the CPU replay
// (rounded product, then rounded add). When both operands are bf16 the fp32
// product is exact (8 x 8 significant bits), so a fused multiply-add rounds
// identically and is used.
template <bool kExactProducts>
__device__ __forceinline__ float mul_add(float acc, float x, float w) {
  if constexpr (kExactProducts) return __fmaf_rn(x, w, acc);
  else return __fadd_rn(acc, __fmul_rn(x, w));
}

// Shared-memory layout of the fp32 token tile: per token row, per 256-element
// chunk c, the 8 elements of lane L = (h / 8) % 32 are split into two
// 16-byte halves stored at [c][half][L] so that a warp reading one half of
// its chunk reads 512 contiguous bytes (no bank conflicts).
__device__ __forceinline__ int tile_pos(int c, int half, int lane) { return c * 256 + half * 128 + lane * 4; }

// Stage the 16 bytes `u` holding elements h .. h + 16/sizeof(XT) - 1 of a row
// (h a multiple of 16/sizeof(XT)) into the row's tile as fp32 (exact).
template <typename XT>
__device__ __forceinline__ void stage_f32(float* row, int h, const uint4& u);
template <>
__device__ __forceinline__ void stage_f32<__nv_bfloat16>(float* row, int h, const uint4& u) {
  const int c = h >> 8, L = (h >> 3) & 31;
  *reinterpret_cast<float4*>(row + tile_pos(c, 0, L)) =
      make_float4(bf16_lo_to_f32(u.x), bf16_hi_to_f32(u.x), bf16_lo_to_f32(u.y), bf16_hi_to_f32(u.y));
  *reinterpret_cast<float4*>(row + tile_pos(c, 1, L)) =
      make_float4(bf16_lo_to_f32(u.z), bf16_hi_to_f32(u.z), bf16_lo_to_f32(u.w), bf16_hi_to_f32(u.w));
}
template <>
__device__ __forceinline__ void stage_f32<float>(float* row, int h, const uint4& u) {
  *reinterpret_cast<uint4*>(row + tile_pos(h >> 8, (h >> 2) & 1, (h >> 3) & 31)) = u;
}

// Stage nt rows of x (H elements each) into xs as fp32 in the tile_pos
// layout (row stride rowf). All loads of a round are issued before its
// stores, so staging costs one memory round trip per 8 vectors a thread.
template <typename XT>
__device__ __forceinline__ void stage_tile(const XT* __restrict__ x, int nt, int H, int rowf, float* xs) {
  constexpr int kVec = 16 / sizeof(XT);
  constexpr int kUnroll = 8;
  const int nvec = nt * H / kVec;  // H % 8 == 0, so rows are whole vectors
  const int vrow = H / kVec;
  const uint4* src = reinterpret_cast<const uint4*>(x);
  for (int i0 = threadIdx.x; i0 < nvec; i0 += blockDim.x * kUnroll) {
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i < nvec) v[u] = __ldg(src + i);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i < nvec) {
        const int t = i / vrow;
        stage_f32<XT>(xs + (size_t)t * rowf, (i - t * vrow) * kVec, v[u]);
      }
    }
  }
}

// The x tile of TT tokens (fp32, tile_pos layout) against one router-weight
// row: acc[t] = the fixed-order logit of token t, returned on every lane.
// Lane L owns the elements h with (h/8) % 32 == L, adds its products in
// increasing h, and the 32 lane sums are combined by an xor butterfly.
template <typename XT, typename WT, int TT>
__device__ __forceinline__ void expert_logits(const float* xs, int rowf, int nchunk, const WT* __restrict__ wrow,
                                              int H, int nt, int lane, float (&acc)[TT]) {
  constexpr bool kExact = std::is_same<XT, __nv_bfloat16>::value && std::is_same<WT, __nv_bfloat16>::value;
  constexpr int kBatch = kWBatch<WT>;
#pragma unroll
  for (int t = 0; t < TT; ++t) acc[t] = 0.f;
  for (int c0 = 0; c0 < nchunk; c0 += kBatch) {
    // a batch of loads in flight, held in stored form (converted per chunk)
    RawW8<WT> raw[kBatch];
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const int h0 = (c0 + b) * 256 + lane * 8;
      raw[b].load(wrow + h0, c0 + b < nchunk && h0 < H);
    }
    // tokens innermost: the TT accumulation chains interleave; each token
    // still adds its elements in increasing h
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      if (c0 + b < nchunk) {
        float w[1][8];
        raw[b].to_f32(w[0]);
        const bool hok = (c0 + b) * 256 + lane * 8 < H;
        const float* px = xs + tile_pos(c0 + b, 0, lane);
#pragma unroll
        for (int t = 0; t < TT; ++t) {
          if (t < nt) {
            float4 lo = make_float4(0.f, 0.f, 0.f, 0.f), hi = lo;
            if (hok) {
              lo = *reinterpret_cast<const float4*>(px + (size_t)t * rowf);
              hi = *reinterpret_cast<const float4*>(px + (size_t)t * rowf + 128);
            }
            const float xv[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
            for (int v = 0; v < 8; ++v) acc[t] = mul_add<kExact>(acc[t], xv[v], w[0][v]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < TT; ++t) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1)
      acc[t] = __fadd_rn(acc[t], __shfl_xor_sync(0xffffffffu, acc[t], off));
  }
}

// Ask L2 for a router-weight row (H elements): lane L touches every 32nd
// 128-byte line.
template <typename WT>
__device__ __forceinline__ void prefetch_row_l2(const WT* __restrict__ wrow, int H, int lane) {
  const char* p = reinterpret_cast<const char*>(wrow);
  const int bytes = H * (int)sizeof(WT);
  for (int off = lane * 128; off < bytes; off += 32 * 128)
    asm volatile("prefetch.global.L2 [%0];\n" ::"l"(p + off));
}

// Grid: (ceil(E/8), ceil(T/TT)); warp w of a CTA owns expert blockIdx.x*8+w.
// The TT-token tile of x is staged once in shared memory as fp32 (one
// cooperative round trip of 16-byte loads, converted once per CTA rather
// than once per expert); router-weight chunks are loaded kBatch at a time so
// their latencies overlap.
template <typename XT, typename WT, int TT>
__global__ void __launch_bounds__(kRouterWarps * 32)
router_logits_kernel(const XT* __restrict__ x, const WT* __restrict__ wr, int T, int H, int E,
                     float* __restrict__ logits) {
  pdl_begin();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* xs = reinterpret_cast<float*>(smem_raw);  // [TT][nchunk * 256] fp32, tile_pos layout
  const int nchunk = (H + 255) / 256;
  const int rowf = nchunk * 256;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * kRouterWarps + warp;
  const int t0 = blockIdx.y * TT;
  const int nt = min(TT, T - t0);
  stage_tile<XT>(x + (size_t)t0 * H, nt, H, rowf, xs);
  __syncthreads();
  if (e >= E) return;
  float acc[TT];
  expert_logits<XT, WT, TT>(xs, rowf, nchunk, wr + (size_t)e * H, H, nt, lane, acc);
  if (lane == 0) {
#pragma unroll
    for (int t = 0; t < TT; ++t)
      if (t < nt) logits[(size_t)(t0 + t) * E + e] = acc[t];
  }
}

// Large-batch form for bf16 x and router weight: each warp computes an
// 8-token x 8-expert block of logits in registers, reading x and the weight
// rows straight from global memory (16-byte loads, coalesced across the
// warp). Lane L still owns exactly the elements h with (h/8) % 32 == L, adds
// its exact bf16 x bf16 products in increasing h, and the 32 lane sums are
// combined by the same xor butterfly, so every logit is bit-identical to
// router_logits_kernel's. CTA: 4 token blocks x 2 expert blocks of warps.
constexpr int kBlkT = 8, kBlkE = 8, kBlkWarpsT = 4, kBlkWarpsE = 2;

__global__ void __launch_bounds__(kBlkWarpsT * kBlkWarpsE * 32)
router_logits_block_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ wr, int T,
                           int H, int E, float* __restrict__ logits) {
  pdl_begin();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = (blockIdx.y * kBlkWarpsT + warp % kBlkWarpsT) * kBlkT;
  const int e0 = (blockIdx.x * kBlkWarpsE + warp / kBlkWarpsT) * kBlkE;
  if (t0 >= T || e0 >= E) return;
  float acc[kBlkT][kBlkE];
#pragma unroll
  for (int t = 0; t < kBlkT; ++t)
#pragma unroll
    for (int e = 0; e < kBlkE; ++e) acc[t][e] = 0.f;
  const int nchunk = (H + 255) / 256;
  for (int c = 0; c < nchunk; ++c) {
    const int h0 = c * 256 + lane * 8;
    const bool hok = h0 < H;
    uint4 xv[kBlkT], wv[kBlkE];
#pragma unroll
    for (int t = 0; t < kBlkT; ++t)
      xv[t] = (hok && t0 + t < T) ? __ldg(reinterpret_cast<const uint4*>(x + (size_t)(t0 + t) * H + h0))
                                  : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int e = 0; e < kBlkE; ++e)
      wv[e] = (hok && e0 + e < E) ? __ldg(reinterpret_cast<const uint4*>(wr + (size_t)(e0 + e) * H + h0))
                                  : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int v = 0; v < 8; ++v) {  // element h0 + v, in increasing h
      float xf[kBlkT], wf[kBlkE];
#pragma unroll
      for (int t = 0; t < kBlkT; ++t) {
        const uint32_t u = (v < 2) ? xv[t].x : (v < 4) ? xv[t].y : (v < 6) ? xv[t].z : xv[t].w;
        xf[t] = (v & 1) ? bf16_hi_to_f32(u) : bf16_lo_to_f32(u);
      }
#pragma unroll
      for (int e = 0; e < kBlkE; ++e) {
        const uint32_t u = (v < 2) ? wv[e].x : (v < 4) ? wv[e].y : (v < 6) ? wv[e].z : wv[e].w;
        wf[e] = (v & 1) ? bf16_hi_to_f32(u) : bf16_lo_to_f32(u);
      }
#pragma unroll
      for (int t = 0; t < kBlkT; ++t)
#pragma unroll
        for (int e = 0; e < kBlkE; ++e) acc[t][e] = __fmaf_rn(xf[t], wf[e], acc[t][e]);
    }
  }
#pragma unroll
  for (int t = 0; t < kBlkT; ++t)
#pragma unroll
    for (int e = 0; e < kBlkE; ++e)
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1)
        acc[t][e] = __fadd_rn(acc[t][e], __shfl_xor_sync(0xffffffffu, acc[t][e], off));
  // lane (t * 8 + e) % 32 writes two of the 64 results
#pragma unroll
  for (int t = 0; t < kBlkT; ++t)
#pragma unroll
    for (int e = 0; e < kBlkE; ++e)
      if (lane == ((t * kBlkE + e) & 31) && t0 + t < T && e0 + e < E)
        logits[(size_t)(t0 + t) * E + e0 + e] = acc[t][e];
}

// exp(x) for x <= 0: Cody-Waite reduction with a two-part ln2, then the
// degree-7 Taylor polynomial of e^r in Horner form, then scaling by 2^n.
// Constants are fp32 bit patterns shared with the CPU restatement.
__device__ __forceinline__ float exp_fixed(float x) {
  const float kLog2e = __uint_as_float(0x3FB8AA3Bu);
  const float kLn2Hi = __uint_as_float(0x3F318000u);
  const float kLn2Lo = __uint_as_float(0xB95E8083u);
  const float c[8] = {__uint_as_float(0x3F800000u), __uint_as_float(0x3F800000u),
                      __uint_as_float(0x3F000000u), __uint_as_float(0x3E2AAAABu),
                      __uint_as_float(0x3D2AAAABu), __uint_as_float(0x3C088889u),
                      __uint_as_float(0x3AB60B61u), __uint_as_float(0x39500D01u)};
  const float n = rintf(__fmul_rn(x, kLog2e));
  float r = __fsub_rn(x, __fmul_rn(n, kLn2Hi));
  r = __fsub_rn(r, __fmul_rn(n, kLn2Lo));
  float p = c[7];
#pragma unroll
  for (int i = 6; i >= 0; --i) p = __fadd_rn(__fmul_rn(p, r), c[i]);
  int ni = (int)n;
  ni = ni < -126 ? -126 : (ni > 127 ? 127 : ni);
  const float two_n = __uint_as_float((uint32_t)(ni + 127) << 23);
  const float out = __fmul_rn(p, two_n);
  return x < -87.0f ? 0.0f : out;
}

// softmax (fp32, exp_fixed), top-k (ties -> lower index) and
// renormalisation of one token held by one warp: v[i] is the logit of
// expert lane + 32 i (entries at or beyond E are ignored). Writes probs (when
// non-null), topk_idx and topk_w of token t.
template <int EPL>
__device__ __forceinline__ void softmax_topk_warp(float (&v)[EPL], int lane, int t, int E, int top_k,
                                                  int renormalize, float* __restrict__ probs,
                                                  int32_t* __restrict__ topk_idx, float* __restrict__ topk_w) {
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    if (e >= E) v[i] = -INFINITY;
    m = fmaxf(m, v[i]);
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? exp_fixed(__fsub_rn(v[i], m)) : 0.f;
    s = __fadd_rn(s, v[i]);
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    if (e < E) {
      v[i] = __fdiv_rn(v[i], s);
      if (probs) probs[(size_t)t * E + e] = v[i];
    } else {
      v[i] = -1.0f;  // below every probability: never picked
    }
  }
  // k rounds of warp argmax; larger value wins, equal values -> lower index.
  uint32_t taken = 0;
  float my_val = 0.f;
  int my_idx = 0;
  float sum_sel = 0.f;
  for (int j = 0; j < top_k; ++j) {
    float bv = -2.0f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = lane + 32 * i;
      const bool free_slot = !((taken >> i) & 1u);
      if (free_slot && (v[i] > bv || (v[i] == bv && e < bi))) { bv = v[i]; bi = e; }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    sum_sel = __fadd_rn(sum_sel, bv);
    if (lane == j) { my_val = bv; my_idx = bi; }
  }
  if (lane < top_k) {
    topk_idx[(size_t)t * top_k + lane] = my_idx;
    topk_w[(size_t)t * top_k + lane] = renormalize ? __fdiv_rn(my_val, sum_sel) : my_val;
  }
}

// One warp per token. EPL = experts held per lane (E <= 32*EPL).
template <int EPL>
__global__ void __launch_bounds__(256)
router_topk_kernel(const float* __restrict__ logits, int T, int E, int top_k, int renormalize,
                   float* __restrict__ probs, int32_t* __restrict__ topk_idx,
                   float* __restrict__ topk_w) {
  pdl_begin();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + warp;
  if (t >= T) return;
  const float* lrow = logits + (size_t)t * E;
  float v[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? lrow[e] : -INFINITY;
  }
  softmax_topk_warp<EPL>(v, lane, t, E, top_k, renormalize, probs, topk_idx, topk_w);
}

// Fused router for decode batches (T < 256, E <= 256): logits, softmax,
// top-k and, optionally, the fixed-point encoding of x for the decode FFN, in
// one launch. A cluster of 8 CTAs shares a tile of TT tokens: CTA q stages
// the tile as fp32 and computes the logits of experts q*EC .. q*EC+EC-1
// (EC = ceil(E/8), warp w taking experts w, w+8, ... of them) with the same
// fixed reduction order as router_logits_kernel; the logits go to global
// memory and to the CTA's shared memory. CTA q also encodes the groups
// g = q, q+8, ... of every token of the tile (fx rows, as fx_rows_kernel).
// After a cluster barrier, token t of the tile is taken by warp t/8 of CTA
// t%8, which reads all E logits through distributed shared memory and runs
// softmax_topk_warp. A second cluster barrier keeps every CTA's shared
// memory alive until all reads are done. No CTA leaves before either
// barrier, so the barriers always complete.
constexpr int kFusedCluster = 8;
constexpr int kFusedWarps = 16;  // one expert per warp for E <= 128
constexpr int kTopkScratch = 8 + 8 + 256 + 32 + 32 + 4;  // words of shared memory for softmax_topk_group

// Softmax and top-k of one token by the nw = ceil(E/32) warps wl = 0..nw-1
// of a group (named barrier bar_id), one expert per lane (e = 32 wl + lane),
// with results bit-identical to softmax_topk_warp<8>:
//  * the maximum and exp_fixed(v - max) as there;
//  * the sum in the same order: "lane" L adds e = L, L+32, ... (L + 224) to
//    0, then the xor butterfly 16..1 (run by warp 0 over the exps in shared
//    memory; terms with e >= E are 0 there and change nothing);
//  * the same division; and instead of k rounds of warp argmax, the rank of
//    each probability among all E (larger first, equal -> lower index), the
//    order in which those rounds pick. A NaN is never picked; when fewer
//    than k values can be (non-finite logits), the remaining picks are the
//    padding slots e = E, E+1, ... < 256 with value -1, then (0x7fffffff,
//    -2), exactly as the rounds would make them. The selected values are
//    summed in pick order.
__device__ void softmax_topk_group(float v, int wl, int nw, int lane, int bar_id, int t, int E, int top_k,
                                   int renormalize, float* __restrict__ probs, int32_t* __restrict__ topk_idx,
                                   float* __restrict__ topk_w, float* scr) {
  float* wmax = scr;                                  // [8]
  int* wnan = reinterpret_cast<int*>(scr + 8);         // [8]
  float* ps = scr + 16;                               // [256]
  float* selv = ps + 256;                             // [32]
  int* seli = reinterpret_cast<int*>(selv + 32);      // [32]
  float* ssum = reinterpret_cast<float*>(seli + 32);  // [2]
  const int nthreads = nw * 32;
  const int e = wl * 32 + lane;
  auto gsync = [&]() { asm volatile("bar.sync %0, %1;\n" ::"r"(bar_id), "r"(nthreads) : "memory"); };
  if (e >= E) v = -INFINITY;
  float m = v;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if (lane == 0) wmax[wl] = m;
  gsync();
  m = wmax[0];
  for (int i = 1; i < nw; ++i) m = fmaxf(m, wmax[i]);
  const float pe = e < E ? exp_fixed(__fsub_rn(v, m)) : 0.f;
  ps[e] = pe;
  gsync();
  if (wl == 0) {
    float sm = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int ee = lane + 32 * i;
      if (ee < E) sm = __fadd_rn(sm, ps[ee]);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) sm = __fadd_rn(sm, __shfl_xor_sync(0xffffffffu, sm, off));
    if (lane == 0) ssum[0] = sm;
  }
  gsync();  // also: warp 0 has read every exp before ps is overwritten below
  const float s = ssum[0];
  float q = -1.0f;
  if (e < E) {
    q = __fdiv_rn(pe, s);
    if (probs) probs[(size_t)t * E + e] = q;
  }
  ps[e] = q;
  const bool is_nan = e < E && q != q;
  const unsigned nb = __ballot_sync(0xffffffffu, is_nan);
  if (lane == 0) wnan[wl] = __popc(nb);
  gsync();
  if (e < E && !is_nan) {
    int rank = 0;
    const int E4 = E & ~3;
    for (int j = 0; j < E4; j += 4) {
      const float4 o = *reinterpret_cast<const float4*>(ps + j);
      rank += (o.x > q || (o.x == q && j < e)) + (o.y > q || (o.y == q && j + 1 < e)) +
              (o.z > q || (o.z == q && j + 2 < e)) + (o.w > q || (o.w == q && j + 3 < e));
    }
    for (int j = E4; j < E; ++j) rank += (ps[j] > q || (ps[j] == q && j < e));
    if (rank < top_k) {
      selv[rank] = q;
      seli[rank] = e;
    }
  }
  gsync();
  if (wl == 0 && lane == 0) {
    int valid = E;
    for (int i = 0; i < nw; ++i) valid -= wnan[i];
    for (int r = valid; r < top_k; ++r) {
      const int ep = E + (r - valid);
      selv[r] = ep < 256 ? -1.0f : -2.0f;
      seli[r] = ep < 256 ? ep : 0x7fffffff;
    }
    float ss = 0.f;
    for (int r = 0; r < top_k; ++r) ss = __fadd_rn(ss, selv[r]);
    ssum[1] = ss;
  }
  gsync();
  if (e < top_k) {
    topk_idx[(size_t)t * top_k + e] = seli[e];
    topk_w[(size_t)t * top_k + e] = renormalize ? __fdiv_rn(selv[e], ssum[1]) : selv[e];
  }
}

// The dispatch of a one-token batch from its picks (softmax_topk_group's
// scratch, after it returns), with launch_dispatch's results: row r of the
// k valid picks is the r-th smallest expert id (one token: rows in expert
// order), offsets[e] = the valid picks below e, active = the picked experts
// ascending, row_token = 0, inv = the pick's row (-1 for an id outside
// [0, E), which launch_dispatch drops too). The picks are distinct experts.
__device__ void dispatch_one_token(const float* scr, int wl, int nw, int lane, int E, int top_k,
                                   const DispatchOut& disp) {
  const int* seli = reinterpret_cast<const int*>(scr + 16 + 256 + 32);
  const int tid = wl * 32 + lane;
  for (int e = tid; e <= E; e += nw * 32) {
    int c = 0;
    for (int j = 0; j < top_k; ++j) c += (unsigned)seli[j] < (unsigned)E && seli[j] < e;
    disp.offsets[e] = c;
  }
  if (tid < top_k) {
    const int ej = seli[tid];
    const bool ok = (unsigned)ej < (unsigned)E;
    int rank = 0;
    for (int j = 0; j < top_k; ++j) rank += (unsigned)seli[j] < (unsigned)E && seli[j] < ej;
    disp.inv[tid] = ok ? rank : -1;
    if (ok) {
      disp.row_token[rank] = 0;
      disp.active[1 + rank] = ej;
    }
  }
  if (tid == 0) {
    int nv = 0;
    for (int j = 0; j < top_k; ++j) nv += (unsigned)seli[j] < (unsigned)E;
    disp.active[0] = nv;
  }
}

template <int G>
__device__ __forceinline__ void encode_tile_groups(const float* xs, int rowf, int nt, int H, int q, int t0,
                                                   uint8_t* __restrict__ xq, int2* __restrict__ xc) {
  constexpr int kTpg = G / 8;                  // threads per group (one word each)
  constexpr int kGroupsPerRound = kFusedWarps * 32 / kTpg;
  const int NG = H / G;
  const int ngc = (NG + kFusedCluster - 1) / kFusedCluster;  // groups of a token handled by this CTA
  const int units = nt * ngc;
  for (int u0 = 0; u0 < units; u0 += kGroupsPerRound) {
    const int u = u0 + (int)threadIdx.x / kTpg;
    const int t = u / ngc;
    const int g = q + kFusedCluster * (u - t * ngc);
    const bool ok = u < units && g < NG;
    const int w = (ok ? g : 0) * kTpg + (int)(threadIdx.x % kTpg);  // word index in the row
    float v[8];
    if (ok) {
      const int h = w * 8, c = h >> 8, L = (h >> 3) & 31;
      const float4 lo = *reinterpret_cast<const float4*>(xs + (size_t)t * rowf + tile_pos(c, 0, L));
      const float4 hi = *reinterpret_cast<const float4*>(xs + (size_t)t * rowf + tile_pos(c, 1, L));
      v[0] = lo.x; v[1] = lo.y; v[2] = lo.z; v[3] = lo.w; v[4] = hi.x; v[5] = hi.y; v[6] = hi.z; v[7] = hi.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = 0.f;
    }
    float m = 0.f;
    bool nonfinite = false;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float a = fabsf(v[j]);
      nonfinite |= !(a <= 3.0e38f);
      m = fmaxf(m, a);
    }
#pragma unroll
    for (int off = 1; off < kTpg; off <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    bool bad;
    const int e = fx_exponent<G>(m, bad);
    int a[8];
    int s = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      a[j] = fx_encode<G>(v[j], e);
      s += a[j];
    }
#pragma unroll
    for (int off = 1; off < kTpg; off <<= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (ok) {
      const size_t row = (size_t)(t0 + t);
      *reinterpret_cast<uint4*>(xq + (row * (H / 8) + w) * 16) = fx_word(a);
      if ((threadIdx.x % kTpg) == 0) {
        const int M = fx_magic(e);
        xc[row * NG + g] = make_int2(M - 8 * s, M);
      }
      if (bad || nonfinite) fx_flag_bad();
    }
  }
}

template <typename XT, typename WT, int TT>
__global__ void __launch_bounds__(kFusedWarps * 32, 2)  // two CTAs per SM: a 32-cluster batch fits one wave
router_fused_kernel(const XT* __restrict__ x, const WT* __restrict__ wr, int T, int H, int E, int top_k,
                    int renormalize, float* __restrict__ logits, float* __restrict__ probs,
                    int32_t* __restrict__ topk_idx, float* __restrict__ topk_w, int G, uint8_t* __restrict__ xq,
                    int2* __restrict__ xc, DispatchOut disp) {
  cg::cluster_group cluster = cg::this_cluster();
  const int q = (int)cluster.block_rank();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int nchunk = (H + 255) / 256;
  const int rowf = nchunk * 256;
  const int EC = (E + kFusedCluster - 1) / kFusedCluster;
  float* xs = reinterpret_cast<float*>(smem_raw);  // [TT][rowf]
  float* lg = xs + (size_t)TT * rowf;              // [TT][EC] this CTA's logits
  float* scr = lg + ((size_t)TT * EC + 3) / 4 * 4;  // [kTopkScratch] top-k scratch
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.y * TT;
  const int nt = min(TT, T - t0);
  // The router weights are constant: each warp asks L2 for its experts'
  // rows before waiting for the previous kernel, so the fetch from HBM
  // overlaps that kernel's tail and the staging of x.
  for (int el = warp; el < EC && q * EC + el < E; el += kFusedWarps)
    prefetch_row_l2<WT>(wr + (size_t)(q * EC + el) * H, H, lane);
  pdl_wait();
  pdl_trigger();
  stage_tile<XT>(x + (size_t)t0 * H, nt, H, rowf, xs);
  __syncthreads();
  for (int el = warp; el < EC; el += kFusedWarps) {
    const int e = q * EC + el;
    if (e >= E) break;
    float acc[TT];
    expert_logits<XT, WT, TT>(xs, rowf, nchunk, wr + (size_t)e * H, H, nt, lane, acc);
    if (lane == 0) {
#pragma unroll
      for (int t = 0; t < TT; ++t) {
        if (t < nt) {
          logits[(size_t)(t0 + t) * E + e] = acc[t];
          lg[t * EC + el] = acc[t];
        }
      }
    }
  }
  if (xq != nullptr) {
    if (G == 64) encode_tile_groups<64>(xs, rowf, nt, H, q, t0, xq, xc);
    else encode_tile_groups<32>(xs, rowf, nt, H, q, t0, xq, xc);
  }
  cluster.sync();
  // token t of the tile: CTA t % 8, warps 0 .. ceil(E/32)-1 (TT <= 8: one
  // token per CTA), every logit read through distributed shared memory
  {
    const int nw = (E + 31) / 32;
    const int t = q;
    if (t < nt && warp < nw) {
      const int e = warp * 32 + lane;
      float v = -INFINITY;
      if (e < E) {
        const float* remote = cluster.map_shared_rank(lg, e / EC);
        v = remote[t * EC + e % EC];
      }
      softmax_topk_group(v, warp, nw, lane, 1, t0 + t, E, top_k, renormalize, probs, topk_idx, topk_w, scr);
      if (disp.offsets != nullptr && T == 1) dispatch_one_token(scr, warp, nw, lane, E, top_k, disp);
    }
  }
  cluster.sync();
}

// sigmoid(x) from exp_fixed (so the CPU restatement replays it bit for bit).
__device__ __forceinline__ float sigmoid_fixed(float x) {
  if (x >= 0.0f) return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_fixed(-x)));
  const float e = exp_fixed(x);
  return __fdiv_rn(e, __fadd_rn(1.0f, e));
}

// DeepSeek-V3 routing (transformers 5.5.0 models/deepseek_v3/modeling_deepseek_v3.py
// DeepseekV3MoE.route_tokens_to_experts): s = sigmoid(logit); choice c = s +
// bias[e]; the E experts form n_group groups of E/n_group, a group scores
// the sum of its two largest c, the topk_group best groups stay and the
// others' c become 0; the top_k largest c are picked and weighted by their
// s, renormalised by (sum + 1e-20) when asked, times `scale`. Ties -> lower
// index (groups and experts). One warp per token.
template <int EPL>
__global__ void __launch_bounds__(256)
router_topk_grouped_kernel(const float* __restrict__ logits, const float* __restrict__ bias, int T, int E,
                           int top_k, int n_group, int topk_group, int renormalize, float scale,
                           int32_t* __restrict__ topk_idx, float* __restrict__ topk_w) {
  pdl_begin();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + warp;
  if (t >= T) return;
  const float* lrow = logits + (size_t)t * E;
  float sc[EPL], c[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    if (e < E) {
      sc[i] = sigmoid_fixed(lrow[e]);
      c[i] = bias ? __fadd_rn(sc[i], bias[e]) : sc[i];
    } else {
      sc[i] = 0.f;
      c[i] = -INFINITY;
    }
  }
  if (n_group > 1) {
    const int gs = E / n_group;
    float mine = -INFINITY;  // lane g: score of group g
    for (int g = 0; g < n_group; ++g) {
      float a = -INFINITY, b = -INFINITY;  // two largest c of this lane's members of group g
#pragma unroll
      for (int i = 0; i < EPL; ++i) {
        const int e = lane + 32 * i;
        if (e < E && e / gs == g) {
          if (c[i] > a) { b = a; a = c[i]; } else if (c[i] > b) { b = c[i]; }
        }
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, a, off), ob = __shfl_xor_sync(0xffffffffu, b, off);
        const float na = fmaxf(a, oa);
        b = fmaxf(fminf(a, oa), fmaxf(b, ob));
        a = na;
      }
      if (lane == g) mine = __fadd_rn(a, b);
    }
    uint32_t keep = 0;
    for (int r = 0; r < topk_group; ++r) {
      float bv = (lane < n_group && !((keep >> lane) & 1u)) ? mine : -INFINITY;
      int bi = (lane < n_group && !((keep >> lane) & 1u)) ? lane : 0x7fffffff;
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      keep |= 1u << bi;
    }
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = lane + 32 * i;
      if (e < E && !((keep >> (e / gs)) & 1u)) c[i] = 0.0f;  // masked_fill(~mask, 0.0)
    }
  }
  uint32_t taken = 0;
  float my_val = 0.f, sum_sel = 0.f;
  int my_idx = 0;
  for (int j = 0; j < top_k; ++j) {
    float bv = -INFINITY, bs = 0.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = lane + 32 * i;
      if (e < E && !((taken >> i) & 1u) && (c[i] > bv || (c[i] == bv && e < bi))) { bv = c[i]; bi = e; bs = sc[i]; }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      const float os = __shfl_xor_sync(0xffffffffu, bs, off);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; bs = os; }
    }
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    sum_sel = __fadd_rn(sum_sel, bs);
    if (lane == j) { my_val = bs; my_idx = bi; }
  }
  if (lane < top_k) {
    const float w = renormalize ? __fdiv_rn(my_val, __fadd_rn(sum_sel, 1e-20f)) : my_val;
    topk_idx[(size_t)t * top_k + lane] = my_idx;
    topk_w[(size_t)t * top_k + lane] = __fmul_rn(w, scale);
  }
}

template <typename XT, typename WT, int TT>
void launch_logits_tt(const void* x, const void* wr, int T, int H, int E, float* logits,
                      cudaStream_t st) {
  const size_t smem = (size_t)TT * ((H + 255) / 256 * 256) * sizeof(float);
  auto kern = router_logits_kernel<XT, WT, TT>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((E + kRouterWarps - 1) / kRouterWarps, (T + TT - 1) / TT);
  launch_pdl(kern, dim3(grid), dim3(kRouterWarps * 32), smem, st, static_cast<const XT*>(x), static_cast<const WT*>(wr),
                                              T, H, E, logits);
}

// Token tile: 8 rows for small batches; 32 rows (4x fewer router-weight
// re-reads from L2) for large ones when the tile fits in shared memory.
template <typename XT, typename WT>
void launch_logits(const void* x, const void* wr, int T, int H, int E, float* logits,
                   cudaStream_t st) {
  const size_t row = (size_t)((H + 255) / 256 * 256) * sizeof(float);
  // CTAs for a token tile of tt rows; small batches take smaller tiles so
  // that there are at least two CTAs per SM to hide the accumulation chains
  const long long eblk = (E + kRouterWarps - 1) / kRouterWarps, want = 2LL * device_sm_count();
  auto ctas = [&](int tt) { return eblk * ((T + tt - 1) / tt); };
  if (kRouterTokens * row > kMaxTileBytes)  // very wide layers: 4-token tiles
    launch_logits_tt<XT, WT, 4>(x, wr, T, H, E, logits, st);
  else if (T >= 256 && 32 * row <= 160 * 1024)
    launch_logits_tt<XT, WT, 32>(x, wr, T, H, E, logits, st);
  else if (ctas(kRouterTokens) >= want || T <= 1)
    launch_logits_tt<XT, WT, kRouterTokens>(x, wr, T, H, E, logits, st);
  else if (ctas(4) >= want)
    launch_logits_tt<XT, WT, 4>(x, wr, T, H, E, logits, st);
  else
    launch_logits_tt<XT, WT, 2>(x, wr, T, H, E, logits, st);
}

}  // namespace

namespace {
void launch_router_logits(const void* x, int x_dtype, const void* wr, int w_dtype, int T, int H, int E, float* logits,
                          cudaStream_t st) {
  if (x_dtype == PHMOE_DTYPE_BF16 && w_dtype == PHMOE_DTYPE_BF16 && T >= kBlockRouterMinTokens) {
    dim3 grid((E + kBlkE * kBlkWarpsE - 1) / (kBlkE * kBlkWarpsE), (T + kBlkT * kBlkWarpsT - 1) / (kBlkT * kBlkWarpsT));
    launch_pdl(router_logits_block_kernel, dim3(grid), dim3(kBlkWarpsT * kBlkWarpsE * 32), 0, st, 
        static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(wr), T, H, E, logits);
  } else if (x_dtype == PHMOE_DTYPE_BF16 && w_dtype == PHMOE_DTYPE_BF16)
    launch_logits<__nv_bfloat16, __nv_bfloat16>(x, wr, T, H, E, logits, st);
  else if (x_dtype == PHMOE_DTYPE_BF16 && w_dtype == PHMOE_DTYPE_F32)
    launch_logits<__nv_bfloat16, float>(x, wr, T, H, E, logits, st);
  else if (x_dtype == PHMOE_DTYPE_F32 && w_dtype == PHMOE_DTYPE_BF16)
    launch_logits<float, __nv_bfloat16>(x, wr, T, H, E, logits, st);
  else
    launch_logits<float, float>(x, wr, T, H, E, logits, st);
}
}  // namespace

int launch_router_grouped(const void* x, int x_dtype, const void* wr, int w_dtype, int T, int H, int E, int top_k,
                          int renormalize, const float* bias, int n_group, int topk_group, float scale,
                          float* logits, int32_t* topk_idx, float* topk_w, cudaStream_t st) {
  if (T == 0) return PHMOE_OK;
  if (E > 1024) return PHMOE_ERR_UNSUPPORTED;
  launch_router_logits(x, x_dtype, wr, w_dtype, T, H, E, logits, st);
  const int grid = (T + 7) / 8;
  if (E <= 128)
    launch_pdl(router_topk_grouped_kernel<4>, dim3(grid), dim3(256), 0, st, logits, bias, T, E, top_k, n_group, topk_group, renormalize,
                                                        scale, topk_idx, topk_w);
  else if (E <= 256)
    launch_pdl(router_topk_grouped_kernel<8>, dim3(grid), dim3(256), 0, st, logits, bias, T, E, top_k, n_group, topk_group, renormalize,
                                                        scale, topk_idx, topk_w);
  else
    launch_pdl(router_topk_grouped_kernel<32>, dim3(grid), dim3(256), 0, st, logits, bias, T, E, top_k, n_group, topk_group, renormalize,
                                                         scale, topk_idx, topk_w);
  note_launches(2);
  return PHMOE_OK;
}

namespace {
template <typename XT, typename WT, int TT>
void launch_fused_tt(const void* x, const void* wr, int T, int H, int E, int top_k, int renormalize, float* logits,
                     float* probs, int32_t* topk_idx, float* topk_w, int G, uint8_t* xq, int2* xc,
                     const DispatchOut& disp, cudaStream_t st) {
  const int EC = (E + kFusedCluster - 1) / kFusedCluster;
  const size_t smem =
      ((size_t)TT * ((H + 255) / 256 * 256) + ((size_t)TT * EC + 3) / 4 * 4 + kTopkScratch) * sizeof(float);
  static_assert(TT <= kFusedCluster, "one token per CTA in the top-k step");
  auto kern = router_fused_kernel<XT, WT, TT>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  launch_pdl_cluster(kern, dim3(kFusedCluster, (T + TT - 1) / TT), dim3(kFusedWarps * 32), dim3(kFusedCluster, 1, 1),
                     smem, st, static_cast<const XT*>(x), static_cast<const WT*>(wr), T, H, E, top_k, renormalize,
                     logits, probs, topk_idx, topk_w, G, xq, xc, disp);
}

template <typename XT, typename WT>
void launch_fused(const void* x, const void* wr, int T, int H, int E, int top_k, int renormalize, float* logits,
                  float* probs, int32_t* topk_idx, float* topk_w, int G, uint8_t* xq, int2* xc,
                  const DispatchOut& disp, cudaStream_t st) {
  // token tiles: at least ~one CTA per SM where the batch allows
  if (T <= 16)
    launch_fused_tt<XT, WT, 1>(x, wr, T, H, E, top_k, renormalize, logits, probs, topk_idx, topk_w, G, xq, xc, disp,
                               st);
  else if (T <= 128)
    launch_fused_tt<XT, WT, 2>(x, wr, T, H, E, top_k, renormalize, logits, probs, topk_idx, topk_w, G, xq, xc, disp,
                               st);
  else
    launch_fused_tt<XT, WT, 4>(x, wr, T, H, E, top_k, renormalize, logits, probs, topk_idx, topk_w, G, xq, xc, disp,
                               st);
}
}  // namespace

int router_device_error(bool reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_router_error, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_router_error, &zero, sizeof(int));
  }
  return v;
}

bool router_fused_supported(int T, int H, int E) {
  // shared memory of the largest tile (4 tokens): x tile, logits, top-k scratch
  const size_t bytes = ((size_t)4 * ((H + 255) / 256 * 256) + 4 * 32 + kTopkScratch) * 4;
  return T > 0 && T < kBlockRouterMinTokens && E <= 256 && bytes <= kMaxTileBytes;
}

int launch_router(const void* x, int x_dtype, const void* wr, int w_dtype, int T, int H, int E,
                  int top_k, int renormalize, float* logits, float* probs, int32_t* topk_idx,
                  float* topk_w, cudaStream_t st, int G, uint8_t* xq, int2* xc, const DispatchOut* disp) {
  if (T == 0) return PHMOE_OK;
  if (router_fused_supported(T, H, E)) {
    // the one-token dispatch rides along (the batch is one cluster)
    const DispatchOut d = (disp != nullptr && T == 1) ? *disp : DispatchOut{nullptr, nullptr, nullptr, nullptr};
    const bool xb = x_dtype == PHMOE_DTYPE_BF16, wb = w_dtype == PHMOE_DTYPE_BF16;
    if (xb && wb)
      launch_fused<__nv_bfloat16, __nv_bfloat16>(x, wr, T, H, E, top_k, renormalize, logits, probs, topk_idx, topk_w,
                                                 G, xq, xc, d, st);
    else if (xb)
      launch_fused<__nv_bfloat16, float>(x, wr, T, H, E, top_k, renormalize, logits, probs, topk_idx, topk_w, G, xq,
                                         xc, d, st);
    else if (wb)
      launch_fused<float, __nv_bfloat16>(x, wr, T, H, E, top_k, renormalize, logits, probs, topk_idx, topk_w, G, xq,
                                         xc, d, st);
    else
      launch_fused<float, float>(x, wr, T, H, E, top_k, renormalize, logits, probs, topk_idx, topk_w, G, xq, xc, d,
                                 st);
    note_launches(1);
    return (xq ? kRouterEncodedX : 0) | (d.offsets ? kRouterDispatched : 0);
  }
  launch_router_logits(x, x_dtype, wr, w_dtype, T, H, E, logits, st);
  const int grid = (T + 7) / 8;
  if (E <= 128)
    launch_pdl(router_topk_kernel<4>, dim3(grid), dim3(256), 0, st, logits, T, E, top_k, renormalize, probs, topk_idx, topk_w);
  else if (E <= 256)
    launch_pdl(router_topk_kernel<8>, dim3(grid), dim3(256), 0, st, logits, T, E, top_k, renormalize, probs, topk_idx, topk_w);
  else
    launch_pdl(router_topk_kernel<32>, dim3(grid), dim3(256), 0, st, logits, T, E, top_k, renormalize, probs, topk_idx, topk_w);
  note_launches(2);
  return PHMOE_OK;
}

}  // namespace phmoe
