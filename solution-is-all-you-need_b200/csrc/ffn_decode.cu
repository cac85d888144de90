// Grouped SwiGLU expert FFN, decode form (few tokens per expert).
//
// Reference: Qwen3MoeExperts.forward loop body (transformers 5.5.0
// models/qwen3_moe/modeling_qwen3_moe.py:245-247):
//   gate, up = linear(x_e, gate_up_proj[e]).chunk(2); h = silu(gate) * up;
//   y_e = linear(h, down_proj[e])
// on weights dequantised as (nibble - 8) * scale (gguf_loader.py:372-378).
//
// At decode sizes the layer streams ~2.5 MB of packed weights per expert hit
// and does a few FMAs per weight: the bound is HBM. Both kernels are
// persistent (one CTA per SM, a contiguous range of work items each) and
// stream "tasks" (a work item's K-chunk) through a ring of shared-memory
// stages; from shared memory each lane reads the int4 words of its A
// fragments and turns each 32-bit word (8 consecutive weights) into four
// bf16x2 pairs with one lop3 each (packed layout in phmoe.h); the pairs feed
// mma.sync m16n8k16 directly, with the 8 tokens of a pass as the N side.
// Dequantised weights are never written back to shared memory (bf16 would
// be 4x the int4 bytes).
//
// gate/up kernel (the larger half of the bytes): warp-specialised.
//  * item = (expert, 64 gate rows and the 64 matching up rows, pass of 8
//    tokens); task = one 512-element K chunk of an item (32 KB of weights).
//    Items are ordered (expert, row block, pass) so extra passes re-read
//    weights still in L2.
//  * A producer warp issues, per task, two TMA tensor copies of weights (a
//    64-row x 2 x 128-byte box of gate rows and one of up rows, 128-byte
//    swizzled so the fragment reads are nearly conflict free), two TMA copies
//    of the matching fp16 scale slices, and one bulk copy per activation row;
//    all complete on the stage's "full" mbarrier.
//  * Consumer warp w owns 16-row group w%4 and K quarter w/4 of every task,
//    waits on "full", computes and releases "empty" (one arrival per warp);
//    its accumulators cover the item's whole K, so the only cross-warp step
//    is a 4-way sum (fixed order) at the item's end, after which the
//    quarter-0 warp applies SwiGLU and stores h as bf16 hi/lo planes. The
//    unpacked weights are 128 + nibble: the +136 offset is removed after the
//    MMA with one extra MMA per K step against an all-ones A (it yields
//    sum_k x_k), and the fp16 group scale multiplies the fp32 partial of
//    each group.
// down kernel: 16 warps copy each task (128 rows x 512 K) with 16-byte
//  cp.async into padded rows and compute it between two CTA barriers; warp w
//  owns rows 16(w%8)..+15 and half of each K-chunk (w/8).
//
// Lane c of a quad holds K elements 16c..16c+15 of a 64-group (8c..8c+7 of a
// 32-group) for A and reads the same activations for B; inside one MMA the K
// order is a permutation applied to both operands, which a dot product does
// not see.
//
// Precision: bf16 activations enter the gate/up MMAs exactly; fp32
// activations are split into bf16 hi + lo parts (two MMAs each, ~16
// significant bits). The intermediate h goes to the down projection as fp16
// (11 significant bits; with fp32 activations as fp16 hi + lo, ~22 bits),
// against weights unpacked exactly to fp16; an |h| above the fp16 range is
// clamped to 65504 and raises bit 2 of the device error word.
//
// Every mbarrier wait is bounded: a waiting warp sleeps inside try_wait (a
// suspend-time hint, woken when the phase completes, so waiting warps take no
// issue slots from computing ones); after kWaitLimitNs of %globaltimer time
// (or kSpinLimit tries) it raises the CTA's abort flag and the device error
// word (phmoe_device_error) and all warps leave; the producer first waits
// (bounded) for its copies in flight.
#include <cuda.h>  // CUtensorMap (types only; the encoder is fetched from the driver at run time)
#include <string.h>

#include "common.cuh"
#include "pipeline.cuh"
#include "launch.h"

namespace phmoe {

// Error bits raised by the decode FFN kernels (read by phmoe_device_error;
// every writer ORs its bit in, so several conditions of one call all show):
//   1  a pipeline wait timed out and its CTA abandoned its work
//   2  a SwiGLU value was clamped to the fp16 range
__device__ int g_ffn_error;

namespace {

constexpr int kConsumers = 16;                  // gate/up consumer warps
constexpr int kGuThreads = (kConsumers + 1) * 32;  // + 1 producer warp
constexpr int kDownThreads = 16 * 32;
constexpr int kTok = 8;                         // tokens per pass (the MMA N dimension)
constexpr uint32_t kSpinLimit = 1u << 24;       // try_wait polls before giving up
constexpr uint32_t kSuspendNs = 20000;            // try_wait suspend-time hint
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ void cp_async4(uint32_t saddr, const void* g) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(saddr), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(saddr), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
// Bounded wait for copies still in flight when a producer leaves.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait_suspend(bar, parity, kSuspendNs) && global_ns() - t0 <= kWaitLimitNs) {
  }
}
// Arrive on `bar` once every cp.async this thread issued so far has landed.
__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(bar) : "memory");
}

// Bounded wait on a barrier phase. Returns false when this CTA aborts.
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait_suspend(bar, parity, kSuspendNs)) return true;
    if (*abort_flag) return false;
    if (global_ns() - t0 > kWaitLimitNs) break;
  }
  *abort_flag = 1;
  atomicOr(&g_ffn_error, 1);
  return false;
}

__device__ __forceinline__ void warp_arrive(uint32_t bar, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
}

// Control block of the row-block gate/up kernel: stage ring plus
// double-buffered reduction barriers for each of the four row groups.
template <int S>
struct RbCtl {
  uint64_t full[S];
  uint64_t empty[S];
  uint64_t red_full[8];   // [buf][rg]: the three kq > 0 warps have written
  uint64_t red_empty[8];  // [buf][rg]: the kq = 0 warp has read
  int abort_flag;
};


// ---------------------------------------------------------------------------
// fragments
// ---------------------------------------------------------------------------

// A words of one row and one group for this lane (G/32 words).
template <int G>
struct RowWords {
  uint32_t w[G / 32];
};

template <int G>
__device__ __forceinline__ RowWords<G> lds_row(const uint8_t* p) {
  RowWords<G> r;
  if constexpr (G == 64) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    r.w[0] = v.x; r.w[1] = v.y;
  } else {
    r.w[0] = *reinterpret_cast<const uint32_t*>(p);
  }
  return r;
}

// B words of one group for this lane: bf16 pairs of its G/4 elements.
template <int G>
struct BWords {
  uint32_t hi[G / 8];
  uint32_t lo[G / 8];
};

template <int G>
__device__ __forceinline__ void lds_b_plane(const uint8_t* p, uint32_t (&d)[G / 8]) {
  const uint4 a = *reinterpret_cast<const uint4*>(p);
  d[0] = a.x; d[1] = a.y; d[2] = a.z; d[3] = a.w;
  if constexpr (G == 64) {
    const uint4 b = *reinterpret_cast<const uint4*>(p + 16);
    d[4] = b.x; d[5] = b.y; d[6] = b.z; d[7] = b.w;
  }
}

__device__ __forceinline__ void split4(const float4 v, uint32_t& h0, uint32_t& h1, uint32_t& l0,
                                       uint32_t& l1) {
  split_bf16x2(v.x, v.y, h0, l0);
  split_bf16x2(v.z, v.w, h1, l1);
}

template <int G>
__device__ __forceinline__ void lds_b_f32(const uint8_t* p, BWords<G>& b) {
#pragma unroll
  for (int i = 0; i < G / 16; ++i)
    split4(reinterpret_cast<const float4*>(p)[i], b.hi[2 * i], b.hi[2 * i + 1], b.lo[2 * i], b.lo[2 * i + 1]);
}

// gate/up partial of one group: acc_g/acc_u += s * (A.B - 136 * sum(B)) for
// rows (r, r+8) of the gate and up tiles. A is unpacked biased (128 + n).
template <int G, bool kTwo>
__device__ __forceinline__ void gateup_group(const RowWords<G>& g0, const RowWords<G>& g8,
                                             const RowWords<G>& u0, const RowWords<G>& u8,
                                             const BWords<G>& b, float sg0, float sg8, float su0,
                                             float su8, float (&acc_g)[4], float (&acc_u)[4]) {
  float tg[4] = {0.f, 0.f, 0.f, 0.f}, tu[4] = {0.f, 0.f, 0.f, 0.f}, td[4] = {0.f, 0.f, 0.f, 0.f};
  const uint32_t ones[4] = {kBf16x2One, kBf16x2One, kBf16x2One, kBf16x2One};
#pragma unroll
  for (int w = 0; w < G / 32; ++w) {
    uint32_t pg0[4], pg8[4], pu0[4], pu8[4];
    unpack_word_biased(g0.w[w], pg0);
    unpack_word_biased(g8.w[w], pg8);
    unpack_word_biased(u0.w[w], pu0);
    unpack_word_biased(u8.w[w], pu8);
#pragma unroll
    for (int h = 0; h < 2; ++h) {  // two MMA steps per word
      const int s = 2 * w + h;
      const uint32_t ag[4] = {pg0[2 * h], pg8[2 * h], pg0[2 * h + 1], pg8[2 * h + 1]};
      const uint32_t au[4] = {pu0[2 * h], pu8[2 * h], pu0[2 * h + 1], pu8[2 * h + 1]};
      mma_bf16_16816(tg, ag, b.hi[2 * s], b.hi[2 * s + 1], tg);
      mma_bf16_16816(tu, au, b.hi[2 * s], b.hi[2 * s + 1], tu);
      mma_bf16_16816(td, ones, b.hi[2 * s], b.hi[2 * s + 1], td);
      if constexpr (kTwo) {
        mma_bf16_16816(tg, ag, b.lo[2 * s], b.lo[2 * s + 1], tg);
        mma_bf16_16816(tu, au, b.lo[2 * s], b.lo[2 * s + 1], tu);
        mma_bf16_16816(td, ones, b.lo[2 * s], b.lo[2 * s + 1], td);
      }
    }
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float d = -136.0f * td[q];  // td = sum of this group's activations (per token)
    const float sg = q < 2 ? sg0 : sg8, su = q < 2 ? su0 : su8;
    acc_g[q] = fmaf(sg, tg[q] + d, acc_g[q]);
    acc_u[q] = fmaf(su, tu[q] + d, acc_u[q]);
  }
}

// gateup_group for up to NB 8-token column blocks: the A fragments are
// unpacked once and reused for every block b < nb (B of block b at
// b_base + b * b_stride).
template <int G, bool kTwo, int NB>
__device__ __forceinline__ void gateup_group_mt(const RowWords<G>& g0, const RowWords<G>& g8,
                                                const RowWords<G>& u0, const RowWords<G>& u8,
                                                const uint8_t* b_base, int b_stride, int nb, float sg0, float sg8,
                                                float su0, float su8, float (&acc_g)[NB][4], float (&acc_u)[NB][4]) {
  uint32_t pg0[G / 32][4], pg8[G / 32][4], pu0[G / 32][4], pu8[G / 32][4];
#pragma unroll
  for (int w = 0; w < G / 32; ++w) {
    unpack_word_biased(g0.w[w], pg0[w]);
    unpack_word_biased(g8.w[w], pg8[w]);
    unpack_word_biased(u0.w[w], pu0[w]);
    unpack_word_biased(u8.w[w], pu8[w]);
  }
  const uint32_t ones[4] = {kBf16x2One, kBf16x2One, kBf16x2One, kBf16x2One};
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    if (b < nb) {
      BWords<G> bw;
      if constexpr (kTwo) lds_b_f32<G>(b_base + b * b_stride, bw);
      else lds_b_plane<G>(b_base + b * b_stride, bw.hi);
      float tg[4] = {0.f, 0.f, 0.f, 0.f}, tu[4] = {0.f, 0.f, 0.f, 0.f}, td[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int w = 0; w < G / 32; ++w) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int s = 2 * w + h;
          const uint32_t ag[4] = {pg0[w][2 * h], pg8[w][2 * h], pg0[w][2 * h + 1], pg8[w][2 * h + 1]};
          const uint32_t au[4] = {pu0[w][2 * h], pu8[w][2 * h], pu0[w][2 * h + 1], pu8[w][2 * h + 1]};
          mma_bf16_16816(tg, ag, bw.hi[2 * s], bw.hi[2 * s + 1], tg);
          mma_bf16_16816(tu, au, bw.hi[2 * s], bw.hi[2 * s + 1], tu);
          mma_bf16_16816(td, ones, bw.hi[2 * s], bw.hi[2 * s + 1], td);
          if constexpr (kTwo) {
            mma_bf16_16816(tg, ag, bw.lo[2 * s], bw.lo[2 * s + 1], tg);
            mma_bf16_16816(tu, au, bw.lo[2 * s], bw.lo[2 * s + 1], tu);
            mma_bf16_16816(td, ones, bw.lo[2 * s], bw.lo[2 * s + 1], td);
          }
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float d = -136.0f * td[q];
        const float sg = q < 2 ? sg0 : sg8, su = q < 2 ? su0 : su8;
        acc_g[b][q] = fmaf(sg, tg[q] + d, acc_g[b][q]);
        acc_u[b][q] = fmaf(su, tu[q] + d, acc_u[b][q]);
      }
    }
  }
}

// down partial of one group: acc += s * A.(B_hi [+ B_lo]), A unpacked exactly
// to fp16, B the fp16 h plane(s).
template <int G, bool kTwo>
__device__ __forceinline__ void down_group(const RowWords<G>& a0, const RowWords<G>& a8,
                                           const BWords<G>& b, float s0, float s8, float (&acc)[4]) {
  float t[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int w = 0; w < G / 32; ++w) {
    uint32_t p0[4], p8[4];
    unpack_word_f16(a0.w[w], p0);
    unpack_word_f16(a8.w[w], p8);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int s = 2 * w + h;
      const uint32_t a[4] = {p0[2 * h], p8[2 * h], p0[2 * h + 1], p8[2 * h + 1]};
      mma_f16_16816(t, a, b.hi[2 * s], b.hi[2 * s + 1], t);
      if constexpr (kTwo) mma_f16_16816(t, a, b.lo[2 * s], b.lo[2 * s + 1], t);
    }
  }
  acc[0] = fmaf(s0, t[0], acc[0]);
  acc[1] = fmaf(s0, t[1], acc[1]);
  acc[2] = fmaf(s8, t[2], acc[2]);
  acc[3] = fmaf(s8, t[3], acc[3]);
}

// h as the down projection reads it: fp16, clamped to the fp16 range (a
// clamp raises bit 2 of the device error word); with fp32 activations the
// rounding remainder goes to a second fp16 plane.
template <bool kTwo>
__device__ __forceinline__ void store_h(float hv, __half* __restrict__ h_hi, __half* __restrict__ h_lo, size_t o) {
  if (fabsf(hv) > 65504.0f) {
    hv = copysignf(65504.0f, hv);
    atomicOr(&g_ffn_error, 2);
  }
  const __half hb = __float2half_rn(hv);
  h_hi[o] = hb;
  if constexpr (kTwo) h_lo[o] = __float2half_rn(hv - __half2float(hb));
}

// ---------------------------------------------------------------------------
// work items
// ---------------------------------------------------------------------------

// Per active slot s: expert id, first row, row count, and the prefix
// table[s] of items before slot s (an expert with n rows has
// tiles * ceil(n / 8) items). Every CTA builds the same copy in shared memory.
struct Meta {
  int* e;
  int* row0;
  int* n;
  int* table;  // [na + 1]
};

template <int TB = kTok>  // tokens per item
__device__ int build_meta(const int32_t* __restrict__ offsets, const int32_t* __restrict__ active, int tiles,
                          Meta m) {
  const int na = active[0];
  for (int s = threadIdx.x; s < na; s += blockDim.x) {
    const int e = active[1 + s];
    const int r0 = offsets[e];
    m.e[s] = e;
    m.row0[s] = r0;
    m.n[s] = offsets[e + 1] - r0;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    int carry = 0;
    for (int s0 = 0; s0 < na; s0 += 32) {
      const int s = s0 + lane;
      const int v = s < na ? ((m.n[s] + TB - 1) / TB) * tiles : 0;
      int incl = v;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += t;
      }
      if (s < na) m.table[s + 1] = carry + incl;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) m.table[0] = 0;
  }
  __syncthreads();
  return m.table[na];
}

// Position of a CTA in its task sequence: (active slot, tile, pass, K-chunk).
// Tasks are visited in order, so a cursor only ever advances by one; no
// integer division happens in the loops (a runtime division costs several
// instructions on the SM's narrow XU pipe).
struct Cursor {
  int slot, tile, pass, kc, passes;
};

template <int TB = kTok>
__device__ __forceinline__ int passes_of(int n) { return (n + TB - 1) / TB; }

template <int TB = kTok>
__device__ Cursor cursor_at(int q, int na, int tiles, const Meta& m) {
  int lo = 0, hi = na;  // table[lo] <= q < table[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (m.table[mid] <= q) lo = mid;
    else hi = mid;
  }
  Cursor c;
  c.slot = lo;
  c.passes = passes_of<TB>(m.n[lo]);
  const int local = q - m.table[lo];
  c.tile = local / c.passes;
  c.pass = local - c.tile * c.passes;
  c.kc = 0;
  return c;
}

template <int TB = kTok>
__device__ __forceinline__ void cursor_next(Cursor& c, int tiles, int nkc, const Meta& m) {
  if (++c.kc < nkc) return;
  c.kc = 0;
  if (++c.pass < c.passes) return;
  c.pass = 0;
  if (++c.tile < tiles) return;
  c.tile = 0;
  ++c.slot;                          // may step one past the last slot: arrays hold E + 1 entries
  c.passes = passes_of<TB>(m.n[c.slot]);
}

__device__ __forceinline__ void cta_range(int total, int& q0, int& q1) {
  q0 = (int)((long long)total * blockIdx.x / gridDim.x);
  q1 = (int)((long long)total * (blockIdx.x + 1) / gridDim.x);
}

// ---------------------------------------------------------------------------
// gate/up + SwiGLU, row-block form
// ---------------------------------------------------------------------------
// Item = (expert, 64-row block of gate rows and the matching up rows, pass of
// 8 tokens); task = one 512-element K chunk of the item (32 KB of weights).
// Consumer warp w owns 16-row group rg = w % 4 and K quarter kq = w / 4 of
// every task, so its accumulators run over the whole K range of the item and
// the only cross-warp step is a 4-way sum (fixed order kq 0, 1, 2, 3) at the
// end of each item, after which the kq = 0 warp applies SwiGLU. Scales arrive
// with the weights (4-byte async copies) and are read as fp16 pairs.
constexpr int kRbRows = 64;   // gate rows per item (and as many up rows)
constexpr int kRbKc = 512;    // K elements per task

template <int G, typename XT>
struct RbCfg {
  static constexpr bool kF32 = std::is_same<XT, float>::value;
  static constexpr int kGpq = 128 / G;                       // groups per consumer warp per task
  static constexpr int kBlock = 2 * kRbRows * 128;           // one 64-row box of 2 K-chunks (16 KB)
  static constexpr int kScaleRow = kRbKc / G * 2;            // bytes of scales per row per task
  static constexpr int kPairs = kRbKc / G / 2;
  static constexpr int kBRowBytes = kRbKc * (int)sizeof(XT);
  static constexpr int kBPad = (G == 32 && !kF32) ? 64 : 16;
  static constexpr int kBStride = kBRowBytes + kBPad;
  static constexpr int kW = 0;                                // [gate box][up box]
  static constexpr int kS = 2 * kBlock;                       // [128 rows][kScaleRow]
  static constexpr int kB = kS + 2 * kRbRows * kScaleRow;     // [8 tokens][kBStride]
  static constexpr int kStage = (kB + kTok * kBStride + 1023) / 1024 * 1024;
  static constexpr int kStages = kF32 ? 3 : 4;
  static constexpr int kRed = 4 * 3 * 32 * 8 * 4;             // [rg][kq-1][lane][8] floats
  static constexpr size_t smem(int E) {
    return 1024 + (size_t)kStages * kStage + 2 * kRed + sizeof(RbCtl<kStages>) + (size_t)(4 * E + 4) * 4;
  }
};

// Byte offset of (row R of a `rows`-row box of 128-byte K-chunks, byte kb of
// the task's K slice) as TMA writes it with the 128-byte swizzle.
__device__ __forceinline__ int swz_off_rows(int R, int kb, int rows) {
  const int c0 = kb & 127;
  return ((kb >> 7) * rows + R) * 128 + ((((c0 >> 4) ^ (R & 7)) << 4) | (c0 & 15));
}

// Byte offset of (row R of a 64-row box, byte kb of the task's K slice).
__device__ __forceinline__ int swz_off64(int R, int kb) {
  const int c0 = kb & 127;
  return ((kb >> 7) * kRbRows + R) * 128 + ((((c0 >> 4) ^ (R & 7)) << 4) | (c0 & 15));
}

template <int G, typename XT>
__global__ void __launch_bounds__(kGuThreads, 1)
ffn_gateup_rb_kernel(const __grid_constant__ CUtensorMap w13_map, int map3d, int box_chunks,
                     const __grid_constant__ CUtensorMap s_map, int s_tma, const XT* __restrict__ x,
                     const int32_t* __restrict__ row_token, const int32_t* __restrict__ offsets,
                     const int32_t* __restrict__ active, const uint16_t* __restrict__ w13_s, int H, int I, int E,
                     __half* __restrict__ h_hi, __half* __restrict__ h_lo) {
  pdl_begin();
  using C = RbCfg<G, XT>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* red = reinterpret_cast<float*>(smem + S * C::kStage);  // [2][rg][kq-1][lane][8]
  RbCtl<S>* ctl = reinterpret_cast<RbCtl<S>*>(smem + S * C::kStage + 2 * C::kRed);
  int* mbase = reinterpret_cast<int*>(ctl + 1);
  const Meta meta{mbase, mbase + (E + 1), mbase + 2 * (E + 1), mbase + 3 * (E + 1)};
  volatile int* abort_flag = &ctl->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = (I + kRbRows - 1) / kRbRows;
  const int NG = H / G;
  const int nkc = (H + kRbKc - 1) / kRbKc;
  const int na = active[0];

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&ctl->full[s]), 1 + 32);  // expect_tx arrival + one cp.async arrival per lane
      mbar_init(smem_u32(&ctl->empty[s]), kConsumers);
    }
    for (int i = 0; i < 8; ++i) {
      mbar_init(smem_u32(&ctl->red_full[i]), 3);
      mbar_init(smem_u32(&ctl->red_empty[i]), 1);
    }
    ctl->abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  const int total = build_meta(offsets, active, tiles, meta);  // its barriers publish the init too
  int q0, q1;
  cta_range(total, q0, q1);
  const int ntask = (q1 - q0) * nkc;
  if (ntask == 0) return;

  if (warp == kConsumers) {
    // ---------------- producer warp ----------------
    Cursor cu = cursor_at(q0, na, tiles, meta);
    auto token = [&](const Cursor& k) -> int {  // lane holds the token id of pass row lane % 8
      const int rr = k.pass * kTok + (lane & (kTok - 1));
      return rr < meta.n[k.slot] ? __ldg(row_token + meta.row0[k.slot] + rr) : -1;
    };
    int tok = token(cu);
    int issued = 0;
    for (int t = 0; t < ntask; ++t) {
      const int s = t % S;
      if (t >= S && !wait_phase(smem_u32(&ctl->empty[s]), (t / S - 1) & 1, abort_flag)) break;
      Cursor nx = cu;
      cursor_next(nx, tiles, nkc, meta);
      const int tok_next = (t + 1 < ntask && nx.kc == 0) ? token(nx) : tok;
      const int k0 = cu.kc * kRbKc;
      const int kel = min(kRbKc, H - k0);
      const int nt = min(kTok, meta.n[cu.slot] - cu.pass * kTok);
      const uint32_t full = smem_u32(&ctl->full[s]);
      uint8_t* st = smem + s * C::kStage;
      if (lane == 0)
        mbar_arrive_expect_tx(full, 2u * (uint32_t)(box_chunks * kRbRows * 128) + (uint32_t)(nt * kel * (int)sizeof(XT)) +
                                        (s_tma ? 2u * kRbRows * C::kScaleRow : 0u));
      __syncwarp();
      const int grow = meta.e[cu.slot] * 2 * I + cu.tile * kRbRows;  // first gate row; up rows are I further
      if (lane < 2) {
        const uint32_t dst = smem_u32(st + C::kW + lane * C::kBlock);
        const int row = grow + lane * I;
        if (map3d) {
          tma_load_3d(dst, &w13_map, 0, row, k0 / 256, full);
        } else {
          for (int ch = 0; ch < box_chunks; ++ch)
            tma_load_2d(dst + ch * kRbRows * 128, &w13_map, k0 / 2 + ch * 128, row, full);
        }
      }
      if (lane < nt)  // lane n < 8 holds the token id of pass row n
        bulk_g2s(smem_u32(st + C::kB + lane * C::kBStride), x + (size_t)tok * H + k0, kel * (int)sizeof(XT), full);
      // scales: 64 gate rows then 64 up rows, kel/G groups each: two TMA boxes
      // when the scale rows are 16-byte aligned, else pairs of groups by
      // 4-byte async copies
      if (s_tma) {
        if (lane == 2 || lane == 3)
          tma_load_2d(smem_u32(st + C::kS + (lane - 2) * kRbRows * C::kScaleRow), &s_map, k0 / G,
                      grow + (lane - 2) * I, full);
      } else for (int q = lane; q < 2 * kRbRows * C::kPairs; q += 32) {
        const int rr = q / C::kPairs, pp = q - rr * C::kPairs;
        const int i = cu.tile * kRbRows + (rr & (kRbRows - 1));
        if (pp * 2 * G < kel && i < I) {
          const size_t srow = (size_t)grow + (rr >= kRbRows ? I : 0) + (rr & (kRbRows - 1));
          cp_async4(smem_u32(st + C::kS + rr * C::kScaleRow + pp * 4), w13_s + srow * NG + k0 / G + 2 * pp);
        }
      }
      cp_async_arrive_noinc(full);
      ++issued;
      tok = tok_next;
      cu = nx;
    }
    for (int t = max(0, issued - S); t < issued; ++t) {
      const uint32_t full = smem_u32(&ctl->full[t % S]);
      drain_wait(full, (t / S) & 1);
    }
    return;
  }

  // ---------------- consumer warps ----------------
  const int rg = warp & 3, kq = warp >> 2;
  const int r = lane >> 2, c = lane & 3;
  constexpr int kGpq = C::kGpq;
  const int R0 = rg * 16 + r;
  int o0[kGpq], o8[kGpq], ob[kGpq];
#pragma unroll
  for (int j = 0; j < kGpq; ++j) {
    const int g = kq * kGpq + j;  // group within the task
    const int kb = (G == 64) ? g * 32 + 8 * c : g * 16 + 4 * c;
    o0[j] = C::kW + swz_off64(R0, kb);
    o8[j] = C::kW + swz_off64(R0 + 8, kb);
    ob[j] = C::kB + r * C::kBStride + g * G * (int)sizeof(XT) + (G == 64 ? 16 : 8) * c * (int)sizeof(XT);
  }
  // scales of this warp's groups for gate rows R0, R0+8 and up rows R0, R0+8
  const int osg0 = C::kS + R0 * C::kScaleRow + kq * kGpq * 2;
  const int osg8 = osg0 + 8 * C::kScaleRow;
  const int osu0 = osg0 + kRbRows * C::kScaleRow;
  const int osu8 = osu0 + 8 * C::kScaleRow;
  Cursor cu = cursor_at(q0, na, tiles, meta);
  float acc_g[4] = {0.f, 0.f, 0.f, 0.f}, acc_u[4] = {0.f, 0.f, 0.f, 0.f};
  int item = 0;
  for (int t = 0; t < ntask; ++t) {
    const int s = t % S;
    if (cu.kc == 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q) { acc_g[q] = 0.f; acc_u[q] = 0.f; }
    }
    const int ngt = min(kRbKc, H - cu.kc * kRbKc) / G;
    if (!wait_phase(smem_u32(&ctl->full[s]), (t / S) & 1, abort_flag)) return;
    const uint8_t* st = smem + s * C::kStage;
    __half2 sg0[kGpq / 2 > 0 ? kGpq / 2 : 1], sg8[kGpq / 2 > 0 ? kGpq / 2 : 1];
    __half2 su0[kGpq / 2 > 0 ? kGpq / 2 : 1], su8[kGpq / 2 > 0 ? kGpq / 2 : 1];
#pragma unroll
    for (int p = 0; p < kGpq / 2; ++p) {
      sg0[p] = *reinterpret_cast<const __half2*>(st + osg0 + 4 * p);
      sg8[p] = *reinterpret_cast<const __half2*>(st + osg8 + 4 * p);
      su0[p] = *reinterpret_cast<const __half2*>(st + osu0 + 4 * p);
      su8[p] = *reinterpret_cast<const __half2*>(st + osu8 + 4 * p);
    }
#pragma unroll
    for (int j = 0; j < kGpq; ++j) {
      if (kq * kGpq + j < ngt) {
        const RowWords<G> ag0 = lds_row<G>(st + o0[j]);
        const RowWords<G> ag8 = lds_row<G>(st + o8[j]);
        const RowWords<G> au0 = lds_row<G>(st + o0[j] + C::kBlock);
        const RowWords<G> au8 = lds_row<G>(st + o8[j] + C::kBlock);
        BWords<G> b;
        if constexpr (C::kF32) lds_b_f32<G>(st + ob[j], b);
        else lds_b_plane<G>(st + ob[j], b.hi);
        const int p = j >> 1;
        const bool hi = j & 1;
        gateup_group<G, C::kF32>(ag0, ag8, au0, au8, b,
                                 hi ? __high2float(sg0[p]) : __low2float(sg0[p]),
                                 hi ? __high2float(sg8[p]) : __low2float(sg8[p]),
                                 hi ? __high2float(su0[p]) : __low2float(su0[p]),
                                 hi ? __high2float(su8[p]) : __low2float(su8[p]), acc_g, acc_u);
      }
    }
    warp_arrive(smem_u32(&ctl->empty[s]), lane);  // this warp is done with the stage
    if (cu.kc == nkc - 1) {
      const int buf = item & 1, use = item >> 1;
      const int bi = buf * 4 + rg;  // barrier index
      float* rb = red + (size_t)buf * (C::kRed / 4) + (size_t)rg * 3 * 32 * 8;
      if (kq > 0) {
        if (use > 0 && !wait_phase(smem_u32(&ctl->red_empty[bi]), (use - 1) & 1, abort_flag)) return;
        float4* dst = reinterpret_cast<float4*>(rb + ((kq - 1) * 32 + lane) * 8);
        dst[0] = make_float4(acc_g[0], acc_g[1], acc_g[2], acc_g[3]);
        dst[1] = make_float4(acc_u[0], acc_u[1], acc_u[2], acc_u[3]);
        warp_arrive(smem_u32(&ctl->red_full[bi]), lane);
      } else {
        if (!wait_phase(smem_u32(&ctl->red_full[bi]), use & 1, abort_flag)) return;
        float gs[4] = {acc_g[0], acc_g[1], acc_g[2], acc_g[3]};
        float us[4] = {acc_u[0], acc_u[1], acc_u[2], acc_u[3]};
#pragma unroll
        for (int w = 0; w < 3; ++w) {
          const float4* src = reinterpret_cast<const float4*>(rb + (w * 32 + lane) * 8);
          const float4 a = src[0], b = src[1];
          gs[0] += a.x; gs[1] += a.y; gs[2] += a.z; gs[3] += a.w;
          us[0] += b.x; us[1] += b.y; us[2] += b.z; us[3] += b.w;
        }
        warp_arrive(smem_u32(&ctl->red_empty[bi]), lane);
        const int n = meta.n[cu.slot], row0 = meta.row0[cu.slot];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int i = cu.tile * kRbRows + R0 + (q >= 2 ? 8 : 0);
          const int rr = cu.pass * kTok + 2 * c + (q & 1);
          if (rr < n && i < I) {
            store_h<C::kF32>(silu_f32(gs[q]) * us[q], h_hi, h_lo, (size_t)(row0 + rr) * I + i);
          }
        }
      }
      ++item;
    }
    cursor_next(cu, tiles, nkc, meta);
  }
}

// down projection
// ---------------------------------------------------------------------------
template <int G>
struct DownCfg {
  static constexpr int kStages = 3;
  static constexpr int kRows = 128;
  static constexpr int kKch = 512;
  static constexpr int kWch = kKch / 32;
  static constexpr int kPairs = kKch / G / 2;
  static constexpr int kWStride = kKch / 2 + (G == 64 ? 32 : 16);
  static constexpr int kScaleRow = kKch / G * 2;
  static constexpr int kBRowBytes = kKch * 2;  // one bf16 plane
  static constexpr int kBch = kBRowBytes / 16;
  static constexpr int kBStride = kBRowBytes + (G == 64 ? 16 : 64);
  static constexpr int kW = 0;
  static constexpr int kS = kRows * kWStride;
  static constexpr int kB = kS + kRows * kScaleRow;             // [2 planes][kTok][kBStride]
  static constexpr int kStage = (kB + 2 * kTok * kBStride + 127) / 128 * 128;
  static constexpr int kRed = 8 * 4 * 32 * 4;
};

template <int G, bool kTwo>
__global__ void __launch_bounds__(kDownThreads, 1)
ffn_down_kernel(const __half* __restrict__ h_hi, const __half* __restrict__ h_lo,
                const int32_t* __restrict__ offsets, const int32_t* __restrict__ active,
                const uint8_t* __restrict__ w2_q, const uint16_t* __restrict__ w2_s, int H, int I, int E,
                float* __restrict__ y) {
  pdl_begin();
  using C = DownCfg<G>;
  constexpr int S = C::kStages;
  extern __shared__ __align__(128) uint8_t smem[];
  float* red = reinterpret_cast<float*>(smem + S * C::kStage);  // [8][4][32]
  int* mbase = reinterpret_cast<int*>(smem + S * C::kStage + C::kRed);
  const Meta meta{mbase, mbase + (E + 1), mbase + 2 * (E + 1), mbase + 3 * (E + 1)};
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, c = lane & 3;
  const int rb = warp & 7, kh = warp >> 3;  // row block, K half
  const int tiles = H / C::kRows;
  const int NG = I / G;
  const int nkc = (I + C::kKch - 1) / C::kKch;
  const size_t row_bytes = (size_t)I / 2;
  const int na = active[0];

  const int total = build_meta(offsets, active, tiles, meta);
  int q0, q1;
  cta_range(total, q0, q1);
  const int ntask = (q1 - q0) * nkc;
  if (ntask == 0) return;

  auto issue = [&](const Cursor& cu, int task) {
    uint8_t* st = smem + (task % S) * C::kStage;
    const int k0 = cu.kc * C::kKch;
    const int kel = min(C::kKch, I - k0);
    const size_t rbase = (size_t)meta.e[cu.slot] * H + (size_t)cu.tile * C::kRows;
#pragma unroll
    for (int q = threadIdx.x; q < C::kRows * C::kWch; q += kDownThreads) {
      const int rr = q / C::kWch, cc = q % C::kWch;
      if (cc * 32 < kel)
        cp_async16(smem_u32(st + C::kW + rr * C::kWStride + cc * 16), w2_q + (rbase + rr) * row_bytes + k0 / 2 + cc * 16);
    }
#pragma unroll
    for (int q = threadIdx.x; q < C::kRows * C::kPairs; q += kDownThreads) {
      const int rr = q / C::kPairs, pp = q % C::kPairs;
      if (pp * 2 * G < kel)
        cp_async4(smem_u32(st + C::kS + rr * C::kScaleRow + pp * 4), w2_s + (rbase + rr) * NG + k0 / G + 2 * pp);
    }
    // h rows of the pass (one fp16 plane, two with fp32 activations), this K-chunk
    const int row_p = meta.row0[cu.slot] + cu.pass * kTok;
    const int nt = min(kTok, meta.n[cu.slot] - cu.pass * kTok);
#pragma unroll
    for (int q = threadIdx.x; q < (kTwo ? 2 : 1) * kTok * C::kBch; q += kDownThreads) {
      const int pl = q / (kTok * C::kBch);
      const int n = (q / C::kBch) % kTok, cc = q % C::kBch;
      if (n < nt && cc * 8 < kel) {
        const __half* src = (pl ? h_lo : h_hi) + (size_t)(row_p + n) * I + k0;
        cp_async16(smem_u32(st + C::kB + (pl * kTok + n) * C::kBStride + cc * 16),
                   reinterpret_cast<const uint8_t*>(src) + cc * 16);
      }
    }
  };

  Cursor ci = cursor_at(q0, na, tiles, meta);
  for (int s = 0; s < S - 1; ++s) {
    if (s < ntask) issue(ci, s);
    cp_async_commit();
    cursor_next(ci, tiles, nkc, meta);
  }
  Cursor cm = cursor_at(q0, na, tiles, meta);

  float acc[4];
  const int lr0 = rb * 16 + r;
  const int a_off = (G == 64) ? 8 * c : 4 * c;
  const int b_off = (G == 64 ? 32 : 16) * c;
  for (int task = 0; task < ntask; ++task) {
    if (task + S - 1 < ntask) issue(ci, task + S - 1);
    cp_async_commit();
    cursor_next(ci, tiles, nkc, meta);
    if (cm.kc == 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[q] = 0.f;
    }
    const int ngt = min(C::kKch, I - cm.kc * C::kKch) / G;
    const int n = meta.n[cm.slot], p0 = cm.pass * kTok;
    const bool tok_ok = p0 + r < n;  // B rows beyond the pass hold stale data: use zeros
    cp_async_wait<S - 1>();
    __syncthreads();
    const uint8_t* st = smem + (task % S) * C::kStage;
    const __half* sc = reinterpret_cast<const __half*>(st + C::kS);
    constexpr int kScH = C::kScaleRow / 2;
#pragma unroll 2
    for (int g = kh; g < ngt; g += 2) {
      const uint8_t* ab = st + C::kW + g * (G / 2) + a_off;
      const RowWords<G> a0 = lds_row<G>(ab + lr0 * C::kWStride);
      const RowWords<G> a8 = lds_row<G>(ab + (lr0 + 8) * C::kWStride);
      BWords<G> b;
      if (tok_ok) {
        const uint8_t* bb = st + C::kB + r * C::kBStride + g * G * 2 + b_off;
        lds_b_plane<G>(bb, b.hi);
        if constexpr (kTwo) lds_b_plane<G>(bb + kTok * C::kBStride, b.lo);
      } else {
#pragma unroll
        for (int i = 0; i < G / 8; ++i) b.hi[i] = b.lo[i] = 0u;
      }
      down_group<G, kTwo>(a0, a8, b, __half2float(sc[lr0 * kScH + g]), __half2float(sc[(lr0 + 8) * kScH + g]), acc);
    }
    if (cm.kc == nkc - 1) {
      if (kh == 1) {
#pragma unroll
        for (int q = 0; q < 4; ++q) red[(rb * 4 + q) * 32 + lane] = acc[q];
      }
      __syncthreads();
      if (kh == 0) {
        const int row0 = meta.row0[cm.slot];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float v = acc[q] + red[(rb * 4 + q) * 32 + lane];
          const int hrow = cm.tile * C::kRows + lr0 + (q >= 2 ? 8 : 0);
          const int rr = p0 + 2 * c + (q & 1);
          if (rr < n) y[(size_t)(row0 + rr) * H + hrow] = v;
        }
      }
    }
    cursor_next(cm, tiles, nkc, meta);
    __syncthreads();  // stage (task % S) and `red` are free again
  }
  cp_async_wait<0>();
}

// ---------------------------------------------------------------------------
// gate/up + SwiGLU, multi-token form (batches with >= ~12 rows per expert)
// ---------------------------------------------------------------------------
// As the row-block form, but an item covers up to 32 tokens of one expert:
// each lane unpacks its A fragments once per group and applies them to every
// 8-token column block of the item (up to four mma.sync per fragment and row
// pair), so the unpack cost is shared by up to 32 tokens. Item = (expert, 64
// gate rows + the 64 matching up rows, block of up to 32 tokens); task = one
// 512-element K chunk. Eight consumer warps = 4 row groups x 2 K halves (288
// threads leave registers for the accumulators). Each warp keeps one
// accumulator per 128-element K quarter of the task, and the item's end sum
// is ((q0 + q1) + q2) + q3 like the row-block form's, so both forms give
// bit-identical h for every row: which one runs never changes the result.
constexpr int kMtConsumers = 8;
constexpr int kMtThreads = (kMtConsumers + 1) * 32;
constexpr int kMtRows = 64;
constexpr int kMtKc = 512;
constexpr int kMtTok = 32;
constexpr int kMtNb = kMtTok / kTok;  // 8-token column blocks per item
// expected rows per expert from which a launch takes the multi-token form
#ifndef PHMOE_DECODE_MT_MIN_ROWS
#define PHMOE_DECODE_MT_MIN_ROWS 20
#endif
constexpr int kMtMinRowsPerExpert = PHMOE_DECODE_MT_MIN_ROWS;

template <int S>
struct MtCtl {
  uint64_t full[S];
  uint64_t empty[S];
  uint64_t red_full[4];   // [rg]: the K-half-1 warp has written its partials
  uint64_t red_empty[4];  // [rg]: the K-half-0 warp has read them
  int abort_flag;
};

template <int G, typename XT>
struct MtCfg {
  static constexpr bool kF32 = std::is_same<XT, float>::value;
  static constexpr int kGpq = 128 / G;                        // groups per K quarter per task
  static constexpr int kBlock = 2 * kMtRows * 128;            // one 64-row box of 2 K-chunks (16 KB)
  static constexpr int kScaleRow = kMtKc / G * 2;
  static constexpr int kPairs = kMtKc / G / 2;
  static constexpr int kBRowBytes = kMtKc * (int)sizeof(XT);
  static constexpr int kBPad = (G == 32 && !kF32) ? 64 : 16;
  static constexpr int kBStride = kBRowBytes + kBPad;
  static constexpr int kW = 0;                                // [gate box][up box]
  static constexpr int kS = 2 * kBlock;                       // [128 rows][kScaleRow]
  static constexpr int kB = kS + 2 * kMtRows * kScaleRow;     // [32 tokens][kBStride]
  static constexpr int kStage = (kB + kMtTok * kBStride + 1023) / 1024 * 1024;
  static constexpr int kRed = 4 * 32 * (8 * kMtNb) * 4;       // [rg][lane][nb][8] floats
  // three stages where they fit next to the metadata of up to 256 experts
  static constexpr int kStages = (1024 + 3 * kStage + kRed + 256 + (4 * 256 + 4) * 4 <= 232448) ? 3 : 2;
  static constexpr size_t smem(int E) {
    return 1024 + (size_t)kStages * kStage + kRed + sizeof(MtCtl<kStages>) + (size_t)(4 * E + 4) * 4;
  }
};

template <int G, typename XT>
__global__ void __launch_bounds__(kMtThreads, 1)
ffn_gateup_mt_kernel(const __grid_constant__ CUtensorMap w13_map, int map3d, int box_chunks,
                     const __grid_constant__ CUtensorMap s_map, int s_tma, const XT* __restrict__ x,
                     const int32_t* __restrict__ row_token, const int32_t* __restrict__ offsets,
                     const int32_t* __restrict__ active, const uint16_t* __restrict__ w13_s, int H, int I, int E,
                     __half* __restrict__ h_hi, __half* __restrict__ h_lo) {
  pdl_begin();
  using C = MtCfg<G, XT>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* red = reinterpret_cast<float*>(smem + S * C::kStage);
  MtCtl<S>* ctl = reinterpret_cast<MtCtl<S>*>(smem + S * C::kStage + C::kRed);
  int* mbase = reinterpret_cast<int*>(ctl + 1);
  const Meta meta{mbase, mbase + (E + 1), mbase + 2 * (E + 1), mbase + 3 * (E + 1)};
  volatile int* abort_flag = &ctl->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = (I + kMtRows - 1) / kMtRows;
  const int NG = H / G;
  const int nkc = (H + kMtKc - 1) / kMtKc;
  const int na = active[0];

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&ctl->full[s]), 1 + 32);
      mbar_init(smem_u32(&ctl->empty[s]), kMtConsumers);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(smem_u32(&ctl->red_full[i]), 1);
      mbar_init(smem_u32(&ctl->red_empty[i]), 1);
    }
    ctl->abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  const int total = build_meta<kMtTok>(offsets, active, tiles, meta);
  int q0, q1;
  cta_range(total, q0, q1);
  const int ntask = (q1 - q0) * nkc;
  if (ntask == 0) return;

  if (warp == kMtConsumers) {
    // ---------------- producer warp ----------------
    Cursor cu = cursor_at<kMtTok>(q0, na, tiles, meta);
    auto token = [&](const Cursor& k) -> int {  // lane holds the token id of block row `lane`
      const int rr = k.pass * kMtTok + lane;
      return rr < meta.n[k.slot] ? __ldg(row_token + meta.row0[k.slot] + rr) : -1;
    };
    int tok = token(cu);
    int issued = 0;
    for (int t = 0; t < ntask; ++t) {
      const int s = t % S;
      if (t >= S && !wait_phase(smem_u32(&ctl->empty[s]), (t / S - 1) & 1, abort_flag)) break;
      Cursor nx = cu;
      cursor_next<kMtTok>(nx, tiles, nkc, meta);
      const int tok_next = (t + 1 < ntask && nx.kc == 0) ? token(nx) : tok;
      const int k0 = cu.kc * kMtKc;
      const int kel = min(kMtKc, H - k0);
      const int nt = min(kMtTok, meta.n[cu.slot] - cu.pass * kMtTok);
      const uint32_t full = smem_u32(&ctl->full[s]);
      uint8_t* st = smem + s * C::kStage;
      if (lane == 0)
        mbar_arrive_expect_tx(full, 2u * (uint32_t)(box_chunks * kMtRows * 128) + (uint32_t)(nt * kel * (int)sizeof(XT)) +
                                        (s_tma ? 2u * kMtRows * C::kScaleRow : 0u));
      __syncwarp();
      const int grow = meta.e[cu.slot] * 2 * I + cu.tile * kMtRows;  // first gate row; up rows are I further
      if (lane < 2) {
        const uint32_t dst = smem_u32(st + C::kW + lane * C::kBlock);
        const int row = grow + lane * I;
        if (map3d) {
          tma_load_3d(dst, &w13_map, 0, row, k0 / 256, full);
        } else {
          for (int ch = 0; ch < box_chunks; ++ch)
            tma_load_2d(dst + ch * kMtRows * 128, &w13_map, k0 / 2 + ch * 128, row, full);
        }
      }
      if (lane < nt)  // lane n < 32 holds the token id of block row n
        bulk_g2s(smem_u32(st + C::kB + lane * C::kBStride), x + (size_t)tok * H + k0, kel * (int)sizeof(XT), full);
      if (s_tma) {
        if (lane == 2 || lane == 3)
          tma_load_2d(smem_u32(st + C::kS + (lane - 2) * kMtRows * C::kScaleRow), &s_map, k0 / G,
                      grow + (lane - 2) * I, full);
      } else {
        for (int q = lane; q < 2 * kMtRows * C::kPairs; q += 32) {
          const int rr = q / C::kPairs, pp = q - rr * C::kPairs;
          const int i = cu.tile * kMtRows + (rr & (kMtRows - 1));
          if (pp * 2 * G < kel && i < I) {
            const size_t srow = (size_t)grow + (rr >= kMtRows ? I : 0) + (rr & (kMtRows - 1));
            cp_async4(smem_u32(st + C::kS + rr * C::kScaleRow + pp * 4), w13_s + srow * NG + k0 / G + 2 * pp);
          }
        }
      }
      cp_async_arrive_noinc(full);
      ++issued;
      tok = tok_next;
      cu = nx;
    }
    for (int t = max(0, issued - S); t < issued; ++t) {
      const uint32_t full = smem_u32(&ctl->full[t % S]);
      drain_wait(full, (t / S) & 1);
    }
    return;
  }

  // ---------------- consumer warps ----------------
  const int rg = warp & 3, kh = warp >> 2;
  const int r = lane >> 2, c = lane & 3;
  constexpr int kGpq = C::kGpq;
  const int R0 = rg * 16 + r;
  constexpr int kScH = C::kScaleRow / 2;
  Cursor cu = cursor_at<kMtTok>(q0, na, tiles, meta);
  float acc_g[2][kMtNb][4], acc_u[2][kMtNb][4];  // [K quarter of this half][block][fragment]
  int item = 0;
  for (int t = 0; t < ntask; ++t) {
    const int s = t % S;
    if (cu.kc == 0) {
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int b = 0; b < kMtNb; ++b)
#pragma unroll
          for (int q = 0; q < 4; ++q) { acc_g[h][b][q] = 0.f; acc_u[h][b][q] = 0.f; }
    }
    const int nb = (min(kMtTok, meta.n[cu.slot] - cu.pass * kMtTok) + kTok - 1) / kTok;  // warp-uniform
    const int ngt = min(kMtKc, H - cu.kc * kMtKc) / G;
    if (!wait_phase(smem_u32(&ctl->full[s]), (t / S) & 1, abort_flag)) return;
    const uint8_t* st = smem + s * C::kStage;
    const __half* sc = reinterpret_cast<const __half*>(st + C::kS);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll 1
      for (int j = 0; j < kGpq; ++j) {
        const int g = (2 * kh + h) * kGpq + j;  // group within the task
        if (g < ngt) {
          const int kb = (G == 64) ? g * 32 + 8 * c : g * 16 + 4 * c;
          const RowWords<G> ag0 = lds_row<G>(st + C::kW + swz_off64(R0, kb));
          const RowWords<G> ag8 = lds_row<G>(st + C::kW + swz_off64(R0 + 8, kb));
          const RowWords<G> au0 = lds_row<G>(st + C::kW + C::kBlock + swz_off64(R0, kb));
          const RowWords<G> au8 = lds_row<G>(st + C::kW + C::kBlock + swz_off64(R0 + 8, kb));
          const float sg0 = __half2float(sc[R0 * kScH + g]), sg8 = __half2float(sc[(R0 + 8) * kScH + g]);
          const float su0 = __half2float(sc[(kMtRows + R0) * kScH + g]);
          const float su8 = __half2float(sc[(kMtRows + R0 + 8) * kScH + g]);
          const int ob =
              C::kB + r * C::kBStride + g * G * (int)sizeof(XT) + (G == 64 ? 16 : 8) * c * (int)sizeof(XT);
          gateup_group_mt<G, C::kF32, kMtNb>(ag0, ag8, au0, au8, st + ob, kTok * C::kBStride, nb, sg0, sg8, su0,
                                             su8, acc_g[h], acc_u[h]);
        }
      }
    }
    warp_arrive(smem_u32(&ctl->empty[s]), lane);
    if (cu.kc == nkc - 1) {
      float4* rb = reinterpret_cast<float4*>(red) + ((size_t)rg * 32 + lane) * (2 * kMtNb);
      if (kh == 0) {  // hands q0 + q1 to the K-half-1 warp
        if (item > 0 && !wait_phase(smem_u32(&ctl->red_empty[rg]), (item - 1) & 1, abort_flag)) return;
#pragma unroll
        for (int b = 0; b < kMtNb; ++b) {
          if (b < nb) {
            rb[2 * b] = make_float4(acc_g[0][b][0] + acc_g[1][b][0], acc_g[0][b][1] + acc_g[1][b][1],
                                    acc_g[0][b][2] + acc_g[1][b][2], acc_g[0][b][3] + acc_g[1][b][3]);
            rb[2 * b + 1] = make_float4(acc_u[0][b][0] + acc_u[1][b][0], acc_u[0][b][1] + acc_u[1][b][1],
                                        acc_u[0][b][2] + acc_u[1][b][2], acc_u[0][b][3] + acc_u[1][b][3]);
          }
        }
        warp_arrive(smem_u32(&ctl->red_full[rg]), lane);
      } else {  // ((q0 + q1) + q2) + q3, then SwiGLU
        if (!wait_phase(smem_u32(&ctl->red_full[rg]), item & 1, abort_flag)) return;
        const int n = meta.n[cu.slot], row0 = meta.row0[cu.slot];
#pragma unroll
        for (int b = 0; b < kMtNb; ++b) {
          if (b < nb) {
            const float4 og = rb[2 * b], ou = rb[2 * b + 1];
            const float gs[4] = {(og.x + acc_g[0][b][0]) + acc_g[1][b][0], (og.y + acc_g[0][b][1]) + acc_g[1][b][1],
                                 (og.z + acc_g[0][b][2]) + acc_g[1][b][2], (og.w + acc_g[0][b][3]) + acc_g[1][b][3]};
            const float us[4] = {(ou.x + acc_u[0][b][0]) + acc_u[1][b][0], (ou.y + acc_u[0][b][1]) + acc_u[1][b][1],
                                 (ou.z + acc_u[0][b][2]) + acc_u[1][b][2], (ou.w + acc_u[0][b][3]) + acc_u[1][b][3]};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int i = cu.tile * kMtRows + R0 + (q >= 2 ? 8 : 0);
              const int rr = cu.pass * kMtTok + b * kTok + 2 * c + (q & 1);
              if (rr < n && i < I) {
                store_h<C::kF32>(silu_f32(gs[q]) * us[q], h_hi, h_lo, (size_t)(row0 + rr) * I + i);
              }
            }
          }
        }
        warp_arrive(smem_u32(&ctl->red_empty[rg]), lane);
      }
      ++item;
    }
    cursor_next<kMtTok>(cu, tiles, nkc, meta);
  }
}

// ---------------------------------------------------------------------------
// down projection, TMA-fed form (I % 256 == 0)
// ---------------------------------------------------------------------------
// Item = (expert, 128 output rows, pass of 8 tokens); task = one 512-element
// K chunk. A producer warp copies per task one TMA box of weights (128 rows x
// 2 x 128 bytes, 128-byte swizzle), the matching scales (a TMA box when the
// scale rows are 16-byte aligned, else one bulk copy of the block's
// contiguous scale rows, else 4-byte async copies) and the two h planes of
// the pass (one TMA box each: 8 groups x 8 rows x 64 elements, 128-byte
// swizzle). Consumer warp w owns 16-row group w%8 and K half w/8; the two
// halves are summed (fixed order) at the item's end.
constexpr int kDnRows = 128;
constexpr int kDnKc = 512;
constexpr int kDnScaleBytes = 4096;  // scale region of a stage

template <int S>
struct DnCtl {
  uint64_t full[S];
  uint64_t empty[S];
  uint64_t red_full[16];   // [buf][rg]
  uint64_t red_empty[16];
  int abort_flag;
};

template <int G>
struct DnCfg {
  static constexpr int kGph = 256 / G;                 // groups per consumer warp per task
  static constexpr int kW = 0;                         // [2 chunks][128 rows][128 B]
  static constexpr int kS = 2 * kDnRows * 128;         // scales
  static constexpr int kB = kS + kDnScaleBytes;        // [2 planes][8 groups][8 rows][128 B]
  static constexpr int kPlane = 8 * kTok * 128;
  static constexpr int kStage = kB + 2 * kPlane;
  static constexpr int kStages = 4;
  static constexpr int kRed = 8 * 32 * 16;             // [rg][lane][4 floats]
  static constexpr size_t smem(int E) {
    return 1024 + (size_t)kStages * kStage + 2 * kRed + sizeof(DnCtl<kStages>) + (size_t)(4 * E + 4) * 4;
  }
};

// B words of group g (within a task) for token row r from one h plane laid
// out [64-element block][8 rows][128 B] with 128-byte swizzle.
template <int G>
__device__ __forceinline__ void lds_b_swz(const uint8_t* plane, int g, int r, int c, uint32_t (&d)[G / 8]) {
  if constexpr (G == 64) {
    const uint8_t* row = plane + g * (kTok * 128) + r * 128;
    const uint4 a = *reinterpret_cast<const uint4*>(row + (((2 * c) ^ (r & 7)) << 4));
    const uint4 b = *reinterpret_cast<const uint4*>(row + (((2 * c + 1) ^ (r & 7)) << 4));
    d[0] = a.x; d[1] = a.y; d[2] = a.z; d[3] = a.w;
    d[4] = b.x; d[5] = b.y; d[6] = b.z; d[7] = b.w;
  } else {
    const uint8_t* row = plane + (g >> 1) * (kTok * 128) + r * 128;
    const uint4 a = *reinterpret_cast<const uint4*>(row + ((((g & 1) * 4 + c) ^ (r & 7)) << 4));
    d[0] = a.x; d[1] = a.y; d[2] = a.z; d[3] = a.w;
  }
}

template <int G, bool kTwo>
__global__ void __launch_bounds__(kGuThreads, 1)
ffn_down_tma_kernel(const __grid_constant__ CUtensorMap w_map, const __grid_constant__ CUtensorMap s_map,
                    const __grid_constant__ CUtensorMap hi_map, const __grid_constant__ CUtensorMap lo_map,
                    int s_mode, const int32_t* __restrict__ offsets, const int32_t* __restrict__ active,
                    const uint16_t* __restrict__ w2_s, int H, int I, int E, float* __restrict__ y) {
  pdl_begin();
  using C = DnCfg<G>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* red = reinterpret_cast<float*>(smem + S * C::kStage);  // [2][rg][lane][4]
  DnCtl<S>* ctl = reinterpret_cast<DnCtl<S>*>(smem + S * C::kStage + 2 * C::kRed);
  int* mbase = reinterpret_cast<int*>(ctl + 1);
  const Meta meta{mbase, mbase + (E + 1), mbase + 2 * (E + 1), mbase + 3 * (E + 1)};
  volatile int* abort_flag = &ctl->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = H / kDnRows;
  const int NG = I / G;
  const int nkc = (I + kDnKc - 1) / kDnKc;
  const int na = active[0];
  // scale rows in shared memory: s_mode 0 = TMA box / async copies of the
  // task's groups; 1 = every group of the block (one bulk copy)
  const int srow = s_mode == 1 ? NG * 2 : (kDnKc / G) * 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&ctl->full[s]), 1 + 32);
      mbar_init(smem_u32(&ctl->empty[s]), kConsumers);
    }
    for (int i = 0; i < 16; ++i) {
      mbar_init(smem_u32(&ctl->red_full[i]), 1);
      mbar_init(smem_u32(&ctl->red_empty[i]), 1);
    }
    ctl->abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  const int total = build_meta(offsets, active, tiles, meta);
  int q0, q1;
  cta_range(total, q0, q1);
  const int ntask = (q1 - q0) * nkc;
  if (ntask == 0) return;

  if (warp == kConsumers) {
    // ---------------- producer warp ----------------
    Cursor cu = cursor_at(q0, na, tiles, meta);
    int issued = 0;
    const uint32_t sbytes_block = (uint32_t)kDnRows * (uint32_t)NG * 2;
    for (int t = 0; t < ntask; ++t) {
      const int s = t % S;
      if (t >= S && !wait_phase(smem_u32(&ctl->empty[s]), (t / S - 1) & 1, abort_flag)) break;
      const int k0 = cu.kc * kDnKc;
      const int kel = min(kDnKc, I - k0);
      const uint32_t full = smem_u32(&ctl->full[s]);
      uint8_t* st = smem + s * C::kStage;
      const int wrow = meta.e[cu.slot] * H + cu.tile * kDnRows;
      const int hrow = meta.row0[cu.slot] + cu.pass * kTok;
      const uint32_t sbytes = s_mode == 0 ? (uint32_t)kDnRows * (kDnKc / G) * 2 : (s_mode == 1 ? sbytes_block : 0u);
      if (lane == 0)
        mbar_arrive_expect_tx(full, (uint32_t)(2 * kDnRows * 128) + sbytes + (kTwo ? 2u : 1u) * C::kPlane);
      __syncwarp();
      if (lane == 0) tma_load_3d(smem_u32(st + C::kW), &w_map, 0, wrow, k0 / 256, full);
      if (lane == 1) tma_load_3d(smem_u32(st + C::kB), &hi_map, 0, hrow, k0 / 64, full);
      if (kTwo && lane == 2) tma_load_3d(smem_u32(st + C::kB + C::kPlane), &lo_map, 0, hrow, k0 / 64, full);
      if (s_mode == 0) {
        if (lane == 3) tma_load_2d(smem_u32(st + C::kS), &s_map, k0 / G, wrow, full);
      } else if (s_mode == 1) {
        if (lane == 3) bulk_g2s(smem_u32(st + C::kS), w2_s + (size_t)wrow * NG, sbytes_block, full);
      } else {
        constexpr int kPairs = kDnKc / G / 2;
        for (int q = lane; q < kDnRows * kPairs; q += 32) {
          const int rr = q / kPairs, pp = q - rr * kPairs;
          if (pp * 2 * G < kel)
            cp_async4(smem_u32(st + C::kS + rr * srow + pp * 4), w2_s + (size_t)(wrow + rr) * NG + k0 / G + 2 * pp);
        }
      }
      cp_async_arrive_noinc(full);
      ++issued;
      cursor_next(cu, tiles, nkc, meta);
    }
    for (int t = max(0, issued - S); t < issued; ++t) {
      const uint32_t full = smem_u32(&ctl->full[t % S]);
      drain_wait(full, (t / S) & 1);
    }
    return;
  }

  // ---------------- consumer warps ----------------
  const int rg = warp & 7, kh = warp >> 3;
  const int r = lane >> 2, c = lane & 3;
  const int lr0 = rg * 16 + r;
  const int a_off = (G == 64) ? 8 * c : 4 * c;
  Cursor cu = cursor_at(q0, na, tiles, meta);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  int item = 0;
  for (int t = 0; t < ntask; ++t) {
    const int s = t % S;
    if (cu.kc == 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[q] = 0.f;
    }
    const int ngt = min(kDnKc, I - cu.kc * kDnKc) / G;
    if (!wait_phase(smem_u32(&ctl->full[s]), (t / S) & 1, abort_flag)) return;
    const uint8_t* st = smem + s * C::kStage;
    const __half* sc = reinterpret_cast<const __half*>(st + C::kS);
    const int goff = s_mode == 1 ? cu.kc * (kDnKc / G) : 0;
#pragma unroll
    for (int j = 0; j < C::kGph; ++j) {
      const int g = kh * C::kGph + j;
      if (g < ngt) {
        const int kb = g * (G / 2) + a_off;
        const RowWords<G> a0 = lds_row<G>(st + C::kW + swz_off_rows(lr0, kb, kDnRows));
        const RowWords<G> a8 = lds_row<G>(st + C::kW + swz_off_rows(lr0 + 8, kb, kDnRows));
        BWords<G> b;
        lds_b_swz<G>(st + C::kB, g, r, c, b.hi);
        if constexpr (kTwo) lds_b_swz<G>(st + C::kB + C::kPlane, g, r, c, b.lo);
        down_group<G, kTwo>(a0, a8, b, __half2float(sc[(lr0 * srow) / 2 + goff + g]),
                      __half2float(sc[((lr0 + 8) * srow) / 2 + goff + g]), acc);
      }
    }
    warp_arrive(smem_u32(&ctl->empty[s]), lane);
    if (cu.kc == nkc - 1) {
      const int buf = item & 1, use = item >> 1;
      const int bi = buf * 8 + rg;
      float4* rb = reinterpret_cast<float4*>(red + (size_t)buf * (C::kRed / 4)) + rg * 32 + lane;
      if (kh == 1) {
        if (use > 0 && !wait_phase(smem_u32(&ctl->red_empty[bi]), (use - 1) & 1, abort_flag)) return;
        *rb = make_float4(acc[0], acc[1], acc[2], acc[3]);
        warp_arrive(smem_u32(&ctl->red_full[bi]), lane);
      } else {
        if (!wait_phase(smem_u32(&ctl->red_full[bi]), use & 1, abort_flag)) return;
        const float4 o = *rb;
        warp_arrive(smem_u32(&ctl->red_empty[bi]), lane);
        const float v[4] = {acc[0] + o.x, acc[1] + o.y, acc[2] + o.z, acc[3] + o.w};
        const int n = meta.n[cu.slot], row0 = meta.row0[cu.slot];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int hr = cu.tile * kDnRows + lr0 + (q >= 2 ? 8 : 0);
          const int rr = cu.pass * kTok + 2 * c + (q & 1);
          if (rr < n) y[(size_t)(row0 + rr) * H + hr] = v[q];
        }
      }
      ++item;
    }
    cursor_next(cu, tiles, nkc, meta);
  }
}

template <typename K>
void set_smem(K kern, size_t bytes) {
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// Tensor map over w13_q viewed as [rows = E*2I][K bytes = H/2], for 16-row
// boxes of `box_chunks` 128-byte K-chunks with 128-byte swizzle. First choice:
// a 3-D view (128 B, rows, K-chunks) so one copy moves the whole box; if the
// driver rejects it, a 2-D view copied one 128-byte chunk at a time (same
// shared-memory layout). Returns 0 (2-D), 1 (3-D) or -1 (no map).
int make_w13_map(CUtensorMap* map, const uint8_t* w13_q, long long rows, int H, int box_chunks, int box_rows = 16) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return -1;
  {
    const cuuint64_t dims[3] = {128, (cuuint64_t)rows, (cuuint64_t)(H / 256)};
    const cuuint64_t strides[2] = {(cuuint64_t)(H / 2), 128};
    const cuuint32_t box[3] = {128, (cuuint32_t)box_rows, (cuuint32_t)box_chunks};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(w13_q), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
      return 1;
  }
  const cuuint64_t dims[2] = {(cuuint64_t)(H / 2), (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(H / 2)};
  const cuuint32_t box[2] = {128, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  if (enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(w13_q), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
    return 0;
  return -1;
}

constexpr size_t kMaxSmem = 227 * 1024;

// Tensor map over the fp16 scales [E*2I rows][H/G] for boxes of one task's
// groups x `rows` rows; false when the rows are not 16-byte aligned.
bool make_scale_map(CUtensorMap* map, const uint16_t* w13_s, long long rows, int H, int G, int kc, int box_rows) {
  if (((H / G) * 2) % 16) return false;
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)(H / G), (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(H / G) * 2};
  const cuuint32_t box[2] = {(cuuint32_t)(kc / G), (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint16_t*>(w13_s), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int G, typename XT>
int launch_gateup_mt(const void* x, const int32_t* row_token, const int32_t* offsets, const int32_t* active,
                     const uint8_t* w13_q, const uint16_t* w13_s, int H, int I, int E, __half* h_hi,
                     __half* h_lo, int grid, cudaStream_t st) {
  const size_t smem = MtCfg<G, XT>::smem(E);
  if (smem > kMaxSmem) return PHMOE_ERR_UNSUPPORTED;
  const int box_chunks = std::min(H, kMtKc) / 256;
  alignas(64) CUtensorMap map, smap;
  const int mode = make_w13_map(&map, w13_q, (long long)E * 2 * I, H, box_chunks, kMtRows);
  if (mode < 0) return PHMOE_ERR_CUDA;
  const int s_tma = make_scale_map(&smap, w13_s, (long long)E * 2 * I, H, G, kMtKc, kMtRows) ? 1 : 0;
  if (!s_tma) memset(&smap, 0, sizeof(smap));
  auto k = ffn_gateup_mt_kernel<G, XT>;
  set_smem(k, smem);
  launch_pdl(k, dim3(grid), dim3(kMtThreads), smem, st, map, mode, box_chunks, smap, s_tma, static_cast<const XT*>(x), row_token, offsets,
                                    active, w13_s, H, I, E, h_hi, h_lo);
  return PHMOE_OK;
}

template <int G, typename XT>
int launch_gateup_rb(const void* x, const int32_t* row_token, const int32_t* offsets, const int32_t* active,
                     const uint8_t* w13_q, const uint16_t* w13_s, int H, int I, int E, __half* h_hi,
                     __half* h_lo, int grid, cudaStream_t st) {
  const int box_chunks = std::min(H, kRbKc) / 256;
  alignas(64) CUtensorMap map, smap;
  const int mode = make_w13_map(&map, w13_q, (long long)E * 2 * I, H, box_chunks, kRbRows);
  if (mode < 0) return PHMOE_ERR_CUDA;
  // scales as a 2-D fp16 tensor [E*2I rows][H/G]: boxes of one task's groups x 64 rows
  int s_tma = 0;
  if (((H / G) * 2) % 16 == 0) {
    EncodeTiledFn enc = encode_fn();
    const cuuint64_t dims[2] = {(cuuint64_t)(H / G), (cuuint64_t)E * 2 * I};
    const cuuint64_t strides[1] = {(cuuint64_t)(H / G) * 2};
    const cuuint32_t box[2] = {(cuuint32_t)(kRbKc / G), (cuuint32_t)kRbRows};
    const cuuint32_t estr[2] = {1, 1};
    s_tma = enc && enc(&smap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint16_t*>(w13_s), dims, strides, box,
                       estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  }
  if (!s_tma) memset(&smap, 0, sizeof(smap));
  const size_t smem = RbCfg<G, XT>::smem(E);
  if (smem > kMaxSmem) return PHMOE_ERR_UNSUPPORTED;
  auto k = ffn_gateup_rb_kernel<G, XT>;
  set_smem(k, smem);
  launch_pdl(k, dim3(grid), dim3(kGuThreads), smem, st, map, mode, box_chunks, smap, s_tma, static_cast<const XT*>(x), row_token,
                                    offsets, active, w13_s, H, I, E, h_hi, h_lo);
  return PHMOE_OK;
}

template <int G>
size_t down_smem(int E) {
  using C = DownCfg<G>;
  return (size_t)C::kStages * C::kStage + C::kRed + (size_t)(4 * E + 4) * 4;
}

template <int G, bool kTwo>
void launch_down(const __half* h_hi, const __half* h_lo, const int32_t* offsets,
                 const int32_t* active, const uint8_t* w2_q, const uint16_t* w2_s, int H, int I, int E, float* y,
                 int grid, cudaStream_t st) {
  const size_t smem = down_smem<G>(E);
  auto k = ffn_down_kernel<G, kTwo>;
  set_smem(k, smem);
  launch_pdl(k, dim3(grid), dim3(kDownThreads), smem, st, h_hi, h_lo, offsets, active, w2_q, w2_s, H, I, E, y);
}

// TMA-fed down projection; returns false (nothing launched) when the shape
// or the tensor maps do not allow it.
template <int G, bool kTwo>
bool launch_down_tma(const __half* h_hi, const __half* h_lo, long long R, const int32_t* offsets,
                     const int32_t* active, const uint8_t* w2_q, const uint16_t* w2_s, int H, int I, int E, float* y,
                     int grid, cudaStream_t st) {
  if (I % 256 || H % kDnRows || R <= 0) return false;
  const size_t smem = DnCfg<G>::smem(E);
  if (smem > kMaxSmem) return false;
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  alignas(64) CUtensorMap wm, sm, hm, lm;
  const cuuint32_t e3[3] = {1, 1, 1}, e2[2] = {1, 1};
  {
    const cuuint64_t dims[3] = {128, (cuuint64_t)E * H, (cuuint64_t)(I / 256)};
    const cuuint64_t strides[2] = {(cuuint64_t)(I / 2), 128};
    const cuuint32_t box[3] = {128, (cuuint32_t)kDnRows, 2};
    if (enc(&wm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(w2_q), dims, strides, box, e3,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return false;
  }
  const __half* planes[2] = {h_hi, h_lo};
  CUtensorMap* pm[2] = {&hm, &lm};
  for (int p = 0; p < 2; ++p) {
    const cuuint64_t dims[3] = {64, (cuuint64_t)R, (cuuint64_t)(I / 64)};
    const cuuint64_t strides[2] = {(cuuint64_t)I * 2, 128};
    const cuuint32_t box[3] = {64, (cuuint32_t)kTok, 8};
    if (enc(pm[p], CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<__half*>(planes[p]), dims, strides, box, e3,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return false;
  }
  const int NG = I / G;
  int s_mode = 2;
  memset(&sm, 0, sizeof(sm));
  if ((NG * 2) % 16 == 0) {
    const cuuint64_t dims[2] = {(cuuint64_t)NG, (cuuint64_t)E * H};
    const cuuint64_t strides[1] = {(cuuint64_t)NG * 2};
    const cuuint32_t box[2] = {(cuuint32_t)(kDnKc / G), (cuuint32_t)kDnRows};
    if (enc(&sm, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint16_t*>(w2_s), dims, strides, box, e2,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
      s_mode = 0;
  }
  if (s_mode == 2 && (size_t)kDnRows * NG * 2 <= (size_t)kDnScaleBytes &&
      (reinterpret_cast<uintptr_t>(w2_s) & 15) == 0)
    s_mode = 1;
  auto k = ffn_down_tma_kernel<G, kTwo>;
  set_smem(k, smem);
  launch_pdl(k, dim3(grid), dim3(kGuThreads), smem, st, wm, sm, hm, lm, s_mode, offsets, active, w2_s, H, I, E, y);
  return true;
}

}  // namespace

int ffn_device_error(bool reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_ffn_error, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_ffn_error, &zero, sizeof(int));
  }
  return v;
}

int launch_ffn_decode(const void* x, int x_dtype, const int32_t* row_token,
                      const int32_t* offsets, const int32_t* active, const uint8_t* w13_q,
                      const uint16_t* w13_s, const uint8_t* w2_q, const uint16_t* w2_s, int T,
                      int H, int E, int top_k, int I, int G, float* h, float* y,
                      cudaStream_t st, cudaEvent_t mid_event, long long rows_hint) {
  const long long R = (long long)T * top_k;
  if (R == 0) return PHMOE_OK;
  if (G != 32 && G != 64) return PHMOE_ERR_UNSUPPORTED;
  __half* h_hi = reinterpret_cast<__half*>(h);  // fp16 planes: hi, then lo (fp32 activations only)
  __half* h_lo = h_hi + (size_t)R * I;
  const int grid = device_sm_count();
  const bool f32 = x_dtype == PHMOE_DTYPE_F32;
  // multi-token gate/up items from kMtMinRowsPerExpert expected rows per
  // expert (each unpacked weight then feeds two or more 8-token MMA blocks);
  // both forms give bit-identical h, so this choice is for speed only
  const long long rows = rows_hint >= 0 ? rows_hint : R;
  const bool mt = rows >= (long long)kMtMinRowsPerExpert * E;
  int s = PHMOE_ERR_UNSUPPORTED;
  if (mt) {
    if (G == 64)
      s = f32 ? launch_gateup_mt<64, float>(x, row_token, offsets, active, w13_q, w13_s, H, I, E, h_hi, h_lo, grid, st)
              : launch_gateup_mt<64, __nv_bfloat16>(x, row_token, offsets, active, w13_q, w13_s, H, I, E, h_hi, h_lo,
                                                    grid, st);
    else
      s = f32 ? launch_gateup_mt<32, float>(x, row_token, offsets, active, w13_q, w13_s, H, I, E, h_hi, h_lo, grid, st)
              : launch_gateup_mt<32, __nv_bfloat16>(x, row_token, offsets, active, w13_q, w13_s, H, I, E, h_hi, h_lo,
                                                    grid, st);
  }
  if (s != PHMOE_OK) {  // 8-token items (small batches, or the multi-token form did not fit)
    if (G == 64)
      s = f32 ? launch_gateup_rb<64, float>(x, row_token, offsets, active, w13_q, w13_s, H, I, E, h_hi, h_lo, grid, st)
              : launch_gateup_rb<64, __nv_bfloat16>(x, row_token, offsets, active, w13_q, w13_s, H, I, E, h_hi, h_lo,
                                                    grid, st);
    else
      s = f32 ? launch_gateup_rb<32, float>(x, row_token, offsets, active, w13_q, w13_s, H, I, E, h_hi, h_lo, grid, st)
              : launch_gateup_rb<32, __nv_bfloat16>(x, row_token, offsets, active, w13_q, w13_s, H, I, E, h_hi, h_lo,
                                                    grid, st);
  }
  if (s) return s;
  if (mid_event) cudaEventRecord(mid_event, st);
  bool tma;
  if (G == 64)
    tma = f32 ? launch_down_tma<64, true>(h_hi, h_lo, R, offsets, active, w2_q, w2_s, H, I, E, y, grid, st)
              : launch_down_tma<64, false>(h_hi, h_lo, R, offsets, active, w2_q, w2_s, H, I, E, y, grid, st);
  else
    tma = f32 ? launch_down_tma<32, true>(h_hi, h_lo, R, offsets, active, w2_q, w2_s, H, I, E, y, grid, st)
              : launch_down_tma<32, false>(h_hi, h_lo, R, offsets, active, w2_q, w2_s, H, I, E, y, grid, st);
  if (!tma) {
    if (G == 64 && f32) launch_down<64, true>(h_hi, h_lo, offsets, active, w2_q, w2_s, H, I, E, y, grid, st);
    else if (G == 64) launch_down<64, false>(h_hi, h_lo, offsets, active, w2_q, w2_s, H, I, E, y, grid, st);
    else if (f32) launch_down<32, true>(h_hi, h_lo, offsets, active, w2_q, w2_s, H, I, E, y, grid, st);
    else launch_down<32, false>(h_hi, h_lo, offsets, active, w2_q, w2_s, H, I, E, y, grid, st);
  }
  note_launches(2);
  return PHMOE_OK;
}

}  // namespace phmoe
