// Grouped SwiGLU expert FFN, decode form (few tokens per expert).
//
// Reference: Qwen3MoeExperts.forward loop body (transformers 5.5.0
// models/qwen3_moe/modeling_qwen3_moe.py:245-247):
//   gate, up = linear(x_e, gate_up_proj[e]).chunk(2); h = silu(gate) * up;
//   y_e = linear(h, down_proj[e])
// on weights dequantised as (nibble - 8) * scale (gguf_loader.py:372-378).
//
// At decode sizes the layer streams ~2.5 MB of packed weights per expert hit
// and does a few multiply-adds per weight: the bound is HBM, and the kernels
// are built to spend as few instructions per weight byte as possible.
//
// Numerics: exact integer dot products on the int8 tensor cores.
//  * The activations of the rows and the SwiGLU output h are "fx rows"
//    (common.cuh): per row and group of G elements a power-of-two exponent
//    and integers |A| <= 8191 (16383 for G = 32) split into two signed
//    bytes, A = 256 hi + lo. fx_rows_kernel encodes x; the gate/up epilogue
//    encodes h.
//  * A weight word (8 nibbles) becomes two registers of unsigned bytes with
//    one AND and one shift + AND (nib_bytes); mma.sync m16n8k32 u8 x s8
//    gives the exact int32 sums sum(n * hi) and C0 + sum(n * lo) per group
//    (one MMA type for both planes); one IMAD joins them, and the result
//    read as a float minus the group's magic constant is
//    sum((n - 8) * A) * 2^e exactly (no int-to-float conversion). The fp16
//    weight scale multiplies it and fp32 accumulates over the groups.
//  * Every group's dot product is exact: the only roundings are the
//    encodings of x and h (to 2^-13 of the group's largest |value| or
//    better) and the fp32 accumulation. The exponent adapts per group, so any
//    finite value below ~1e34 is held; larger or non-finite values are
//    clamped and raise bit value 2 of the device error word.
//
// gate/up kernel (persistent, one CTA per SM, warp-specialised):
//  * item = (expert, 64 gate rows and the 64 matching up rows, pass of 8
//    tokens); task = one 512-element K chunk of an item (32 KB of weights).
//    Three producer warps issue side by side (each copy instruction waits
//    behind the consumers' shared-memory loads): two TMA tensor copies of
//    weights (128-byte swizzle) and two of the fp16 scale slices; one bulk
//    copy per token of its fx row slice; 8-byte async copies of the fx
//    constants (transposed to [group][token] so a lane reads its two tokens'
//    constants with one 16-byte load). All complete on the stage's "full"
//    mbarrier. Consumer warp w owns 16-row group w%4 and K quarter w/4 of
//    every task; its accumulators cover the item's whole K. An expert with
//    more than 8 rows takes one pass per 8 of them (its weights come from L2
//    after the first). (A form that unpacked each weight once for up to 32
//    tokens was slower at every batch once the producers were split.)
//  * epilogue (4 warps, one per 16-row group): the four K-quarter partials
//    summed in fixed order ((q0 + q1) + q2) + q3, h = silu(gate) * up in
//    fp32, then the fx encoding of h per (row, group): the group's |max| and
//    sum of integers are exchanged between the warps holding the group's rows
//    (mbarriers with bounded waits), the bytes are staged in shared memory
//    and stored as 16-byte words.
// down kernel (TMA-fed for I % 256 == 0 and H % 256 == 0, else an
//  all-thread cp.async form): item = (expert, 256 output rows, pass of 8
//  tokens), tasks of 256 K elements, 16 warps of 16 output rows each over
//  the whole K, the same integer dot products against the fx h rows, fp32 y.
//
// Fragment layout of one m16n8k32 step: lane (r, c) holds for weight rows
// mma_row(r) and mma_row(r) + 8 of its 16-row tile one packed word each (its
// bytes are K slots 4c..4c+3 and 16+4c..16+4c+3), and the fx word of token r
// for the same 8 K elements; inside one MMA the K order is a permutation
// applied to both operands, which a dot product does not see.
//
// Every mbarrier wait is bounded: a waiting warp sleeps inside try_wait (a
// suspend-time hint, woken when the phase completes); after kWaitLimitNs of
// %globaltimer time (or kSpinLimit tries) it raises the CTA's abort flag and
// the device error word (phmoe_device_error) and all warps leave; the
// producer first waits (bounded) for its copies in flight.
#include <cuda.h>  // CUtensorMap (types only; the encoder is fetched from the driver at run time)
#include <string.h>

#include "common.cuh"
#include "pipeline.cuh"
#include "launch.h"

namespace phmoe {

// Error bits raised by the decode FFN kernels (read by phmoe_device_error;
// every writer ORs its bit in, so several conditions of one call all show):
//   1  a pipeline wait timed out and its CTA abandoned its work
//   2  an activation or SwiGLU value was beyond the fixed-point range (about
//      1e34) or not finite, and was clamped
__device__ int g_ffn_error;

namespace {

constexpr int kConsumers = 16;                  // consumer (MMA) warps
constexpr int kEpiWarps = 4;                    // gate/up epilogue warps (one per 16-row group)
constexpr int kRbProducers = 3;                // gate/up row-block kernel: weights+scales, x rows, constants
constexpr int kRbThreads = (kConsumers + kEpiWarps + kRbProducers) * 32;
constexpr int kDownThreads = 16 * 32;
constexpr int kTok = 8;                         // tokens per pass (the MMA N dimension)
constexpr uint32_t kSpinLimit = 1u << 24;       // try_wait polls before giving up
constexpr uint32_t kSuspendNs = 20000;          // try_wait suspend-time hint
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ void cp_async4(uint32_t saddr, const void* g) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(saddr), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t saddr, const void* g) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(saddr), "l"(g) : "memory");
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

// ---------------------------------------------------------------------------
// fixed-point encoding of activation rows
// ---------------------------------------------------------------------------
// One thread per 8-element word, G/8 threads per group. Rows 0..rows-1 of x,
// or (index != null) rows index[i] for i < *count (the rows a caller wants
// encoded out of a larger buffer). q [rows][K * 2 bytes], consts [rows][K/G].
template <typename XT, int G>
__global__ void __launch_bounds__(256)
fx_rows_kernel(const XT* __restrict__ x, int K, long long rows, const int32_t* __restrict__ index,
               const int32_t* __restrict__ count, uint8_t* __restrict__ q, int2* __restrict__ consts) {
  pdl_begin();
  constexpr int kTpg = G / 8;
  const int wpr = K / 8;
  const long long n = count ? (long long)*count : rows;
  const long long nw = n * wpr;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long w0 = (long long)blockIdx.x * blockDim.x; w0 < nw; w0 += stride) {
    const long long w = w0 + threadIdx.x;
    const bool ok = w < nw;
    long long row = 0;
    int wi = 0;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = 0.f;
    if (ok) {
      const long long i = w / wpr;
      wi = (int)(w - i * wpr);
      row = index ? (long long)__ldg(index + i) : i;
      const XT* p = x + row * K + (long long)wi * 8;
      if constexpr (std::is_same<XT, float>::value) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(p));
        const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      } else {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
        v[0] = bf16_lo_to_f32(u.x); v[1] = bf16_hi_to_f32(u.x); v[2] = bf16_lo_to_f32(u.y);
        v[3] = bf16_hi_to_f32(u.y); v[4] = bf16_lo_to_f32(u.z); v[5] = bf16_hi_to_f32(u.z);
        v[6] = bf16_lo_to_f32(u.w); v[7] = bf16_hi_to_f32(u.w);
      }
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
      *reinterpret_cast<uint4*>(q + ((size_t)row * wpr + wi) * 16) = fx_word(a);
      if ((threadIdx.x & (kTpg - 1)) == 0) {
        const int M = fx_magic(e);
        consts[(size_t)row * (K / G) + wi / kTpg] = make_int2(M - 8 * s, M);
      }
      if (bad || nonfinite) atomicOr(&g_ffn_error, 2);
    }
  }
}

// ---------------------------------------------------------------------------
// fragments and group dot products
// ---------------------------------------------------------------------------

// Packed weight words of one row and one group for this lane (G/32 words).
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

// fx words of one group for this lane (one per m16n8k32 step): .x .y = the
// high-byte B fragment, .z .w = the low-byte one.
template <int G>
struct FxB {
  uint4 s[G / 32];
};

template <int G>
__device__ __forceinline__ FxB<G> lds_fxb(const uint8_t* p) {
  FxB<G> b;
#pragma unroll
  for (int i = 0; i < G / 32; ++i) b.s[i] = reinterpret_cast<const uint4*>(p)[i];
  return b;
}

// One group's contribution for weight rows (r, r+8) of one tile and the 8
// tokens of a pass: acc += s_row * (sum((n - 8) * A) * 2^e). cc: the fx
// constants {C0, M} of tokens 2c (columns 0, 2) and 2c+1 (columns 1, 3).
template <int G>
__device__ __forceinline__ void fx_group_tile(const RowWords<G>& w0, const RowWords<G>& w8, const FxB<G>& b,
                                              const int4& cc, float s0, float s8, float (&acc)[4]) {
  int lo[4], hi[4];
#pragma unroll
  for (int s = 0; s < G / 32; ++s) {
    uint32_t a[4];
    nib_bytes(w0.w[s], a[0], a[2]);
    nib_bytes(w8.w[s], a[1], a[3]);
    if (s == 0) {
      mma_u8s8_16832_first(lo, a, b.s[s].z, b.s[s].w, cc.x, cc.z);
      mma_u8s8_16832_first(hi, a, b.s[s].x, b.s[s].y, 0, 0);
    } else {
      mma_u8s8_16832(lo, a, b.s[s].z, b.s[s].w);
      mma_u8s8_16832(hi, a, b.s[s].x, b.s[s].y);
    }
  }
  const float m0 = __int_as_float(cc.y), m1 = __int_as_float(cc.w);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float f = __fsub_rn(__int_as_float(hi[q] * 256 + lo[q]), (q & 1) ? m1 : m0);
    acc[q] = fmaf(q < 2 ? s0 : s8, f, acc[q]);
  }
}

// gate and up tiles of one group, sharing the B words and constants.
template <int G>
__device__ __forceinline__ void gateup_group_fx(const RowWords<G>& g0, const RowWords<G>& g8,
                                                const RowWords<G>& u0, const RowWords<G>& u8, const FxB<G>& b,
                                                const int4& cc, float sg0, float sg8, float su0, float su8,
                                                float (&acc_g)[4], float (&acc_u)[4]) {
  int gl[4], ul[4], gh[4], uh[4];
#pragma unroll
  for (int s = 0; s < G / 32; ++s) {
    uint32_t ag[4], au[4];
    nib_bytes(g0.w[s], ag[0], ag[2]);
    nib_bytes(g8.w[s], ag[1], ag[3]);
    nib_bytes(u0.w[s], au[0], au[2]);
    nib_bytes(u8.w[s], au[1], au[3]);
    if (s == 0) {
      mma_u8s8_16832_first(gl, ag, b.s[s].z, b.s[s].w, cc.x, cc.z);
      mma_u8s8_16832_first(gh, ag, b.s[s].x, b.s[s].y, 0, 0);
      mma_u8s8_16832_first(ul, au, b.s[s].z, b.s[s].w, cc.x, cc.z);
      mma_u8s8_16832_first(uh, au, b.s[s].x, b.s[s].y, 0, 0);
    } else {
      mma_u8s8_16832(gl, ag, b.s[s].z, b.s[s].w);
      mma_u8s8_16832(gh, ag, b.s[s].x, b.s[s].y);
      mma_u8s8_16832(ul, au, b.s[s].z, b.s[s].w);
      mma_u8s8_16832(uh, au, b.s[s].x, b.s[s].y);
    }
  }
  const float m0 = __int_as_float(cc.y), m1 = __int_as_float(cc.w);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float m = (q & 1) ? m1 : m0;
    acc_g[q] = fmaf(q < 2 ? sg0 : sg8, __fsub_rn(__int_as_float(gh[q] * 256 + gl[q]), m), acc_g[q]);
    acc_u[q] = fmaf(q < 2 ? su0 : su8, __fsub_rn(__int_as_float(uh[q] * 256 + ul[q]), m), acc_u[q]);
  }
}


// ---------------------------------------------------------------------------
// work items
// ---------------------------------------------------------------------------

// Per active slot s: expert id, first row, row count, and the prefix
// table[s] of items before slot s (an expert with n rows has
// tiles * ceil(n / TB) items). Every CTA builds the same copy in shared memory.
struct Meta {
  int* e;
  int* row0;
  int* n;
  int* table;  // [na + 1]
};

template <int TB = kTok>  // tokens per item
__device__ int build_meta(const int32_t* __restrict__ offsets, const int32_t* __restrict__ active, int E, int tiles,
                          Meta m) {
  // active[0..E] and offsets[0..E] are loaded side by side (one round trip
  // to memory instead of three dependent ones) into table and n, then
  // reordered by active slot in shared memory.
  for (int i = threadIdx.x; i <= E; i += blockDim.x) {
    m.table[i] = __ldg(active + i);
    m.n[i] = __ldg(offsets + i);
  }
  __syncthreads();
  const int na = m.table[0];
  constexpr int kPer = 4;  // slots per thread held in registers across the barrier
  int nreg[kPer];
  if (na <= kPer * (int)blockDim.x) {
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int s = threadIdx.x + i * blockDim.x;
      if (s < na) {
        const int e = m.table[1 + s];
        const int r0 = m.n[e];
        m.e[s] = e;
        m.row0[s] = r0;
        nreg[i] = m.n[e + 1] - r0;
      }
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int s = threadIdx.x + i * blockDim.x;
      if (s < na) m.n[s] = nreg[i];
    }
  } else {  // more active experts than kPer per thread: reload from global memory
    __syncthreads();
    for (int s = threadIdx.x; s < na; s += blockDim.x) {
      const int e = __ldg(active + 1 + s);
      const int r0 = __ldg(offsets + e);
      m.e[s] = e;
      m.row0[s] = r0;
      m.n[s] = __ldg(offsets + e + 1) - r0;
    }
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

// Weight row (within an 8-row block) of MMA row r of a lane's tile. A lane
// (r, c) loads 8 bytes of rows r and r + 8 at K byte 8c (+ 32 per group); in
// the 128-byte swizzle rows r and r ^ 1 at K halves c >> 1 = 0 and 1 share a
// 16-byte bank slot, so with rows in order each half-warp (MMA rows 0-3,
// 4-7) took two passes. Rows 0, 2, 4, 6 for MMA rows 0-3 and 1, 3, 5, 7 for
// 4-7 give every lane of a half-warp its own slot. The dot products do not
// depend on which MMA row holds a weight row; the scales, the h slot and
// the output row follow the same map.
__device__ __forceinline__ int mma_row(int r) { return 2 * (r & 3) + (r >> 2); }

// Byte offset of (row R of a `rows`-row box of 128-byte K-chunks, byte kb of
// the task's K slice) as TMA writes it with the 128-byte swizzle.
__device__ __forceinline__ int swz_off_rows(int R, int kb, int rows) {
  const int c0 = kb & 127;
  return ((kb >> 7) * rows + R) * 128 + ((((c0 >> 4) ^ (R & 7)) << 4) | (c0 & 15));
}

// ---------------------------------------------------------------------------
// gate/up epilogue: SwiGLU output -> fx rows
// ---------------------------------------------------------------------------
// Run by the four warps (rg = 0..3) that hold an item's 64 I rows after the
// K sum: lane (r, c) of warp rg holds for token columns tb + 2c + (q & 1) the
// I rows tile * 64 + rg * 16 + r (+ 8 for q >= 2), i.e. element r of words
// 2 rg and 2 rg + 1 of the item's 8 words. With G = 64 the item is one group
// (all four warps), with G = 32 two (warps 0-1 and 2-3). One buffer per item
// parity holds the exchange of per-warp maxima and integer sums and the byte
// staging of the item's rows.
template <int TB>
struct EpiBuf {
  float xm[4][TB];
  int xs[4][TB];
  uint8_t hs[TB][128];
};

// Per-warp |max| of token columns tb + 2c, tb + 2c + 1 into xm.
template <int TB>
__device__ __forceinline__ void epi_block_max(EpiBuf<TB>* eb, int rg, int lane, int tb, const float (&hv)[4]) {
  const int r = lane >> 2, c = lane & 3;
  float m0 = fmaxf(fabsf(hv[0]), fabsf(hv[2])), m1 = fmaxf(fabsf(hv[1]), fabsf(hv[3]));
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, off));
    m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, off));
  }
  if (r == 0) {
    eb->xm[rg][tb + 2 * c] = m0;
    eb->xm[rg][tb + 2 * c + 1] = m1;
  }
}

// After the max exchange: the group exponents of this lane's two token
// columns (e[]), the integers of its four values, the per-warp integer sums
// into xs and the bytes into the staging rows.
template <int G, int TB>
__device__ __forceinline__ void epi_block_encode(EpiBuf<TB>* eb, int rg, int lane, int tb, const float (&hv)[4],
                                                 bool any_valid, int (&e)[2]) {
  const int r = lane >> 2, c = lane & 3;
  const int w0 = (G == 64) ? 0 : (rg & 2), nw = (G == 64) ? 4 : 2;  // warps holding this group's rows
  float M0 = 0.f, M1 = 0.f;
  for (int w = w0; w < w0 + nw; ++w) {
    M0 = fmaxf(M0, eb->xm[w][tb + 2 * c]);
    M1 = fmaxf(M1, eb->xm[w][tb + 2 * c + 1]);
  }
  bool bad0, bad1;
  e[0] = fx_exponent<G>(M0, bad0);
  e[1] = fx_exponent<G>(M1, bad1);
  int a[4];
  a[0] = fx_encode<G>(hv[0], e[0]);
  a[1] = fx_encode<G>(hv[1], e[1]);
  a[2] = fx_encode<G>(hv[2], e[0]);
  a[3] = fx_encode<G>(hv[3], e[1]);
  int s0 = a[0] + a[2], s1 = a[1] + a[3];
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    s0 += __shfl_xor_sync(0xffffffffu, s0, off);
    s1 += __shfl_xor_sync(0xffffffffu, s1, off);
  }
  if (r == 0) {
    eb->xs[rg][tb + 2 * c] = s0;
    eb->xs[rg][tb + 2 * c + 1] = s1;
  }
  const int slot = fx_slot(mma_row(r));  // this lane holds I rows rg*16 + mma_row(r) (+ 8)
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint8_t* p = &eb->hs[tb + 2 * c + (q & 1)][(2 * rg + (q >> 1)) * 16 + slot];
    p[0] = (uint8_t)(((a[q] + 128) >> 8) & 255);
    p[8] = (uint8_t)(a[q] & 255);
  }
  if ((bad0 || bad1) && any_valid) atomicOr(&g_ffn_error, 2);
}

// After the sum exchange: the group constants (one writer lane per token
// column and group) and the 16-byte word stores of the 8 staged rows of
// block tb. Rows at or beyond n (the expert's row count) are not stored.
template <int G, int TB>
__device__ __forceinline__ void epi_block_store(EpiBuf<TB>* eb, int rg, int lane, int tb, const int (&e)[2],
                                                int tile, int prow0, int n, int row0, int I,
                                                uint8_t* __restrict__ hq, int2* __restrict__ hc) {
  const int r = lane >> 2, c = lane & 3;
  const bool writer = (G == 64) ? rg == 0 : (rg & 1) == 0;
  if (writer && r == 0) {
    const int w0 = (G == 64) ? 0 : (rg & 2), nw = (G == 64) ? 4 : 2;
    const int grp = (G == 64) ? tile : 2 * tile + (rg >> 1);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int t = tb + 2 * c + j;
      const int rr = prow0 + t;
      if (rr < n) {
        int S = 0;
        for (int w = w0; w < w0 + nw; ++w) S += eb->xs[w][t];
        const int M = fx_magic(e[j]);
        hc[(size_t)(row0 + rr) * (I / G) + grp] = make_int2(M - 8 * S, M);
      }
    }
  }
  const int tid = rg * 32 + lane;  // the four warps store the block's 8 rows x 8 words
  if (tid < 64) {
    const int t = tb + (tid >> 3), w = tid & 7;
    const int rr = prow0 + t;
    if (rr < n)
      *reinterpret_cast<uint4*>(hq + (size_t)(row0 + rr) * I * 2 + (size_t)(tile * 8 + w) * 16) =
          *reinterpret_cast<const uint4*>(&eb->hs[t][w * 16]);
  }
}

// ---------------------------------------------------------------------------
// gate/up + SwiGLU, row-block form
// ---------------------------------------------------------------------------
constexpr int kRbRows = 64;   // gate rows per item (and as many up rows)
constexpr int kRbKc = 512;    // K elements per task

template <int S>
struct RbCtl {
  uint64_t full[S];
  uint64_t empty[S];
  uint64_t red_full[8];   // [buf][rg]: the four K-quarter warps have written their partials
  uint64_t red_empty[8];  // [buf][rg]: the epilogue warp has read them
  uint64_t epi[4];        // [buf][2]: the epilogue warps' max and sum exchanges
  int abort_flag;
};

template <int G, int NS = 4>
struct RbCfg {
  static constexpr int kGpq = 128 / G;                       // groups per consumer warp per task
  static constexpr int kCg = kRbKc / G;                      // groups per task
  static constexpr int kBlock = 2 * kRbRows * 128;           // one 64-row box of 2 K-chunks (16 KB)
  static constexpr int kScaleRow = kRbKc / G * 2;            // bytes of scales per row per task
  static constexpr int kPairs = kRbKc / G / 2;
  static constexpr int kBStride = kRbKc * 2 + 16;            // fx row slice + pad
  static constexpr int kW = 0;                                // [gate box][up box]
  static constexpr int kS = 2 * kBlock;                       // [128 rows][kScaleRow]
  static constexpr int kB = kS + 2 * kRbRows * kScaleRow;     // [8 tokens][kBStride]
  static constexpr int kC = kB + kTok * kBStride;             // [kCg groups][8 tokens] int2
  static constexpr int kStage = (kC + kCg * kTok * 8 + 1023) / 1024 * 1024;
  static constexpr int kStages = NS;
  static constexpr int kRed = 4 * 4 * 32 * 8 * 4;             // [rg][kq][lane][8] floats
  static constexpr int kEpi = (int)sizeof(EpiBuf<kTok>);
  static constexpr size_t smem(int E) {
    return 1024 + (size_t)kStages * kStage + 2 * kRed + 2 * kEpi + sizeof(RbCtl<kStages>) +
           (size_t)(4 * E + 4) * 4;
  }
};

template <int G, int NS>
__global__ void __launch_bounds__(kRbThreads, 1)
ffn_gateup_rb_kernel(const __grid_constant__ CUtensorMap w13_map, int map3d, int box_chunks,
                     const __grid_constant__ CUtensorMap s_map, int s_tma, const uint8_t* __restrict__ xq,
                     const int2* __restrict__ xc, const int32_t* __restrict__ row_token,
                     const int32_t* __restrict__ offsets, const int32_t* __restrict__ active,
                     const uint16_t* __restrict__ w13_s, int H, int I, int E, uint8_t* __restrict__ hq,
                     int2* __restrict__ hc) {
  pdl_begin();
  using C = RbCfg<G, NS>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* red = reinterpret_cast<float*>(smem + S * C::kStage);  // [2][rg][kq][lane][8]
  EpiBuf<kTok>* epib = reinterpret_cast<EpiBuf<kTok>*>(smem + S * C::kStage + 2 * C::kRed);
  RbCtl<S>* ctl = reinterpret_cast<RbCtl<S>*>(smem + S * C::kStage + 2 * C::kRed + 2 * C::kEpi);
  int* mbase = reinterpret_cast<int*>(ctl + 1);
  const Meta meta{mbase, mbase + (E + 1), mbase + 2 * (E + 1), mbase + 3 * (E + 1)};
  volatile int* abort_flag = &ctl->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = I / kRbRows;
  const int NG = H / G;
  const int nkc = (H + kRbKc - 1) / kRbKc;
  const int na = active[0];

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      // expect_tx arrivals of the weight and x producers + one cp.async
      // arrival per lane of the constants producer
      mbar_init(smem_u32(&ctl->full[s]), 2 + 32);
      mbar_init(smem_u32(&ctl->empty[s]), kConsumers);
    }
    for (int i = 0; i < 8; ++i) {
      mbar_init(smem_u32(&ctl->red_full[i]), 4);
      mbar_init(smem_u32(&ctl->red_empty[i]), 1);
    }
    for (int i = 0; i < 4; ++i) mbar_init(smem_u32(&ctl->epi[i]), kEpiWarps);
    ctl->abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  const int total = build_meta(offsets, active, E, tiles, meta);  // its barriers publish the init too
  int q0, q1;
  cta_range(total, q0, q1);
  const int ntask = (q1 - q0) * nkc;
  if (ntask == 0) return;

  if (warp >= kConsumers && warp < kConsumers + kEpiWarps) {
    // ---------------- epilogue warps ----------------
    // Warp rg finishes the I rows rg*16..rg*16+15 of every item: the sum of
    // the four K-quarter partials in fixed order ((q0 + q1) + q2) + q3, the
    // SwiGLU, and with the other three the fx encoding of h.
    const int rg = warp - kConsumers;
    const int c = lane & 3;
    Cursor ci = cursor_at(q0, na, tiles, meta);
    for (int it = 0; it < q1 - q0; ++it) {
      const int buf = it & 1, use = it >> 1;
      const int bi = buf * 4 + rg;
      if (!wait_phase(smem_u32(&ctl->red_full[bi]), use & 1, abort_flag)) return;
      const float* rb = red + (size_t)buf * (C::kRed / 4) + (size_t)rg * 4 * 32 * 8 + lane * 8;
      float gs[4], us[4];
      {
        const float4 a = reinterpret_cast<const float4*>(rb)[0], b = reinterpret_cast<const float4*>(rb)[1];
        gs[0] = a.x; gs[1] = a.y; gs[2] = a.z; gs[3] = a.w;
        us[0] = b.x; us[1] = b.y; us[2] = b.z; us[3] = b.w;
      }
#pragma unroll
      for (int w = 1; w < 4; ++w) {
        const float4 a = reinterpret_cast<const float4*>(rb + w * 32 * 8)[0];
        const float4 b = reinterpret_cast<const float4*>(rb + w * 32 * 8)[1];
        gs[0] += a.x; gs[1] += a.y; gs[2] += a.z; gs[3] += a.w;
        us[0] += b.x; us[1] += b.y; us[2] += b.z; us[3] += b.w;
      }
      warp_arrive(smem_u32(&ctl->red_empty[bi]), lane);
      const int n = meta.n[ci.slot], row0 = meta.row0[ci.slot];
      const int prow0 = ci.pass * kTok;
      float hv[4];
      bool any = false;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const bool ok = prow0 + 2 * c + (q & 1) < n;
        hv[q] = ok ? silu_fast(gs[q]) * us[q] : 0.f;
        any |= ok;
      }
      EpiBuf<kTok>* eb = epib + buf;
      epi_block_max<kTok>(eb, rg, lane, 0, hv);
      warp_arrive(smem_u32(&ctl->epi[buf * 2]), lane);
      if (!wait_phase(smem_u32(&ctl->epi[buf * 2]), use & 1, abort_flag)) return;
      int e[2];
      epi_block_encode<G, kTok>(eb, rg, lane, 0, hv, any, e);
      warp_arrive(smem_u32(&ctl->epi[buf * 2 + 1]), lane);
      if (!wait_phase(smem_u32(&ctl->epi[buf * 2 + 1]), use & 1, abort_flag)) return;
      epi_block_store<G, kTok>(eb, rg, lane, 0, e, ci.tile, prow0, n, row0, I, hq, hc);
      cursor_next(ci, tiles, 1, meta);
    }
    return;
  }

  if (warp >= kConsumers + kEpiWarps) {
    // ---------------- producer warps ----------------
    // Issuing a copy waits behind the consumers' shared-memory loads (about
    // 150 cycles per TMA or bulk instruction at full load), so the copies of
    // a task are split over three warps that issue side by side: role 0 the
    // weight and scale boxes, role 1 the fx rows of x, role 2 the fx
    // constants (and the scales when they go by 4-byte async copies).
    const int role = warp - kConsumers - kEpiWarps;
    Cursor cu = cursor_at(q0, na, tiles, meta);
    auto token = [&](const Cursor& k) -> int {  // lane holds the token id of pass row lane % 8
      const int rr = k.pass * kTok + (lane & (kTok - 1));
      return rr < meta.n[k.slot] ? __ldg(row_token + meta.row0[k.slot] + rr) : -1;
    };
    int tok = role != 0 ? token(cu) : -1;
    int issued = 0;
    for (int t = 0; t < ntask; ++t) {
      const int s = t % S;
      if (t >= S && !wait_phase(smem_u32(&ctl->empty[s]), (t / S - 1) & 1, abort_flag)) break;
      Cursor nx = cu;
      cursor_next(nx, tiles, nkc, meta);
      const int tok_next = (role != 0 && t + 1 < ntask && nx.kc == 0) ? token(nx) : tok;
      const int k0 = cu.kc * kRbKc;
      const int kel = min(kRbKc, H - k0);
      const int nt = min(kTok, meta.n[cu.slot] - cu.pass * kTok);
      const uint32_t full = smem_u32(&ctl->full[s]);
      uint8_t* st = smem + s * C::kStage;
      const int grow = meta.e[cu.slot] * 2 * I + cu.tile * kRbRows;  // first gate row; up rows are I further
      if (role == 0) {
        if (lane == 0)
          mbar_arrive_expect_tx(full, 2u * (uint32_t)(box_chunks * kRbRows * 128) +
                                          (s_tma ? 2u * kRbRows * C::kScaleRow : 0u));
        __syncwarp();
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
        // scales: 64 gate rows then 64 up rows, kel/G groups each (two TMA
        // boxes when the scale rows are 16-byte aligned; role 2 otherwise)
        if (s_tma && (lane == 2 || lane == 3))
          tma_load_2d(smem_u32(st + C::kS + (lane - 2) * kRbRows * C::kScaleRow), &s_map, k0 / G,
                      grow + (lane - 2) * I, full);
      } else if (role == 1) {
        if (lane == 0) mbar_arrive_expect_tx(full, (uint32_t)(nt * kel * 2));
        __syncwarp();
        if (lane < nt)  // lane n < 8 holds the token id of pass row n
          bulk_g2s(smem_u32(st + C::kB + lane * C::kBStride), xq + (size_t)tok * H * 2 + (size_t)k0 * 2, kel * 2,
                   full);
      } else {
        // fx constants of the task's groups, transposed to [group][token]
        // (lane L copies for pass row L % 8, whose token id it holds)
        for (int q = lane; q < C::kCg * kTok; q += 32) {
          const int tt = q & (kTok - 1), j = q >> 3;
          if (tt < nt && j * G < kel)
            cp_async8(smem_u32(st + C::kC + (j * kTok + tt) * 8), xc + (size_t)tok * NG + k0 / G + j);
        }
        if (!s_tma) {  // scales as pairs of groups by 4-byte async copies
          for (int q = lane; q < 2 * kRbRows * C::kPairs; q += 32) {
            const int rr = q / C::kPairs, pp = q - rr * C::kPairs;
            if (pp * 2 * G < kel) {
              const size_t srow = (size_t)grow + (rr >= kRbRows ? I : 0) + (rr & (kRbRows - 1));
              cp_async4(smem_u32(st + C::kS + rr * C::kScaleRow + pp * 4), w13_s + srow * NG + k0 / G + 2 * pp);
            }
          }
        }
        cp_async_arrive_noinc(full);
      }
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
  const int R0 = rg * 16 + mma_row(r);
  int o0[kGpq], o8[kGpq], ob[kGpq];
#pragma unroll
  for (int j = 0; j < kGpq; ++j) {
    const int g = kq * kGpq + j;  // group within the task
    const int kb = (G == 64) ? g * 32 + 8 * c : g * 16 + 4 * c;
    o0[j] = C::kW + swz_off_rows(R0, kb, kRbRows);
    o8[j] = C::kW + swz_off_rows(R0 + 8, kb, kRbRows);
    ob[j] = C::kB + r * C::kBStride + g * G * 2 + (G == 64 ? 32 : 16) * c;
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
      const int g = kq * kGpq + j;
      if (g < ngt) {
        const RowWords<G> ag0 = lds_row<G>(st + o0[j]);
        const RowWords<G> ag8 = lds_row<G>(st + o8[j]);
        const RowWords<G> au0 = lds_row<G>(st + o0[j] + C::kBlock);
        const RowWords<G> au8 = lds_row<G>(st + o8[j] + C::kBlock);
        const int p = j >> 1;
        const bool hi = j & 1;
        const float fsg0 = hi ? __high2float(sg0[p]) : __low2float(sg0[p]);
        const float fsg8 = hi ? __high2float(sg8[p]) : __low2float(sg8[p]);
        const float fsu0 = hi ? __high2float(su0[p]) : __low2float(su0[p]);
        const float fsu8 = hi ? __high2float(su8[p]) : __low2float(su8[p]);
        const FxB<G> b = lds_fxb<G>(st + ob[j]);
        const int4 cc = *reinterpret_cast<const int4*>(st + C::kC + (g * kTok + 2 * c) * 8);
        gateup_group_fx<G>(ag0, ag8, au0, au8, b, cc, fsg0, fsg8, fsu0, fsu8, acc_g, acc_u);
      }
    }
    warp_arrive(smem_u32(&ctl->empty[s]), lane);  // this warp is done with the stage
    if (cu.kc == nkc - 1) {  // hand this K quarter's partials to the epilogue warp
      const int buf = item & 1, use = item >> 1;
      const int bi = buf * 4 + rg;  // barrier index
      if (use > 0 && !wait_phase(smem_u32(&ctl->red_empty[bi]), (use - 1) & 1, abort_flag)) return;
      float4* dst = reinterpret_cast<float4*>(red + (size_t)buf * (C::kRed / 4) + ((size_t)(rg * 4 + kq) * 32 + lane) * 8);
      dst[0] = make_float4(acc_g[0], acc_g[1], acc_g[2], acc_g[3]);
      dst[1] = make_float4(acc_u[0], acc_u[1], acc_u[2], acc_u[3]);
      warp_arrive(smem_u32(&ctl->red_full[bi]), lane);
      ++item;
    }
    cursor_next(cu, tiles, nkc, meta);
  }
}

// ---------------------------------------------------------------------------
// down projection, TMA-fed form (I % 256 == 0, H % 256 == 0)
// ---------------------------------------------------------------------------
// Item = (expert, 256 output rows, pass of 8 tokens); task = one 256-element
// K chunk (one 128-byte chunk of every weight row, 32 KB). A producer warp
// copies per task one TMA box of weights (256 rows x 128 bytes, 128-byte
// swizzle), the fx h rows of the pass (one TMA box: 4 blocks of 64 elements
// x 8 rows, 128-byte swizzle), the rows' scale slices (8- or 16-byte async
// copies, one per weight row) and the fx constants (8-byte async copies into
// [group][token]). Consumer warp w owns output rows 16w..16w+15 and every
// group of the task, so all 16 warps do equal work for any I that is a
// multiple of 256, and each warp's accumulators hold its rows' whole K: the
// item ends with a plain store, no cross-warp sum.
constexpr int kDnRows = 256;
constexpr int kDnKc = 256;
constexpr int kDnThreads = (kConsumers + 2) * 32;  // 16 consumer + 2 producer warps

template <int S>
struct DnCtl {
  uint64_t full[S];
  uint64_t empty[S];
  int abort_flag;
};

template <int G, int NS>
struct DnCfg {
  static constexpr int kGt = kDnKc / G;                // groups per task
  static constexpr int kW = 0;                         // [256 rows][128 B]
  static constexpr int kS = kDnRows * 128;             // [256 rows][kGt] fp16 scales
  static constexpr int kB = kS + kDnRows * kGt * 2;    // [4 blocks of 64][8 rows][128 B]
  static constexpr int kPlane = (kDnKc / 64) * kTok * 128;
  static constexpr int kC = kB + kPlane;               // [kGt groups][8 tokens] int2
  // stages start on 1024-byte boundaries: the 128-byte swizzle of the TMA
  // boxes (weights, h) is a function of the shared-memory address bits 7-9
  static constexpr int kStage = (kC + kGt * kTok * 8 + 1023) / 1024 * 1024;
  static constexpr int kStages = NS;
  static constexpr size_t smem(int E) {
    return 1024 + (size_t)kStages * kStage + sizeof(DnCtl<kStages>) + (size_t)(4 * E + 4) * 4;
  }
  static_assert(kS % 1024 == 0 && kB % 1024 == 0, "TMA destinations must keep the swizzle phase");
};

// fx words of group g (within a task) for token row r from the h box laid
// out [64-element block][8 rows][128 B] with 128-byte swizzle.
template <int G>
__device__ __forceinline__ FxB<G> lds_fxb_swz(const uint8_t* plane, int g, int r, int c) {
  FxB<G> b;
  if constexpr (G == 64) {
    const uint8_t* row = plane + g * (kTok * 128) + r * 128;
    b.s[0] = *reinterpret_cast<const uint4*>(row + (((2 * c) ^ (r & 7)) << 4));
    b.s[1] = *reinterpret_cast<const uint4*>(row + (((2 * c + 1) ^ (r & 7)) << 4));
  } else {
    const uint8_t* row = plane + (g >> 1) * (kTok * 128) + r * 128;
    b.s[0] = *reinterpret_cast<const uint4*>(row + ((((g & 1) * 4 + c) ^ (r & 7)) << 4));
  }
  return b;
}

// s_vec: the scale slice of a row for one task (kGt halves: 8 bytes for
// G = 64, 16 for G = 32) is copied with one async copy when w2_s and the
// scale rows allow it, else as 4-byte pairs.
template <int G, int NS>
__global__ void __launch_bounds__(kDnThreads, 1)
ffn_down_tma_kernel(const __grid_constant__ CUtensorMap w_map, const __grid_constant__ CUtensorMap h_map,
                    int s_vec, const int2* __restrict__ hc, int R, const int32_t* __restrict__ offsets,
                    const int32_t* __restrict__ active, const uint16_t* __restrict__ w2_s, int H, int I, int E,
                    float* __restrict__ y, const __grid_constant__ RowScatter scat) {
  // No wait here: the item table comes from the dispatch, which ran before
  // the gate/up kernel (see pdl_wait), and the weights and scales do not
  // change; the producers wait for the gate/up kernel only before they copy
  // its h rows.
  using C = DnCfg<G, NS>;
  constexpr int S = C::kStages;
  constexpr int kGt = C::kGt;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  DnCtl<S>* ctl = reinterpret_cast<DnCtl<S>*>(smem + S * C::kStage);
  int* mbase = reinterpret_cast<int*>(ctl + 1);
  const Meta meta{mbase, mbase + (E + 1), mbase + 2 * (E + 1), mbase + 3 * (E + 1)};
  volatile int* abort_flag = &ctl->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = H / kDnRows;
  const int NG = I / G;
  const int nkc = I / kDnKc;
  const int na = active[0];

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&ctl->full[s]), 1 + 32);  // TMA warp's expect_tx + one cp.async arrival per lane
      mbar_init(smem_u32(&ctl->empty[s]), kConsumers);
    }
    ctl->abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  const int total = build_meta(offsets, active, E, tiles, meta);
  int q0, q1;
  cta_range(total, q0, q1);
  const int ntask = (q1 - q0) * nkc;
  if (ntask == 0) return;

  if (warp >= kConsumers) {
    // ---------------- producer warps ----------------
    // role 0: the weight and h boxes (TMA); role 1: the scale slices and the
    // fx constants (async copies). Two warps issue side by side: each copy
    // instruction waits behind the consumers' shared-memory loads. The first
    // stages' weights and scales go out before griddepcontrol.wait, while
    // the gate/up kernel finishes; h and its constants after it.
    const int role = warp - kConsumers;
    const uint16_t* s_all = w2_s;
    auto issue_static = [&](const Cursor& c, int t) {
      const uint32_t full = smem_u32(&ctl->full[t % S]);
      uint8_t* st = smem + (t % S) * C::kStage;
      const int wrow = meta.e[c.slot] * H + c.tile * kDnRows;
      if (role == 0) {
        if (lane == 0) {
          mbar_arrive_expect_tx(full, (uint32_t)(kDnRows * 128 + C::kPlane));  // weights now, h later
          tma_load_3d(smem_u32(st + C::kW), &w_map, 0, wrow, c.kc, full);
        }
      } else {
        const uint16_t* sbase = s_all + (size_t)wrow * NG + c.kc * kGt;
        if (s_vec) {
#pragma unroll
          for (int rr = lane; rr < kDnRows; rr += 32) {
            const uint32_t dst = smem_u32(st + C::kS + rr * kGt * 2);
            if constexpr (G == 64) cp_async8(dst, sbase + (size_t)rr * NG);
            else cp_async16(dst, sbase + (size_t)rr * NG);
          }
        } else {
          for (int q = lane; q < kDnRows * (kGt / 2); q += 32) {
            const int rr = q / (kGt / 2), pp = q - rr * (kGt / 2);
            cp_async4(smem_u32(st + C::kS + rr * kGt * 2 + pp * 4), sbase + (size_t)rr * NG + 2 * pp);
          }
        }
      }
    };
    auto issue_dynamic = [&](const Cursor& c, int t) {
      const uint32_t full = smem_u32(&ctl->full[t % S]);
      uint8_t* st = smem + (t % S) * C::kStage;
      const int hrow = meta.row0[c.slot] + c.pass * kTok;
      if (role == 0) {
        if (lane == 0) tma_load_3d(smem_u32(st + C::kB), &h_map, 0, hrow, c.kc * (kDnKc / 64), full);
      } else {
        for (int q = lane; q < kGt * kTok; q += 32) {  // fx constants, transposed to [group][token]
          const int tt = q & (kTok - 1), j = q >> 3;
          if (hrow + tt < R)
            cp_async8(smem_u32(st + C::kC + (j * kTok + tt) * 8), hc + (size_t)(hrow + tt) * NG + c.kc * kGt + j);
        }
        cp_async_arrive_noinc(full);
      }
    };
    Cursor cu = cursor_at(q0, na, tiles, meta);
    {
      Cursor c = cu;
      for (int t = 0; t < min(S, ntask); ++t) {
        issue_static(c, t);
        cursor_next(c, tiles, nkc, meta);
      }
    }
    pdl_wait();  // the gate/up kernel's h rows and constants are complete and visible
    if (role == 0) pdl_trigger();
    int issued = 0;
    for (int t = 0; t < ntask; ++t) {
      if (t >= S) {
        if (!wait_phase(smem_u32(&ctl->empty[t % S]), (t / S - 1) & 1, abort_flag)) break;
        issue_static(cu, t);
      }
      issue_dynamic(cu, t);
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
  const int r = lane >> 2, c = lane & 3;
  const int lr0 = warp * 16 + mma_row(r);
  const int a_off = (G == 64) ? 8 * c : 4 * c;
  // row lr0 + 8 has the swizzle phase of row lr0 and lies 8 x 128 bytes further
  int ow0[kGt];
#pragma unroll
  for (int g = 0; g < kGt; ++g) ow0[g] = C::kW + swz_off_rows(lr0, g * (G / 2) + a_off, kDnRows);
  Cursor cu = cursor_at(q0, na, tiles, meta);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int t = 0; t < ntask; ++t) {
    const int s = t % S;
    if (cu.kc == 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[q] = 0.f;
    }
    if (!wait_phase(smem_u32(&ctl->full[s]), (t / S) & 1, abort_flag)) return;
    const uint8_t* st = smem + s * C::kStage;
    const __half* sc = reinterpret_cast<const __half*>(st + C::kS);
#pragma unroll
    for (int g = 0; g < kGt; ++g) {
      const RowWords<G> a0 = lds_row<G>(st + ow0[g]);
      const RowWords<G> a8 = lds_row<G>(st + ow0[g] + 8 * 128);
      const float s0 = __half2float(sc[lr0 * kGt + g]), s8 = __half2float(sc[(lr0 + 8) * kGt + g]);
      const FxB<G> b = lds_fxb_swz<G>(st + C::kB, g, r, c);
      const int4 cc = *reinterpret_cast<const int4*>(st + C::kC + (g * kTok + 2 * c) * 8);
      fx_group_tile<G>(a0, a8, b, cc, s0, s8, acc);
    }
    warp_arrive(smem_u32(&ctl->empty[s]), lane);
    if (cu.kc == nkc - 1) {
      const int n = meta.n[cu.slot], row0 = meta.row0[cu.slot];
      float* dst[2];  // this lane's two output rows (token columns 2c, 2c + 1)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int rr = cu.pass * kTok + 2 * c + j;
        dst[j] = nullptr;
        if (rr < n) {
          const int row = row0 + rr;
          if (scat.src == nullptr) {
            dst[j] = y + (size_t)row * H;
          } else {
            const int s = __ldg(scat.src + row), d = __ldg(scat.row + row);
            if (s >= 0 && s < scat.nbase && d >= 0 && d < scat.cap) dst[j] = scat.base[s] + (size_t)d * H;
          }
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int hr = cu.tile * kDnRows + lr0 + (q >= 2 ? 8 : 0);
        if (dst[q & 1] != nullptr) dst[q & 1][hr] = acc[q];
      }
    }
    cursor_next(cu, tiles, nkc, meta);
  }
}

// ---------------------------------------------------------------------------
// down projection, all-thread form (I % 256 != 0)
// ---------------------------------------------------------------------------
// 16 warps copy each task (128 rows x up to 512 K) with cp.async into padded
// rows and compute it between two CTA barriers; warp w owns rows 16(w%8)..+15
// and every other group of the task (w/8).
template <int G>
struct DownCfg {
  static constexpr int kStages = 3;
  static constexpr int kRows = 128;
  static constexpr int kKch = 512;
  static constexpr int kWch = kKch / 32;
  static constexpr int kPairs = kKch / G / 2;
  static constexpr int kCg = kKch / G;
  static constexpr int kWStride = kKch / 2 + (G == 64 ? 32 : 16);
  static constexpr int kScaleRow = kKch / G * 2;
  static constexpr int kBRowBytes = kKch * 2;  // fx row slice
  static constexpr int kBch = kBRowBytes / 16;
  static constexpr int kBStride = kBRowBytes + 16;
  static constexpr int kW = 0;
  static constexpr int kS = kRows * kWStride;
  static constexpr int kB = kS + kRows * kScaleRow;             // [kTok][kBStride]
  static constexpr int kC = kB + kTok * kBStride;               // [kCg][kTok] int2
  static constexpr int kStage = (kC + kCg * kTok * 8 + 127) / 128 * 128;
  static constexpr int kRed = 8 * 4 * 32 * 4;
};

template <int G>
__global__ void __launch_bounds__(kDownThreads, 1)
ffn_down_kernel(const uint8_t* __restrict__ hq, const int2* __restrict__ hc, const int32_t* __restrict__ offsets,
                const int32_t* __restrict__ active, const uint8_t* __restrict__ w2_q,
                const uint16_t* __restrict__ w2_s, int H, int I, int E, float* __restrict__ y) {
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

  const int total = build_meta(offsets, active, E, tiles, meta);
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
    // fx h rows of the pass and their constants, this K-chunk
    const int row_p = meta.row0[cu.slot] + cu.pass * kTok;
    const int nt = min(kTok, meta.n[cu.slot] - cu.pass * kTok);
#pragma unroll
    for (int q = threadIdx.x; q < kTok * C::kBch; q += kDownThreads) {
      const int n = q / C::kBch, cc = q % C::kBch;
      if (n < nt && cc * 8 < kel)
        cp_async16(smem_u32(st + C::kB + n * C::kBStride + cc * 16),
                   hq + (size_t)(row_p + n) * I * 2 + (size_t)k0 * 2 + cc * 16);
    }
    for (int q = threadIdx.x; q < C::kCg * kTok; q += kDownThreads) {
      const int tt = q & (kTok - 1), j = q >> 3;
      if (tt < nt && j * G < kel)
        cp_async8(smem_u32(st + C::kC + (j * kTok + tt) * 8), hc + (size_t)(row_p + tt) * NG + k0 / G + j);
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
      const FxB<G> b = lds_fxb<G>(st + C::kB + r * C::kBStride + g * G * 2 + b_off);
      const int4 cc = *reinterpret_cast<const int4*>(st + C::kC + (g * kTok + 2 * c) * 8);
      fx_group_tile<G>(a0, a8, b, cc, __half2float(sc[lr0 * kScH + g]), __half2float(sc[(lr0 + 8) * kScH + g]),
                       acc);
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
// launchers
// ---------------------------------------------------------------------------

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

// Tensor map over w13_q viewed as [rows = E*2I][K bytes = H/2], for boxes of
// `box_rows` rows x `box_chunks` 128-byte K-chunks with 128-byte swizzle.
// First choice: a 3-D view (128 B, rows, K-chunks) so one copy moves the
// whole box; if the driver rejects it, a 2-D view copied one 128-byte chunk
// at a time (same shared-memory layout). Returns 0 (2-D), 1 (3-D) or -1.
int make_w13_map(CUtensorMap* map, const uint8_t* w13_q, long long rows, int H, int box_chunks, int box_rows) {
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

// Tensor map over the fp16 scales [rows][H/G] for boxes of one task's
// groups x `box_rows` rows; false when the rows are not 16-byte aligned.
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

template <int G>
int launch_gateup(const uint8_t* xq, const int2* xc, const int32_t* row_token, const int32_t* offsets,
                  const int32_t* active, const uint8_t* w13_q, const uint16_t* w13_s, int H, int I, int E,
                  uint8_t* hq, int2* hc, int grid, cudaStream_t st) {
  const int rows = kRbRows;
  const int kc = kRbKc;
  const bool rb4 = RbCfg<G, 4>::smem(E) <= kMaxSmem;  // four stages where they fit, else three
  const size_t smem = rb4 ? RbCfg<G, 4>::smem(E) : RbCfg<G, 3>::smem(E);
  if (smem > kMaxSmem) return PHMOE_ERR_UNSUPPORTED;
  const int box_chunks = std::min(H, kc) / 256;
  alignas(64) CUtensorMap map, smap;
  const int mode = make_w13_map(&map, w13_q, (long long)E * 2 * I, H, box_chunks, rows);
  if (mode < 0) return PHMOE_ERR_CUDA;
  const int s_tma = make_scale_map(&smap, w13_s, (long long)E * 2 * I, H, G, kc, rows) ? 1 : 0;
  if (!s_tma) memset(&smap, 0, sizeof(smap));
  auto k = rb4 ? ffn_gateup_rb_kernel<G, 4> : ffn_gateup_rb_kernel<G, 3>;
  set_smem(k, smem);
  launch_pdl(k, dim3(grid), dim3(kRbThreads), smem, st, map, mode, box_chunks, smap, s_tma, xq, xc, row_token,
             offsets, active, w13_s, H, I, E, hq, hc);
  return PHMOE_OK;
}

// TMA-fed down projection; returns false (nothing launched) when the shape
// or the tensor maps do not allow it.
template <int G>
bool launch_down_tma(const uint8_t* hq, const int2* hc, long long R, const int32_t* offsets, const int32_t* active,
                     const uint8_t* w2_q, const uint16_t* w2_s, int H, int I, int E, float* y, int grid,
                     cudaStream_t st, const RowScatter& sc) {
  if (I % kDnKc || H % kDnRows || R <= 0 || R > (1LL << 30)) return false;
  const bool five = DnCfg<G, 5>::smem(E) <= kMaxSmem;  // five stages where they fit, else four
  const size_t smem = five ? DnCfg<G, 5>::smem(E) : DnCfg<G, 4>::smem(E);
  if (smem > kMaxSmem) return false;
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  alignas(64) CUtensorMap wm, hm;
  const cuuint32_t e3[3] = {1, 1, 1};
  {  // weights as [I/256 chunks][E*H rows][128 bytes]
    const cuuint64_t dims[3] = {128, (cuuint64_t)E * H, (cuuint64_t)(I / 256)};
    const cuuint64_t strides[2] = {(cuuint64_t)(I / 2), 128};
    const cuuint32_t box[3] = {128, (cuuint32_t)kDnRows, 1};
    if (enc(&wm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(w2_q), dims, strides, box, e3,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return false;
  }
  {  // fx h rows viewed as 16-bit elements: [I/64 blocks][R rows][64]
    const cuuint64_t dims[3] = {64, (cuuint64_t)R, (cuuint64_t)(I / 64)};
    const cuuint64_t strides[2] = {(cuuint64_t)I * 2, 128};
    const cuuint32_t box[3] = {64, (cuuint32_t)kTok, (cuuint32_t)(kDnKc / 64)};
    if (enc(&hm, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<uint8_t*>(hq), dims, strides, box, e3,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return false;
  }
  // one 8- (G = 64) or 16-byte (G = 32) copy per row's scale slice: the
  // slice starts at (row * I/G + k0/G) * 2 bytes, a multiple of the copy size
  // when w2_s is 16-byte aligned (I % 256 == 0 makes I/G a multiple of 4 or 8)
  const int s_vec = (reinterpret_cast<uintptr_t>(w2_s) & 15) == 0 ? 1 : 0;
  if (five) {
    auto k = ffn_down_tma_kernel<G, 5>;
    set_smem(k, smem);
    launch_pdl(k, dim3(grid), dim3(kDnThreads), smem, st, wm, hm, s_vec, hc, (int)R, offsets, active, w2_s, H, I,
               E, y, sc);
  } else {
    auto k = ffn_down_tma_kernel<G, 4>;
    set_smem(k, smem);
    launch_pdl(k, dim3(grid), dim3(kDnThreads), smem, st, wm, hm, s_vec, hc, (int)R, offsets, active, w2_s, H, I,
               E, y, sc);
  }
  return true;
}

template <int G>
void launch_down(const uint8_t* hq, const int2* hc, const int32_t* offsets, const int32_t* active,
                 const uint8_t* w2_q, const uint16_t* w2_s, int H, int I, int E, float* y, int grid,
                 cudaStream_t st) {
  using C = DownCfg<G>;
  const size_t smem = (size_t)C::kStages * C::kStage + C::kRed + (size_t)(4 * E + 4) * 4;
  auto k = ffn_down_kernel<G>;
  set_smem(k, smem);
  launch_pdl(k, dim3(grid), dim3(kDownThreads), smem, st, hq, hc, offsets, active, w2_q, w2_s, H, I, E, y);
}

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

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

uint8_t* ffn_decode_xq(float* y) { return reinterpret_cast<uint8_t*>(y); }
int2* ffn_decode_xc(float* y, int T, int H) {
  return reinterpret_cast<int2*>(reinterpret_cast<uint8_t*>(y) + align256((size_t)T * H * 2));
}

size_t fx_rows_bytes(long long rows, int K, int G) {
  return align256((size_t)rows * K * 2) + (size_t)rows * (K / G) * 8;
}

int launch_fx_rows(const void* x, int x_dtype, long long rows, int K, int G, const int32_t* index,
                   const int32_t* count, uint8_t* q, int2* consts, cudaStream_t st) {
  if (rows <= 0) return PHMOE_OK;
  if ((G != 32 && G != 64) || K % G) return PHMOE_ERR_UNSUPPORTED;
  const long long words = rows * (K / 8);
  const long long want = (words + 255) / 256;
  const int grid = (int)std::min<long long>(want, 8LL * device_sm_count());
  const bool f32 = x_dtype == PHMOE_DTYPE_F32;
  if (G == 64) {
    if (f32)
      launch_pdl(fx_rows_kernel<float, 64>, dim3(grid), dim3(256), 0, st, static_cast<const float*>(x), K, rows,
                 index, count, q, consts);
    else
      launch_pdl(fx_rows_kernel<__nv_bfloat16, 64>, dim3(grid), dim3(256), 0, st,
                 static_cast<const __nv_bfloat16*>(x), K, rows, index, count, q, consts);
  } else {
    if (f32)
      launch_pdl(fx_rows_kernel<float, 32>, dim3(grid), dim3(256), 0, st, static_cast<const float*>(x), K, rows,
                 index, count, q, consts);
    else
      launch_pdl(fx_rows_kernel<__nv_bfloat16, 32>, dim3(grid), dim3(256), 0, st,
                 static_cast<const __nv_bfloat16*>(x), K, rows, index, count, q, consts);
  }
  note_launches(1);
  return PHMOE_OK;
}

int launch_ffn_decode(const void* x, int x_dtype, const int32_t* row_token,
                      const int32_t* offsets, const int32_t* active, const uint8_t* w13_q,
                      const uint16_t* w13_s, const uint8_t* w2_q, const uint16_t* w2_s, int T,
                      int H, int E, int top_k, int I, int G, float* h, float* y,
                      cudaStream_t st, cudaEvent_t mid_event, const int32_t* enc_index,
                      const int32_t* enc_count, bool x_encoded, const RowScatter* scatter, bool* scattered) {
  const long long R = (long long)T * top_k;
  if (R == 0) return PHMOE_OK;
  if (G != 32 && G != 64) return PHMOE_ERR_UNSUPPORTED;
  // fx rows of x in y's memory (the down kernel writes y only after gate/up
  // has read them), fx rows of h in h's
  uint8_t* xq = ffn_decode_xq(y);
  int2* xc = ffn_decode_xc(y, T, H);
  uint8_t* hq = reinterpret_cast<uint8_t*>(h);
  int2* hc = reinterpret_cast<int2*>(hq + align256((size_t)R * I * 2));
  if (!x_encoded)
    if (int s = launch_fx_rows(x, x_dtype, T, H, G, enc_index, enc_count, xq, xc, st)) return s;
  const int grid = device_sm_count();
  const int s = G == 64 ? launch_gateup<64>(xq, xc, row_token, offsets, active, w13_q, w13_s, H, I, E, hq, hc, grid, st)
                        : launch_gateup<32>(xq, xc, row_token, offsets, active, w13_q, w13_s, H, I, E, hq, hc, grid, st);
  if (s) return s;
  if (mid_event) cudaEventRecord(mid_event, st);
  RowScatter sc{};
  if (scatter != nullptr) sc = *scatter;
  const bool tma = G == 64 ? launch_down_tma<64>(hq, hc, R, offsets, active, w2_q, w2_s, H, I, E, y, grid, st, sc)
                           : launch_down_tma<32>(hq, hc, R, offsets, active, w2_q, w2_s, H, I, E, y, grid, st, sc);
  if (scattered != nullptr) *scattered = tma && sc.src != nullptr;
  if (!tma) {
    if (G == 64) launch_down<64>(hq, hc, offsets, active, w2_q, w2_s, H, I, E, y, grid, st);
    else launch_down<32>(hq, hc, offsets, active, w2_q, w2_s, H, I, E, y, grid, st);
  }
  note_launches(2);
  return PHMOE_OK;
}

}  // namespace phmoe
