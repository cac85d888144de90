// Grouped SwiGLU expert FFN, decode form (few tokens per expert).
//
// Reference: Qwen3MoeExperts.forward loop body (transformers 5.5.0
// models/qwen3_moe/modeling_qwen3_moe.py:245-247):
//   gate, up = linear(x_e, gate_up_proj[e]).chunk(2); h = silu(gate) * up;
//   y_e = linear(h, down_proj[e])
// on weights dequantised as (nibble - 8) * scale (gguf_loader.py:372-378).
//
// Design. At decode sizes the layer streams ~2.5 MB of packed weights per
// expert hit and does a few FMAs per weight: the bound is HBM. Both kernels
// are persistent (one 512-thread CTA per SM, a contiguous range of work items
// each) and run a multi-stage cp.async pipeline over "tasks" (a work item's
// K-chunk). A stage holds everything a task reads: the packed int4 weight
// rows, their fp16 scales and the K-chunk of the activation rows (B). While
// the 16 warps compute task t, tasks t+1.. are in flight from HBM/L2, so the
// compute loop issues no global loads. Rows are padded so that every
// fragment read is bank-conflict free (fp32 activations excepted).
//
// From shared memory each lane reads the int4 words of its A fragments and
// turns each 32-bit word (8 consecutive weights) into four bf16x2 pairs with
// one lop3 each (see the packed layout in phmoe.h); the pairs feed mma.sync
// m16n8k16 directly, with the 8 tokens of a pass as the N side. Dequantised
// weights are never written back to shared memory (bf16 would be 4x the int4
// bytes). In gate/up the unpacked values are 128 + nibble and the +136
// offset is removed after the MMA with one extra MMA per K step against an
// all-ones A (it yields sum_k x_k); the fp16 group scale multiplies the fp32
// partial of each group. Both steps are exact factorisations.
//
// Lane c of a quad holds K elements 16c..16c+15 of a 64-group (8c..8c+7 of a
// 32-group) for A and reads the same activations for B; inside one MMA the K
// order is a permutation applied to both operands, which a dot product does
// not see.
//
// Precision: bf16 activations enter the MMA exactly; fp32 activations and the
// intermediate h are split into bf16 hi + lo parts (two MMAs each), keeping
// ~16 significant bits.
//
// gate/up kernel: item = (expert, 16 intermediate rows, pass of 8 tokens) ->
//   32 weight rows (16 gate + 16 up); the 16 warps split each K-chunk and are
//   reduced through shared memory in warp order (deterministic); SwiGLU in
//   the epilogue, h stored as bf16 hi/lo planes.
// down kernel: item = (expert, 128 output rows, pass); warp w owns rows
//   16(w%8)..+15 and half of each K-chunk (w/8); the halves are added in a
//   fixed order.
// Items are ordered (expert, tile, pass) so the extra passes of an expert
// with more than 8 rows re-read weights that are still in L2.
#include "common.cuh"
#include "launch.h"

namespace phmoe {

namespace {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kTok = 8;  // tokens per pass (the MMA N dimension)

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(saddr), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t saddr, const void* g) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(saddr), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

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

// down partial of one group: acc += s * A.(B_hi + B_lo), A unpacked exactly.
template <int G>
__device__ __forceinline__ void down_group(const RowWords<G>& a0, const RowWords<G>& a8,
                                           const BWords<G>& b, float s0, float s8, float (&acc)[4]) {
  float t[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int w = 0; w < G / 32; ++w) {
    uint32_t p0[4], p8[4];
    unpack_word(a0.w[w], p0);
    unpack_word(a8.w[w], p8);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int s = 2 * w + h;
      const uint32_t a[4] = {p0[2 * h], p8[2 * h], p0[2 * h + 1], p8[2 * h + 1]};
      mma_bf16_16816(t, a, b.hi[2 * s], b.hi[2 * s + 1], t);
      mma_bf16_16816(t, a, b.lo[2 * s], b.lo[2 * s + 1], t);
    }
  }
  acc[0] = fmaf(s0, t[0], acc[0]);
  acc[1] = fmaf(s0, t[1], acc[1]);
  acc[2] = fmaf(s8, t[2], acc[2]);
  acc[3] = fmaf(s8, t[3], acc[3]);
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
      const int v = s < na ? ((m.n[s] + kTok - 1) / kTok) * tiles : 0;
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

__device__ __forceinline__ int passes_of(int n) { return (n + kTok - 1) / kTok; }

__device__ Cursor cursor_at(int q, int na, int tiles, const Meta& m) {
  int lo = 0, hi = na;  // table[lo] <= q < table[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (m.table[mid] <= q) lo = mid;
    else hi = mid;
  }
  Cursor c;
  c.slot = lo;
  c.passes = passes_of(m.n[lo]);
  const int local = q - m.table[lo];
  c.tile = local / c.passes;
  c.pass = local - c.tile * c.passes;
  c.kc = 0;
  return c;
}

__device__ __forceinline__ void cursor_next(Cursor& c, int tiles, int nkc, const Meta& m) {
  if (++c.kc < nkc) return;
  c.kc = 0;
  if (++c.pass < c.passes) return;
  c.pass = 0;
  if (++c.tile < tiles) return;
  c.tile = 0;
  ++c.slot;                          // may step one past the last slot: arrays hold E + 1 entries
  c.passes = passes_of(m.n[c.slot]);
}

__device__ __forceinline__ void cta_range(int total, int& q0, int& q1) {
  q0 = (int)((long long)total * blockIdx.x / gridDim.x);
  q1 = (int)((long long)total * (blockIdx.x + 1) / gridDim.x);
}

// ---------------------------------------------------------------------------
// gate/up + SwiGLU
// ---------------------------------------------------------------------------
// KCH = K elements per task: 2048 (3 stages) amortises the per-task barriers
// over twice the bytes; 1024 (5 stages, 3 for fp32) when 2048 does not fit.
template <int G, typename XT, int KCH>
struct GateUpCfg {
  static constexpr bool kF32 = std::is_same<XT, float>::value;
  static constexpr int kStages = KCH == 2048 ? 3 : (kF32 ? 3 : 5);
  static constexpr int kRows = 32;
  static constexpr int kKch = KCH;
  static constexpr int kWch = kKch / 32;                             // 16-byte weight chunks per row
  static constexpr int kPairs = kKch / G / 2;                        // 4-byte scale pairs per row
  static constexpr int kWStride = kKch / 2 + (G == 64 ? 32 : 16);    // conflict-free A reads
  static constexpr int kScaleRow = kKch / G * 2;
  static constexpr int kBRowBytes = kKch * (int)sizeof(XT);
  static constexpr int kBch = kBRowBytes / 16;                       // 16-byte B chunks per token
  static constexpr int kBPad = (G == 32 && !kF32) ? 64 : 16;         // conflict-free B reads
  static constexpr int kBStride = kBRowBytes + kBPad;
  static constexpr int kW = 0;
  static constexpr int kS = kRows * kWStride;
  static constexpr int kB = kS + kRows * kScaleRow;
  static constexpr int kStage = (kB + kTok * kBStride + 127) / 128 * 128;
  static constexpr int kRed = kWarps * 8 * 32 * 4;
};

template <int G, typename XT, int KCH>
__global__ void __launch_bounds__(kThreads, 1)
ffn_gateup_kernel(const XT* __restrict__ x, const int32_t* __restrict__ row_token,
                  const int32_t* __restrict__ offsets, const int32_t* __restrict__ active,
                  const uint8_t* __restrict__ w13_q, const uint16_t* __restrict__ w13_s, int H, int I,
                  int E, __nv_bfloat16* __restrict__ h_hi, __nv_bfloat16* __restrict__ h_lo) {
  using C = GateUpCfg<G, XT, KCH>;
  constexpr int S = C::kStages;
  extern __shared__ __align__(128) uint8_t smem[];
  float* red = reinterpret_cast<float*>(smem + S * C::kStage);  // [kWarps][8][32]
  int* mbase = reinterpret_cast<int*>(smem + S * C::kStage + C::kRed);
  const Meta meta{mbase, mbase + (E + 1), mbase + 2 * (E + 1), mbase + 3 * (E + 1)};
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, c = lane & 3;
  const int tiles = I / 16;
  const int NG = H / G;
  const int nkc = (H + C::kKch - 1) / C::kKch;
  const size_t row_bytes = (size_t)H / 2;
  const int na = active[0];

  const int total = build_meta(offsets, active, tiles, meta);
  int q0, q1;
  cta_range(total, q0, q1);
  const int ntask = (q1 - q0) * nkc;
  if (ntask == 0) return;

  // B-copy assignment of this thread: token bn, 16-byte chunks bc, bc+64, ...
  const int bn = threadIdx.x >> 6;
  const int bc = threadIdx.x & 63;
  auto token_of = [&](const Cursor& cu) -> int {
    const int rr = cu.pass * kTok + bn;
    return rr < meta.n[cu.slot] ? __ldg(row_token + meta.row0[cu.slot] + rr) : -1;
  };
  auto issue = [&](const Cursor& cu, int task, int tok) {
    uint8_t* st = smem + (task % S) * C::kStage;
    const int k0 = cu.kc * C::kKch;
    const int kel = min(C::kKch, H - k0);
    const size_t erow = (size_t)meta.e[cu.slot] * 2 * I;
    const int i0 = cu.tile * 16;
#pragma unroll
    for (int q = threadIdx.x; q < C::kRows * C::kWch; q += kThreads) {
      const int rr = q / C::kWch, cc = q % C::kWch;
      if (cc * 32 < kel) {
        const size_t grow = erow + (rr < 16 ? i0 + rr : I + i0 + rr - 16);
        cp_async16(smem_u32(st + C::kW + rr * C::kWStride + cc * 16), w13_q + grow * row_bytes + k0 / 2 + cc * 16);
      }
    }
#pragma unroll
    for (int q = threadIdx.x; q < C::kRows * C::kPairs; q += kThreads) {
      const int rr = q / C::kPairs, pp = q % C::kPairs;
      if (pp * 2 * G < kel) {
        const size_t grow = erow + (rr < 16 ? i0 + rr : I + i0 + rr - 16);
        cp_async4(smem_u32(st + C::kS + rr * C::kScaleRow + pp * 4), w13_s + grow * NG + k0 / G + 2 * pp);
      }
    }
    if (tok >= 0) {
      const uint8_t* src = reinterpret_cast<const uint8_t*>(x + (size_t)tok * H + k0);
      const int bch = kel * (int)sizeof(XT) / 16;
#pragma unroll
      for (int cc = bc; cc < C::kBch; cc += 64)
        if (cc < bch) cp_async16(smem_u32(st + C::kB + bn * C::kBStride + cc * 16), src + cc * 16);
    }
  };

  Cursor ci = cursor_at(q0, na, tiles, meta);  // next task to issue
  for (int s = 0; s < S - 1; ++s) {
    if (s < ntask) issue(ci, s, token_of(ci));
    cp_async_commit();
    cursor_next(ci, tiles, nkc, meta);
  }
  Cursor ct = ci;  // task S-1: its token id is loaded one iteration ahead
  int next_tok = (S - 1 < ntask) ? token_of(ct) : -1;
  cursor_next(ct, tiles, nkc, meta);
  Cursor cm = cursor_at(q0, na, tiles, meta);  // task being computed

  float acc_g[4], acc_u[4];
  const int a_off = (G == 64) ? 8 * c : 4 * c;
  const int b_off = (G == 64 ? 16 : 8) * c * (int)sizeof(XT);
  for (int task = 0; task < ntask; ++task) {
    if (task + S - 1 < ntask) issue(ci, task + S - 1, next_tok);
    cp_async_commit();
    cursor_next(ci, tiles, nkc, meta);
    next_tok = (task + S < ntask) ? token_of(ct) : -1;  // consumed by the next iteration's issue
    cursor_next(ct, tiles, nkc, meta);
    if (cm.kc == 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q) { acc_g[q] = 0.f; acc_u[q] = 0.f; }
    }
    const int ngt = min(C::kKch, H - cm.kc * C::kKch) / G;
    cp_async_wait<S - 1>();
    __syncthreads();
    const uint8_t* st = smem + (task % S) * C::kStage;
    const __half* sc = reinterpret_cast<const __half*>(st + C::kS);
    constexpr int kScH = C::kScaleRow / 2;
#pragma unroll 2
    for (int g = warp; g < ngt; g += kWarps) {
      const uint8_t* ab = st + C::kW + g * (G / 2) + a_off;
      const RowWords<G> ag0 = lds_row<G>(ab + r * C::kWStride);
      const RowWords<G> ag8 = lds_row<G>(ab + (r + 8) * C::kWStride);
      const RowWords<G> au0 = lds_row<G>(ab + (16 + r) * C::kWStride);
      const RowWords<G> au8 = lds_row<G>(ab + (24 + r) * C::kWStride);
      BWords<G> b;
      const uint8_t* bb = st + C::kB + r * C::kBStride + g * G * (int)sizeof(XT) + b_off;
      if constexpr (C::kF32) lds_b_f32<G>(bb, b);
      else lds_b_plane<G>(bb, b.hi);
      gateup_group<G, C::kF32>(ag0, ag8, au0, au8, b, __half2float(sc[r * kScH + g]),
                               __half2float(sc[(r + 8) * kScH + g]), __half2float(sc[(16 + r) * kScH + g]),
                               __half2float(sc[(24 + r) * kScH + g]), acc_g, acc_u);
    }
    if (cm.kc == nkc - 1) {
      // reduce the K-slices in warp order, then SwiGLU
      float* mine = red + warp * 8 * 32;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        mine[q * 32 + lane] = acc_g[q];
        mine[(4 + q) * 32 + lane] = acc_u[q];
      }
      __syncthreads();
      // 128 threads finish the 4 x 32 fragment slots: thread (q, ln) sums
      // slot q of lane ln over the warps in order 0..15.
      if (threadIdx.x < 128) {
        const int q = threadIdx.x >> 5, ln = threadIdx.x & 31;
        float gs = 0.f, us = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
          gs += red[w * 256 + q * 32 + ln];
          us += red[w * 256 + (4 + q) * 32 + ln];
        }
        const int n = meta.n[cm.slot], row0 = meta.row0[cm.slot];
        const int i = cm.tile * 16 + (ln >> 2) + (q >= 2 ? 8 : 0);
        const int rr = cm.pass * kTok + 2 * (ln & 3) + (q & 1);
        if (rr < n) {
          const float hv = silu_f32(gs) * us;
          const __nv_bfloat16 hb = __float2bfloat16_rn(hv);
          const __nv_bfloat16 lb = __float2bfloat16_rn(hv - __bfloat162float(hb));
          const size_t o = (size_t)(row0 + rr) * I + i;
          h_hi[o] = hb;
          h_lo[o] = lb;
        }
      }
    }
    cursor_next(cm, tiles, nkc, meta);
    __syncthreads();  // stage (task % S) and `red` are free again
  }
  cp_async_wait<0>();
}

// ---------------------------------------------------------------------------
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

template <int G>
__global__ void __launch_bounds__(kThreads, 1)
ffn_down_kernel(const __nv_bfloat16* __restrict__ h_hi, const __nv_bfloat16* __restrict__ h_lo,
                const int32_t* __restrict__ offsets, const int32_t* __restrict__ active,
                const uint8_t* __restrict__ w2_q, const uint16_t* __restrict__ w2_s, int H, int I, int E,
                float* __restrict__ y) {
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
    for (int q = threadIdx.x; q < C::kRows * C::kWch; q += kThreads) {
      const int rr = q / C::kWch, cc = q % C::kWch;
      if (cc * 32 < kel)
        cp_async16(smem_u32(st + C::kW + rr * C::kWStride + cc * 16), w2_q + (rbase + rr) * row_bytes + k0 / 2 + cc * 16);
    }
#pragma unroll
    for (int q = threadIdx.x; q < C::kRows * C::kPairs; q += kThreads) {
      const int rr = q / C::kPairs, pp = q % C::kPairs;
      if (pp * 2 * G < kel)
        cp_async4(smem_u32(st + C::kS + rr * C::kScaleRow + pp * 4), w2_s + (rbase + rr) * NG + k0 / G + 2 * pp);
    }
    // h rows of the pass (both planes), this K-chunk
    const int row_p = meta.row0[cu.slot] + cu.pass * kTok;
    const int nt = min(kTok, meta.n[cu.slot] - cu.pass * kTok);
#pragma unroll
    for (int q = threadIdx.x; q < 2 * kTok * C::kBch; q += kThreads) {
      const int pl = q / (kTok * C::kBch);
      const int n = (q / C::kBch) % kTok, cc = q % C::kBch;
      if (n < nt && cc * 8 < kel) {
        const __nv_bfloat16* src = (pl ? h_lo : h_hi) + (size_t)(row_p + n) * I + k0;
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
        lds_b_plane<G>(bb + kTok * C::kBStride, b.lo);
      } else {
#pragma unroll
        for (int i = 0; i < G / 8; ++i) b.hi[i] = b.lo[i] = 0u;
      }
      down_group<G>(a0, a8, b, __half2float(sc[lr0 * kScH + g]), __half2float(sc[(lr0 + 8) * kScH + g]), acc);
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

template <typename K>
void set_smem(K kern, size_t bytes) {
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

constexpr size_t kMaxSmem = 227 * 1024;

template <int G, typename XT, int KCH>
size_t gateup_smem(int E) {
  using C = GateUpCfg<G, XT, KCH>;
  return (size_t)C::kStages * C::kStage + C::kRed + (size_t)(4 * E + 4) * 4;
}

template <int G>
size_t down_smem(int E) {
  using C = DownCfg<G>;
  return (size_t)C::kStages * C::kStage + C::kRed + (size_t)(4 * E + 4) * 4;
}

template <int G, typename XT, int KCH>
void launch_gateup_k(const void* x, const int32_t* row_token, const int32_t* offsets, const int32_t* active,
                     const uint8_t* w13_q, const uint16_t* w13_s, int H, int I, int E, __nv_bfloat16* h_hi,
                     __nv_bfloat16* h_lo, int grid, cudaStream_t st) {
  const size_t smem = gateup_smem<G, XT, KCH>(E);
  auto k = ffn_gateup_kernel<G, XT, KCH>;
  set_smem(k, smem);
  k<<<grid, kThreads, smem, st>>>(static_cast<const XT*>(x), row_token, offsets, active, w13_q, w13_s, H, I,
                                  E, h_hi, h_lo);
}

// 2048-element tasks for bf16 activations when H needs them and they fit.
template <int G, typename XT>
void launch_gateup(const void* x, const int32_t* row_token, const int32_t* offsets, const int32_t* active,
                   const uint8_t* w13_q, const uint16_t* w13_s, int H, int I, int E, __nv_bfloat16* h_hi,
                   __nv_bfloat16* h_lo, int grid, cudaStream_t st) {
  if constexpr (!std::is_same<XT, float>::value) {
    if (H > 1024 && gateup_smem<G, XT, 2048>(E) <= kMaxSmem) {
      launch_gateup_k<G, XT, 2048>(x, row_token, offsets, active, w13_q, w13_s, H, I, E, h_hi, h_lo, grid, st);
      return;
    }
  }
  launch_gateup_k<G, XT, 1024>(x, row_token, offsets, active, w13_q, w13_s, H, I, E, h_hi, h_lo, grid, st);
}

template <int G>
void launch_down(const __nv_bfloat16* h_hi, const __nv_bfloat16* h_lo, const int32_t* offsets,
                 const int32_t* active, const uint8_t* w2_q, const uint16_t* w2_s, int H, int I, int E, float* y,
                 int grid, cudaStream_t st) {
  const size_t smem = down_smem<G>(E);
  auto k = ffn_down_kernel<G>;
  set_smem(k, smem);
  k<<<grid, kThreads, smem, st>>>(h_hi, h_lo, offsets, active, w2_q, w2_s, H, I, E, y);
}

}  // namespace

int launch_ffn_decode(const void* x, int x_dtype, const int32_t* row_token,
                      const int32_t* offsets, const int32_t* active, const uint8_t* w13_q,
                      const uint16_t* w13_s, const uint8_t* w2_q, const uint16_t* w2_s, int T,
                      int H, int E, int top_k, int I, int G, float* h, float* y,
                      cudaStream_t st, cudaEvent_t mid_event) {
  const long long R = (long long)T * top_k;
  if (R == 0) return PHMOE_OK;
  if (G != 32 && G != 64) return PHMOE_ERR_UNSUPPORTED;
  __nv_bfloat16* h_hi = reinterpret_cast<__nv_bfloat16*>(h);
  __nv_bfloat16* h_lo = h_hi + (size_t)R * I;
  const int grid = device_sm_count();
  const bool f32 = x_dtype == PHMOE_DTYPE_F32;
  if (G == 64) {
    if (f32) launch_gateup<64, float>(x, row_token, offsets, active, w13_q, w13_s, H, I, E, h_hi, h_lo, grid, st);
    else launch_gateup<64, __nv_bfloat16>(x, row_token, offsets, active, w13_q, w13_s, H, I, E, h_hi, h_lo, grid, st);
  } else {
    if (f32) launch_gateup<32, float>(x, row_token, offsets, active, w13_q, w13_s, H, I, E, h_hi, h_lo, grid, st);
    else launch_gateup<32, __nv_bfloat16>(x, row_token, offsets, active, w13_q, w13_s, H, I, E, h_hi, h_lo, grid, st);
  }
  if (mid_event) cudaEventRecord(mid_event, st);
  if (G == 64) launch_down<64>(h_hi, h_lo, offsets, active, w2_q, w2_s, H, I, E, y, grid, st);
  else launch_down<32>(h_hi, h_lo, offsets, active, w2_q, w2_s, H, I, E, y, grid, st);
  note_launches(2);
  return PHMOE_OK;
}

}  // namespace phmoe
