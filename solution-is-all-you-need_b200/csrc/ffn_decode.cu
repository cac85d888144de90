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
// are persistent (one 256-thread CTA per SM) and run a 4-stage cp.async
// pipeline: while the 8 warps compute task t, the packed int4 weights and
// fp16 scales of tasks t+1..t+3 are in flight from HBM into shared memory
// (~100 KB per SM), so memory latency is covered by the pipeline rather than
// by occupancy. Weight rows are stored with a 32-byte (G=64) / 16-byte (G=32)
// pad so that the fragment reads below are bank-conflict free.
//
// From shared memory each lane reads the int4 bytes of its A fragments, turns
// them into bf16 (nibble - 8) in registers (exact) and issues mma.sync
// m16n8k16 with tokens as the N=8 side. The dequantised weights are never
// written back to shared memory (bf16 would be 4x the int4 bytes). The fp16
// group scale multiplies the fp32 partial of each group (exact factorisation).
// Activations (B) are prefetched into registers one group ahead.
//
// The K order inside a group is permuted identically for A and B (a dot
// product does not depend on the order): for G=64 lane c of a quad holds
// elements 8c..8c+7 (low nibbles) and 32+8c..32+8c+7 (high nibbles), exactly
// the activations it loads with two 16-byte loads.
//
// Precision: bf16 activations enter the MMA exactly; fp32 activations and the
// intermediate h are split into bf16 hi + lo parts (two MMAs each), keeping
// ~16 significant bits.
//
// gate/up kernel: item = (expert, token pass, 16 intermediate rows) -> 32
//   weight rows (16 gate + 16 up); the 8 warps split K and are reduced through
//   shared memory in warp order (deterministic); SwiGLU in the epilogue.
// down kernel: item = (expert, token pass, 128 output rows); warp w owns rows
//   16w..16w+15 over all of K.
// A token pass covers up to 8*NCH of the expert's rows; experts with more
// rows get more passes (more items).
#include "common.cuh"
#include "launch.h"

namespace phmoe {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 4;

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

// B fragments for one group and one 8-token chunk: per MMA step (2 per
// 32-bit weight word: low then high nibbles) the two b registers, for the
// "hi" part and (split inputs) the "lo" part.
template <int G>
struct GroupB {
  static constexpr int kSteps = 2 * (G / 32);
  uint32_t hi[kSteps][2];
  uint32_t lo[kSteps][2];
};

// Activations of one group (global group index g). Step order: word 0 low,
// word 0 high, word 1 low, word 1 high. G=64: word w low covers elements
// 8c+4w..+3, high covers 32+8c+4w..+3. G=32: low 4c..4c+3, high 16+4c..+3.
template <int G>
__device__ __forceinline__ void load_b_bf16(const __nv_bfloat16* row, int g, int c, bool ok,
                                            uint32_t (&d)[GroupB<G>::kSteps][2]) {
  if constexpr (G == 64) {
    uint4 x0 = make_uint4(0, 0, 0, 0), x1 = make_uint4(0, 0, 0, 0);
    if (ok) {
      x0 = __ldg(reinterpret_cast<const uint4*>(row + g * 64 + 8 * c));
      x1 = __ldg(reinterpret_cast<const uint4*>(row + g * 64 + 32 + 8 * c));
    }
    d[0][0] = x0.x; d[0][1] = x0.y;
    d[1][0] = x1.x; d[1][1] = x1.y;
    d[2][0] = x0.z; d[2][1] = x0.w;
    d[3][0] = x1.z; d[3][1] = x1.w;
  } else {
    uint2 x0 = make_uint2(0, 0), x1 = make_uint2(0, 0);
    if (ok) {
      x0 = __ldg(reinterpret_cast<const uint2*>(row + g * 32 + 4 * c));
      x1 = __ldg(reinterpret_cast<const uint2*>(row + g * 32 + 16 + 4 * c));
    }
    d[0][0] = x0.x; d[0][1] = x0.y;
    d[1][0] = x1.x; d[1][1] = x1.y;
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

template <int G, typename XT>
__device__ __forceinline__ void load_b_x(const XT* row, int g, int c, bool ok, GroupB<G>& b) {
  if constexpr (std::is_same<XT, float>::value) load_b_f32<G>(row, g, c, ok, b);
  else load_b_bf16<G>(row, g, c, ok, b.hi);
}

template <int G>
__device__ __forceinline__ void load_b_planes(const __nv_bfloat16* hi_row, const __nv_bfloat16* lo_row,
                                              int g, int c, bool ok, GroupB<G>& b) {
  load_b_bf16<G>(hi_row, g, c, ok, b.hi);
  load_b_bf16<G>(lo_row, g, c, ok, b.lo);
}

// Packed words of one row of one group for this lane, from shared memory.
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

// tmp += A(rows r, r+8 of one group) * B(chunk), all MMA steps of the group.
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
// work items
// ---------------------------------------------------------------------------

// table[s] = items of the active experts before slot s (s = 0..na); an
// expert with n rows has ceil(n / tok_per_pass) passes of `tiles` items.
// Every CTA builds the same table. Returns the total item count.
__device__ int build_item_table(const int32_t* __restrict__ offsets, const int32_t* __restrict__ active,
                                int tok_per_pass, int tiles, int* table) {
  const int na = active[0];
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    int carry = 0;
    for (int s0 = 0; s0 < na; s0 += 32) {
      const int s = s0 + lane;
      int v = 0;
      if (s < na) {
        const int e = active[1 + s];
        const int n = offsets[e + 1] - offsets[e];
        v = ((n + tok_per_pass - 1) / tok_per_pass) * tiles;
      }
      int incl = v;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += t;
      }
      if (s < na) table[s + 1] = carry + incl;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) table[0] = 0;
  }
  __syncthreads();
  return table[na];
}

struct Item {
  int e, row0, n, p0, tile;
};

__device__ __forceinline__ Item decode_item(int q, const int* table, const int32_t* __restrict__ offsets,
                                            const int32_t* __restrict__ active, int tiles, int tok_per_pass) {
  int lo = 0, hi = active[0];  // table[lo] <= q < table[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (table[mid] <= q) lo = mid;
    else hi = mid;
  }
  const int local = q - table[lo];
  const int pass = local / tiles;
  Item it;
  it.e = active[1 + lo];
  it.row0 = offsets[it.e];
  it.n = offsets[it.e + 1] - it.row0;
  it.p0 = pass * tok_per_pass;
  it.tile = local - pass * tiles;
  return it;
}

// ---------------------------------------------------------------------------
// gate/up + SwiGLU
// ---------------------------------------------------------------------------
template <int G>
struct GateUpCfg {
  static constexpr int kRows = 32;
  static constexpr int kKch = 2048;  // K elements per task
  static constexpr int kStride = kKch / 2 + (G == 64 ? 32 : 16);
  static constexpr int kScaleRow = kKch / G * 2;  // scale bytes per row per task
  static constexpr int kWBytes = kRows * kStride;
  static constexpr int kStage = kWBytes + kRows * kScaleRow;
};

template <int G, typename XT, int NCH>
__global__ void __launch_bounds__(kThreads, 1)
ffn_gateup_kernel(const XT* __restrict__ x, const int32_t* __restrict__ row_token,
                  const int32_t* __restrict__ offsets, const int32_t* __restrict__ active,
                  const uint8_t* __restrict__ w13_q, const uint16_t* __restrict__ w13_s, int H, int I,
                  __nv_bfloat16* __restrict__ h_hi, __nv_bfloat16* __restrict__ h_lo) {
  using C = GateUpCfg<G>;
  constexpr bool kTwo = std::is_same<XT, float>::value;
  constexpr int kTok = 8 * NCH;
  extern __shared__ __align__(128) uint8_t smem[];
  float* red = reinterpret_cast<float*>(smem + kStages * C::kStage);  // [kWarps][NCH*8][32]
  int* table = reinterpret_cast<int*>(red + kWarps * NCH * 8 * 32);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, c = lane & 3;
  const int tiles = I / 16;
  const int NG = H / G;
  const int nkc = (H + C::kKch - 1) / C::kKch;
  const size_t row_bytes = (size_t)H / 2;

  const int total = build_item_table(offsets, active, kTok, tiles, table);
  const int my_items = blockIdx.x < total ? (total - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  const int my_tasks = my_items * nkc;

  auto issue = [&](int task) {
    const int j = task / nkc, kc = task - j * nkc;
    const Item it = decode_item(blockIdx.x + j * gridDim.x, table, offsets, active, tiles, kTok);
    uint8_t* st = smem + (task % kStages) * C::kStage;
    const int k0 = kc * C::kKch;
    const int kel = min(C::kKch, H - k0);
    const int nch16 = kel / 32;  // 16-byte chunks per row
    const size_t erow = (size_t)it.e * 2 * I;
    const int i0 = it.tile * 16;
    for (int q = threadIdx.x; q < C::kRows * nch16; q += kThreads) {
      const int rr = q / nch16, cc = q - rr * nch16;
      const size_t grow = erow + (rr < 16 ? i0 + rr : I + i0 + rr - 16);
      cp_async16(smem_u32(st + rr * C::kStride + cc * 16), w13_q + grow * row_bytes + k0 / 2 + cc * 16);
    }
    const int npair = kel / G / 2;
    uint8_t* sc = st + C::kWBytes;
    for (int q = threadIdx.x; q < C::kRows * npair; q += kThreads) {
      const int rr = q / npair, pp = q - rr * npair;
      const size_t grow = erow + (rr < 16 ? i0 + rr : I + i0 + rr - 16);
      cp_async4(smem_u32(sc + rr * C::kScaleRow + pp * 4), w13_s + grow * NG + k0 / G + 2 * pp);
    }
  };

#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    if (s < my_tasks) issue(s);
    cp_async_commit();
  }

  float acc[NCH][2][4];
  for (int task = 0; task < my_tasks; ++task) {
    if (task + kStages - 1 < my_tasks) issue(task + kStages - 1);
    cp_async_commit();
    const int j = task / nkc, kc = task - j * nkc;
    const Item it = decode_item(blockIdx.x + j * gridDim.x, table, offsets, active, tiles, kTok);
    if (kc == 0) {
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
        for (int q = 0; q < 4; ++q) { acc[ch][0][q] = 0.f; acc[ch][1][q] = 0.f; }
    }
    const int nvch = min(NCH, (it.n - it.p0 + 7) / 8);  // chunks holding tokens
    const XT* xrow[NCH];
    bool xok[NCH];
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      const int rr = it.p0 + ch * 8 + r;
      xok[ch] = rr < it.n;
      xrow[ch] = x + (size_t)(xok[ch] ? row_token[it.row0 + rr] : 0) * H;
    }
    const int k0 = kc * C::kKch;
    const int ngt = min(C::kKch, H - k0) / G;
    const int kg0 = k0 / G;
    GroupB<G> b0[NCH], b1[NCH];
    if (warp < ngt) {
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch)
        if (ch < nvch) load_b_x<G, XT>(xrow[ch], kg0 + warp, c, xok[ch], b0[ch]);
    }
    cp_async_wait<kStages - 1>();
    __syncthreads();
    const uint8_t* st = smem + (task % kStages) * C::kStage;
    const __half* sc = reinterpret_cast<const __half*>(st + C::kWBytes);
    constexpr int kScH = C::kScaleRow / 2;
    const int lane_off = (G == 64) ? 8 * c : 4 * c;

    auto compute = [&](int g, const GroupB<G> (&b)[NCH]) {
      const uint8_t* base = st + g * (G / 2) + lane_off;
      const RowWords<G> ag0 = lds_row<G>(base + r * C::kStride);
      const RowWords<G> ag8 = lds_row<G>(base + (r + 8) * C::kStride);
      const RowWords<G> au0 = lds_row<G>(base + (16 + r) * C::kStride);
      const RowWords<G> au8 = lds_row<G>(base + (24 + r) * C::kStride);
      const float sg0 = __half2float(sc[r * kScH + g]);
      const float sg8 = __half2float(sc[(r + 8) * kScH + g]);
      const float su0 = __half2float(sc[(16 + r) * kScH + g]);
      const float su8 = __half2float(sc[(24 + r) * kScH + g]);
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {
        if (ch < nvch) {
          float tg[4] = {0.f, 0.f, 0.f, 0.f}, tu[4] = {0.f, 0.f, 0.f, 0.f};
          mma_group<G, kTwo>(tg, ag0, ag8, b[ch]);
          mma_group<G, kTwo>(tu, au0, au8, b[ch]);
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
    };

    // groups g = warp, warp+8, ...; B for the next group is in flight while
    // the current one computes.
    for (int g = warp; g < ngt; g += 2 * kWarps) {
      const int g1 = g + kWarps, g2 = g + 2 * kWarps;
      if (g1 < ngt) {
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch)
          if (ch < nvch) load_b_x<G, XT>(xrow[ch], kg0 + g1, c, xok[ch], b1[ch]);
      }
      compute(g, b0);
      if (g1 < ngt) {
        if (g2 < ngt) {
#pragma unroll
          for (int ch = 0; ch < NCH; ++ch)
            if (ch < nvch) load_b_x<G, XT>(xrow[ch], kg0 + g2, c, xok[ch], b0[ch]);
        }
        compute(g1, b1);
      }
    }

    if (kc == nkc - 1) {
      // reduce the 8 K-slices in warp order, then SwiGLU
      float* mine = red + (size_t)warp * NCH * 8 * 32;
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          mine[(ch * 8 + q) * 32 + lane] = acc[ch][0][q];
          mine[(ch * 8 + 4 + q) * 32 + lane] = acc[ch][1][q];
        }
      __syncthreads();
      if (warp < nvch) {
        const int ch = warp;
        float gs[4] = {0.f, 0.f, 0.f, 0.f}, us[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
          const float* src = red + (size_t)w * NCH * 8 * 32;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            gs[q] += src[(ch * 8 + q) * 32 + lane];
            us[q] += src[(ch * 8 + 4 + q) * 32 + lane];
          }
        }
        const int i0 = it.tile * 16;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int i = i0 + r + (q >= 2 ? 8 : 0);
          const int rr = it.p0 + ch * 8 + 2 * c + (q & 1);
          if (rr < it.n) {
            const float hv = silu_f32(gs[q]) * us[q];
            const __nv_bfloat16 hb = __float2bfloat16_rn(hv);
            const __nv_bfloat16 lb = __float2bfloat16_rn(hv - __bfloat162float(hb));
            const size_t o = (size_t)(it.row0 + rr) * I + i;
            h_hi[o] = hb;
            h_lo[o] = lb;
          }
        }
      }
    }
    __syncthreads();  // stage (task % kStages) and `red` are free again
  }
  cp_async_wait<0>();
}

// ---------------------------------------------------------------------------
// down projection
// ---------------------------------------------------------------------------
template <int G>
struct DownCfg {
  static constexpr int kRows = 128;
  static constexpr int kKch = 512;
  static constexpr int kStride = kKch / 2 + (G == 64 ? 32 : 16);
  static constexpr int kScaleRow = kKch / G * 2;
  static constexpr int kWBytes = kRows * kStride;
  static constexpr int kStage = kWBytes + kRows * kScaleRow;
};

template <int G, int NCH>
__global__ void __launch_bounds__(kThreads, 1)
ffn_down_kernel(const __nv_bfloat16* __restrict__ h_hi, const __nv_bfloat16* __restrict__ h_lo,
                const int32_t* __restrict__ offsets, const int32_t* __restrict__ active,
                const uint8_t* __restrict__ w2_q, const uint16_t* __restrict__ w2_s, int H, int I,
                float* __restrict__ y) {
  using C = DownCfg<G>;
  constexpr int kTok = 8 * NCH;
  extern __shared__ __align__(128) uint8_t smem[];
  int* table = reinterpret_cast<int*>(smem + kStages * C::kStage);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, c = lane & 3;
  const int tiles = H / C::kRows;
  const int NG = I / G;
  const int nkc = (I + C::kKch - 1) / C::kKch;
  const size_t row_bytes = (size_t)I / 2;

  const int total = build_item_table(offsets, active, kTok, tiles, table);
  const int my_items = blockIdx.x < total ? (total - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  const int my_tasks = my_items * nkc;

  auto issue = [&](int task) {
    const int j = task / nkc, kc = task - j * nkc;
    const Item it = decode_item(blockIdx.x + j * gridDim.x, table, offsets, active, tiles, kTok);
    uint8_t* st = smem + (task % kStages) * C::kStage;
    const int k0 = kc * C::kKch;
    const int kel = min(C::kKch, I - k0);
    const int nch16 = kel / 32;
    const size_t rbase = (size_t)it.e * H + (size_t)it.tile * C::kRows;
    for (int q = threadIdx.x; q < C::kRows * nch16; q += kThreads) {
      const int rr = q / nch16, cc = q - rr * nch16;
      cp_async16(smem_u32(st + rr * C::kStride + cc * 16), w2_q + (rbase + rr) * row_bytes + k0 / 2 + cc * 16);
    }
    const int npair = kel / G / 2;
    uint8_t* sc = st + C::kWBytes;
    for (int q = threadIdx.x; q < C::kRows * npair; q += kThreads) {
      const int rr = q / npair, pp = q - rr * npair;
      cp_async4(smem_u32(sc + rr * C::kScaleRow + pp * 4), w2_s + (rbase + rr) * NG + k0 / G + 2 * pp);
    }
  };

#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    if (s < my_tasks) issue(s);
    cp_async_commit();
  }

  float acc[NCH][4];
  const int lr0 = warp * 16 + r;
  for (int task = 0; task < my_tasks; ++task) {
    if (task + kStages - 1 < my_tasks) issue(task + kStages - 1);
    cp_async_commit();
    const int j = task / nkc, kc = task - j * nkc;
    const Item it = decode_item(blockIdx.x + j * gridDim.x, table, offsets, active, tiles, kTok);
    if (kc == 0) {
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[ch][q] = 0.f;
    }
    const int nvch = min(NCH, (it.n - it.p0 + 7) / 8);
    const __nv_bfloat16* hr[NCH];
    const __nv_bfloat16* lr[NCH];
    bool ok[NCH];
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      const int rr = it.p0 + ch * 8 + r;
      ok[ch] = rr < it.n;
      const size_t off = (size_t)(it.row0 + (ok[ch] ? rr : 0)) * I;
      hr[ch] = h_hi + off;
      lr[ch] = h_lo + off;
    }
    const int k0 = kc * C::kKch;
    const int ngt = min(C::kKch, I - k0) / G;
    const int kg0 = k0 / G;
    GroupB<G> b0[NCH], b1[NCH];
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch)
      if (ch < nvch) load_b_planes<G>(hr[ch], lr[ch], kg0, c, ok[ch], b0[ch]);
    cp_async_wait<kStages - 1>();
    __syncthreads();
    const uint8_t* st = smem + (task % kStages) * C::kStage;
    const __half* sc = reinterpret_cast<const __half*>(st + C::kWBytes);
    constexpr int kScH = C::kScaleRow / 2;
    const int lane_off = (G == 64) ? 8 * c : 4 * c;

    auto compute = [&](int g, const GroupB<G> (&b)[NCH]) {
      const uint8_t* base = st + g * (G / 2) + lane_off;
      const RowWords<G> a0 = lds_row<G>(base + lr0 * C::kStride);
      const RowWords<G> a8 = lds_row<G>(base + (lr0 + 8) * C::kStride);
      const float s0 = __half2float(sc[lr0 * kScH + g]);
      const float s8 = __half2float(sc[(lr0 + 8) * kScH + g]);
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {
        if (ch < nvch) {
          float t[4] = {0.f, 0.f, 0.f, 0.f};
          mma_group<G, true>(t, a0, a8, b[ch]);
          acc[ch][0] = fmaf(s0, t[0], acc[ch][0]);
          acc[ch][1] = fmaf(s0, t[1], acc[ch][1]);
          acc[ch][2] = fmaf(s8, t[2], acc[ch][2]);
          acc[ch][3] = fmaf(s8, t[3], acc[ch][3]);
        }
      }
    };

    for (int g = 0; g < ngt; g += 2) {
      if (g + 1 < ngt) {
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch)
          if (ch < nvch) load_b_planes<G>(hr[ch], lr[ch], kg0 + g + 1, c, ok[ch], b1[ch]);
      }
      compute(g, b0);
      if (g + 1 < ngt) {
        if (g + 2 < ngt) {
#pragma unroll
          for (int ch = 0; ch < NCH; ++ch)
            if (ch < nvch) load_b_planes<G>(hr[ch], lr[ch], kg0 + g + 2, c, ok[ch], b0[ch]);
        }
        compute(g + 1, b1);
      }
    }

    if (kc == nkc - 1) {
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int hrow = it.tile * C::kRows + lr0 + (q >= 2 ? 8 : 0);
          const int rr = it.p0 + ch * 8 + 2 * c + (q & 1);
          if (rr < it.n) y[(size_t)(it.row0 + rr) * H + hrow] = acc[ch][q];
        }
      }
    }
    __syncthreads();  // stage (task % kStages) is free again
  }
  cp_async_wait<0>();
}

template <int G, typename XT, int NCH>
void launch_gateup(const void* x, const int32_t* row_token, const int32_t* offsets,
                   const int32_t* active, const uint8_t* w13_q, const uint16_t* w13_s, int H, int I,
                   int E, __nv_bfloat16* h_hi, __nv_bfloat16* h_lo, int grid, cudaStream_t st) {
  const size_t smem = (size_t)kStages * GateUpCfg<G>::kStage + (size_t)kWarps * NCH * 8 * 32 * 4 +
                      (size_t)(E + 2) * 4;
  auto kern = ffn_gateup_kernel<G, XT, NCH>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  kern<<<grid, kThreads, smem, st>>>(static_cast<const XT*>(x), row_token, offsets, active, w13_q, w13_s,
                                      H, I, h_hi, h_lo);
}

template <int G, int NCH>
void launch_down(const __nv_bfloat16* h_hi, const __nv_bfloat16* h_lo, const int32_t* offsets,
                 const int32_t* active, const uint8_t* w2_q, const uint16_t* w2_s, int H, int I, int E,
                 float* y, int grid, cudaStream_t st) {
  const size_t smem = (size_t)kStages * DownCfg<G>::kStage + (size_t)(E + 2) * 4;
  auto kern = ffn_down_kernel<G, NCH>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  kern<<<grid, kThreads, smem, st>>>(h_hi, h_lo, offsets, active, w2_q, w2_s, H, I, y);
}

template <int G, int NCH>
void launch_all(const void* x, int x_dtype, const int32_t* row_token, const int32_t* offsets,
                const int32_t* active, const uint8_t* w13_q, const uint16_t* w13_s,
                const uint8_t* w2_q, const uint16_t* w2_s, int H, int I, int E, int R,
                __nv_bfloat16* h_hi, __nv_bfloat16* h_lo, float* y, cudaStream_t st,
                cudaEvent_t mid_event) {
  const int sms = device_sm_count();
  // upper bounds on the item counts (every row its own pass at worst)
  const long long max_active = std::min<long long>(E, R);
  const long long passes = max_active + R / (8 * NCH);
  const int g1 = (int)std::max<long long>(1, std::min<long long>(sms, passes * (I / 16)));
  const int g2 = (int)std::max<long long>(1, std::min<long long>(sms, passes * (H / 128)));
  if (x_dtype == PHMOE_DTYPE_BF16)
    launch_gateup<G, __nv_bfloat16, NCH>(x, row_token, offsets, active, w13_q, w13_s, H, I, E, h_hi, h_lo, g1, st);
  else
    launch_gateup<G, float, 1>(x, row_token, offsets, active, w13_q, w13_s, H, I, E, h_hi, h_lo, g1, st);
  if (mid_event) cudaEventRecord(mid_event, st);
  launch_down<G, NCH>(h_hi, h_lo, offsets, active, w2_q, w2_s, H, I, E, y, g2, st);
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
  __nv_bfloat16* h_hi = reinterpret_cast<__nv_bfloat16*>(h);
  __nv_bfloat16* h_lo = h_hi + (size_t)R * I;
  const long long mean = (R + E - 1) / E;
  const int nch = (mean <= 2 || x_dtype == PHMOE_DTYPE_F32) ? 1 : 2;
#define PHMOE_FFN_CASE(GG, NN)                                                                  \
  if (G == GG && nch == NN) {                                                                   \
    launch_all<GG, NN>(x, x_dtype, row_token, offsets, active, w13_q, w13_s, w2_q, w2_s, H, I, E, \
                       (int)R, h_hi, h_lo, y, st, mid_event);                                  \
    return PHMOE_OK;                                                                            \
  }
  PHMOE_FFN_CASE(64, 1)
  PHMOE_FFN_CASE(64, 2)
  PHMOE_FFN_CASE(32, 1)
  PHMOE_FFN_CASE(32, 2)
#undef PHMOE_FFN_CASE
  return PHMOE_ERR_UNSUPPORTED;
}

}  // namespace phmoe
