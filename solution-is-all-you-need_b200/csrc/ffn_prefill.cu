// Grouped SwiGLU expert FFN for large batches (prefill): two persistent
// grouped GEMMs on the 5th-generation tensor cores (tcgen05, accumulators in
// tensor memory), fed by TMA.
//
//   gather  : X[r] = fp16(x[row_token[r]])    (rows in expert order)
//   gate/up : h[r, i] = silu(X_e W_g^T)[r, i] * (X_e W_u^T)[r, i]   (fp16 h)
//   down    : y[r, :] = h_e[r] W_d^T                                 (fp32 y)
//
// This replaces the per-expert loop of Qwen3MoeExperts.forward
// (transformers 5.5.0 modeling_qwen3_moe.py:245-247) for batches where every
// expert sees many rows. PHANTOM runs that loop as bf16 GEMMs on weights it
// dequantised to bf16 at load time (python/phantom/loader/gguf_loader.py:
// 799-805); here the int4 weights stay packed in HBM and are dequantised per
// tile in shared memory. The MMA operands are fp16, not bf16: the
// dequantised weight fp16_rn((nibble - 8) * scale) is one exactly rounded
// f16x2 multiply of the fp16 scale, it carries 11 significant bits instead of
// 8 (at Mixtral's I = 14336 bf16 weights and h alone put the layer ~0.05 off
// the fp32 result), and bf16 activations convert to fp16 exactly inside the
// fp16 range. Values beyond the fp16 range keep their magnitude through
// power-of-two exponents (multiplying by 2^n is exact, so rows that stay in
// range are untouched - exponent 0, factor 1.0):
//   * gather: a row of x with |x| > 65504 is stored as x * 2^-sx[r] (its
//     largest finite |x| brought into [2^15, 2^16)); the gate/up epilogue
//     multiplies the accumulators by 2^sx[r];
//   * gate/up: a 128-column block of h with |h| > 65504 is stored as
//     h * 2^-eb[r, b] and raises the row's exponent er[r] (atomicMax);
//   * fixup: blocks of a row with eb[r, b] < er[r] are rescaled to er[r]
//     (a short kernel that reads er[] and leaves at once when all are 0);
//   * down: the epilogue multiplies row r of y by 2^er[r].
// Infinite and NaN inputs propagate as they would in fp32.
//
// Tile: 256 rows (two M=128 MMAs sharing one dequantised B tile) x 256
// output columns (N=256: a 128x128 MMA keeps the tensor core only about half
// busy, a 128x256 one fills it) x 64 K per pipeline stage (one 128-byte
// swizzle span). The two 128x256 fp32 accumulators fill all 512 TMEM
// columns, so the epilogue drains them before the next tile starts.
// Roles per CTA (576 threads, one CTA per SM, grid = SM count):
//   warp 0      : TMA producer - A rows (fp16, 128B swizzle) and raw int4
//                 weight rows into a 3-stage ring
//   warp 1      : allocates 512 TMEM columns; lane 0 issues tcgen05.mma
//                 (M128 N256 K16, fp16 -> fp32) and commits stage and
//                 accumulator barriers
//   warps 2-9   : dequantise the raw int4 tile into a 2-stage ring of fp16 B
//                 tiles (K-major, 128B swizzle, as the MMA descriptor says),
//                 one B row of 64 elements per thread per stage
//   warps 10-17 : epilogue - tcgen05.ld the accumulators (warp w reads TMEM
//                 lanes 32*(w%4)..+31), SwiGLU or fp32 store, release them
// For gate/up the 256 B rows of a tile are 128 gate rows and the 128 matching
// up rows, so one accumulator holds both halves of the SwiGLU.
//
// Every wait is bounded: a wait that runs out sets the CTA's abort flag and
// the device error word (phmoe_device_error); all roles then leave their
// loops, the producer waits (bounded) for its copies in flight, the MMA
// thread waits for its last commit, and TMEM is released before exit.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>

#include "common.cuh"
#include "pipeline.cuh"
#include "launch.h"

namespace phmoe {

// Error bits raised by the prefill kernels (read by phmoe_device_error;
// every writer ORs its bit in):
//   1  a pipeline wait timed out and its CTA abandoned its work
__device__ int g_prefill_error;

namespace {

constexpr int kBM = 128;                          // rows per MMA
constexpr int kHalves = 2;                        // MMAs per B tile along M
constexpr int kTileM = kBM * kHalves;             // rows per tile
constexpr int kBN = 256;                          // MMA N: B rows (output columns) per tile
constexpr int kBK = 64;                           // K per stage
constexpr int kLoadStages = 3;                    // ring of A rows + raw int4 (TMA)
constexpr int kBStages = 2;                       // ring of dequantised B tiles
constexpr int kAHalfBytes = kBM * kBK * 2;        // 16 KB
constexpr int kABytes = kTileM * kBK * 2;         // 32 KB
constexpr int kBBytes = kBN * kBK * 2;            // 32 KB
constexpr int kRawBytes = kBN * kBK / 2;          // 8 KB
constexpr int kLoadBytes = kABytes + kRawBytes;   // one load stage
constexpr int kBOffset = kLoadStages * kLoadBytes;
constexpr int kCtlOffset = kBOffset + kBStages * kBBytes;
constexpr int kDequantWarps = 8;
constexpr int kEpiWarps = 8;
constexpr int kThreads = (2 + kDequantWarps + kEpiWarps) * 32;
constexpr uint32_t kTmemCols = 512;               // 2 halves x 256 fp32 columns
// Waits suspend in mbarrier.try_wait (woken when the phase completes) for at
// most kSuspendNs per try; a wait that has not completed after kWaitLimitNs
// of %globaltimer time gives up.
constexpr uint32_t kSuspendNs = 20000;
constexpr unsigned long long kWaitLimitNs = 2000000000ull;
constexpr uint32_t kDrainPolls = 1u << 22;
static_assert(kLoadBytes % 1024 == 0 && kBBytes % 1024 == 0, "stages must keep 1024-byte alignment");
static_assert(kDequantWarps * 32 == kBN, "one dequant thread per B row");

// Instruction descriptor of tcgen05.mma kind::f16: fp32 D (bits 4-5 = 1),
// fp16 A and B (bits 7-9, 10-12 = 0), both K-major, N >> 3 at bit 17,
// M >> 4 at bit 24.
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
constexpr float kF16Max = 65504.0f;

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// Shared-memory matrix descriptor: K-major tile of 128-byte rows with the
// 128-byte swizzle, 8-row groups 1024 bytes apart (SBO), version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(kIdesc), "r"(accumulate) : "memory");
}
// Arrive once on `bar` when every tcgen05.mma this thread issued so far is done.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
               : "memory");
}
// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

// (w & 0x000F000F) | 0x64006400: the nibbles at bits 0-3 and 16-19 as the
// fp16 pair (1024 + n), exact (fp16's unit in the last place at 1024 is 1).
__device__ __forceinline__ uint32_t nib_pair_f16(uint32_t v) {
  uint32_t r;
  asm("lop3.b32 %0, %1, 0x000F000F, 0x64006400, 0xEA;" : "=r"(r) : "r"(v));
  return r;
}
// One packed word (elements e0..e7) -> fp16 pairs (e_{2i} - 8, e_{2i+1} - 8) * s,
// each rounded once: (1024 + n) - 1032 is exact, and so is its product's
// single rounding in mul.rn.
__device__ __forceinline__ void dequant_word_f16(uint32_t w, uint32_t s2, uint32_t (&o)[4]) {
  const uint32_t one = 0x3C003C00u, m1032 = 0xE408E408u;  // (1, 1), (-1032, -1032)
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t t;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(t) : "r"(nib_pair_f16(w >> (4 * i))), "r"(one), "r"(m1032));
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o[i]) : "r"(t), "r"(s2));
  }
}
// fp32 pair -> fp16x2 (round to nearest even); `over` is set when either
// value lies beyond the fp16 range (and so rounds to infinity).
__device__ __forceinline__ uint32_t pack_f16x2(float a, float b, bool& over) {
  over |= fabsf(a) > kF16Max || fabsf(b) > kF16Max;
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
// 2^e as fp32 for e in [-126, 127] (exact).
__device__ __forceinline__ float pow2i(int e) { return __int_as_float((127 + e) << 23); }
// Unbiased exponent of a positive finite or infinite fp32 (128 for inf).
__device__ __forceinline__ int exponent_of(float m) { return (int)((__float_as_uint(m) >> 23) & 0xFFu) - 127; }

struct Ctl {
  uint64_t full[kLoadStages];   // A rows + raw weights landed (TMA transaction bytes)
  uint64_t empty[kLoadStages];  // MMAs reading the load stage finished (tcgen05.commit)
  uint64_t bready[kBStages];    // dequantised B tile written (one arrival per dequant warp)
  uint64_t bempty[kBStages];    // MMAs reading the B tile finished (tcgen05.commit)
  uint64_t acc_full;            // accumulators complete (tcgen05.commit)
  uint64_t acc_empty;           // accumulators read out (one arrival per epilogue warp)
  uint64_t drain;               // final commit before TMEM is released
  uint32_t tmem_base;
  int abort_flag;
};

// Bounded wait of one thread; false when this CTA aborts (the first thread
// to run out of time raises the abort flag and the device error word).
__device__ __forceinline__ bool lane_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  while (true) {
    if (mbar_try_wait_suspend(bar, parity, kSuspendNs)) return true;
    if (*abort_flag) return false;
    if (global_ns() - t0 > kWaitLimitNs) break;
  }
  *abort_flag = 1;
  atomicOr(&g_prefill_error, 1);
  return false;
}
// Warp form: lane 0 waits, the result is the same for the whole warp.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int lane) {
  int ok = 1;
  if (lane == 0) ok = lane_wait(bar, parity, abort_flag) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// Tiles of active slot s are prefix[s] .. prefix[s+1]-1; a slot's tiles are
// its ceil(n/256) row tiles times the column tiles, row tile fastest (tiles
// of one weight column block run side by side, so its weights are read from
// HBM once and from L2 after that).
__device__ int build_tiles(const int32_t* __restrict__ offsets, const int32_t* __restrict__ active, int ncol,
                           int* prefix) {
  const int na = __ldg(active);
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    int carry = 0;
    for (int s0 = 0; s0 < na; s0 += 32) {
      const int s = s0 + lane;
      int v = 0;
      if (s < na) {
        const int e = __ldg(active + 1 + s);
        const int n = __ldg(offsets + e + 1) - __ldg(offsets + e);
        v = ((n + kTileM - 1) / kTileM) * ncol;
      }
      int incl = v;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += t;
      }
      if (s < na) prefix[s] = carry + incl - v;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) prefix[na] = carry;
  }
  __syncthreads();
  return prefix[na];
}

struct Tile {
  int e, row0, n, m0, col;
};

__device__ __forceinline__ Tile tile_at(int t, int na, const int* prefix, const int32_t* __restrict__ offsets,
                                        const int32_t* __restrict__ active) {
  int lo = 0, hi = na;  // prefix[lo] <= t < prefix[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (prefix[mid] <= t) lo = mid; else hi = mid;
  }
  const int e = __ldg(active + 1 + lo);
  const int r0 = __ldg(offsets + e);
  const int n = __ldg(offsets + e + 1) - r0;
  const int mt = (n + kTileM - 1) / kTileM;
  const int local = t - prefix[lo];
  return Tile{e, r0, n, (local % mt) * kTileM, local / mt};
}

// The SwiGLU block of one row (128 columns: gate accumulators at taddr,
// up at taddr + 128) when some |h| exceeds the fp16 range: one pass finds
// the largest |h|, a second stores h * 2^-eb with that value in
// [2^14, 2^15); returns eb (0 for lanes with `over` false, which store
// nothing). Warp-collective (tcgen05.ld).
__device__ __noinline__ int swiglu_block_rescaled(uint32_t taddr, float rs, bool over, __half* dst_row) {
  constexpr int kHalfN = kBN / 2;
  float m = 0.0f;
#pragma unroll 1
  for (int c = 0; c < kHalfN; c += 32) {
    uint32_t g[32], u[32];
    tmem_ld32(taddr + c, g);
    tmem_ld32(taddr + kHalfN + c, u);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 32; ++i)
      m = fmaxf(m, fabsf(silu_f32(__uint_as_float(g[i]) * rs) * (__uint_as_float(u[i]) * rs)));
  }
  const int eb = over ? exponent_of(m) - 14 : 0;
  const float hs = pow2i(-eb);
#pragma unroll 1
  for (int c = 0; c < kHalfN; c += 32) {
    uint32_t g[32], u[32];
    tmem_ld32(taddr + c, g);
    tmem_ld32(taddr + kHalfN + c, u);
    tmem_ld_wait();
    uint32_t packed[16];
    bool unused = false;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float h0 = silu_f32(__uint_as_float(g[2 * i]) * rs) * (__uint_as_float(u[2 * i]) * rs);
      const float h1 = silu_f32(__uint_as_float(g[2 * i + 1]) * rs) * (__uint_as_float(u[2 * i + 1]) * rs);
      packed[i] = pack_f16x2(h0 * hs, h1 * hs, unused);
    }
    if (over) {
      uint4* dst = reinterpret_cast<uint4*>(dst_row + c);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        dst[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
    }
  }
  return eb;
}

// kGateUp: B rows of a tile are gate rows col*64.. and up rows I+col*64..
// (wrows = 2I per expert), output h = SwiGLU as fp16 [R, n_out = I].
// Otherwise B rows are col*128.. of [E*H, K/2] (wrows = H) and the output is
// fp32 y [R, n_out = H].
template <bool kGateUp>
__global__ void __launch_bounds__(kThreads, 1)
prefill_gemm_kernel(const __grid_constant__ CUtensorMap a_map, const __grid_constant__ CUtensorMap w_map,
                    const uint16_t* __restrict__ w_s, const int32_t* __restrict__ offsets,
                    const int32_t* __restrict__ active, int K, int n_out, int wrows, int G,
                    __half* __restrict__ h_out, float* __restrict__ y_out, const int32_t* __restrict__ row_exp,
                    int32_t* __restrict__ h_row_exp, uint8_t* __restrict__ h_blk_exp) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Ctl* ctl = reinterpret_cast<Ctl*>(smem + kCtlOffset);
  int* prefix = reinterpret_cast<int*>(ctl + 1);
  volatile int* abort_flag = &ctl->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = K / kBK;
  const int ncol = kGateUp ? n_out / (kBN / 2) : n_out / kBN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kLoadStages; ++s) {
      mbar_init(smem_u32(&ctl->full[s]), 1);
      mbar_init(smem_u32(&ctl->empty[s]), 1);
    }
    for (int s = 0; s < kBStages; ++s) {
      mbar_init(smem_u32(&ctl->bready[s]), kDequantWarps);
      mbar_init(smem_u32(&ctl->bempty[s]), 1);
    }
    mbar_init(smem_u32(&ctl->acc_full), 1);
    mbar_init(smem_u32(&ctl->acc_empty), kEpiWarps);
    mbar_init(smem_u32(&ctl->drain), 1);
    ctl->abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n"
                 ::"r"(smem_u32(&ctl->tmem_base)), "r"(kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    tc_fence_before();
  }
  const int na = __ldg(active);
  const int total = build_tiles(offsets, active, ncol, prefix);  // its __syncthreads publishes the above
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        const Tile tl = tile_at(t, na, prefix, offsets, active);
        const int wrow = kGateUp ? tl.e * wrows + tl.col * (kBN / 2) : tl.e * wrows + tl.col * kBN;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % kLoadStages;
          if (it >= kLoadStages &&
              !lane_wait(smem_u32(&ctl->empty[s]), ((it / kLoadStages) - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t full = smem_u32(&ctl->full[s]);
          uint8_t* st = smem + s * kLoadBytes;
          mbar_arrive_expect_tx(full, kLoadBytes);
          tma_load_2d(smem_u32(st), &a_map, kb * kBK, tl.row0 + tl.m0, full);
          const uint32_t raw = smem_u32(st + kABytes);
          if (kGateUp) {
            tma_load_2d(raw, &w_map, kb * (kBK / 2), wrow, full);
            tma_load_2d(raw + (kBN / 2) * (kBK / 2), &w_map, kb * (kBK / 2), wrow + n_out, full);
          } else {
            tma_load_2d(raw, &w_map, kb * (kBK / 2), wrow, full);
          }
        }
      }
      // leave only when every copy issued into shared memory has landed
      for (int t = it - kLoadStages < 0 ? 0 : it - kLoadStages; t < it; ++t) {
        const uint32_t full = smem_u32(&ctl->full[t % kLoadStages]);
        for (uint32_t i = 0; i < kDrainPolls && !mbar_try_wait(full, (t / kLoadStages) & 1); ++i) {
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int it = 0, tcount = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x, ++tcount) {
        const Tile tl = tile_at(t, na, prefix, offsets, active);
        const int halves = (tl.n - tl.m0 > kBM) ? 2 : 1;
        if (tcount >= 1 && !lane_wait(smem_u32(&ctl->acc_empty), (tcount - 1) & 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d0 = tmem_base;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int sl = it % kLoadStages, sb = it % kBStages;
          if (!lane_wait(smem_u32(&ctl->full[sl]), (it / kLoadStages) & 1, abort_flag) ||
              !lane_wait(smem_u32(&ctl->bready[sb]), (it / kBStages) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + sl * kLoadBytes);
          const uint32_t b_base = smem_u32(smem + kBOffset + sb * kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t bdesc = sw128_desc(b_base + k * 32);
            umma_f16(d0, sw128_desc(a_base + k * 32), bdesc, (kb | k) != 0);
            if (halves == 2) umma_f16(d0 + kBN, sw128_desc(a_base + kAHalfBytes + k * 32), bdesc, (kb | k) != 0);
          }
          umma_commit(smem_u32(&ctl->bempty[sb]));
          umma_commit(smem_u32(&ctl->empty[sl]));
        }
        if (ok) umma_commit(smem_u32(&ctl->acc_full));
      }
      // every MMA must be finished before TMEM is released, abort or not
      umma_commit(smem_u32(&ctl->drain));
      for (uint32_t i = 0; i < kDrainPolls && !mbar_try_wait(smem_u32(&ctl->drain), 0); ++i) {
      }
    }
    __syncwarp();
  } else if (warp < 2 + kDequantWarps) {
    // ---------------- dequantise int4 -> fp16 B tile ----------------
    const int r = threadIdx.x - 64;  // B row
    const int ng = K / G;
    const int gstep = kBK / G;        // groups per stage
    const int g2 = 32 / G;            // group offset of elements 32..63 (1 for G=32, 0 for G=64)
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
      const Tile tl = tile_at(t, na, prefix, offsets, active);
      constexpr int kHalfN = kBN / 2;
      const int srow = kGateUp ? tl.e * wrows + (r < kHalfN ? tl.col * kHalfN + r : n_out + tl.col * kHalfN + (r - kHalfN))
                               : tl.e * wrows + tl.col * kBN + r;
      const uint16_t* sp = w_s + (size_t)srow * ng;
      // scales of elements 0..31 and 32..63 of stages kb, kb+1 (prefetched two stages ahead)
      uint32_t sc0 = (uint32_t)__ldg(sp) | ((uint32_t)__ldg(sp + g2) << 16);
      uint32_t sc1 = nkb > 1 ? ((uint32_t)__ldg(sp + gstep) | ((uint32_t)__ldg(sp + gstep + g2) << 16)) : 0u;
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const uint32_t sc = sc0;
        sc0 = sc1;
        sc1 = kb + 2 < nkb ? ((uint32_t)__ldg(sp + (kb + 2) * gstep) | ((uint32_t)__ldg(sp + (kb + 2) * gstep + g2) << 16))
                           : 0u;
        const int sl = it % kLoadStages, sb = it % kBStages;
        if (!warp_wait(smem_u32(&ctl->full[sl]), (it / kLoadStages) & 1, abort_flag, lane) ||
            (it >= kBStages &&
             !warp_wait(smem_u32(&ctl->bempty[sb]), ((it / kBStages) - 1) & 1, abort_flag, lane))) {
          ok = false;
          break;
        }
        const uint8_t* rawrow = smem + sl * kLoadBytes + kABytes + r * (kBK / 2);
        const uint4 raw0 = *reinterpret_cast<const uint4*>(rawrow);
        const uint4 raw1 = *reinterpret_cast<const uint4*>(rawrow + 16);
        const uint32_t s2a = (sc & 0xFFFFu) * 0x10001u;  // scale of elements 0..31, both halves
        const uint32_t s2b = (sc >> 16) * 0x10001u;      // scale of elements 32..63
        uint8_t* brow = smem + kBOffset + sb * kBBytes + (r >> 3) * 1024 + (r & 7) * 128;
        const uint32_t words[8] = {raw0.x, raw0.y, raw0.z, raw0.w, raw1.x, raw1.y, raw1.z, raw1.w};
#pragma unroll
        for (int c = 0; c < 8; ++c) {  // word c = elements 8c..8c+7 = 16-byte chunk c of the row
          uint32_t o[4];
          dequant_word_f16(words[c], c < 4 ? s2a : s2b, o);
          *reinterpret_cast<uint4*>(brow + ((c ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&ctl->bready[sb]));
      }
    }
  } else {
    // ---------------- epilogue ----------------
    const int ew = warp - 2 - kDequantWarps;
    const int half = ew >> 2;
    const int quarter = warp & 3;  // TMEM lanes this warp may read
    const int lrow = half * kBM + quarter * 32 + lane;
    int tcount = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++tcount) {
      const Tile tl = tile_at(t, na, prefix, offsets, active);
      const int halves = (tl.n - tl.m0 > kBM) ? 2 : 1;
      if (!warp_wait(smem_u32(&ctl->acc_full), tcount & 1, abort_flag, lane)) break;
      tc_fence_after();
      if (half < halves) {
        const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(half * kBN);
        const bool valid = tl.m0 + lrow < tl.n;
        const size_t row = (size_t)(tl.row0 + tl.m0 + lrow);
        // row_exp[row]: 2^row_exp undoes the power-of-two scaling of this
        // GEMM's A row (x for gate/up, h for down); 0 for rows in range.
        const float rs = valid ? pow2i(__ldg(row_exp + row)) : 1.0f;
        if (kGateUp) {
          constexpr int kHalfN = kBN / 2;  // gate columns, then as many up columns
          // h is stored as fp16; a row whose block went beyond the fp16
          // range is redone by swiglu_block_rescaled (the accumulators stay
          // in TMEM until acc_empty; tcgen05.ld is warp-collective, so the
          // whole warp takes that call).
          bool over = false;
          int eb = 0;
#pragma unroll 1
          for (int c = 0; c < kHalfN; c += 32) {
            uint32_t g[32], u[32];
            tmem_ld32(taddr + c, g);
            tmem_ld32(taddr + kHalfN + c, u);
            tmem_ld_wait();
            uint32_t packed[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float g0 = __uint_as_float(g[2 * i]) * rs, g1 = __uint_as_float(g[2 * i + 1]) * rs;
              const float h0 = silu_f32(g0) * (__uint_as_float(u[2 * i]) * rs);
              const float h1 = silu_f32(g1) * (__uint_as_float(u[2 * i + 1]) * rs);
              packed[i] = pack_f16x2(h0, h1, over);
            }
            if (valid) {
              uint4* dst = reinterpret_cast<uint4*>(h_out + row * n_out + tl.col * kHalfN + c);
#pragma unroll
              for (int i = 0; i < 4; ++i)
                dst[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
            }
          }
          over = over && valid;
          if (__any_sync(0xffffffffu, over))
            eb = swiglu_block_rescaled(taddr, rs, over, h_out + row * n_out + tl.col * kHalfN);
          if (valid) {
            h_blk_exp[row * (size_t)(n_out / kHalfN) + tl.col] = (uint8_t)eb;
            if (eb) atomicMax(h_row_exp + row, eb);
          }
        } else {
#pragma unroll 1
          for (int c = 0; c < kBN; c += 32) {
            uint32_t v[32];
            tmem_ld32(taddr + c, v);
            tmem_ld_wait();
            if (rs != 1.0f) {
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * rs);
            }
            if (valid) {
              uint4* dst = reinterpret_cast<uint4*>(y_out + row * n_out + tl.col * kBN + c);
#pragma unroll
              for (int i = 0; i < 8; ++i) dst[i] = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctl->acc_empty));
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem_base), "r"(kTmemCols)
                 : "memory");
  }
}

constexpr size_t kSmemFixed = 1024 + (size_t)kCtlOffset + sizeof(Ctl);

size_t prefill_smem(int E) { return kSmemFixed + (size_t)(E + 1) * sizeof(int); }

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  }
  return fn;
}

// 2-D map over a row-major [rows, cols] matrix.
bool make_map(CUtensorMap* map, CUtensorMapDataType dt, size_t elt, const void* base, uint64_t cols, uint64_t rows,
              uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz) {
  EncodeFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * elt};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool kGateUp>
int launch_gemm(const CUtensorMap& a_map, const CUtensorMap& w_map, const uint16_t* w_s, const int32_t* offsets,
                const int32_t* active, int K, int n_out, int wrows, int G, int E, __half* h_out,
                float* y_out, const int32_t* row_exp, int32_t* h_row_exp, uint8_t* h_blk_exp, cudaStream_t st) {
  auto k = prefill_gemm_kernel<kGateUp>;
  const size_t smem = prefill_smem(E);
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return PHMOE_ERR_CUDA;
  k<<<device_sm_count(), kThreads, smem, st>>>(a_map, w_map, w_s, offsets, active, K, n_out, wrows, G, h_out,
                                               y_out, row_exp, h_row_exp, h_blk_exp);
  note_launches(1);
  return PHMOE_OK;
}

}  // namespace

int prefill_device_error(bool reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_prefill_error, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_prefill_error, &zero, sizeof(int));
  }
  return v;
}

bool prefill_supported(int H, int I, int G, int E) {
  return (G == 32 || G == 64) && H % kBN == 0 && I % (kBN / 2) == 0 && E >= 1 &&
         prefill_smem(E) <= 227 * 1024;
}

namespace {

constexpr int kGatherThreads = 128;
constexpr int kFixupWarps = 8;

// X[r] = fp16(x[row_token[r]] * 2^-sx[r]) for the rows of experts
// (r < offsets[E]). bf16 -> fp16 is exact inside the fp16 range, where
// sx[r] = 0; a row with |x| > 65504 gets sx[r] = (exponent of its largest
// finite |x|) - 15, which brings that value into [2^15, 2^16) where every
// bf16 value is an fp16 value. Also zeroes er[r], the row's h exponent that
// the gate/up epilogue raises. One CTA per row.
__global__ void __launch_bounds__(kGatherThreads)
gather_to_f16_kernel(const __nv_bfloat16* __restrict__ x, int T, const int32_t* __restrict__ row_token,
                     const int32_t* __restrict__ offsets, int E, int H, __half* __restrict__ xg,
                     int32_t* __restrict__ sx, int32_t* __restrict__ er) {
  __shared__ uint32_t warp_max[kGatherThreads / 32];
  const int r = blockIdx.x;
  if (r >= __ldg(offsets + E)) return;
  const int t = __ldg(row_token + r);
  if (t < 0 || t >= T) {
    if (threadIdx.x == 0) sx[r] = er[r] = 0;
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)t * H);
  uint4* dst = reinterpret_cast<uint4*>(xg + (size_t)r * H);
  bool over = false;
  uint32_t mag = 0;  // largest finite |x| of this thread, as bf16 bits (they order like the values)
  for (int c = threadIdx.x; c < H / 8; c += kGatherThreads) {
    const uint4 v = __ldg(src + c);
    const uint32_t in[4] = {v.x, v.y, v.z, v.w};
    uint32_t out[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t a = in[i] & 0x7FFFu, b = (in[i] >> 16) & 0x7FFFu;
      if (a < 0x7F80u) mag = max(mag, a);
      if (b < 0x7F80u) mag = max(mag, b);
      out[i] = pack_f16x2(bf16_lo_to_f32(in[i]), bf16_hi_to_f32(in[i]), over);
    }
    dst[c] = make_uint4(out[0], out[1], out[2], out[3]);
  }
  int e = 0;
  if (__syncthreads_or(over)) {
    mag = __reduce_max_sync(0xffffffffu, mag);
    if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = mag;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < kGatherThreads / 32; ++w) mag = max(mag, warp_max[w]);
    e = max(0, (int)(mag >> 7) - 127 - 15);
    const float s = pow2i(-e);
    bool unused = false;
    for (int c = threadIdx.x; c < H / 8; c += kGatherThreads) {
      const uint4 v = __ldg(src + c);
      const uint32_t in[4] = {v.x, v.y, v.z, v.w};
      uint32_t out[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) out[i] = pack_f16x2(bf16_lo_to_f32(in[i]) * s, bf16_hi_to_f32(in[i]) * s, unused);
      dst[c] = make_uint4(out[0], out[1], out[2], out[3]);
    }
  }
  if (threadIdx.x == 0) {
    sx[r] = e;
    er[r] = 0;
  }
}

// Rows whose 128-column blocks of h were stored with different exponents:
// block b of row r holds h * 2^-eb[r, b]; rescale the blocks below the row's
// exponent er[r] to it (exact unless a value falls into the fp16 subnormals).
// One warp per row, 4 halves per lane per block; rows with er[r] = 0 - all
// of them unless something exceeded the fp16 range - cost one load.
__global__ void __launch_bounds__(kFixupWarps * 32)
h_fixup_kernel(const int32_t* __restrict__ offsets, int E, const int32_t* __restrict__ er,
               const uint8_t* __restrict__ eb, int I, __half* __restrict__ h) {
  const int rows = __ldg(offsets + E);
  const int nblk = I / (kBN / 2);
  const int lane = threadIdx.x & 31;
  for (int r = blockIdx.x * kFixupWarps + (threadIdx.x >> 5); r < rows; r += gridDim.x * kFixupWarps) {
    const int e = __ldg(er + r);
    if (e == 0) continue;
    for (int b = 0; b < nblk; ++b) {
      const int d = e - (int)__ldg(eb + (size_t)r * nblk + b);
      if (d <= 0) continue;
      const float s = pow2i(-d);
      uint2* p = reinterpret_cast<uint2*>(h + (size_t)r * I + b * (kBN / 2)) + lane;
      uint2 v = *p;
      __half2* hv = reinterpret_cast<__half2*>(&v);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float2 f = __half22float2(hv[i]);
        hv[i] = __floats2half2_rn(f.x * s, f.y * s);
      }
      *p = v;
    }
  }
}

}  // namespace

// x is bf16 [T, H]; h is scratch of R*I*4 bytes: the fp16 h [R, I], then the
// row exponents sx[R] and er[R] (int32) and the block exponents
// eb[R, I/128] (uint8), which need 8 + I/128 <= 2*I bytes per row;
// y [R, H] fp32 doubles as the gathered fp16 activation rows until the down GEMM.
int launch_ffn_prefill(const void* x, const int32_t* row_token, const int32_t* offsets, const int32_t* active,
                       const uint8_t* w13_q, const uint16_t* w13_s, const uint8_t* w2_q, const uint16_t* w2_s,
                       int T, int H, int E, int top_k, int I, int G, float* h, float* y, cudaStream_t st,
                       cudaEvent_t mid_event) {
  const int R = T * top_k;
  if (R == 0) return PHMOE_OK;
  __half* xg = reinterpret_cast<__half*>(y);
  __half* hb = reinterpret_cast<__half*>(h);
  int32_t* sx = reinterpret_cast<int32_t*>(hb + (size_t)R * I);
  int32_t* er = sx + R;
  uint8_t* eb = reinterpret_cast<uint8_t*>(er + R);
  gather_to_f16_kernel<<<R, kGatherThreads, 0, st>>>(static_cast<const __nv_bfloat16*>(x), T, row_token, offsets, E,
                                                      H, xg, sx, er);
  note_launches(1);
  CUtensorMap a1, w1, a2, w2;
  if (!make_map(&a1, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, xg, H, R, kBK, kTileM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&w1, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w13_q, H / 2, (uint64_t)E * 2 * I, kBK / 2, kBN / 2,
                CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_map(&a2, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, hb, I, R, kBK, kTileM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&w2, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w2_q, I / 2, (uint64_t)E * H, kBK / 2, kBN,
                CU_TENSOR_MAP_SWIZZLE_NONE))
    return PHMOE_ERR_CUDA;
  if (int s = launch_gemm<true>(a1, w1, w13_s, offsets, active, H, I, 2 * I, G, E, hb, nullptr, sx, er, eb, st))
    return s;
  const int fixup_ctas = std::min((R + kFixupWarps - 1) / kFixupWarps, device_sm_count() * 8);
  h_fixup_kernel<<<fixup_ctas, kFixupWarps * 32, 0, st>>>(offsets, E, er, eb, I, hb);
  note_launches(1);
  if (mid_event) cudaEventRecord(mid_event, st);
  return launch_gemm<false>(a2, w2, w2_s, offsets, active, I, H, H, G, E, nullptr, y, er, nullptr, nullptr, st);
}

}  // namespace phmoe
