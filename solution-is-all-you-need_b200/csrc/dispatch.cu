// Token dispatch: per-expert histogram, exclusive scan, and a stable
// permutation of the T*k (token, slot) assignments ordered by expert, then
// by token index. Replaces the one_hot / nonzero / where grouping of
// Qwen3MoeExperts.forward (transformers 5.5.0
// models/qwen3_moe/modeling_qwen3_moe.py:234-244), which needs a host sync
// per expert; here everything stays on the device.
//
// Assignment a = t*k + j. Inside one expert a token appears at most once, so
// "ascending a" is "ascending token". The rank of an assignment among the
// earlier assignments of its expert is found chunk by chunk (1024
// assignments per chunk): warp-level __match_any_sync ranks inside a warp,
// a per-(warp, expert) count table ranks the warps, and a running base per
// expert carries the chunks. The result is independent of thread timing.
#include "common.cuh"
#include "launch.h"

namespace phmoe {

namespace {

constexpr int kDispThreads = 1024;
constexpr int kDispWarps = kDispThreads / 32;
constexpr int kSingleCtaMaxRows = 16384;
// Decode batches (up to kSmallRows assignments) take a 256-thread CTA: the
// same algorithm with a quarter of the barrier participants and an
// 8-warp (instead of 32-warp) per-expert prefix.
constexpr int kSmallThreads = 256;
constexpr int kSmallRows = 2048;

// Exclusive scan of one int per thread over a kThreads-thread block.
template <int kThreads = kDispThreads>
__device__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
  constexpr int kWarps = kThreads / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += n;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int s = lane < kWarps ? warp_sums[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, s, off);
      if (lane >= off) s += n;
    }
    if (lane < kWarps) warp_sums[lane] = s;
  }
  __syncthreads();
  const int prefix = warp > 0 ? warp_sums[warp - 1] : 0;
  *total = warp_sums[kWarps - 1];
  __syncthreads();
  return prefix + incl - v;
}

// Offsets + active list from per-expert totals held in smem `cnt[E]`.
// Writes offsets[E+1], active[E+1] and leaves base[e] = offsets[e] in smem.
template <int kThreads = kDispThreads>
__device__ void scan_experts(const int* cnt, int E, int* base, int32_t* offsets, int32_t* active,
                             int* warp_sums) {
  int carry = 0, carry_act = 0;
  for (int e0 = 0; e0 < E; e0 += kThreads) {
    const int e = e0 + threadIdx.x;
    const int c = e < E ? cnt[e] : 0;
    int tot, tot_act;
    const int ex = block_exclusive_scan<kThreads>(c, warp_sums, &tot);
    const int ex_act = block_exclusive_scan<kThreads>(c > 0 ? 1 : 0, warp_sums, &tot_act);
    if (e < E) {
      base[e] = carry + ex;
      offsets[e] = carry + ex;
      if (c > 0) active[1 + carry_act + ex_act] = e;
    }
    carry += tot;
    carry_act += tot_act;
  }
  if (threadIdx.x == 0) {
    offsets[E] = carry;
    active[0] = carry_act;
  }
}

// Rank the assignments [a0, a0 + kThreads) and write their permuted rows.
// `base[e]` (smem) is the first free row of expert e and is advanced.
// `wcnt` is smem [kThreads / 32][E].
template <int kThreads = kDispThreads>
__device__ void rank_chunk(const int32_t* __restrict__ idx, int R, int top_k, int E, int a0,
                           int* base, int* wcnt, int32_t* row_token, int32_t* inv) {
  constexpr int kDispWarps = kThreads / 32;
  constexpr int kDispThreads = kThreads;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int a = a0 + threadIdx.x;
  const int e_raw = a < R ? idx[a] : 0;
  const bool valid = a < R && (unsigned)e_raw < (unsigned)E;
  const int e = valid ? e_raw : 0;
  if (a < R && !valid) inv[a] = -1;  // out-of-range expert id: dropped, combine skips it
  for (int i = threadIdx.x; i < kDispWarps * E; i += kDispThreads) wcnt[i] = 0;
  __syncthreads();
  const int key = valid ? e : -1 - lane;  // invalid lanes match nobody
  const uint32_t same = __match_any_sync(0xffffffffu, key);
  const uint32_t lt = (1u << lane) - 1u;
  const int rank = __popc(same & lt);
  if (valid && rank == 0) wcnt[warp * E + e] = __popc(same);
  __syncthreads();
  // Exclusive prefix over warps, per expert.
  for (int ee = threadIdx.x; ee < E; ee += kDispThreads) {
    int run = 0;
    for (int w = 0; w < kDispWarps; ++w) {
      const int c = wcnt[w * E + ee];
      wcnt[w * E + ee] = run;
      run += c;
    }
  }
  __syncthreads();
  int pos = 0;
  if (valid) {
    pos = base[e] + wcnt[warp * E + e] + rank;
    row_token[pos] = a / top_k;
    inv[a] = pos;
  }
  __syncthreads();
  // Advance base: the last assignment of each expert in this chunk moves it.
  if (valid) {
    const uint32_t gt = ~((2u << lane) - 1u);
    const bool last_in_warp = (same & gt) == 0;
    if (last_in_warp) atomicMax(&base[e], pos + 1);
  }
  __syncthreads();
}

template <int kDispThreads>
__global__ void __launch_bounds__(kDispThreads)
dispatch_single_kernel(const int32_t* __restrict__ idx, int T, int top_k, int E,
                       int32_t* __restrict__ offsets, int32_t* __restrict__ row_token,
                       int32_t* __restrict__ inv, int32_t* __restrict__ active) {
  pdl_begin();
  extern __shared__ int smem[];
  int* cnt = smem;               // [E]
  int* base = cnt + E;           // [E]
  int* warp_sums = base + E;     // [32]
  int* wcnt = warp_sums + 32;    // [kDispWarps * E]
  const int R = T * top_k;
  for (int e = threadIdx.x; e < E; e += kDispThreads) cnt[e] = 0;
  __syncthreads();
  for (int a = threadIdx.x; a < R; a += kDispThreads) {
    const int e = idx[a];
    if ((unsigned)e < (unsigned)E) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  scan_experts<kDispThreads>(cnt, E, base, offsets, active, warp_sums);
  __syncthreads();
  for (int a0 = 0; a0 < R; a0 += kDispThreads)
    rank_chunk<kDispThreads>(idx, R, top_k, E, a0, base, wcnt, row_token, inv);
}

// Multi-CTA form for large T*k: count per chunk, scan, then rank per chunk.
__global__ void __launch_bounds__(kDispThreads)
dispatch_count_kernel(const int32_t* __restrict__ idx, int R, int E, int32_t* __restrict__ blkcnt) {
  pdl_begin();
  extern __shared__ int cnt[];
  for (int e = threadIdx.x; e < E; e += kDispThreads) cnt[e] = 0;
  __syncthreads();
  const int a = blockIdx.x * kDispThreads + threadIdx.x;
  if (a < R) {
    const int e = idx[a];
    if ((unsigned)e < (unsigned)E) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += kDispThreads) blkcnt[(size_t)blockIdx.x * E + e] = cnt[e];
}

__global__ void __launch_bounds__(kDispThreads)
dispatch_scan_kernel(int nblk, int E, int32_t* __restrict__ blkcnt, int32_t* __restrict__ offsets,
                     int32_t* __restrict__ active) {
  pdl_begin();
  extern __shared__ int smem[];
  int* cnt = smem;            // [E]
  int* base = cnt + E;        // [E]
  int* warp_sums = base + E;  // [32]
  for (int e = threadIdx.x; e < E; e += kDispThreads) {
    int s = 0;
    for (int b = 0; b < nblk; ++b) s += blkcnt[(size_t)b * E + e];
    cnt[e] = s;
  }
  __syncthreads();
  scan_experts(cnt, E, base, offsets, active, warp_sums);
  __syncthreads();
  // blkcnt[b][e] <- first row of chunk b's assignments to expert e.
  for (int e = threadIdx.x; e < E; e += kDispThreads) {
    int run = base[e];
    for (int b = 0; b < nblk; ++b) {
      const int c = blkcnt[(size_t)b * E + e];
      blkcnt[(size_t)b * E + e] = run;
      run += c;
    }
  }
}

__global__ void __launch_bounds__(kDispThreads)
dispatch_rank_kernel(const int32_t* __restrict__ idx, int R, int top_k, int E,
                     const int32_t* __restrict__ blkbase, int32_t* __restrict__ row_token,
                     int32_t* __restrict__ inv) {
  pdl_begin();
  extern __shared__ int smem[];
  int* base = smem;         // [E]
  int* wcnt = base + E;     // [kDispWarps * E]
  for (int e = threadIdx.x; e < E; e += kDispThreads) base[e] = blkbase[(size_t)blockIdx.x * E + e];
  __syncthreads();
  rank_chunk(idx, R, top_k, E, blockIdx.x * kDispThreads, base, wcnt, row_token, inv);
}

}  // namespace

size_t dispatch_scratch_bytes(int T, int top_k, int E) {
  const long long R = (long long)T * top_k;
  if (R <= kSingleCtaMaxRows) return 0;
  const long long nblk = (R + kDispThreads - 1) / kDispThreads;
  return (size_t)(nblk * E * sizeof(int32_t));
}

int launch_dispatch(const int32_t* topk_idx, int T, int top_k, int E, int32_t* offsets,
                    int32_t* row_token, int32_t* inv, int32_t* active, void* scratch,
                    cudaStream_t st) {
  const int R = T * top_k;
  if (R <= kSmallRows) {
    auto k = dispatch_single_kernel<kSmallThreads>;
    const size_t smem = (size_t)(2 * E + 32 + (kSmallThreads / 32) * E) * sizeof(int);
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    launch_pdl(k, dim3(1), dim3(kSmallThreads), smem, st, topk_idx, T, top_k, E, offsets, row_token, inv, active);
    note_launches(1);
    return PHMOE_OK;
  }
  if (R <= kSingleCtaMaxRows) {
    auto k = dispatch_single_kernel<kDispThreads>;
    const size_t smem = (size_t)(2 * E + 32 + kDispWarps * E) * sizeof(int);
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    launch_pdl(k, dim3(1), dim3(kDispThreads), smem, st, topk_idx, T, top_k, E, offsets, row_token, inv, active);
    note_launches(1);
    return PHMOE_OK;
  }
  const int nblk = (R + kDispThreads - 1) / kDispThreads;
  int32_t* blkcnt = static_cast<int32_t*>(scratch);
  launch_pdl(dispatch_count_kernel, dim3(nblk), dim3(kDispThreads), E * sizeof(int), st, topk_idx, R, E, blkcnt);
  launch_pdl(dispatch_scan_kernel, dim3(1), dim3(kDispThreads), (2 * E + 32) * sizeof(int), st, nblk, E, blkcnt,
                                                                            offsets, active);
  const size_t smem = (size_t)(E + kDispWarps * E) * sizeof(int);
  if (smem > 48 * 1024) {
    cudaFuncSetAttribute(dispatch_rank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  }
  launch_pdl(dispatch_rank_kernel, dim3(nblk), dim3(kDispThreads), smem, st, topk_idx, R, top_k, E, blkcnt, row_token,
                                                        inv);
  note_launches(3);
  return PHMOE_OK;
}

}  // namespace phmoe
