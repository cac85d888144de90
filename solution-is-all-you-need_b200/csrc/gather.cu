// Row gather dst[i] = src[index[i]]: the pack step of the expert-parallel
// dispatch (rows in expert order, ready for the all-to-all) and the
// un-permute of its return path. PHANTOM has no expert parallelism, so this
// has no counterpart in the reference.
//
// One CTA per 4 destination rows; its 128 threads stride over each row's
// 16-byte chunks. Rows are plain byte strings, so the same kernel moves bf16
// activations and fp32 expert outputs. Bandwidth bound: 2 * n_rows *
// row_bytes of HBM traffic.
#include <stdint.h>

#include "launch.h"

namespace phmoe {
namespace {

constexpr int kGatherThreads = 128;
constexpr int kRowsPerCta = 4;

__global__ void __launch_bounds__(kGatherThreads)
gather_rows_kernel(const uint4* __restrict__ src, long long src_rows, const int32_t* __restrict__ index,
                   int n_rows, int chunks, uint4* __restrict__ dst) {
  const int r0 = blockIdx.x * kRowsPerCta;
#pragma unroll
  for (int j = 0; j < kRowsPerCta; ++j) {
    const int r = r0 + j;
    if (r >= n_rows) return;
    const int s = index[r];
    uint4* d = dst + (size_t)r * chunks;
    if (s < 0 || (long long)s >= src_rows) {
      for (int c = threadIdx.x; c < chunks; c += kGatherThreads) d[c] = make_uint4(0, 0, 0, 0);
    } else {
      const uint4* p = src + (size_t)s * chunks;
      for (int c = threadIdx.x; c < chunks; c += kGatherThreads) d[c] = __ldg(p + c);
    }
  }
}

}  // namespace

void launch_gather_rows(const void* src, long long src_rows, const int32_t* index, int n_rows,
                        long long row_bytes, void* dst, cudaStream_t st) {
  if (n_rows <= 0 || row_bytes <= 0) return;
  const int chunks = (int)(row_bytes / 16);
  const int grid = (n_rows + kRowsPerCta - 1) / kRowsPerCta;
  gather_rows_kernel<<<grid, kGatherThreads, 0, st>>>(static_cast<const uint4*>(src), src_rows, index, n_rows,
                                                     chunks, static_cast<uint4*>(dst));
  note_launches(1);
}

}  // namespace phmoe
