// Combine: out[t] = sum_j w[t,j] * y[inv[t,j]] in slot order j = 0..k-1.
//
// Reference: Qwen3MoeExperts.forward multiplies each expert's rows by their
// routing weight and index_add_s them into the token rows
// (transformers 5.5.0 models/qwen3_moe/modeling_qwen3_moe.py:248-249); on a GPU
// index_add_ uses atomics, so its summation order varies run to run. Here each
// output element is one thread's fixed-order fp32 sum: bitwise deterministic.
#include "common.cuh"
#include "launch.h"

namespace phmoe {

namespace {

template <typename OT>
__device__ __forceinline__ void store4(OT* p, float4 v);

template <>
__device__ __forceinline__ void store4<float>(float* p, float4 v) {
  *reinterpret_cast<float4*>(p) = v;
}

template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* p, float4 v) {
  uint2 u;
  u.x = pack_bf16x2(v.x, v.y);
  u.y = pack_bf16x2(v.z, v.w);
  *reinterpret_cast<uint2*>(p) = u;
}

template <typename OT>
__global__ void __launch_bounds__(256)
combine_kernel(const float* __restrict__ y, const int32_t* __restrict__ inv,
               const float* __restrict__ topk_w, int T, int top_k, int H, OT* __restrict__ out) {
  pdl_begin();
  const int t = blockIdx.x;
  const int h = (blockIdx.y * blockDim.x + threadIdx.x) * 4;
  if (h >= H) return;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  const int32_t* inv_t = inv + (size_t)t * top_k;
  const float* w_t = topk_w + (size_t)t * top_k;
  // Slots in batches of 8: all loads of a batch are issued before the sums,
  // which then run in slot order.
  for (int j0 = 0; j0 < top_k; j0 += 8) {
    int row[8];
    float w[8];
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const bool ok = j0 + u < top_k;
      row[u] = ok ? __ldg(inv_t + j0 + u) : -1;  // -1 also marks a dropped assignment
      w[u] = ok ? __ldg(w_t + j0 + u) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u)
      v[u] = row[u] >= 0 ? __ldg(reinterpret_cast<const float4*>(y + (size_t)row[u] * H + h))
                         : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (row[u] >= 0) {
        acc.x = fmaf(w[u], v[u].x, acc.x);
        acc.y = fmaf(w[u], v[u].y, acc.y);
        acc.z = fmaf(w[u], v[u].z, acc.z);
        acc.w = fmaf(w[u], v[u].w, acc.w);
      }
    }
  }
  store4<OT>(out + (size_t)t * H + h, acc);
}

}  // namespace

int launch_combine(const float* y, const int32_t* inv, const float* topk_w, int T, int top_k,
                   int H, void* out, int out_dtype, cudaStream_t st) {
  if (T == 0) return PHMOE_OK;
  dim3 grid(T, (H / 4 + 255) / 256);
  if (out_dtype == PHMOE_DTYPE_BF16)
    launch_pdl(combine_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, st, y, inv, topk_w, T, top_k, H,
                                                         static_cast<__nv_bfloat16*>(out));
  else
    launch_pdl(combine_kernel<float>, dim3(grid), dim3(256), 0, st, y, inv, topk_w, T, top_k, H, static_cast<float*>(out));
  note_launches(1);
  return PHMOE_OK;
}

}  // namespace phmoe
