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
  const int t = blockIdx.x;
  const int h = (blockIdx.y * blockDim.x + threadIdx.x) * 4;
  if (h >= H) return;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j = 0; j < top_k; ++j) {
    const int row = __ldg(inv + (size_t)t * top_k + j);
    if (row < 0) continue;  // assignment dropped by dispatch (expert id out of range)
    const float w = __ldg(topk_w + (size_t)t * top_k + j);
    const float4 v = __ldg(reinterpret_cast<const float4*>(y + (size_t)row * H + h));
    acc.x = fmaf(w, v.x, acc.x);
    acc.y = fmaf(w, v.y, acc.y);
    acc.z = fmaf(w, v.z, acc.z);
    acc.w = fmaf(w, v.w, acc.w);
  }
  store4<OT>(out + (size_t)t * H + h, acc);
}

}  // namespace

int launch_combine(const float* y, const int32_t* inv, const float* topk_w, int T, int top_k,
                   int H, void* out, int out_dtype, cudaStream_t st) {
  if (T == 0) return PHMOE_OK;
  dim3 grid(T, (H / 4 + 255) / 256);
  if (out_dtype == PHMOE_DTYPE_BF16)
    combine_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(y, inv, topk_w, T, top_k, H,
                                                         static_cast<__nv_bfloat16*>(out));
  else
    combine_kernel<float><<<grid, 256, 0, st>>>(y, inv, topk_w, T, top_k, H, static_cast<float*>(out));
  note_launches(1);
  return PHMOE_OK;
}

}  // namespace phmoe
