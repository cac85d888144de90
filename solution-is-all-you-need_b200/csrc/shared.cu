// Shared experts as extra routed slots.
//
// Models with shared experts add to the routed output the output of an
// always-on SwiGLU expert, optionally scaled by a per-token sigmoid gate:
// Qwen2-MoE (transformers 5.5.0 models/qwen2_moe/modeling_qwen2_moe.py,
// Qwen2MoeSparseMoeBlock.forward: routed + sigmoid(x . w_sg) * shared(x));
// DeepSeek-style blocks (n_shared_experts always-on experts, no gate, routed
// weights scaled by routed_scaling_factor). A shared expert of intermediate
// size m * I is the sum of m experts of size I (SwiGLU separates over the
// intermediate dimension), so the packed weights hold them as experts
// E .. E+m-1 after the E routed ones, and this kernel appends m slots to
// every token's routing: slot k + i -> expert E + i with weight g(t).
// Dispatch, the expert FFN and combine then run unchanged over E + m
// experts and k + m slots (combine adds the routed slots first, then the
// shared ones, as the reference adds the shared output last).
#include "common.cuh"
#include "launch.h"

namespace phmoe {

namespace {

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  v[0] = bf16_lo_to_f32(u.x); v[1] = bf16_hi_to_f32(u.x);
  v[2] = bf16_lo_to_f32(u.y); v[3] = bf16_hi_to_f32(u.y);
  v[4] = bf16_lo_to_f32(u.z); v[5] = bf16_hi_to_f32(u.z);
  v[6] = bf16_lo_to_f32(u.w); v[7] = bf16_hi_to_f32(u.w);
}
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// One warp per token: g = sigmoid(x[t] . gate_w) in fp32 (1 without a gate),
// then the k routed slots (weights times routed_scale) and the m shared ones.
template <typename XT, typename WT>
__global__ void __launch_bounds__(256)
shared_slots_kernel(const XT* __restrict__ x, const WT* __restrict__ gate_w, const int32_t* __restrict__ idx,
                    const float* __restrict__ w, int T, int H, int k, int E, int m, float routed_scale,
                    int32_t* __restrict__ idx_out, float* __restrict__ w_out) {
  pdl_begin();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  float g = 1.0f;
  if (gate_w) {
    float acc = 0.f;
    for (int h0 = lane * 8; h0 < H; h0 += 256) {
      float xv[8], wv[8];
      load8<XT>(x + (size_t)t * H + h0, xv);
      load8<WT>(gate_w + h0, wv);
#pragma unroll
      for (int v = 0; v < 8; ++v) acc = fmaf(xv[v], wv[v], acc);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    g = 1.0f / (1.0f + expf(-acc));
  }
  const int kk = k + m;
  for (int j = lane; j < kk; j += 32) {
    const size_t o = (size_t)t * kk + j;
    if (j < k) {
      idx_out[o] = idx[(size_t)t * k + j];
      w_out[o] = w[(size_t)t * k + j] * routed_scale;
    } else {
      idx_out[o] = E + (j - k);
      w_out[o] = g;
    }
  }
}

template <typename XT, typename WT>
void launch_slots(const void* x, const void* gate_w, const int32_t* idx, const float* w, int T, int H, int k,
                  int E, int m, float scale, int32_t* idx_out, float* w_out, cudaStream_t st) {
  launch_pdl(shared_slots_kernel<XT, WT>, dim3((T + 7) / 8), dim3(256), 0, st, static_cast<const XT*>(x),
                                                           static_cast<const WT*>(gate_w), idx, w, T, H, k, E, m,
                                                           scale, idx_out, w_out);
}

}  // namespace

int launch_shared_slots(const void* x, int x_dtype, const void* gate_w, int w_dtype, const int32_t* idx,
                        const float* w, int T, int H, int k, int E, int m, float routed_scale, int32_t* idx_out,
                        float* w_out, cudaStream_t st) {
  if (T == 0) return PHMOE_OK;
  const bool xb = x_dtype == PHMOE_DTYPE_BF16, wb = w_dtype == PHMOE_DTYPE_BF16;
  if (xb && wb) launch_slots<__nv_bfloat16, __nv_bfloat16>(x, gate_w, idx, w, T, H, k, E, m, routed_scale, idx_out, w_out, st);
  else if (xb) launch_slots<__nv_bfloat16, float>(x, gate_w, idx, w, T, H, k, E, m, routed_scale, idx_out, w_out, st);
  else if (wb) launch_slots<float, __nv_bfloat16>(x, gate_w, idx, w, T, H, k, E, m, routed_scale, idx_out, w_out, st);
  else launch_slots<float, float>(x, gate_w, idx, w, T, H, k, E, m, routed_scale, idx_out, w_out, st);
  note_launches(1);
  return PHMOE_OK;
}

}  // namespace phmoe
