// phmoe_moe_layer_noalloc: the whole MoE layer with its scratch memory in a
// fixed array that this library owns on every GPU, for callers that cannot
// allocate device memory themselves.
//
// Who those callers are: hosts that only receive device buffers from another
// framework (a serving runtime whose caching allocator has already reserved
// nearly all of the GPU's memory, so a cudaMalloc from outside it fails or
// fragments the pool), hosts whose policy forbids new device allocations
// once the model is loaded (cudaFree synchronises the whole device and
// cudaMalloc may, which stalls every other stream of the process), and
// foreign-language bindings that have no way to call an allocator at all.
// They pass inputs and outputs as usual; the layer's intermediate buffers
// (logits, routing tables, SwiGLU output, per-row expert output) live in
// `g_static_scratch` below instead of a caller-provided workspace.
//
// Limits and sharing rules (also stated in include/phmoe.h):
//  * The scratch holds PHMOE_STATIC_SCRATCH_BYTES (16 MiB). A call whose
//    phmoe_workspace_size(...) exceeds that is rejected with
//    PHMOE_ERR_WORKSPACE before anything is launched. At the Qwen3-30B-A3B
//    shape (H 2048, 128 experts, top-8, I 768) that is up to 184 tokens.
//  * Every GPU on which the library's device code is loaded holds the 16 MiB
//    until the process exits.
//  * All calls on a device share the one array and it keeps whatever the last
//    call left in it. Nothing in it needs to start at zero: every sub-buffer
//    the layer reads is written earlier in the same call (router -> logits and
//    top-k, dispatch -> offsets, row lists and inverse map, gate/up -> SwiGLU
//    output, down -> expert output), so nothing is cleared. Two calls that
//    overlap on the GPU (different streams, or different host threads without
//    ordering between their streams) race on the array and corrupt each
//    other's results; order them on one stream.
//  * The first call on each device looks up the array's device address with
//    cudaGetSymbolAddress (with that device current) and caches it; make that
//    first call before any stream capture begins on the device.
//  * Nothing here calls cudaMalloc, cudaFree or any allocating library
//    routine; the work itself is phmoe_moe_layer's, unchanged.
//
// The reference has no counterpart: its kernels cudaMalloc their scratch on
// every call (kernels/sparse_moe/sparse_matmul.cu:264-273).
#include <stdio.h>

#include <atomic>
#include <mutex>

#include "launch.h"
#include "phmoe.h"

namespace phmoe {
namespace {

constexpr size_t kStaticScratchBytes = PHMOE_STATIC_SCRATCH_BYTES;

// In host code this name is only a handle for the CUDA runtime; the device
// address comes from cudaGetSymbolAddress below.
__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::atomic<void*> g_scratch_ptr[kMaxDevices];
std::mutex g_setup_mutex;

// Device address of g_static_scratch on the current device (looked up once
// per device and cached).
int static_scratch(void** out) {
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "phmoe_moe_layer_noalloc: cudaGetDevice failed: %s", cudaGetErrorString(err));
    return record_error(PHMOE_ERR_CUDA, msg);
  }
  if (dev < 0 || dev >= kMaxDevices) {
    char msg[128];
    snprintf(msg, sizeof(msg), "phmoe_moe_layer_noalloc: device %d is beyond the %d this library tracks", dev,
             kMaxDevices);
    return record_error(PHMOE_ERR_UNSUPPORTED, msg);
  }
  void* p = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    p = g_scratch_ptr[dev].load(std::memory_order_relaxed);
    if (p == nullptr) {
      err = cudaGetSymbolAddress(&p, g_static_scratch);
      if (err != cudaSuccess || p == nullptr) {
        char msg[256];
        snprintf(msg, sizeof(msg), "phmoe_moe_layer_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                 cudaGetErrorString(err));
        cudaGetLastError();  // do not leave the error for the caller's next check
        return record_error(PHMOE_ERR_CUDA, msg);
      }
      g_scratch_ptr[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return PHMOE_OK;
}

}  // namespace
}  // namespace phmoe

using namespace phmoe;

extern "C" int phmoe_moe_layer_noalloc(const void* x, int x_dtype, const void* router_w, int w_dtype,
                                       const uint8_t* w13_q, const uint16_t* w13_s, const uint8_t* w2_q,
                                       const uint16_t* w2_s, int T, int H, int E, int top_k, int I,
                                       int group_size, int renormalize, int path, void* out,
                                       int32_t* topk_idx_out, float* topk_w_out, void* stream) {
  const size_t need = phmoe_workspace_size(T, H, E, top_k, I, path);
  if (need > kStaticScratchBytes) {
    char msg[320];
    snprintf(msg, sizeof(msg),
             "phmoe_moe_layer_noalloc: T=%d needs %zu bytes of scratch but the library's static scratch holds "
             "%zu; use fewer tokens per call or phmoe_moe_layer with a caller workspace",
             T, need, kStaticScratchBytes);
    return record_error(PHMOE_ERR_WORKSPACE, msg);
  }
  // need == 0 means invalid dimensions; phmoe_moe_layer reports which.
  void* scratch = nullptr;
  if (T > 0 && need > 0) {
    if (int s = static_scratch(&scratch)) return s;
  }
  return phmoe_moe_layer(x, x_dtype, router_w, w_dtype, w13_q, w13_s, w2_q, w2_s, T, H, E, top_k, I,
                         group_size, renormalize, path, out, topk_idx_out, topk_w_out, scratch,
                         kStaticScratchBytes, stream);
}
