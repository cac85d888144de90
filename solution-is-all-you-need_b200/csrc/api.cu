// C ABI of the phantom-moe layer (declared in include/phmoe.h).
//
// Every entry validates its arguments, launches stream-ordered work and
// returns a status code; nothing allocates, synchronises or exits. The
// reference's native entries instead cudaMalloc/cudaFree and create a cuBLAS
// handle per call and exit() on error (kernels/sparse_moe/sparse_matmul.cu:
// 264-314, kernels/common/cuda_utils.h:31-52).
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <string>
#include <vector>

#include "common.cuh"
#include "launch.h"

namespace phmoe {

namespace {

thread_local std::string g_last_error;

int fail(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int check_launch(const char* what) {
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess)
    return fail(PHMOE_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(err), cudaGetErrorString(err));
  return PHMOE_OK;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
bool dtype_ok(int d) { return d == PHMOE_DTYPE_F32 || d == PHMOE_DTYPE_BF16; }
size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

constexpr size_t kAlign = 256;

// Workspace carve-up shared by phmoe_workspace_size and phmoe_moe_layer.
struct Layout {
  size_t logits, idx, w, offsets, active, row_token, inv, disp, h, y, total;
};

Layout make_layout(int T, int H, int E, int k, int I) {
  Layout L{};
  const size_t R = (size_t)T * k;
  size_t off = 0;
  auto take = [&](size_t bytes) { const size_t o = off; off = round_up(off + bytes, kAlign); return o; };
  L.logits = take((size_t)T * E * 4);
  L.idx = take(R * 4);
  L.w = take(R * 4);
  L.offsets = take((size_t)(E + 1) * 4);
  L.active = take((size_t)(E + 1) * 4);
  L.row_token = take(R * 4);
  L.inv = take(R * 4);
  L.disp = take(dispatch_scratch_bytes(T, k, E));
  L.h = take(R * (size_t)I * 4);
  L.y = take(R * (size_t)H * 4);
  L.total = off;
  return L;
}

int check_router_dims(int T, int H, int E, int top_k) {
  if (T < 0) return fail(PHMOE_ERR_INVALID_ARG, "T must be >= 0 (got %d)", T);
  if (H <= 0 || H % 8) return fail(PHMOE_ERR_INVALID_ARG, "H must be a positive multiple of 8 (got %d)", H);
  if (E < 1 || E > 1024) return fail(PHMOE_ERR_INVALID_ARG, "E must be in [1, 1024] (got %d)", E);
  if (top_k < 1 || top_k > E || top_k > 32)
    return fail(PHMOE_ERR_INVALID_ARG, "top_k must be in [1, min(E, 32)] (got %d, E=%d)", top_k, E);
  return PHMOE_OK;
}

// The router stages an 8-token tile of x in shared memory (227 KB per CTA).
int check_router_smem(int H, int x_dtype) {
  (void)x_dtype;  // the router stages a 4- to 32-token tile as fp32 whatever the input type
  const size_t bytes = (size_t)4 * ((H + 255) / 256 * 256) * 4;
  if (bytes > 232448)
    return fail(PHMOE_ERR_UNSUPPORTED, "H=%d too large for the router's token tile", H);
  return PHMOE_OK;
}

// The FFN kernels copy scales in pairs of groups (4-byte async copies), load
// gate/up weights as TMA boxes of 128-byte K-chunks (H % 256) and tile the
// down projection in 128-row blocks.
int check_ffn_dims(int H, int I, int G) {
  if (G != 32 && G != 64) return fail(PHMOE_ERR_UNSUPPORTED, "group_size must be 32 or 64 (got %d)", G);
  if (H <= 0 || H % 256)
    return fail(PHMOE_ERR_UNSUPPORTED, "H must be a positive multiple of 256 (got %d)", H);
  if (I <= 0 || I % 16 || I % (2 * G))
    return fail(PHMOE_ERR_UNSUPPORTED, "I must be a positive multiple of 16 and of 2*group_size (got %d)", I);
  return PHMOE_OK;
}

// The prefill GEMMs take bf16 activations, tile output columns by 256 (down)
// and 128 (gate/up, with the 128 matching up rows) and K by 64.
int check_prefill_dims(int x_dtype, int H, int I, int G, int E) {
  if (x_dtype != PHMOE_DTYPE_BF16) return fail(PHMOE_ERR_UNSUPPORTED, "the prefill path takes bf16 activations");
  if (G != 32 && G != 64) return fail(PHMOE_ERR_UNSUPPORTED, "group_size must be 32 or 64 (got %d)", G);
  if (H <= 0 || H % 256) return fail(PHMOE_ERR_UNSUPPORTED, "prefill needs H %% 256 == 0 (got %d)", H);
  if (I <= 0 || I % 128) return fail(PHMOE_ERR_UNSUPPORTED, "prefill needs I %% 128 == 0 (got %d)", I);
  if (!prefill_supported(H, I, G, E)) return fail(PHMOE_ERR_UNSUPPORTED, "prefill not built for E=%d", E);
  return PHMOE_OK;
}

// Average rows per expert from which PHMOE_PATH_AUTO takes the prefill GEMMs.
constexpr int kPrefillRowsPerExpert = 64;

// Resolves PHMOE_PATH_AUTO and checks the chosen path's limits.
int resolve_path(int path, int x_dtype, int T, int top_k, int H, int I, int G, int E, int* chosen) {
  if (path < PHMOE_PATH_AUTO || path > PHMOE_PATH_PREFILL)
    return fail(PHMOE_ERR_INVALID_ARG, "bad path code %d", path);
  if (path == PHMOE_PATH_AUTO) {
    const bool g_ok = G == 32 || G == 64;
    const bool prefill_ok = g_ok && x_dtype == PHMOE_DTYPE_BF16 && H % 256 == 0 && I % 128 == 0 &&
                            prefill_supported(H, I, G, E);
    const bool decode_ok = g_ok && H % 256 == 0 && I % 16 == 0 && I % (2 * G) == 0;
    const bool big = (long long)T * top_k >= (long long)kPrefillRowsPerExpert * E;
    path = (prefill_ok && (big || !decode_ok)) ? PHMOE_PATH_PREFILL : PHMOE_PATH_DECODE;
  }
  *chosen = path;
  return path == PHMOE_PATH_PREFILL ? check_prefill_dims(x_dtype, H, I, G, E) : check_ffn_dims(H, I, G);
}

}  // namespace

namespace {
std::atomic<unsigned long long> g_launches{0};

// Stage-timing events for phmoe_profile_begin/end (process-global).
struct Profile {
  int max_calls = 0;
  int calls = 0;
  std::vector<cudaEvent_t> ev;  // max_calls * (PHMOE_NUM_STAGES + 1)
};
Profile g_prof;

cudaEvent_t prof_event(int call, int boundary) {
  return g_prof.ev[(size_t)call * (PHMOE_NUM_STAGES + 1) + boundary];
}
}  // namespace

void note_launches(int n) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }

int device_sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

int record_error(int status, const char* msg) { return fail(status, "%s", msg); }

}  // namespace phmoe

using namespace phmoe;

extern "C" {

int phmoe_version(void) { return 100; }

const char* phmoe_status_string(int status) {
  switch (status) {
    case PHMOE_OK: return "ok";
    case PHMOE_ERR_INVALID_ARG: return "invalid argument";
    case PHMOE_ERR_UNSUPPORTED: return "unsupported shape or dtype";
    case PHMOE_ERR_WORKSPACE: return "workspace too small or misaligned";
    case PHMOE_ERR_CUDA: return "CUDA error";
    case PHMOE_ERR_ALIGNMENT: return "pointer not 16-byte aligned";
    default: return "unknown status";
  }
}

const char* phmoe_last_error(void) { return g_last_error.c_str(); }

int phmoe_select_path(int path, int x_dtype, int T, int top_k, int H, int E, int I, int group_size) {
  g_last_error.clear();
  if (int s = check_router_dims(T, H, E, top_k)) return s;
  if (!dtype_ok(x_dtype)) return fail(PHMOE_ERR_INVALID_ARG, "bad dtype code");
  int chosen = PHMOE_PATH_DECODE;
  if (int s = resolve_path(path, x_dtype, T, top_k, H, I, group_size, E, &chosen)) return s;
  return chosen;
}

size_t phmoe_workspace_size(int T, int H, int E, int top_k, int I, int path) {
  if (T < 0 || H <= 0 || E < 1 || top_k < 1 || I <= 0) return 0;
  if (path < PHMOE_PATH_AUTO || path > PHMOE_PATH_PREFILL) return 0;
  return make_layout(T, H, E, top_k, I).total;
}

int phmoe_router(const void* x, int x_dtype, const void* router_w, int w_dtype, int T, int H,
                 int E, int top_k, int renormalize, float* logits, float* probs,
                 int32_t* topk_idx, float* topk_w, void* stream) {
  g_last_error.clear();
  if (int s = check_router_dims(T, H, E, top_k)) return s;
  if (!dtype_ok(x_dtype) || !dtype_ok(w_dtype)) return fail(PHMOE_ERR_INVALID_ARG, "bad dtype code");
  if (int s = check_router_smem(H, x_dtype)) return s;
  if (T == 0) return PHMOE_OK;
  if (!x || !router_w || !logits || !topk_idx || !topk_w)
    return fail(PHMOE_ERR_INVALID_ARG, "null pointer argument");
  if (!aligned(x, 16) || !aligned(router_w, 16))
    return fail(PHMOE_ERR_ALIGNMENT, "x and router_w must be 16-byte aligned");
  launch_router(x, x_dtype, router_w, w_dtype, T, H, E, top_k, renormalize, logits, probs, topk_idx,
                topk_w, static_cast<cudaStream_t>(stream));
  return check_launch("phmoe_router");
}

size_t phmoe_dispatch_scratch_size(int T, int top_k, int E) {
  if (T < 0 || top_k < 1 || E < 1) return 0;
  return dispatch_scratch_bytes(T, top_k, E);
}

int phmoe_dispatch(const int32_t* topk_idx, int T, int top_k, int E, int32_t* expert_offsets,
                   int32_t* row_token, int32_t* inv, int32_t* active, void* scratch,
                   size_t scratch_bytes, void* stream) {
  g_last_error.clear();
  if (T < 0 || top_k < 1 || top_k > 32 || E < 1 || E > 1024)
    return fail(PHMOE_ERR_INVALID_ARG, "bad dispatch dims T=%d k=%d E=%d", T, top_k, E);
  if (!expert_offsets || !active) return fail(PHMOE_ERR_INVALID_ARG, "null pointer argument");
  if (T > 0 && (!topk_idx || !row_token || !inv)) return fail(PHMOE_ERR_INVALID_ARG, "null pointer argument");
  const size_t need = dispatch_scratch_bytes(T, top_k, E);
  if (scratch_bytes < need || (need && !scratch))
    return fail(PHMOE_ERR_WORKSPACE, "dispatch scratch needs %zu bytes", need);
  launch_dispatch(topk_idx, T, top_k, E, expert_offsets, row_token, inv, active, scratch,
                  static_cast<cudaStream_t>(stream));
  return check_launch("phmoe_dispatch");
}

int phmoe_expert_ffn_decode(const void* x, int x_dtype, const int32_t* row_token,
                            const int32_t* expert_offsets, const int32_t* active,
                            const uint8_t* w13_q, const uint16_t* w13_s, const uint8_t* w2_q,
                            const uint16_t* w2_s, int T, int H, int E, int top_k, int I,
                            int group_size, float* h, float* y, void* stream) {
  g_last_error.clear();
  if (int s = check_router_dims(T, H, E, top_k)) return s;
  if (int s = check_ffn_dims(H, I, group_size)) return s;
  if (!dtype_ok(x_dtype)) return fail(PHMOE_ERR_INVALID_ARG, "bad dtype code");
  if (T == 0) return PHMOE_OK;
  if (!x || !row_token || !expert_offsets || !active || !w13_q || !w13_s || !w2_q || !w2_s || !h || !y)
    return fail(PHMOE_ERR_INVALID_ARG, "null pointer argument");
  if (!aligned(x, 16) || !aligned(w13_q, 16) || !aligned(w2_q, 16) || !aligned(h, 16) || !aligned(y, 16))
    return fail(PHMOE_ERR_ALIGNMENT, "x, weights, h and y must be 16-byte aligned");
  if (!aligned(w13_s, 4) || !aligned(w2_s, 4)) return fail(PHMOE_ERR_ALIGNMENT, "scales must be 4-byte aligned");
  const int s = launch_ffn_decode(x, x_dtype, row_token, expert_offsets, active, w13_q, w13_s, w2_q,
                                  w2_s, T, H, E, top_k, I, group_size, h, y,
                                  static_cast<cudaStream_t>(stream));
  if (s) return fail(s, "no decode kernel for group_size=%d", group_size);
  return check_launch("phmoe_expert_ffn_decode");
}

int phmoe_expert_ffn_prefill(const void* x, int x_dtype, const int32_t* row_token,
                             const int32_t* expert_offsets, const int32_t* active,
                             const uint8_t* w13_q, const uint16_t* w13_s, const uint8_t* w2_q,
                             const uint16_t* w2_s, int T, int H, int E, int top_k, int I,
                             int group_size, float* h, float* y, void* stream) {
  g_last_error.clear();
  if (int s = check_router_dims(T, H, E, top_k)) return s;
  if (int s = check_prefill_dims(x_dtype, H, I, group_size, E)) return s;
  if (T == 0) return PHMOE_OK;
  if (!x || !row_token || !expert_offsets || !active || !w13_q || !w13_s || !w2_q || !w2_s || !h || !y)
    return fail(PHMOE_ERR_INVALID_ARG, "null pointer argument");
  if (!aligned(x, 16) || !aligned(w13_q, 16) || !aligned(w2_q, 16) || !aligned(h, 16) || !aligned(y, 16))
    return fail(PHMOE_ERR_ALIGNMENT, "x, weights, h and y must be 16-byte aligned");
  if (!aligned(w13_s, 2) || !aligned(w2_s, 2)) return fail(PHMOE_ERR_ALIGNMENT, "scales must be 2-byte aligned");
  const int s = launch_ffn_prefill(x, row_token, expert_offsets, active, w13_q, w13_s, w2_q, w2_s, T, H, E,
                                   top_k, I, group_size, h, y, static_cast<cudaStream_t>(stream));
  if (s) return fail(s, "prefill launch failed (tensor map or kernel attribute)");
  return check_launch("phmoe_expert_ffn_prefill");
}

size_t phmoe_fx_rows_size(long long rows, int K, int group_size) {
  if (rows < 0 || K <= 0 || (group_size != 32 && group_size != 64) || K % group_size) return 0;
  return fx_rows_bytes(rows, K, group_size);
}

int phmoe_fx_rows(const void* x, int x_dtype, long long rows, int K, int group_size, void* out, void* stream) {
  g_last_error.clear();
  if (!dtype_ok(x_dtype)) return fail(PHMOE_ERR_INVALID_ARG, "bad dtype code");
  if (group_size != 32 && group_size != 64) return fail(PHMOE_ERR_UNSUPPORTED, "group_size must be 32 or 64");
  if (rows < 0 || K <= 0 || K % group_size)
    return fail(PHMOE_ERR_INVALID_ARG, "K must be a positive multiple of group_size (got %d)", K);
  if (rows == 0) return PHMOE_OK;
  if (!x || !out) return fail(PHMOE_ERR_INVALID_ARG, "null pointer argument");
  if (!aligned(x, 16) || !aligned(out, 256)) return fail(PHMOE_ERR_ALIGNMENT, "x must be 16- and out 256-byte aligned");
  uint8_t* q = static_cast<uint8_t*>(out);
  int2* consts = reinterpret_cast<int2*>(q + (fx_rows_bytes(rows, K, group_size) - (size_t)rows * (K / group_size) * 8));
  if (int st = launch_fx_rows(x, x_dtype, rows, K, group_size, nullptr, nullptr, q, consts,
                              static_cast<cudaStream_t>(stream)))
    return fail(st, "fx row encoding not built for these arguments");
  return check_launch("phmoe_fx_rows");
}

int phmoe_combine(const float* y, const int32_t* inv, const float* topk_w, int T, int top_k,
                  int H, void* out, int out_dtype, void* stream) {
  g_last_error.clear();
  if (T < 0 || top_k < 1 || top_k > 32 || H <= 0 || H % 4)
    return fail(PHMOE_ERR_INVALID_ARG, "bad combine dims T=%d k=%d H=%d", T, top_k, H);
  if (!dtype_ok(out_dtype)) return fail(PHMOE_ERR_INVALID_ARG, "bad dtype code");
  if (T == 0) return PHMOE_OK;
  if (!y || !inv || !topk_w || !out) return fail(PHMOE_ERR_INVALID_ARG, "null pointer argument");
  if (!aligned(y, 16) || !aligned(out, 16)) return fail(PHMOE_ERR_ALIGNMENT, "y and out must be 16-byte aligned");
  launch_combine(y, inv, topk_w, T, top_k, H, out, out_dtype, static_cast<cudaStream_t>(stream));
  return check_launch("phmoe_combine");
}

int phmoe_gather_rows(const void* src, long long src_rows, const int32_t* index, int n_rows,
                      long long row_bytes, void* dst, void* stream) {
  g_last_error.clear();
  if (n_rows < 0 || src_rows < 0 || row_bytes <= 0 || row_bytes % 16 || row_bytes / 16 > (1LL << 30))
    return fail(PHMOE_ERR_INVALID_ARG, "bad gather dims n_rows=%d src_rows=%lld row_bytes=%lld", n_rows,
                src_rows, row_bytes);
  if (n_rows == 0) return PHMOE_OK;
  if (!index || !dst || (src_rows > 0 && !src)) return fail(PHMOE_ERR_INVALID_ARG, "null pointer argument");
  if (!aligned(src, 16) || !aligned(dst, 16)) return fail(PHMOE_ERR_ALIGNMENT, "src and dst must be 16-byte aligned");
  launch_gather_rows(src, src_rows, index, n_rows, row_bytes, dst, static_cast<cudaStream_t>(stream));
  return check_launch("phmoe_gather_rows");
}

int phmoe_moe_layer(const void* x, int x_dtype, const void* router_w, int w_dtype,
                    const uint8_t* w13_q, const uint16_t* w13_s, const uint8_t* w2_q,
                    const uint16_t* w2_s, int T, int H, int E, int top_k, int I,
                    int group_size, int renormalize, int path, void* out, int32_t* topk_idx_out,
                    float* topk_w_out, void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  if (int s = check_router_dims(T, H, E, top_k)) return s;
  if (!dtype_ok(x_dtype) || !dtype_ok(w_dtype)) return fail(PHMOE_ERR_INVALID_ARG, "bad dtype code");
  int chosen = PHMOE_PATH_DECODE;
  if (int s = resolve_path(path, x_dtype, T, top_k, H, I, group_size, E, &chosen)) return s;
  if (int s = check_router_smem(H, x_dtype)) return s;
  if (T == 0) return PHMOE_OK;
  if (!x || !router_w || !w13_q || !w13_s || !w2_q || !w2_s || !out || !workspace)
    return fail(PHMOE_ERR_INVALID_ARG, "null pointer argument");
  if (!aligned(x, 16) || !aligned(router_w, 16) || !aligned(w13_q, 16) || !aligned(w2_q, 16) || !aligned(out, 16))
    return fail(PHMOE_ERR_ALIGNMENT, "x, router_w, packed weights and out must be 16-byte aligned");
  if (!aligned(w13_s, 4) || !aligned(w2_s, 4)) return fail(PHMOE_ERR_ALIGNMENT, "scales must be 4-byte aligned");
  const Layout L = make_layout(T, H, E, top_k, I);
  if (!aligned(workspace, kAlign)) return fail(PHMOE_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  if (workspace_bytes < L.total)
    return fail(PHMOE_ERR_WORKSPACE, "workspace needs %zu bytes (got %zu)", L.total, workspace_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  float* logits = reinterpret_cast<float*>(ws + L.logits);
  int32_t* idx = topk_idx_out ? topk_idx_out : reinterpret_cast<int32_t*>(ws + L.idx);
  float* wts = topk_w_out ? topk_w_out : reinterpret_cast<float*>(ws + L.w);
  int32_t* offsets = reinterpret_cast<int32_t*>(ws + L.offsets);
  int32_t* active = reinterpret_cast<int32_t*>(ws + L.active);
  int32_t* row_token = reinterpret_cast<int32_t*>(ws + L.row_token);
  int32_t* inv = reinterpret_cast<int32_t*>(ws + L.inv);
  float* h = reinterpret_cast<float*>(ws + L.h);
  float* y = reinterpret_cast<float*>(ws + L.y);

  const bool prof = g_prof.calls < g_prof.max_calls;
  const int pc = g_prof.calls;
  auto mark = [&](int b) { if (prof) cudaEventRecord(prof_event(pc, b), st); };

  mark(0);
  const bool decode = chosen != PHMOE_PATH_PREFILL;
  const DispatchOut disp{offsets, row_token, inv, active};
  const int rflags =
      launch_router(x, x_dtype, router_w, w_dtype, T, H, E, top_k, renormalize, logits, nullptr, idx, wts, st,
                    group_size, decode ? ffn_decode_xq(y) : nullptr, decode ? ffn_decode_xc(y, T, H) : nullptr, &disp);
  const bool x_encoded = (rflags & kRouterEncodedX) != 0;
  if (int s = check_launch("router")) return s;
  mark(1);
  if (!(rflags & kRouterDispatched)) launch_dispatch(idx, T, top_k, E, offsets, row_token, inv, active, ws + L.disp, st);
  if (int s = check_launch("dispatch")) return s;
  mark(2);
  if (chosen == PHMOE_PATH_PREFILL) {
    if (int s = launch_ffn_prefill(x, row_token, offsets, active, w13_q, w13_s, w2_q, w2_s, T, H, E, top_k, I,
                                   group_size, h, y, st, prof ? prof_event(pc, 3) : nullptr))
      return fail(s, "prefill launch failed (tensor map or kernel attribute)");
  } else if (int s = launch_ffn_decode(x, x_dtype, row_token, offsets, active, w13_q, w13_s, w2_q, w2_s, T, H,
                                       E, top_k, I, group_size, h, y, st, prof ? prof_event(pc, 3) : nullptr,
                                       nullptr, nullptr, x_encoded)) {
    return fail(s, "no decode kernel for group_size=%d", group_size);
  }
  if (int s = check_launch("expert_ffn")) return s;
  mark(4);
  launch_combine(y, inv, wts, T, top_k, H, out, x_dtype, st);
  mark(5);
  if (prof) g_prof.calls++;
  return check_launch("combine");
}

size_t phmoe_workspace_size_ex(int T, int H, int E, int top_k, int I, int num_shared, int path) {
  if (T < 0 || H <= 0 || E < 1 || top_k < 1 || I <= 0 || num_shared < 0) return 0;
  if (path < PHMOE_PATH_AUTO || path > PHMOE_PATH_PREFILL) return 0;
  // the whole layer over E + m experts and k + m slots, plus the router's [T, k] choice
  return make_layout(T, H, E + num_shared, top_k + num_shared, I).total + round_up((size_t)T * top_k * 8, kAlign);
}

// Checks of the extended router options; PHMOE_OK when valid.
int check_routing_ex(int E, int scoring, int n_group, int topk_group, float routed_scale) {
  if (scoring != PHMOE_SCORING_SOFTMAX && scoring != PHMOE_SCORING_SIGMOID)
    return fail(PHMOE_ERR_INVALID_ARG, "bad scoring code %d", scoring);
  if (n_group > 1) {
    if (scoring != PHMOE_SCORING_SIGMOID)
      return fail(PHMOE_ERR_UNSUPPORTED, "group-limited routing is implemented for sigmoid scoring");
    if (n_group > 32 || E % n_group || E / n_group < 2)
      return fail(PHMOE_ERR_INVALID_ARG, "n_group must divide E into groups of >= 2 experts (n_group <= 32)");
    if (topk_group < 1 || topk_group > n_group)
      return fail(PHMOE_ERR_INVALID_ARG, "topk_group must be in [1, n_group]");
  }
  if (!(routed_scale > 0.f)) return fail(PHMOE_ERR_INVALID_ARG, "routed_scale must be > 0");
  return PHMOE_OK;
}

void route_ex(const void* x, int x_dtype, const void* router_w, int w_dtype, int T, int H, int E, int top_k,
              int renormalize, int scoring, const float* score_bias, int n_group, int topk_group, float scale,
              float* logits, int32_t* idx, float* w, cudaStream_t st) {
  if (scoring == PHMOE_SCORING_SOFTMAX && n_group <= 1 && !score_bias && scale == 1.0f)
    launch_router(x, x_dtype, router_w, w_dtype, T, H, E, top_k, renormalize, logits, nullptr, idx, w, st);
  else
    launch_router_grouped(x, x_dtype, router_w, w_dtype, T, H, E, top_k, renormalize, score_bias,
                          scoring == PHMOE_SCORING_SIGMOID ? n_group : 1, topk_group, scale, logits, idx, w, st);
}

int phmoe_router_ex(const void* x, int x_dtype, const void* router_w, int w_dtype, int T, int H,
                    int E, int top_k, int renormalize, int scoring, const float* score_bias,
                    int n_group, int topk_group, float routed_scale, float* logits,
                    int32_t* topk_idx, float* topk_w, void* stream) {
  g_last_error.clear();
  if (int s = check_router_dims(T, H, E, top_k)) return s;
  if (int s = check_routing_ex(E, scoring, n_group, topk_group, routed_scale)) return s;
  if (scoring == PHMOE_SCORING_SOFTMAX && (score_bias || routed_scale != 1.0f))
    return fail(PHMOE_ERR_UNSUPPORTED, "score_bias and routed_scale apply to sigmoid scoring");
  if (!dtype_ok(x_dtype) || !dtype_ok(w_dtype)) return fail(PHMOE_ERR_INVALID_ARG, "bad dtype code");
  if (int s = check_router_smem(H, x_dtype)) return s;
  if (T == 0) return PHMOE_OK;
  if (!x || !router_w || !logits || !topk_idx || !topk_w) return fail(PHMOE_ERR_INVALID_ARG, "null pointer argument");
  if (!aligned(x, 16) || !aligned(router_w, 16)) return fail(PHMOE_ERR_ALIGNMENT, "x and router_w must be 16-byte aligned");
  route_ex(x, x_dtype, router_w, w_dtype, T, H, E, top_k, renormalize, scoring, score_bias, n_group, topk_group,
           routed_scale, logits, topk_idx, topk_w, static_cast<cudaStream_t>(stream));
  return check_launch("phmoe_router_ex");
}

int phmoe_moe_layer_ex(const void* x, int x_dtype, const void* router_w, int w_dtype,
                       const uint8_t* w13_q, const uint16_t* w13_s, const uint8_t* w2_q,
                       const uint16_t* w2_s, int T, int H, int E, int top_k, int I,
                       int group_size, int renormalize, int scoring, const float* score_bias,
                       int n_group, int topk_group, int num_shared, const void* shared_gate_w,
                       float routed_scale, int path, void* out, int32_t* topk_idx_out,
                       float* topk_w_out, void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  if (num_shared < 0 || num_shared > 32) return fail(PHMOE_ERR_INVALID_ARG, "num_shared must be in [0, 32]");
  if (int s = check_router_dims(T, H, E, top_k)) return s;
  if (int s = check_routing_ex(E, scoring, n_group, topk_group, routed_scale)) return s;
  if (!dtype_ok(x_dtype) || !dtype_ok(w_dtype)) return fail(PHMOE_ERR_INVALID_ARG, "bad dtype code");
  const int Et = E + num_shared, kt = top_k + num_shared;
  if (Et > 1024) return fail(PHMOE_ERR_INVALID_ARG, "E + num_shared must be <= 1024");
  int chosen = PHMOE_PATH_DECODE;
  if (int s = resolve_path(path, x_dtype, T, kt, H, I, group_size, Et, &chosen)) return s;
  if (int s = check_router_smem(H, x_dtype)) return s;
  if (T == 0) return PHMOE_OK;
  if (!x || !router_w || !w13_q || !w13_s || !w2_q || !w2_s || !out || !workspace)
    return fail(PHMOE_ERR_INVALID_ARG, "null pointer argument");
  if (!aligned(x, 16) || !aligned(router_w, 16) || !aligned(w13_q, 16) || !aligned(w2_q, 16) || !aligned(out, 16) ||
      (shared_gate_w && !aligned(shared_gate_w, 16)))
    return fail(PHMOE_ERR_ALIGNMENT, "x, router_w, shared_gate_w, packed weights and out must be 16-byte aligned");
  if (!aligned(w13_s, 4) || !aligned(w2_s, 4)) return fail(PHMOE_ERR_ALIGNMENT, "scales must be 4-byte aligned");
  const Layout L = make_layout(T, H, Et, kt, I);
  const size_t need = phmoe_workspace_size_ex(T, H, E, top_k, I, num_shared, path);
  if (!aligned(workspace, kAlign)) return fail(PHMOE_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  if (workspace_bytes < need) return fail(PHMOE_ERR_WORKSPACE, "workspace needs %zu bytes (got %zu)", need, workspace_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  float* logits = reinterpret_cast<float*>(ws + L.logits);  // [T, Et] >= [T, E]
  int32_t* r_idx = topk_idx_out ? topk_idx_out : reinterpret_cast<int32_t*>(ws + L.total);
  float* r_w = topk_w_out ? topk_w_out : reinterpret_cast<float*>(ws + L.total + (size_t)T * top_k * 4);
  int32_t* idx = reinterpret_cast<int32_t*>(ws + L.idx);
  float* wts = reinterpret_cast<float*>(ws + L.w);
  int32_t* offsets = reinterpret_cast<int32_t*>(ws + L.offsets);
  int32_t* active = reinterpret_cast<int32_t*>(ws + L.active);
  int32_t* row_token = reinterpret_cast<int32_t*>(ws + L.row_token);
  int32_t* inv = reinterpret_cast<int32_t*>(ws + L.inv);
  float* h = reinterpret_cast<float*>(ws + L.h);
  float* y = reinterpret_cast<float*>(ws + L.y);

  route_ex(x, x_dtype, router_w, w_dtype, T, H, E, top_k, renormalize, scoring, score_bias, n_group, topk_group,
           1.0f, logits, r_idx, r_w, st);
  if (int s = check_launch("router")) return s;
  launch_shared_slots(x, x_dtype, shared_gate_w, w_dtype, r_idx, r_w, T, H, top_k, E, num_shared, routed_scale,
                      idx, wts, st);
  if (int s = check_launch("shared_slots")) return s;
  launch_dispatch(idx, T, kt, Et, offsets, row_token, inv, active, ws + L.disp, st);
  if (int s = check_launch("dispatch")) return s;
  if (chosen == PHMOE_PATH_PREFILL) {
    if (int s = launch_ffn_prefill(x, row_token, offsets, active, w13_q, w13_s, w2_q, w2_s, T, H, Et, kt, I,
                                   group_size, h, y, st, nullptr))
      return fail(s, "prefill launch failed (tensor map or kernel attribute)");
  } else if (int s = launch_ffn_decode(x, x_dtype, row_token, offsets, active, w13_q, w13_s, w2_q, w2_s, T, H,
                                       Et, kt, I, group_size, h, y, st, nullptr)) {
    return fail(s, "no decode kernel for group_size=%d", group_size);
  }
  if (int s = check_launch("expert_ffn")) return s;
  launch_combine(y, inv, wts, T, kt, H, out, x_dtype, st);
  return check_launch("combine");
}

int phmoe_quantize_int4(const void* w, int w_dtype, long long rows, int K, int group_size,
                        uint8_t* packed, uint16_t* scales, void* stream) {
  g_last_error.clear();
  if (!dtype_ok(w_dtype)) return fail(PHMOE_ERR_INVALID_ARG, "bad dtype code");
  if (group_size != 32 && group_size != 64) return fail(PHMOE_ERR_UNSUPPORTED, "group_size must be 32 or 64");
  if (rows < 0 || K <= 0 || K % group_size) return fail(PHMOE_ERR_INVALID_ARG, "K must be a positive multiple of group_size");
  if (rows == 0) return PHMOE_OK;
  if (!w || !packed || !scales) return fail(PHMOE_ERR_INVALID_ARG, "null pointer argument");
  launch_quantize(w, w_dtype, rows, K, group_size, packed, scales, static_cast<cudaStream_t>(stream));
  return check_launch("phmoe_quantize_int4");
}

int phmoe_gguf_q4_0_to_packed(const void* blocks, long long rows, int K, uint8_t* packed,
                              uint16_t* scales, void* stream) {
  g_last_error.clear();
  if (rows < 0 || K <= 0 || K % 32) return fail(PHMOE_ERR_INVALID_ARG, "K must be a positive multiple of 32");
  if (rows == 0) return PHMOE_OK;
  if (!blocks || !packed || !scales) return fail(PHMOE_ERR_INVALID_ARG, "null pointer argument");
  if (!aligned(blocks, 2) || !aligned(packed, 16) || !aligned(scales, 2))
    return fail(PHMOE_ERR_ALIGNMENT, "blocks must be 2-byte, packed 16-byte and scales 2-byte aligned");
  launch_gguf_q4_0(blocks, rows, K, packed, scales, static_cast<cudaStream_t>(stream));
  return check_launch("phmoe_gguf_q4_0_to_packed");
}

int phmoe_gguf_q4_k_to_packed(const void* blocks, long long rows, int K, int group_size,
                              uint8_t* packed, uint16_t* scales, void* stream) {
  g_last_error.clear();
  if (group_size != 32 && group_size != 64) return fail(PHMOE_ERR_UNSUPPORTED, "group_size must be 32 or 64");
  if (rows < 0 || K <= 0 || K % 256) return fail(PHMOE_ERR_INVALID_ARG, "K must be a positive multiple of 256");
  if (rows == 0) return PHMOE_OK;
  if (!blocks || !packed || !scales) return fail(PHMOE_ERR_INVALID_ARG, "null pointer argument");
  launch_gguf_q4_k(blocks, rows, K, group_size, packed, scales, static_cast<cudaStream_t>(stream));
  return check_launch("phmoe_gguf_q4_k_to_packed");
}

int phmoe_gguf_q4_k_dequantize(const void* blocks, long long n, float* out, void* stream) {
  g_last_error.clear();
  if (n < 0 || n % 256) return fail(PHMOE_ERR_INVALID_ARG, "n must be a non-negative multiple of 256");
  if (n == 0) return PHMOE_OK;
  if (!blocks || !out) return fail(PHMOE_ERR_INVALID_ARG, "null pointer argument");
  launch_gguf_q4_k_dequant(blocks, n, out, static_cast<cudaStream_t>(stream));
  return check_launch("phmoe_gguf_q4_k_dequantize");
}

unsigned long long phmoe_kernel_launch_count(void) { return g_launches.load(); }

int phmoe_device_error(int reset) {
  const int a = ffn_device_error(reset != 0);
  const int b = prefill_device_error(reset != 0);
  const int c = ep_device_error(reset != 0);
  const int d = router_device_error(reset != 0);
  if (a < 0 || b < 0 || c < 0 || d < 0) return -1;
  return a | b | c | d;
}

// ---- expert parallelism in peer memory ----

int phmoe_ep_create_ex(int rank, int world, int max_tokens, int top_k, int H, int E, int slots_per_rank,
                       int x_dtype, void** ctx, void* ipc_handle_out) {
  g_last_error.clear();
  if (!ctx || !ipc_handle_out) return fail(PHMOE_ERR_INVALID_ARG, "null pointer argument");
  *ctx = nullptr;
  if (!dtype_ok(x_dtype)) return fail(PHMOE_ERR_INVALID_ARG, "bad dtype code");
  if (world < 1 || world > PHMOE_EP_MAX_WORLD || rank < 0 || rank >= world)
    return fail(PHMOE_ERR_INVALID_ARG, "rank %d of world %d (world must be 1..%d)", rank, world, PHMOE_EP_MAX_WORLD);
  if (E < 1 || E > 1024 || E % world) return fail(PHMOE_ERR_INVALID_ARG, "E=%d must split evenly over %d ranks", E, world);
  if (max_tokens < 1 || top_k < 1 || top_k > E || top_k > 32 || H <= 0 || H % 8)
    return fail(PHMOE_ERR_INVALID_ARG, "bad dims max_tokens=%d top_k=%d H=%d", max_tokens, top_k, H);
  const int slots = slots_per_rank ? slots_per_rank : E / world;
  if (slots < E / world || (long long)slots * world > 1024)
    return fail(PHMOE_ERR_INVALID_ARG, "slots_per_rank=%d must be >= E/world=%d with world*slots <= 1024",
                slots_per_rank, E / world);
  EpContext* c = nullptr;
  const int s = ep_create(rank, world, max_tokens, top_k, H, E, slots, x_dtype == PHMOE_DTYPE_F32 ? 4 : 2, &c,
                          ipc_handle_out);
  if (s) return fail(s, "could not allocate or export the exchange region (%s)", cudaGetErrorString(cudaGetLastError()));
  *ctx = c;
  return PHMOE_OK;
}

int phmoe_ep_create(int rank, int world, int max_tokens, int top_k, int H, int E, int x_dtype, void** ctx,
                    void* ipc_handle_out) {
  return phmoe_ep_create_ex(rank, world, max_tokens, top_k, H, E, 0, x_dtype, ctx, ipc_handle_out);
}

int phmoe_ep_connect(void* ctx, const void* ipc_handles) {
  g_last_error.clear();
  if (!ctx || !ipc_handles) return fail(PHMOE_ERR_INVALID_ARG, "null pointer argument");
  if (int s = ep_connect(static_cast<EpContext*>(ctx), ipc_handles))
    return fail(s, "could not open a peer's exchange region (%s)", cudaGetErrorString(cudaGetLastError()));
  return PHMOE_OK;
}

int phmoe_ep_destroy(void* ctx) {
  g_last_error.clear();
  ep_destroy(static_cast<EpContext*>(ctx));
  return PHMOE_OK;
}

size_t phmoe_ep_workspace_size(const void* ctx, int I) {
  if (!ctx || I <= 0) return 0;
  return ep_workspace_bytes(static_cast<const EpContext*>(ctx), I);
}

int phmoe_ep_layer_ex(void* ctx, const void* x, int x_dtype, const void* router_w, int w_dtype,
                      const uint8_t* w13_q, const uint16_t* w13_s, const uint8_t* w2_q, const uint16_t* w2_s, int T,
                      int I, int group_size, int renormalize, int path, const int32_t* vmap, void* out,
                      int32_t* topk_idx_out, float* topk_w_out, void* workspace, size_t workspace_bytes,
                      void* stream) {
  g_last_error.clear();
  if (!ctx) return fail(PHMOE_ERR_INVALID_ARG, "null context");
  EpContext* c = static_cast<EpContext*>(ctx);
  int rank, world, max_tokens, top_k, H, E;
  if (!ep_info(c, &rank, &world, &max_tokens, &top_k, &H, &E))
    return fail(PHMOE_ERR_INVALID_ARG, "context not connected (phmoe_ep_connect)");
  const int slots = ep_slots(c);
  if (!vmap && slots != E / world)
    return fail(PHMOE_ERR_INVALID_ARG, "a context with %d slots per rank (E/world = %d) needs the expert map",
                slots, E / world);
  if (vmap && !aligned(vmap, 4)) return fail(PHMOE_ERR_ALIGNMENT, "vmap must be 4-byte aligned");
  if (T < 0 || T > max_tokens) return fail(PHMOE_ERR_INVALID_ARG, "T=%d outside [0, %d]", T, max_tokens);
  if (!dtype_ok(x_dtype) || !dtype_ok(w_dtype)) return fail(PHMOE_ERR_INVALID_ARG, "bad dtype code");
  if (int s = check_router_smem(H, x_dtype)) return s;
  // the path is chosen for the rows a rank expects (T*k over its local slots)
  int chosen = PHMOE_PATH_DECODE;
  if (int s = resolve_path(path, x_dtype, T > 0 ? T : 1, top_k, H, I, group_size, slots, &chosen)) return s;
  if ((T > 0 && (!x || !router_w || !out)) || !w13_q || !w13_s || !w2_q || !w2_s || !workspace)
    return fail(PHMOE_ERR_INVALID_ARG, "null pointer argument");
  if (!aligned(x, 16) || !aligned(router_w, 16) || !aligned(w13_q, 16) || !aligned(w2_q, 16) || !aligned(out, 16))
    return fail(PHMOE_ERR_ALIGNMENT, "x, router_w, packed weights and out must be 16-byte aligned");
  if (!aligned(w13_s, 4) || !aligned(w2_s, 4)) return fail(PHMOE_ERR_ALIGNMENT, "scales must be 4-byte aligned");
  if (!aligned(workspace, kAlign)) return fail(PHMOE_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  const size_t need = ep_workspace_bytes(c, I);
  if (workspace_bytes < need) return fail(PHMOE_ERR_WORKSPACE, "workspace needs %zu bytes (got %zu)", need, workspace_bytes);
  // stage events as phmoe_moe_layer records them; here stage 1 also holds the
  // row exchange out, stage 4 the return of the results
  const bool prof = g_prof.calls < g_prof.max_calls;
  cudaEvent_t marks[PHMOE_NUM_STAGES + 1] = {};
  if (prof)
    for (int b = 0; b <= PHMOE_NUM_STAGES; ++b) marks[b] = prof_event(g_prof.calls, b);
  const int s = ep_layer(c, x, x_dtype, router_w, w_dtype, w13_q, w13_s, w2_q, w2_s, T, I, group_size, renormalize,
                         chosen, out, topk_idx_out, topk_w_out, workspace, static_cast<cudaStream_t>(stream),
                         prof ? marks : nullptr, vmap);
  if (prof) g_prof.calls++;
  if (s) return fail(s, "expert FFN launch failed");
  return check_launch("phmoe_ep_layer");
}

int phmoe_ep_layer(void* ctx, const void* x, int x_dtype, const void* router_w, int w_dtype, const uint8_t* w13_q,
                   const uint16_t* w13_s, const uint8_t* w2_q, const uint16_t* w2_s, int T, int I, int group_size,
                   int renormalize, int path, void* out, int32_t* topk_idx_out, float* topk_w_out, void* workspace,
                   size_t workspace_bytes, void* stream) {
  return phmoe_ep_layer_ex(ctx, x, x_dtype, router_w, w_dtype, w13_q, w13_s, w2_q, w2_s, T, I, group_size,
                           renormalize, path, nullptr, out, topk_idx_out, topk_w_out, workspace, workspace_bytes,
                           stream);
}

int phmoe_profile_begin(int max_calls) {
  g_last_error.clear();
  if (max_calls < 0 || max_calls > (1 << 20)) return fail(PHMOE_ERR_INVALID_ARG, "bad max_calls %d", max_calls);
  for (cudaEvent_t e : g_prof.ev) cudaEventDestroy(e);
  g_prof = Profile{};
  g_prof.ev.resize((size_t)max_calls * (PHMOE_NUM_STAGES + 1));
  for (auto& e : g_prof.ev) {
    const cudaError_t err = cudaEventCreate(&e);
    if (err != cudaSuccess) {
      g_prof.ev.clear();
      return fail(PHMOE_ERR_CUDA, "cudaEventCreate: %s", cudaGetErrorString(err));
    }
  }
  g_prof.max_calls = max_calls;
  return PHMOE_OK;
}

int phmoe_profile_end(float* stage_ms, int n_stages, int* calls) {
  g_last_error.clear();
  int status = PHMOE_OK;
  if (stage_ms)
    for (int s = 0; s < n_stages; ++s) stage_ms[s] = 0.f;
  const int n = g_prof.calls;
  if (n > 0) {
    const cudaError_t err = cudaEventSynchronize(prof_event(n - 1, PHMOE_NUM_STAGES));
    if (err != cudaSuccess) status = fail(PHMOE_ERR_CUDA, "cudaEventSynchronize: %s", cudaGetErrorString(err));
  }
  for (int c = 0; c < n && status == PHMOE_OK; ++c)
    for (int s = 0; s < PHMOE_NUM_STAGES && s < n_stages; ++s) {
      float ms = 0.f;
      if (cudaEventElapsedTime(&ms, prof_event(c, s), prof_event(c, s + 1)) == cudaSuccess && stage_ms)
        stage_ms[s] += ms;
    }
  if (calls) *calls = n;
  for (cudaEvent_t e : g_prof.ev) cudaEventDestroy(e);
  g_prof = Profile{};
  return status;
}

}  // extern "C"
