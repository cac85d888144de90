// Internal launchers shared between the kernel files and the C ABI layer.
// Arguments are validated by the ABI layer (api.cu) before these run.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace phmoe {

// Router. With xq != null and a batch the fused single-launch router takes
// (router_fused_supported), it also writes the fixed-point rows of x for the
// decode FFN (group size G) to xq / xc and sets kRouterEncodedX in its
// result; callers then pass x_encoded to launch_ffn_decode. With disp !=
// null and a one-token batch it also writes launch_dispatch's outputs (the
// token's k rows in expert order) and sets kRouterDispatched; callers then
// skip launch_dispatch. The result is 0 when it did neither.
constexpr int kRouterEncodedX = 1;
constexpr int kRouterDispatched = 2;
struct DispatchOut {
  int32_t* offsets;    // [E+1]
  int32_t* row_token;  // [T*k]
  int32_t* inv;        // [T, k]
  int32_t* active;     // [E+1]
};
bool router_fused_supported(int T, int H, int E);
int launch_router(const void* x, int x_dtype, const void* wr, int w_dtype, int T, int H, int E,
                  int top_k, int renormalize, float* logits, float* probs, int32_t* topk_idx,
                  float* topk_w, cudaStream_t st, int G = 0, uint8_t* xq = nullptr, int2* xc = nullptr,
                  const DispatchOut* disp = nullptr);
int router_device_error(bool reset);

size_t dispatch_scratch_bytes(int T, int top_k, int E);
int launch_dispatch(const int32_t* topk_idx, int T, int top_k, int E, int32_t* offsets,
                    int32_t* row_token, int32_t* inv, int32_t* active, void* scratch,
                    cudaStream_t st);

// Decode FFN over dispatched rows (exact integer tensor-core dot products on
// fixed-point rows, ffn_decode.cu). The activation rows of x are encoded
// first: all T rows, or (enc_index != null) rows enc_index[i] for
// i < *enc_count (device memory), e.g. the rows that arrived from peers in a
// receive buffer of T rows. h is scratch of T*k*I*4 bytes; y ([T*k, H]
// fp32) also holds the encoded activations until the down kernel writes it.
// mid_event (may be null) is recorded between the gate/up and down kernels.
int launch_ffn_decode(const void* x, int x_dtype, const int32_t* row_token,
                      const int32_t* offsets, const int32_t* active, const uint8_t* w13_q,
                      const uint16_t* w13_s, const uint8_t* w2_q, const uint16_t* w2_s, int T,
                      int H, int E, int top_k, int I, int G, float* h, float* y,
                      cudaStream_t st, cudaEvent_t mid_event = nullptr,
                      const int32_t* enc_index = nullptr, const int32_t* enc_count = nullptr,
                      bool x_encoded = false, const struct RowScatter* scatter = nullptr,
                      bool* scattered = nullptr);
// Where the decode down projection stores its output rows (expert
// parallelism: straight into the source ranks' return buffers): row r of y
// goes to base[src[r]] + row[r] * H instead of y + r * H; a row whose src is
// outside [0, nbase) or whose row is outside [0, cap) is not stored.
// launch_ffn_decode sets *scattered when its down kernel did this (the TMA
// form); otherwise the rows are in y as usual.
struct RowScatter {
  float* base[8];
  const int32_t* src;
  const int32_t* row;
  int nbase;
  int cap;
};
// Where launch_ffn_decode keeps the fixed-point rows of x inside y (the
// router may write them there first).
uint8_t* ffn_decode_xq(float* y);
int2* ffn_decode_xc(float* y, int T, int H);

// Fixed-point rows (common.cuh) of `rows` rows of K elements (or of rows
// index[i], i < *count): q [rows][K*2 bytes], consts [rows][K/G] {C0, M}.
size_t fx_rows_bytes(long long rows, int K, int G);
int launch_fx_rows(const void* x, int x_dtype, long long rows, int K, int G, const int32_t* index,
                   const int32_t* count, uint8_t* q, int2* consts, cudaStream_t st);

// Prefill form (tcgen05 grouped GEMMs): bf16 x only; h is R*I*4 bytes of
// scratch and y doubles as the gathered activations until the down GEMM.
bool prefill_supported(int H, int I, int G, int E);
int launch_ffn_prefill(const void* x, const int32_t* row_token, const int32_t* offsets, const int32_t* active,
                       const uint8_t* w13_q, const uint16_t* w13_s, const uint8_t* w2_q, const uint16_t* w2_s,
                       int T, int H, int E, int top_k, int I, int G, float* h, float* y, cudaStream_t st,
                       cudaEvent_t mid_event = nullptr);
int prefill_device_error(bool reset);

int launch_combine(const float* y, const int32_t* inv, const float* topk_w, int T, int top_k,
                   int H, void* out, int out_dtype, cudaStream_t st);

void launch_gather_rows(const void* src, long long src_rows, const int32_t* index, int n_rows,
                        long long row_bytes, void* dst, cudaStream_t st);

int launch_quantize(const void* w, int w_dtype, long long rows, int K, int G, uint8_t* packed,
                    uint16_t* scales, cudaStream_t st);
int launch_gguf_q4_0(const void* blocks, long long rows, int K, uint8_t* packed, uint16_t* scales, cudaStream_t st);
int launch_gguf_q4_k(const void* blocks, long long rows, int K, int G, uint8_t* packed, uint16_t* scales,
                     cudaStream_t st);
int launch_gguf_q4_k_dequant(const void* blocks, long long n, float* out, cudaStream_t st);
int launch_router_grouped(const void* x, int x_dtype, const void* wr, int w_dtype, int T, int H, int E, int top_k,
                          int renormalize, const float* bias, int n_group, int topk_group, float scale,
                          float* logits, int32_t* topk_idx, float* topk_w, cudaStream_t st);
int launch_shared_slots(const void* x, int x_dtype, const void* gate_w, int w_dtype, const int32_t* idx,
                        const float* w, int T, int H, int k, int E, int m, float routed_scale, int32_t* idx_out,
                        float* w_out, cudaStream_t st);

int device_sm_count();

// Error word the FFN kernels raise when a pipeline wait times out (0 = ok).
int ffn_device_error(bool reset);

// Host-side count of kernels enqueued by this library (see phmoe.h).
void note_launches(int n);

// Sets the text phmoe_last_error returns on this host thread; returns status.
int record_error(int status, const char* msg);

// Expert-parallel exchange in peer memory (ep_p2p.cu).
struct EpContext;
// slots: local expert slots per rank (0: E/world; more for replicated placements)
int ep_create(int rank, int world, int max_tokens, int top_k, int H, int E, int slots, int x_elt, EpContext** out,
              void* handle_out);
int ep_connect(EpContext* c, const void* handles);
void ep_destroy(EpContext* c);
size_t ep_workspace_bytes(const EpContext* c, int I);
int ep_layer(EpContext* c, const void* x, int x_dtype, const void* router_w, int w_dtype, const uint8_t* w13_q,
             const uint16_t* w13_s, const uint8_t* w2_q, const uint16_t* w2_s, int T, int I, int G, int renormalize,
             int path, void* out, int32_t* topk_idx_out, float* topk_w_out, void* workspace, cudaStream_t st,
             const cudaEvent_t* marks,   // PHMOE_NUM_STAGES + 1 events, or null
             const int32_t* vmap);       // [E] expert -> virtual expert (device), or null for the home placement
int ep_info(const EpContext* c, int* rank, int* world, int* max_tokens, int* top_k, int* H, int* E);
int ep_slots(const EpContext* c);
int ep_device_error(bool reset);

}  // namespace phmoe
