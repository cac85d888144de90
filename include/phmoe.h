/*
 * phmoe.h - C ABI of the B200 (sm_100a) sparse-MoE layer.
 *
 * The reference (FreakyAdy/Solution-is-all-You-need, "PHANTOM") runs MoE
 * layers through transformers' Qwen3MoeSparseMoeBlock / MixtralSparseMoeBlock
 * (transformers 5.5.0 models/qwen3_moe/modeling_qwen3_moe.py:275-286, reached
 * from python/phantom/phantom_cli.py:1393-1430). Its own native kernels use
 * the convention `extern "C" float fn(device pointers, dims, cudaStream_t)`
 * (kernels/sparse_moe/sparse_matmul.cu:240-254, gate_predict.cu:200-214).
 * This ABI keeps that shape - raw device pointers, plain integer dims and a
 * stream - with three changes: every entry returns a status code instead of
 * calling exit() (kernels/common/cuda_utils.h:31-52); scratch memory is a
 * caller-provided workspace instead of cudaMalloc per call
 * (sparse_matmul.cu:264-273); and nothing synchronises the stream.
 *
 * All pointers are device pointers unless stated. `stream` is a
 * cudaStream_t passed as void* (NULL = legacy default stream). Entries are
 * reentrant as long as concurrent calls use distinct workspaces.
 *
 * Packed int4 layout (build-defined, generalising GGUF Q4_0,
 * python/phantom/loader/gguf_loader.py:362-381): a weight row of K elements
 * is K/2 bytes; value = (nibble - 8) * scale, with one fp16 scale per G
 * consecutive elements (G = 32 or 64) in a separate [rows, K/G] array.
 * Every 8 consecutive elements e0..e7 form one little-endian 32-bit word
 * holding e_{2i} in bits [4i, 4i+4) and e_{2i+1} in bits [16+4i, 16+4i+4):
 * bytes (e0|e2<<4, e4|e6<<4, e1|e3<<4, e5|e7<<4). GGUF Q4_0 blocks map to it
 * losslessly with G = 32 (a nibble shuffle; the block's d becomes the scale).
 */
#ifndef PHMOE_H_
#define PHMOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define PHMOE_OK 0
#define PHMOE_ERR_INVALID_ARG (-1)  /* a size, pointer or flag is out of range */
#define PHMOE_ERR_UNSUPPORTED (-2)  /* shape/dtype combination not built */
#define PHMOE_ERR_WORKSPACE (-3)    /* workspace too small or misaligned */
#define PHMOE_ERR_CUDA (-4)         /* a CUDA runtime call failed */
#define PHMOE_ERR_ALIGNMENT (-5)    /* a pointer is not 16-byte aligned */

/* ---- element types ---- */
#define PHMOE_DTYPE_F32 0
#define PHMOE_DTYPE_BF16 1

/* ---- FFN path selection for phmoe_moe_layer ---- */
#define PHMOE_PATH_AUTO 0    /* decode kernel for small batches, prefill kernel above */
#define PHMOE_PATH_DECODE 1  /* register-dequant grouped GEMV (mma.sync) */
#define PHMOE_PATH_PREFILL 2 /* TMA + tcgen05/TMEM grouped GEMM */

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int phmoe_version(void);

/* Human-readable text for a status code. Never returns NULL. */
const char* phmoe_status_string(int status);

/* Detail text of the last failing call on this host thread ("" if none). */
const char* phmoe_last_error(void);

/*
 * Bytes of workspace phmoe_moe_layer needs for T tokens (256-byte aligned
 * sub-buffers). Returns 0 on invalid arguments.
 */
size_t phmoe_workspace_size(int T, int H, int E, int top_k, int I, int path);

/*
 * The FFN path phmoe_moe_layer takes for these arguments: PHMOE_PATH_DECODE
 * or PHMOE_PATH_PREFILL (PHMOE_PATH_AUTO picks the prefill GEMMs for bf16
 * activations from 64 rows per expert on average, where the shapes allow),
 * or a negative status when the requested path cannot run them. Host-only.
 */
int phmoe_select_path(int path, int x_dtype, int T, int top_k, int H, int E, int I, int group_size);

/*
 * Router: logits = x . Wr^T (fp32, fixed reduction order), fp32 softmax,
 * top-k with ties to the lower expert index, optional renormalisation.
 * Replaces Qwen3MoeTopKRouter.forward (modeling_qwen3_moe.py:263-272) and
 * PhantomTopKRouter.forward (tests/test_moe_routing.py:56-72).
 *   x         [T, H]  x_dtype         router_w [E, H] w_dtype
 *   logits    [T, E]  fp32 (required: also the softmax staging buffer)
 *   probs     [T, E]  fp32 (may be NULL)
 *   topk_idx  [T, k]  int32           topk_w   [T, k] fp32
 * Limits: H % 8 == 0, 1 <= E <= 1024, 1 <= top_k <= min(E, 32).
 */
int phmoe_router(const void* x, int x_dtype, const void* router_w, int w_dtype, int T, int H,
                 int E, int top_k, int renormalize, float* logits, float* probs,
                 int32_t* topk_idx, float* topk_w, void* stream);

/*
 * Dispatch: group the T*k (token, slot) assignments by expert, ordered by
 * token index inside each expert (replaces the one_hot/where loop,
 * modeling_qwen3_moe.py:234-244).
 *   expert_offsets [E+1]  exclusive scan of per-expert counts
 *   row_token      [T*k]  token of each permuted row
 *   inv            [T*k]  permuted row of assignment t*k+j
 *   active         [E+1]  active[0] = number of experts hit, active[1..] their ids ascending
 * `scratch` needs phmoe_dispatch_scratch_size(T, k, E) bytes.
 */
size_t phmoe_dispatch_scratch_size(int T, int top_k, int E);
int phmoe_dispatch(const int32_t* topk_idx, int T, int top_k, int E, int32_t* expert_offsets,
                   int32_t* row_token, int32_t* inv, int32_t* active, void* scratch,
                   size_t scratch_bytes, void* stream);

/*
 * Grouped SwiGLU expert FFN over dispatched rows, decode form: exact integer
 * dot products on the int8 tensor cores. The activations and the SwiGLU
 * output h are encoded as fixed-point rows (phmoe_fx_rows); the int4
 * nibbles enter the MMAs as unsigned bytes, the group sums are exact int32,
 * and the fp16 group scales and fp32 accumulation are applied per group.
 * Replaces Qwen3MoeExperts.forward's per-expert loop body
 * (modeling_qwen3_moe.py:245-247).
 *   x        [T, H] x_dtype, gathered through row_token
 *   w13_q    [E, 2I, H/2] uint8 (gate rows 0..I-1, up rows I..2I-1)
 *   w13_s    [E, 2I, H/G] fp16        w2_q [E, H, I/2] uint8   w2_s [E, H, I/G] fp16
 *   h        scratch of T*k*I*4 bytes (fixed-point rows of the SwiGLU output)
 *   y        [T*k, H] fp32 output (permuted rows); also holds the encoded
 *            activations until the down projection writes it
 * Limits: G in {32, 64}; H % 256 == 0 (gate/up weight tiles are copied by TMA
 * in 128-byte rows); I % 16 == 0 and I % (2G) == 0; w13_s and w2_s 4-byte
 * aligned; w13_q 16-byte aligned.
 */
int phmoe_expert_ffn_decode(const void* x, int x_dtype, const int32_t* row_token,
                            const int32_t* expert_offsets, const int32_t* active,
                            const uint8_t* w13_q, const uint16_t* w13_s, const uint8_t* w2_q,
                            const uint16_t* w2_s, int T, int H, int E, int top_k, int I,
                            int group_size, float* h, float* y, void* stream);

/*
 * Grouped SwiGLU expert FFN, prefill form: the dispatched rows are gathered
 * into expert order, then two persistent grouped GEMMs run on the tcgen05
 * tensor cores (TMA-fed, accumulators in tensor memory) with fp16 operands:
 * the bf16 rows convert to fp16 exactly, the int4 weights are dequantised per
 * tile in shared memory to fp16_rn((nibble - 8) * scale) (the semantics of
 * gguf_loader.py:362-381 with 11 significant bits), and the SwiGLU output h
 * is rounded to fp16 between the two GEMMs. Rows of x beyond the fp16 range
 * are stored with a power-of-two row exponent, 128-column blocks of h with a
 * power-of-two block exponent (a short fixup pass brings a row's blocks to
 * one exponent), and the fp32 epilogues undo both exactly, so values up to
 * the bf16/fp32 range keep their magnitude; rows inside the fp16 range are
 * computed exactly as without them. Replaces the same loop as
 * phmoe_expert_ffn_decode, for batches where every expert sees many rows.
 * Same arguments; x must be bf16; h is scratch of T*k*I*4 bytes (the fp16 h
 * uses half, the exponents part of the rest); y doubles as the gathered rows
 * until the down GEMM.
 * Limits: G in {32, 64}; H % 256 == 0; I % 128 == 0; E such that the tile
 * table fits in shared memory (E <= 1024).
 */
int phmoe_expert_ffn_prefill(const void* x, int x_dtype, const int32_t* row_token,
                             const int32_t* expert_offsets, const int32_t* active,
                             const uint8_t* w13_q, const uint16_t* w13_s, const uint8_t* w2_q,
                             const uint16_t* w2_s, int T, int H, int E, int top_k, int I,
                             int group_size, float* h, float* y, void* stream);

/*
 * Fixed-point rows, the operand format of the decode FFN (no counterpart in
 * the reference, which multiplies in fp32). Each group of G consecutive
 * elements of a row gets an exponent e (the group's largest |value| scaled
 * into [4096, 8191] for G = 64, [8192, 16383] for G = 32; |value| below
 * ~1e34) and integers A = rint(v * 2^-e). Layout of `out`
 * (phmoe_fx_rows_size bytes, 256-byte aligned):
 *   q       [rows][K*2 bytes]: A = 256 * hi + lo with hi = (A + 128) >> 8
 *           and lo = A - 256 * hi (both signed bytes); per 8-element word
 *           16 bytes, the high bytes then the low bytes (the low byte is
 *           A & 255), each in element order 0, 4, 1, 5, 2, 6, 3, 7;
 *   consts  [rows][K/G] int32 pairs {C0, M} at byte offset
 *           phmoe_fx_rows_size - rows*(K/G)*8: M = bits of the float
 *           1.5 * 2^(23+e), C0 = M - 8 * sum(A).
 * Values beyond the range, infinities and NaNs are clamped and raise bit
 * value 2 of phmoe_device_error.
 */
size_t phmoe_fx_rows_size(long long rows, int K, int group_size);
int phmoe_fx_rows(const void* x, int x_dtype, long long rows, int K, int group_size, void* out, void* stream);

/*
 * Combine: out[t] = sum_j topk_w[t,j] * y[inv[t,j]] in slot order j = 0..k-1
 * (deterministic; replaces the weight multiply + index_add_,
 * modeling_qwen3_moe.py:248-249). out is [T, H] in out_dtype.
 */
int phmoe_combine(const float* y, const int32_t* inv, const float* topk_w, int T, int top_k,
                  int H, void* out, int out_dtype, void* stream);

/*
 * Row gather: dst[i] = src[index[i]] for i < n_rows, rows of row_bytes bytes;
 * a row whose index is outside [0, src_rows) is zero-filled. Used by the
 * expert-parallel layer to pack rows in expert order before the dispatch
 * all-to-all and to restore arrival order before the return all-to-all. No
 * counterpart in the reference (PHANTOM has no expert parallelism).
 * Limits: row_bytes % 16 == 0; src and dst 16-byte aligned.
 */
int phmoe_gather_rows(const void* src, long long src_rows, const int32_t* index, int n_rows,
                      long long row_bytes, void* dst, void* stream);

/*
 * Expert parallelism with the token exchange in peer memory (NVLink /
 * NVSwitch). No counterpart in the reference (PHANTOM has no expert
 * parallelism). E experts split evenly over `world` ranks (one process per
 * GPU, all on one node): rank r holds experts [r*E/world, (r+1)*E/world).
 *
 * Set-up (once per group, outside any stream capture):
 *   phmoe_ep_create   allocates this rank's exchange region (flags, counts,
 *                     received rows, returned rows; sized for max_tokens
 *                     tokens per rank) and writes its CUDA IPC handle
 *                     (PHMOE_EP_HANDLE_BYTES) to ipc_handle_out;
 *   the caller gathers every rank's handle, in rank order, and passes the
 *   world * PHMOE_EP_HANDLE_BYTES bytes to phmoe_ep_connect on every rank;
 *   phmoe_ep_destroy after all ranks have stopped calling the layer.
 * Per layer, on every rank in the same order (the call takes an epoch from a
 * host counter, so all ranks must make the same number of calls):
 *   phmoe_ep_layer    router and dispatch over all E experts; the rows for
 *                     each rank's experts are stored into that rank's region;
 *                     grouped FFN over the rows that arrived (w13_q etc. are
 *                     this rank's E/world experts); fp32 results stored back
 *                     into each source's region; combine. Completion is
 *                     signalled by epoch flags; a wait that exceeds 2 s sets
 *                     phmoe_device_error bit 2 and the layer continues with
 *                     the rows that did arrive instead of hanging.
 *   T (0..max_tokens) may differ between ranks. `path` as for
 *   phmoe_moe_layer, chosen for the T*k rows a rank expects over its E/world
 *   experts. workspace >= phmoe_ep_workspace_size(ctx, I) bytes, 256-byte
 *   aligned. The result equals phmoe_moe_layer on the full layer for this
 *   rank's tokens when both take the same FFN path.
 */
#define PHMOE_EP_MAX_WORLD 8
#define PHMOE_EP_HANDLE_BYTES 64
int phmoe_ep_create(int rank, int world, int max_tokens, int top_k, int H, int E, int x_dtype, void** ctx,
                    void* ipc_handle_out);
int phmoe_ep_connect(void* ctx, const void* ipc_handles);
int phmoe_ep_destroy(void* ctx);
size_t phmoe_ep_workspace_size(const void* ctx, int I);
int phmoe_ep_layer(void* ctx, const void* x, int x_dtype, const void* router_w, int w_dtype, const uint8_t* w13_q,
                   const uint16_t* w13_s, const uint8_t* w2_q, const uint16_t* w2_s, int T, int I, int group_size,
                   int renormalize, int path, void* out, int32_t* topk_idx_out, float* topk_w_out, void* workspace,
                   size_t workspace_bytes, void* stream);

/*
 * Replicated placements (hot experts copied onto several ranks, to even out
 * skewed routing). phmoe_ep_create_ex sizes every rank for slots_per_rank
 * local expert slots (>= E/world; 0 means E/world; world * slots <= 1024);
 * rank r's slot j is the virtual expert r * slots + j. phmoe_ep_layer_ex
 * takes this rank's map vmap [E] int32 (device memory): the virtual expert
 * each of its expert ids is sent to, i.e. the copy it uses; w13_q etc. hold
 * the rank's `slots` local experts (padding slots may repeat any expert; they
 * receive no rows). Rows with a map entry outside [0, world * slots) are
 * dropped. With vmap = NULL it is phmoe_ep_layer (home placement only). Every
 * row's result is the same whichever copy computes it, so the output equals
 * phmoe_ep_layer's.
 */
int phmoe_ep_create_ex(int rank, int world, int max_tokens, int top_k, int H, int E, int slots_per_rank,
                       int x_dtype, void** ctx, void* ipc_handle_out);
int phmoe_ep_layer_ex(void* ctx, const void* x, int x_dtype, const void* router_w, int w_dtype,
                      const uint8_t* w13_q, const uint16_t* w13_s, const uint8_t* w2_q, const uint16_t* w2_s, int T,
                      int I, int group_size, int renormalize, int path, const int32_t* vmap, void* out,
                      int32_t* topk_idx_out, float* topk_w_out, void* workspace, size_t workspace_bytes,
                      void* stream);

/*
 * The whole layer (Qwen3MoeSparseMoeBlock.forward, modeling_qwen3_moe.py:281-286,
 * on [T, H] rows): router -> dispatch -> grouped FFN -> combine, all
 * stream-ordered, no host synchronisation, no allocation.
 *   out           [T, H] same dtype as x
 *   topk_idx_out  [T, k] int32 (may be NULL)   topk_w_out [T, k] fp32 (may be NULL)
 *   workspace     >= phmoe_workspace_size(T, H, E, k, I, path) bytes, 256-byte aligned
 */
int phmoe_moe_layer(const void* x, int x_dtype, const void* router_w, int w_dtype,
                    const uint8_t* w13_q, const uint16_t* w13_s, const uint8_t* w2_q,
                    const uint16_t* w2_s, int T, int H, int E, int top_k, int I,
                    int group_size, int renormalize, int path, void* out, int32_t* topk_idx_out,
                    float* topk_w_out, void* workspace, size_t workspace_bytes, void* stream);

/*
 * phmoe_moe_layer without a workspace argument, for callers that cannot
 * allocate device memory: hosts handed buffers by another framework whose
 * allocator already holds the GPU's free memory, hosts that forbid device
 * allocation after load (cudaFree synchronises the device, cudaMalloc may),
 * and foreign-language bindings with no allocator to call. No counterpart in
 * the reference (its kernels cudaMalloc scratch per call).
 *
 * Scratch comes from a fixed array of PHMOE_STATIC_SCRATCH_BYTES inside the
 * library, held on every GPU that loads the library until the process exits.
 * Calls needing more (phmoe_workspace_size(...) > PHMOE_STATIC_SCRATCH_BYTES;
 * at H 2048, E 128, top-8, I 768 that is beyond 184 tokens) return
 * PHMOE_ERR_WORKSPACE without launching anything. All calls on a device share
 * the array, which keeps the last call's contents (nothing in it has to start
 * at zero); calls that overlap on the GPU race on it, so order them on one
 * stream. The first call on each device looks up the array's address
 * (cudaGetSymbolAddress); make it before any stream capture on that device.
 * Allocates nothing. Same arguments and results as phmoe_moe_layer.
 */
#define PHMOE_STATIC_SCRATCH_BYTES ((size_t)16 << 20)
int phmoe_moe_layer_noalloc(const void* x, int x_dtype, const void* router_w, int w_dtype,
                            const uint8_t* w13_q, const uint16_t* w13_s, const uint8_t* w2_q,
                            const uint16_t* w2_s, int T, int H, int E, int top_k, int I,
                            int group_size, int renormalize, int path, void* out,
                            int32_t* topk_idx_out, float* topk_w_out, void* stream);

/* Router scoring functions. */
enum { PHMOE_SCORING_SOFTMAX = 0, PHMOE_SCORING_SIGMOID = 1 };

/*
 * Router with the DeepSeek-V3 selection (transformers 5.5.0
 * models/deepseek_v3/modeling_deepseek_v3.py DeepseekV3MoE.route_tokens_to_experts):
 * scoring PHMOE_SCORING_SIGMOID: s = sigmoid(logit) (fp32; a fixed exp
 * routine, bit-reproducible), choice c = s + score_bias[e] (score_bias [E]
 * fp32 or NULL); with n_group > 1 the experts form n_group groups of
 * E/n_group (>= 2), a group scores the sum of its two largest c, only the
 * topk_group best groups stay (the others' c become 0); the top_k largest c
 * are picked (ties -> lower index) and weighted by s, divided by
 * (sum + 1e-20) when renormalize, times routed_scale.
 * scoring PHMOE_SCORING_SOFTMAX with n_group <= 1, no bias and
 * routed_scale == 1 is phmoe_router. Logits as phmoe_router.
 */
int phmoe_router_ex(const void* x, int x_dtype, const void* router_w, int w_dtype, int T, int H,
                    int E, int top_k, int renormalize, int scoring, const float* score_bias,
                    int n_group, int topk_group, float routed_scale, float* logits,
                    int32_t* topk_idx, float* topk_w, void* stream);

/*
 * Extended MoE layer: shared experts and the DeepSeek-V3 router.
 *
 * Shared experts (Qwen2-MoE's gated shared expert, transformers 5.5.0
 * models/qwen2_moe/modeling_qwen2_moe.py Qwen2MoeSparseMoeBlock.forward:
 * out = routed + sigmoid(x . w_sg) * shared(x); DeepSeek's ungated ones,
 * DeepseekV3MoE.forward): the packed expert tensors hold E + num_shared
 * experts, the E routed ones and then the shared expert split along its
 * intermediate dimension into num_shared experts of size I (a shared expert
 * of size m * I is the sum of those m SwiGLU experts). Every token goes to
 * its top_k routed experts (weights times routed_scale) and to all
 * num_shared shared experts with weight sigmoid(x . shared_gate_w)
 * (shared_gate_w: [H] in w_dtype), or 1 when shared_gate_w is NULL.
 * Routing: scoring / score_bias / n_group / topk_group as phmoe_router_ex.
 * topk_idx_out / topk_w_out (optional, [T, top_k]) receive the routed choice
 * before routed_scale. Other arguments and limits as phmoe_moe_layer;
 * workspace_bytes >= phmoe_workspace_size_ex(...).
 */
size_t phmoe_workspace_size_ex(int T, int H, int E, int top_k, int I, int num_shared, int path);
int phmoe_moe_layer_ex(const void* x, int x_dtype, const void* router_w, int w_dtype,
                       const uint8_t* w13_q, const uint16_t* w13_s, const uint8_t* w2_q,
                       const uint16_t* w2_s, int T, int H, int E, int top_k, int I,
                       int group_size, int renormalize, int scoring, const float* score_bias,
                       int n_group, int topk_group, int num_shared, const void* shared_gate_w,
                       float routed_scale, int path, void* out, int32_t* topk_idx_out,
                       float* topk_w_out, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Symmetric int4 group quantiser on the GPU (load-time utility; the
 * reference has no quantiser and reads pre-quantised GGUF files):
 * scale = fp16(absmax(group)/7), q = clamp(rint(w/scale), -8, 7).
 *   w [rows, K] fp32 or bf16 -> packed [rows, K/2] uint8, scales [rows, K/G] fp16.
 */
int phmoe_quantize_int4(const void* w, int w_dtype, long long rows, int K, int group_size,
                        uint8_t* packed, uint16_t* scales, void* stream);

/*
 * GGUF importers (load-time): llama.cpp-quantised expert tensors straight
 * into the packed layout on the GPU, without a bf16 round trip. They replace
 * the dequantise-at-load step of the reference's GGUF loader
 * (python/phantom/loader/gguf_loader.py:799-805 -> dequantize_tensor_cuda,
 * gguf_loader.py:538), whose Q4_0 and Q4_K semantics they follow
 * (gguf_loader.py:588-596 and 648-666). `blocks` holds `rows` rows of K
 * elements each as consecutive GGUF blocks (a GGUF tensor's data as stored:
 * K is its innermost dimension).
 *
 * phmoe_gguf_q4_0_to_packed: Q4_0 (18-byte blocks of 32) -> packed int4 with
 *   group_size 32, bit-exact: the same values, nibbles re-ordered, d copied
 *   as the fp16 group scale. K % 32 == 0; packed 16-byte aligned.
 * phmoe_gguf_q4_k_to_packed: Q4_K (144-byte super-blocks of 256) -> each
 *   element dequantised in fp32 as the reference does, then re-quantised with
 *   phmoe_quantize_int4's rule (group_size 32 or 64). Q4_K is asymmetric
 *   (scale and min per 32 elements), so this step is lossy: the error per
 *   element is at most half a step of the new group scale. K % 256 == 0.
 * phmoe_gguf_q4_k_dequantize: Q4_K -> fp32 values (n elements, n % 256 == 0),
 *   the reference's dequantised weights, for checks.
 */
int phmoe_gguf_q4_0_to_packed(const void* blocks, long long rows, int K, uint8_t* packed,
                              uint16_t* scales, void* stream);
int phmoe_gguf_q4_k_to_packed(const void* blocks, long long rows, int K, int group_size,
                              uint8_t* packed, uint16_t* scales, void* stream);
int phmoe_gguf_q4_k_dequantize(const void* blocks, long long n, float* out, void* stream);

/*
 * Instrumentation for benchmarks (no counterpart in the reference, whose
 * entries return their own elapsed ms from a CudaTimer,
 * kernels/common/cuda_utils.h:341-357, sparse_matmul.cu:256-257).
 *
 * phmoe_kernel_launch_count: number of kernels this library has enqueued in
 * this process (host-side counter; replays of a captured CUDA graph are not
 * counted again).
 *
 * phmoe_profile_begin(max_calls): the next max_calls phmoe_moe_layer calls
 * record CUDA events between their stages on the caller's stream
 * (stages: 0 router, 1 dispatch, 2 FFN gate/up, 3 FFN down, 4 combine).
 * phmoe_profile_end waits for the last recorded event, writes the summed
 * device time per stage (ms) into stage_ms[0..n_stages-1], the number of
 * calls recorded into *calls, and releases the events. Process-global and
 * not thread-safe; do not profile inside stream capture.
 */
#define PHMOE_NUM_STAGES 5

/*
 * Device-side error bits of the current device: 0 when all is well; bit 0
 * (1) when a pipeline wait of an FFN kernel timed out (its CTA abandoned its
 * work after a bounded wait instead of hanging); bit 1 (2) when an
 * activation or SwiGLU value could not be held and was clamped (the decode
 * path's fixed-point rows: beyond ~1e34, infinite or NaN; the prefill path
 * has no such limit below the fp32 range); bit 2 (4) when an expert-parallel peer
 * flag did not arrive within 2 s.
 * Synchronous; reset != 0 clears it. Not part of the hot path.
 */
int phmoe_device_error(int reset);
unsigned long long phmoe_kernel_launch_count(void);
int phmoe_profile_begin(int max_calls);
int phmoe_profile_end(float* stage_ms, int n_stages, int* calls);

#ifdef __cplusplus
}
#endif

#endif /* PHMOE_H_ */
