// Expert-parallel MoE layer with the token exchange done in peer memory over
// NVLink / NVSwitch: each rank writes the rows it routes to another rank's
// experts straight into that rank's receive buffer, and the expert outputs
// come back the same way. No host synchronisation and no collective library
// on the data path; completion is signalled with per-source epoch flags
// (system-scope release stores, acquire loads). PHANTOM has no expert
// parallelism; the layer semantics are those of phmoe_moe_layer (transformers'
// Qwen3MoeSparseMoeBlock.forward, modeling_qwen3_moe.py:281-286) with the
// E experts split evenly over the ranks (rank r holds [r*E/P, (r+1)*E/P)).
//
// Per layer on rank `me` (one stream, in order; every kernel is launched
// with programmatic dependent launch and waits for its predecessor first):
//   router + dispatch over all E experts (rows come out expert-major, hence
//     destination-major);
//   ep_send_kernel   - row r goes to rank d = owner of its expert, slot
//     i = r - offsets[d*Epr] of d's receive block for `me`; the first CTA
//     also stores `me`'s per-expert counts for every d; the last CTA to
//     count (each CTA releases its stores with one system fence) stores d's
//     arrival flag for `me` = epoch;
//   ep_prepare_kernel - waits (bounded) for every source's flag, then builds
//     the local expert grouping of the arrived rows (per local expert: source
//     by source, each source's rows in its own order) and, per local row, the
//     source rank and its row in the source's dispatch order;
//   grouped FFN (decode or prefill kernels) over the arrived rows; the
//     decode down kernel stores each fp32 output row straight into its
//     source's return buffer at that row (RowScatter) and ep_flag_kernel
//     then raises the return flags; after the prefill kernels,
//     ep_return_kernel copies the rows back and its last CTA raises them;
//   ep_wait_kernel   - waits (bounded) for every destination's return flag;
//   combine over the returned rows in slot order.
// Replicated placements (hot experts copied onto several ranks): every rank
// holds S >= E/P local slots and the layer takes this rank's map from expert
// to virtual expert (rank * S + slot of the copy it sends to); the router's
// ids are remapped to virtual ids before the dispatch, so the rows still come
// out destination-major and every step below runs with S in place of E/P.
// Reusing the single receive/return buffers is safe without further
// handshakes: a source writes epoch e+1 rows only after its combine of epoch
// e, which waited for this rank's return of epoch e, which came after this
// rank's FFN finished reading the epoch-e rows.
//
// Waits give up after kWaitNs (2 s) of %globaltimer time, set the device error word
// (phmoe_device_error bit 2) and continue with empty data instead of hanging.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "common.cuh"
#include "pipeline.cuh"
#include "launch.h"

namespace phmoe {

__device__ int g_ep_error;  // 0 = ok, 4 = a peer flag did not arrive in time

namespace {

constexpr int kMaxWorld = 8;
constexpr int kCopyThreads = 256;
// The row exchange kernels run one CTA of kXferThreads per SM: every thread
// ends with a system-scope fence (its peer stores acknowledged) before the
// last-CTA count, so all fences overlap in one wave instead of queueing over
// several waves of small CTAs.
constexpr int kXferThreads = 1024;
constexpr unsigned long long kWaitNs = 2000000000ull;

struct Peers {
  char* base[kMaxWorld];  // every rank's region, as mapped in this process (own one included)
};

// Byte offsets inside a rank's region (identical on every rank).
struct Region {
  size_t flags_in, flags_back, counts_in, recv_x, y_back, done, epoch, total;
};

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

Region region_layout(int world, int cap, int epr, int H, int elt) {
  Region L{};
  size_t off = 0;
  auto take = [&](size_t bytes) { const size_t o = off; off = align_up(off + bytes, 256); return o; };
  L.flags_in = take(kMaxWorld * 4);
  L.flags_back = take(kMaxWorld * 4);
  L.counts_in = take((size_t)kMaxWorld * (epr + 1) * 4);  // per source: epr counts, then its base row
  L.done = take(2 * 4);                                     // last-CTA counters (send, return)
  L.epoch = take(4);                                        // the current layer call's epoch (from 1)
  L.recv_x = take((size_t)world * cap * H * elt);
  L.y_back = take((size_t)cap * H * 4);
  L.total = off;
  return L;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Bounded wait for *flag == epoch; false (and the error bit) on timeout.
__device__ bool wait_flag(const uint32_t* flag, uint32_t epoch) {
  if (ld_acquire_sys(flag) == epoch) return true;
  const unsigned long long t0 = global_ns();
  while (ld_acquire_sys(flag) != epoch) {
    if (global_ns() - t0 > kWaitNs) {
      atomicOr(&g_ep_error, 4);
      return false;
    }
    __nanosleep(200);
  }
  return true;
}

// Copies this CTA's rows, r = blockIdx.x + j * gridDim.x < n: the (row,
// 16-byte chunk) pairs are spread over all threads, four loads in flight per
// thread. row(r) gives a row's source and destination (dst null: the row is
// not copied).
struct RowCopy {
  const uint4* src;
  uint4* dst;
};
template <typename RowFn>
__device__ __forceinline__ void copy_rows(int n, int chunks, RowFn row) {
  const int mine = (int)blockIdx.x < n ? (n - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int total = mine * chunks;
  for (int q0 = threadIdx.x; q0 < total; q0 += 4 * blockDim.x) {
    uint4 v[4];
    uint4* d[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int q = q0 + u * blockDim.x;
      d[u] = nullptr;
      if (q < total) {
        const int j = q / chunks, c = q - j * chunks;
        const RowCopy rc = row((int)blockIdx.x + j * (int)gridDim.x);
        if (rc.dst != nullptr) {
          v[u] = __ldg(rc.src + c);
          d[u] = rc.dst + c;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (d[u] != nullptr) *d[u] = v[u];
  }
}

// The epoch of the current layer call: a word of this rank's region, set to
// 1 at creation and advanced by the call's last exchange kernel
// (ep_wait_kernel), so the layer can be captured in a CUDA graph and
// replayed. Read after the kernel's programmatic-launch wait, i.e. after the
// previous call's advance.
__device__ __forceinline__ uint32_t call_epoch(const char* region, const Region& L) {
  return *reinterpret_cast<const volatile uint32_t*>(region + L.epoch);
}

// System-scope acquire-release fence (the count hand-offs below need no
// sequentially consistent fence; fence.sc.sys measured ~3-4 us per step of
// the exchange's chain).
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// True for the one CTA that finishes last; that CTA resets the counter for
// the next layer. The CTA barrier orders every thread's stores before
// thread 0's system-scope fence, which is cumulative: the CTA's stores (to
// peers too) are visible system-wide before its count (release), and the
// last CTA's fence after reading the count (acquire) orders them all before
// the release stores of its flags.
// (One fence per CTA instead of one per thread: a fence in every thread cost
// ~2.4 us more per copy kernel of a 148 x 1024 grid.)
__device__ bool last_cta(int* counter) {
  __shared__ bool last;
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_acq_rel_sys();
    last = atomicAdd(counter, 1) == (int)(gridDim.x - 1);
    if (last) *counter = 0;
    if (last) fence_acq_rel_sys();
  }
  __syncthreads();
  return last;
}

__global__ void __launch_bounds__(kXferThreads)
ep_send_kernel(const char* __restrict__ x, const int32_t* __restrict__ row_token, const int32_t* __restrict__ offsets,
               int R, int T, int epr, int world, int me, int cap, int row_bytes, const __grid_constant__ Peers peers,
               Region L) {
  pdl_begin();
  const uint32_t epoch = call_epoch(peers.base[me], L);
  const int chunks = row_bytes / 16;
  const int nvalid = R > 0 ? __ldg(offsets + epr * world) : 0;
  if (blockIdx.x == 0) {
    // counts and base row for each destination (they depend on the dispatch
    // only): written first, so CTA 0's release before its count covers them
    for (int d = 0; d < world; ++d) {
      int32_t* cnt = reinterpret_cast<int32_t*>(peers.base[d] + L.counts_in) + (size_t)me * (epr + 1);
      for (int l = threadIdx.x; l <= epr; l += blockDim.x) {
        int32_t v = 0;
        if (R > 0)
          v = l < epr ? __ldg(offsets + d * epr + l + 1) - __ldg(offsets + d * epr + l) : __ldg(offsets + d * epr);
        cnt[l] = v;
      }
    }
  }
  copy_rows(nvalid, chunks, [&](int r) -> RowCopy {
    int d = 0;
    while (d + 1 < world && __ldg(offsets + (d + 1) * epr) <= r) ++d;
    const int i = r - __ldg(offsets + d * epr);
    const int t = __ldg(row_token + r);
    if (i >= cap || t < 0 || t >= T) return RowCopy{nullptr, nullptr};
    return RowCopy{reinterpret_cast<const uint4*>(x + (size_t)t * row_bytes),
                   reinterpret_cast<uint4*>(peers.base[d] + L.recv_x + ((size_t)me * cap + i) * row_bytes)};
  });
  int* done = reinterpret_cast<int*>(peers.base[me] + L.done);
  if (!last_cta(done)) return;
  // every CTA's rows (and CTA 0's counts) are ordered before these
  if (threadIdx.x < world)
    st_release_sys(reinterpret_cast<uint32_t*>(peers.base[threadIdx.x] + L.flags_in) + me, epoch);
}

constexpr int kPrepThreads = 1024;

// One CTA. Local grouping of the arrived rows: for local expert l, the rows of
// source 0, then source 1, ... each in the source's order. Outputs:
// off[epr+1], active[epr+1], row_token (index into the receive buffer),
// ret_src / ret_row (where each local row goes back).
__global__ void __launch_bounds__(kPrepThreads)
ep_prepare_kernel(const char* __restrict__ local, Region L, int world, int cap, int epr,
                  int32_t* __restrict__ off, int32_t* __restrict__ active, int32_t* __restrict__ row_token,
                  int32_t* __restrict__ ret_src, int32_t* __restrict__ ret_row) {
  pdl_begin();
  const uint32_t epoch = call_epoch(local, L);
  __shared__ int s_ok[kMaxWorld];
  extern __shared__ int sm[];
  int* cnt = sm;                           // [world][epr]
  int* base = cnt + world * epr;           // [world]
  int* seg = base + world;                 // [world][epr] exclusive scan over l per source
  int* loff = seg + world * epr;           // [epr + 1]
  if (threadIdx.x < world)
    s_ok[threadIdx.x] = wait_flag(reinterpret_cast<const uint32_t*>(local + L.flags_in) + threadIdx.x, epoch);
  __syncthreads();
  const int32_t* cin = reinterpret_cast<const int32_t*>(local + L.counts_in);
  for (int q = threadIdx.x; q < world * (epr + 1); q += blockDim.x) {
    const int s = q / (epr + 1), l = q % (epr + 1);
    int v = s_ok[s] ? cin[(size_t)s * (epr + 1) + l] : 0;
    if (l < epr) {
      cnt[s * epr + l] = v < 0 ? 0 : (v > cap ? cap : v);
    } else {
      base[s] = v;
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  if (warp < world) {  // warp s: exclusive scan of source s's counts over the local experts
    const int s = warp;
    int carry = 0;
    for (int l0 = 0; l0 < epr; l0 += 32) {
      const int l = l0 + lane;
      const int v = l < epr ? cnt[s * epr + l] : 0;
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      if (l < epr) seg[s * epr + l] = carry + incl - v;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
  } else if (warp == world) {  // per-expert totals: their exclusive scan and the active list
    int carry = 0, na = 0;
    for (int l0 = 0; l0 < epr; l0 += 32) {
      const int l = l0 + lane;
      int n = 0;
      if (l < epr)
        for (int s = 0; s < world; ++s) n += cnt[s * epr + l];
      int incl = n;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      if (l < epr) loff[l] = carry + incl - n;
      const unsigned m = __ballot_sync(0xffffffffu, l < epr && n > 0);
      if (l < epr && n > 0) active[1 + na + __popc(m & ((1u << lane) - 1u))] = l;
      na += __popc(m);
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      loff[epr] = carry;
      active[0] = na;
    }
  }
  __syncthreads();
  for (int l = threadIdx.x; l <= epr; l += blockDim.x) off[l] = loff[l];
  // rows: one warp per (expert, source) segment
  for (int q = warp; q < epr * world; q += nwarps) {
    const int l = q / world, s = q % world;
    int p = loff[l];
    for (int s2 = 0; s2 < s; ++s2) p += cnt[s2 * epr + l];
    const int n = cnt[s * epr + l], st = seg[s * epr + l];
    for (int j = lane; j < n; j += 32) {
      row_token[p + j] = s * cap + st + j;
      ret_src[p + j] = s;
      ret_row[p + j] = base[s] + st + j;
    }
  }
}

__global__ void __launch_bounds__(kXferThreads)
ep_return_kernel(const float* __restrict__ y, const int32_t* __restrict__ off, int epr,
                 const int32_t* __restrict__ ret_src, const int32_t* __restrict__ ret_row, int world, int me, int cap,
                 int H, const __grid_constant__ Peers peers, Region L) {
  pdl_begin();
  const uint32_t epoch = call_epoch(peers.base[me], L);
  const int nrows = __ldg(off + epr);
  const int chunks = H * 4 / 16;
  copy_rows(nrows, chunks, [&](int r) -> RowCopy {
    const int s = __ldg(ret_src + r), row = __ldg(ret_row + r);
    if (s < 0 || s >= world || row < 0 || row >= cap) return RowCopy{nullptr, nullptr};
    return RowCopy{reinterpret_cast<const uint4*>(y + (size_t)r * H),
                   reinterpret_cast<uint4*>(peers.base[s] + L.y_back + (size_t)row * H * 4)};
  });
  int* done = reinterpret_cast<int*>(peers.base[me] + L.done) + 1;
  if (!last_cta(done)) return;
  if (threadIdx.x < world)
    st_release_sys(reinterpret_cast<uint32_t*>(peers.base[threadIdx.x] + L.flags_back) + me, epoch);
}

// vidx[i] = vmap[idx[i]]: expert ids to virtual experts (-1, i.e. dropped
// by the dispatch, for ids outside [0, E) or maps outside [0, V)).
__global__ void __launch_bounds__(kCopyThreads)
ep_remap_kernel(const int32_t* __restrict__ idx, const int32_t* __restrict__ vmap, int R, int E, int V,
                int32_t* __restrict__ vidx) {
  pdl_begin();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < R; i += gridDim.x * blockDim.x) {
    const int e = __ldg(idx + i);
    const int v = (unsigned)e < (unsigned)E ? __ldg(vmap + e) : -1;
    vidx[i] = (unsigned)v < (unsigned)V ? v : -1;
  }
}

// The return flags when the down projection stored its rows straight into
// the sources' return buffers (RowScatter): after the down kernel (the
// programmatic-launch wait makes its stores visible to this grid), a
// system-scope acquire-release fence orders them before each source's flag.
__global__ void ep_flag_kernel(const __grid_constant__ Peers peers, Region L, int world, int me) {
  pdl_begin();
  const uint32_t epoch = call_epoch(peers.base[me], L);
  if (threadIdx.x < world) {
    fence_acq_rel_sys();
    st_release_sys(reinterpret_cast<uint32_t*>(peers.base[threadIdx.x] + L.flags_back) + me, epoch);
  }
}

// Waits for the return flags, then advances the epoch word for the next
// layer call (every rank advances its own in step: one per call).
__global__ void ep_wait_kernel(char* __restrict__ local, Region L, int world) {
  pdl_begin();
  const uint32_t epoch = call_epoch(local, L);
  __syncthreads();  // every thread has read this call's epoch
  if (threadIdx.x < world) wait_flag(reinterpret_cast<const uint32_t*>(local + L.flags_back) + threadIdx.x, epoch);
  __syncthreads();
  if (threadIdx.x == 0) *reinterpret_cast<volatile uint32_t*>(local + L.epoch) = epoch + 1;
}

}  // namespace

struct EpContext {
  // epr: local expert slots per rank (E/world, more with replicas); V = world * epr virtual experts
  int rank = 0, world = 1, max_tokens = 0, top_k = 1, H = 0, E = 0, epr = 0, V = 0, elt = 2, cap = 0, device = 0;
  Region L{};
  char* local = nullptr;
  Peers peers{};
  bool opened[kMaxWorld] = {};
  bool connected = false;
};

int ep_device_error(bool reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_ep_error, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_ep_error, &zero, sizeof(int));
  }
  return v;
}

int ep_create(int rank, int world, int max_tokens, int top_k, int H, int E, int slots, int x_elt, EpContext** out,
              void* handle_out) {
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world || E % world || max_tokens < 1 || top_k < 1 ||
      H <= 0 || (H * x_elt) % 16 || (slots != 0 && slots < E / world))
    return PHMOE_ERR_INVALID_ARG;
  EpContext* c = new EpContext();
  c->rank = rank;
  c->world = world;
  c->max_tokens = max_tokens;
  c->top_k = top_k;
  c->H = H;
  c->E = E;
  c->epr = slots ? slots : E / world;
  c->V = world * c->epr;
  c->elt = x_elt;
  c->cap = max_tokens * top_k;
  c->L = region_layout(world, c->cap, c->epr, H, x_elt);
  const uint32_t first_epoch = 1;
  if (cudaGetDevice(&c->device) != cudaSuccess || cudaMalloc(&c->local, c->L.total) != cudaSuccess ||
      cudaMemset(c->local, 0, c->L.total) != cudaSuccess ||
      cudaMemcpy(c->local + c->L.epoch, &first_epoch, 4, cudaMemcpyHostToDevice) != cudaSuccess) {
    if (c->local) cudaFree(c->local);
    delete c;
    return PHMOE_ERR_CUDA;
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, c->local) != cudaSuccess) {
    cudaFree(c->local);
    delete c;
    return PHMOE_ERR_CUDA;
  }
  memcpy(handle_out, &h, sizeof(h));
  c->peers.base[rank] = c->local;
  *out = c;
  return PHMOE_OK;
}

int ep_connect(EpContext* c, const void* handles) {
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const char*>(handles) + (size_t)r * sizeof(h), sizeof(h));
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return PHMOE_ERR_CUDA;
    c->peers.base[r] = static_cast<char*>(p);
    c->opened[r] = true;
  }
  c->connected = true;
  return PHMOE_OK;
}

void ep_destroy(EpContext* c) {
  if (!c) return;
  for (int r = 0; r < c->world; ++r)
    if (c->opened[r]) cudaIpcCloseMemHandle(c->peers.base[r]);
  if (c->local) cudaFree(c->local);
  delete c;
}

size_t ep_workspace_bytes(const EpContext* c, int I) {
  const size_t capr = (size_t)c->world * c->cap;  // rows this rank may receive
  size_t off = 0;
  auto take = [&](size_t b) { off = align_up(off + b, 256); };
  take((size_t)c->max_tokens * c->E * 4);               // logits
  take((size_t)c->cap * 4);                             // idx
  take((size_t)c->cap * 4);                             // w
  take((size_t)(c->V + 1) * 4);                         // offsets (per virtual expert)
  take((size_t)(c->V + 1) * 4);                         // active
  take((size_t)c->cap * 4);                             // row_token
  take((size_t)c->cap * 4);                             // inv
  take((size_t)c->cap * 4);                             // virtual expert ids
  take(dispatch_scratch_bytes(c->max_tokens, c->top_k, c->V));
  take((size_t)(c->epr + 1) * 4 * 2);                   // local offsets, active
  take(capr * 4 * 3);                                   // local row_token, ret_src, ret_row
  take(capr * (size_t)I * 4);                           // h
  take(capr * (size_t)c->H * 4);                        // y (local expert order)
  return off;
}

int ep_layer(EpContext* c, const void* x, int x_dtype, const void* router_w, int w_dtype, const uint8_t* w13_q,
             const uint16_t* w13_s, const uint8_t* w2_q, const uint16_t* w2_s, int T, int I, int G, int renormalize,
             int path, void* out, int32_t* topk_idx_out, float* topk_w_out, void* workspace, cudaStream_t st,
             const cudaEvent_t* marks, const int32_t* vmap) {
  const int E = c->E, V = c->V, k = c->top_k, epr = c->epr, world = c->world;
  auto mark = [&](int b) { if (marks) cudaEventRecord(marks[b], st); };
  const size_t capr = (size_t)world * c->cap;
  char* ws = static_cast<char*>(workspace);
  size_t off = 0;
  auto take = [&](size_t b) { char* p = ws + off; off = align_up(off + b, 256); return p; };
  float* logits = reinterpret_cast<float*>(take((size_t)c->max_tokens * E * 4));
  int32_t* idx = reinterpret_cast<int32_t*>(take((size_t)c->cap * 4));
  float* wts = reinterpret_cast<float*>(take((size_t)c->cap * 4));
  int32_t* offsets = reinterpret_cast<int32_t*>(take((size_t)(V + 1) * 4));
  int32_t* active = reinterpret_cast<int32_t*>(take((size_t)(V + 1) * 4));
  int32_t* row_token = reinterpret_cast<int32_t*>(take((size_t)c->cap * 4));
  int32_t* inv = reinterpret_cast<int32_t*>(take((size_t)c->cap * 4));
  int32_t* vidx = reinterpret_cast<int32_t*>(take((size_t)c->cap * 4));
  void* disp = take(dispatch_scratch_bytes(c->max_tokens, k, V));
  int32_t* loff = reinterpret_cast<int32_t*>(take((size_t)(epr + 1) * 4 * 2));
  int32_t* lact = loff + (epr + 1);
  int32_t* lrow = reinterpret_cast<int32_t*>(take(capr * 4 * 3));
  int32_t* ret_src = lrow + capr;
  int32_t* ret_row = ret_src + capr;
  float* h = reinterpret_cast<float*>(take(capr * (size_t)I * 4));
  float* y = reinterpret_cast<float*>(take(capr * (size_t)c->H * 4));
  if (topk_idx_out) idx = topk_idx_out;
  if (topk_w_out) wts = topk_w_out;

  const int R = T * k;
  const int row_bytes = c->H * c->elt;
  mark(0);
  if (T > 0) launch_router(x, x_dtype, router_w, w_dtype, T, c->H, E, k, renormalize, logits, nullptr, idx, wts, st);
  mark(1);
  const int sms = device_sm_count();
  if (T > 0 && vmap) {  // replicated placement: dispatch by virtual expert
    launch_pdl(ep_remap_kernel, dim3(R < sms * 4 * kCopyThreads ? (R + kCopyThreads - 1) / kCopyThreads : sms * 4),
               dim3(kCopyThreads), 0, st, static_cast<const int32_t*>(idx), vmap, R, E, V, vidx);
    note_launches(1);
    launch_dispatch(vidx, T, k, V, offsets, row_token, inv, active, disp, st);
  } else if (T > 0) {
    launch_dispatch(idx, T, k, E, offsets, row_token, inv, active, disp, st);
  }
  launch_pdl(ep_send_kernel, dim3(R > 0 ? (R < sms ? R : sms) : 1), dim3(kXferThreads), 0, st,
             static_cast<const char*>(x), static_cast<const int32_t*>(row_token), static_cast<const int32_t*>(offsets),
             R, T, epr, world, c->rank, c->cap, row_bytes, c->peers, c->L);
  const size_t psmem = (size_t)(2 * world * epr + world + epr + 1) * sizeof(int);
  launch_pdl(ep_prepare_kernel, dim3(1), dim3(kPrepThreads), psmem, st, static_cast<const char*>(c->local), c->L,
             world, c->cap, epr, loff, lact, lrow, ret_src, ret_row);
  const char* recv = c->local + c->L.recv_x;
  mark(2);
  const cudaEvent_t mid = marks ? marks[3] : nullptr;
  // the decode down kernel stores each row straight into its source's
  // return buffer (no separate return copy)
  RowScatter scatter{};
  for (int r = 0; r < world; ++r) scatter.base[r] = reinterpret_cast<float*>(c->peers.base[r] + c->L.y_back);
  scatter.src = ret_src;
  scatter.row = ret_row;
  scatter.nbase = world;
  scatter.cap = c->cap;
  bool scattered = false;
  int s;
  if (path == PHMOE_PATH_PREFILL)
    s = launch_ffn_prefill(recv, lrow, loff, lact, w13_q, w13_s, w2_q, w2_s, (int)capr, c->H, epr, 1, I, G, h, y, st,
                           mid);
  else
    s = launch_ffn_decode(recv, x_dtype, lrow, loff, lact, w13_q, w13_s, w2_q, w2_s, (int)capr, c->H, epr, 1, I, G, h,
                          y, st, mid, lrow, loff + epr,  // encode only the rows that arrived
                          false, &scatter, &scattered);
  if (s) return s;
  mark(4);
  if (scattered)
    launch_pdl(ep_flag_kernel, dim3(1), dim3(32), 0, st, c->peers, c->L, world, c->rank);
  else
    launch_pdl(ep_return_kernel, dim3(sms), dim3(kXferThreads), 0, st, static_cast<const float*>(y),
               static_cast<const int32_t*>(loff), epr, static_cast<const int32_t*>(ret_src),
               static_cast<const int32_t*>(ret_row), world, c->rank, c->cap, c->H, c->peers, c->L);
  launch_pdl(ep_wait_kernel, dim3(1), dim3(32), 0, st, c->local, c->L, world);
  if (T > 0)
    launch_combine(reinterpret_cast<const float*>(c->local + c->L.y_back), inv, wts, T, k, c->H, out, x_dtype, st);
  mark(5);
  note_launches(4 + (T > 0 ? 3 : 0));
  return PHMOE_OK;
}

int ep_slots(const EpContext* c) { return c->epr; }

int ep_info(const EpContext* c, int* rank, int* world, int* max_tokens, int* top_k, int* H, int* E) {
  *rank = c->rank;
  *world = c->world;
  *max_tokens = c->max_tokens;
  *top_k = c->top_k;
  *H = c->H;
  *E = c->E;
  return c->connected ? 1 : 0;
}

}  // namespace phmoe
