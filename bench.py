#!/usr/bin/env python3
"""Benchmark of the B200 sparse-MoE layer (BASELINE config 2 at N=1).

Workload: one Qwen3-30B-A3B-shaped MoE layer (hidden 2048, 128 experts,
top-8 renormalised, intermediate 768, SwiGLU, int4 group-64 experts, bf16
activations N(0,1), router weight N(0, 0.02^2), seed 1), decode batch of
``--tokens`` tokens (default 64) per GPU. A step is one layer forward. Eight
distinct layers' weights (seeds 1..8, 2.6 GB) are cycled step by step, so
every step streams its experts from HBM (the working set is ~20x the 126 MB
L2); no explicit flush is needed.

* ``value``: tokens/s over K steps replayed from CUDA graphs, inputs resident
  in HBM, timed with CUDA events; max over ranks for N > 1.
* ``e2e``: the same through the public API (``phantom_moe.HostPipeline``
  over ``MoeLayer``s), every step copying its activations host->device from
  pinned memory and its output back, the copies on their own streams
  (overlapping the neighbouring steps' layers), timed with CUDA events from
  before the first copy in to after the last copy out; ``e2e.sync`` is the
  same with one stream and a host synchronisation per step.
* ``roofline``: the dominant kernels, the decode expert FFN (fixed-point
  encoding of x, gate/up, down), called back to back over the cycled layers
  inside one CUDA graph and timed with CUDA events around the replays (per
  call: device time of the three kernels, programmatic launch between them
  as in the layer); algorithmic bytes = packed int4 weights + fp16 scales
  of every expert hit + x fx rows read + h written and read + y written.
  The per-stage times of the layer (CUDA events the library records between
  its kernels, which also stop the kernels' launch overlap) are in
  ``stages``.
* ``cpu_baseline``: transformers' Qwen3MoeSparseMoeBlock (the MoE code
  PHANTOM runs) in fp32 on the host cores, same layer and batch.

With N > 1 (torchrun), experts are sharded expert-parallel (128/N per
rank), each rank routes its own ``--tokens`` tokens (weak scaling), and the
rows and expert outputs move through peer memory over NVLink inside one
library call per layer (``--ep-exchange nccl``: NCCL all-to-alls instead).

``--impl reference`` times the reference's CPU path alone (rank 0).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "solution-is-all-you-need_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

H, E, K_TOP, I, G = 2048, 128, 8, 768, 64
SWEEP = (1, 4, 16, 64, 256)
METRIC = "MoE-layer tokens/s (Qwen3-30B-A3B-shaped layer, int4 g64, bf16 decode)"
EXPERT_BYTES = (2 * I * H // 2 + 2 * I * (H // G) * 2) + (H * I // 2 + H * (I // G) * 2)  # 2,506,752
W13_BYTES = 2 * I * H // 2 + 2 * I * (H // G) * 2  # 1,671,168 per expert


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def dist_info():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ---------------------------------------------------------------------------
# weights
# ---------------------------------------------------------------------------

def make_layer(seed: int, device, expert_range=None):
    """Router weight (bf16 [E, H]) and packed experts of one layer, drawn
    N(0, 0.02^2) from ``seed``. ``expert_range`` keeps only those experts
    (expert-parallel shard); the full draw is made so shards agree."""
    import phantom_moe as pm
    g = torch.Generator(device=device).manual_seed(seed)
    wr = (torch.randn(E, H, device=device, generator=g) * 0.02).to(torch.bfloat16)
    w13 = torch.randn(E, 2 * I, H, device=device, generator=g) * 0.02
    lo, hi = expert_range if expert_range else (0, E)
    p13 = pm.quantize_int4(w13[lo:hi].contiguous(), G)
    del w13
    w2 = torch.randn(E, H, I, device=device, generator=g) * 0.02
    p2 = pm.quantize_int4(w2[lo:hi].contiguous(), G)
    del w2
    return wr, pm.PackedExperts(p13[0], p13[1], p2[0], p2[1], G)


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------

class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"phmoe_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = [r.split(", ") for r in self.path.read_text().strip().splitlines() if r.count(",") >= 8]
        try:
            self.path.unlink()
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        loaded = sorted(sm)[len(sm) // 2:] if sm else []
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": reasons, "samples": len(rows),
                "power_w_max": max((float(r[3]) for r in rows if r[3].replace(".", "").isdigit()), default=None)}


def bench_config(ws: int, T: int, args) -> dict:
    """The workload description both arms print as ``config`` (identical for
    the same N and flags): what is computed, not what was measured."""
    cfg = {"workload": f"qwen3-30b-a3b moe layer decode T={T}" + (" per GPU, expert-parallel" if ws > 1 else ""),
           "hidden": H, "experts": E, "top_k": K_TOP, "intermediate": I, "group_size": G, "tokens_per_gpu": T,
           "global_batch": ws * T, "parallelism": f"ep{ws}" if ws > 1 else "single-gpu",
           "l2": f"inputs larger than L2: {args.layers} layers' weights cycled per step",
           "graph": ("CUDA graph per layer" if ws == 1 or getattr(args, "ep_exchange", "peer") == "peer"
                     else "eager layer calls (NCCL all-to-alls)")}
    if ws > 1:
        cfg["experts_per_gpu"] = E // ws
        cfg["exchange"] = ("peer-memory stores over NVLink with epoch flags (phmoe_ep_layer)"
                           if args.ep_exchange == "peer" else
                           "NCCL all_to_all_single: counts, bf16 rows out, fp32 rows back")
    return cfg


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def run_single_gpu(args, device):
    import phantom_moe as pm
    from phantom_moe import _lib
    lib = pm.load_library()
    L = args.layers
    t0 = time.time()
    layers = [make_layer(1 + l, device) for l in range(L)]
    torch.cuda.synchronize()
    log(f"[bench] built {L} layers in {time.time() - t0:.1f}s")
    stream = torch.cuda.Stream(device)
    results = {}
    headline = None
    Ts = sorted(set(SWEEP) | {args.tokens}) if args.sweep else [args.tokens]
    for T in Ts:
        g = torch.Generator(device=device).manual_seed(1000 + T)
        xs = [torch.randn(T, H, device=device, generator=g).to(torch.bfloat16) for _ in range(L)]
        outs = [torch.empty(T, H, device=device, dtype=torch.bfloat16) for _ in range(L)]
        wsp = torch.empty(pm.workspace_bytes(T, H, E, K_TOP, I), dtype=torch.uint8, device=device)
        # unique experts hit per layer (algorithmic bytes)
        U = []
        for l in range(L):
            _, idx, _ = pm.moe_layer(xs[l], layers[l][0], *_pk(layers[l][1]), K_TOP, return_routing=True)
            U.append(int(torch.unique(idx).numel()))
        torch.cuda.synchronize()
        # capture one graph per layer
        graphs = []
        with torch.cuda.stream(stream):
            for l in range(L):  # warm-up outside capture
                pm.moe_layer(xs[l], layers[l][0], *_pk(layers[l][1]), K_TOP, out=outs[l], workspace=wsp)
            stream.synchronize()
            n0 = lib.phmoe_kernel_launch_count()
            for l in range(L):
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=stream):
                    pm.moe_layer(xs[l], layers[l][0], *_pk(layers[l][1]), K_TOP, out=outs[l], workspace=wsp)
                graphs.append(gr)
            launches_per_step = (lib.phmoe_kernel_launch_count() - n0) / L
        K, W = args.steps, args.warmup
        with torch.cuda.stream(stream):
            for i in range(W):
                graphs[i % L].replay()
            stream.synchronize()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record(stream)
            for i in range(K):
                graphs[i % L].replay()
            ev1.record(stream)
            ev1.synchronize()
        ms = ev0.elapsed_time(ev1) / K
        # per-stage device time (eager calls queued behind a sleep so launch gaps do not count)
        stage = profile_stages(pm, lib, layers, xs, outs, stream, n_calls=min(64, max(8, K)))
        mean_u = float(np.mean(U))
        R = T * K_TOP
        gateup_bytes = mean_u * W13_BYTES + R * H * 2 + R * I * 4
        ffn_bytes = mean_u * EXPERT_BYTES + R * H * 2 + 2 * R * I * 4 + R * H * 4
        layer_bytes = mean_u * EXPERT_BYTES + E * H * 2 + 2 * T * H * 2
        res = {"tokens": T, "ms_per_step": ms, "tokens_per_s": T / (ms / 1e3),
               "unique_experts_mean": mean_u, "layer_GBps": layer_bytes / (ms / 1e3) / 1e9,
               "stage_ms": stage, "gateup_GBps": gateup_bytes / (stage["ffn_gateup"] / 1e3) / 1e9,
               "ffn_GBps": ffn_bytes / ((stage["ffn_gateup"] + stage["ffn_down"]) / 1e3) / 1e9,
               "launches_per_step": launches_per_step}
        results[T] = res
        log(f"[bench] T={T:4d} {ms * 1e3:8.1f} us/step {res['tokens_per_s'] / 1e6:7.3f} Mtok/s "
            f"layer {res['layer_GBps']:7.0f} GB/s gateup {res['gateup_GBps']:7.0f} GB/s U={mean_u:.1f} "
            f"stages(us) " + " ".join(f"{k}={v * 1e3:.1f}" for k, v in stage.items()))
        if T == args.tokens:
            headline = dict(res, graphs=graphs, xs=xs, outs=outs, wsp=wsp, gateup_bytes=gateup_bytes)
        else:
            del graphs
    return layers, results, headline


def _pk(p):
    return p.w13_q, p.w13_scales, p.w2_q, p.w2_scales


def profile_stages(pm, lib, layers, xs, outs, stream, n_calls):
    from phantom_moe import _lib
    import ctypes
    L = len(layers)
    with torch.cuda.stream(stream):
        _lib.call("phmoe_profile_begin", n_calls)
        torch.cuda._sleep(50_000_000)  # ~25 ms: the CPU queues every call before the GPU starts
        for i in range(n_calls):
            l = i % L
            pm.moe_layer(xs[l], layers[l][0], *_pk(layers[l][1]), K_TOP, out=outs[l])
        arr = (ctypes.c_float * _lib.NUM_STAGES)()
        n = ctypes.c_int(0)
        _lib.call("phmoe_profile_end", arr, _lib.NUM_STAGES, ctypes.byref(n))
    return {name: arr[i] / max(n.value, 1) for i, name in enumerate(_lib.STAGE_NAMES)}


def e2e_single(args, device, layers, T):
    """Public-API path with host<->device copies inside the timed region.

    ``phantom_moe.HostPipeline`` over the bench's layers: every step copies
    its tokens host->device from pinned memory, runs the layer (a CUDA graph
    per layer and device slot) and copies its output device->host; the
    copies run on their own streams, so those of neighbouring steps overlap
    the layer. ``sync`` is the same steps issued on one stream with a host
    synchronisation after each."""
    import phantom_moe as pm
    L = len(layers)
    g = torch.Generator().manual_seed(2000 + T)
    xh = [torch.randn(T, H, generator=g).to(torch.bfloat16).pin_memory() for _ in range(L)]
    oh = [torch.empty(T, H, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    moe = [pm.MoeLayer(layers[l][0], *_pk(layers[l][1]), K_TOP) for l in range(L)]
    pipe = pm.HostPipeline(moe, T, H, device=device, depth=2)
    for i in range(args.warmup):
        pipe.submit(xh[i % L], oh[i % 2])
    pipe.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(pipe.copy_in)
    for i in range(args.steps):
        pipe.submit(xh[i % L], oh[i % 2])
    ev1.record(pipe.copy_out)
    ev1.synchronize()
    pipe.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    # the same steps, synchronous: copy in, replay, copy out, wait
    xd = torch.zeros(T, H, dtype=torch.bfloat16, device=device)  # graphed() warms up on its contents
    od = torch.empty(T, H, dtype=torch.bfloat16, device=device)
    run = [m.graphed(xd, od) for m in moe]
    st = torch.cuda.current_stream(device)
    for i in range(args.warmup):
        xd.copy_(xh[i % L], non_blocking=True)
        oh[0].copy_(run[i % L](), non_blocking=True)
        st.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(st)
    for i in range(args.steps):
        xd.copy_(xh[i % L], non_blocking=True)
        oh[0].copy_(run[i % L](), non_blocking=True)
        st.synchronize()
    s1.record(st)
    s1.synchronize()
    ms_sync = s0.elapsed_time(s1) / args.steps
    return {"value": T / (ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": T * H * 2,
            "d2h_bytes_per_step": T * H * 2, "ms_per_step": ms,
            "api": "phantom_moe.HostPipeline(MoeLayer per layer).submit(x_host, out_host) per step: pinned host -> "
                   "device copy of the step's tokens, the layer (CUDA graph), device -> host copy of its output, "
                   "each on its own stream ordered by events; timed from before the first copy in to after the "
                   "last copy out",
            "sync": {"value": T / (ms_sync / 1e3), "ms_per_step": ms_sync,
                     "api": "MoeLayer(...).graphed(x, out) per step on one stream, copies in and out, "
                            "host synchronised after every step"}}


def cpu_baseline(layers_host_fn, T, budget_s):
    """transformers' Qwen3MoeSparseMoeBlock, fp32, all host threads."""
    from oracle import tf_ref
    threads = tf_ref.host_threads()
    torch.set_num_threads(threads)
    wr, w13_q, w13_s, w2_q, w2_s = layers_host_fn()
    blk = tf_ref.build_block("qwen3", wr, w13_q, w13_s, w2_q, w2_s, K_TOP, G)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(3000 + T)).to(torch.bfloat16).float().numpy()
    tf_ref.forward(blk, x)  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        tf_ref.forward(blk, x)
        n += 1
        el = time.perf_counter() - t0
        if (el >= budget_s and n >= 3) or n >= 1000:
            break
    return {"value": n * T / el, "unit": "tokens/s", "cores": threads, "kind": "reference",
            "sample": f"transformers 5.5.0 Qwen3MoeSparseMoeBlock fp32 (eager experts loop), layer seed 1, "
                      f"T={T}, {n} forwards in {el:.1f}s, torch threads={threads}, cpu={tf_ref.cpu_model()}"}


def host_layer0_gpu():
    """Layer-0 weights (seed 1) packed by this library's CUDA quantiser and
    copied to the host (our arm's CPU-baseline leg; the bytes equal
    :func:`host_layer0_cpu`'s, as the GPU parity tests check)."""
    wr, pk = make_layer(1, torch.device("cuda", torch.cuda.current_device()))
    return (wr.float().cpu().numpy(), pk.w13_q.cpu().numpy(), pk.w13_scales.cpu().numpy(),
            pk.w2_q.cpu().numpy(), pk.w2_scales.cpu().numpy())


def host_layer0_cpu():
    """Layer-0 weights (seed 1): the same torch draw as :func:`make_layer`,
    quantised on the host by the oracle's quantiser. The reference arm uses
    this so that it never loads this library."""
    from oracle import moe_oracle as O
    g = torch.Generator().manual_seed(1)
    wr = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16).float().numpy()
    w13 = torch.randn(E, 2 * I, H, generator=g) * 0.02
    parts13 = [O.quantize_int4(w13[e].numpy(), G) for e in range(E)]
    del w13
    w2 = torch.randn(E, H, I, generator=g) * 0.02
    parts2 = [O.quantize_int4(w2[e].numpy(), G) for e in range(E)]
    return (wr, np.stack([p for p, _ in parts13]), np.stack([s for _, s in parts13]),
            np.stack([p for p, _ in parts2]), np.stack([s for _, s in parts2]))


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def load_traffic(T):
    """DRAM bytes (read + write) per call of the decode FFN's two weight
    kernels at batch T, from the ncu capture summarised in profiles/."""
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        d = json.loads(p.read_text())
        g, dn = d.get(f"ffn_gateup_T{T}"), d.get(f"ffn_down_T{T}")
        if g is not None and dn is not None:
            return float(g) + float(dn)
    return None


def ffn_chain_timing(pm, layers, T, device, calls=64, replays=8):
    """The decode expert FFN alone (phmoe_expert_ffn_decode: fx encoding of
    x, gate/up, down) over the cycled layers, `calls` back-to-back calls
    captured in one CUDA graph on fixed dispatched rows; returns (us per
    call, algorithmic bytes per call)."""
    from phantom_moe import _lib
    L = len(layers)
    g = torch.Generator(device=device).manual_seed(4242 + T)
    R = T * K_TOP
    ins, us = [], []
    for l in range(L):
        x = torch.randn(T, H, device=device, generator=g).to(torch.bfloat16)
        idx, _, _ = pm.router(x, layers[l][0], K_TOP)
        offsets, row_token, _, active = pm.dispatch(idx, E)
        h = torch.empty(R * I, dtype=torch.float32, device=device)
        y = torch.empty(R, H, dtype=torch.float32, device=device)
        ins.append((x, row_token, offsets, active, h, y) + tuple(_pk(layers[l][1])))
        us.append(int(torch.unique(idx).numel()))
    stream = torch.cuda.Stream(device)

    def call(i):
        x, rt, off, act, h, y, w13q, w13s, w2q, w2s = ins[i % L]
        _lib.call("phmoe_expert_ffn_decode", x.data_ptr(), 1, rt.data_ptr(), off.data_ptr(), act.data_ptr(),
                  w13q.data_ptr(), w13s.data_ptr(), w2q.data_ptr(), w2s.data_ptr(), T, H, E, K_TOP, I, G,
                  h.data_ptr(), y.data_ptr(), stream.cuda_stream)

    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for i in range(L):
            call(i)
        stream.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            for i in range(calls):
                call(i)
        gr.replay()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(replays):
            gr.replay()
        e1.record(stream)
        e1.synchronize()
    per_call_us = e0.elapsed_time(e1) * 1e3 / (replays * calls)
    mean_u = float(np.mean(us))
    nbytes = mean_u * EXPERT_BYTES + R * H * 2 + 2 * R * I * 2 + R * H * 4
    del gr
    return per_call_us, nbytes


def run_prefill(args, device):
    """Mixtral-8x7B-shaped layer (H 4096, 8 experts, top-2,
    I 14336, int4 g64), bf16 prefill batch of 4096 tokens (seed 2), through
    the tcgen05 prefill GEMMs. Timed with CUDA events over back-to-back layer
    calls (3 ms each; the 750 MB of packed weights and 64 MB of activations
    stream from HBM every step). Roofline: tensor, 2*3*H*I*k*T FLOPs per step."""
    import phantom_moe as pm
    from phantom_moe import _lib
    import ctypes
    Hm, Em, km, Im, Tm = 4096, 8, 2, 14336, args.prefill_tokens
    g = torch.Generator(device=device).manual_seed(2)
    x = torch.randn(Tm, Hm, device=device, generator=g).to(torch.bfloat16)
    wr = (torch.randn(Em, Hm, device=device, generator=g) * 0.02).to(torch.bfloat16)
    w13 = torch.randn(Em, 2 * Im, Hm, device=device, generator=g) * 0.02
    p13 = pm.quantize_int4(w13, G)
    del w13
    w2 = torch.randn(Em, Hm, Im, device=device, generator=g) * 0.02
    p2 = pm.quantize_int4(w2, G)
    del w2
    torch.cuda.empty_cache()
    wts = (p13[0], p13[1], p2[0], p2[1])
    out = torch.empty_like(x)
    wsp = torch.empty(pm.workspace_bytes(Tm, Hm, Em, km, Im, "prefill"), dtype=torch.uint8, device=device)
    st = torch.cuda.current_stream(device)
    for _ in range(max(3, args.warmup // 4)):
        pm.moe_layer(x, wr, *wts, km, path="prefill", out=out, workspace=wsp)
    steps = max(5, min(args.steps, 30))
    n0 = pm.load_library().phmoe_kernel_launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.synchronize()
    ev0.record(st)
    for _ in range(steps):
        pm.moe_layer(x, wr, *wts, km, path="prefill", out=out, workspace=wsp)
    ev1.record(st)
    ev1.synchronize()
    ms = ev0.elapsed_time(ev1) / steps
    launches = (pm.load_library().phmoe_kernel_launch_count() - n0) / steps
    _lib.call("phmoe_profile_begin", steps)
    torch.cuda._sleep(20_000_000)
    for _ in range(steps):
        pm.moe_layer(x, wr, *wts, km, path="prefill", out=out, workspace=wsp)
    arr = (ctypes.c_float * _lib.NUM_STAGES)()
    n = ctypes.c_int(0)
    _lib.call("phmoe_profile_end", arr, _lib.NUM_STAGES, ctypes.byref(n))
    stage = {name: arr[i] / max(n.value, 1) for i, name in enumerate(_lib.STAGE_NAMES)}
    flops = 2.0 * 3 * Hm * Im * km * Tm
    ffn_ms = stage["ffn_gateup"] + stage["ffn_down"]
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    burst = float(peaks.get("bf16_tflops", 1590.0))
    sustained = float(peaks.get("bf16_tflops_sustained", 1400.0))
    layer_tf = flops / (ms / 1e3) / 1e12
    ffn_tf = flops / (ffn_ms / 1e3) / 1e12
    res = {"workload": f"mixtral-8x7b moe layer prefill T={Tm} (BASELINE config 3), 1 GPU",
           "tokens_per_s": Tm / (ms / 1e3), "ms_per_step": ms, "steps": steps, "dtype": "fp16 MMA operands, fp32 accumulate",
           "stage_us": {k: round(v * 1e3, 1) for k, v in stage.items()},
           "roofline": {"kernel": "ffn (gate/up + down GEMMs)", "bound": "tensor", "achieved": ffn_tf,
                        "peak": burst, "unit": "TFLOP/s", "frac": ffn_tf / burst,
                        "frac_of_sustained": ffn_tf / sustained, "layer_tflops": layer_tf,
                        "peak_kind": "measured" if peaks else "fallback"},
           "gpu_launches_per_step": launches}
    log(f"[bench] prefill config 3: {ms * 1e3:.0f} us/layer {Tm / ms / 1e3:.3f} Mtok/s layer {layer_tf:.0f} TF/s "
        f"ffn {ffn_tf:.0f} TF/s ({ffn_tf / burst:.2f} of burst, {ffn_tf / sustained:.2f} of sustained)")
    del x, wr, wts, p13, p2, out, wsp
    torch.cuda.empty_cache()
    return res


def run_ours(args):
    ws, rank, local = dist_info()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if ws > 1:
        if args.zipf:
            import torch.distributed as dist
            z = run_ep_zipf(args, ws, rank, device)
            if rank == 0:
                print(json.dumps({"zipf": z}), flush=True)
            dist.barrier()
            dist.destroy_process_group()
            return
        return run_ep(args, ws, rank, device)
    if args.stack:
        print(json.dumps({"stack": run_stack(args, device)}), flush=True)
        return
    if args.prefill_only:
        print(json.dumps({"prefill": run_prefill(args, device)}), flush=True)
        return
    with ClockSampler(local) as clk:
        layers, results, hl = run_single_gpu(args, device)
        # sustained replay of the headline step while the sampler runs
        t_end = time.time() + args.clock_soak
        st = torch.cuda.current_stream(device)
        while time.time() < t_end:
            for i in range(200):
                hl["graphs"][i % len(hl["graphs"])].replay()
            st.synchronize()
    clocks = clk.summary()
    e2e = e2e_single(args, device, layers, args.tokens)
    T = args.tokens
    res = results[T]
    peak, peak_kind = load_peaks()
    gateup_bytes = hl["gateup_bytes"]
    import phantom_moe as pm
    ffn_us, ffn_bytes = ffn_chain_timing(pm, layers, T, device)
    achieved = ffn_bytes / (ffn_us / 1e6) / 1e9
    log(f"[bench] decode FFN alone at T={T}: {ffn_us:.1f} us per call, {achieved:.0f} GB/s")
    del layers, hl
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    prefill = run_prefill(args, device) if args.prefill else None
    hf = run_hf_generate(args, device) if args.hf_generate else None
    cpu = None
    if not args.no_cpu_baseline:
        cpu = cpu_baseline(host_layer0_gpu, T, args.cpu_budget)
    line = {
        "metric": METRIC, "value": res["tokens_per_s"], "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02^2) weights, int4 g64)",
        "config": bench_config(1, T, args),
        "sweep": {str(k): _sweep_entry(v) for k, v in results.items()},
        "roofline": {"kernel": "decode expert FFN (fx encode + ffn_gateup + ffn_down), back-to-back calls "
                               "in a CUDA graph", "bound": "hbm", "achieved": achieved, "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": load_traffic(T), "algorithmic_bytes_per_launch": ffn_bytes,
                     "us_per_call": ffn_us,
                     "stage_events": {"note": "per-stage CUDA events inside the layer call (they also stop "
                                              "the launch overlap between kernels, so each stage includes "
                                              "its kernel's launch and drain)",
                                      "ffn_gateup_GBps": gateup_bytes / (res["stage_ms"]["ffn_gateup"] / 1e3) / 1e9,
                                      "ffn_GBps": res["ffn_GBps"]}},
        "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks,
        "gpu_launches": int(round(res["launches_per_step"] * args.steps)),
        "prefill": prefill,
    }
    if hf is not None:
        line["hf_generate"] = hf
    print(json.dumps(line), flush=True)


def run_hf_generate(args, device):
    """End-to-end decode through transformers' generate: a Qwen3-30B-A3B-shaped
    model (real MoE layer shapes, ``--hf-layers`` decoder layers, random
    weights, bf16), greedy decoding of ``--hf-new-tokens`` tokens for a batch
    of ``--tokens`` sequences; transformers' own experts path (its default
    ``grouped_mm`` on bf16 weights, and the per-expert ``eager`` loop) against
    the same model after ``phantom_moe.install_into`` (int4 g64 experts on
    this library's kernels). Timed with CUDA events around each generate."""
    import transformers as tf
    import phantom_moe as pm
    B, N, P = args.tokens, args.hf_new_tokens, 16
    cfg = tf.Qwen3MoeConfig(hidden_size=H, num_hidden_layers=args.hf_layers, num_attention_heads=32,
                            num_key_value_heads=4, head_dim=128, vocab_size=32000, num_experts=E,
                            num_experts_per_tok=K_TOP, moe_intermediate_size=I, norm_topk_prob=True,
                            intermediate_size=6144, max_position_embeddings=4096)
    torch.manual_seed(0)
    with torch.device(device):
        model = tf.Qwen3MoeForCausalLM(cfg).to(torch.bfloat16).eval()
    with torch.no_grad():
        for p in model.parameters():
            if p.dim() >= 2:
                p.normal_(0.0, 0.02)
    ids = torch.randint(0, cfg.vocab_size, (B, P), device=device, generator=torch.Generator(device=device).manual_seed(1))

    def timed(reps=2):
        with torch.no_grad():
            model.generate(ids, max_new_tokens=4, min_new_tokens=4, do_sample=False)  # warm-up
            best = None
            for _ in range(reps):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                model.generate(ids, max_new_tokens=N, min_new_tokens=N, do_sample=False)
                e1.record()
                e1.synchronize()
                ms = e0.elapsed_time(e1)
                best = ms if best is None else min(best, ms)
        return B * N / (best / 1e3)

    out = {"workload": f"qwen3-30b-a3b-shaped model, {args.hf_layers} layers, batch {B}, prompt {P}, "
                       f"{N} new tokens, greedy", "unit": "generated tokens/s"}
    model.config._experts_implementation = "grouped_mm"
    out["transformers_grouped_mm_bf16"] = timed()
    model.config._experts_implementation = "eager"
    out["transformers_eager_loop_bf16"] = timed(reps=1)
    model.config._experts_implementation = "grouped_mm"
    pm.install_into(model)
    out["phantom_moe_int4"] = timed()
    out["speedup_vs_grouped_mm"] = out["phantom_moe_int4"] / out["transformers_grouped_mm_bf16"]
    out["speedup_vs_eager_loop"] = out["phantom_moe_int4"] / out["transformers_eager_loop_bf16"]
    del model
    torch.cuda.empty_cache()
    return out


def run_stack(args, device):
    """BASELINE config 4 on one GPU: a stack of ``--stack`` Qwen3-30B-A3B-shaped
    MoE layers (MoE FFN only, attention omitted; layer l's weights drawn from
    seed 100 + l, int4 g64, 15.4 GB for 48 layers), decode T = ``--tokens``,
    each layer on its own seeded input, the whole stack captured as one CUDA
    graph per step (weights read from HBM: the stack is 120x the L2)."""
    import phantom_moe as pm
    Ls, T = args.stack, args.tokens
    layers = [make_layer(100 + l, device) for l in range(Ls)]
    g = torch.Generator(device=device).manual_seed(3000 + T)
    xs = [torch.randn(T, H, device=device, generator=g).to(torch.bfloat16) for _ in range(Ls)]
    outs = [torch.empty_like(x) for x in xs]
    moe = [pm.MoeLayer(wr, *_pk(pk), K_TOP) for wr, pk in layers]
    side = torch.cuda.Stream(device=device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for l in range(Ls):
            moe[l](xs[l], out=outs[l])
    torch.cuda.current_stream(device).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for l in range(Ls):
            moe[l](xs[l], out=outs[l])
    st = torch.cuda.current_stream(device)
    for _ in range(args.warmup):
        graph.replay()
    st.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(st)
    for _ in range(args.steps):
        graph.replay()
    ev1.record(st)
    ev1.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    wbytes = sum(pk.w13_q.numel() + pk.w13_scales.numel() * 2 + pk.w2_q.numel() + pk.w2_scales.numel() * 2
                 for _, pk in layers)
    del graph, moe, layers
    torch.cuda.empty_cache()
    return {"workload": f"{Ls}-layer qwen3-30b-a3b MoE stack (MoE FFN only), decode T={T}, 1 GPU, CUDA graph",
            "layers": Ls, "tokens_per_gpu": T, "ms_per_step": ms, "tokens_per_s": T / (ms / 1e3),
            "us_per_layer": ms * 1e3 / Ls, "packed_weight_GB": wbytes / 1e9}


def run_ep_prefill(args, ws, rank, device):
    """BASELINE config 3 under expert parallelism: the Mixtral-8x7B-shaped
    layer (H 4096, 8 experts, top-2, I 14336, int4 g64) with its experts
    sharded 8/N per rank and --prefill-tokens tokens in total (strong scaling:
    4096/N per rank, seed 2, the same draw on every rank), through the peer
    exchange and the tcgen05 prefill GEMMs. Max over ranks."""
    import torch.distributed as dist
    import phantom_moe as pm
    from phantom_moe import ep
    Hm, Em, km, Im, Tt = 4096, 8, 2, 14336, args.prefill_tokens
    T = Tt // ws
    lo, hi = ep.shard_range(Em, ws, rank)
    g = torch.Generator(device=device).manual_seed(2)
    x = torch.randn(Tt, Hm, device=device, generator=g).to(torch.bfloat16)[rank * T:(rank + 1) * T].contiguous()
    wr = (torch.randn(Em, Hm, device=device, generator=g) * 0.02).to(torch.bfloat16)
    w13 = torch.randn(Em, 2 * Im, Hm, device=device, generator=g) * 0.02
    p13 = pm.quantize_int4(w13[lo:hi].contiguous(), G)
    del w13
    w2 = torch.randn(Em, Hm, Im, device=device, generator=g) * 0.02
    p2 = pm.quantize_int4(w2[lo:hi].contiguous(), G)
    del w2
    torch.cuda.empty_cache()
    wts = (p13[0], p13[1], p2[0], p2[1])
    exchange = ep.PeerExchange(None, T, km, Hm, Em) if args.ep_exchange == "peer" else None
    stream = torch.cuda.current_stream(device)

    def step():
        return ep.moe_layer_ep(x, wr, *wts, km, True, G, None, path="prefill", exchange=exchange)

    # parity of the first call against the single-GPU prefill layer (all experts)
    gg = torch.Generator(device=device).manual_seed(2)
    torch.randn(Tt, Hm, device=device, generator=gg)
    torch.randn(Em, Hm, device=device, generator=gg)
    full13 = pm.quantize_int4(torch.randn(Em, 2 * Im, Hm, device=device, generator=gg) * 0.02, G)
    full2 = pm.quantize_int4(torch.randn(Em, Hm, Im, device=device, generator=gg) * 0.02, G)
    torch.cuda.empty_cache()
    ref = pm.moe_layer(x, wr, full13[0], full13[1], full2[0], full2[1], km, path="prefill")
    got = step()
    mism = torch.tensor([int((got != ref).sum().item()), ref.numel()], device=device, dtype=torch.int64)
    dist.all_reduce(mism)
    del full13, full2, ref, got
    torch.cuda.empty_cache()
    for _ in range(3):
        step()
    dist.barrier()
    torch.cuda.synchronize()
    steps = max(5, min(args.steps, 20))
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        step()
    ev1.record(stream)
    ev1.synchronize()
    dist.barrier()
    t = torch.tensor([ev0.elapsed_time(ev1) / steps], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    if exchange is not None:
        exchange.close()
    del x, wr, wts, p13, p2
    torch.cuda.empty_cache()
    flops = 2.0 * 3 * Hm * Im * km * Tt
    return {"workload": f"config 3: mixtral-8x7b moe layer prefill, {Tt} tokens over {ws} GPUs "
                        f"({T} per GPU), {Em // ws} experts per GPU, strong scaling",
            "exchange": args.ep_exchange, "tokens_per_s": Tt / (ms / 1e3), "ms_per_step": ms, "steps": steps,
            "tflops_all_gpus": flops / (ms / 1e3) / 1e12,
            "ep_parity": {"compared": "first call, every rank's tokens, EP prefill layer vs single-GPU prefill layer",
                          "elements": int(mism[1].item()), "mismatches": int(mism[0].item()),
                          "result": "bit-exact" if int(mism[0].item()) == 0 else "MISMATCH"}}


def run_ep_stack(args, ws, rank, device):
    """BASELINE config 4 under expert parallelism: ``--stack-ep`` (default 48)
    Qwen3-30B-A3B-shaped MoE layers (attention omitted), 128/N experts of each
    layer per GPU, ``--tokens`` decode tokens per GPU, the peer-memory
    exchange in every layer; a step is one pass through the whole stack. Max
    over ranks."""
    import torch.distributed as dist
    import phantom_moe as pm
    from phantom_moe import ep
    Ls, T = args.stack_ep, args.tokens
    lo, hi = ep.shard_range(E, ws, rank)
    layers = [make_layer(100 + l, device, expert_range=(lo, hi)) for l in range(Ls)]
    g = torch.Generator(device=device).manual_seed(3000 + T + 7919 * rank)
    x0 = torch.randn(T, H, device=device, generator=g).to(torch.bfloat16)
    exchange = ep.PeerExchange(None, T, K_TOP, H, E)
    stream = torch.cuda.current_stream(device)

    def run_stack():
        h = x0
        for wr, pk in layers:
            h = ep.moe_layer_ep(h, wr, *_pk(pk), K_TOP, True, G, None, exchange=exchange)
        return h

    for _ in range(2):
        run_stack()
    dist.barrier()
    torch.cuda.synchronize()
    steps = max(3, min(args.steps, 10))
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        run_stack()
    ev1.record(stream)
    ev1.synchronize()
    dist.barrier()
    t = torch.tensor([ev0.elapsed_time(ev1) / steps], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    exchange.close()
    wbytes = sum(pk.w13_q.numel() + pk.w13_scales.numel() * 2 + pk.w2_q.numel() + pk.w2_scales.numel() * 2
                 for _, pk in layers)
    del layers
    torch.cuda.empty_cache()
    return {"workload": f"config 4: {Ls}-layer qwen3-30b-a3b MoE stack (MoE FFN only), decode T={T} per GPU, "
                        f"{E // ws} experts per GPU per layer, peer exchange per layer",
            "layers": Ls, "ms_per_step": ms, "tokens_per_s": ws * T / (ms / 1e3), "us_per_layer": ms * 1e3 / Ls,
            "steps": steps, "packed_weight_GB_per_gpu": wbytes / 1e9}


def run_ep_zipf(args, ws, rank, device, replicate=True):
    """BASELINE config 5 under expert parallelism: 8192 tokens in total
    (8192 / N per rank), router logits biased by log of a Zipf(1.2) prior over
    the experts (a constant input feature x[:, 0] = 1 meeting router column
    0 = log p_i), against the same layer without the bias, and with hot
    experts replicated (``phantom_moe.ep.plan_replicas`` over the Zipf case's
    expert loads, ``--replica-slots`` extra slots per rank); reports the load
    imbalance, every rank's received rows and the step time (max over ranks)."""
    import torch.distributed as dist
    import phantom_moe as pm
    from phantom_moe import ep
    T = 8192 // ws
    lo, hi = ep.shard_range(E, ws, rank)
    wr, pk_full = make_layer(7, device)
    full = _pk(pk_full)
    shard = tuple(t[lo:hi] for t in full)
    g = torch.Generator(device=device).manual_seed(4000 + 7919 * rank)
    x = torch.randn(T, H, device=device, generator=g)
    prior = torch.log(torch.arange(1, E + 1, device=device, dtype=torch.float32) ** -1.2)
    wr_skew = wr.float()
    wr_skew[:, 0] = prior
    x_skew = x.clone()
    x_skew[:, 0] = 1.0
    cases = {"balanced": (x.to(torch.bfloat16), wr), "zipf": (x_skew.to(torch.bfloat16), wr_skew.to(torch.bfloat16))}
    if replicate:
        cases["zipf_replicated"] = None
    stream = torch.cuda.current_stream(device)
    res = {}
    for name in cases:
        placement = None
        if name == "zipf_replicated":
            xc, wc = cases["zipf"]
            placement = ep.plan_replicas(res["zipf"]["expert_rows"], ws, args.replica_slots)
            weights = placement.local_weights(rank, *full)
        else:
            xc, wc = cases[name]
            weights = shard
        exchange = (ep.PeerExchange(None, T, K_TOP, H, E, placement=placement)
                    if args.ep_exchange == "peer" else None)
        st = {}
        ep.moe_layer_ep(xc, wc, *weights, K_TOP, True, G, None, stats=st, placement=placement)  # row counts
        loads = torch.tensor(st["recv_rows"], device=device, dtype=torch.float32)
        all_loads = [torch.zeros_like(loads) for _ in range(ws)]
        dist.all_gather(all_loads, loads)
        for _ in range(args.warmup):
            ep.moe_layer_ep(xc, wc, *weights, K_TOP, True, G, None, exchange=exchange, placement=placement)
        dist.barrier()
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for _ in range(args.steps):
            ep.moe_layer_ep(xc, wc, *weights, K_TOP, True, G, None, exchange=exchange, placement=placement)
        ev1.record(stream)
        ev1.synchronize()
        dist.barrier()
        t = torch.tensor([ev0.elapsed_time(ev1) / args.steps], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        idx, _, _ = pm.router(xc, wc, K_TOP)
        cnt = torch.bincount(idx.view(-1).long(), minlength=E).float()
        dist.all_reduce(cnt)
        recv = [float(v) for v in torch.stack(all_loads).sum(dim=1).tolist()]
        res[name] = {"ms_per_step": ms, "tokens_per_s": 8192 / (ms / 1e3),
                     "expert_load_max_over_mean": float(cnt.max() / cnt.mean()),
                     "rows_received_per_rank": recv, "rank_load_max_over_mean": max(recv) / (sum(recv) / ws),
                     "expert_rows": [int(v) for v in cnt.tolist()]}
        if placement is not None:
            res[name]["slots_per_rank"] = placement.slots_per_rank
            res[name]["copies_of_hottest"] = len(placement.copies(int(cnt.argmax())))
        if exchange is not None:
            exchange.close()
        del weights
    for v in res.values():
        del v["expert_rows"]
    res["zipf_over_balanced_time"] = res["zipf"]["ms_per_step"] / res["balanced"]["ms_per_step"]
    if replicate:
        res["zipf_replicated_over_balanced_time"] = (res["zipf_replicated"]["ms_per_step"] /
                                                     res["balanced"]["ms_per_step"])
    del full, shard, pk_full
    torch.cuda.empty_cache()
    return {"workload": f"config 5: 8192 tokens over {ws} GPUs, Zipf(1.2) router prior, top-8 of 128",
            "exchange": args.ep_exchange, **res}


def _sweep_entry(v):
    return {"tokens_per_s": round(v["tokens_per_s"], 1), "us_per_step": round(v["ms_per_step"] * 1e3, 2),
            "layer_GBps": round(v["layer_GBps"], 1), "gateup_GBps": round(v["gateup_GBps"], 1),
            "unique_experts": v["unique_experts_mean"],
            "stage_us": {k: round(s * 1e3, 2) for k, s in v["stage_ms"].items()}}


def run_ep(args, ws, rank, device):
    """N > 1: experts sharded E/N per rank, each rank routes its own
    ``--tokens`` tokens (weak scaling); rows move through peer memory
    (``--ep-exchange nccl``: NCCL all-to-alls). Unless ``--no-ep-extras``,
    BASELINE configs 5 (Zipf skew) and 3 (Mixtral prefill) are measured at
    this N too and reported in the same line. Every rank runs the same
    collectives in the same order."""
    import torch.distributed as dist
    import phantom_moe as pm
    from phantom_moe import ep
    lib = pm.load_library()
    L, T = args.layers, args.tokens
    lo, hi = ep.shard_range(E, ws, rank)
    layers = [make_layer(1 + l, device, expert_range=(lo, hi)) for l in range(L)]
    g = torch.Generator(device=device).manual_seed(1000 + T + 7919 * rank)
    xs = [torch.randn(T, H, device=device, generator=g).to(torch.bfloat16) for _ in range(L)]
    torch.cuda.synchronize()

    exchange = ep.PeerExchange(None, T, K_TOP, H, E) if args.ep_exchange == "peer" else None

    def step(i, x=None, stats=None):
        l = i % L
        return ep.moe_layer_ep(xs[l] if x is None else x, layers[l][0], *_pk(layers[l][1]), K_TOP, True, G,
                               None, stats=stats, exchange=None if stats is not None else exchange)

    # parity: the first step's output on every rank against the single-GPU
    # layer (all 128 experts) on the same tokens; the exchange returns fp32
    # rows and every row's result is independent of its batch, so the two
    # must agree bit for bit
    wr0, pk0 = make_layer(1, device)
    ref0 = pm.moe_layer(xs[0], wr0, *_pk(pk0), K_TOP, path="decode")
    got0 = step(0)
    mism = torch.tensor([int((got0 != ref0).sum().item()), ref0.numel()], device=device, dtype=torch.int64)
    dist.all_reduce(mism)
    parity = {"compared": "first step, every rank's T tokens, EP layer vs single-GPU phmoe_moe_layer with all "
                          f"{E} experts", "elements": int(mism[1].item()), "mismatches": int(mism[0].item()),
              "result": "bit-exact" if int(mism[0].item()) == 0 else "MISMATCH"}
    del wr0, pk0, ref0, got0
    torch.cuda.empty_cache()
    # imbalance and local experts hit, per layer (outside the timed region)
    hit, recv = [], []
    for l in range(L):
        st = {}
        step(l, stats=st)
        hit.append(st["local_experts_hit"])
        recv.append(sum(st["recv_rows"]))
    stream = torch.cuda.current_stream(device)
    # the peer-exchange layer as one CUDA graph per layer (its epoch lives in
    # device memory, so replays stay in step across ranks: every rank warms
    # up, captures and replays the same sequence)
    graphs, gouts = [], []
    if exchange is not None:
        gstream = torch.cuda.Stream(device)
        with torch.cuda.stream(gstream):
            for l in range(L):
                step(l)
            gstream.synchronize()
            for l in range(L):
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=gstream):
                    gouts.append(step(l))
                graphs.append(gr)
        torch.cuda.synchronize()
        dist.barrier()

    def run_step(i):
        if graphs:
            graphs[i % L].replay()
        else:
            step(i)

    def timed(fn, K, W):
        for i in range(W):
            fn(i)
        dist.barrier()
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for i in range(K):
            fn(i)
        ev1.record(stream)
        ev1.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        t = torch.tensor([ev0.elapsed_time(ev1) / K], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    n0 = lib.phmoe_kernel_launch_count()
    with ClockSampler(torch.cuda.current_device()) as clk:
        ms = timed(run_step, args.steps, args.warmup)
        launches = lib.phmoe_kernel_launch_count() - n0
        # sustained steps while the sampler runs (same count on every rank)
        n_soak = int(args.clock_soak / max(ms / 1e3, 1e-6))
        n_soak = torch.tensor([n_soak], device=device)
        dist.all_reduce(n_soak, op=dist.ReduceOp.MIN)
        for i in range(int(n_soak.item())):
            run_step(i)
        torch.cuda.synchronize()
    clocks = clk.summary()
    # end to end: pinned host tokens in, output back to the host, every step
    gh = torch.Generator().manual_seed(2000 + T + 7919 * rank)
    xh = [torch.randn(T, H, generator=gh).to(torch.bfloat16).pin_memory() for _ in range(L)]
    oh = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()
    xd = torch.empty(T, H, dtype=torch.bfloat16, device=device)

    def layer_on(i, xx):
        """The layer on input xx: the captured graph of layer i % L (its
        input buffer refilled first), or an eager call."""
        l = i % L
        if graphs:
            xs[l].copy_(xx, non_blocking=True)
            graphs[l].replay()
            return gouts[l]
        return step(i, x=xx)

    def e2e_step(i):
        xd.copy_(xh[i % L], non_blocking=True)
        out = layer_on(i, xd)
        oh.copy_(out, non_blocking=True)
        stream.synchronize()

    ms_e2e_sync = timed(e2e_step, args.steps, args.warmup)
    # the same through HostPipeline: copies on their own streams, the layer
    # (eager, with its peer exchange) on the pipeline's compute stream
    pipe = pm.HostPipeline([lambda xx, out, l=l: out.copy_(layer_on(l, xx)) for l in range(L)], T, H, device=device)
    ohp = [torch.empty(T, H, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    for i in range(args.warmup):
        pipe.submit(xh[i % L], ohp[i % 2])
    pipe.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(pipe.copy_in)
    for i in range(args.steps):
        pipe.submit(xh[i % L], ohp[i % 2])
    p1.record(pipe.copy_out)
    p1.synchronize()
    pipe.synchronize()
    dist.barrier()
    t = torch.tensor([p0.elapsed_time(p1) / args.steps], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_e2e = float(t.item())
    del pipe
    # per-stage device time on this rank (events the library records inside the layer)
    from phantom_moe import _lib
    import ctypes
    nprof = 32
    dist.barrier()
    _lib.call("phmoe_profile_begin", nprof)
    for i in range(nprof):
        step(i)
    arr = (ctypes.c_float * _lib.NUM_STAGES)()
    ncalls = ctypes.c_int(0)
    _lib.call("phmoe_profile_end", arr, _lib.NUM_STAGES, ctypes.byref(ncalls))
    ep_stage_names = ["router", "dispatch+send+prepare", "ffn_gateup", "ffn_down", "return+wait+combine"]
    stage_us = {nm: round(arr[i] / max(ncalls.value, 1) * 1e3, 1) for i, nm in enumerate(ep_stage_names)}
    # per-GPU weight bytes streamed per step (mean over layers and ranks)
    stats = torch.tensor([float(np.mean(hit)), float(max(recv)), float(np.mean(recv))], device=device)
    gathered = [torch.empty_like(stats) for _ in range(ws)]
    dist.all_gather(gathered, stats)
    if rank == 0:
        g_hit = float(np.mean([s[0].item() for s in gathered]))
        recv_all = [s[1].item() for s in gathered]
        recv_mean = float(np.mean([s[2].item() for s in gathered]))
        peak, peak_kind = load_peaks()
        bytes_gpu = g_hit * EXPERT_BYTES
        achieved = bytes_gpu / (ms / 1e3) / 1e9
        line = {
            "metric": METRIC, "value": ws * T / (ms / 1e3), "unit": "tokens/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02^2) weights, int4 g64)",
            "config": bench_config(ws, T, args),
            "ep_stats": {"local_experts_hit_mean": g_hit, "recv_rows_max_over_ranks": max(recv_all),
                         "recv_rows_mean": recv_mean, "stage_us_rank0": stage_us},
            "roofline": {"kernel": "layer (per GPU)", "bound": "hbm", "achieved": achieved, "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak, "traffic": None,
                         "algorithmic_bytes_per_launch": bytes_gpu},
            "cpu_baseline": None,
            "e2e": {"value": ws * T / (ms_e2e / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": T * H * 2,
                    "d2h_bytes_per_step": T * H * 2, "ms_per_step": ms_e2e,
                    "api": "phantom_moe.HostPipeline over moe_layer_ep (peer exchange) per step on every rank: "
                           "pinned host -> device copy of the rank's tokens, the layer, device -> host copy of "
                           "its output, copies on their own streams; max over ranks",
                    "sync": {"value": ws * T / (ms_e2e_sync / 1e3), "ms_per_step": ms_e2e_sync,
                             "api": "the same on one stream, host synchronised after every step"}},
            "clocks": clocks, "gpu_launches": int(launches * args.steps // (args.steps + args.warmup)),
            "ep_parity": parity,
        }
    if exchange is not None:
        exchange.close()
    # the same layer with the token exchange as NCCL all-to-alls: split sizes
    # read on the host every layer, and equal fixed-capacity blocks (T * k rows
    # per rank pair, no host synchronisation)
    nccl = None
    if args.ep_extras and args.ep_exchange == "peer":
        def nccl_step(i, cap=None):
            l = i % L
            return ep.moe_layer_ep(xs[l], layers[l][0], *_pk(layers[l][1]), K_TOP, True, G, None, path="decode",
                                   fixed_capacity=cap)
        ms_hc = timed(nccl_step, args.steps, args.warmup)
        ms_fc = timed(lambda i: nccl_step(i, T * K_TOP), args.steps, args.warmup)
        row_in, row_out = H * 2, H * 4  # bf16 rows out, fp32 results back
        nccl = {"host_counted": {"ms_per_step": ms_hc, "tokens_per_s": ws * T / (ms_hc / 1e3),
                                 "bytes_per_rank_per_step": int(T * K_TOP * (row_in + row_out)),
                                 "note": "all_to_all_single with split sizes copied to the host every layer "
                                         "(one device synchronisation per layer)"},
                "fixed_capacity": {"ms_per_step": ms_fc, "tokens_per_s": ws * T / (ms_fc / 1e3),
                                   "bytes_per_rank_per_step": int(ws * T * K_TOP * (row_in + row_out)),
                                   "note": f"equal splits of T*k = {T * K_TOP} rows per rank pair, no host "
                                           "synchronisation; the padded blocks move world x more bytes"},
                "peer_memory_ms_per_step": ms}
    # BASELINE configs 5 and 3 at this N (every rank runs both; rank 0 reports)
    extras = {}
    if args.ep_extras:
        del layers
        torch.cuda.empty_cache()
        extras["config5_zipf"] = run_ep_zipf(args, ws, rank, device, replicate=args.ep_extras_replicate)
        extras["config3_prefill_ep"] = run_ep_prefill(args, ws, rank, device)
        extras["config4_stack_ep"] = run_ep_stack(args, ws, rank, device)
    if rank == 0:
        if nccl is not None:
            line["nccl_exchange"] = nccl
        line.update(extras)
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    # a result that differs from the single-GPU layer is not a valid measurement
    bad = parity["mismatches"] + extras.get("config3_prefill_ep", {}).get("ep_parity", {}).get("mismatches", 0)
    if bad:
        log(f"[bench] expert-parallel output differs from the single-GPU layer in {bad} elements")
        raise SystemExit(3)


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------

def run_reference(args):
    """The reference's MoE path (transformers' Qwen3MoeSparseMoeBlock in fp32,
    the code PHANTOM runs) on the host cores, on the global batch our arm
    processes at this N. Runs on rank 0 only, never touches a GPU and never
    imports this library: the weights are drawn and quantised on the host."""
    ws, rank, local = dist_info()
    if rank != 0:
        return
    from oracle import tf_ref
    T = args.tokens
    Tg = ws * T
    threads = tf_ref.host_threads()
    torch.set_num_threads(threads)
    wr, w13_q, w13_s, w2_q, w2_s = host_layer0_cpu()
    blk = tf_ref.build_block("qwen3", wr, w13_q, w13_s, w2_q, w2_s, K_TOP, G)
    del w13_q, w13_s, w2_q, w2_s
    x = torch.randn(Tg, H, generator=torch.Generator().manual_seed(3000 + T)).to(torch.bfloat16).float().numpy()
    for _ in range(max(1, args.warmup)):
        tf_ref.forward(blk, x)
    steps = max(1, args.steps)
    t0 = time.perf_counter()
    for _ in range(steps):
        tf_ref.forward(blk, x)
    el = time.perf_counter() - t0
    v = steps * Tg / el
    sample = (f"transformers 5.5.0 Qwen3MoeSparseMoeBlock fp32 on the host (the MoE code PHANTOM runs), "
              f"{Tg} tokens per forward, {steps} forwards, torch threads={threads}, cpu={tf_ref.cpu_model()}")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": ws,
        "steps": steps, "warmup": args.warmup, "ms_per_step": el / steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": bench_config(ws, T, args),
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "reference", "sample": sample},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=64, help="decode tokens per GPU (headline)")
    ap.add_argument("--layers", type=int, default=8, help="distinct layers cycled (L2 defeat)")
    ap.add_argument("--no-sweep", dest="sweep", action="store_false")
    ap.add_argument("--no-prefill", dest="prefill", action="store_false",
                    help="skip the config-3 (Mixtral prefill) measurement")
    ap.add_argument("--prefill-only", action="store_true",
                    help="run only the config-3 prefill measurement (profiling)")
    ap.add_argument("--prefill-tokens", type=int, default=4096)
    ap.add_argument("--ep-exchange", choices=["peer", "nccl"], default="peer",
                    help="N > 1: token exchange through peer memory (default) or NCCL all-to-all")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of CPU-baseline work")
    ap.add_argument("--clock-soak", type=float, default=2.0, help="seconds of sustained replay for clocks")
    ap.add_argument("--hf-generate", action="store_true",
                    help="also time transformers generate with and without install_into (an extra JSON object)")
    ap.add_argument("--stack-ep", type=int, default=48,
                    help="N > 1: layers of the config-4 stack leg in the default line")
    ap.add_argument("--stack", type=int, default=0,
                    help="only time a decode step through this many MoE layers (config 4 on one GPU)")
    ap.add_argument("--no-ep-extras", dest="ep_extras", action="store_false",
                    help="N > 1: skip the config-5 (Zipf) and config-3 (expert-parallel prefill) legs")
    ap.add_argument("--no-ep-extras-replicate", dest="ep_extras_replicate", action="store_false",
                    help="N > 1: the default line's config-5 leg skips the hot-expert replication case")
    ap.add_argument("--replica-slots", type=int, default=8,
                    help="N > 1, config 5: extra expert slots per rank for copies of hot experts")
    ap.add_argument("--zipf", action="store_true",
                    help="N > 1: only the config-5 Zipf-skewed routing measurement (8192 tokens in total)")
    ap.add_argument("--hf-layers", type=int, default=4)
    ap.add_argument("--hf-new-tokens", type=int, default=32)
    return ap


def main():
    args = build_parser().parse_args()
    if args.warmup < 3:
        args.warmup = 3
    ws, rank, local = dist_info()
    if ws > 1 and args.impl == "ours":
        import datetime
        import torch.distributed as dist
        # keep stdout to the one JSON line (NCCL's version banner goes to stdout)
        if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
            os.environ["NCCL_DEBUG"] = "WARN"
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
