"""Helpers for the expert-parallel tests: checker ops over the numpy oracle
(so the exchange logic of phantom_moe.ep runs on CPU gloo ranks), seeded
cases, and the per-rank worker spawned by the tests."""

from __future__ import annotations

import datetime
import os
import sys
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[1]
for p in (str(REPO), str(REPO / "solution-is-all-you-need_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

from oracle import moe_oracle as O  # noqa: E402


class OracleOps:
    """The compute steps of the layer on the CPU oracle (torch CPU tensors in
    and out), standing in for the CUDA kernels in gloo tests."""

    def router(self, x, router_weight, top_k, renormalize):
        _, _, idx, w = O.route_fixed_order(x.numpy(), router_weight.numpy(), top_k, renormalize)
        return torch.from_numpy(idx.astype(np.int32)), torch.from_numpy(w.astype(np.float32))

    def dispatch(self, idx, num_experts):
        counts, offsets, row_token, _, inv = O.dispatch(idx.numpy(), num_experts)
        hit = np.nonzero(counts)[0].astype(np.int32)
        active = np.zeros(num_experts + 1, np.int32)
        active[0] = hit.size
        active[1:1 + hit.size] = hit
        return (torch.from_numpy(offsets), torch.from_numpy(row_token), torch.from_numpy(inv),
                torch.from_numpy(active))

    def gather(self, src, index):
        out = torch.zeros(index.numel(), src.shape[1], dtype=src.dtype)
        ok = (index >= 0) & (index < src.shape[0])
        out[ok] = src[index[ok].long()]
        return out

    def ffn(self, x, row_token, offsets, active, w13_q, w13_scales, w2_q, w2_scales, group_size, path="auto"):
        xs = x.numpy()
        off = offsets.numpy()
        rt = row_token.numpy()
        y = np.zeros((rt.size, xs.shape[1]), np.float32)
        for e in range(w13_q.shape[0]):
            a, b = int(off[e]), int(off[e + 1])
            if a == b:
                continue
            d13 = O.dequantize_int4(w13_q[e].numpy(), w13_scales[e].numpy(), group_size)
            d2 = O.dequantize_int4(w2_q[e].numpy(), w2_scales[e].numpy(), group_size)
            y[a:b] = O.expert_ffn(xs[rt[a:b]], d13, d2)
        return torch.from_numpy(y)

    def combine(self, y, inv, topk_w, out_dtype):
        yn, iv, w = y.numpy(), inv.numpy(), topk_w.numpy()
        out = np.zeros((iv.shape[0], yn.shape[1]), np.float32)
        for j in range(iv.shape[1]):  # slot order, as the combine kernel sums
            out += w[:, j:j + 1] * yn[iv[:, j]]
        return torch.from_numpy(out).to(out_dtype)


# (H, E, k, I, G)
DIMS = (64, 8, 3, 64, 32)


def make_case(case: str, world: int):
    """Seeded tokens per rank, router weight and packed experts."""
    H, E, k, I, G = DIMS
    g = torch.Generator().manual_seed({"ragged": 21, "skew": 22}[case] + world)
    tokens = {2: [7, 4], 4: [5, 0, 3, 6]}[world]
    xs = [torch.randn(t, H, generator=g) for t in tokens]
    wr = torch.randn(E, H, generator=g) * 0.02
    if case == "skew":  # every token prefers the last rank's experts
        xs = [x.abs() for x in xs]
        lo = E - E // world
        wr[:lo] = -0.05
        wr[lo:] = 0.05 + 0.01 * torch.randn(E - lo, H, generator=g).abs()
    w13 = (torch.randn(E, 2 * I, H, generator=g) * 0.02).numpy()
    w2 = (torch.randn(E, H, I, generator=g) * 0.02).numpy()
    p13, s13 = O.quantize_int4(w13, G)
    p2, s2 = O.quantize_int4(w2, G)
    return xs, wr, (torch.from_numpy(p13), torch.from_numpy(s13), torch.from_numpy(p2), torch.from_numpy(s2))


def replica_plan(xs, wr, world: int):
    """The replicated placement every rank derives from the routing of all
    tokens (one extra slot per rank for each home expert)."""
    from phantom_moe import ep
    H, E, k, I, G = DIMS
    idx, _ = OracleOps().router(torch.cat(xs), wr, k, True)
    load = np.bincount(idx.numpy().reshape(-1), minlength=E)
    return ep.plan_replicas(load.tolist(), world, E // world)


def gloo_worker(rank: int, world: int, port: int, case: str, out_dir: str, replicate: bool = False,
                fixed: bool = False):
    import torch.distributed as dist
    from phantom_moe import ep
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        H, E, k, I, G = DIMS
        xs, wr, (p13, s13, p2, s2) = make_case(case, world)
        stats = {}
        if replicate:
            pl = replica_plan(xs, wr, world)
            local = pl.local_weights(rank, p13, s13, p2, s2)
            out, idx, w = ep.moe_layer_ep(xs[rank], wr, *local, k, True, G, None, return_routing=True,
                                          ops=OracleOps(), stats=stats, placement=pl)
        else:
            lo, hi = ep.shard_range(E, world, rank)
            cap = max(x.shape[0] for x in xs) * k if fixed else None  # the same on every rank
            out, idx, w = ep.moe_layer_ep(xs[rank], wr, p13[lo:hi], s13[lo:hi], p2[lo:hi], s2[lo:hi], k, True, G,
                                          None, return_routing=True, ops=OracleOps(), stats=stats,
                                          fixed_capacity=cap)
        np.savez(Path(out_dir) / f"rank{rank}.npz", out=out.numpy(), idx=idx.numpy(), w=w.numpy(),
                 send=np.array(stats["send_rows"]), recv=np.array(stats["recv_rows"]))
    finally:
        dist.destroy_process_group()
