"""Expert-parallel layer on the GPU: ranks emulated on one device (the
all-to-alls become concatenations) and, with two or more GPUs, real NCCL
ranks. Both must reproduce the single-GPU layer bit for bit."""

from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch

import phantom_moe as pm
from phantom_moe import ep

H, E, K, I, G = 2048, 128, 8, 768, 64


def _layer(seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    wr = (torch.randn(E, H, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    w13 = torch.randn(E, 2 * I, H, device=dev, generator=g) * 0.02
    p13 = pm.quantize_int4(w13, G)
    del w13
    w2 = torch.randn(E, H, I, device=dev, generator=g) * 0.02
    p2 = pm.quantize_int4(w2, G)
    return wr, (p13[0], p13[1], p2[0], p2[1])


def _shards(packed, world):
    out = []
    for r in range(world):
        lo, hi = ep.shard_range(E, world, r)
        out.append(tuple(t[lo:hi] for t in packed))
    return out


@pytest.mark.gpu
def test_gather_rows_matches_indexing(cuda_device):
    dev = cuda_device
    g = torch.Generator(device=dev).manual_seed(4)
    for dtype, width in ((torch.bfloat16, 2048), (torch.float32, 2048), (torch.bfloat16, 8)):
        src = torch.randn(37, width, device=dev, generator=g).to(dtype)
        index = torch.randint(-3, 40, (101,), device=dev, generator=g, dtype=torch.int32)
        got = pm.gather_rows(src, index)
        ok = (index >= 0) & (index < 37)
        want = torch.zeros_like(got)
        want[ok] = src[index[ok].long()]
        assert torch.equal(got, want)
    assert pm.gather_rows(src, index[:0]).shape == (0, 8)


@pytest.mark.gpu
@pytest.mark.parametrize("world,tokens", [(2, [64, 64]), (4, [5, 0, 17, 64]), (8, [64] * 8)])
def test_ep_emulated_equals_single_gpu(cuda_device, world, tokens):
    dev = cuda_device
    wr, packed = _layer(31, dev)
    g = torch.Generator(device=dev).manual_seed(32 + world)
    xs = [torch.randn(t, H, device=dev, generator=g).to(torch.bfloat16) for t in tokens]
    outs = ep.moe_layer_ep_emulated(xs, wr, _shards(packed, world), K, True, G)
    ref = pm.moe_layer(torch.cat(xs), wr, *packed, K)
    torch.cuda.synchronize()
    assert torch.equal(torch.cat(outs), ref)


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_emulated_replicated_equals_single_gpu(cuda_device, world):
    """Hot experts copied onto other ranks (plan_replicas), ranks emulated on
    one GPU with the CUDA kernels: the same output bit for bit."""
    dev = cuda_device
    wr, packed = _layer(63, dev)
    load = [200.0 / (e + 1) for e in range(E)]  # the low (rank 0) experts hot
    pl = ep.plan_replicas(load, world, 4)
    assert pl.slots_per_rank > E // world
    tokens = [64, 5, 0, 40, 64, 17, 9, 33][:world]
    g = torch.Generator(device=dev).manual_seed(64 + world)
    xs = [torch.randn(t, H, device=dev, generator=g).to(torch.bfloat16) for t in tokens]
    shards = [pl.local_weights(r, *packed) for r in range(world)]
    outs = ep.moe_layer_ep_emulated(xs, wr, shards, K, True, G, path="decode", placement=pl)
    ref = pm.moe_layer(torch.cat(xs), wr, *packed, K, path="decode")
    t0 = 0
    for r, t in enumerate(tokens):
        assert torch.equal(outs[r], ref[t0:t0 + t]), r
        t0 += t


@pytest.mark.gpu
def test_ep_emulated_zipf_skew(cuda_device):
    """BASELINE config 5 shape: 8192 tokens, router logits biased by log of a
    Zipf(1.2) prior (folded into the router weight through a constant input
    feature), 4 emulated ranks."""
    dev = cuda_device
    wr, packed = _layer(41, dev)
    T = 8192
    g = torch.Generator(device=dev).manual_seed(42)
    x = torch.randn(T, H, device=dev, generator=g)
    x[:, 0] = 1.0
    prior = torch.log(torch.arange(1, E + 1, device=dev, dtype=torch.float32) ** -1.2)
    wr = wr.float()
    wr[:, 0] = prior
    x, wr = x.to(torch.bfloat16), wr.to(torch.bfloat16)
    xs = list(x.split(T // 4))
    for path in ("decode", "prefill"):  # each rank runs the same kernels as the single GPU
        outs = ep.moe_layer_ep_emulated(xs, wr, _shards(packed, 4), K, True, G, path=path)
        ref, idx, _ = pm.moe_layer(x, wr, *packed, K, path=path, return_routing=True)
        torch.cuda.synchronize()
        assert torch.equal(torch.cat(outs), ref), path
    load = torch.bincount(idx.view(-1).long(), minlength=E).float()
    assert load.max() / load.mean() > 5.0  # the skew is real


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        wr, packed = _layer(51, dev)
        lo, hi = ep.shard_range(E, world, rank)
        tokens = [64, 3, 0, 40, 64, 1, 17, 9][:world]
        g = torch.Generator(device=dev).manual_seed(52)
        xs = [torch.randn(t, H, device=dev, generator=g).to(torch.bfloat16) for t in tokens]
        stats = {}
        out = ep.moe_layer_ep(xs[rank], wr, *(t[lo:hi] for t in packed), K, True, G, None, stats=stats)
        out2 = ep.moe_layer_ep(xs[rank], wr, *(t[lo:hi] for t in packed), K, True, G, None)
        ref = pm.moe_layer(torch.cat(xs), wr, *packed, K)
        t0 = sum(tokens[:rank])
        torch.cuda.synchronize()
        ok = torch.equal(out, ref[t0:t0 + tokens[rank]]) and torch.equal(out, out2)
        np.save(os.path.join(out_dir, f"ok{rank}.npy"), np.array([ok, sum(stats["recv_rows"])]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_ep_nccl_ranks_equal_single_gpu(cuda_device, tmp_path):
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    torch.multiprocessing.start_processes(_nccl_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                                          join=True, start_method="spawn")
    res = [np.load(tmp_path / f"ok{r}.npy") for r in range(world)]
    assert all(bool(r[0]) for r in res)
    assert sum(int(r[1]) for r in res) == sum([64, 3, 0, 40, 64, 1, 17, 9][:world]) * K


def _peer_worker(rank, world, port, out_dir, case):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    lib = pm.load_library()
    result = {}
    try:
        wr, packed = _layer(61, dev)
        lo, hi = ep.shard_range(E, world, rank)
        shard = tuple(t[lo:hi] for t in packed)
        if case == "layer":
            ok = True
            ex = ep.PeerExchange(None, max_tokens=64, top_k=K, hidden_size=H, num_experts=E)
            tokens = [64, 3, 0, 40, 64, 1, 17, 9][:world]
            t0 = sum(tokens[:rank])
            for it in range(3):  # consecutive calls reuse the exchange buffers
                g = torch.Generator(device=dev).manual_seed(70 + it)
                xs = [torch.randn(t, H, device=dev, generator=g).to(torch.bfloat16) for t in tokens]
                out = ep.moe_layer_ep(xs[rank], wr, *shard, K, True, G, None, path="decode", exchange=ex)
                ref = pm.moe_layer(torch.cat(xs), wr, *packed, K, path="decode")
                torch.cuda.synchronize()
                ok = ok and torch.equal(out, ref[t0:t0 + tokens[rank]])
            ex.close()
            ex2 = ep.PeerExchange(None, max_tokens=1024, top_k=K, hidden_size=H, num_experts=E)
            tokens = [1024, 512, 0, 1000, 1024, 7, 300, 64][:world]
            t0 = sum(tokens[:rank])
            g = torch.Generator(device=dev).manual_seed(80)
            xs = [torch.randn(t, H, device=dev, generator=g).to(torch.bfloat16) for t in tokens]
            out = ep.moe_layer_ep(xs[rank], wr, *shard, K, True, G, None, path="prefill", exchange=ex2)
            ref = pm.moe_layer(torch.cat(xs), wr, *packed, K, path="prefill")
            torch.cuda.synchronize()
            ok = ok and torch.equal(out, ref[t0:t0 + tokens[rank]])
            ex2.close()
            result = {"ok": ok, "err": lib.phmoe_device_error(1)}
        elif case == "replicated":
            # a load that makes rank 0's experts hot, so the planner copies them
            # onto the other ranks; every rank derives the same placement
            load = [100 if e < E // world else 1 for e in range(E)]
            pl = ep.plan_replicas(load, world, E // world)
            local = pl.local_weights(rank, *packed)
            ok = pl.slots_per_rank > E // world and local[0].shape[0] == pl.slots_per_rank
            ex = ep.PeerExchange(None, max_tokens=64, top_k=K, hidden_size=H, num_experts=E, placement=pl)
            tokens = [64, 40, 0, 64, 17, 64, 5, 33][:world]
            t0 = sum(tokens[:rank])
            for it in range(2):  # consecutive calls reuse the exchange buffers
                g = torch.Generator(device=dev).manual_seed(90 + it)
                xs = [torch.randn(t, H, device=dev, generator=g).to(torch.bfloat16) for t in tokens]
                out = ep.moe_layer_ep(xs[rank], wr, *local, K, True, G, None, path="decode", exchange=ex,
                                      placement=pl)
                ref = pm.moe_layer(torch.cat(xs), wr, *packed, K, path="decode")
                torch.cuda.synchronize()
                ok = ok and torch.equal(out, ref[t0:t0 + tokens[rank]])
            ex.close()
            result = {"ok": ok, "err": lib.phmoe_device_error(1)}
        elif case == "graphed":
            # the layer captured in CUDA graphs: its epoch is a device word
            # advanced by every call, so replays keep the ranks in step
            ex = ep.PeerExchange(None, max_tokens=64, top_k=K, hidden_size=H, num_experts=E)
            tokens = [64, 3, 0, 40, 64, 1, 17, 9][:world]
            t0 = sum(tokens[:rank])
            inputs, refs = [], []
            for l in range(3):
                g = torch.Generator(device=dev).manual_seed(100 + l)
                xs = [torch.randn(t, H, device=dev, generator=g).to(torch.bfloat16) for t in tokens]
                inputs.append(xs[rank].clone())
                refs.append(pm.moe_layer(torch.cat(xs), wr, *packed, K, path="decode")[t0:t0 + tokens[rank]])
            s = torch.cuda.Stream(dev)
            graphs, outs = [], []
            with torch.cuda.stream(s):
                for l in range(3):  # eager warm-up, the same number of calls on every rank
                    ep.moe_layer_ep(inputs[l], wr, *shard, K, True, G, None, path="decode", exchange=ex)
                s.synchronize()
                for l in range(3):
                    gr = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(gr, stream=s):
                        outs.append(ep.moe_layer_ep(inputs[l], wr, *shard, K, True, G, None, path="decode",
                                                    exchange=ex))
                    graphs.append(gr)
            torch.cuda.synchronize()
            ok = True
            for l in (0, 1, 2, 2, 0, 1):  # out of order, same order on every rank
                graphs[l].replay()
                torch.cuda.synchronize()
                ok = ok and torch.equal(outs[l], refs[l])
            del graphs
            ex.close()
            result = {"ok": ok, "err": lib.phmoe_device_error(1)}
        else:  # "timeout": rank 1 never calls the layer, so rank 0's flags never arrive
            ex = ep.PeerExchange(None, max_tokens=8, top_k=K, hidden_size=H, num_experts=E)
            if rank == 0:
                x = torch.randn(8, H, device=dev).to(torch.bfloat16)
                ep.moe_layer_ep(x, wr, *shard, K, True, G, None, path="decode", exchange=ex)
                torch.cuda.synchronize()
            result = {"err": lib.phmoe_device_error(1), "alive": int(torch.ones(1, device=dev).sum().item())}
            ex.close()
        np.save(os.path.join(out_dir, f"peer{rank}.npy"), np.array([result.get("ok", True), result["err"],
                                                                     result.get("alive", 1)]))
    finally:
        dist.destroy_process_group()


def _run_peer(case, tmp_path):
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    torch.multiprocessing.start_processes(_peer_worker, args=(world, _free_port(), str(tmp_path), case),
                                          nprocs=world, join=True, start_method="spawn")
    return [np.load(tmp_path / f"peer{r}.npy") for r in range(world)]


@pytest.mark.gpu
def test_ep_peer_exchange_equals_single_gpu(cuda_device, tmp_path):
    """Rows and results moved through peer memory (no collective on the data
    path): three consecutive decode calls with ragged and empty ranks, then a
    prefill call, each equal to the single-GPU layer bit for bit."""
    res = _run_peer("layer", tmp_path)
    assert all(bool(r[0]) for r in res)
    assert all(int(r[1]) == 0 for r in res)


@pytest.mark.gpu
def test_ep_peer_exchange_replicated_placement(cuda_device, tmp_path):
    """Hot experts copied onto other ranks (phmoe_ep_create_ex / _layer_ex):
    every row goes to the copy its source is assigned, and the output still
    equals the single-GPU layer bit for bit."""
    res = _run_peer("replicated", tmp_path)
    assert all(bool(r[0]) for r in res)
    assert all(int(r[1]) == 0 for r in res)


@pytest.mark.gpu
def test_ep_peer_exchange_in_cuda_graph(cuda_device, tmp_path):
    """The peer-exchange layer captured in CUDA graphs (the exchange's epoch
    is a device word every call advances) and replayed out of order: every
    replay equals the single-GPU layer bit for bit."""
    res = _run_peer("graphed", tmp_path)
    assert all(bool(r[0]) for r in res)
    assert all(int(r[1]) == 0 for r in res)


@pytest.mark.gpu
def test_ep_peer_wait_times_out_without_hanging(cuda_device, tmp_path):
    """A rank that never calls the layer: the other rank's bounded flag waits
    run out (2 s each), set device error bit 2 and return; its GPU context
    stays usable."""
    res = _run_peer("timeout", tmp_path)
    assert int(res[0][1]) & 4
    assert int(res[0][2]) == 1
    assert all(int(r[1]) == 0 for r in res[1:])
