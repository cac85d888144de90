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
