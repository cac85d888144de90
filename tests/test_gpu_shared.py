"""Shared experts on the GPU (phmoe_moe_layer_shared through moe_layer):
Qwen2-MoE's gated shared expert against transformers' block (golden) and
the oracle; DeepSeek-style ungated shared experts with routed scaling; both
FFN paths."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import phantom_moe as pm
from conftest import load_golden
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


def cu(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.to(dtype) if dtype is not None else t


@pytest.mark.parametrize("path", ["decode", "prefill"])
def test_qwen2moe_golden(cuda_device, path):
    z = load_golden("qwen2moe_block_small.npz")
    T, H, E, I, m, _ = (int(v) for v in z["dims"])
    k, g = int(z["top_k"]), int(z["group"])
    dt = torch.bfloat16 if path == "prefill" else torch.float32  # the prefill GEMMs take bf16 activations
    x = cu(z["x"], dt)
    out, idx, w = pm.moe_layer(x, cu(z["wr"], dt), cu(z["w13_q"]), cu(z["w13_s"]), cu(z["w2_q"]), cu(z["w2_s"]),
                               k, renormalize=False, group_size=g, path=path, return_routing=True, num_shared=m,
                               shared_gate_weight=cu(z["shared_gate"], dt))
    xr = x.float().cpu().numpy()
    ref, i_ref, w_ref = O.moe_layer_reference_shared(xr, cu(z["wr"], dt).float().cpu().numpy(), z["w13_q"],
                                                     z["w13_s"], z["w2_q"], z["w2_s"], k, m, g, renormalize=False,
                                                     shared_gate=cu(z["shared_gate"], dt).float().cpu().numpy())
    assert np.array_equal(idx.cpu().numpy(), i_ref)
    mx, mr = O.parity_stats(out.float().cpu().numpy(), ref)
    assert mx <= O.MAX_ABS_TOL and mr <= O.MEAN_REL_TOL, (mx, mr)
    if dt == torch.float32:  # fp32 end to end: also the transformers block itself
        mx, mr = O.parity_stats(out.cpu().numpy(), z["out"])
        assert mx <= 1e-3 and mr <= O.DECODE_FP32_MEAN_REL, (mx, mr)


@pytest.mark.parametrize("T,path,gated,scale", [(3, "decode", True, 1.0), (64, "decode", False, 2.5),
                                                (700, "prefill", True, 1.0), (300, "auto", False, 2.5)])
def test_shared_layer_shapes(cuda_device, T, path, gated, scale):
    """Qwen2-MoE-A2.7B-like shape (H 2048, 60 experts, top-4, I 1408, shared
    5632 = 4 x 1408) and DeepSeek-style ungated shared experts with
    routed_scaling_factor."""
    dev = cuda_device
    H, E, k, I, m, G = 2048, 60, 4, 1408, 4, 64
    gen = torch.Generator(device=dev).manual_seed(T)
    gu = torch.randn(E, 2 * I, H, device=dev, generator=gen) * 0.02
    dn = torch.randn(E, H, I, device=dev, generator=gen) * 0.02
    sg, su = (torch.randn(m * I, H, device=dev, generator=gen) * 0.02 for _ in range(2))
    sd = torch.randn(H, m * I, device=dev, generator=gen) * 0.02
    pk = pm.pack_experts_shared(gu, dn, sg, su, sd, G)
    assert pk.num_shared == m and pk.w13_q.shape[0] == E + m
    wr = (torch.randn(E, H, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
    gate = (torch.randn(H, device=dev, generator=gen) * 0.05).to(torch.bfloat16) if gated else None
    x = torch.randn(T, H, device=dev, generator=gen).to(torch.bfloat16)
    out, idx, w = pm.moe_layer(x, wr, pk.w13_q, pk.w13_scales, pk.w2_q, pk.w2_scales, k, renormalize=True,
                               group_size=G, path=path, return_routing=True, num_shared=m,
                               shared_gate_weight=gate, routed_scale=scale)
    host = [t.cpu().numpy() for t in (pk.w13_q, pk.w13_scales, pk.w2_q, pk.w2_scales)]
    ref, i_ref, _ = O.moe_layer_reference_shared(x.float().cpu().numpy(), wr.float().cpu().numpy(), *host, k, m, G,
                                                 shared_gate=None if gate is None else gate.float().cpu().numpy(),
                                                 routed_scale=scale)
    assert np.array_equal(idx.cpu().numpy(), i_ref)
    mx, mr = O.parity_stats(out.float().cpu().numpy(), ref)
    assert mx <= 0.05 and mr <= O.MEAN_REL_TOL, (mx, mr)  # bf16 output: |out| ~ 10 gives a 0.03 half-ulp
    assert pm.load_library().phmoe_device_error(1) == 0


def test_pack_experts_shared_bytes(cuda_device):
    dev = cuda_device
    E, H, I, m = 4, 256, 128, 2
    gen = torch.Generator(device=dev).manual_seed(9)
    gu, dn = torch.randn(E, 2 * I, H, device=dev, generator=gen), torch.randn(E, H, I, device=dev, generator=gen)
    sg, su, sd = (torch.randn(m * I, H, device=dev, generator=gen), torch.randn(m * I, H, device=dev, generator=gen),
                  torch.randn(H, m * I, device=dev, generator=gen))
    pk = pm.pack_experts_shared(gu, dn, sg, su, sd, 64)
    s13 = np.concatenate([sg.cpu().numpy().reshape(m, I, H), su.cpu().numpy().reshape(m, I, H)], axis=1)
    s2 = sd.cpu().numpy().reshape(H, m, I).transpose(1, 0, 2)
    p13, q13 = O.quantize_int4(np.concatenate([gu.cpu().numpy(), s13]), 64)
    p2, q2 = O.quantize_int4(np.concatenate([dn.cpu().numpy(), s2]), 64)
    assert np.array_equal(pk.w13_q.cpu().numpy(), p13) and np.array_equal(pk.w2_q.cpu().numpy(), p2)
    assert np.array_equal(pk.w13_scales.cpu().numpy(), q13) and np.array_equal(pk.w2_scales.cpu().numpy(), q2)
    with pytest.raises(ValueError):
        pm.pack_experts_shared(gu, dn, sg[:100], su[:100], sd[:, :100], 64)


@pytest.mark.parametrize("E,ng,tg,k,dt", [(256, 8, 4, 8, torch.bfloat16), (16, 4, 2, 4, torch.float32),
                                          (64, 1, 1, 6, torch.bfloat16)])
def test_router_ex_bit_exact(cuda_device, E, ng, tg, k, dt):
    """DeepSeek-V3 routing on the GPU against the oracle's replay: same
    indices in the same order, weights bit-exact (DeepSeek-V3 shape H 7168,
    256 experts in 8 groups, 4 kept, top-8)."""
    dev = cuda_device
    H = 7168 if E == 256 else 512
    gen = torch.Generator(device=dev).manual_seed(E + k)
    x = torch.randn(40, H, device=dev, generator=gen).to(dt)
    wr = (torch.randn(E, H, device=dev, generator=gen) * 0.02).to(dt)
    bias = torch.randn(E, device=dev, generator=gen) * 0.05
    idx, w, logits = pm.router_ex(x, wr, k, True, "sigmoid", bias, ng, tg, 2.5)
    lg, _, i_ref, w_ref = O.route_sigmoid_grouped(x.float().cpu().numpy(), wr.float().cpu().numpy(), k, True,
                                                  bias.cpu().numpy(), ng, tg, 2.5)
    assert np.array_equal(logits.cpu().numpy().view(np.uint32), lg.view(np.uint32))
    assert np.array_equal(idx.cpu().numpy(), i_ref)
    assert np.array_equal(w.cpu().numpy().view(np.uint32), w_ref.view(np.uint32))


def test_router_ex_rejects(cuda_device):
    x = torch.zeros(4, 256, device=cuda_device)
    wr = torch.zeros(12, 256, device=cuda_device)
    for kw in (dict(n_group=5, topk_group=1), dict(n_group=4, topk_group=5), dict(scoring="softmax", n_group=4)):
        args = dict(renormalize=True, scoring="sigmoid", score_bias=None, topk_group=1, routed_scale=1.0)
        args.update(kw)
        with pytest.raises(pm.PhmoeError):
            pm.router_ex(x, wr, 2, **args)


@pytest.mark.parametrize("path", ["decode", "prefill"])
def test_deepseek_layer(cuda_device, path):
    """DeepSeek-style layer: sigmoid routing with bias over 64 experts in 8
    groups (3 kept), top-6, 2 ungated shared experts, routed_scale 2.5."""
    dev = cuda_device
    H, E, k, I, m, G, T = 1024, 64, 6, 256, 2, 64, 200
    gen = torch.Generator(device=dev).manual_seed(21)
    gu = torch.randn(E, 2 * I, H, device=dev, generator=gen) * 0.02
    dn = torch.randn(E, H, I, device=dev, generator=gen) * 0.02
    sg, su = (torch.randn(m * I, H, device=dev, generator=gen) * 0.02 for _ in range(2))
    sd = torch.randn(H, m * I, device=dev, generator=gen) * 0.02
    pk = pm.pack_experts_shared(gu, dn, sg, su, sd, G)
    wr = (torch.randn(E, H, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
    bias = torch.randn(E, device=dev, generator=gen) * 0.05
    x = torch.randn(T, H, device=dev, generator=gen).to(torch.bfloat16)
    out, idx, w = pm.moe_layer(x, wr, pk.w13_q, pk.w13_scales, pk.w2_q, pk.w2_scales, k, group_size=G, path=path,
                               return_routing=True, num_shared=m, routed_scale=2.5, scoring="sigmoid",
                               score_bias=bias, n_group=8, topk_group=3)
    host = [t.cpu().numpy() for t in (pk.w13_q, pk.w13_scales, pk.w2_q, pk.w2_scales)]
    ref, i_ref, w_ref = O.moe_layer_reference_shared(x.float().cpu().numpy(), wr.float().cpu().numpy(), *host, k, m,
                                                     G, routed_scale=2.5, scoring="sigmoid",
                                                     score_bias=bias.cpu().numpy(), n_group=8, topk_group=3)
    assert np.array_equal(idx.cpu().numpy(), i_ref)
    assert np.array_equal(w.cpu().numpy(), w_ref)
    mx, mr = O.parity_stats(out.float().cpu().numpy(), ref)
    assert mx <= 0.05 and mr <= O.MEAN_REL_TOL, (mx, mr)
