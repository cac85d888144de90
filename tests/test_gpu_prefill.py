"""Prefill FFN (tcgen05 grouped GEMMs) through the C ABI.

* against an fp32 emulation of exactly what the kernels compute (weights
  rounded once to fp16, SwiGLU output rounded to fp16): catches any layout,
  descriptor or tiling error, which would show as O(1) differences;
* the whole layer against the fp32 reference on the exact dequantised
  weights, within the north-star tolerance (max-abs 2e-2, mean-rel 5e-3),
  at the small fixtures, Qwen3 shapes and BASELINE config 3 (Mixtral).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import phantom_moe as pm
from conftest import load_golden
from oracle import moe_oracle as O
from torch_ref import ffn_rows_torch, layer_torch

torch.backends.cuda.matmul.allow_tf32 = False


def _packed_layer(E, H, I, G, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    wr = (torch.randn(E, H, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    w13 = torch.randn(E, 2 * I, H, device=dev, generator=g) * 0.02
    p13 = pm.quantize_int4(w13, G)
    del w13
    w2 = torch.randn(E, H, I, device=dev, generator=g) * 0.02
    p2 = pm.quantize_int4(w2, G)
    return wr, (p13[0], p13[1], p2[0], p2[1])


def _rel(a, b):
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.mark.gpu
@pytest.mark.parametrize("T,H,E,k,I,G", [(300, 512, 8, 2, 256, 64), (97, 256, 16, 4, 128, 32),
                                         (1, 256, 4, 1, 128, 64), (640, 1024, 4, 2, 384, 64)])
def test_prefill_ffn_matches_f16_emulation(cuda_device, T, H, E, k, I, G):
    dev = cuda_device
    wr, packed = _packed_layer(E, H, I, G, 7 + T, dev)
    x = torch.randn(T, H, device=dev, generator=torch.Generator(device=dev).manual_seed(T)).to(torch.bfloat16)
    idx, w, _ = pm.router(x, wr, k)
    offsets, row_token, inv, active = pm.dispatch(idx, E)
    y = pm.expert_ffn_prefill(x, row_token, offsets, active, *packed, k, G)
    ref = ffn_rows_torch(x, row_token, offsets, *packed, G, operand_dtype=torch.float16)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()
    assert _rel(y, ref) < 1e-4, _rel(y, ref)
    exact = ffn_rows_torch(x, row_token, offsets, *packed, G)
    mx, mr = O.parity_stats(y.cpu().numpy(), exact.cpu().numpy())
    assert mx <= O.MAX_ABS_TOL and mr <= O.MEAN_REL_TOL, (mx, mr)


@pytest.mark.gpu
def test_prefill_tile_boundaries(cuda_device):
    """Experts with 1, 128, 129, 255, 256, 257 and 513 rows (k = 1): partial
    halves, full tiles and a tile that starts one row before the end."""
    dev = cuda_device
    E, H, I, G = 8, 256, 128, 64
    _, packed = _packed_layer(E, H, I, G, 99, dev)
    sizes = [1, 128, 129, 255, 256, 257, 0, 513]
    ids = torch.cat([torch.full((n,), e, dtype=torch.int32) for e, n in enumerate(sizes)])
    ids = ids[torch.randperm(ids.numel(), generator=torch.Generator().manual_seed(3))]
    T = ids.numel()
    idx = ids.view(T, 1).to(dev)
    x = torch.randn(T, H, device=dev).to(torch.bfloat16)
    offsets, row_token, inv, active = pm.dispatch(idx, E)
    y = pm.expert_ffn_prefill(x, row_token, offsets, active, *packed, 1, G)
    ref = ffn_rows_torch(x, row_token, offsets, *packed, G, operand_dtype=torch.float16)
    torch.cuda.synchronize()
    assert _rel(y, ref) < 1e-4
    per_row = (y - ref).norm(dim=1) / ref.norm(dim=1).clamp_min(1e-6)
    assert float(per_row.max()) < 1e-3  # no row left unwritten or misplaced


@pytest.mark.gpu
def test_prefill_rejects_unsupported_shapes(cuda_device):
    """The G=32 fixture has I = 64, below the gate/up column tile (128 = 128
    gate + 128 up rows per tile): an explicit prefill request is refused and
    auto falls back to the decode kernels."""
    g = load_golden("qwen3_block_small_g32.npz")
    args = [torch.from_numpy(np.ascontiguousarray(g[n])).to(cuda_device) for n in ("w13_q", "w13_s", "w2_q", "w2_s")]
    xb = torch.from_numpy(g["x"]).to(torch.bfloat16).to(cuda_device)
    wr = torch.from_numpy(g["wr"]).to(cuda_device)
    with pytest.raises(pm.PhmoeError, match="prefill needs I"):
        pm.moe_layer(xb, wr, *args, int(g["top_k"]), group_size=int(g["group"]), path="prefill")
    pm.moe_layer(xb, wr, *args, int(g["top_k"]), group_size=int(g["group"]), path="auto")


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["qwen3_block_small.npz", "mixtral_block_small.npz"])
def test_prefill_layer_small_fixtures(cuda_device, name):
    dev = cuda_device
    g = load_golden(name)
    G, k = int(g["group"]), int(g["top_k"])
    xb = torch.from_numpy(g["x"]).to(torch.bfloat16)
    x_np = xb.float().numpy()
    ref, ref_idx, _ = O.moe_layer_reference_packed(x_np, g["wr"], g["w13_q"], g["w13_s"], g["w2_q"], g["w2_s"], k, G)
    args = [torch.from_numpy(np.ascontiguousarray(g[n])).to(dev) for n in ("w13_q", "w13_s", "w2_q", "w2_s")]
    out, idx, _ = pm.moe_layer(xb.to(dev), torch.from_numpy(g["wr"]).to(dev), *args, k, group_size=G,
                               path="prefill", return_routing=True)
    torch.cuda.synchronize()
    assert np.array_equal(idx.cpu().numpy(), ref_idx)
    mx, mr = O.parity_stats(out.float().cpu().numpy(), ref)
    assert mx <= O.MAX_ABS_TOL and mr <= O.MEAN_REL_TOL, (mx, mr)


def _layer_vs_torch(dev, E, H, k, I, G, T, seed, path):
    """The layer's computation in fp32 (the stages, combined to fp32) against
    the fp32 reference; and the layer's bf16 output against that fp32 result
    rounded once to bf16. (A bf16 output alone cannot meet a 2e-2 max-abs
    bound once |out| >= 8, where bf16's half-ulp is 0.031.)"""
    wr, packed = _packed_layer(E, H, I, G, seed, dev)
    x = torch.randn(T, H, device=dev, generator=torch.Generator(device=dev).manual_seed(seed + 1)).to(torch.bfloat16)
    out, idx, w = pm.moe_layer(x, wr, *packed, k, group_size=G, path=path, return_routing=True)
    offsets, row_token, inv, active = pm.dispatch(idx, E)
    R = T * k
    use_prefill = path == "prefill" or (path == "auto" and R >= 64 * E)
    ffn = pm.expert_ffn_prefill if use_prefill else pm.expert_ffn_decode
    y = ffn(x, row_token, offsets, active, *packed, k, G)
    out32 = pm.combine(y, inv, w, torch.float32)
    ref = layer_torch(x, idx, w, offsets, row_token, inv, packed, G)
    torch.cuda.synchronize()
    assert torch.equal(out, out32.to(torch.bfloat16))
    mx, mr = O.parity_stats(out32.cpu().numpy(), ref.cpu().numpy())
    return mx, mr, out


@pytest.mark.gpu
def test_prefill_mixtral_config3(cuda_device):
    """H 4096, 8 experts, top-2, I 14336, T 4096, bf16,
    seed 2 - the prefill path against fp32 on the exact dequantised weights."""
    mx, mr, _ = _layer_vs_torch(cuda_device, 8, 4096, 2, 14336, 64, 4096, 2, "prefill")
    assert mx <= O.MAX_ABS_TOL and mr <= O.MEAN_REL_TOL, (mx, mr)
    assert pm.load_library().phmoe_device_error(1) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("T", [256, 1024])
def test_prefill_qwen3_and_auto_path(cuda_device, T):
    mx, mr, out = _layer_vs_torch(cuda_device, 128, 2048, 8, 768, 64, T, 11, "prefill")
    assert mx <= O.MAX_ABS_TOL and mr <= O.MEAN_REL_TOL, (mx, mr)
    mx2, mr2, out_auto = _layer_vs_torch(cuda_device, 128, 2048, 8, 768, 64, T, 11, "auto")
    assert mx2 <= O.MAX_ABS_TOL and mr2 <= O.MEAN_REL_TOL
    if T * 8 >= 64 * 128:  # auto takes the prefill GEMMs from 64 rows per expert
        assert torch.equal(out_auto, out)


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1024, 700])
def test_decode_many_rows_per_expert(cuda_device, T):
    """Decode path at 40-64 rows per expert: 5-8 passes of 8 tokens per row
    tile of every expert, ragged last passes included."""
    mx, mr, _ = _layer_vs_torch(cuda_device, 128, 2048, 8, 768, 64, T, 13, "decode")
    assert mx <= O.MAX_ABS_TOL and mr <= O.MEAN_REL_TOL, (mx, mr)
    assert pm.load_library().phmoe_device_error(1) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("T,I", [(5, 768), (64, 512), (64, 768)])
def test_decode_group32(cuda_device, T, I):
    """Decode path with 32-element scale groups at Qwen3's hidden size: the
    down projection's 256-element K tasks hold 8 groups, and I = 768 takes
    three tasks per item."""
    mx, mr, _ = _layer_vs_torch(cuda_device, 32, 2048, 4, I, 32, T, 21, "decode")
    assert mx <= O.MAX_ABS_TOL and mr <= O.MEAN_REL_TOL, (mx, mr)


@pytest.mark.gpu
def test_decode_many_rows_fp32_activations(cuda_device):
    """fp32 activations at 32 rows per expert (four passes per row tile)."""
    dev = cuda_device
    E, H, k, I, G, T = 128, 2048, 8, 768, 64, 512
    wr, packed = _packed_layer(E, H, I, G, 17, dev)
    wr = wr.float()
    x = torch.randn(T, H, device=dev, generator=torch.Generator(device=dev).manual_seed(18))
    out, idx, w = pm.moe_layer(x, wr, *packed, k, group_size=G, path="decode", return_routing=True)
    offsets, row_token, inv, _ = pm.dispatch(idx, E)
    ref = layer_torch(x, idx, w, offsets, row_token, inv, packed, G)
    torch.cuda.synchronize()
    mx, mr = O.parity_stats(out.cpu().numpy(), ref.cpu().numpy())
    assert mx <= 1e-3 and mr <= O.DECODE_FP32_MEAN_REL, (mx, mr)  # fp32 in, fp32 out: 14-bit operands


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_decode_batch_invariance(cuda_device, dtype):
    """A token's decode-path output does not depend on the batch around it:
    the first 8 tokens of a 1024-token batch (64 rows per expert: eight passes
    per row tile, block router) give bit-identical rows when run alone (one
    pass, per-token router)."""
    dev = cuda_device
    E, H, k, I, G, T = 128, 2048, 8, 768, 64, 1024
    wr, packed = _packed_layer(E, H, I, G, 23, dev)
    x = torch.randn(T, H, device=dev, generator=torch.Generator(device=dev).manual_seed(24)).to(dtype)
    wr = wr.to(dtype)
    big, idx_big, _ = pm.moe_layer(x, wr, *packed, k, group_size=G, path="decode", return_routing=True)
    for n in (1, 8, 37):
        small, idx_small, _ = pm.moe_layer(x[:n], wr, *packed, k, group_size=G, path="decode",
                                           return_routing=True)
        torch.cuda.synchronize()
        assert torch.equal(idx_small, idx_big[:n]), n
        assert torch.equal(small, big[:n]), n
    assert pm.load_library().phmoe_device_error(1) == 0


@pytest.mark.gpu
def test_decode_batch_invariance_few_experts(cuda_device):
    """16 experts with ~32 rows each (the local shape of 8-way expert
    parallelism): rows are bit-identical to the same tokens run alone."""
    dev = cuda_device
    E, H, k, I, G, T = 16, 2048, 2, 768, 64, 256
    wr, packed = _packed_layer(E, H, I, G, 29, dev)
    x = torch.randn(T, H, device=dev, generator=torch.Generator(device=dev).manual_seed(30)).to(torch.bfloat16)
    big = pm.moe_layer(x, wr, *packed, k, group_size=G, path="decode")
    for n in (1, 5):
        small = pm.moe_layer(x[:n], wr, *packed, k, group_size=G, path="decode")
        torch.cuda.synchronize()
        assert torch.equal(small, big[:n]), n
    mx, mr, _ = _layer_vs_torch(dev, E, H, k, I, G, T, 31, "decode")
    assert mx <= O.MAX_ABS_TOL and mr <= O.MEAN_REL_TOL, (mx, mr)


def _row_scaled_parity(got, ref):
    """parity_stats with every row divided by its own largest |reference|:
    rows of very different magnitude are each held to the contract."""
    s = np.maximum(np.abs(ref).max(axis=1, keepdims=True), 1e-30)
    return O.parity_stats(got / s, ref / s)


def _large_layer(dev, E=32, H=1024, I=512, G=64, seed=11):
    gen = torch.Generator(device=dev).manual_seed(seed)
    wr = (torch.randn(E, H, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
    pk = pm.pack_experts(torch.randn(E, 2 * I, H, device=dev, generator=gen) * 0.02,
                         torch.randn(E, H, I, device=dev, generator=gen) * 0.02, G)
    return wr, pk, gen


def _prefill_vs_oracle(x, wr, pk, k, G):
    out, idx, _ = pm.moe_layer(x, wr, pk.w13_q, pk.w13_scales, pk.w2_q, pk.w2_scales, k, group_size=G,
                               path="prefill", return_routing=True, check_errors=True)
    host = [t.cpu().numpy() for t in (pk.w13_q, pk.w13_scales, pk.w2_q, pk.w2_scales)]
    ref, i_ref, _ = O.moe_layer_reference_packed(x.float().cpu().numpy(), wr.float().cpu().numpy(), *host, k, G)
    assert np.array_equal(idx.cpu().numpy(), i_ref)
    got = out.float().cpu().numpy()
    assert np.all(np.isfinite(got))
    return got, ref


@pytest.mark.gpu
@pytest.mark.parametrize("scale", [1e3, 1e5, 1e6])
def test_prefill_layer_activations_beyond_fp16(cuda_device, scale):
    """At 1e3 the activations fit fp16 but the SwiGLU output (~1e5) does not;
    at 1e5-1e6 both are beyond it (h ~1e9-1e11). Rows of x and 128-column
    blocks of h take power-of-two exponents, so the prefill layer matches the
    fp32 oracle within the contract tolerance taken relative to each row's
    scale, and no device error bit is raised."""
    dev = cuda_device
    T, k, G = 300, 4, 64
    wr, pk, gen = _large_layer(dev, G=G)
    x = (torch.randn(T, 1024, device=dev, generator=gen) * scale).to(torch.bfloat16)
    got, ref = _prefill_vs_oracle(x, wr, pk, k, G)
    mx, mr = _row_scaled_parity(got, ref)
    assert mx <= O.MAX_ABS_TOL and mr <= O.MEAN_REL_TOL, (mx, mr)


@pytest.mark.gpu
@pytest.mark.parametrize("G", [32, 64])
def test_prefill_outlier_rows_and_features(cuda_device, G):
    """A batch of ordinary rows with outliers mixed in: 8 rows scaled by 1e5,
    8 by 2e3 (h alone beyond fp16), and 6 rows with one feature at 3e5 (a
    "massive activation"). Within a row the h blocks then need different
    exponents, which the fixup pass brings to the row's largest. Ordinary rows
    give bit-identical output to the same rows run without the outliers."""
    dev = cuda_device
    T, k = 257, 4
    wr, pk, gen = _large_layer(dev, G=G, seed=5)
    base = torch.randn(T, 1024, device=dev, generator=gen)
    x = base.clone()
    x[3:11] *= 1e5
    x[40:48] *= 2e3
    x[100:106, 17] = 3e5
    x = x.to(torch.bfloat16)
    got, ref = _prefill_vs_oracle(x, wr, pk, k, G)
    mx, mr = _row_scaled_parity(got, ref)
    assert mx <= O.MAX_ABS_TOL and mr <= O.MEAN_REL_TOL, (mx, mr)
    plain = pm.moe_layer(base.to(torch.bfloat16), wr, pk.w13_q, pk.w13_scales, pk.w2_q, pk.w2_scales, k,
                         group_size=G, path="prefill", check_errors=True).float().cpu().numpy()
    keep = np.ones(T, dtype=bool)
    keep[3:11] = keep[40:48] = keep[100:106] = False
    # routing of a row depends only on that row; the FFN rows of other tokens
    # share tiles but not accumulators
    assert np.array_equal(got[keep], plain[keep])
