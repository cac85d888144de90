"""Pin the CPU oracle against the reference's own outputs (golden fixtures).

The fixtures were produced by tests/golden/make_golden.py from the reference's
``GGUFLoader.dequantize_tensor`` (python/phantom/loader/gguf_loader.py:362-381),
``PhantomTopKRouter`` (tests/test_moe_routing.py:43-72) and transformers'
``Qwen3MoeSparseMoeBlock`` / ``MixtralSparseMoeBlock`` (the path PHANTOM runs).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import moe_oracle as O


def to_bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16).float().numpy()


# ---- int4 / Q4_0 ----------------------------------------------------------

def test_q4_0_known_answer_audit_suite():
    g = load_golden("q4_0_kat.npz")
    # tests/audit_suite.py:36-41: all nibbles 0x8 with d = 1.5 dequantise to 0.
    out = O.dequantize_q4_0(g["kat_raw"].tobytes(), 32)
    assert np.array_equal(out, np.zeros(32, np.float32))
    assert np.array_equal(g["kat_out"], np.zeros(32, np.float32))


def test_q4_0_random_blocks_match_reference_loader():
    g = load_golden("q4_0_kat.npz")
    n = g["out_bf16"].size
    ours = O.dequantize_q4_0(g["raw"].tobytes(), n)
    # the reference returns bf16 (gguf_loader.py:380)
    assert np.array_equal(to_bf16(ours), g["out_bf16"])


def test_q4_0_import_is_lossless_group32():
    g = load_golden("q4_0_kat.npz")
    raw = g["raw"].tobytes()
    rows, K = 4, 512
    packed, scales = O.q4_0_to_packed(raw, rows, K)
    assert packed.shape == (rows, K // 2) and scales.shape == (rows, K // 32)
    ours = O.dequantize_int4(packed, scales, 32).reshape(-1)
    assert np.array_equal(ours, O.dequantize_q4_0(raw, rows * K))


def test_quantizer_roundtrip_bounds():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((8, 256)) * 0.02).astype(np.float32)
    for G in (32, 64):
        p, s = O.quantize_int4(w, G)
        d = O.dequantize_int4(p, s, G)
        step = np.repeat(s.astype(np.float32), G, axis=1)
        assert np.all(np.abs(d - w) <= 0.5 * step + 1e-7 + np.abs(w) * 2e-3)
    z = np.zeros((2, 64), np.float32)
    p, s = O.quantize_int4(z, 64)
    assert np.all(p == 0x88) and np.all(s == 0)


def small_block_dense(g):
    """Dense expert weights of a small-block fixture, regenerated from its seed
    (tests/golden/make_golden.py:small_block_inputs)."""
    T, H, E, I, seed = (int(v) for v in g["dims"])
    gen = torch.Generator().manual_seed(seed)
    torch.randn(T, H, generator=gen)
    torch.randn(E, H, generator=gen)
    w13 = (torch.randn(E, 2 * I, H, generator=gen) * 0.02).numpy()
    w2 = (torch.randn(E, H, I, generator=gen) * 0.02).numpy()
    return w13, w2


def test_quantizer_matches_fixture_bytes():
    for name in ("qwen3_block_small.npz", "qwen3_block_small_g32.npz", "mixtral_block_small.npz"):
        g = load_golden(name)
        w13, w2 = small_block_dense(g)
        G = int(g["group"])
        p13, s13 = O.quantize_int4(w13, G)
        p2, s2 = O.quantize_int4(w2, G)
        assert np.array_equal(p13, g["w13_q"]) and np.array_equal(s13, g["w13_s"])
        assert np.array_equal(p2, g["w2_q"]) and np.array_equal(s2, g["w2_s"])


# ---- exp / router --------------------------------------------------------

def test_fixed_exp_accuracy():
    x = np.linspace(-87.0, 0.0, 200001, dtype=np.float32)
    ours = O.fixed_exp(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    ulp = np.spacing(ref.astype(np.float32)).astype(np.float64)
    assert np.max(np.abs(ours - ref) / ulp) <= 2.0
    assert O.fixed_exp(np.array([-100.0], np.float32))[0] == 0.0
    assert O.fixed_exp(np.array([0.0], np.float32))[0] == 1.0


def test_phantom_topk_router_golden():
    g = load_golden("router_phantom.npz")
    x = g["x"].reshape(-1, g["x"].shape[-1])
    for route in (O.route_reference, O.route_fixed_order):
        _, _, idx, w = route(x, g["gate"], 2, True)
        assert np.array_equal(idx, g["indices"].reshape(-1, 2))
        np.testing.assert_allclose(w, g["weights"].reshape(-1, 2), rtol=0, atol=2e-6)
    # tests/test_moe_routing.py:149-158 invariants
    assert np.allclose(w.sum(-1), 1.0, atol=1e-5)


@pytest.mark.parametrize("name,kind", [("qwen3_block_small.npz", "qwen3"),
                                       ("qwen3_block_small_g32.npz", "qwen3"),
                                       ("mixtral_block_small.npz", "mixtral")])
def test_block_golden(name, kind):
    g = load_golden(name)
    G, k = int(g["group"]), int(g["top_k"])
    d13 = O.dequantize_int4(g["w13_q"], g["w13_s"], G)
    d2 = O.dequantize_int4(g["w2_q"], g["w2_s"], G)
    for router in ("reference", "fixed"):
        out, idx, w = O.moe_layer_reference(g["x"], g["wr"], d13, d2, k, True, router=router)
        assert np.array_equal(idx, g["idx"])
        np.testing.assert_allclose(w, g["scores"], rtol=0, atol=2e-6)
        np.testing.assert_allclose(out, g["out"], rtol=0, atol=2e-5)
        mx, mr = O.parity_stats(out, g["out"])
        assert mx < 1e-4 and mr < 1e-5
    _, probs, _, _ = O.route_fixed_order(g["x"], g["wr"], k)
    np.testing.assert_allclose(probs, g["probs"], rtol=0, atol=2e-6)


def _cfg1_inputs():
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(16, 2048, generator=gen)
    wr = torch.randn(128, 2048, generator=gen) * 0.02
    return x.numpy(), wr.numpy()


def test_cfg1_router_golden():
    """BASELINE config 1 (Qwen3-30B-A3B-shaped, fp32, seed 0): the fixed-order
    router picks exactly transformers' experts."""
    import hashlib
    g = load_golden("qwen3_cfg1.npz")
    x, wr = _cfg1_inputs()
    assert hashlib.sha256(x.tobytes()).hexdigest() == str(g["sha_x"])
    assert hashlib.sha256(wr.tobytes()).hexdigest() == str(g["sha_wr"])
    _, probs, idx, w = O.route_fixed_order(x, wr, 8)
    assert np.array_equal(idx, g["idx"])
    np.testing.assert_allclose(w, g["scores"], rtol=0, atol=2e-6)
    np.testing.assert_allclose(probs, g["probs"], rtol=0, atol=1e-6)
    assert O.topk_margin(probs, 8).min() > 1e-6


# ---- dispatch ------------------------------------------------------------

def test_dispatch_oracle_invariants():
    rng = np.random.default_rng(3)
    T, E, k = 37, 16, 4
    idx = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    counts, offsets, row_token, row_slot, inv = O.dispatch(idx, E)
    assert counts.sum() == T * k and offsets[-1] == T * k
    for e in range(E):
        rows = np.arange(offsets[e], offsets[e + 1])
        toks = row_token[rows]
        assert np.all(np.diff(toks) > 0)  # ordered by token
        assert np.all(idx[toks, row_slot[rows]] == e)
    for t in range(T):
        for j in range(k):
            r = inv[t, j]
            assert row_token[r] == t and row_slot[r] == j


def test_torch_reference_nibble_order():
    """The GPU-side fp32 reference helpers read the same packed layout."""
    from torch_ref import dequant_torch
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((6, 256)) * 0.02).astype(np.float32)
    for G in (32, 64):
        p, s = O.quantize_int4(w, G)
        got = dequant_torch(torch.from_numpy(p), torch.from_numpy(s), G).numpy()
        assert np.array_equal(got, O.dequantize_int4(p, s, G))


def test_qwen2moe_shared_expert_golden():
    """transformers' Qwen2MoeSparseMoeBlock (routed + sigmoid-gated shared
    expert, norm_topk_prob False) against the oracle's shared-expert form on
    the same packed weights (shared expert as 4 slices after the routed
    experts)."""
    z = load_golden("qwen2moe_block_small.npz")
    T, H, E, I, m, _ = (int(v) for v in z["dims"])
    out, idx, w = O.moe_layer_reference_shared(z["x"], z["wr"], z["w13_q"], z["w13_s"], z["w2_q"], z["w2_s"],
                                               int(z["top_k"]), m, int(z["group"]), renormalize=False,
                                               shared_gate=z["shared_gate"])
    assert np.array_equal(np.sort(idx, 1), np.sort(z["idx"], 1))
    mx, mr = O.parity_stats(out, z["out"])
    assert mx <= 1e-5 and mr <= 1e-5, (mx, mr)


def test_deepseek_routing_golden():
    """transformers' DeepseekV3MoE.route_tokens_to_experts (sigmoid, score
    bias, 4 groups of 4 experts with 2 kept, top-4, renormalised, x2.5) on
    the same logits: same expert sets, weights within 1e-6."""
    z = load_golden("deepseek_route.npz")
    E, ng, tg, k = (int(v) for v in z["cfg"])
    _, _, idx, w = O.route_sigmoid_grouped(None, None, k, True, z["bias"], ng, tg, float(z["scale"]),
                                           logits=z["logits"])
    o1, o2 = np.argsort(idx, 1), np.argsort(z["idx"], 1)
    assert np.array_equal(np.take_along_axis(idx, o1, 1), np.take_along_axis(z["idx"], o2, 1))
    assert np.abs(np.take_along_axis(w, o1, 1) - np.take_along_axis(z["w"], o2, 1)).max() <= 1e-6
