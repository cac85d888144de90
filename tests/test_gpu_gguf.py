"""GGUF importers on the GPU (through the C ABI) against the oracle, and a
GGUF file through the whole MoE layer."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import phantom_moe as pm
from oracle import moe_oracle as O
from phantom_moe import gguf as G
from tests.gguf_writer import random_q4_0, random_q4_k, write_gguf

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("rows,K", [(1, 32), (7, 96), (64, 2048), (3, 14336)])
def test_q4_0_import_bit_exact(cuda_device, rows, K):
    raw = random_q4_0(np.random.default_rng(rows * K), rows, K)
    p, s = G.q4_0_to_packed(np.frombuffer(raw, dtype=np.uint8), rows, K, cuda_device)
    rp, rs = O.q4_0_to_packed(raw, rows, K)
    assert np.array_equal(p.cpu().numpy(), rp)
    assert np.array_equal(s.cpu().numpy().view(np.uint16), rs.view(np.uint16))


def test_q4_k_dequantise_matches_reference(cuda_device):
    z = np.load(GOLDEN / "q4_k_ref.npz")
    out = G.q4_k_dequantize(z["raw"], z["out_f32"].size, cuda_device)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), z["out_f32"].view(np.uint32))


@pytest.mark.parametrize("rows,K,g", [(5, 256, 32), (5, 256, 64), (33, 2048, 32), (2, 4096, 64)])
def test_q4_k_import_bit_exact(cuda_device, rows, K, g):
    raw = random_q4_k(np.random.default_rng(rows + K + g), rows, K)
    p, s = G.q4_k_to_packed(np.frombuffer(raw, dtype=np.uint8), rows, K, g, cuda_device)
    rp, rs = O.q4_k_to_packed(raw, rows, K, g)
    assert np.array_equal(p.cpu().numpy(), rp)
    assert np.array_equal(s.cpu().numpy().view(np.uint16), rs.view(np.uint16))


def test_importer_rejects_bad_sizes(cuda_device):
    with pytest.raises(ValueError):
        G.q4_0_to_packed(np.zeros(17, dtype=np.uint8), 1, 32, cuda_device)
    with pytest.raises(pm.PhmoeError):
        pm.load_library()  # loaded
        from phantom_moe import _lib
        _lib.call("phmoe_gguf_q4_k_to_packed", None, 1, 100, 32, None, None, None)


@pytest.mark.parametrize("qtype", [2, 12])
def test_gguf_layer_end_to_end(cuda_device, tmp_path, qtype):
    """A llama.cpp-layout MoE block (router F32, experts Q4_0 or Q4_K) read
    from a GGUF file, imported on the GPU and run through moe_layer, against
    the oracle on the imported weights; for Q4_0 the imported weights equal
    the file's values exactly."""
    rng = np.random.default_rng(77 + qtype)
    E, H, I, k, T = 8, 512, 256, 2, 24
    # weights of a realistic size (|w| up to ~0.1): Q4_0 d ~ 0.01, Q4_K d, dmin ~ 1e-4 (6-bit scales up to 63)
    mk = (lambda r, a, b: random_q4_0(r, a, b, 0.01)) if qtype == 2 else (lambda r, a, b: random_q4_k(r, a, b, 1e-4))
    gate, up, down = mk(rng, E * I, H), mk(rng, E * I, H), mk(rng, E * H, I)
    router = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    path = tmp_path / "moe.gguf"
    write_gguf(path, {"general.architecture": "qwen3moe", "qwen3moe.expert_count": E,
                      "qwen3moe.expert_used_count": k, "qwen3moe.embedding_length": H,
                      "qwen3moe.expert_feed_forward_length": I, "qwen3moe.block_count": 1},
               [("blk.0.ffn_gate_inp.weight", (H, E), 0, router.tobytes()),
                ("blk.0.ffn_gate_exps.weight", (H, I, E), qtype, gate),
                ("blk.0.ffn_up_exps.weight", (H, I, E), qtype, up),
                ("blk.0.ffn_down_exps.weight", (I, H, E), qtype, down)])
    with pm.GGUFFile(path) as gf:
        spec = pm.detect_moe(gf)
        L = pm.load_moe_layer(gf, 0, cuda_device, router_dtype=torch.float32)
    assert (spec.num_experts, spec.top_k) == (E, k) and L["group_size"] == 32
    if qtype == 2:  # lossless: the packed weights dequantise to the file's values
        w_gate = O.dequantize_q4_0(gate, E * I * H).reshape(E, I, H)
        got = O.dequantize_int4(L["w13_q"].cpu().numpy(), L["w13_scales"].cpu().numpy(), 32)
        assert np.array_equal(got[:, :I], w_gate)
    x = torch.randn(T, H, device=cuda_device, generator=torch.Generator(device=cuda_device).manual_seed(5))
    out, idx, w = pm.moe_layer(x, L["router_weight"], L["w13_q"], L["w13_scales"], L["w2_q"], L["w2_scales"], k,
                               group_size=32, return_routing=True)
    host = [L[n].cpu().numpy() for n in ("w13_q", "w13_scales", "w2_q", "w2_scales")]
    ref, i_ref, _ = O.moe_layer_reference_packed(x.cpu().numpy(), router, *host, k, 32)
    assert np.array_equal(idx.cpu().numpy(), i_ref)
    mx, mr = O.parity_stats(out.cpu().numpy(), ref)
    assert mx <= O.MAX_ABS_TOL and mr <= O.MEAN_REL_TOL, (mx, mr)
