"""GGUF import on the CPU: the oracle's Q4_0/Q4_K restatements against the
reference's own dequantiser (golden fixtures), the GGUF reader, and MoE
metadata detection (gguf_loader.py:252-301, format_detect.py:98-127)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import moe_oracle as O
from phantom_moe import gguf as G
from tests.gguf_writer import random_q4_0, random_q4_k, write_gguf

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_q4_k_oracle_matches_reference_dequantiser():
    """dequantize_tensor_cuda (gguf_loader.py:648-666, the loader's path) in
    fp32, on 48 random super-blocks: bit-exact."""
    z = np.load(GOLDEN / "q4_k_ref.npz")
    out = O.dequantize_q4_k(z["raw"].tobytes(), z["out_f32"].size)
    assert np.array_equal(out.view(np.uint32), z["out_f32"].view(np.uint32))
    if "ggml" in z:  # llama.cpp's own Python dequantiser agrees with the loader's path
        assert np.array_equal(z["ggml"], z["out_f32"])
    # the reference's CPU branch (gguf_loader.py:453-489) orders nibbles differently
    assert not np.allclose(z["out_cpu_branch_bf16"], z["out_f32"], atol=1e-2)


def test_q4_0_oracle_matches_reference_cuda_dequantiser():
    z = np.load(GOLDEN / "q4_k_ref.npz")
    out = O.dequantize_q4_0(z["q4_0_raw"].tobytes(), z["q4_0_out_f32"].size)
    assert np.array_equal(out, z["q4_0_out_f32"])


def test_q4_0_packed_is_lossless():
    rng = np.random.default_rng(3)
    raw = random_q4_0(rng, 6, 256)
    packed, scales = O.q4_0_to_packed(raw, 6, 256)
    assert np.array_equal(O.dequantize_int4(packed, scales, 32), O.dequantize_q4_0(raw, 6 * 256).reshape(6, 256))


def test_q4_k_requantised_error_bound():
    rng = np.random.default_rng(4)
    raw = random_q4_k(rng, 4, 512)
    w = O.dequantize_q4_k(raw, 4 * 512).reshape(4, 512)
    for g in (32, 64):
        packed, scales = O.q4_k_to_packed(raw, 4, 512, g)
        back = O.dequantize_int4(packed, scales, g)
        step = np.repeat(scales.astype(np.float32), g, axis=1)
        assert np.all(np.abs(back - w) <= 0.5 * step * (1 + 1e-3) + 1e-7)


def test_reader_roundtrip(tmp_path):
    rng = np.random.default_rng(5)
    E, H, I = 4, 256, 256
    gate, up, down = random_q4_0(rng, E * I, H), random_q4_k(rng, E * I, H), random_q4_0(rng, E * H, I)
    router = rng.standard_normal((E, H)).astype(np.float32)
    meta = {"general.architecture": "qwen3moe", "qwen3moe.expert_count": E, "qwen3moe.expert_used_count": 2,
            "qwen3moe.embedding_length": H, "qwen3moe.expert_feed_forward_length": I,
            "qwen3moe.block_count": 1, "general.name": "tiny", "some.list": [1, 2, 3], "some.float": 0.5}
    path = tmp_path / "m.gguf"
    write_gguf(path, meta, [("blk.0.ffn_gate_inp.weight", (H, E), 0, router.tobytes()),
                            ("blk.0.ffn_gate_exps.weight", (H, I, E), 2, gate),
                            ("blk.0.ffn_up_exps.weight", (H, I, E), 12, up),
                            ("blk.0.ffn_down_exps.weight", (I, H, E), 2, down)])
    with G.GGUFFile(path) as gf:
        assert gf.metadata["general.name"] == "tiny" and gf.metadata["some.list"] == [1, 2, 3]
        assert gf.metadata["some.float"] == 0.5
        t = gf.tensors["blk.0.ffn_gate_exps.weight"]
        assert t.shape == (E, I, H) and t.type_name == "Q4_0" and t.n_bytes == len(gate)
        assert gf.tensor_bytes("blk.0.ffn_up_exps.weight").tobytes() == up
        assert gf.tensor_bytes("blk.0.ffn_down_exps.weight").tobytes() == down
        assert np.array_equal(gf.tensor_bytes("blk.0.ffn_gate_inp.weight").view(np.float32).reshape(E, H), router)
        spec = G.detect_moe(gf)
    assert spec == G.MoeSpec("qwen3moe", E, 2, H, I, 1)
    assert G.detect_moe(str(path)).num_experts == E


def test_reader_matches_gguf_package(tmp_path):
    """Cross-check the reader with llama.cpp's gguf package writer."""
    gguf = pytest.importorskip("gguf")
    rng = np.random.default_rng(6)
    path = tmp_path / "p.gguf"
    w = gguf.GGUFWriter(str(path), "llama")  # llama.cpp writes Mixtral as llama with experts
    w.add_uint32("llama.expert_count", 8)
    w.add_uint32("llama.expert_used_count", 2)
    w.add_uint32("llama.embedding_length", 4096)
    w.add_uint32("llama.feed_forward_length", 14336)
    raw = np.frombuffer(random_q4_0(rng, 2, 64), dtype=np.uint8)
    w.add_tensor("t", raw.reshape(2, 36), raw_dtype=gguf.GGMLQuantizationType.Q4_0)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with G.GGUFFile(path) as gf:
        assert gf.tensors["t"].shape == (2, 64) and gf.tensor_bytes("t").tobytes() == raw.tobytes()
        spec = G.detect_moe(gf)
    assert spec.family == "mixtral" and (spec.num_experts, spec.top_k, spec.intermediate_size) == (8, 2, 14336)


def test_detect_moe_from_transformers_configs():
    tf = pytest.importorskip("transformers")
    q3 = G.detect_moe(tf.Qwen3MoeConfig(hidden_size=2048, num_experts=128, num_experts_per_tok=8,
                                        moe_intermediate_size=768, norm_topk_prob=True))
    assert (q3.family, q3.num_experts, q3.top_k, q3.intermediate_size, q3.norm_topk_prob) == \
        ("qwen3_moe", 128, 8, 768, True)
    mx = G.detect_moe(tf.MixtralConfig(hidden_size=4096, intermediate_size=14336))
    assert (mx.num_experts, mx.top_k, mx.intermediate_size) == (8, 2, 14336)
    q2 = G.detect_moe(tf.Qwen2MoeConfig(hidden_size=2048, num_experts=60, num_experts_per_tok=4,
                                        moe_intermediate_size=1408, shared_expert_intermediate_size=5632))
    assert (q2.num_experts, q2.shared_intermediate_size, q2.shared_expert_gate) == (60, 5632, True)
    ds = G.detect_moe({"model_type": "deepseek_v3", "hidden_size": 7168, "n_routed_experts": 256,
                       "num_experts_per_tok": 8, "moe_intermediate_size": 2048, "n_shared_experts": 1,
                       "scoring_func": "sigmoid", "routed_scaling_factor": 2.5, "n_group": 8, "topk_group": 4})
    assert (ds.num_experts, ds.shared_intermediate_size, ds.scoring, ds.n_group, ds.topk_group) == \
        (256, 2048, "sigmoid", 8, 4)
    assert G.detect_moe({"model_type": "llama", "hidden_size": 4096}) is None
