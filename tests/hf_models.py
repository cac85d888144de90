"""Tiny random-init transformers MoE models for the integration tests (test
infrastructure): Qwen3-MoE, Mixtral and Qwen2-MoE (with a shared expert)
with shapes the packed kernels take (H 256, I 128, 8 experts, top-2)."""

from __future__ import annotations

import torch


def tiny_model(kind: str, seed: int = 0, dtype=torch.float32):
    import transformers as tf
    torch.manual_seed(seed)
    common = dict(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                  vocab_size=256, max_position_embeddings=128, num_experts_per_tok=2)
    if kind == "qwen3_moe":
        cfg = tf.Qwen3MoeConfig(num_experts=8, moe_intermediate_size=128, norm_topk_prob=True, head_dim=64, **common)
        model = tf.Qwen3MoeForCausalLM(cfg)
    elif kind == "mixtral":
        cfg = tf.MixtralConfig(num_local_experts=8, intermediate_size=128, **common)
        model = tf.MixtralForCausalLM(cfg)
    elif kind == "qwen2_moe":
        cfg = tf.Qwen2MoeConfig(num_experts=8, moe_intermediate_size=128, shared_expert_intermediate_size=512,
                                intermediate_size=512, norm_topk_prob=False, **common)
        model = tf.Qwen2MoeForCausalLM(cfg)
    elif kind == "deepseek_v3":
        cfg = tf.DeepseekV3Config(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=4,
                                  vocab_size=256, max_position_embeddings=128, n_routed_experts=16, n_group=4,
                                  topk_group=2, num_experts_per_tok=4, moe_intermediate_size=128, n_shared_experts=2,
                                  routed_scaling_factor=2.5, first_k_dense_replace=0, intermediate_size=512,
                                  q_lora_rank=64, kv_lora_rank=64, qk_rope_head_dim=32, qk_nope_head_dim=32,
                                  v_head_dim=32, norm_topk_prob=True)
        model = tf.DeepseekV3ForCausalLM(cfg)
    else:
        raise ValueError(kind)
    with torch.no_grad():  # weights of a realistic scale (init std 0.02 everywhere)
        for name, p in model.named_parameters():
            if p.dim() >= 2:
                p.normal_(0.0, 0.02)
        for name, b in model.named_buffers():
            if name.endswith("e_score_correction_bias"):
                b.normal_(0.0, 0.05)
    cfg._experts_implementation = "eager"
    return model.to(dtype).eval()
