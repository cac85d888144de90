"""install_into on the CPU: block discovery and the loud refusal of CPU
models (there is no CPU path)."""

from __future__ import annotations

import pytest

pytest.importorskip("transformers")

import phantom_moe as pm  # noqa: E402
from tests.hf_models import tiny_model  # noqa: E402


@pytest.mark.parametrize("kind,cls", [("qwen3_moe", "Qwen3MoeSparseMoeBlock"), ("mixtral", "MixtralSparseMoeBlock"),
                                      ("qwen2_moe", "Qwen2MoeSparseMoeBlock"), ("deepseek_v3", "DeepseekV3MoE")])
def test_find_blocks(kind, cls):
    model = tiny_model(kind)
    blocks = pm.find_moe_blocks(model)
    assert len(blocks) == 2 and all(type(m).__name__ == cls for _, m in blocks)
    spec = pm.detect_moe(model.config)
    assert (spec.num_experts, spec.top_k) == ((16, 4) if kind == "deepseek_v3" else (8, 2))
    if kind == "deepseek_v3":
        assert (spec.scoring, spec.n_group, spec.topk_group, spec.shared_intermediate_size) == ("sigmoid", 4, 2, 256)


def test_install_refuses_cpu_model():
    model = tiny_model("qwen3_moe")
    with pytest.raises(ValueError, match="CUDA"):
        pm.install_into(model)
    assert not any(hasattr(m, "_phmoe") for _, m in pm.find_moe_blocks(model))
