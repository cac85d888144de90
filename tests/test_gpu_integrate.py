"""install_into on the GPU: a patched transformers model against the same
model running transformers' own MoE blocks on the int4-dequantised expert
weights (block by block on identical inputs, and end to end)."""

from __future__ import annotations

import copy

import numpy as np
import pytest
import torch

pytest.importorskip("transformers")

import phantom_moe as pm  # noqa: E402
from oracle import moe_oracle as O  # noqa: E402
from tests.hf_models import tiny_model  # noqa: E402

pytestmark = pytest.mark.gpu


def _dequantised_copy(model, group=64):
    """A copy whose expert (and shared-expert) weights are their int4 values."""
    ref = copy.deepcopy(model)
    for _, blk in pm.find_moe_blocks(ref):
        ex = blk.experts
        with torch.no_grad():
            for p in (ex.gate_up_proj, ex.down_proj):
                q, s = O.quantize_int4(p.detach().float().cpu().numpy(), group)
                p.copy_(torch.from_numpy(O.dequantize_int4(q, s, group)).to(p.dtype))
            se = getattr(blk, "shared_expert", None) or getattr(blk, "shared_experts", None)
            if se is not None:
                for lin in (se.gate_proj, se.up_proj, se.down_proj):
                    q, s = O.quantize_int4(lin.weight.detach().float().cpu().numpy(), group)
                    lin.weight.copy_(torch.from_numpy(O.dequantize_int4(q, s, group)).to(lin.weight.dtype))
    return ref


@pytest.mark.parametrize("kind", ["qwen3_moe", "mixtral", "qwen2_moe", "deepseek_v3"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_install_into_matches_transformers(cuda_device, kind, dtype):
    """Each patched block against transformers' own block in fp32 on the
    int4-dequantised weights and the same inputs; then the whole model's
    logits. (A bf16 transformers block is no reference: it rounds the router
    logits to bf16 before top-k and its own result carries ~1e-2 error.)"""
    model = tiny_model(kind, seed=3).to(cuda_device, dtype)
    ref = _dequantised_copy(model).float()
    ref_blocks = dict(pm.find_moe_blocks(ref))
    ids = torch.randint(0, 256, (2, 24), device=cuda_device, generator=torch.Generator(device=cuda_device).manual_seed(4))
    with torch.no_grad():
        logits_ref = ref(ids).logits.float()
    names = pm.install_into(model, path="decode")
    assert len(names) == 2
    tol = (1e-3, O.DECODE_FP32_MEAN_REL) if dtype == torch.float32 else (0.05, O.MEAN_REL_TOL)
    gen = torch.Generator(device=cuda_device).manual_seed(5)
    with torch.no_grad():
        for n, blk in pm.find_moe_blocks(model):
            x = torch.randn(2, 24, 256, device=cuda_device, generator=gen).to(dtype)
            got = blk(x).float()
            want = ref_blocks[n](x.float()).float()
            mx, mr = O.parity_stats(got.cpu().numpy(), want.cpu().numpy())
            assert mx <= tol[0] and mr <= tol[1], (n, mx, mr)
        logits = model(ids).logits.float()
    mx, mr = O.parity_stats(logits.cpu().numpy(), logits_ref.cpu().numpy())
    assert mr <= (1e-3 if dtype == torch.float32 else 5e-2), (mx, mr)
    # dense expert weights were released
    assert all(b.experts.gate_up_proj.numel() == 0 for _, b in pm.find_moe_blocks(model))


def test_generate_and_uninstall(cuda_device):
    model = tiny_model("qwen3_moe", seed=5).to(cuda_device, torch.bfloat16)
    ids = torch.randint(0, 256, (1, 8), device=cuda_device, generator=torch.Generator(device=cuda_device).manual_seed(6))
    pm.install_into(model, keep_dense=True)
    out = model.generate(ids, max_new_tokens=6, do_sample=False)
    assert out.shape == (1, 14)
    assert pm.uninstall(model) and not any(hasattr(b, "_phmoe") for _, b in pm.find_moe_blocks(model))
    out2 = model.generate(ids, max_new_tokens=2, do_sample=False)  # transformers' own blocks again
    assert out2.shape == (1, 10)
