"""Drop-in integration with transformers models.

The MoE path PHANTOM executes is transformers' sparse-MoE block, reached from
``from_pretrained`` (python/phantom/phantom_cli.py:1393-1410,
phantom_tui.py:2140-2153): ``Qwen3MoeSparseMoeBlock.forward`` (transformers
5.5.0 models/qwen3_moe/modeling_qwen3_moe.py:281-286), and likewise
``MixtralSparseMoeBlock``, ``Qwen2MoeSparseMoeBlock`` and ``DeepseekV3MoE``
(models/deepseek_v3/modeling_deepseek_v3.py). ``install_into``
packs each block's weights once into the int4 layout on the GPU (router
``gate.weight [E, H]``, ``experts.gate_up_proj [E, 2I, H]``,
``experts.down_proj [E, H, I]``, and for Qwen2-MoE the shared expert and its
sigmoid gate, for DeepSeek-V3 the shared experts, the score-correction bias
and the group settings) and replaces the block's ``forward`` with
:func:`moe_layer`, so ``model.generate`` runs the experts on this library's
kernels. Routing semantics follow each block's router: top-k
renormalisation per ``norm_topk_prob`` (Mixtral always renormalises);
DeepSeek-V3's sigmoid scoring, group-limited choice and routed scaling.
"""

from __future__ import annotations

import dataclasses
import types
from typing import List, Optional, Tuple

import torch

from .layer import MoeLayer, PackedExperts, pack_experts, pack_experts_shared

SUPPORTED_BLOCKS = ("Qwen3MoeSparseMoeBlock", "MixtralSparseMoeBlock", "Qwen2MoeSparseMoeBlock", "DeepseekV3MoE")


@dataclasses.dataclass
class InstalledMoe:
    """What a patched block runs: packed experts and routing settings."""
    kind: str
    packed: PackedExperts
    router_weight: torch.Tensor
    top_k: int
    renormalize: bool
    path: str
    shared_gate: Optional[torch.Tensor]
    original_forward: object
    dense_kept: bool
    routing: dict = dataclasses.field(default_factory=dict)  # extra moe_layer routing arguments
    layer: Optional[MoeLayer] = None  # the bound layer the patched forward calls


def find_moe_blocks(model: torch.nn.Module) -> List[Tuple[str, torch.nn.Module]]:
    """(name, module) of every supported sparse-MoE block in ``model``."""
    return [(n, m) for n, m in model.named_modules() if type(m).__name__ in SUPPORTED_BLOCKS]


def _router_dtype(t: torch.Tensor) -> torch.dtype:
    return t.dtype if t.dtype in (torch.bfloat16, torch.float32) else torch.bfloat16


def _pack_block(blk: torch.nn.Module, group_size: int, path: str, keep_dense: bool) -> InstalledMoe:
    kind = type(blk).__name__
    gate, experts = blk.gate, blk.experts
    dev = experts.gate_up_proj.device
    if dev.type != "cuda":
        raise ValueError(f"{kind}: install_into needs the model on a CUDA device (got {dev}); "
                         "phantom_moe has no CPU path")
    gu, dn = experts.gate_up_proj.detach(), experts.down_proj.detach()
    rdt = _router_dtype(gate.weight)
    shared_gate = None
    with torch.no_grad():
        se = blk.shared_expert if kind == "Qwen2MoeSparseMoeBlock" else getattr(blk, "shared_experts", None)
        if se is not None:
            packed = pack_experts_shared(gu.float(), dn.float(), se.gate_proj.weight.float(), se.up_proj.weight.float(),
                                         se.down_proj.weight.float(), group_size)
        else:
            packed = pack_experts(gu.float(), dn.float(), group_size)
        if kind == "Qwen2MoeSparseMoeBlock":
            shared_gate = blk.shared_expert_gate.weight.detach().reshape(-1).to(rdt).contiguous()
    routing = {}
    if kind == "DeepseekV3MoE":
        renorm, top_k = bool(blk.norm_topk_prob), int(blk.top_k)
        routing = dict(scoring="sigmoid", score_bias=gate.e_score_correction_bias.detach().float().contiguous(),
                       n_group=int(blk.n_group), topk_group=int(blk.topk_group),
                       routed_scale=float(blk.routed_scaling_factor))
    else:
        renorm = True if kind == "MixtralSparseMoeBlock" else bool(getattr(gate, "norm_topk_prob", True))
        top_k = int(gate.top_k)
    st = InstalledMoe(kind, packed, gate.weight.detach().to(rdt).contiguous(), top_k, renorm, path,
                      shared_gate, blk.forward, keep_dense, routing)
    p = packed
    st.layer = MoeLayer(st.router_weight, p.w13_q, p.w13_scales, p.w2_q, p.w2_scales, top_k, renorm, p.group_size,
                        path=path, num_shared=p.num_shared, shared_gate_weight=shared_gate, **routing)
    if not keep_dense:  # the packed copy replaces the dense expert weights
        empty = torch.empty(0, device=dev, dtype=gu.dtype)
        experts.gate_up_proj.data = empty
        experts.down_proj.data = empty
        se = blk.shared_expert if kind == "Qwen2MoeSparseMoeBlock" else getattr(blk, "shared_experts", None)
        if se is not None:
            for lin in (se.gate_proj, se.up_proj, se.down_proj):
                lin.weight.data = torch.empty(0, device=dev, dtype=lin.weight.dtype)
    return st


def _forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
    st: InstalledMoe = self._phmoe
    shape = hidden_states.shape
    x = hidden_states.reshape(-1, shape[-1])
    dt = x.dtype
    if dt not in (torch.bfloat16, torch.float32):
        x = x.to(torch.bfloat16)
    out = st.layer(x.contiguous())
    return out.to(dt).reshape(shape)


def install_into(model: torch.nn.Module, group_size: int = 64, path: str = "auto",
                 keep_dense: bool = False) -> List[str]:
    """Replace the forward of every supported MoE block of ``model`` (already
    on a CUDA device) with this library's layer; returns the block names.

    The expert weights are quantised to int4 (``group_size`` 32 or 64) once;
    unless ``keep_dense`` the dense expert tensors are released afterwards
    (``uninstall`` needs them kept)."""
    names = []
    for name, blk in find_moe_blocks(model):
        if hasattr(blk, "_phmoe"):
            continue
        blk._phmoe = _pack_block(blk, group_size, path, keep_dense)
        blk.forward = types.MethodType(_forward, blk)
        names.append(name)
    return names


def uninstall(model: torch.nn.Module) -> List[str]:
    """Restore the original forward of blocks installed with keep_dense=True."""
    names = []
    for name, blk in find_moe_blocks(model):
        st = getattr(blk, "_phmoe", None)
        if st is None:
            continue
        if not st.dense_kept:
            raise RuntimeError(f"{name}: installed without keep_dense=True, the dense weights are gone")
        blk.__dict__.pop("forward", None)  # the class forward again
        del blk._phmoe
        names.append(name)
    return names
