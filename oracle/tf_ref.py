"""The reference's own CPU MoE path, for timing (test/bench infrastructure).

PHANTOM runs MoE layers through transformers' ``Qwen3MoeSparseMoeBlock`` /
``MixtralSparseMoeBlock`` (python/phantom/phantom_cli.py:1393-1430 ->
transformers 5.5.0 models/qwen3_moe/modeling_qwen3_moe.py:275-286). This
module instantiates that block in fp32 on the CPU with the dequantised int4
expert weights, so ``bench.py`` can time the reference path on the same
workload as the CUDA layer. Only ``bench.py``'s CPU legs and tests use it.
"""

from __future__ import annotations

import os

import numpy as np
import torch

from . import moe_oracle as O


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def build_block(kind: str, wr: np.ndarray, w13_q, w13_s, w2_q, w2_s, top_k: int, group: int = 64,
                renormalize: bool = True):
    """transformers block (fp32, CPU, eager experts loop) holding the
    dequantised weights of one layer."""
    E, I2, Hh = w13_q.shape
    H, I = Hh * 2, I2 // 2
    if kind == "qwen3":
        from transformers.models.qwen3_moe.configuration_qwen3_moe import Qwen3MoeConfig
        from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeSparseMoeBlock
        cfg = Qwen3MoeConfig(hidden_size=H, num_experts=E, num_experts_per_tok=top_k,
                             moe_intermediate_size=I, norm_topk_prob=renormalize)
        cfg._experts_implementation = "eager"
        blk = Qwen3MoeSparseMoeBlock(cfg)
    else:
        from transformers.models.mixtral.configuration_mixtral import MixtralConfig
        from transformers.models.mixtral.modeling_mixtral import MixtralSparseMoeBlock
        cfg = MixtralConfig(hidden_size=H, num_local_experts=E, num_experts_per_tok=top_k, intermediate_size=I)
        cfg._experts_implementation = "eager"
        blk = MixtralSparseMoeBlock(cfg)
    blk = blk.eval()
    with torch.no_grad():
        blk.gate.weight.copy_(torch.from_numpy(np.asarray(wr, dtype=np.float32)))
        for e in range(E):
            blk.experts.gate_up_proj[e].copy_(torch.from_numpy(O.dequantize_int4(w13_q[e], w13_s[e], group)))
            blk.experts.down_proj[e].copy_(torch.from_numpy(O.dequantize_int4(w2_q[e], w2_s[e], group)))
    return blk


def forward(blk, x: np.ndarray) -> np.ndarray:
    with torch.inference_mode():
        out = blk(torch.from_numpy(np.asarray(x, dtype=np.float32))[None])
        if isinstance(out, tuple):
            out = out[0]
    return out[0].numpy()
