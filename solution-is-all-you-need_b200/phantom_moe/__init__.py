"""phantom_moe - B200-native (sm_100a) sparse-MoE layer.

Drop-in for the MoE block that PHANTOM (FreakyAdy/Solution-is-all-You-need)
runs through transformers (python/phantom/phantom_cli.py:1393-1430 ->
Qwen3MoeSparseMoeBlock.forward, transformers 5.5.0
models/qwen3_moe/modeling_qwen3_moe.py:281-286), with int4 group-quantised
experts. The compute is hand-written CUDA in ``libphmoe.so`` behind the C ABI
of ``include/phmoe.h``; this package validates tensors and calls it.
"""

from ._lib import PhmoeError, load as load_library
from .gguf import GGUFFile, MoeSpec, detect_moe, load_moe_layer
from .integrate import find_moe_blocks, install_into, uninstall
from .pipeline import HostPipeline
from .layer import (
    DEVICE_ERROR_BITS,
    DeviceError,
    MoeLayer,
    PackedExperts,
    check_device_errors,
    check_expert_weights,
    combine,
    dispatch,
    expert_ffn_decode,
    expert_ffn_prefill,
    gather_rows,
    moe_layer,
    pack_experts,
    pack_experts_shared,
    quantize_int4,
    router,
    router_ex,
    workspace_bytes,
)

__all__ = [
    "DEVICE_ERROR_BITS",
    "DeviceError",
    "GGUFFile",
    "HostPipeline",
    "MoeLayer",
    "MoeSpec",
    "PhmoeError",
    "PackedExperts",
    "check_device_errors",
    "check_expert_weights",
    "combine",
    "detect_moe",
    "dispatch",
    "expert_ffn_decode",
    "find_moe_blocks",
    "expert_ffn_prefill",
    "gather_rows",
    "install_into",
    "load_library",
    "load_moe_layer",
    "moe_layer",
    "pack_experts",
    "pack_experts_shared",
    "quantize_int4",
    "router",
    "router_ex",
    "uninstall",
    "workspace_bytes",
]

__version__ = "0.1.0"
