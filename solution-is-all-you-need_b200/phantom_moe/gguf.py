"""GGUF import: llama.cpp-quantised MoE expert tensors into the packed layout.

The reference loads GGUF models by dequantising every tensor to bf16 at load
time (python/phantom/loader/gguf_loader.py:799-805 -> ``dequantize_tensor_cuda``,
gguf_loader.py:538) and then runs the experts on dense bf16 weights. Here the
quantised expert tensors go straight into the packed int4 layout the FFN
kernels read, on the GPU:

* Q4_0 -> group 32, bit-exact (``phmoe_gguf_q4_0_to_packed``);
* Q4_K -> dequantised in fp32 exactly as the reference does, re-quantised to
  the symmetric format (``phmoe_gguf_q4_k_to_packed``; lossy, because the
  symmetric format has no per-group minimum).

Also here: a small GGUF file reader (header, metadata, tensor table; data
memory-mapped) and the MoE metadata detection of the reference's loaders
(gguf_loader.py:252-301 for GGUF metadata, format_detect.py:98-127 for
transformers configs), extended to the MoE families the layer serves.
"""

from __future__ import annotations

import dataclasses
import mmap
import os
import struct
from typing import Any, Dict, Optional, Tuple

import numpy as np
import torch

from . import _lib
from .layer import _ptr, _stream

# GGML tensor types (llama.cpp ggml.h numbering) and their block geometry:
# type -> (elements per block, bytes per block)
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0, GGML_Q4_K, GGML_Q6_K, GGML_BF16 = 0, 1, 2, 8, 12, 14, 30
_BLOCK = {
    0: (1, 4), 1: (1, 2), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34), 9: (32, 36),
    10: (256, 84), 11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210), 15: (256, 292), 30: (1, 2),
}
_TYPE_NAMES = {0: "F32", 1: "F16", 2: "Q4_0", 3: "Q4_1", 6: "Q5_0", 7: "Q5_1", 8: "Q8_0", 9: "Q8_1",
               10: "Q2_K", 11: "Q3_K", 12: "Q4_K", 13: "Q5_K", 14: "Q6_K", 15: "Q8_K", 30: "BF16"}

# GGUF metadata value types -> struct format (scalars)
_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
_STRING, _ARRAY = 8, 9


@dataclasses.dataclass
class TensorInfo:
    name: str
    dims: Tuple[int, ...]      # GGUF order: dims[0] is the innermost (contiguous) dimension
    ggml_type: int
    offset: int                # from the start of the data section

    @property
    def shape(self) -> Tuple[int, ...]:
        """Row-major shape (outermost first)."""
        return tuple(reversed(self.dims))

    @property
    def n_elements(self) -> int:
        n = 1
        for d in self.dims:
            n *= d
        return n

    @property
    def n_bytes(self) -> int:
        per, nbytes = _BLOCK[self.ggml_type]
        return self.n_elements // per * nbytes

    @property
    def type_name(self) -> str:
        return _TYPE_NAMES.get(self.ggml_type, str(self.ggml_type))


class GGUFFile:
    """Read-only view of a GGUF (v2/v3) file: ``metadata`` (key -> value),
    ``tensors`` (name -> :class:`TensorInfo`) and :meth:`tensor_bytes`
    (a zero-copy uint8 view of one tensor's data)."""

    def __init__(self, path: str | os.PathLike):
        self.path = os.fspath(path)
        with open(self.path, "rb") as f:
            self._mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        buf = self._mm
        if buf[:4] != b"GGUF":
            raise ValueError(f"{self.path}: not a GGUF file")
        self.version, = struct.unpack_from("<I", buf, 4)
        if self.version not in (2, 3):
            raise ValueError(f"{self.path}: unsupported GGUF version {self.version}")
        n_tensors, n_kv = struct.unpack_from("<QQ", buf, 8)
        pos = 24
        self.metadata: Dict[str, Any] = {}
        for _ in range(n_kv):
            key, pos = self._string(pos)
            vtype, = struct.unpack_from("<I", buf, pos)
            value, pos = self._value(vtype, pos + 4)
            self.metadata[key] = value
        self.tensors: Dict[str, TensorInfo] = {}
        for _ in range(n_tensors):
            name, pos = self._string(pos)
            nd, = struct.unpack_from("<I", buf, pos)
            dims = struct.unpack_from(f"<{nd}Q", buf, pos + 4)
            pos += 4 + 8 * nd
            gtype, off = struct.unpack_from("<IQ", buf, pos)
            pos += 12
            if gtype not in _BLOCK:
                raise ValueError(f"{name}: unsupported GGML type {gtype}")
            self.tensors[name] = TensorInfo(name, tuple(int(d) for d in dims), int(gtype), int(off))
        align = int(self.metadata.get("general.alignment", 32))
        self.data_offset = (pos + align - 1) // align * align

    def _string(self, pos: int) -> Tuple[str, int]:
        n, = struct.unpack_from("<Q", self._mm, pos)
        return bytes(self._mm[pos + 8: pos + 8 + n]).decode("utf-8"), pos + 8 + n

    def _value(self, vtype: int, pos: int) -> Tuple[Any, int]:
        if vtype in _SCALAR:
            fmt = _SCALAR[vtype]
            return struct.unpack_from(fmt, self._mm, pos)[0], pos + struct.calcsize(fmt)
        if vtype == _STRING:
            return self._string(pos)
        if vtype == _ARRAY:
            etype, count = struct.unpack_from("<IQ", self._mm, pos)
            pos += 12
            out = []
            for _ in range(count):
                v, pos = self._value(etype, pos)
                out.append(v)
            return out, pos
        raise ValueError(f"unsupported GGUF metadata type {vtype}")

    def tensor_bytes(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        start = self.data_offset + t.offset
        return np.frombuffer(self._mm, dtype=np.uint8, count=t.n_bytes, offset=start)

    def close(self) -> None:
        self._mm.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


# ---------------------------------------------------------------------------
# GPU importers (C ABI)
# ---------------------------------------------------------------------------

def _blocks_on(blocks, device) -> torch.Tensor:
    if isinstance(blocks, np.ndarray):
        a = np.ascontiguousarray(blocks).view(np.uint8).reshape(-1)
        if not a.flags.writeable:  # a memory-mapped file: torch wants writeable memory
            a = a.copy()
        blocks = torch.from_numpy(a)
    if blocks.dtype != torch.uint8:
        raise TypeError("GGUF blocks must be uint8 bytes")
    return blocks.reshape(-1).to(device, non_blocking=True).contiguous()


def q4_0_to_packed(blocks, rows: int, K: int, device=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """GGUF Q4_0 data of a [rows, K] tensor -> (packed uint8 [rows, K/2],
    scales fp16 [rows, K/32]) on the GPU; lossless (group size 32)."""
    device = torch.device(device or "cuda")
    b = _blocks_on(blocks, device)
    if K % 32 or b.numel() != rows * (K // 32) * 18:
        raise ValueError("Q4_0 data size does not match rows x K")
    packed = torch.empty(rows, K // 2, dtype=torch.uint8, device=device)
    scales = torch.empty(rows, K // 32, dtype=torch.float16, device=device)
    with torch.cuda.device(device):
        _lib.call("phmoe_gguf_q4_0_to_packed", _ptr(b), rows, K, _ptr(packed), _ptr(scales), _stream())
    return packed, scales


def q4_k_to_packed(blocks, rows: int, K: int, group_size: int = 32,
                   device=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """GGUF Q4_K data of a [rows, K] tensor -> packed int4 re-quantised with
    ``group_size`` (32 or 64) from the reference's fp32 dequantised values."""
    device = torch.device(device or "cuda")
    b = _blocks_on(blocks, device)
    if K % 256 or b.numel() != rows * (K // 256) * 144:
        raise ValueError("Q4_K data size does not match rows x K")
    packed = torch.empty(rows, K // 2, dtype=torch.uint8, device=device)
    scales = torch.empty(rows, K // group_size, dtype=torch.float16, device=device)
    with torch.cuda.device(device):
        _lib.call("phmoe_gguf_q4_k_to_packed", _ptr(b), rows, K, group_size, _ptr(packed), _ptr(scales),
                  _stream())
    return packed, scales


def q4_k_dequantize(blocks, n: int, device=None) -> torch.Tensor:
    """GGUF Q4_K data -> fp32 [n] (the reference's dequantised values)."""
    device = torch.device(device or "cuda")
    b = _blocks_on(blocks, device)
    if n % 256 or b.numel() != n // 256 * 144:
        raise ValueError("Q4_K data size does not match n")
    out = torch.empty(n, dtype=torch.float32, device=device)
    with torch.cuda.device(device):
        _lib.call("phmoe_gguf_q4_k_dequantize", _ptr(b), n, _ptr(out), _stream())
    return out


def import_expert_tensor(data, ggml_type: int, rows: int, K: int, group_size: Optional[int] = None,
                         device=None) -> Tuple[torch.Tensor, torch.Tensor, int]:
    """One quantised [rows, K] expert tensor -> (packed, scales, group_size).

    Q4_0 keeps its native group of 32 (lossless); Q4_K is re-quantised with
    ``group_size`` (default 32)."""
    if ggml_type == GGML_Q4_0:
        if group_size not in (None, 32):
            raise ValueError("Q4_0 imports losslessly with group_size 32 only")
        p, s = q4_0_to_packed(data, rows, K, device)
        return p, s, 32
    if ggml_type == GGML_Q4_K:
        g = group_size or 32
        p, s = q4_k_to_packed(data, rows, K, g, device)
        return p, s, g
    raise ValueError(f"expert tensors of GGML type {_TYPE_NAMES.get(ggml_type, ggml_type)} are not supported "
                     "(Q4_0 and Q4_K are)")


def _dense(gf: GGUFFile, name: str, device) -> torch.Tensor:
    t = gf.tensors[name]
    raw = gf.tensor_bytes(name)
    if t.ggml_type == GGML_F32:
        a = torch.from_numpy(raw.view(np.float32).copy())
    elif t.ggml_type == GGML_F16:
        a = torch.from_numpy(raw.view(np.float16).copy()).float()
    elif t.ggml_type == GGML_BF16:
        a = torch.from_numpy(raw.view(np.int16).copy()).view(torch.bfloat16).float()
    else:
        raise ValueError(f"{name}: router weights must be F32/F16/BF16, got {t.type_name}")
    return a.reshape(t.shape).to(device)


def load_moe_layer(gf: GGUFFile, layer: int, device=None, group_size: Optional[int] = None,
                   router_dtype: torch.dtype = torch.bfloat16) -> Dict[str, Any]:
    """The MoE tensors of block ``layer`` of a llama.cpp GGUF file, imported:
    ``router_weight`` [E, H] (``blk.N.ffn_gate_inp``), ``w13_q``/``w13_scales``
    (gate rows then up rows per expert, from ``ffn_gate_exps`` [E, I, H] and
    ``ffn_up_exps``), ``w2_q``/``w2_scales`` (``ffn_down_exps`` [E, H, I]),
    ``group_size``, and the shared-expert tensors when the block has them
    (``ffn_{gate,up,down}_shexp``, ``ffn_gate_inp_shexp``)."""
    device = torch.device(device or "cuda")
    pre = f"blk.{layer}."
    gate, up, down = (gf.tensors[pre + n] for n in ("ffn_gate_exps.weight", "ffn_up_exps.weight",
                                                      "ffn_down_exps.weight"))
    E, I, H = gate.shape
    if up.shape != (E, I, H) or down.shape != (E, H, I):
        raise ValueError(f"block {layer}: expert tensor shapes {gate.shape} {up.shape} {down.shape} disagree")
    if not (gate.ggml_type == up.ggml_type):
        raise ValueError("gate and up experts must share one quantisation type")
    gq, gs, g1 = import_expert_tensor(gf.tensor_bytes(gate.name), gate.ggml_type, E * I, H, group_size, device)
    uq, us, _ = import_expert_tensor(gf.tensor_bytes(up.name), up.ggml_type, E * I, H, g1, device)
    dq, ds, g2 = import_expert_tensor(gf.tensor_bytes(down.name), down.ggml_type, E * H, I, g1, device)
    if g1 != g2:
        raise ValueError("gate/up and down experts import with different group sizes")
    w13_q = torch.cat([gq.view(E, I, H // 2), uq.view(E, I, H // 2)], dim=1).contiguous()
    w13_s = torch.cat([gs.view(E, I, H // g1), us.view(E, I, H // g1)], dim=1).contiguous()
    out: Dict[str, Any] = {
        "router_weight": _dense(gf, pre + "ffn_gate_inp.weight", device).to(router_dtype).contiguous(),
        "w13_q": w13_q, "w13_scales": w13_s,
        "w2_q": dq.view(E, H, I // 2), "w2_scales": ds.view(E, H, I // g1),
        "group_size": g1, "num_experts": E, "hidden_size": H, "intermediate_size": I,
    }
    if pre + "ffn_gate_shexp.weight" in gf.tensors:
        sg, su, sd = (gf.tensors[pre + n] for n in ("ffn_gate_shexp.weight", "ffn_up_shexp.weight",
                                                      "ffn_down_shexp.weight"))
        Is = sg.shape[0]
        q1, s1, _ = import_expert_tensor(gf.tensor_bytes(sg.name), sg.ggml_type, Is, H, g1, device)
        q2, s2, _ = import_expert_tensor(gf.tensor_bytes(su.name), su.ggml_type, Is, H, g1, device)
        q3, s3, _ = import_expert_tensor(gf.tensor_bytes(sd.name), sd.ggml_type, H, Is, g1, device)
        out["shared"] = {"w13_q": torch.cat([q1, q2], 0).unsqueeze(0), "w13_scales": torch.cat([s1, s2], 0).unsqueeze(0),
                         "w2_q": q3.unsqueeze(0), "w2_scales": s3.unsqueeze(0), "intermediate_size": Is}
        if pre + "ffn_gate_inp_shexp.weight" in gf.tensors:
            out["shared"]["gate_weight"] = _dense(gf, pre + "ffn_gate_inp_shexp.weight", device).reshape(1, H)
    return out


# ---------------------------------------------------------------------------
# MoE metadata detection
# ---------------------------------------------------------------------------

@dataclasses.dataclass
class MoeSpec:
    """What the layer needs to know about a model's MoE blocks."""
    family: str
    num_experts: int
    top_k: int
    hidden_size: int
    intermediate_size: int             # per routed expert
    num_layers: int = 0
    norm_topk_prob: bool = True        # renormalise the picked probabilities
    shared_intermediate_size: int = 0  # 0: no shared expert
    shared_expert_gate: bool = False   # sigmoid gate on the shared expert (Qwen2-MoE)
    scoring: str = "softmax"           # "softmax" or "sigmoid" (DeepSeek-V3)
    routed_scaling_factor: float = 1.0
    n_group: int = 1
    topk_group: int = 1

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0


def detect_moe(source) -> Optional[MoeSpec]:
    """MoE configuration from a GGUF file (path or :class:`GGUFFile`), a
    transformers config object, or a config dict; None for a dense model.

    GGUF keys follow the reference's GGUF loader (gguf_loader.py:252-301:
    ``{arch}.expert_count``, ``{arch}.expert_used_count``,
    ``{arch}.embedding_length``, ``{arch}.block_count``) plus llama.cpp's
    ``expert_feed_forward_length`` / ``expert_shared_feed_forward_length``;
    transformers configs follow format_detect.py:98-127 (DeepSeek
    ``n_routed_experts``, Mixtral ``num_local_experts``, Qwen2-MoE
    ``num_experts``) and add Qwen3-MoE (``model_type`` "qwen3_moe").
    """
    if isinstance(source, (str, os.PathLike)):
        with GGUFFile(source) as gf:
            return _detect_gguf(gf.metadata)
    if isinstance(source, GGUFFile):
        return _detect_gguf(source.metadata)
    if isinstance(source, dict):
        return _detect_config(source)
    cfg = source.to_dict()
    for key in ("num_experts", "num_local_experts", "n_routed_experts"):  # attribute-mapped names
        if hasattr(source, key):
            cfg[key] = getattr(source, key)
    return _detect_config(cfg)


def _detect_gguf(kv: Dict[str, Any]) -> Optional[MoeSpec]:
    arch = kv.get("general.architecture", "llama")
    p = arch + "."
    E = int(kv.get(p + "expert_count", 0))
    if E <= 0:
        return None
    H = int(kv.get(p + "embedding_length", 0))
    ffn = int(kv.get(p + "expert_feed_forward_length", kv.get(p + "feed_forward_length", 0)))
    spec = MoeSpec(family=arch, num_experts=E, top_k=int(kv.get(p + "expert_used_count", 0)), hidden_size=H,
                   intermediate_size=ffn, num_layers=int(kv.get(p + "block_count", 0)))
    if arch == "llama":          # Mixtral GGUFs use the llama architecture with experts
        spec.family = "mixtral"
    shared = int(kv.get(p + "expert_shared_feed_forward_length", 0))
    n_shared = int(kv.get(p + "expert_shared_count", 0))
    if arch.startswith("deepseek"):
        spec.shared_intermediate_size = n_shared * ffn
        spec.norm_topk_prob = bool(kv.get(p + "expert_weights_norm", True))
        spec.routed_scaling_factor = float(kv.get(p + "expert_weights_scale", 1.0))
        spec.scoring = "sigmoid" if int(kv.get(p + "expert_gating_func", 1)) == 2 else "softmax"
    elif arch == "qwen2moe":
        spec.shared_intermediate_size = shared
        spec.shared_expert_gate = shared > 0
        spec.norm_topk_prob = False
    return spec


def _detect_config(cfg: Dict[str, Any]) -> Optional[MoeSpec]:
    mt = str(cfg.get("model_type", "")).lower()
    archs = [str(a).lower() for a in (cfg.get("architectures") or [])]
    H = int(cfg.get("hidden_size", 0))
    L = int(cfg.get("num_hidden_layers", 0))
    if "deepseek" in mt or any("deepseek" in a for a in archs):
        E = int(cfg.get("n_routed_experts") or 0)
        if not E:
            return None
        I = int(cfg["moe_intermediate_size"])
        return MoeSpec("deepseek", E, int(cfg.get("num_experts_per_tok", 8)), H, I, L,
                       norm_topk_prob=bool(cfg.get("norm_topk_prob", True)),
                       shared_intermediate_size=int(cfg.get("n_shared_experts") or 0) * I,
                       scoring=str(cfg.get("scoring_func", "sigmoid" if "v3" in mt or any("v3" in a for a in archs)
                                           else "softmax")),
                       routed_scaling_factor=float(cfg.get("routed_scaling_factor", 1.0)),
                       n_group=int(cfg.get("n_group") or 1), topk_group=int(cfg.get("topk_group") or 1))
    if "mixtral" in mt or any("mixtral" in a for a in archs):
        return MoeSpec("mixtral", int(cfg.get("num_local_experts", 8)), int(cfg.get("num_experts_per_tok", 2)), H,
                       int(cfg["intermediate_size"]), L, norm_topk_prob=True)
    if mt == "qwen2_moe":
        return MoeSpec("qwen2_moe", int(cfg.get("num_experts") or cfg.get("num_local_experts") or 60), int(cfg.get("num_experts_per_tok", 4)), H,
                       int(cfg["moe_intermediate_size"]), L, norm_topk_prob=bool(cfg.get("norm_topk_prob", False)),
                       shared_intermediate_size=int(cfg.get("shared_expert_intermediate_size", 0)),
                       shared_expert_gate=True)
    if mt == "qwen3_moe":
        return MoeSpec("qwen3_moe", int(cfg.get("num_experts") or cfg.get("num_local_experts") or 128), int(cfg.get("num_experts_per_tok", 8)), H,
                       int(cfg["moe_intermediate_size"]), L, norm_topk_prob=bool(cfg.get("norm_topk_prob", True)))
    return None
