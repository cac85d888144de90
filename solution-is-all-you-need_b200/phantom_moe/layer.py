"""Host side of the MoE layer: tensor validation + calls into the C ABI.

``moe_layer`` is the drop-in for ``Qwen3MoeSparseMoeBlock.forward`` /
``MixtralSparseMoeBlock.forward`` (transformers 5.5.0
models/qwen3_moe/modeling_qwen3_moe.py:281-286, models/mixtral/modeling_mixtral.py:119-137),
the MoE path PHANTOM executes (python/phantom/phantom_cli.py:1393-1430), with
the weights in packed int4 form. The stage functions (``router``,
``dispatch``, ``expert_ffn_decode``, ``combine``, ``quantize_int4``) expose
each kernel on its own for tests and for the expert-parallel path.

All work is enqueued on ``torch.cuda.current_stream()``; nothing here
synchronises the device. There is no CPU path: CPU tensors are rejected.
"""

from __future__ import annotations

import threading
from dataclasses import dataclass

import torch

from . import _lib

_DT = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16}
_PATHS = {"auto": _lib.PATH_AUTO, "decode": _lib.PATH_DECODE, "prefill": _lib.PATH_PREFILL}
_SCORING = {"softmax": _lib.SCORING_SOFTMAX, "sigmoid": _lib.SCORING_SIGMOID}


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _need_cuda(name: str, t: torch.Tensor) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor (got {t.device}); phantom_moe has no CPU path")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _need_dtype(name: str, t: torch.Tensor, dtypes) -> None:
    if t.dtype not in dtypes:
        raise TypeError(f"{name} must have dtype in {[str(d) for d in dtypes]} (got {t.dtype})")


def _need_shape(name: str, t: torch.Tensor, shape) -> None:
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {tuple(shape)} (got {tuple(t.shape)})")


class _Workspace:
    """Per-(device, stream) scratch buffer, grown on demand through torch's
    caching allocator. Calls on one stream are ordered, so they may share it.

    A CUDA graph captured around ``moe_layer`` bakes the workspace address in,
    so a buffer is never released once handed out: when a larger one is
    needed the old one is kept in ``_retired`` for the life of the process
    (or until :meth:`clear`, which the caller may only use when no captured
    graph that used the workspace will be replayed again)."""

    def __init__(self):
        self._bufs: dict[tuple[int, int], torch.Tensor] = {}
        self._retired: list[torch.Tensor] = []
        self._lock = threading.Lock()

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor:
        key = (device.index if device.index is not None else torch.cuda.current_device(), _stream())
        with self._lock:
            buf = self._bufs.get(key)
            if buf is None or buf.numel() < nbytes:
                if buf is not None:
                    self._retired.append(buf)
                buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
                self._bufs[key] = buf
            return buf

    def clear(self) -> None:
        with self._lock:
            self._bufs.clear()
            self._retired.clear()


WORKSPACE = _Workspace()


class DeviceError(RuntimeError):
    """A kernel of this library raised a bit of the device error word
    (``phmoe_device_error``). ``bits`` holds the word; see
    :data:`DEVICE_ERROR_BITS` for the meanings."""

    def __init__(self, bits: int):
        self.bits = bits
        names = [txt for b, txt in DEVICE_ERROR_BITS.items() if bits & b] or [f"unknown bits {bits:#x}"]
        super().__init__("phantom_moe device error: " + "; ".join(names))


DEVICE_ERROR_BITS = {
    1: "an FFN pipeline wait timed out (its CTA abandoned its work; results are incomplete)",
    2: "an activation could not be held by the decode FFN's fixed-point rows (beyond ~1e34, inf or NaN)",
    4: "an expert-parallel peer flag did not arrive within 2 s (a peer stopped calling the layer)",
}


def check_device_errors(reset: bool = True) -> None:
    """Raise :class:`DeviceError` if any kernel of this library raised a bit
    of the current device's error word since it was last cleared (``reset``
    clears it). Waits for the device (``cudaMemcpyFromSymbol``): call it
    between steps, not on a latency-critical path."""
    bits = _lib.load().phmoe_device_error(int(bool(reset)))
    if bits < 0:
        raise RuntimeError("phmoe_device_error: reading the device error word failed")
    if bits:
        raise DeviceError(bits)


@dataclass
class PackedExperts:
    """Packed int4 expert weights for one layer.

    w13_q [E, 2I, H/2] uint8 (gate rows 0..I-1, up rows I..2I-1, as
    ``gate_up_proj`` is split by ``chunk(2)``, modeling_qwen3_moe.py:245),
    w13_scales [E, 2I, H/G] fp16, w2_q [E, H, I/2] uint8, w2_scales [E, H, I/G] fp16.
    """

    w13_q: torch.Tensor
    w13_scales: torch.Tensor
    w2_q: torch.Tensor
    w2_scales: torch.Tensor
    group_size: int = 64
    num_shared: int = 0  # trailing experts that are slices of a shared expert (pack_experts_shared)

    @property
    def num_experts(self) -> int:
        return self.w13_q.shape[0]

    @property
    def hidden_size(self) -> int:
        return self.w2_q.shape[1]

    @property
    def intermediate_size(self) -> int:
        return self.w13_q.shape[1] // 2


def check_expert_weights(w13_q, w13_scales, w2_q, w2_scales, H: int, group_size: int):
    """Validate packed expert tensors; returns (E, I)."""
    for n, t in (("w13_q", w13_q), ("w13_scales", w13_scales), ("w2_q", w2_q), ("w2_scales", w2_scales)):
        _need_cuda(n, t)
    _need_dtype("w13_q", w13_q, (torch.uint8,))
    _need_dtype("w2_q", w2_q, (torch.uint8,))
    _need_dtype("w13_scales", w13_scales, (torch.float16,))
    _need_dtype("w2_scales", w2_scales, (torch.float16,))
    if group_size not in (32, 64):
        raise ValueError(f"group_size must be 32 or 64 (got {group_size})")
    if w13_q.dim() != 3:
        raise ValueError("w13_q must be [E, 2I, H/2]")
    E, I2, Hh = w13_q.shape
    if I2 % 2:
        raise ValueError("w13_q dim 1 must be 2*I")
    I = I2 // 2
    _need_shape("w13_q", w13_q, (E, 2 * I, H // 2))
    _need_shape("w13_scales", w13_scales, (E, 2 * I, H // group_size))
    _need_shape("w2_q", w2_q, (E, H, I // 2))
    _need_shape("w2_scales", w2_scales, (E, H, I // group_size))
    return E, I


# ---------------------------------------------------------------------------
# stage entry points
# ---------------------------------------------------------------------------

def router(x: torch.Tensor, router_weight: torch.Tensor, top_k: int, renormalize: bool = True,
           return_probs: bool = False):
    """Fused router (Qwen3MoeTopKRouter.forward, modeling_qwen3_moe.py:263-272).

    Returns ``(topk_idx int32[T,k], topk_w fp32[T,k], logits fp32[T,E])`` and
    ``probs fp32[T,E]`` when ``return_probs``.
    """
    _need_cuda("x", x)
    _need_cuda("router_weight", router_weight)
    _need_dtype("x", x, _DT)
    _need_dtype("router_weight", router_weight, _DT)
    T, H = x.shape
    E = router_weight.shape[0]
    _need_shape("router_weight", router_weight, (E, H))
    dev = x.device
    logits = torch.empty(T, E, dtype=torch.float32, device=dev)
    probs = torch.empty(T, E, dtype=torch.float32, device=dev) if return_probs else None
    idx = torch.empty(T, top_k, dtype=torch.int32, device=dev)
    w = torch.empty(T, top_k, dtype=torch.float32, device=dev)
    _lib.call("phmoe_router", _ptr(x), _DT[x.dtype], _ptr(router_weight), _DT[router_weight.dtype],
              T, H, E, top_k, int(bool(renormalize)), _ptr(logits), _ptr(probs), _ptr(idx), _ptr(w),
              _stream())
    if return_probs:
        return idx, w, logits, probs
    return idx, w, logits


def router_ex(x: torch.Tensor, router_weight: torch.Tensor, top_k: int, renormalize: bool = True,
              scoring: str = "sigmoid", score_bias: torch.Tensor | None = None, n_group: int = 1,
              topk_group: int = 1, routed_scale: float = 1.0):
    """DeepSeek-V3 style router (``phmoe_router_ex``): returns
    ``(topk_idx int32[T,k], topk_w fp32[T,k], logits fp32[T,E])``."""
    _need_cuda("x", x)
    _need_cuda("router_weight", router_weight)
    T, H = x.shape
    E = router_weight.shape[0]
    logits = torch.empty(T, E, dtype=torch.float32, device=x.device)
    idx = torch.empty(T, top_k, dtype=torch.int32, device=x.device)
    w = torch.empty(T, top_k, dtype=torch.float32, device=x.device)
    _lib.call("phmoe_router_ex", _ptr(x), _DT[x.dtype], _ptr(router_weight), _DT[router_weight.dtype], T, H, E,
              top_k, int(bool(renormalize)), _SCORING[scoring], _ptr(score_bias), n_group, topk_group,
              float(routed_scale), _ptr(logits), _ptr(idx), _ptr(w), _stream())
    return idx, w, logits


def dispatch(topk_idx: torch.Tensor, num_experts: int):
    """Expert grouping ordered by token (modeling_qwen3_moe.py:234-244).

    Returns ``(offsets int32[E+1], row_token int32[T*k], inv int32[T,k],
    active int32[E+1])``; ``active[0]`` = experts hit, ``active[1:1+n]`` their ids.
    """
    _need_cuda("topk_idx", topk_idx)
    _need_dtype("topk_idx", topk_idx, (torch.int32,))
    T, k = topk_idx.shape
    dev = topk_idx.device
    E = int(num_experts)
    offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
    active = torch.empty(E + 1, dtype=torch.int32, device=dev)
    row_token = torch.empty(T * k, dtype=torch.int32, device=dev)
    inv = torch.empty(T, k, dtype=torch.int32, device=dev)
    lib = _lib.load()
    nscr = lib.phmoe_dispatch_scratch_size(T, k, E)
    scratch = torch.empty(max(nscr, 1), dtype=torch.uint8, device=dev)
    _lib.call("phmoe_dispatch", _ptr(topk_idx), T, k, E, _ptr(offsets), _ptr(row_token), _ptr(inv),
              _ptr(active), _ptr(scratch), nscr, _stream())
    return offsets, row_token, inv, active


def expert_ffn_decode(x: torch.Tensor, row_token, offsets, active, w13_q, w13_scales, w2_q,
                      w2_scales, top_k: int, group_size: int = 64):
    """Grouped SwiGLU FFN over dispatched rows (modeling_qwen3_moe.py:245-247).

    ``row_token`` holds R rows (the token each row reads); returns y fp32[R, H]
    in permuted-row order.
    """
    _need_cuda("x", x)
    _need_dtype("x", x, _DT)
    T, H = x.shape
    E, I = check_expert_weights(w13_q, w13_scales, w2_q, w2_scales, H, group_size)
    R = row_token.numel()
    if R != T * top_k:
        raise ValueError(f"row_token must have T*top_k = {T * top_k} rows (got {R})")
    dev = x.device
    h = torch.empty(max(R * I, 1), dtype=torch.float32, device=dev)
    y = torch.empty(R, H, dtype=torch.float32, device=dev)
    _lib.call("phmoe_expert_ffn_decode", _ptr(x), _DT[x.dtype], _ptr(row_token), _ptr(offsets),
              _ptr(active), _ptr(w13_q), _ptr(w13_scales), _ptr(w2_q), _ptr(w2_scales), T, H, E,
              top_k, I, group_size, _ptr(h), _ptr(y), _stream())
    return y


def expert_ffn_prefill(x: torch.Tensor, row_token, offsets, active, w13_q, w13_scales, w2_q,
                       w2_scales, top_k: int, group_size: int = 64):
    """Grouped SwiGLU FFN as two tcgen05 grouped GEMMs (large batches; bf16
    ``x``). Same inputs and result layout as :func:`expert_ffn_decode`."""
    _need_cuda("x", x)
    _need_dtype("x", x, (torch.bfloat16,))
    T, H = x.shape
    E, I = check_expert_weights(w13_q, w13_scales, w2_q, w2_scales, H, group_size)
    R = row_token.numel()
    if R != T * top_k:
        raise ValueError(f"row_token must have T*top_k = {T * top_k} rows (got {R})")
    dev = x.device
    h = torch.empty(max(R * I, 1), dtype=torch.float32, device=dev)
    y = torch.empty(R, H, dtype=torch.float32, device=dev)
    _lib.call("phmoe_expert_ffn_prefill", _ptr(x), _DT[x.dtype], _ptr(row_token), _ptr(offsets),
              _ptr(active), _ptr(w13_q), _ptr(w13_scales), _ptr(w2_q), _ptr(w2_scales), T, H, E,
              top_k, I, group_size, _ptr(h), _ptr(y), _stream())
    return y


def combine(y: torch.Tensor, inv: torch.Tensor, topk_w: torch.Tensor, out_dtype=torch.bfloat16):
    """out[t] = sum_j w[t,j] * y[inv[t,j]] (modeling_qwen3_moe.py:248-249)."""
    _need_cuda("y", y)
    T, k = inv.shape
    H = y.shape[1]
    out = torch.empty(T, H, dtype=out_dtype, device=y.device)
    _lib.call("phmoe_combine", _ptr(y), _ptr(inv), _ptr(topk_w), T, k, H, _ptr(out), _DT[out_dtype],
              _stream())
    return out


def gather_rows(src: torch.Tensor, index: torch.Tensor, out: torch.Tensor | None = None):
    """``out[i] = src[index[i]]`` for a 2-D CUDA tensor (rows of a multiple of
    16 bytes); rows whose index is out of range come back zero."""
    _need_cuda("src", src)
    _need_cuda("index", index)
    _need_dtype("index", index, (torch.int32,))
    if src.dim() != 2 or not src.is_contiguous():
        raise ValueError("src must be a contiguous 2-D tensor")
    n = index.numel()
    if out is None:
        out = torch.empty(n, src.shape[1], dtype=src.dtype, device=src.device)
    elif out.shape != (n, src.shape[1]) or out.dtype != src.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous [len(index), src.shape[1]] tensor of src's dtype")
    _lib.call("phmoe_gather_rows", _ptr(src), src.shape[0], _ptr(index), n,
              src.shape[1] * src.element_size(), _ptr(out), _stream())
    return out


def quantize_int4(w: torch.Tensor, group_size: int = 64):
    """GPU symmetric int4 group quantiser: ``w[..., K]`` (fp32/bf16, CUDA) ->
    ``(packed uint8[..., K/2], scales fp16[..., K/G])``."""
    _need_cuda("w", w)
    _need_dtype("w", w, _DT)
    K = w.shape[-1]
    rows = w.numel() // K if K else 0
    packed = torch.empty(*w.shape[:-1], K // 2, dtype=torch.uint8, device=w.device)
    scales = torch.empty(*w.shape[:-1], K // group_size, dtype=torch.float16, device=w.device)
    _lib.call("phmoe_quantize_int4", _ptr(w), _DT[w.dtype], rows, K, group_size, _ptr(packed),
              _ptr(scales), _stream())
    return packed, scales


def pack_experts(gate_up_proj: torch.Tensor, down_proj: torch.Tensor, group_size: int = 64) -> PackedExperts:
    """Quantise dense expert weights in transformers' layout
    (``gate_up_proj [E, 2I, H]``, ``down_proj [E, H, I]``,
    modeling_qwen3_moe.py:221-222) into :class:`PackedExperts` on the GPU."""
    w13_q, w13_s = quantize_int4(gate_up_proj.contiguous(), group_size)
    w2_q, w2_s = quantize_int4(down_proj.contiguous(), group_size)
    return PackedExperts(w13_q, w13_s, w2_q, w2_s, group_size)


def pack_experts_shared(gate_up_proj: torch.Tensor, down_proj: torch.Tensor, shared_gate_proj: torch.Tensor,
                        shared_up_proj: torch.Tensor, shared_down_proj: torch.Tensor,
                        group_size: int = 64) -> PackedExperts:
    """Routed experts (``gate_up_proj [E, 2I, H]``, ``down_proj [E, H, I]``)
    plus one shared SwiGLU expert (``gate_proj`` / ``up_proj`` weights
    ``[Is, H]``, ``down_proj`` weight ``[H, Is]``, Qwen2MoeMLP layout) with
    Is = m * I, packed as E + m experts: the shared expert is cut along its
    intermediate dimension into m experts of size I, whose outputs add up to
    the shared expert's (the int4 groups run along H for gate/up and along
    Is for down, so no group straddles two slices)."""
    E, two_i, H = gate_up_proj.shape
    I = two_i // 2
    Is = shared_gate_proj.shape[0]
    if Is % I:
        raise ValueError(f"shared intermediate size {Is} must be a multiple of the routed experts' {I}")
    m = Is // I
    dt = gate_up_proj.dtype
    s13 = torch.cat([shared_gate_proj.reshape(m, I, H), shared_up_proj.reshape(m, I, H)], dim=1).to(dt)
    s2 = shared_down_proj.reshape(H, m, I).permute(1, 0, 2).to(dt)
    packed = pack_experts(torch.cat([gate_up_proj, s13], 0), torch.cat([down_proj, s2], 0), group_size)
    packed.num_shared = m
    return packed


# ---------------------------------------------------------------------------
# the layer
# ---------------------------------------------------------------------------

def select_path(path: str, dtype: torch.dtype, T: int, top_k: int, H: int, E: int, I: int,
                group_size: int = 64) -> str:
    """The FFN path ('decode' or 'prefill') the layer takes for these
    arguments (``phmoe_select_path``); raises when ``path`` cannot run."""
    if path not in _PATHS:
        raise ValueError(f"path must be one of {list(_PATHS)}")
    if dtype not in _DT:
        raise ValueError(f"unsupported dtype {dtype}")
    rc = _lib.load().phmoe_select_path(_PATHS[path], _DT[dtype], T, top_k, H, E, I, group_size)
    _lib.check("phmoe_select_path", rc if rc < 0 else 0)
    return "prefill" if rc == _lib.PATH_PREFILL else "decode"


def workspace_bytes(T: int, H: int, E: int, top_k: int, I: int, path: str = "auto") -> int:
    """Scratch bytes ``moe_layer`` needs for T tokens (``phmoe_workspace_size``)."""
    n = _lib.load().phmoe_workspace_size(T, H, E, top_k, I, _PATHS[path])
    if n == 0:
        raise ValueError("invalid layer dimensions")
    return int(n)


class MoeLayer:
    """One sparse-MoE layer bound to its weights: the weights and options are
    validated once, and each call checks only the activations and reuses the
    bound arguments (the per-call host work of :func:`moe_layer`, which builds
    one of these per call, drops to one C call). Same arguments and results
    as :func:`moe_layer` (single GPU)."""

    def __init__(self, router_weight: torch.Tensor, w13_q: torch.Tensor, w13_scales: torch.Tensor,
                 w2_q: torch.Tensor, w2_scales: torch.Tensor, top_k: int, renormalize: bool = True,
                 group_size: int = 64, *, path: str = "auto", num_shared: int = 0,
                 shared_gate_weight: torch.Tensor | None = None, routed_scale: float = 1.0,
                 scoring: str = "softmax", score_bias: torch.Tensor | None = None, n_group: int = 1,
                 topk_group: int = 1, check_errors: bool = False):
        _need_cuda("router_weight", router_weight)
        _need_dtype("router_weight", router_weight, _DT)
        H = router_weight.shape[-1]
        E, I = check_expert_weights(w13_q, w13_scales, w2_q, w2_scales, H, group_size)
        if num_shared:
            if num_shared < 0 or num_shared >= E:
                raise ValueError("num_shared must be in [0, number of packed experts)")
            E -= num_shared
            if shared_gate_weight is not None:
                _need_cuda("shared_gate_weight", shared_gate_weight)
                if shared_gate_weight.numel() != H or shared_gate_weight.dtype != router_weight.dtype:
                    raise ValueError("shared_gate_weight must hold H values of router_weight's dtype")
        elif shared_gate_weight is not None:
            raise ValueError("shared_gate_weight needs num_shared > 0")
        if scoring not in _SCORING:
            raise ValueError(f"scoring must be one of {list(_SCORING)}")
        if score_bias is not None:
            _need_cuda("score_bias", score_bias)
            _need_dtype("score_bias", score_bias, (torch.float32,))
            _need_shape("score_bias", score_bias, (E,))
        _need_shape("router_weight", router_weight, (E, H))
        if path not in _PATHS:
            raise ValueError(f"path must be one of {list(_PATHS)}")
        self.H, self.E, self.I, self.top_k, self.group_size = H, E, I, top_k, group_size
        self.device = router_weight.device
        self.num_shared = num_shared
        # keep the tensors alive for as long as the bound pointers are used
        self._tensors = (router_weight, w13_q, w13_scales, w2_q, w2_scales, shared_gate_weight, score_bias)
        lib = _lib.load()
        self._extended = (bool(num_shared) or routed_scale != 1.0 or scoring != "softmax" or score_bias is not None
                          or n_group > 1)
        pc = _PATHS[path]
        head = (_ptr(router_weight), _DT[router_weight.dtype], _ptr(w13_q), _ptr(w13_scales), _ptr(w2_q),
                _ptr(w2_scales))
        if self._extended:
            self._name = "phmoe_moe_layer_ex"
            self._size = lambda T: lib.phmoe_workspace_size_ex(T, H, E, top_k, I, num_shared, pc)
            self._tail = (H, E, top_k, I, group_size, int(bool(renormalize)), _SCORING[scoring], _ptr(score_bias),
                          n_group, topk_group, num_shared, _ptr(shared_gate_weight), float(routed_scale), pc)
        else:
            self._name = "phmoe_moe_layer"
            self._size = lambda T: lib.phmoe_workspace_size(T, H, E, top_k, I, pc)
            self._tail = (H, E, top_k, I, group_size, int(bool(renormalize)), pc)
        self._fn = getattr(lib, self._name)
        self._head = head
        self._need: dict[int, int] = {}
        # check_errors: after every call wait for the device and raise
        # DeviceError if a kernel raised the device error word (a debugging
        # aid: it synchronises, and does not work inside stream capture)
        self.check_errors = bool(check_errors)

    def workspace_bytes(self, T: int) -> int:
        n = self._need.get(T)
        if n is None:
            n = self._need[T] = self._size(T)
        return n

    def __call__(self, hidden_states: torch.Tensor, out: torch.Tensor | None = None, return_routing: bool = False,
                 workspace: torch.Tensor | None = None):
        x = hidden_states
        if not isinstance(x, torch.Tensor) or x.device != self.device:
            raise ValueError(f"hidden_states must be a CUDA tensor on {self.device}; phantom_moe has no CPU path")
        if x.dtype not in _DT:
            raise TypeError(f"hidden_states must be bf16 or fp32 (got {x.dtype})")
        if not x.is_contiguous():
            raise ValueError("hidden_states must be contiguous")
        shape = x.shape
        H = self.H
        if shape[-1] != H:
            raise ValueError(f"hidden_states must end in H={H} (got {tuple(shape)})")
        T = x.numel() // H
        dev = x.device
        if out is None:
            out = torch.empty(shape, dtype=x.dtype, device=dev)
        elif (not isinstance(out, torch.Tensor) or out.device != dev or out.dtype != x.dtype
              or out.numel() != T * H or not out.is_contiguous()):
            raise ValueError("out must be a contiguous CUDA tensor matching hidden_states in dtype and size")
        idx = wts = None
        if return_routing:
            idx = torch.empty(T, self.top_k, dtype=torch.int32, device=dev)
            wts = torch.empty(T, self.top_k, dtype=torch.float32, device=dev)
        need = self.workspace_bytes(T)
        if workspace is None:
            ws = WORKSPACE.get(dev, need)
        else:
            _need_cuda("workspace", workspace)
            _need_dtype("workspace", workspace, (torch.uint8,))
            if workspace.numel() < need:
                raise ValueError(f"workspace needs {need} bytes (got {workspace.numel()})")
            ws = workspace
        rc = self._fn(x.data_ptr(), _DT[x.dtype], *self._head, T, *self._tail, out.data_ptr(), _ptr(idx), _ptr(wts),
                      ws.data_ptr(), ws.numel(), _stream())
        if rc:
            _lib.check(self._name, rc)
        if self.check_errors:
            check_device_errors()
        out = out.reshape(shape)
        if return_routing:
            return out, idx, wts
        return out

    def graphed(self, x: torch.Tensor, out: torch.Tensor):
        """Capture this layer on the fixed buffers ``x`` -> ``out`` into a CUDA
        graph and return a function that replays it on the current stream (one
        launch instead of one per kernel). Refill ``x`` in place between
        replays; ``x`` and ``out`` must stay allocated while the graph is used.
        The capture first runs the layer once on ``x``'s current contents, so
        ``x`` should hold valid activations (zeros will do), not uninitialised
        memory."""
        side = torch.cuda.Stream(device=x.device)
        side.wait_stream(torch.cuda.current_stream(x.device))
        with torch.cuda.stream(side):  # warm-up outside the capture (workspace, tensor maps)
            self(x, out=out)
        torch.cuda.current_stream(x.device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self(x, out=out)
        keep = (graph, x, out)

        def replay():
            keep[0].replay()
            return keep[2]
        return replay


def moe_layer(hidden_states: torch.Tensor, router_weight: torch.Tensor, w13_q: torch.Tensor,
              w13_scales: torch.Tensor, w2_q: torch.Tensor, w2_scales: torch.Tensor, top_k: int,
              renormalize: bool = True, group_size: int = 64, ep_group=None, *,
              path: str = "auto", return_routing: bool = False, out: torch.Tensor | None = None,
              workspace: torch.Tensor | None = None, num_shared: int = 0,
              shared_gate_weight: torch.Tensor | None = None, routed_scale: float = 1.0,
              scoring: str = "softmax", score_bias: torch.Tensor | None = None, n_group: int = 1,
              topk_group: int = 1, check_errors: bool = False):
    """Sparse-MoE layer: router -> dispatch -> grouped int4 SwiGLU FFN -> combine.

    ``hidden_states`` is ``[T, H]`` or ``[B, S, H]`` (bf16 or fp32); the result
    has the same shape and dtype. ``router_weight`` is ``[E, H]`` (bf16/fp32).
    With ``ep_group`` (a ``torch.distributed`` group of P > 1 ranks) the expert
    tensors hold this rank's E/P experts and tokens are exchanged with NCCL
    all-to-all (see :mod:`phantom_moe.ep`).

    ``return_routing`` adds ``(topk_idx int32[T,k], topk_w fp32[T,k])``.
    ``workspace`` (uint8 CUDA tensor of at least ``workspace_bytes(...)``)
    overrides the per-stream cached scratch buffer.

    Shared experts (Qwen2-MoE, DeepSeek): with ``num_shared = m > 0`` the
    expert tensors hold E routed experts followed by the m slices of the
    shared expert (:func:`pack_experts_shared`); the router picks among the
    first E, every token also goes to the m slices with weight
    ``sigmoid(x . shared_gate_weight)`` (``[H]`` or ``[1, H]``; 1 when None),
    and the routed weights are multiplied by ``routed_scale``.

    DeepSeek-V3 routing: ``scoring="sigmoid"`` with an optional fp32
    ``score_bias [E]`` (``e_score_correction_bias``, used for the choice
    only) and group-limited selection (``n_group`` groups, the
    ``topk_group`` best kept); see ``phmoe_router_ex`` in ``phmoe.h``.

    ``check_errors``: wait for the device after the call and raise
    :class:`DeviceError` if a kernel raised the device error word (see
    :func:`check_device_errors`).
    """
    if ep_group is not None:
        from . import ep as _ep
        if _ep.ep_world_size(ep_group) > 1:
            if num_shared:
                raise NotImplementedError("shared experts are not supported with expert parallelism")
            return _ep.moe_layer_ep(hidden_states, router_weight, w13_q, w13_scales, w2_q, w2_scales,
                                    top_k, renormalize, group_size, ep_group, path=path,
                                    return_routing=return_routing)
    _need_cuda("hidden_states", hidden_states)
    layer = MoeLayer(router_weight, w13_q, w13_scales, w2_q, w2_scales, top_k, renormalize, group_size, path=path,
                     num_shared=num_shared, shared_gate_weight=shared_gate_weight, routed_scale=routed_scale,
                     scoring=scoring, score_bias=score_bias, n_group=n_group, topk_group=topk_group,
                     check_errors=check_errors)
    return layer(hidden_states, out=out, return_routing=return_routing, workspace=workspace)
