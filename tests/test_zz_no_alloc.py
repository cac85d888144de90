"""phmoe_moe_layer_noalloc: the layer with the library's static scratch
instead of a caller workspace, called through the C ABI.

Named so pytest collects it last; it must also pass alone in a fresh process.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import phantom_moe
from phantom_moe import _lib
from oracle import moe_oracle as O

STATIC_SCRATCH_BYTES = 16 << 20  # PHMOE_STATIC_SCRATCH_BYTES in include/phmoe.h
DT = {torch.float32: 0, torch.bfloat16: 1}


def _ptr(t):
    return None if t is None else t.data_ptr()


def _weights(E, H, I, G, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    wr = torch.randn(E, H, generator=g, device=dev) * 0.02
    w13 = torch.randn(E, 2 * I, H, generator=g, device=dev) * 0.02
    w2 = torch.randn(E, H, I, generator=g, device=dev) * 0.02
    w13_q, w13_s = phantom_moe.quantize_int4(w13, G)
    w2_q, w2_s = phantom_moe.quantize_int4(w2, G)
    return wr, w13_q, w13_s, w2_q, w2_s


def _layer_args(x, wr, w13_q, w13_s, w2_q, w2_s, k, I, G, out, idx, wts):
    T, H = x.shape
    E = wr.shape[0]
    return [_ptr(x), DT[x.dtype], _ptr(wr), DT[wr.dtype], _ptr(w13_q), _ptr(w13_s), _ptr(w2_q),
            _ptr(w2_s), T, H, E, k, I, G, 1, 0, _ptr(out), _ptr(idx), _ptr(wts)]


def test_noalloc_rejects_sizes_beyond_static_scratch():
    """Host-side check only: nothing is launched, so no GPU is needed."""
    lib = phantom_moe.load_library()
    T, H, E, k, I = 1024, 2048, 128, 8, 768
    assert lib.phmoe_workspace_size(T, H, E, k, I, 0) > STATIC_SCRATCH_BYTES
    st = lib.phmoe_moe_layer_noalloc(None, 1, None, 1, None, None, None, None, T, H, E, k, I, 64, 1, 0,
                                     None, None, None, None)
    assert st == -3  # PHMOE_ERR_WORKSPACE
    assert b"static scratch" in lib.phmoe_last_error()
    # the largest Qwen3-shaped decode batch that fits, as the header states
    assert lib.phmoe_workspace_size(184, H, E, k, I, 0) <= STATIC_SCRATCH_BYTES
    assert lib.phmoe_workspace_size(185, H, E, k, I, 0) > STATIC_SCRATCH_BYTES


def _run_pair(lib, x, wr, w13_q, w13_s, w2_q, w2_s, k, I, G, stream):
    """One call through phmoe_moe_layer with a fresh workspace and one through
    phmoe_moe_layer_noalloc; returns both results (out, idx, wts)."""
    T, H = x.shape
    E = wr.shape[0]
    dev = x.device
    ws = torch.empty(lib.phmoe_workspace_size(T, H, E, k, I, 0), dtype=torch.uint8, device=dev)
    assert ws.numel() <= STATIC_SCRATCH_BYTES
    ref = (torch.empty_like(x), torch.empty(T, k, dtype=torch.int32, device=dev),
           torch.empty(T, k, dtype=torch.float32, device=dev))
    _lib.call("phmoe_moe_layer", *_layer_args(x, wr, w13_q, w13_s, w2_q, w2_s, k, I, G, *ref),
              _ptr(ws), ctypes.c_size_t(ws.numel()), stream)
    got = (torch.full_like(x, float("nan")), torch.full((T, k), -7, dtype=torch.int32, device=dev),
           torch.full((T, k), float("nan"), dtype=torch.float32, device=dev))
    _lib.call("phmoe_moe_layer_noalloc", *_layer_args(x, wr, w13_q, w13_s, w2_q, w2_s, k, I, G, *got), stream)
    torch.cuda.synchronize(dev)
    return ref, got


def _assert_same(ref, got, what):
    """Both entries run the same kernels on the same inputs, and the layer is
    deterministic: every output bit must agree (a scratch-aliasing bug that
    changes a few rows would show here)."""
    (ro, ri, rw), (go, gi, gw) = ref, got
    assert torch.equal(gi, ri), what
    assert torch.equal(gw, rw), what
    assert torch.equal(go, ro), (what, int((go != ro).sum()))
    mx, mr = O.parity_stats(go.float().cpu().numpy(), ro.float().cpu().numpy())
    assert np.isfinite(mx) and mx <= O.MAX_ABS_TOL and mr <= O.MEAN_REL_TOL, (what, mx, mr)


@pytest.mark.gpu
@pytest.mark.parametrize("T,H,E,k,I,G,dtype", [
    (64, 2048, 128, 8, 768, 64, torch.bfloat16),   # Qwen3-30B-A3B shape, decode
    (13, 512, 32, 4, 256, 32, torch.float32),
])
def test_noalloc_matches_workspace_entry_two_calls(cuda_device, T, H, E, k, I, G, dtype):
    dev = cuda_device
    lib = _lib.load()
    wr, w13_q, w13_s, w2_q, w2_s = _weights(E, H, I, G, 5, dev)
    wr = wr.to(dtype)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call in range(2):  # two calls in a row: the second runs over the first's leftovers
        gx = torch.Generator(device="cpu").manual_seed(100 + call)
        x = torch.randn(T, H, generator=gx).to(dtype).to(dev)
        _assert_same(*_run_pair(lib, x, wr, w13_q, w13_s, w2_q, w2_s, k, I, G, stream), f"call {call}")
    assert lib.phmoe_device_error(1) == 0


@pytest.mark.gpu
def test_noalloc_layout_changes_between_calls(cuda_device):
    """A call that fills the scratch almost to its limit (184 tokens at the
    Qwen3 shape), then smaller calls with other T, E and k: each sub-buffer
    moves between calls and sits over the previous call's leftovers, which
    nothing may depend on."""
    dev = cuda_device
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    shapes = [(184, 2048, 128, 8, 768, 64, 11), (37, 2048, 64, 6, 768, 64, 12), (5, 1024, 16, 2, 512, 32, 13),
              (184, 2048, 128, 8, 768, 64, 14)]
    for n, (T, H, E, k, I, G, seed) in enumerate(shapes):
        wr, w13_q, w13_s, w2_q, w2_s = _weights(E, H, I, G, seed, dev)
        wr = wr.to(torch.bfloat16)
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(200 + n)).to(torch.bfloat16).to(dev)
        _assert_same(*_run_pair(lib, x, wr, w13_q, w13_s, w2_q, w2_s, k, I, G, stream), (T, E, k))
    assert lib.phmoe_device_error(1) == 0
