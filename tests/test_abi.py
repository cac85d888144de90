"""The C-ABI library loads and exports every symbol include/phmoe.h declares;
host-side argument checks reject bad calls before any CUDA work (no GPU needed)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from conftest import REPO

import phantom_moe
from phantom_moe import _lib

HEADER = REPO / "include" / "phmoe.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(phmoe_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    return phantom_moe.load_library()


def test_library_built_in_tree():
    assert _lib.LIB_PATH.exists(), "run __graft_entry__.build() first"
    assert "solution-is-all-you-need_b200" in str(_lib.LIB_PATH)


def test_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), f"{n} declared in phmoe.h but not exported"
    assert set(names) <= set(_lib.SIGNATURES), f"ctypes table misses {set(names) - set(_lib.SIGNATURES)}"


def test_version_and_status(lib):
    assert lib.phmoe_version() >= 100
    assert lib.phmoe_status_string(0) == b"ok"
    assert lib.phmoe_status_string(-4) == b"CUDA error"
    assert lib.phmoe_status_string(12345) == b"unknown status"


def test_workspace_size(lib):
    n = lib.phmoe_workspace_size(16, 2048, 128, 8, 768, 0)
    R = 16 * 8
    assert n >= R * 768 * 4 + R * 2048 * 4 + 16 * 128 * 4
    assert n % 256 == 0
    assert lib.phmoe_workspace_size(-1, 2048, 128, 8, 768, 0) == 0
    assert lib.phmoe_workspace_size(16, 2048, 128, 8, 768, 9) == 0
    assert lib.phmoe_workspace_size(0, 2048, 128, 8, 768, 0) > 0


@pytest.mark.parametrize("T,H,E,k,status", [
    (-1, 2048, 128, 8, _lib.PHMOE_ERR_INVALID_ARG),
    (4, 2047, 128, 8, _lib.PHMOE_ERR_INVALID_ARG),
    (4, 2048, 0, 1, _lib.PHMOE_ERR_INVALID_ARG),
    (4, 2048, 2000, 8, _lib.PHMOE_ERR_INVALID_ARG),
    (4, 2048, 8, 9, _lib.PHMOE_ERR_INVALID_ARG),
    (4, 2048, 64, 33, _lib.PHMOE_ERR_INVALID_ARG),
])
def test_router_rejects_bad_dims(lib, T, H, E, k, status):
    rc = lib.phmoe_router(None, 1, None, 1, T, H, E, k, 1, None, None, None, None, None)
    assert rc == status
    assert lib.phmoe_last_error()


def test_router_rejects_null_and_misaligned(lib):
    assert lib.phmoe_router(None, 1, None, 1, 4, 256, 8, 2, 1, None, None, None, None, None) == \
        _lib.PHMOE_ERR_INVALID_ARG
    buf = (ctypes.c_char * 4096)()
    base = ctypes.addressof(buf)
    odd = base + (16 - base % 16) + 2
    rc = lib.phmoe_router(odd, 1, odd, 1, 4, 256, 8, 2, 1, odd, None, odd, odd, None)
    assert rc == _lib.PHMOE_ERR_ALIGNMENT


def test_layer_rejects_bad_group_and_path(lib):
    args = [None, 1, None, 1, None, None, None, None, 4, 2048, 128, 8, 768]
    assert lib.phmoe_moe_layer(*args, 48, 1, 0, None, None, None, None, 0, None) == _lib.PHMOE_ERR_UNSUPPORTED
    assert lib.phmoe_moe_layer(*args, 64, 1, 7, None, None, None, None, 0, None) == _lib.PHMOE_ERR_INVALID_ARG
    # T = 0 is a valid no-op
    rc = lib.phmoe_moe_layer(None, 1, None, 1, None, None, None, None, 0, 2048, 128, 8, 768, 64, 1, 0,
                             None, None, None, None, 0, None)
    assert rc == 0


def test_layer_rejects_small_workspace(lib):
    buf = (ctypes.c_char * 8192)()
    base = ctypes.addressof(buf)
    p = base + (256 - base % 256)
    rc = lib.phmoe_moe_layer(p, 1, p, 1, p, p, p, p, 4, 2048, 128, 8, 768, 64, 1, 0, p, None, None, p, 16, None)
    assert rc == _lib.PHMOE_ERR_WORKSPACE
    assert b"workspace needs" in lib.phmoe_last_error()


def test_quantize_rejects_bad_args(lib):
    assert lib.phmoe_quantize_int4(None, 0, 4, 100, 64, None, None, None) == _lib.PHMOE_ERR_INVALID_ARG
    assert lib.phmoe_quantize_int4(None, 0, 4, 128, 16, None, None, None) == _lib.PHMOE_ERR_UNSUPPORTED
    assert lib.phmoe_quantize_int4(None, 0, 0, 128, 64, None, None, None) == 0


def test_python_layer_rejects_cpu_tensors():
    import torch
    x = torch.zeros(4, 256, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        phantom_moe.moe_layer(x, x[:8], x, x, x, x, 2)
    with pytest.raises(ValueError, match="CUDA"):
        phantom_moe.router(x, x[:8], 2)


def test_host_pipeline_argument_checks():
    with pytest.raises(ValueError, match="at least one layer"):
        phantom_moe.HostPipeline([], 4, 256, device="cuda")
    with pytest.raises(ValueError, match="depth"):
        phantom_moe.HostPipeline([lambda x, out: None], 4, 256, device="cuda", depth=0)
    with pytest.raises(ValueError, match="CUDA device"):
        phantom_moe.HostPipeline([lambda x, out: None], 4, 256, device="cpu")


def test_prefill_rejects_fp32_and_bad_dims(lib):
    args = [None, None, None, None, None, None, None, 4, 4096, 8, 2]
    assert lib.phmoe_expert_ffn_prefill(None, 0, *args, 14336, 64, None, None, None) == _lib.PHMOE_ERR_UNSUPPORTED
    assert lib.phmoe_expert_ffn_prefill(None, 1, *args, 14272, 64, None, None, None) == _lib.PHMOE_ERR_UNSUPPORTED
    assert lib.phmoe_expert_ffn_prefill(None, 1, *args, 14336, 16, None, None, None) == _lib.PHMOE_ERR_UNSUPPORTED
    # the layer with an explicit prefill path and fp32 activations
    rc = lib.phmoe_moe_layer(None, 0, None, 0, None, None, None, None, 4, 4096, 8, 2, 14336, 64, 1, 2,
                             None, None, None, None, 0, None)
    assert rc == _lib.PHMOE_ERR_UNSUPPORTED
