"""Expert-parallel exchange logic (phantom_moe.ep.moe_layer_ep) on CPU gloo
ranks, with the oracle standing in for the CUDA kernels: every rank's output
must equal the single-process layer on the same tokens."""

from __future__ import annotations

import socket

import numpy as np
import pytest
import torch

from ep_workers import DIMS, OracleOps, gloo_worker, make_case
from oracle import moe_oracle as O


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _single_process(xs, wr, packed):
    H, E, k, I, G = DIMS
    ops = OracleOps()
    x = torch.cat(xs)
    idx, w = ops.router(x, wr, k, True)
    offsets, row_token, inv, active = ops.dispatch(idx, E)
    y = ops.ffn(x, row_token, offsets, active, *packed, G)
    return ops.combine(y, inv, w, torch.float32).numpy(), idx.numpy()


@pytest.mark.parametrize("world,case", [(2, "ragged"), (4, "ragged"), (2, "skew"), (4, "skew")])
def test_ep_gloo_matches_single_process(tmp_path, world, case):
    torch.multiprocessing.start_processes(gloo_worker, args=(world, _free_port(), case, str(tmp_path)),
                                          nprocs=world, join=True, start_method="spawn")
    H, E, k, I, G = DIMS
    xs, wr, packed = make_case(case, world)
    ref, ref_idx = _single_process(xs, wr, packed)
    full = O.moe_layer_reference_packed(torch.cat(xs).numpy(), wr.numpy(), *(t.numpy() for t in packed), k, G)[0]
    res = [dict(np.load(tmp_path / f"rank{r}.npz")) for r in range(world)]
    t0 = 0
    for r in range(world):
        T = xs[r].shape[0]
        got = res[r]["out"]
        assert got.shape == (T, H)
        assert np.array_equal(res[r]["idx"], ref_idx[t0:t0 + T])
        np.testing.assert_allclose(got, ref[t0:t0 + T], rtol=1e-5, atol=1e-6)
        if T:
            mx, mr = O.parity_stats(got, full[t0:t0 + T])
            assert mx <= O.MAX_ABS_TOL and mr <= O.MEAN_REL_TOL
        t0 += T
    send = np.stack([x["send"] for x in res])  # [src, dst]
    recv = np.stack([x["recv"] for x in res])  # [dst, src]
    assert np.array_equal(send, recv.T)
    assert send.sum() == sum(x.shape[0] for x in xs) * k
    if case == "skew":  # the last rank's experts take every token's first picks
        per = E // world
        assert recv[-1].sum() >= sum(x.shape[0] for x in xs) * min(k, per)
