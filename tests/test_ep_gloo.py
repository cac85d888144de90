"""Expert-parallel exchange logic (phantom_moe.ep.moe_layer_ep) on CPU gloo
ranks, with the oracle standing in for the CUDA kernels: every rank's output
must equal the single-process layer on the same tokens."""

from __future__ import annotations

import socket

import numpy as np
import pytest
import torch

from ep_workers import DIMS, OracleOps, gloo_worker, make_case, replica_plan
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


@pytest.mark.parametrize("world,case,fixed", [(2, "ragged", False), (4, "ragged", False), (2, "skew", False),
                                              (4, "skew", False), (2, "ragged", True), (4, "skew", True)])
def test_ep_gloo_matches_single_process(tmp_path, world, case, fixed):
    """fixed: the equal-split all-to-all (fixed_capacity) instead of the
    host-counted one; the same output bit for bit."""
    torch.multiprocessing.start_processes(gloo_worker, args=(world, _free_port(), case, str(tmp_path), False, fixed),
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


@pytest.mark.parametrize("world", [2, 4])
def test_ep_gloo_replicated_placement(tmp_path, world):
    """Hot experts copied onto other ranks (plan_replicas): the same output,
    and the busiest rank receives fewer rows than without copies."""
    torch.multiprocessing.start_processes(gloo_worker, args=(world, _free_port(), "skew", str(tmp_path), True),
                                          nprocs=world, join=True, start_method="spawn")
    H, E, k, I, G = DIMS
    xs, wr, packed = make_case("skew", world)
    ref, ref_idx = _single_process(xs, wr, packed)
    res = [dict(np.load(tmp_path / f"rank{r}.npz")) for r in range(world)]
    t0 = 0
    for r in range(world):
        T = xs[r].shape[0]
        assert np.array_equal(res[r]["idx"], ref_idx[t0:t0 + T])
        # the checker's numpy FFN rounds by batch composition (the CUDA kernels do not)
        np.testing.assert_allclose(res[r]["out"], ref[t0:t0 + T], rtol=1e-5, atol=1e-6)
        t0 += T
    send = np.stack([x["send"] for x in res])
    recv = np.stack([x["recv"] for x in res])
    assert np.array_equal(send, recv.T)
    total = sum(x.shape[0] for x in xs) * k
    assert send.sum() == total
    pl = replica_plan(xs, wr, world)
    assert pl.slots_per_rank > E // world                  # copies were placed
    per = E // world
    assert recv.sum(1).max() < total and recv[-1].sum() < total * min(k, per) / k  # the hot rank is relieved


def test_placement_home_is_identity_and_checks():
    from phantom_moe import ep
    pl = ep.home_placement(8, 4)
    for s in range(4):
        assert pl.virtual_map(s).tolist() == list(range(8))
    assert pl.local_experts(3) == [6, 7]
    with pytest.raises(ValueError, match="at least one rank"):
        ep.Placement([[0, 1], [2]], 4)
    with pytest.raises(ValueError, match="at most once"):
        ep.Placement([[0, 0], [1]], 2)


def test_plan_replicas_spreads_a_zipf_load():
    from phantom_moe import ep
    E, world = 16, 4
    load = [1000.0 / (e + 1) ** 1.2 for e in range(E)]        # hot experts 0.. all on rank 0
    home = ep.home_placement(E, world)
    pl = ep.plan_replicas(load, world, extra_slots=2)
    assert max(pl.rank_loads(load)) < 0.6 * max(home.rank_loads(load))
    assert abs(sum(pl.rank_loads(load)) - sum(load)) < 1e-6  # rows are moved, not lost
    assert all(len(s) <= E // world + 2 for s in pl.slots)
    assert len(pl.copies(0)) >= 2                             # the hottest expert is copied
    for s in range(world):                                     # each source uses one copy of each expert
        vm = pl.virtual_map(s).tolist()
        S = pl.slots_per_rank
        assert all(pl.slots[v // S][v % S] == e for e, v in enumerate(vm))
    w = torch.arange(E * 3, dtype=torch.float32).view(E, 3)
    (lw,) = pl.local_weights(1, w)
    assert lw.shape == (pl.slots_per_rank, 3)
    assert torch.equal(lw[0], w[pl.slots[1][0]])
