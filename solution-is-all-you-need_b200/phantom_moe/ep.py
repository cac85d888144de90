"""Expert-parallel sparse-MoE layer: experts sharded over the ranks of a
``torch.distributed`` group, tokens exchanged with all-to-all (NCCL over
NVLink on B200s).

PHANTOM has no expert parallelism; this follows the layer semantics of
transformers' ``Qwen3MoeSparseMoeBlock.forward`` (modeling_qwen3_moe.py:
281-286) with the experts spread over P GPUs.

Sharding: with E experts and P ranks (E % P == 0) rank r holds experts
``[r*E/P, (r+1)*E/P)`` (see :func:`shard_range`); the router weight is
replicated and every rank routes its own tokens (data parallel). One layer
call on each rank:

1. router + dispatch of the rank's own T tokens. Rows come out expert-major
   (token order inside an expert); since a rank's experts are contiguous,
   that order is also destination-rank-major.
2. all-to-all of the per-expert row counts ``[P, E/P]`` int32, then one
   device-to-host copy of the send and receive counts: the split sizes the
   row all-to-alls need (the only host synchronisation of the layer).
3. rows packed in that order (:func:`phantom_moe.gather_rows`) and sent with
   an all-to-all.
4. the receiver labels arrived rows with their local expert (from the
   counts), dispatches them by expert (stable in arrival order), runs the
   grouped FFN and gathers its fp32 rows back into arrival order.
5. the reverse all-to-all returns the fp32 rows to their source, which
   combines them with its own routing weights in slot order.

Per row the FFN result does not depend on which other rows share the batch,
and the return path carries fp32, so the output equals the single-GPU layer's
bit for bit.

Every rank issues the same collectives in the same order whatever its token
count (zero included). The compute steps go through an ``ops`` object
(:class:`CudaOps` for the product path), so the exchange logic can be tested
on CPU ranks with a checker's ops.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from . import layer as _layer


def ep_world_size(group) -> int:
    import torch.distributed as dist
    if group is None or not dist.is_available() or not dist.is_initialized():
        return 1
    return dist.get_world_size(group)


def shard_range(num_experts: int, world: int, rank: int) -> tuple[int, int]:
    """Experts ``[lo, hi)`` held by ``rank`` of ``world`` ranks."""
    if world < 1 or num_experts % world:
        raise ValueError(f"{num_experts} experts do not split evenly over {world} ranks")
    per = num_experts // world
    return rank * per, (rank + 1) * per


@dataclass
class Placement:
    """Which global experts each rank holds, replicas of hot experts included.

    ``slots[r]`` lists rank r's experts (its home shard first, then the
    copies it hosts); every rank is padded to ``S = max len(slots[r])`` local
    slots, so local slot j of rank r is the virtual expert ``r * S + j``.
    Each source rank sends all its rows for expert e to one copy
    (:meth:`copy_for`): its own copy when it holds one (no NVLink traffic),
    otherwise the copies in turn over the sources that hold none, starting
    after the home copy. The rows are then dispatched by virtual expert,
    which keeps them destination-rank-major, so the exchange is unchanged. A
    row's result does not depend on which copy computes it, so the layer
    output is the same bit for bit."""
    slots: list
    num_experts: int

    def __post_init__(self):
        held = sorted({e for s in self.slots for e in s})
        if held != list(range(self.num_experts)):
            raise ValueError("every expert must be held by at least one rank")
        for s in self.slots:
            if len(set(s)) != len(s):
                raise ValueError("a rank holds an expert at most once")
        self._copies = {e: [] for e in range(self.num_experts)}
        for r, s in enumerate(self.slots):
            for j, e in enumerate(s):
                self._copies[e].append((r, j))

    @property
    def world(self) -> int:
        return len(self.slots)

    @property
    def slots_per_rank(self) -> int:
        return max(len(s) for s in self.slots)

    def copies(self, e: int) -> list:
        """(rank, slot) of every copy of expert e, in rank order."""
        return list(self._copies[e])

    def copy_for(self, e: int, source_rank: int) -> tuple:
        """(rank, slot) of the copy of expert e that ``source_rank`` uses."""
        c = self._copies[e]
        for r, j in c:
            if r == source_rank:
                return r, j
        holders = {r for r, _ in c}
        others = [q for q in range(self.world) if q not in holders]
        return c[(others.index(source_rank) + 1) % len(c)]

    def virtual_map(self, source_rank: int) -> torch.Tensor:
        """int32 [E]: the virtual expert that ``source_rank`` sends expert e's rows to."""
        S = self.slots_per_rank
        vm = []
        for e in range(self.num_experts):
            r, j = self.copy_for(e, source_rank)
            vm.append(r * S + j)
        return torch.tensor(vm, dtype=torch.int32)

    def local_experts(self, rank: int) -> list:
        """Global expert of each of rank's S local slots (padding repeats the
        rank's last expert; padded slots never receive rows)."""
        s = list(self.slots[rank])
        return s + [s[-1]] * (self.slots_per_rank - len(s))

    def local_weights(self, rank: int, *tensors):
        """Rank's slot-stacked copies of full per-expert tensors ``[E, ...]``."""
        idx = torch.tensor(self.local_experts(rank), dtype=torch.long)
        return tuple(t.index_select(0, idx.to(t.device)).contiguous() for t in tensors)

    def rank_loads(self, expert_load) -> list:
        """Rows each rank receives when expert e receives expert_load[e] rows
        spread evenly over the source ranks."""
        P = self.world
        load = [0.0] * P
        for e in range(self.num_experts):
            for s in range(P):
                load[self.copy_for(e, s)[0]] += float(expert_load[e]) / P
        return load


def home_placement(num_experts: int, world: int) -> Placement:
    """No replicas: rank r holds :func:`shard_range`'s experts."""
    return Placement([list(range(*shard_range(num_experts, world, r))) for r in range(world)], num_experts)


def plan_replicas(expert_load, world: int, extra_slots: int) -> Placement:
    """Greedy replication of hot experts: starting from the home shards, up to
    ``extra_slots`` copies per rank are added, each time copying the expert
    whose copies carry the most rows onto the least-loaded rank that has room
    and does not hold it yet, while that improves the rank loads sorted from
    the busiest down (compared in that order, so ties at the top still make
    progress). ``expert_load[e]``: rows routed to expert e (e.g. counted over
    a batch)."""
    E = len(expert_load)
    pl = home_placement(E, world)
    base = len(pl.slots[0])

    def key(p):
        return [round(v, 6) for v in sorted(p.rank_loads(expert_load), reverse=True)]

    while True:
        loads = pl.rank_loads(expert_load)
        cur = key(pl)
        best = None
        for e in sorted(range(E), key=lambda q: -float(expert_load[q]) / len(pl.copies(q))):
            holders = {r for r, _ in pl.copies(e)}
            room = [r for r in range(world) if r not in holders and len(pl.slots[r]) < base + extra_slots]
            if not room:
                continue
            r = min(room, key=lambda q: (loads[q], q))
            trial = Placement([list(s) + ([e] if i == r else []) for i, s in enumerate(pl.slots)], E)
            if key(trial) < cur:
                best = trial
                break
        if best is None:
            return pl
        pl = best


class CudaOps:
    """The product's compute steps: the libphmoe CUDA kernels."""

    def router(self, x, router_weight, top_k, renormalize):
        idx, w, _ = _layer.router(x, router_weight, top_k, renormalize)
        return idx, w

    def dispatch(self, idx, num_experts):
        return _layer.dispatch(idx, num_experts)

    def gather(self, src, index):
        return _layer.gather_rows(src, index)

    def ffn(self, x, row_token, offsets, active, w13_q, w13_scales, w2_q, w2_scales, group_size, path="auto"):
        """Grouped FFN over this rank's arrived rows; ``path`` as in
        :func:`phantom_moe.moe_layer`, 'auto' deciding on the local batch."""
        E, I = w13_q.shape[0], w13_q.shape[1] // 2
        chosen = _layer.select_path(path, x.dtype, x.shape[0], 1, x.shape[1], E, I, group_size)
        ffn = _layer.expert_ffn_prefill if chosen == "prefill" else _layer.expert_ffn_decode
        return ffn(x, row_token, offsets, active, w13_q, w13_scales, w2_q, w2_scales, top_k=1,
                   group_size=group_size)

    def combine(self, y, inv, topk_w, out_dtype):
        return _layer.combine(y, inv, topk_w, out_dtype)


_CUDA_OPS = CudaOps()


@dataclass
class Routed:
    """A rank's routing of its own tokens."""
    idx: torch.Tensor        # int32 [T, k]
    w: torch.Tensor          # fp32 [T, k]
    offsets: torch.Tensor    # int32 [E + 1], rows per expert (expert-major)
    row_token: torch.Tensor  # int32 [T*k]
    inv: torch.Tensor        # int32 [T, k], row of each (token, slot)
    counts: torch.Tensor     # int32 [E], rows per expert = per (destination rank, local expert)


def route_local(x, router_weight, top_k, renormalize, ops, vmap=None, num_virtual=None) -> Routed:
    """Router + dispatch of this rank's tokens. With ``vmap`` (int32 [E],
    :meth:`Placement.virtual_map`) the rows are grouped by virtual expert
    (``num_virtual`` = ranks x slots) instead of by expert."""
    E = router_weight.shape[0]
    idx, w = ops.router(x, router_weight, top_k, renormalize)
    if vmap is None:
        offsets, row_token, inv, _ = ops.dispatch(idx, E)
    else:
        vidx = vmap.to(idx.device)[idx.long()].to(torch.int32)
        offsets, row_token, inv, _ = ops.dispatch(vidx, num_virtual)
    counts = (offsets[1:] - offsets[:-1]).to(torch.int32)
    return Routed(idx, w, offsets, row_token, inv, counts)


def rows_per_rank(counts_host: torch.Tensor, world: int) -> list[int]:
    """Per-rank row totals from per-(rank, local expert) counts."""
    return counts_host.view(world, -1).sum(1).tolist()


def arrived_expert_ids(recv_counts: torch.Tensor, world: int, total: int) -> torch.Tensor:
    """Local expert of each arrived row: source-major blocks, each expert-major."""
    per = recv_counts.numel() // world
    ids = torch.arange(per, dtype=torch.int32, device=recv_counts.device).repeat(world)
    return torch.repeat_interleave(ids, recv_counts.to(torch.int64), output_size=total).to(torch.int32)


def expert_compute(recv_x, recv_counts, world, w13_q, w13_scales, w2_q, w2_scales, group_size, ops, path="auto"):
    """Grouped FFN over rows that arrived from all ranks; fp32 rows back in
    arrival order."""
    total = recv_x.shape[0]
    per = w13_q.shape[0]
    if total == 0:
        return torch.empty(0, recv_x.shape[1], dtype=torch.float32, device=recv_x.device)
    eid = arrived_expert_ids(recv_counts, world, total)
    offsets, row_token, inv, active = ops.dispatch(eid.view(total, 1), per)
    y = ops.ffn(recv_x, row_token, offsets, active, w13_q, w13_scales, w2_q, w2_scales, group_size, path)
    return ops.gather(y, inv.view(-1))


class PeerExchange:
    """Token exchange in peer memory for :func:`moe_layer_ep` (the
    ``phmoe_ep_*`` entries): every rank of ``group`` allocates one exchange
    region sized for ``max_tokens`` tokens per call, the CUDA IPC handles are
    gathered over ``group``, and each rank maps its peers' regions. Layer calls
    then move rows and results with direct stores over NVLink and epoch flags:
    no host synchronisation and no collective on the data path.

    All ranks must create it together, call the layer the same number of
    times, and :meth:`close` it together (the group is used for the handle
    exchange and for barriers only, so gloo or NCCL both work).

    With ``placement`` (a :class:`Placement`, the same on every rank) each
    rank is sized for ``placement.slots_per_rank`` local expert slots and the
    layer sends every row to the copy the placement assigns
    (``phmoe_ep_create_ex`` / ``phmoe_ep_layer_ex``); the expert tensors then
    hold the rank's slots (:meth:`Placement.local_weights`)."""

    def __init__(self, group, max_tokens: int, top_k: int, hidden_size: int, num_experts: int,
                 dtype: torch.dtype = torch.bfloat16, placement: Placement | None = None):
        import torch.distributed as dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.max_tokens, self.top_k, self.hidden_size, self.num_experts = max_tokens, top_k, hidden_size, num_experts
        self.dtype = dtype
        self.placement = placement
        if placement is not None and (placement.world != self.world or placement.num_experts != num_experts):
            raise ValueError(f"placement is for {placement.num_experts} experts over {placement.world} ranks; "
                             f"the exchange has {num_experts} over {self.world}")
        self._vmap = {}
        self._ctx = ctypes.c_void_p()
        handle = (ctypes.c_char * _lib.EP_HANDLE_BYTES)()
        slots = placement.slots_per_rank if placement is not None else 0
        _lib.call("phmoe_ep_create_ex", self.rank, self.world, max_tokens, top_k, hidden_size, num_experts, slots,
                  _layer._DT[dtype], ctypes.byref(self._ctx), handle)
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        _lib.call("phmoe_ep_connect", self._ctx, b"".join(handles))
        dist.barrier(group=group)
        self._ws = {}

    def workspace(self, device, intermediate_size: int) -> torch.Tensor:
        key = (device.index, intermediate_size)
        if key not in self._ws:
            n = _lib.load().phmoe_ep_workspace_size(self._ctx, intermediate_size)
            self._ws[key] = torch.empty(n, dtype=torch.uint8, device=device)
        return self._ws[key]

    def layer(self, x, router_weight, w13_q, w13_scales, w2_q, w2_scales, renormalize=True, group_size=64,
              path="auto", return_routing=False):
        T, H = x.shape
        I = w13_q.shape[1] // 2
        out = torch.empty_like(x)
        idx = torch.empty(T, self.top_k, dtype=torch.int32, device=x.device) if return_routing else None
        w = torch.empty(T, self.top_k, dtype=torch.float32, device=x.device) if return_routing else None
        ws = self.workspace(x.device, I)
        vmap = None
        if self.placement is not None:
            if w13_q.shape[0] != self.placement.slots_per_rank:
                raise ValueError(f"this rank holds {w13_q.shape[0]} expert slots; the placement has "
                                 f"{self.placement.slots_per_rank} per rank")
            if x.device.index not in self._vmap:
                self._vmap[x.device.index] = self.placement.virtual_map(self.rank).to(x.device)
            vmap = self._vmap[x.device.index]
        _lib.call("phmoe_ep_layer_ex", self._ctx, _layer._ptr(x), _layer._DT[x.dtype], _layer._ptr(router_weight),
                  _layer._DT[router_weight.dtype], _layer._ptr(w13_q), _layer._ptr(w13_scales), _layer._ptr(w2_q),
                  _layer._ptr(w2_scales), T, I, group_size, int(bool(renormalize)), _layer._PATHS[path],
                  _layer._ptr(vmap), _layer._ptr(out), _layer._ptr(idx), _layer._ptr(w), _layer._ptr(ws),
                  ws.numel(), _layer._stream())
        return (out, idx, w) if return_routing else out

    def close(self):
        import torch.distributed as dist
        if self._ctx:
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
            _lib.call("phmoe_ep_destroy", self._ctx)
            self._ctx = ctypes.c_void_p()
            dist.barrier(group=self.group)


def _exchange_fixed(x, rt: Routed, recv_counts, world: int, C: int, w13_q, w13_scales, w2_q, w2_scales,
                    group_size: int, ops, path: str, ep_group):
    """The row exchange with equal split sizes: every rank sends every rank a
    block of C rows (its rows for that rank's experts, then zero rows) and
    gets C fp32 result rows back per block, so the all-to-alls need no split
    sizes from the host and the layer no host synchronisation. C must be at
    least the rows any rank sends to one rank (T * k always is). The padded
    blocks carry world * C rows each way instead of the rows routed."""
    import torch.distributed as dist
    dev = x.device
    per = recv_counts.numel() // world
    off = rt.offsets.to(torch.int64)
    starts = off[0:world * per:per]                                  # first row of each destination block
    ends = off[per:world * per + 1:per]
    pos = torch.arange(world * C, device=dev, dtype=torch.int64)
    d, i = pos // C, pos % C
    src = starts[d] + i
    valid = src < ends[d]
    index = torch.where(valid, rt.row_token.to(torch.int64)[src.clamp(max=max(rt.row_token.numel() - 1, 0))],
                        torch.full_like(src, -1)).to(torch.int32) if rt.row_token.numel() else \
        torch.full((world * C,), -1, dtype=torch.int32, device=dev)
    send_x = ops.gather(x, index)
    recv_x = torch.empty_like(send_x)
    dist.all_to_all_single(recv_x, send_x, group=ep_group)
    # local expert of every arrived row; padding rows get id `per` (dropped by the dispatch)
    rc = recv_counts.view(world, per).to(torch.int64)
    cum = rc.cumsum(1)                                               # [src, per]
    eid = torch.searchsorted(cum, i.view(world, C), right=True).view(-1).to(torch.int32)
    offsets, row_token, inv, active = ops.dispatch(eid.view(world * C, 1), per)
    y = ops.ffn(recv_x, row_token, offsets, active, w13_q, w13_scales, w2_q, w2_scales, group_size, path)
    y_arrived = ops.gather(y, inv.view(-1))                          # arrival order; padding rows zero
    y_back = torch.empty_like(y_arrived)
    dist.all_to_all_single(y_back, y_arrived, group=ep_group)
    # assignment a's row: block of its destination, position inside the block
    rows = rt.inv.to(torch.int64)
    dblk = torch.searchsorted(ends, rows.view(-1), right=True).view_as(rows)
    inv2 = torch.where(rows >= 0, dblk * C + rows - starts[dblk.clamp(max=world - 1)], torch.full_like(rows, -1))
    return ops.combine(y_back, inv2.to(torch.int32), rt.w, x.dtype)


def moe_layer_ep(hidden_states, router_weight, w13_q, w13_scales, w2_q, w2_scales, top_k: int,
                 renormalize: bool = True, group_size: int = 64, ep_group=None, *, path: str = "auto",
                 return_routing: bool = False, ops=None, stats: dict | None = None,
                 exchange: PeerExchange | None = None, placement: Placement | None = None,
                 fixed_capacity: int | None = None):
    """The MoE layer with this rank's expert shard (``w13_q`` etc. hold
    ``E/P`` experts, ``router_weight`` all ``E``). Same result as
    :func:`phantom_moe.moe_layer` on the full layer for this rank's tokens.

    ``path`` selects the FFN kernels on each rank ('auto' decides on the
    rank's arrived rows). ``stats`` (a dict) receives ``send_rows`` / ``recv_rows``: the rows this
    rank sent to / received from each rank (load-imbalance reporting), and
    ``local_experts_hit``: how many of this rank's experts received rows.

    With ``exchange`` (a :class:`PeerExchange` over ``ep_group``) the rows
    move through peer memory inside one library call; otherwise through
    ``torch.distributed.all_to_all_single`` (any backend, the checker's
    ``ops`` included; one device-to-host copy of the counts per call).

    With ``placement`` (a :class:`Placement` over the group's ranks, hot
    experts replicated) the expert tensors hold this rank's
    ``placement.slots_per_rank`` local slots (:meth:`Placement.local_weights`)
    and every rank sends each expert's rows to the copy the placement assigns
    it; with ``exchange`` the placement is the one the exchange was created
    with.

    ``fixed_capacity`` (all-to-all path only): exchange blocks of that many
    rows per rank pair, with equal split sizes, so nothing is copied to the
    host and the layer never synchronises; it must be at least the rows any
    rank sends to one rank (``T * top_k`` of the largest rank batch always
    is, the same value on every rank). The padded blocks move
    ``world * fixed_capacity`` rows each way.
    """
    import torch.distributed as dist
    if exchange is not None and placement is not None and exchange.placement is not placement:
        raise ValueError("pass the placement the PeerExchange was created with")
    if exchange is not None:
        _layer._need_cuda("hidden_states", hidden_states)
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1])
        res = exchange.layer(x, router_weight, w13_q, w13_scales, w2_q, w2_scales, renormalize, group_size, path,
                             return_routing)
        if return_routing:
            return res[0].reshape(shape), res[1], res[2]
        return res.reshape(shape)
    ops = _CUDA_OPS if ops is None else ops
    world = dist.get_world_size(ep_group)  # None: the default group
    shape = hidden_states.shape
    H = shape[-1]
    x = hidden_states.reshape(-1, H)
    E = router_weight.shape[0]
    if placement is None:
        if w13_q.shape[0] * world != E:
            raise ValueError(f"this rank holds {w13_q.shape[0]} experts; {E} experts over {world} ranks "
                             f"needs {E // max(world, 1)} per rank")
        rt = route_local(x, router_weight, top_k, renormalize, ops)
    else:
        S = placement.slots_per_rank
        if placement.world != world or placement.num_experts != E:
            raise ValueError(f"placement is for {placement.num_experts} experts over {placement.world} ranks; "
                             f"this layer has {E} experts over {world} ranks")
        if w13_q.shape[0] != S:
            raise ValueError(f"this rank holds {w13_q.shape[0]} expert slots; the placement has {S} per rank")
        rank = dist.get_rank(ep_group)
        rt = route_local(x, router_weight, top_k, renormalize, ops, placement.virtual_map(rank), world * S)
    V = rt.counts.numel()  # experts (or virtual experts) over all ranks
    recv_counts = torch.empty_like(rt.counts)
    dist.all_to_all_single(recv_counts, rt.counts, group=ep_group)
    if fixed_capacity is not None:
        out = _exchange_fixed(x, rt, recv_counts, world, int(fixed_capacity), w13_q, w13_scales, w2_q, w2_scales,
                              group_size, ops, path, ep_group).reshape(shape)
        if stats is not None:  # (reads the counts on the host: outside any timed loop)
            both = torch.cat([rt.counts, recv_counts]).cpu()
            stats["send_rows"] = rows_per_rank(both[:V], world)
            stats["recv_rows"] = rows_per_rank(both[V:], world)
            stats["local_experts_hit"] = int((both[V:].view(world, -1).sum(0) > 0).sum())
        if return_routing:
            return out, rt.idx, rt.w
        return out
    both = torch.cat([rt.counts, recv_counts]).cpu()
    send_rows = rows_per_rank(both[:V], world)
    recv_rows = rows_per_rank(both[V:], world)
    send_x = ops.gather(x, rt.row_token)
    recv_x = x.new_empty((sum(recv_rows), H))
    dist.all_to_all_single(recv_x, send_x, recv_rows, send_rows, group=ep_group)
    y_arrived = expert_compute(recv_x, recv_counts, world, w13_q, w13_scales, w2_q, w2_scales, group_size, ops,
                               path)
    y_back = y_arrived.new_empty((rt.row_token.numel(), H))
    dist.all_to_all_single(y_back, y_arrived, send_rows, recv_rows, group=ep_group)
    out = ops.combine(y_back, rt.inv, rt.w, x.dtype).reshape(shape)
    if stats is not None:
        stats["send_rows"] = send_rows
        stats["recv_rows"] = recv_rows
        stats["local_experts_hit"] = int((both[V:].view(world, -1).sum(0) > 0).sum())
    if return_routing:
        return out, rt.idx, rt.w
    return out


def moe_layer_ep_emulated(xs, router_weight, shards, top_k: int, renormalize: bool = True,
                          group_size: int = 64, ops=None, path: str = "auto", placement: Placement | None = None):
    """Expert-parallel layer for P ranks emulated in one process (one device):
    ``xs[r]`` are rank r's tokens and ``shards[r]`` its ``(w13_q, w13_scales,
    w2_q, w2_scales)`` (with ``placement``: its slot-stacked local experts).
    The all-to-alls become concatenations, so the steps and data movement of
    :func:`moe_layer_ep` can be checked on one GPU. Returns each rank's
    output."""
    ops = _CUDA_OPS if ops is None else ops
    world = len(xs)
    E = router_weight.shape[0]
    if placement is None:
        per = E // world
        rts = [route_local(x, router_weight, top_k, renormalize, ops) for x in xs]
    else:
        per = placement.slots_per_rank
        rts = [route_local(x, router_weight, top_k, renormalize, ops, placement.virtual_map(s), world * per)
               for s, x in enumerate(xs)]
    counts = [rt.counts.cpu() for rt in rts]
    send_rows = [rows_per_rank(c, world) for c in counts]              # [src][dst]
    packed = [ops.gather(x, rt.row_token) for x, rt in zip(xs, rts)]
    starts = [[sum(send_rows[s][:d]) for d in range(world)] for s in range(world)]
    y_arrived = []
    for d in range(world):
        parts = [packed[s][starts[s][d]:starts[s][d] + send_rows[s][d]] for s in range(world)]
        recv_x = torch.cat(parts)
        recv_counts = torch.cat([rts[s].counts[d * per:(d + 1) * per] for s in range(world)])
        y_arrived.append(expert_compute(recv_x, recv_counts, world, *shards[d], group_size, ops, path))
    outs = []
    for s in range(world):
        parts = []
        for d in range(world):
            first = sum(send_rows[q][d] for q in range(s))
            parts.append(y_arrived[d][first:first + send_rows[s][d]])
        y_back = torch.cat(parts).contiguous()
        outs.append(ops.combine(y_back, rts[s].inv, rts[s].w, xs[s].dtype))
    return outs
