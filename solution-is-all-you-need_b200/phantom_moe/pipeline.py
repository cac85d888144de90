"""Host-resident token batches through MoE layers, copies overlapped with compute.

A serving loop that keeps its token batches in host memory pays, per layer
call, a host->device copy of the batch, the layer, and a device->host copy
of the result. Issued on one stream these three serialise; here they run on
three streams ordered by events, so the input copy of step i+1 and the output
copy of step i-1 proceed while step i computes, and the host never blocks
between steps.

Ordering, for step i on device slot s = i % depth:
  copy-in stream : wait until step i-depth's layer has read x[s]; copy the
                   host batch into x[s]; record in_ready[s]
  compute stream : wait in_ready[s] and until step i-depth's result has been
                   copied out of out[s]; run the layer x[s] -> out[s];
                   record computed[s]
  copy-out stream: wait computed[s]; copy out[s] to the host buffer; record
                   copied[s] (returned to the caller)
Every step's input still crosses host->device and every result
device->host; only their overlap with neighbouring steps is new.

PHANTOM runs its MoE blocks inside transformers' forward with the batch
already on the device (python/phantom/phantom_cli.py:1393-1430); this class
is for callers whose batches live in host memory.
"""

from __future__ import annotations

import functools
from typing import Callable, Sequence, Union

import torch

from .layer import MoeLayer

LayerLike = Union[MoeLayer, Callable[[torch.Tensor, torch.Tensor], object]]


class HostPipeline:
    """Run ``layers`` on pinned host batches with the copies overlapped.

    ``layers``: :class:`MoeLayer` objects (each captured once per device slot
    as a CUDA graph on that slot's buffers) or callables ``fn(x, out)`` that
    enqueue their work on the current stream (run eagerly on the compute
    stream). ``T, H, dtype``: the batch shape every step uses.
    ``depth``: device slots (2 lets one step compute while its neighbours
    copy).

    ``submit(x_host, out_host, layer=None)`` enqueues one step: layer
    ``layer`` (default: steps cycle through ``layers``) on ``x_host``
    (pinned ``[T, H]``), the result landing in ``out_host`` (pinned
    ``[T, H]``). It returns an event of its own for this step, recorded
    after the result's copy; the caller may reuse ``x_host`` and read
    ``out_host`` once that event has completed (or after
    :meth:`synchronize`). The event stays valid however many steps follow.
    """

    def __init__(self, layers: Sequence[LayerLike], T: int, H: int, dtype: torch.dtype = torch.bfloat16,
                 device: torch.device | str | int | None = None, depth: int = 2):
        if not layers:
            raise ValueError("HostPipeline needs at least one layer")
        if depth < 1:
            raise ValueError(f"depth must be >= 1 (got {depth})")
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        if dev.type != "cuda":
            raise ValueError(f"HostPipeline runs on a CUDA device (got {dev})")
        self.T, self.H, self.dtype, self.device, self.depth = T, H, dtype, dev, depth
        # zeroed: capturing a slot's graph runs the layer once on the slot, and
        # uninitialised memory can hold inf or NaN, which the decode layer
        # reports in the device error word
        self.x = [torch.zeros(T, H, dtype=dtype, device=dev) for _ in range(depth)]
        self.out = [torch.zeros(T, H, dtype=dtype, device=dev) for _ in range(depth)]
        self.copy_in = torch.cuda.Stream(device=dev)
        self.compute = torch.cuda.Stream(device=dev)
        self.copy_out = torch.cuda.Stream(device=dev)
        self.in_ready = [torch.cuda.Event() for _ in range(depth)]
        self.computed = [torch.cuda.Event() for _ in range(depth)]
        self.copied = [torch.cuda.Event() for _ in range(depth)]
        self._used = [False] * depth
        self._step = 0
        self._run = []
        with torch.cuda.device(dev), torch.cuda.stream(self.compute):
            for layer in layers:
                if isinstance(layer, MoeLayer):
                    self._run.append([layer.graphed(self.x[s], self.out[s]) for s in range(depth)])
                else:
                    self._run.append([functools.partial(layer, self.x[s], self.out[s]) for s in range(depth)])
        self.compute.synchronize()

    def _check_host(self, name: str, t: torch.Tensor) -> None:
        if t.device.type != "cpu" or not t.is_pinned():
            raise ValueError(f"{name} must be a pinned host tensor")
        if tuple(t.shape) != (self.T, self.H) or t.dtype != self.dtype:
            raise ValueError(f"{name} must be {self.dtype} [{self.T}, {self.H}] (got {t.dtype} {tuple(t.shape)})")

    def submit(self, x_host: torch.Tensor, out_host: torch.Tensor, layer: int | None = None) -> torch.cuda.Event:
        self._check_host("x_host", x_host)
        self._check_host("out_host", out_host)
        s = self._step % self.depth
        l = self._step % len(self._run) if layer is None else layer
        if not 0 <= l < len(self._run):
            raise IndexError(f"layer {l} out of range (have {len(self._run)})")
        if self._used[s]:
            self.copy_in.wait_event(self.computed[s])   # step i-depth has read x[s]
        with torch.cuda.stream(self.copy_in):
            self.x[s].copy_(x_host, non_blocking=True)
            self.in_ready[s].record(self.copy_in)
        self.compute.wait_event(self.in_ready[s])
        if self._used[s]:
            self.compute.wait_event(self.copied[s])     # step i-depth's result has left out[s]
        with torch.cuda.stream(self.compute):
            self._run[l][s]()
            self.computed[s].record(self.compute)
        self.copy_out.wait_event(self.computed[s])
        with torch.cuda.stream(self.copy_out):
            out_host.copy_(self.out[s], non_blocking=True)
            self.copied[s].record(self.copy_out)
            done = torch.cuda.Event()
            done.record(self.copy_out)
        self._used[s] = True
        self._step += 1
        return done

    def synchronize(self) -> None:
        for st in (self.copy_in, self.compute, self.copy_out):
            st.synchronize()
