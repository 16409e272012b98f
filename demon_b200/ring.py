"""Slot-sharded streaming ring over one process per GPU.

The ring shards by slot: global slot ``g`` lives on rank ``g % world``.  Every rank holds
the replicated NVFP4 weights and runs its own :class:`~demon_b200.stream.StreamPipeline`
over its slots, so no collective runs per forward.  Collectives (``torch.distributed``:
NCCL over NVLink on GPUs, gloo in the CPU tests) are used only to

* broadcast hot-mutated shared curves from rank 0, tagged with the tick at which they were
  set and applied by every rank at tick ``tag + apply_delay`` (default 2), so all ranks switch
  on the same tick whatever their relative progress, whatever the number of ranks;
* gather finished latents to rank 0.

Nothing here makes the host wait for the device: curves travel through pinned host buffers
with asynchronous copies and are read back on the host only when due, ``apply_delay`` ticks
after the broadcast was enqueued (the tick enqueued in between keeps the device busy), and the
finished latents gathered at tick ``k`` are handed to rank 0's caller at tick ``k + 1``
(:meth:`collect` returns the last ones), when their counts have long arrived.  Every rank takes the same collective steps in the
same order: :meth:`step` broadcasts on every ``curve_every``-th tick and gathers on every tick.
With one rank no collective runs (no process group is needed).
"""
from __future__ import annotations

from typing import Callable, Dict, List, Optional, Sequence

import torch
import torch.distributed as dist


class ShardedRing:
    def __init__(self, pipe, rank: int, world: int, T: int, device, curve_names: Sequence[str] = (),
                 curve_every: int = 4, max_finished: int = 8, group=None, apply_delay: int = 2):
        if apply_delay < 2:
            raise ValueError("apply_delay must be >= 2 (one tick for the broadcast to land)")
        self.pipe = pipe
        self.rank, self.world = rank, world
        self.T, self.device = T, torch.device(device)
        self.curve_names = list(curve_names)
        self.curve_every = curve_every
        self.max_finished = max_finished
        self.group = group
        self.apply_delay = apply_delay
        self.ticks = 0
        self._cuda = self.device.type == "cuda"
        self._curves: List[tuple] = []          # (tick enqueued, host buffer [1 + n, T], event), oldest first
        self._pending: List[tuple] = []         # (apply_at_tick, {name: tensor | None})
        # [1 + n_curves, T] fp32: row 0 = (tag, presence bits), rows 1.. = curve values
        self._cbuf = torch.zeros(1 + len(self.curve_names), T, dtype=torch.float32, device=self.device)
        # finished latents: double-buffered so tick k's gather is read while tick k + 1 gathers
        self._fbuf = [torch.zeros(max_finished, T, 64, dtype=torch.bfloat16, device=self.device) for _ in range(2)]
        self._fcnt = [torch.zeros(1, dtype=torch.int32, device=self.device) for _ in range(2)]
        if rank == 0:
            self._gbuf = [[torch.zeros_like(self._fbuf[0]) for _ in range(world)] for _ in range(2)]
            self._gcnt = [[torch.zeros_like(self._fcnt[0]) for _ in range(world)] for _ in range(2)]
        else:
            self._gbuf = self._gcnt = None
        self._gathered: Optional[tuple] = None  # (buffer index, host counts, event) of the last gather

    def _host(self, *shape, dtype=torch.float32) -> torch.Tensor:
        return torch.zeros(*shape, dtype=dtype, pin_memory=self._cuda)

    def _event(self):
        if not self._cuda:
            return None
        ev = torch.cuda.Event()
        ev.record()
        return ev

    # ------------------------------------------------------------------ slots
    def owns(self, global_slot: int) -> bool:
        return global_slot % self.world == self.rank

    def local_slots(self, n_global: int) -> List[int]:
        return [g for g in range(n_global) if self.owns(g)]

    # ------------------------------------------------------------------ collectives
    def broadcast_curves(self, curves: Optional[Dict[str, Optional[torch.Tensor]]] = None) -> None:
        """Collective: rank 0's ``curves`` (name -> [T] tensor, or None to clear) reach every
        rank and take effect at tick ``tag + apply_delay`` on all of them (tag = this tick)."""
        host = self._host(1 + len(self.curve_names), self.T)
        if self.rank == 0:
            host[0, 0] = float(self.ticks)
            for i, name in enumerate(self.curve_names):
                v = (curves or {}).get(name)
                if v is not None:
                    host[0, 1 + i] = 1.0
                    host[1 + i].copy_(torch.as_tensor(v, dtype=torch.float32).reshape(-1))
        ev = None
        if self.world > 1:
            self._cbuf.copy_(host, non_blocking=True)
            dist.broadcast(self._cbuf, src=0, group=self.group)
            host = self._host(1 + len(self.curve_names), self.T)
            host.copy_(self._cbuf, non_blocking=True)
            ev = self._event()
        self._curves.append((self.ticks, host, ev))

    def _land_curves(self) -> None:
        """Parse the broadcasts due at this tick: enqueued ``apply_delay`` ticks ago, so the ticks
        enqueued since keep the device busy while the host reads them."""
        while self._curves and self.ticks >= self._curves[0][0] + self.apply_delay:
            _, host, ev = self._curves.pop(0)
            if ev is not None:
                ev.synchronize()
            tag = int(host[0, 0])
            upd = {name: (host[1 + i].clone() if host[0, 1 + i] > 0 else None)
                   for i, name in enumerate(self.curve_names)}
            self._pending.append((tag + self.apply_delay, upd))

    def gather_finished(self, finished: List[torch.Tensor]) -> Optional[List[torch.Tensor]]:
        """Collective: every rank's finished latents [1, T, 64] to rank 0.  Returns, on rank 0,
        the latents gathered on the PREVIOUS call in rank order (one tick of latency keeps the
        host from waiting for the device); other ranks get None.  With one rank, the latents of
        this call."""
        if len(finished) > self.max_finished:
            raise ValueError(f"{len(finished)} finished slots exceed max_finished={self.max_finished}")
        if self.world == 1:  # a single rank: nothing to exchange
            return list(finished)
        b = self.ticks % 2
        for i, f in enumerate(finished):
            self._fbuf[b][i].copy_(f.reshape(self.T, 64))
        self._fcnt[b].fill_(len(finished))
        dist.gather(self._fbuf[b], self._gbuf[b] if self.rank == 0 else None, dst=0, group=self.group)
        dist.gather(self._fcnt[b], self._gcnt[b] if self.rank == 0 else None, dst=0, group=self.group)
        if self.rank != 0:
            return None
        prev = self.collect()
        cnt = self._host(self.world, dtype=torch.int32)
        for r in range(self.world):
            cnt[r:r + 1].copy_(self._gcnt[b][r], non_blocking=True)
        self._gathered = (b, cnt, self._event())
        return prev

    def collect(self) -> List[torch.Tensor]:
        """Rank 0: the latents of the last gather not yet returned (empty if none)."""
        if self._gathered is None:
            return []
        b, cnt, ev = self._gathered
        self._gathered = None
        if ev is not None:
            ev.synchronize()
        out = []
        for r in range(self.world):
            n = int(cnt[r])
            out.extend(self._gbuf[b][r][i:i + 1].clone() for i in range(n))
        return out

    # ------------------------------------------------------------------ tick
    def step(self, curve_source: Optional[Callable[[int], Dict[str, torch.Tensor]]] = None):
        """One ring tick on every rank: apply due curve updates, advance the local slots,
        gather the finished latents to rank 0, and every ``curve_every`` ticks broadcast
        rank 0's new shared curves (``curve_source(tick)``).  Returns (this rank's finished
        latents, rank 0's gathered latents of the previous tick or None)."""
        self._land_curves()
        due = [p for p in self._pending if self.ticks >= p[0]]
        self._pending = [p for p in self._pending if self.ticks < p[0]]
        for _, upd in due:
            for name, v in upd.items():
                self.pipe.set_shared_curve(name, v)
        finished = self.pipe.tick_many()
        gathered = self.gather_finished(finished)
        if self.curve_names and self.ticks % self.curve_every == 0:
            self.broadcast_curves(curve_source(self.ticks) if (curve_source and self.rank == 0) else None)
        self.ticks += 1
        return finished, gathered
