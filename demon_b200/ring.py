"""Slot-sharded streaming ring over one process per GPU.

The ring shards by slot: global slot ``g`` lives on rank ``g % world``.  Every rank holds
the replicated NVFP4 weights and runs its own :class:`~demon_b200.stream.StreamPipeline`
over its slots, so no collective runs per forward.  Collectives (``torch.distributed``:
NCCL over NVLink on GPUs, gloo in the CPU tests) are used only to

* broadcast hot-mutated shared curves from rank 0, tagged with the tick at which they were
  set and applied by every rank at the next tick (``tag + 1``), so all ranks switch on the
  same tick whatever their relative progress;
* gather finished latents to rank 0.

Every rank takes the same collective steps in the same order: :meth:`step` broadcasts on
every ``curve_every``-th tick and gathers on every tick.  With one rank no collective runs
(no process group is needed).
"""
from __future__ import annotations

from typing import Callable, Dict, List, Optional, Sequence

import torch
import torch.distributed as dist


class ShardedRing:
    def __init__(self, pipe, rank: int, world: int, T: int, device, curve_names: Sequence[str] = (),
                 curve_every: int = 4, max_finished: int = 8, group=None):
        self.pipe = pipe
        self.rank, self.world = rank, world
        self.T, self.device = T, torch.device(device)
        self.curve_names = list(curve_names)
        self.curve_every = curve_every
        self.max_finished = max_finished
        self.group = group
        self.ticks = 0
        self._pending: Optional[tuple] = None   # (apply_at_tick, {name: tensor | None})
        # [1 + n_curves, T] fp32: row 0 = (tag, presence bits), rows 1.. = curve values
        self._cbuf = torch.zeros(1 + len(self.curve_names), T, dtype=torch.float32, device=self.device)
        self._fbuf = torch.zeros(max_finished, T, 64, dtype=torch.bfloat16, device=self.device)
        self._fcnt = torch.zeros(1, dtype=torch.int32, device=self.device)
        if rank == 0:
            self._gbuf = [torch.zeros_like(self._fbuf) for _ in range(world)]
            self._gcnt = [torch.zeros_like(self._fcnt) for _ in range(world)]
        else:
            self._gbuf = self._gcnt = None

    # ------------------------------------------------------------------ slots
    def owns(self, global_slot: int) -> bool:
        return global_slot % self.world == self.rank

    def local_slots(self, n_global: int) -> List[int]:
        return [g for g in range(n_global) if self.owns(g)]

    # ------------------------------------------------------------------ collectives
    def broadcast_curves(self, curves: Optional[Dict[str, Optional[torch.Tensor]]] = None) -> None:
        """Collective: rank 0's ``curves`` (name -> [T] tensor, or None to clear) reach every
        rank and take effect at the next tick on all of them."""
        buf = self._cbuf
        if self.rank == 0:
            buf.zero_()
            buf[0, 0] = float(self.ticks)
            for i, name in enumerate(self.curve_names):
                v = (curves or {}).get(name)
                if v is not None:
                    buf[0, 1 + i] = 1.0
                    buf[1 + i].copy_(torch.as_tensor(v, dtype=torch.float32).reshape(-1).to(self.device))
        if self.world > 1:
            dist.broadcast(buf, src=0, group=self.group)
        host = buf.cpu()
        tag = int(host[0, 0])
        upd = {name: (host[1 + i].clone() if host[0, 1 + i] > 0 else None)
               for i, name in enumerate(self.curve_names)}
        self._pending = (tag + 1, upd)

    def gather_finished(self, finished: List[torch.Tensor]) -> Optional[List[torch.Tensor]]:
        """Collective: every rank's finished latents [1, T, 64] to rank 0, in rank order
        (rank 0 returns the list, other ranks None)."""
        if len(finished) > self.max_finished:
            raise ValueError(f"{len(finished)} finished slots exceed max_finished={self.max_finished}")
        if self.world == 1:  # a single rank: nothing to exchange
            return list(finished)
        for i, f in enumerate(finished):
            self._fbuf[i].copy_(f.reshape(self.T, 64))
        self._fcnt.fill_(len(finished))
        dist.gather(self._fbuf, self._gbuf, dst=0, group=self.group)
        dist.gather(self._fcnt, self._gcnt, dst=0, group=self.group)
        if self.rank != 0:
            return None
        out = []
        for r in range(self.world):
            n = int(self._gcnt[r].item())
            out.extend(self._gbuf[r][i:i + 1].clone() for i in range(n))
        return out

    # ------------------------------------------------------------------ tick
    def step(self, curve_source: Optional[Callable[[int], Dict[str, torch.Tensor]]] = None):
        """One ring tick on every rank: apply due curve updates, advance the local slots,
        gather the finished latents to rank 0, and every ``curve_every`` ticks broadcast
        rank 0's new shared curves (``curve_source(tick)``)."""
        if self._pending is not None and self.ticks >= self._pending[0]:
            for name, v in self._pending[1].items():
                self.pipe.set_shared_curve(name, v)
            self._pending = None
        finished = self.pipe.tick_many()
        gathered = self.gather_finished(finished)
        if self.curve_names and self.ticks % self.curve_every == 0:
            self.broadcast_curves(curve_source(self.ticks) if (curve_source and self.rank == 0) else None)
        self.ticks += 1
        return finished, gathered
