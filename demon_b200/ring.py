"""Slot-sharded streaming ring over one process per GPU.

The ring shards by slot: global slot ``g`` lives on rank ``g % world``.  Every rank holds
the replicated NVFP4 weights and runs its own :class:`~demon_b200.stream.StreamPipeline`
over its slots, so no collective runs per forward.  Collectives (``torch.distributed``:
NCCL over NVLink on GPUs, gloo in the CPU tests) are used only to

* broadcast rank 0's hot mutations, tagged with the tick at which rank 0 announced them
  and applied by every rank at tick ``tag + apply_delay`` (default 2), so all ranks switch
  on the same tick whatever their relative progress and whatever the number of ranks:
  the shared curves (``set_shared_curve``, acestep/engine/stream.py:1319-1340), the channel
  gain (``set_channel_gain_tensor``, stream.py:1426-1437) and hot LoRAs -- enable with the
  LoRA's A / B factors, strength changes, removal (``enable_lora`` / ``set_lora_strength`` /
  ``disable_lora``, acestep/engine/lora.py:383-526);
* gather finished latents to rank 0.

Every ``curve_every`` ticks each rank takes part in one control broadcast from rank 0: the
curves, a fixed-size header of up to ``MAX_OPS`` mutation ops and a fixed-size manifest (the
names and shapes of an announced LoRA's factors).  Payloads (LoRA factors, a gain tensor)
travel in one more broadcast each, issued by every rank when the announcing header lands,
because only then do the other ranks know their sizes.  Nothing here makes the host wait for
the device: headers travel through pinned host buffers with asynchronous copies and are read
back on the host only when due, ``apply_delay`` ticks after the broadcast was enqueued (the
tick enqueued in between keeps the device busy), and the finished latents gathered at tick
``k`` are handed to rank 0's caller at tick ``k + 1`` (:meth:`collect` returns the last ones),
when their counts have long arrived.  Every rank takes the same collective steps in the same
order.  With one rank no collective runs (no process group is needed) and mutations still
apply at ``tag + apply_delay``.
"""
from __future__ import annotations

import json
import struct
from typing import Callable, Dict, List, Mapping, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

OP_ENABLE, OP_STRENGTH, OP_REMOVE, OP_GAIN = 1, 2, 3, 4
MAX_OPS = 8                 # mutation ops per control broadcast (more wait for the next one)
OP_FIELDS = 5               # code, LoRA slot, manifest bytes, payload elements, strength (f64 bits)
MANIFEST_BYTES = 1 << 16    # names and shapes of one announced LoRA


def _f64_bits(x: float) -> int:
    return struct.unpack("<q", struct.pack("<d", float(x)))[0]


def _bits_f64(b: int) -> float:
    return struct.unpack("<d", struct.pack("<q", int(b)))[0]


class ShardedRing:
    """``lora_targets``: weight name -> NVFP4 linear (``demon_b200.lora.lora_param_names`` of the
    decoder) whose LoRA banks the broadcast LoRA ops update; taken from ``pipe.decoder`` (or the
    module a ``GraphedDecoder`` wraps) when not given."""

    def __init__(self, pipe, rank: int, world: int, T: int, device, curve_names: Sequence[str] = (),
                 curve_every: int = 4, max_finished: int = 8, group=None, apply_delay: int = 2,
                 lora_targets: Optional[Mapping[str, object]] = None):
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
        # broadcasts not yet landed, oldest first: (tick enqueued, curves [1 + n, T], event, header,
        # manifest) in pinned host memory
        self._curves: List[tuple] = []
        self._pending: List[tuple] = []         # (apply_at_tick, {name: tensor | None}, [mutation ops])
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
        # control plane: header [2 + MAX_OPS * OP_FIELDS] int64 (tag, n_ops, ops) and manifest bytes
        self._hbuf = torch.zeros(2 + MAX_OPS * OP_FIELDS, dtype=torch.int64, device=self.device)
        self._mbuf = torch.zeros(MANIFEST_BYTES, dtype=torch.uint8, device=self.device)
        self._queued: List[tuple] = []          # rank 0: (code, slot, strength, manifest bytes, payload)
        self._announced: Dict[int, list] = {}   # rank 0: tag -> payloads of the ops announced then
        self._lora_slot: Dict[str, int] = {}    # rank 0: LoRA id -> slot number in the ops
        self._slot_id: Dict[int, str] = {}      # every rank: slot -> LoRA id (learned from manifests)
        self._lora_targets = lora_targets

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
        """Collective: rank 0's ``curves`` (name -> [T] tensor, or None to clear) and its queued
        mutation ops reach every rank and take effect at tick ``tag + apply_delay`` on all of
        them (tag = this tick)."""
        host = self._host(1 + len(self.curve_names), self.T)
        hh = self._host(self._hbuf.numel(), dtype=torch.int64)
        mh = self._host(MANIFEST_BYTES, dtype=torch.uint8)
        if self.rank == 0:
            host[0, 0] = float(self.ticks)
            for i, name in enumerate(self.curve_names):
                v = (curves or {}).get(name)
                if v is not None:
                    host[0, 1 + i] = 1.0
                    host[1 + i].copy_(torch.as_tensor(v, dtype=torch.float32).reshape(-1))
            self._pack_ops(hh, mh)
        ev = None
        if self.world > 1:
            self._cbuf.copy_(host, non_blocking=True)
            self._hbuf.copy_(hh, non_blocking=True)
            self._mbuf.copy_(mh, non_blocking=True)
            for b in (self._cbuf, self._hbuf, self._mbuf):
                dist.broadcast(b, src=0, group=self.group)
            host = self._host(1 + len(self.curve_names), self.T)
            hh = self._host(self._hbuf.numel(), dtype=torch.int64)
            mh = self._host(MANIFEST_BYTES, dtype=torch.uint8)
            host.copy_(self._cbuf, non_blocking=True)
            hh.copy_(self._hbuf, non_blocking=True)
            mh.copy_(self._mbuf, non_blocking=True)
            ev = self._event()
        self._curves.append((self.ticks, host, ev, hh, mh))

    def _pack_ops(self, hh: torch.Tensor, mh: torch.Tensor) -> None:
        """Rank 0: move up to MAX_OPS queued ops (at most one LoRA enable, whose manifest fills
        the manifest buffer) into this broadcast's header; their payloads wait for the landing."""
        hh[0] = self.ticks
        ops, pay, manifest_used = [], [], False
        while self._queued and len(ops) < MAX_OPS:
            code, slot, strength, manifest, payload = self._queued[0]
            if code == OP_ENABLE:
                if manifest_used:
                    break
                manifest_used = True
                mh[:len(manifest)].copy_(torch.frombuffer(bytearray(manifest), dtype=torch.uint8))
            self._queued.pop(0)
            n = 0 if payload is None else payload.numel()
            ops.append((code, slot, len(manifest) if manifest else 0, n, _f64_bits(strength)))
            pay.append(payload)
        hh[1] = len(ops)
        for i, op in enumerate(ops):
            hh[2 + i * OP_FIELDS:2 + (i + 1) * OP_FIELDS] = torch.tensor(op, dtype=torch.int64)
        self._announced[self.ticks] = pay

    def _land_curves(self) -> None:
        """Parse the broadcasts due at this tick: enqueued ``apply_delay`` ticks ago, so the ticks
        enqueued since keep the device busy while the host reads them."""
        while self._curves and self.ticks >= self._curves[0][0] + self.apply_delay:
            enq, host, ev, hh, mh = self._curves.pop(0)
            if ev is not None:
                ev.synchronize()
            tag = int(host[0, 0])
            upd = {name: (host[1 + i].clone() if host[0, 1 + i] > 0 else None)
                   for i, name in enumerate(self.curve_names)}
            ops = self._land_ops(enq, hh, mh)
            self._pending.append((tag + self.apply_delay, upd, ops))

    # ------------------------------------------------------------------ mutations (rank 0)
    def _require_rank0(self, what: str) -> None:
        if self.rank != 0:
            raise RuntimeError(f"{what}: hot mutations enter the ring on rank 0 only")

    def set_channel_gain(self, gain: Optional[torch.Tensor]) -> None:
        """Rank 0: the channel gain [1, T, 64] (or None to remove it) for every rank's slots
        (StreamPipeline.set_channel_gain_tensor, stream.py:1426-1437)."""
        self._require_rank0("set_channel_gain")
        payload = None
        if gain is not None:
            payload = gain.to(device=self.device, dtype=torch.bfloat16).reshape(-1).contiguous()
            if payload.numel() != self.T * 64:
                raise ValueError(f"gain must hold T x 64 = {self.T * 64} values")
        self._queued.append((OP_GAIN, 0, 0.0, None, payload))

    def enable_lora(self, lora_id: str, pairs: Mapping[str, Tuple[torch.Tensor, torch.Tensor]],
                    strength: float = 1.0) -> None:
        """Rank 0: register and enable a LoRA on every rank at ``strength``.  ``pairs``: weight
        name -> (A [r, K], B [N, r]) in the PEFT layout (``demon_b200.lora.load_lora_pairs``);
        the factors themselves are broadcast (raw B @ A, no alpha / rank factor, lora.py:316-319)."""
        self._require_rank0("enable_lora")
        slot = self._lora_slot.setdefault(lora_id, len(self._lora_slot))
        names = sorted(pairs)
        meta = {"id": lora_id, "params": []}
        flat = []
        for n in names:
            A, B = pairs[n]
            r, K = A.shape
            N = B.shape[0]
            if B.shape[1] != r:
                raise ValueError(f"{n}: lora_B must be [N, r] with r = {r}")
            meta["params"].append([n, int(r), int(K), int(N)])
            flat += [A.to(self.device, torch.bfloat16).reshape(-1), B.to(self.device, torch.bfloat16).reshape(-1)]
        manifest = json.dumps(meta).encode()
        if len(manifest) > MANIFEST_BYTES:
            raise ValueError(f"LoRA manifest of {len(manifest)} bytes exceeds {MANIFEST_BYTES}")
        payload = torch.cat(flat) if flat else torch.zeros(0, dtype=torch.bfloat16, device=self.device)
        self._queued.append((OP_ENABLE, slot, float(strength), manifest, payload))

    def set_lora_strength(self, lora_id: str, strength: float) -> None:
        """Rank 0: change an enabled LoRA's strength on every rank (a kernel scalar: no refit)."""
        self._require_rank0("set_lora_strength")
        self._queued.append((OP_STRENGTH, self._lora_slot[lora_id], float(strength), None, None))

    def disable_lora(self, lora_id: str) -> None:
        """Rank 0: remove a LoRA from every rank's banks."""
        self._require_rank0("disable_lora")
        self._queued.append((OP_REMOVE, self._lora_slot[lora_id], 0.0, None, None))

    # ------------------------------------------------------------------ landing
    def _land_ops(self, tag: int, hh: torch.Tensor, mh: torch.Tensor) -> list:
        """Every rank, at the landing of the header broadcast at ``tag``: the payload broadcasts
        of its ops (same order on every rank) and the ops ready to apply."""
        n = int(hh[1])
        pay = self._announced.pop(tag, [None] * n) if self.rank == 0 else [None] * n
        out = []
        for i in range(n):
            code, slot, mlen, numel, sbits = (int(v) for v in hh[2 + i * OP_FIELDS:2 + (i + 1) * OP_FIELDS])
            data = pay[i]
            if numel and self.world > 1:
                if self.rank != 0:
                    data = torch.empty(numel, dtype=torch.bfloat16, device=self.device)
                dist.broadcast(data, src=0, group=self.group)
            manifest = json.loads(bytes(mh[:mlen].tolist()).decode()) if code == OP_ENABLE else None
            out.append((code, slot, _bits_f64(sbits), manifest, data))
        return out

    def _targets(self):
        if self._lora_targets is None:
            from .lora import lora_param_names
            dec = getattr(self.pipe, "decoder", None)
            dec = getattr(dec, "decoder", dec)   # GraphedDecoder wraps the module
            self._lora_targets = lora_param_names(dec) if dec is not None else {}
        return self._lora_targets

    def _apply_op(self, op) -> None:
        code, slot, strength, manifest, data = op
        if code == OP_GAIN:
            self.pipe.set_channel_gain_tensor(None if data is None else data.view(1, self.T, 64))
            return
        lins = self._targets()
        if code == OP_ENABLE:
            lora_id = manifest["id"]
            self._slot_id[slot] = lora_id
            off = 0
            for name, r, K, N in manifest["params"]:
                A = data[off:off + r * K].view(r, K)
                off += r * K
                B = data[off:off + N * r].view(N, r)
                off += N * r
                lin = lins.get(name)
                if lin is not None:
                    lin.lora.set(lora_id, A, B, strength=strength)
            return
        lora_id = self._slot_id.get(slot)
        if lora_id is None:
            return
        for lin in lins.values():
            if lora_id not in lin.lora.entries:
                continue
            if code == OP_STRENGTH:
                lin.lora.set_strength(lora_id, strength)
            else:
                lin.lora.remove(lora_id)

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
        """One ring tick on every rank: apply the due curve updates and mutation ops, advance
        the local slots, gather the finished latents to rank 0, and every ``curve_every`` ticks
        broadcast rank 0's new shared curves (``curve_source(tick)``) and queued mutations.
        Returns (this rank's finished latents, rank 0's gathered latents of the previous tick or
        None)."""
        self._land_curves()
        due = [p for p in self._pending if self.ticks >= p[0]]
        self._pending = [p for p in self._pending if self.ticks < p[0]]
        for _, upd, ops in due:
            for name, v in upd.items():
                self.pipe.set_shared_curve(name, v)
            for op in ops:
                self._apply_op(op)
        finished = self.pipe.tick_many()
        gathered = self.gather_finished(finished)
        if self.ticks % self.curve_every == 0:
            self.broadcast_curves(curve_source(self.ticks) if (curve_source and self.rank == 0) else None)
        self.ticks += 1
        return finished, gathered
