"""The slot-sharded ring's collective plumbing on two CPU ranks (gloo).

The ring's compute (StreamPipeline on a GPU) is replaced by a fake pipeline that finishes
deterministic latents and records shared-curve updates, so the test covers exactly the
multi-process part: slot ownership, curve broadcast tagged with the tick (applied on every
rank at tag + 2), the hot-LoRA (factors, strength, removal) and channel-gain broadcasts that
switch on the same tick on every rank, the gather of finished latents to rank 0 in rank
order, and the detection of a rank that left.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

T = 16


class FakePipe:
    def __init__(self, rank):
        self.rank, self.t = rank, 0
        self.curves = []          # (tick, name, first value or None)

    def set_shared_curve(self, name, v):
        self.curves.append((self.t, name, None if v is None else float(v[0])))

    def tick_many(self):
        out = []
        if self.t % 2 == self.rank:   # each rank finishes one latent every other tick
            out.append(torch.full((1, T, 64), float(100 * self.rank + self.t)).to(torch.bfloat16))
        self.t += 1
        return out


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from demon_b200.ring import ShardedRing
    pipe = FakePipe(rank)
    ring = ShardedRing(pipe, rank, world, T, "cpu", curve_names=["velocity_scale", "guidance_curve"],
                       curve_every=4, max_finished=2)

    def src(tick):
        return {"velocity_scale": torch.full((T,), 1.0 + tick), "guidance_curve": None if tick % 8 else
                torch.full((T,), 3.0 + tick)}
    gathered = []
    for _ in range(12):
        _, g = ring.step(src)
        if g is not None:
            gathered.append([float(x[0, 0, 0]) for x in g])
    if rank == 0:
        gathered.append([float(x[0, 0, 0]) for x in ring.collect()])
    q.put((rank, [ring.owns(i) for i in range(8)], pipe.curves, gathered))
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_sharded_ring_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, owns, curves, gathered = q.get(timeout=120)
        res[r] = (owns, curves, gathered)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # ownership: global slot g on rank g % 2
    assert res[0][0] == [g % 2 == 0 for g in range(8)]
    assert res[1][0] == [g % 2 == 1 for g in range(8)]
    # curves broadcast at ticks 0, 4, 8 apply at ticks 2, 6, 10 on both ranks, identically
    assert res[0][1] == res[1][1]
    applied = {(t, n): v for t, n, v in res[0][1]}
    assert applied[(2, "velocity_scale")] == 1.0 and applied[(2, "guidance_curve")] == 3.0
    assert applied[(6, "velocity_scale")] == 5.0 and applied[(6, "guidance_curve")] is None
    assert applied[(10, "velocity_scale")] == 9.0 and applied[(10, "guidance_curve")] == 11.0
    assert sorted({t for t, _, _ in res[0][1]}) == [2, 6, 10]
    # rank 0 gathers every finished latent, rank 0's first (tick t finishes on rank t % 2), each
    # tick's set handed over at the next step (the first step returns the empty set before it)
    assert res[1][2] == []
    assert res[0][2] == [[]] + [[100.0 * (t % 2) + t] for t in range(12)]


def _failing_worker(rank, world, port, q, fail_at):
    """Rank 1 dies on the host between two ticks (no collective in flight); rank 0 must learn of
    it through its next collective, which ends with an error inside the short group timeout
    instead of waiting for good."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import time
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    from demon_b200.ring import ShardedRing
    ring = ShardedRing(FakePipe(rank), rank, world, T, "cpu", curve_names=["velocity_scale"], curve_every=1,
                       max_finished=2)

    def src(tick):
        return {"velocity_scale": torch.full((T,), 1.0 + tick)}
    for i in range(8):
        if rank == 1 and i == fail_at:
            _report(q, (rank, "left", i))
            os._exit(3)  # the failure: the process leaves without joining the next collective
        t0 = time.monotonic()
        try:
            ring.step(src)
        except Exception as e:  # noqa: BLE001 -- any collective error is the detection
            _report(q, (rank, f"error after {time.monotonic() - t0:.1f}s: {type(e).__name__}", i))
            os._exit(0)
    _report(q, (rank, "finished", 8))
    os._exit(0)


def _report(q, msg):
    q.put(msg)
    q.close()
    q.join_thread()  # flush before the process exits without cleanup


def test_sharded_ring_rank_failure_is_detected():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q, 3)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, what, i = q.get(timeout=120)
        res[r] = (what, i)
    for p in procs:
        p.join(timeout=60)
    assert res[1] == ("left", 3)
    assert res[0][0].startswith("error"), res[0]
    assert res[0][1] == 3  # the first tick after the peer left
    assert procs[1].exitcode == 3


class FakeLoRAPipe(FakePipe):
    """FakePipe that also records, at every tick, the channel gain and the LoRA banks of two
    NVFP4 linears (the banks are host bookkeeping: no kernel runs on the CPU)."""

    def __init__(self, rank, lins):
        super().__init__(rank)
        self.lins, self.gain, self.log = lins, None, []

    def set_channel_gain_tensor(self, g):
        self.gain = None if g is None else g.clone()

    def tick_many(self):
        banks = {n: sorted((i, e.strength, float(e.A.float().sum()), float(e.B.float().sum()))
                           for i, e in lin.lora.entries.items()) for n, lin in self.lins.items()}
        self.log.append((self.t, None if self.gain is None else float(self.gain.float().sum()), banks))
        return super().tick_many()


def _lora_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from demon_b200.nvfp4 import NVFP4Linear
    from demon_b200.ring import ShardedRing
    lins = {"layers.0.self_attn.q_proj.weight": NVFP4Linear(128, 256, bias=False, device="cpu"),
            "layers.0.mlp.down_proj.weight": NVFP4Linear(256, 128, bias=False, device="cpu")}
    pipe = FakeLoRAPipe(rank, lins)
    ring = ShardedRing(pipe, rank, world, T, "cpu", curve_names=["velocity_scale"], curve_every=4,
                       max_finished=2, lora_targets=lins)
    g = torch.Generator().manual_seed(9)
    pairs = {"layers.0.self_attn.q_proj.weight": (torch.randn(16, 128, generator=g), torch.randn(256, 16, generator=g)),
             "layers.0.mlp.down_proj.weight": (torch.randn(32, 256, generator=g), torch.randn(128, 32, generator=g))}
    gain = torch.rand(1, T, 64, generator=g) + 0.5
    for t in range(16):
        if rank == 0 and t == 1:
            ring.enable_lora("L1", pairs, strength=0.5)
        if rank == 0 and t == 5:
            ring.set_channel_gain(gain)
            ring.set_lora_strength("L1", 1.0)
        if rank == 0 and t == 9:
            ring.disable_lora("L1")
            ring.set_channel_gain(None)
        ring.step()
    q.put((rank, pipe.log))
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_ring_broadcasts_lora_and_gain():
    """Rank 0's hot-LoRA enable (factors broadcast), strength change, removal and channel-gain
    changes reach rank 1 and switch on the same tick on both ranks (announced with the next
    control broadcast every 4 ticks, applied 2 ticks later), with identical factors."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_lora_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, log = q.get(timeout=120)
        res[r] = log
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0] == res[1]                     # same state at every tick on both ranks
    by_t = {t: (gain, banks) for t, gain, banks in res[0]}
    qn = "layers.0.self_attn.q_proj.weight"
    for t in range(16):
        gain, banks = by_t[t]
        ids = [e[:2] for e in banks[qn]]
        if t < 6:        # enable queued at tick 1, announced at 4, applied at 6
            assert ids == [] and gain is None, t
        elif t < 10:     # strength and gain queued at 5, announced at 8, applied at 10
            assert ids == [("L1", 0.5)] and gain is None, t
        elif t < 14:     # removal and gain clear queued at 9, announced at 12, applied at 14
            assert ids == [("L1", 1.0)] and gain is not None, t
        else:
            assert ids == [] and gain is None, t
    assert [e[0] for e in by_t[7][1]["layers.0.mlp.down_proj.weight"]] == ["L1"]
