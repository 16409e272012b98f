"""Benchmark of the DEMON hot path on B200 (driver contract: one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload stream|linear]

Workload ``stream`` (default; BASELINE configs[4], the multi-GPU streaming ring): the
2B-shape ACE-Step DiT (24 layers, hidden 2048, GQA 16/8 heads of 128, MLP 6144; random
init, every DiT linear in NVFP4) drives a ring of 64 slots, T = 1500 latent frames (750
tokens), 8 steps per slot, standard CFG (a positive and a negative forward per slot per
tick), text condition [256, 2048] N(0,1).  The slots are sharded over the N GPUs (64/N per
rank, one process per GPU); each rank runs its own pipeline tick (batched DiT forwards as
CUDA-graph replays, then one fused ODE-step launch), finished latents are gathered to rank 0
and shared curves (velocity_scale, guidance) are mutated on rank 0 every 4 ticks and
broadcast (NCCL).  The ring is kept full: each tick 64/(8N) slots per rank finish and as
many new requests start.  One step = one global tick (all 64 slots advance one step);
``value`` = ticks/s of the whole job (total work fixed: strong scaling), timed with CUDA
events between barriers, max over ranks.  Request inputs are resident in HBM (a pool of 8
request templates); ``e2e`` repeats the run with the templates in pinned host memory (the
new requests' inputs cross H2D, the finished latents D2H, inside the timed region).

Workload ``linear``: one NVFP4 linear, x bf16 [1500, 2048]
(N(0,1), 1% of channels x20), W [6144, 2048] N(0, 0.02), bias 0; one step = quantise +
GEMM on a rotation of buffer sets larger than 2x L2; replicas on N GPUs.

``--impl reference`` times the reference's CPU path on this host's cores: for ``stream``
the CPU restatement of AceStepDiTModel (oracle/dit_ref.py, bit-exact with the reference
module) on one slot's CFG pair plus the CPU ODE-step oracle, scaled to the 64-slot tick;
for ``linear`` the reference's nn.Linear in bf16.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

M1, K1, N1 = 1500, 2048, 6144
FLOP1 = 2.0 * M1 * N1 * K1
CONFIG1 = {"workload": "config1: NVFP4 linear, x bf16 [1500,2048] N(0,1) w/ 1% channels x20, "
                       "W [6144,2048] N(0,0.02), bias 0", "M": M1, "K": K1, "N": N1,
           "l2": "rotating buffer sets, footprint > 2x L2 (no L2 reuse between steps)",
           "gs_mode": "per-row activation global scale, per-tensor weight global scale"}
METRIC = "NVFP4 linear TFLOPS (% FP4 peak); DiT stream ticks/sec, depth 8, 1\u20138 GPUs"
RING, T5, L5, STEPS5 = 64, 1500, 256, 8
CONFIG5 = {"workload": "configs[4]: streaming ring on the NVFP4 DiT (24 layers, hidden 2048, GQA 16/8 x 128, "
                       "MLP 6144, random init), 64 slots sharded over the GPUs, T=1500 frames (750 tokens), "
                       "8 steps, standard CFG, text [256,2048] N(0,1), curves mutated every 4 ticks (NCCL "
                       "broadcast), finished latents gathered to rank 0",
           "slots": RING, "T": T5, "tokens": T5 // 2, "text_len": L5, "steps_per_slot": STEPS5,
           "cfg": "standard (pos + neg forward)",
           "l2": "inputs > L2 (activations of one forward are several GB; weights 0.85 GB NVFP4)"}


def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def peaks():
    p = {}
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        p = json.loads(f.read_text())
    hbm = p.get("hbm_gbs")
    bf16 = p.get("bf16_tflops")
    src = "measured" if hbm and bf16 else "fallback"
    hbm = hbm or 6650.0
    bf16 = bf16 or 1590.0
    return {"hbm_gbs": hbm, "bf16_tflops": bf16, "fp4_tflops": 4.0 * bf16, "source": src,
            "bf16_sustained": p.get("bf16_tflops_sustained") or 1400.0}


class ClockSampler:
    """SM clock and throttle reasons sampled every 20 ms through NVML while the
    timed region runs (the fields of the recipe's nvidia-smi clocks line)."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}

    def __init__(self, gpu_index: int, period: float = 0.02):
        self.idx, self.period = gpu_index, period
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            phys = int(vis.split(",")[self.idx]) if vis else self.idx
            self.h = pynvml.nvmlDeviceGetHandleByIndex(phys)
            self.nv = pynvml
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM))
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        except Exception:
            self.nv = None
        return self

    def _run(self):
        while not self._stop.is_set():
            try:
                mhz = float(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                rs = int(self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h))
                self.samples.append((mhz, rs))
            except Exception:
                pass
            self._stop.wait(self.period)

    def __exit__(self, *a):
        self._stop.set()
        if self.nv is not None:
            self.t.join(timeout=2)

    def summary(self):
        sm = sorted(m for m, _ in self.samples)
        reasons = sorted({n for _, r in self.samples for n, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(sm), "source": "nvml every 20 ms during the timed region"}


def dist_init(world):
    import torch
    import torch.distributed as dist
    if world > 1 and not dist.is_initialized():
        import datetime
        dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    return dist if world > 1 else None


def max_over_ranks(v: float, dist_mod, device):
    import torch
    if dist_mod is None:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist_mod.all_reduce(t, op=dist_mod.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# CPU reference (the reference's nn.Linear in bf16 on host cores)
# ---------------------------------------------------------------------------

def cpu_linear_sample(seconds: float = 10.0):
    import torch
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(M1, K1, generator=g).to(torch.bfloat16)
    w = (torch.randn(N1, K1, generator=g) * 0.02).to(torch.bfloat16)
    b = torch.zeros(N1, dtype=torch.bfloat16)
    torch.nn.functional.linear(x, w, b)
    n, t0 = 0, time.perf_counter()
    while True:
        torch.nn.functional.linear(x, w, b)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds or n >= 2000:
            break
    return {"value": FLOP1 * n / el / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "reference",
            "sample": f"{n} x torch F.linear bf16 [1500,2048]x[2048,6144] (the reference's nn.Linear, "
                      f"turbo.py:286-289) in {el:.1f} s"}


def run_reference(args):
    rank, world, _ = env_rank()
    if rank != 0:
        return
    import torch
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(M1, K1, generator=g).to(torch.bfloat16)
    w = (torch.randn(N1, K1, generator=g) * 0.02).to(torch.bfloat16)
    b = torch.zeros(N1, dtype=torch.bfloat16)
    for _ in range(args.warmup):
        torch.nn.functional.linear(x, w, b)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        torch.nn.functional.linear(x, w, b)
    el = time.perf_counter() - t0
    v = FLOP1 * args.steps / el / 1e12
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el * 1e3 / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": CONFIG1,
        "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "reference",
                         "sample": f"{args.steps} x torch F.linear bf16 (the reference's nn.Linear) on {cores} cores"},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ---------------------------------------------------------------------------
# kernel legs
# ---------------------------------------------------------------------------

class _CudnnBand:
    """The library baseline the attention leg compares against for the sliding window: one
    cuDNN-frontend fused-attention graph with a diagonal band (left bound window + 1, right
    bound window), GQA native, reading q / k / v through their strides."""

    def __init__(self):
        self._graphs = {}
        self._handle = None

    def __call__(self, q, k, v, window):
        import cudnn
        import torch
        B, S, Hq, D = q.shape
        L, Hk = k.shape[1], k.shape[2]
        out = torch.empty(B, S, Hq, D, dtype=torch.bfloat16, device=q.device)
        qv, kv, vv, ov = (t.transpose(1, 2) for t in (q, k, v, out))
        strides = tuple(tuple(t.stride()) for t in (qv, kv, vv, ov))
        if self._handle is None:
            self._handle = cudnn.create_handle()
        key = (B, S, L, Hq, Hk, D, window, strides)
        ent = self._graphs.get(key)
        if ent is None:
            c = cudnn
            g = c.pygraph(io_data_type=c.data_type.BFLOAT16, intermediate_data_type=c.data_type.FLOAT,
                          compute_data_type=c.data_type.FLOAT, handle=self._handle)
            ts = [g.tensor(name=n, dim=[B, h, n_, D], stride=list(st), data_type=c.data_type.BFLOAT16)
                  for n, h, n_, st in (("q", Hq, S, strides[0]), ("k", Hk, L, strides[1]), ("v", Hk, L, strides[2]))]
            o, _ = g.sdpa(q=ts[0], k=ts[1], v=ts[2], is_inference=True, attn_scale=D ** -0.5,
                          diagonal_band_left_bound=window + 1, diagonal_band_right_bound=window)
            o.set_output(True).set_dim([B, Hq, S, D]).set_stride(list(strides[3])).set_data_type(c.data_type.BFLOAT16)
            g.validate()
            g.build_operation_graph()
            g.create_execution_plans([c.heur_mode.A, c.heur_mode.FALLBACK])
            g.check_support()
            g.build_plans()
            ws = torch.empty(max(1, g.get_workspace_size()), dtype=torch.uint8, device=q.device)
            ent = self._graphs[key] = (g, ts + [o], ws)
        g, (tq, tk, tv, to), ws = ent
        cudnn.set_stream(handle=self._handle, stream=torch.cuda.current_stream().cuda_stream)
        g.execute({tq: qv, tk: kv, tv: vv, to: ov}, ws, handle=self._handle)
        return out


def attention_leg(dev, B=128, S=750, L=L5, hq=16, hk=8, reps=20):
    """The DiT's three attention classes at the tick's shapes (B = 2 CFG x 64 slots sequences of
    750 tokens, GQA 16/8 x 128, text 256): demon's sm_100a kernel beside the cuDNN fused
    attention it replaced (SDPA for global and cross, a diagonal-band graph for the window),
    each replayed from a CUDA graph of `reps` launches.  FLOPs count only the scores inside the
    band (4 * B * Hq * D per valid (query, key) pair)."""
    import torch
    from torch.nn.attention import SDPBackend, sdpa_kernel
    from demon_b200.attention import attention
    D = 128
    g = torch.Generator(device=dev).manual_seed(0)
    qkv = torch.randn(B * S, (hq + 2 * hk) * D, device=dev, generator=g).to(torch.bfloat16)
    ld = qkv.stride(0)
    q = qkv.as_strided((B, S, hq, D), (S * ld, ld, D, 1))
    k = qkv.as_strided((B, S, hk, D), (S * ld, ld, D, 1), hq * D)
    v = qkv.as_strided((B, S, hk, D), (S * ld, ld, D, 1), (hq + hk) * D)
    kvx = torch.randn(B * L, 2 * hk * D, device=dev, generator=g).to(torch.bfloat16)
    ldk = kvx.stride(0)
    ck = kvx.as_strided((B, L, hk, D), (L * ldk, ldk, D, 1))
    cv = kvx.as_strided((B, L, hk, D), (L * ldk, ldk, D, 1), hk * D)
    qc = torch.randn(B, S, hq, D, device=dev, generator=g).to(torch.bfloat16)
    band = _CudnnBand()

    def sdpa(qq, kk, vv):
        with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
            return torch.nn.functional.scaled_dot_product_attention(
                qq.transpose(1, 2), kk.transpose(1, 2), vv.transpose(1, 2), enable_gqa=True).transpose(1, 2)
    n_band = sum(min(i + 128, S - 1) - max(i - 128, 0) + 1 for i in range(S))
    classes = {
        "band": (lambda: attention(q, k, v, 128), lambda: band(q, k, v, 128), 4 * B * hq * n_band * D),
        "global": (lambda: attention(q, k, v), lambda: sdpa(q, k, v), 4 * B * hq * S * S * D),
        "cross": (lambda: attention(qc, ck, cv), lambda: sdpa(qc, ck, cv), 4 * B * hq * S * L * D),
    }
    res = {}
    for name, (mine, lib, flops) in classes.items():
        a, b = mine().float(), lib().float()
        diff = float((a - b).norm() / b.norm())
        t = {}
        for tag, fn in (("demon", mine), ("cudnn", lib)):
            for _ in range(2):
                fn()
            torch.cuda.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                for _ in range(reps):
                    fn()
            gr.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            gr.replay()
            e1.record()
            torch.cuda.synchronize()
            t[tag] = e0.elapsed_time(e1) * 1e3 / reps
            del gr
        res[name] = {"demon_us": round(t["demon"], 1), "cudnn_us": round(t["cudnn"], 1),
                     "demon_tflops": round(flops / t["demon"] / 1e6, 1), "cudnn_tflops": round(flops / t["cudnn"] / 1e6, 1),
                     "demon_over_cudnn_time": round(t["demon"] / t["cudnn"], 3), "rel_diff_vs_cudnn": diff}
    per_fwd = {tag: 12 * res["band"][f"{tag}_us"] + 12 * res["global"][f"{tag}_us"] + 24 * res["cross"][f"{tag}_us"]
               for tag in ("demon", "cudnn")}
    res["per_forward_ms"] = {k: round(v / 1e3, 3) for k, v in per_fwd.items()}
    res["shapes"] = f"B={B} sequences x {S} tokens, GQA {hq}/{hk} x 128, text {L}; 12 band + 12 global + 24 cross per forward"
    return res


def ode_workload(dev, nslots=64, T=1500, seed=0):
    """Config-3 slot features at config-5 scale: 64 slots x T=1500 x 64, CFG modes cycling
    standard / RCFG-initialize (cached negative) / RCFG-self, per-slot guidance U(3,7),
    per-frame velocity_scale / sde_denoise / apg_momentum / cfg_rescale splines in [0, 1.5],
    source latents (SDE-curve path), binary latent mask with 40 % spans, channel gain U(0.8, 1.2),
    DCW double with the reference's default scalers (on by default in its DiffusionConfig).
    Returns (OdeTick with the slots added, algorithmic bytes per launch, gain)."""
    import torch
    from demon_b200 import ode
    g = torch.Generator().manual_seed(seed)
    D = 64
    bf = torch.bfloat16

    def spline(lo, hi):
        knots = torch.rand(16, generator=g) * (hi - lo) + lo
        xs = torch.linspace(0, 15, T)
        i = xs.floor().clamp(max=14).long()
        f = xs - i
        return knots[i] * (1 - f) + knots[i + 1] * f

    def lat():
        return torch.randn(T, D, generator=g).to(bf).to(dev)

    tick = ode.OdeTick(dev, T, max_slots=nslots)
    vpos = torch.randn(nslots, T, D, generator=g).to(bf).to(dev)
    vneg = torch.randn(nslots, T, D, generator=g).to(bf).to(dev)
    gain = (torch.rand(T, D, generator=g) * 0.4 + 0.8).to(bf).to(dev)
    elems = T * D
    nbytes = 0
    for i in range(nslots):
        mode = ("full", "initialize", "self")[i % 3]
        m = torch.zeros(T)
        a = int(torch.randint(0, T - int(0.4 * T), (1,), generator=g))
        m[a:a + int(0.4 * T)] = 1.0
        st = ode.SlotStep(
            xt=lat(), t_curr=0.75, t_next=0.5, step_idx=3, total_steps=8, pos=[(vpos[i], None)],
            has_cfg=True, rcfg_mode=mode,
            neg=[(vneg[i], None)] if mode == "full" else None,
            neg_cached=lat() if mode == "initialize" else None,
            initial_noise=lat() if mode == "self" else None,
            momentum=lat(), momentum_fresh=False,
            guidance=float(torch.rand(1, generator=g)) * 4 + 3, apg_momentum=spline(0, 1.5),
            cfg_rescale=spline(0, 1.5), velocity_scale=spline(0, 1.5), sde_denoise_curve=spline(0, 1.5),
            source=lat(), mask=ode.LatentMask(m.to(dev), lat(), lat()),
            dec_out=torch.empty(T, D, dtype=bf, device=dev), dcw=("double", 0.05, 0.02), seed=1000 + i)
        tick.add(st)
        # reads: v_pos, v_neg source, momentum, xt, mask original + noise, source; writes: momentum, xt, dec
        nbytes += elems * 2 * (7 + 3)
    nbytes += elems * 2  # the channel gain, shared by every slot
    return tick, nbytes, gain


def measure_ode(dev, stream, reps=20):
    """HBM roofline of the fused ODE step: two slot sets (2 x 123 MB > 2x L2) alternated."""
    import torch
    from demon_b200 import _native as nat
    ticks = [ode_workload(dev, seed=s) for s in (0, 1)]
    launches = []
    for tk, nbytes, gain in ticks:
        b, nb = tk._stage()
        tk._dev[b][:nb].copy_(tk._host[b][:nb])
        launches.append((tk._dev[b].data_ptr(), len(tk.slots), tk.T, nbytes, gain))
    torch.cuda.synchronize()

    def run(i):
        ptr, n, T, _, gain = launches[i % 2]
        nat.check(nat.load().demon_ode_step(ptr, n, T, 64, nat.ptr(gain), nat.stream_ptr()))

    for i in range(4):
        run(i)
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        for i in range(reps):
            run(i)
    gr.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    gr.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / reps
    nbytes = sum(l[3] for l in launches) / 2
    return {"kernel": "demon::ode_step_kernel", "workload": "64 slots x T=1500 x 64 (config-3 features)",
            "us": us, "bytes": nbytes, "achieved": nbytes / (us * 1e-6) / 1e9, "unit": "GB/s"}


def measure_quantize(sets, stream, reps=8):
    import torch
    from demon_b200 import nvfp4
    nsets = len(sets)
    for s_ in sets:
        nvfp4.quantize(s_["x"])
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        for _ in range(reps):
            for s_ in sets:
                nvfp4.quantize(s_["x"])
    gr.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    gr.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * nsets)
    nbytes = M1 * K1 * 2 + M1 * K1 // 2 + M1 * K1 // 16
    return {"kernel": "demon::quantize_rows_kernel<2,2>", "workload": "x bf16 [1500, 2048], per-row scales",
            "us": us, "bytes": nbytes, "achieved": nbytes / (us * 1e-6) / 1e9, "unit": "GB/s"}




def measure_quantize_big(dev, stream, M=12000, K=2048, reps=10):
    """Quantiser HBM roofline at a tick's activation size (x bf16 [M, 2048], the rank's rows of
    one forward: 2 x slots x 750 tokens), three inputs rotated so L2 holds none of them from one
    launch to the next (at M = 12000, the 8-GPU ring's rank, 3 x 49 MB)."""
    import torch
    from demon_b200 import nvfp4
    xs = [torch.randn(M, K, device=dev).to(torch.bfloat16) for _ in range(3)]
    for x in xs:
        nvfp4.quantize(x)
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        for i in range(reps):
            nvfp4.quantize(xs[i % 3])
    gr.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    gr.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / reps
    nbytes = M * K * 2 + M * K // 2 + M * K // 16 + M * 4
    return {"kernel": "demon::quantize_blocks_kernel<2,2048>", "workload": f"x bf16 [{M}, {K}], per-row scales",
            "us": us, "bytes": nbytes, "achieved": nbytes / (us * 1e-6) / 1e9, "unit": "GB/s"}


def linear_leg(dev, stream, reps=64):
    """Config-1 NVFP4 linear (M=1500, K=2048, N=6144): GEMM device time over a rotation of
    buffer sets larger than 2x L2, one CUDA graph."""
    import torch
    from demon_b200 import nvfp4
    per_set = M1 * K1 // 2 + N1 * K1 // 2 + M1 * N1 * 2
    nsets = max(2, int(2 * 126e6 // per_set) + 1)
    g = torch.Generator(device=dev).manual_seed(11)
    sets = []
    for _ in range(nsets):
        x = torch.randn(M1, K1, generator=g, device=dev)
        x[:, :K1 // 100] *= 20.0
        w = (torch.randn(N1, K1, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        sets.append((nvfp4.quantize(x.to(torch.bfloat16)), nvfp4.pack_weight(w),
                     torch.zeros(N1, dtype=torch.bfloat16, device=dev),
                     torch.empty(M1, N1, dtype=torch.bfloat16, device=dev)))
    for a, w, b, y in sets:
        nvfp4.gemm(a, w, bias=b, out=y)
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        for i in range(reps):
            a, w, b, y = sets[i % nsets]
            nvfp4.gemm(a, w, bias=b, out=y)
    gr.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    gr.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / reps
    pk = peaks()
    tf = FLOP1 / (us * 1e-6) / 1e12
    traffic = None
    f = ROOT / "profiles" / "traffic.json"
    if f.exists():
        traffic = json.loads(f.read_text()).get("nvfp4_gemm_config1")
    return {"kernel": "demon::gemm_kernel<256, 5, 1, 1, 5>", "workload": CONFIG1["workload"], "us": us,
            "achieved": tf, "unit": "TFLOP/s", "peak": pk["fp4_tflops"], "frac": tf / pk["fp4_tflops"],
            "peak_note": "4x the measured burst bf16 cuBLAS figure (kernel timed alone)", "traffic": traffic}


def run_linear(args):
    import torch
    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist_mod = dist_init(world)
    from demon_b200 import _build
    if rank == 0 or not (ROOT / "demon_b200" / "libdemon_b200.so").exists():
        _build.build()
    if dist_mod is not None:
        dist_mod.barrier()
    from demon_b200 import _native as nat
    from demon_b200 import nvfp4

    # rotation of distinct buffer sets, footprint > 2x L2
    per_set = M1 * K1 * 2 + N1 * K1 // 2 + N1 * K1 // 8 + M1 * N1 * 2
    nsets = max(2, int(2 * 126e6 // per_set) + 1)
    g = torch.Generator().manual_seed(1234 + rank)
    sets = []
    for i in range(nsets):
        x = torch.randn(M1, K1, generator=g)
        idx = torch.randperm(K1, generator=g)[: K1 // 100]
        x[:, idx] *= 20.0
        w = (torch.randn(N1, K1, generator=g) * 0.02).to(torch.bfloat16).to(dev)
        sets.append(dict(x=x.to(torch.bfloat16).to(dev), w=nvfp4.pack_weight(w),
                         b=torch.zeros(N1, dtype=torch.bfloat16, device=dev),
                         y=torch.empty(M1, N1, dtype=torch.bfloat16, device=dev)))
        del w
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)

    def step(s):
        a = nvfp4.quantize(s["x"])
        nvfp4.gemm(a, s["w"], bias=s["b"], out=s["y"])

    # eager warm-up (first launches set function attributes), then one CUDA graph per buffer set:
    # a step is a graph replay of [quantise, GEMM], so host launch overhead stays off the clock
    for k in range(args.warmup):
        step(sets[k % nsets])
    torch.cuda.synchronize()
    pool = torch.cuda.graph_pool_handle()
    graphs = []
    for s_ in sets:
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, pool=pool):
            step(s_)
        graphs.append(gr)
    gemm_graph = torch.cuda.CUDAGraph()  # GEMM-only launches over the rotation, for the roofline
    qs = [nvfp4.quantize(s_["x"]) for s_ in sets]
    torch.cuda.synchronize()
    gemm_reps = max(1, 64 // nsets)
    with torch.cuda.graph(gemm_graph, pool=pool):
        for _ in range(gemm_reps):
            for s_, q_ in zip(sets, qs):
                nvfp4.gemm(q_, s_["w"], bias=s_["b"], out=s_["y"])
    for k in range(args.warmup):
        graphs[k % nsets].replay()
    gemm_graph.replay()
    torch.cuda.synchronize()
    if dist_mod is not None:
        dist_mod.barrier()
    torch.cuda.synchronize()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        t_start.record(stream)
        for k in range(args.steps):
            graphs[k % nsets].replay()
        t_end.record(stream)
        g0.record(stream)
        gemm_graph.replay()
        g1.record(stream)
        torch.cuda.synchronize()
    ms_local = t_start.elapsed_time(t_end)
    if dist_mod is not None:
        dist_mod.barrier()
    torch.cuda.synchronize()
    ms = max_over_ranks(ms_local, dist_mod, dev)
    gemm_avg = max_over_ranks(g0.elapsed_time(g1) / (gemm_reps * nsets), dist_mod, dev)
    quant = measure_quantize(sets, stream)
    odek = measure_ode(dev, stream) if args.ode else None
    status = nat.device_status()

    # end to end through the public API: pinned host x -> device, NVFP4Linear, y -> pinned host
    lin = nvfp4.NVFP4Linear(K1, N1, bias=True, device=dev)
    with torch.no_grad():
        lin.weight.copy_((torch.randn(N1, K1, generator=g) * 0.02).to(torch.bfloat16))
        lin.bias.zero_()
    lin.repack()
    xh = sets[0]["x"].cpu().pin_memory()
    yh = torch.empty(M1, N1, dtype=torch.bfloat16).pin_memory()
    xd = torch.empty_like(sets[0]["x"])
    for _ in range(max(3, args.warmup)):
        xd.copy_(xh, non_blocking=True)
        yh.copy_(lin(xd), non_blocking=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        xd.copy_(xh, non_blocking=True)
        yh.copy_(lin(xd), non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), dist_mod, dev)

    if rank == 0:
        pk = peaks()
        achieved = FLOP1 / (gemm_avg * 1e-3) / 1e12
        traffic = None
        tf = ROOT / "profiles" / "traffic.json"
        if tf.exists():
            traffic = json.loads(tf.read_text()).get("nvfp4_gemm_config1")
        cpu = cpu_linear_sample(args.cpu_seconds) if (world == 1 and args.cpu_seconds > 0) else None
        value = FLOP1 * args.steps * world / (ms * 1e-3) / 1e12
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "nvfp4 (e2m1 x ue4m3 blocks, fp32 accumulate)", "data": "synthetic",
            "config": dict(CONFIG1, parallelism=f"replicas x{world}", buffer_sets=nsets),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": pk["fp4_tflops"], "unit": "TFLOP/s",
                         "frac": achieved / pk["fp4_tflops"], "traffic": traffic,
                         "peak_note": f"FP4 dense peak taken as 4x the {pk['source']} bf16 cuBLAS figure "
                                      f"({pk['bf16_tflops']:.0f} TF/s); nominal 9 PF/s -> frac "
                                      f"{achieved / 9000.0:.3f}",
                         "kernel": "demon::gemm_kernel<256, 5, 1, 1, 5>", "gemm_us": gemm_avg * 1e3},
            "e2e": {"value": FLOP1 * args.steps * world / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": M1 * K1 * 2, "d2h_bytes_per_step": M1 * N1 * 2},
            "gpu_launches": 2 * args.steps + gemm_reps * nsets,
            "clocks": clk.summary(),
            "device_status": list(status),
        }
        kern = {"quantize": dict(quant, peak=pk["hbm_gbs"], frac=quant["achieved"] / pk["hbm_gbs"])}
        if odek is not None:
            kern["ode_step"] = dict(odek, peak=pk["hbm_gbs"], frac=odek["achieved"] / pk["hbm_gbs"])
        line["kernels"] = kern
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if dist_mod is not None:
        dist_mod.barrier()
        dist_mod.destroy_process_group()




# ---------------------------------------------------------------------------
# stream workload
# ---------------------------------------------------------------------------

def build_dit(dev):
    import torch
    from demon_b200.dit import DemonDiT, DiTConfig
    return DemonDiT(DiTConfig()).to(dev, torch.bfloat16).init_random_(0).eval()


def request_templates(dev, n=8, seed=7, pin=False):
    """n distinct (text, negative text, context latents, guidance) request inputs."""
    import torch
    g = torch.Generator().manual_seed(seed)
    bf = torch.bfloat16
    out = []
    for _ in range(n):
        t = [torch.randn(1, L5, 2048, generator=g).to(bf), torch.randn(1, L5, 2048, generator=g).to(bf),
             torch.randn(1, T5, 128, generator=g).to(bf)]
        t = [x.pin_memory() if pin else x.to(dev) for x in t]
        out.append((*t, float(torch.rand(1, generator=g)) * 4 + 3))
    return out


def curve_source(tick):
    """Rank 0's shared-curve mutation at `tick`: smooth velocity_scale in [0.8, 1.2], guidance in [3, 7]."""
    import torch
    x = torch.linspace(0, 1, T5)
    return {"velocity_scale": 1.0 + 0.2 * torch.sin(6.283 * (x + 0.1 * tick)),
            "guidance_curve": 5.0 + 2.0 * torch.cos(6.283 * (x - 0.05 * tick))}


class Ring:
    """One rank's share of the 64-slot ring plus its request feed."""

    def __init__(self, dit, dev, rank, world, templates):
        import torch
        from demon_b200.ring import ShardedRing
        from demon_b200.stream import StreamConfig, StreamPipeline
        self.local = RING // world
        self.k_new = max(1, self.local // STEPS5)
        self.rank, self.world = rank, world
        self.tmpl = templates
        self.ones = torch.ones(1, L5, dtype=torch.bfloat16, device=dev)
        self.pipe = StreamPipeline(dit, StreamConfig(infer_steps=STEPS5), pipeline_depth=self.local, device=dev,
                                   use_graphs=True)
        self.ring = ShardedRing(self.pipe, rank, world, T5, dev, curve_names=["velocity_scale", "guidance_curve"],
                                curve_every=4, max_finished=self.local)
        self.n_sub = 0

    def set_templates(self, t):
        self.tmpl = t

    def _request(self):
        from demon_b200.stream import SlotCondition, SlotRequest
        enc, neg, ctx, gsc = self.tmpl[self.n_sub % len(self.tmpl)]
        import torch
        gid = self.n_sub * self.world + self.rank
        self.n_sub += 1
        return SlotRequest(encoder_hidden_states=enc, encoder_attention_mask=self.ones, context_latents=ctx,
                           seed=gid, neg_conditions=[SlotCondition(neg, self.ones)],
                           guidance_curve=torch.tensor(gsc))

    def tick(self, on_finished=None):
        for _ in range(self.k_new):
            self.pipe.submit(self._request())
        fin, gathered = self.ring.step(curve_source)
        if on_finished is not None:
            on_finished(fin)
        return fin


def run_config3(dit, dev, ticks=24, warmup=24):
    """BASELINE config 3 on one GPU: a depth-8 ring at T=750 (375 tokens) on the full DiT with
    heterogeneous slots -- denoise cycling 1.0 / 0.5 / 0.75 (source latents), CFG cycling
    standard / RCFG-initialize / RCFG-self, guidance U(3, 7), velocity_scale / sde_denoise /
    apg_momentum / cfg_rescale as [750] splines in [0, 1.5], binary latent mask with 40 %
    spans, channel gain U(0.8, 1.2), DCW on (the reference's default); one request submitted
    per tick, one slot finished per tick (StreamPipeline.tick).  The rows per forward vary with
    the CFG modes, so the warm-up runs long enough to capture every shape's graph before the
    timed ticks.  Returns ticks/s (CUDA events)."""
    import torch
    from demon_b200.stream import (LatentNoiseMask, SlotCondition, SlotRequest, StreamConfig,
                                   StreamPipeline)
    T, L, D = 750, L5, 2048
    g = torch.Generator().manual_seed(33)
    bf = torch.bfloat16

    def spline(lo, hi):
        knots = torch.rand(16, generator=g) * (hi - lo) + lo
        xs = torch.linspace(0, 15, T)
        i = xs.floor().clamp(max=14).long()
        f = xs - i
        return knots[i] * (1 - f) + knots[i + 1] * f

    ones = torch.ones(1, L, dtype=bf, device=dev)
    reqs = []
    for k in range(12):
        src = torch.randn(1, T, 64, generator=g).to(bf).to(dev)
        m = torch.zeros(T)
        a0 = int(torch.randint(0, T - int(0.4 * T), (1,), generator=g))
        m[a0:a0 + int(0.4 * T)] = 1.0
        mode = ("standard", "initialize", "self")[k % 3]
        kw = dict(guidance_curve=torch.tensor(float(torch.rand(1, generator=g)) * 4 + 3),
                  velocity_scale=spline(0, 1.5), sde_denoise_curve=spline(0, 1.5),
                  apg_momentum=spline(0, 1.5), cfg_rescale_curve=spline(0, 1.5))
        if mode != "self":
            kw["neg_conditions"] = [SlotCondition(torch.randn(1, L, D, generator=g).to(bf).to(dev), ones)]
        if mode != "standard":
            kw["rcfg_mode"] = mode
        reqs.append(SlotRequest(
            encoder_hidden_states=torch.randn(1, L, D, generator=g).to(bf).to(dev), encoder_attention_mask=ones,
            context_latents=torch.randn(1, T, 128, generator=g).to(bf).to(dev), seed=700 + k,
            source_latents=src, denoise=(1.0, 0.5, 0.75)[k % 3],
            latent_mask=LatentNoiseMask(mask=m.to(dev), original_latents=src,
                                        noise=torch.randn(1, T, 64, generator=g).to(bf).to(dev)), **kw))
    pipe = StreamPipeline(dit, StreamConfig(infer_steps=8), pipeline_depth=8, device=dev, use_graphs=True)
    pipe.set_channel_gain_tensor((torch.rand(1, T, 64, generator=g) * 0.4 + 0.8).to(bf).to(dev))
    n = 0
    for _ in range(8 + warmup):
        pipe.submit(reqs[n % len(reqs)])
        n += 1
        pipe.tick()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(ticks):
        pipe.submit(reqs[n % len(reqs)])
        n += 1
        pipe.tick()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / ticks
    pipe.close()
    return {"workload": "configs[2]: depth-8 ring, T=750 (375 tokens), 8 steps, heterogeneous slots "
                        "(denoise 1.0/0.5/0.75, standard / RCFG-initialize / RCFG-self CFG, guidance U(3,7), "
                        "four [750] spline curves, 40 % latent mask, channel gain, DCW), full DiT",
            "value": 1e3 / ms, "unit": "ticks/s", "ms_per_tick": ms, "ticks": ticks}


PHASE_FUNCS = (("Q", "gemm", "gemm"), ("D", "_attention", "attention"), ("D", "adanorm_quantize", "row_kernels"),
               ("Q", "quantize", "row_kernels"), ("D", "head_norm_rope", "row_kernels"),
               ("D", "silu_mul_quantize", "row_kernels"), ("Q", "bf16_linear", "bf16_linears"),
               ("Q", "lora_down", "lora_down"))


def _graph_ms(fn, reps=3):
    """Device ms of fn() captured in one CUDA graph and replayed (CUDA events around the last
    replay): no host launch gaps inside."""
    import torch
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        fn()
    for _ in range(reps - 1):
        gr.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    gr.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    del gr
    return ms


def forward_inputs(dev, B, T=None, L=None, seed=3):
    import torch
    T, L = T or T5, L or L5
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(B, T, 64, generator=g, device=dev).to(torch.bfloat16)
    ctx = torch.randn(B, T, 128, generator=g, device=dev).to(torch.bfloat16)
    enc = torch.randn(B, L, 2048, generator=g, device=dev).to(torch.bfloat16)
    t = torch.full((B,), 0.5, device=dev, dtype=torch.bfloat16)
    return dict(hidden_states=x, timestep=t, timestep_r=t, encoder_hidden_states=enc, context_latents=ctx)


def forward_phases(dit, dev, B, T=None, L=None):
    """Device time of one DiT forward at batch B split by kernel class, without host gaps.

    One eager forward records the calls of each class (the function and its arguments) made by
    layers 0 and 1 (one sliding-window and one full-attention layer; every other layer repeats
    one of them with other weights) and outside the layer loop (embeddings, the encoder K/V of
    all layers, the output projection).  Each class's recorded calls are then captured alone,
    in order, into a CUDA graph and replayed between CUDA events; the in-layer part counts
    num_layers / 2 times.  The whole forward is captured and timed the same way; ``other`` is
    the forward minus the classes (PyTorch glue: concatenations, the AdaLN table sums).  The
    GEMM class gives the roofline: algorithmic FLOPs / its device time."""
    import torch
    from demon_b200 import dit as D
    Q = D.Q
    mods = {"Q": Q, "D": D}
    kw = forward_inputs(dev, B, T, L)
    n_layers = len(dit.layers)
    rep = n_layers / 2.0
    rec = []
    state = {"layer": None, "count": 0}
    with torch.no_grad():
        dit(**kw)
        torch.cuda.synchronize()
        saved = []
        for m, name, cls in PHASE_FUNCS:
            mod = mods[m]
            orig = getattr(mod, name)
            saved.append((mod, name, orig))

            def wrap(*a, _orig=orig, _cls=cls, **k):
                out = _orig(*a, **k)
                if state["layer"] is None or state["layer"] < 2:
                    rec.append((_cls, _orig, a, k, 1.0 if state["layer"] is None else rep))
                return out
            setattr(mod, name, wrap)
        layer_fwd = D.DiTLayer.forward

        def layer_wrap(self, *a, **k):
            state["layer"] = state["count"]
            state["count"] += 1
            try:
                return layer_fwd(self, *a, **k)
            finally:
                state["layer"] = None
        D.DiTLayer.forward = layer_wrap
        try:
            dit(**kw)
        finally:
            for mod, name, orig in saved:
                setattr(mod, name, orig)
            D.DiTLayer.forward = layer_fwd
        torch.cuda.synchronize()
        ms = {"forward": _graph_ms(lambda: dit(**kw))}
        for cls in dict.fromkeys(r_[0] for r_ in rec):
            total = 0.0
            for w in (1.0, rep):
                calls = [(f, a, k) for c, f, a, k, w_ in rec if c == cls and w_ == w]
                if not calls:
                    continue

                def replay(calls=calls):
                    for f, a, k in calls:   # each output is dropped at once: the graph pool reuses it
                        f(*a, **k)
                total += w * _graph_ms(replay)
            ms[cls] = total
    gemms = [(a[0].rows, a[1].rows, a[0].K, k.get("silu_mul", False), w) for c, f, a, k, w in rec if c == "gemm"]
    del rec
    flops = sum(w * 2.0 * m * n * kk for m, n, kk, _, w in gemms)
    ms["other"] = max(0.0, ms["forward"] - sum(v for c, v in ms.items() if c != "forward"))
    # DRAM traffic of the forward's GEMMs: ncu's per-launch bytes at M=12000 for each (N, K),
    # scaled by the launch's rows; launches of other shapes are counted in traffic_flops_covered
    traffic, covered = None, 0.0
    tf = ROOT / "profiles" / "traffic.json"
    if tf.exists():
        per = json.loads(tf.read_text()).get("gemm_M12000", {})
        traffic = 0.0
        for m, n, kk, _, w in gemms:
            b_ = per.get(f"{n}x{kk}")
            if b_ is not None:
                traffic += w * b_ * m / 12000.0
                covered += w * 2.0 * m * n * kk
    alg = sum(w * (m * kk * 0.5625 + n * kk * 0.5625 + m * (n // 2 if sm else n) * 2) for m, n, kk, sm, w in gemms)
    return {"ms": ms, "gemm_launches": sum(w for *_, w in gemms), "gemm_flops": flops,
            "gemm_achieved": flops / (ms["gemm"] * 1e-3) / 1e12, "alg_bytes": alg, "traffic": traffic,
            "traffic_flops_covered": covered / flops if flops else 0.0,
            "method": "per kernel class: the recorded calls of layers 0-1 (x num_layers/2) and outside the "
                      "layer loop, each class captured alone in a CUDA graph and replayed (CUDA events)"}


def tick_phases(r, n=8):
    """Mean device ms per tick of each part of a ring tick over n ticks (CUDA events on the
    launching stream around the decoder forward -- a CUDA-graph replay --, the fused ODE step,
    the finished-latent gather and the control broadcast; the GPU is busy with the forward when
    the ODE and collective events are recorded, so host gaps do not enter them).  A collective's
    time includes waiting for the slowest rank."""
    import torch
    from demon_b200 import ode as O
    acc = {"forward": [], "ode_step": [], "gather": [], "broadcast": []}
    pending = []

    def timed(key, fn):
        def f(*a, **k):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            out = fn(*a, **k)
            e1.record()
            pending.append((key, e0, e1))
            return out
        return f
    pipe, ring = r.pipe, r.ring
    saved = [(pipe, "_forward"), (ring, "gather_finished"), (ring, "broadcast_curves")]
    origs = [getattr(o, nm) for o, nm in saved]
    ode_step = O.OdeTick.step
    try:
        pipe._forward = timed("forward", origs[0])
        ring.gather_finished = timed("gather", origs[1])
        ring.broadcast_curves = timed("broadcast", origs[2])
        O.OdeTick.step = timed("ode_step", ode_step)
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(n):
            r.tick()
        t1.record()
        torch.cuda.synchronize()
    finally:
        for (o, nm), f in zip(saved, origs):
            if o.__dict__.get(nm) is not None:
                del o.__dict__[nm]
        O.OdeTick.step = ode_step
    for key, e0, e1 in pending:
        acc[key].append(e0.elapsed_time(e1))
    out = {k: sum(v) / n for k, v in acc.items()}
    out["tick"] = t0.elapsed_time(t1) / n
    out["other"] = max(0.0, out["tick"] - sum(out[k] for k in acc))
    return out


def count_launches(fn):
    """Kernel launches of our library during fn(): every C-ABI compute call is one launch,
    except a dynamic-scale quantise (three)."""
    from demon_b200 import _native as nat
    L = nat.load()
    names = ["demon_nvfp4_quantize", "demon_nvfp4_gemm", "demon_lora_down", "demon_ode_step", "demon_ode_prepare",
             "demon_bf16_linear", "demon_adanorm_quantize", "demon_silu_mul_quantize", "demon_head_norm_rope"]
    counts = {n: 0 for n in names}
    saved = {n: getattr(L, n) for n in names}

    class Wrap:
        def __init__(self, n, f):
            self.n, self.f = n, f

        def __call__(self, *a):
            counts[self.n] += 3 if (self.n == "demon_nvfp4_quantize" and a[4] == nat.GS_DYNAMIC) else 1
            return self.f(*a)
    try:
        for n in names:
            setattr(L, n, Wrap(n, saved[n]))
        fn()
    finally:
        for n in names:
            setattr(L, n, saved[n])
    return sum(counts.values()), counts


def lora_pairs(dit, dev, rank=64, seed=21, std=0.01):
    """BASELINE config 4's hot LoRA: rank 64, A ~ N(0, 0.01), B ~ N(0, 0.01) (bf16, PEFT
    layout) on every attention q/k/v/o (self and cross) and MLP linear of the DiT."""
    import torch
    from demon_b200.lora import lora_param_names
    g = torch.Generator(device=dev).manual_seed(seed)
    out = {}
    for name, lin in lora_param_names(dit).items():
        if ".self_attn." in name or ".cross_attn." in name or ".mlp." in name:
            A = (torch.randn(rank, lin.in_features, generator=g, device=dev) * std).to(torch.bfloat16)
            B = (torch.randn(lin.out_features, rank, generator=g, device=dev) * std).to(torch.bfloat16)
            out[name] = (A, B)
    return out


def lora_flop_share(pairs, rows, enc_rows):
    """LoRA FLOPs of one forward / its base NVFP4 GEMM FLOPs: 2 M r (K + N) against 2 M N K per
    linear (M = the forward's token rows, or the encoder rows for the cross-attention K / V)."""
    base = extra = 0.0
    for name, (A, B) in pairs.items():
        r, K = A.shape
        N = B.shape[0]
        M = enc_rows if (".cross_attn.k_proj" in name or ".cross_attn.v_proj" in name) else rows
        base += 2.0 * M * N * K
        extra += 2.0 * M * r * (K + N)
    return extra / base


def run_config2(dit, dev):
    """one DiT decoder forward, batch 8 (ring depth 4 x CFG pair), T = 750
    latent frames (375 tokens), text [256, 2048]: the forward as a CUDA-graph replay, with its
    per-class split and GEMM throughput."""
    fp = forward_phases(dit, dev, 8, T=750, L=L5)
    ms = fp["ms"]["forward"]
    return {"workload": "configs[1]: DiT decoder forward, batch 8 (depth 4 x CFG 2), T=750 (375 tokens), "
                        "text [256,2048], all linears NVFP4, random init",
            "ms_per_forward": ms, "forwards_per_s": 1e3 / ms, "gemm_ms": fp["ms"]["gemm"],
            "gemm_tflops": fp["gemm_achieved"], "gemm_flops": fp["gemm_flops"],
            "phases_ms": {k: round(v, 4) for k, v in fp["ms"].items()}}


def run_config4(dit, dev, sweep=32):
    """the hot-LoRA stream.  A depth-8 ring at T = 750 (375 tokens) of
    standard-CFG requests on the DiT with a rank-64 LoRA (A, B ~ N(0, 0.01)) on every attention
    q/k/v/o and MLP linear, enabled at strength 0 while the ring runs, swept 0 -> 1 over 32
    ticks (each tick's strength a kernel scalar; the first non-zero one switches the fused
    projections to per-linear GEMMs and re-captures the decoder graph), then removed (the
    fused graph comes back).  Returns ticks/s of each phase and the LoRA FLOP share."""
    import torch
    from demon_b200.stream import SlotCondition, SlotRequest, StreamConfig, StreamPipeline
    from demon_b200.lora import apply_to_decoder, drop_lora, lora_param_names
    T, depth = 750, 8
    g = torch.Generator().manual_seed(44)
    bf = torch.bfloat16
    ones = torch.ones(1, L5, dtype=bf, device=dev)
    reqs = [SlotRequest(encoder_hidden_states=torch.randn(1, L5, 2048, generator=g).to(bf).to(dev),
                        encoder_attention_mask=ones, context_latents=torch.randn(1, T, 128, generator=g).to(bf).to(dev),
                        seed=900 + k, neg_conditions=[SlotCondition(torch.randn(1, L5, 2048, generator=g).to(bf).to(dev),
                                                                    ones)],
                        guidance_curve=torch.tensor(float(torch.rand(1, generator=g)) * 4 + 3)) for k in range(8)]
    pipe = StreamPipeline(dit, StreamConfig(infer_steps=8), pipeline_depth=depth, device=dev, use_graphs=True)
    n = [0]

    def run_ticks(k, strength_at=None):
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(k):
            if strength_at is not None:
                s_ = strength_at(i)
                for name in pairs:
                    lins[name].lora.set_strength("sweep", s_)
            pipe.submit(reqs[n[0] % len(reqs)])
            n[0] += 1
            pipe.tick()
        e1.record()
        torch.cuda.synchronize()
        return k / (e0.elapsed_time(e1) * 1e-3)
    pairs, lins = {}, {}
    run_ticks(depth + 8)                               # fill + capture the fused graph
    base = run_ticks(16)
    pairs = lora_pairs(dit, dev)
    lins = lora_param_names(dit)
    apply_to_decoder(dit, pairs, [("sweep", True, 0.0, pairs)], linears=lins)   # enabled at strength 0
    at_zero = run_ticks(8)                             # contributes nothing: the fused graph stays
    gen0 = pipe.decoder._gen
    first = run_ticks(1, lambda i: 1.0 / sweep)        # first non-zero strength: re-capture
    recaptured = pipe.decoder._gen != gen0
    rest = run_ticks(sweep - 1, lambda i: (i + 2) / sweep)   # in-place strength updates: replays
    drop_lora(lins, "sweep")                           # the enable / remove cycle ends
    run_ticks(1)                                       # re-capture of the fused graph
    after = run_ticks(8)
    share = lora_flop_share(pairs, 2 * depth * (T // 2), 2 * depth * L5)
    pipe.close()
    return {"workload": "configs[3]: depth-8 ring, T=750 (375 tokens), standard CFG, hot LoRA rank 64 "
                        "(A, B ~ N(0,0.01)) on every attention q/k/v/o (self + cross) and MLP linear, strength "
                        f"0 -> 1 over {sweep} ticks, one enable / remove cycle",
            "base_ticks_per_s": base, "enabled_at_strength0_ticks_per_s": at_zero,
            "first_nonzero_tick_ticks_per_s": first, "lora_ticks_per_s": rest,
            "after_remove_ticks_per_s": after, "lora_linears": len(pairs), "lora_flop_share": share,
            "graph_recaptured_on_first_nonzero": recaptured}


def ring_lora_leg(r, dit, dev, dist_mod, ticks=8):
    """A hot LoRA through the sharded ring at N GPUs: rank 0 enables config 4's rank-64 LoRA
    (its A / B factors are broadcast to every rank), every rank applies it on the same tick,
    ``ticks`` ticks are timed with it on (max over ranks), then rank 0 removes it."""
    import torch
    from demon_b200.lora import lora_param_names
    ring = r.ring
    pairs = lora_pairs(dit, dev) if r.rank == 0 else None
    payload = sum(A.numel() + B.numel() for A, B in pairs.values()) * 2 if pairs else 0
    if r.rank == 0:
        ring.enable_lora("ring-lora", pairs, strength=1.0)
    for _ in range(ring.curve_every + ring.apply_delay + 1):   # announce, land, apply, re-capture
        r.tick()
    torch.cuda.synchronize()
    held = sum(1 for lin in lora_param_names(dit).values() if "ring-lora" in lin.lora.entries)
    held_min = int(-max_over_ranks(-float(held), dist_mod, dev))
    if dist_mod is not None:
        dist_mod.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(ticks):
        r.tick()
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), dist_mod, dev)
    if r.rank == 0:
        ring.disable_lora("ring-lora")
    for _ in range(ring.curve_every + ring.apply_delay + 1):
        r.tick()
    torch.cuda.synchronize()
    left = sum(1 for lin in lora_param_names(dit).values() if "ring-lora" in lin.lora.entries)
    return {"ticks_per_s": ticks / (ms * 1e-3), "ticks": ticks, "linears_with_lora_min_over_ranks": held_min,
            "linears_with_lora_after_remove": left, "payload_bytes_broadcast": payload,
            "note": "rank-64 LoRA on every attention and MLP linear enabled on rank 0 and broadcast (NCCL) "
                    "to every rank with the ring's control broadcast; timed with it on"}


def cpu_stream_sample(budget_s: float, max_steps: int | None = None, min_steps: int = 1):
    """The reference's CPU path for whole slot-steps of the tick: one slot's CFG pair (B=2, 750
    tokens) through all 24 layers of the CPU restatement of AceStepDiTModel (oracle/dit_ref.py,
    bit-exact with the reference module; the 24 layers share two layers' weights, which changes
    no arithmetic) and then the CPU ODE-step oracle on [1500, 64] (CFG, APG, curves, DCW),
    repeated while the budget lasts (at least ``min_steps``, at most ``max_steps``).  Returns
    the measured seconds per slot-step and the sample's size."""
    import numpy as np
    import torch
    from oracle.dit_ref import DiTRef
    from oracle import ode_oracle as OO
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    D, NL = 2048, 24
    g = torch.Generator().manual_seed(0)
    sd = {}
    for i in range(2):
        p = f"layers.{i}"
        for nm, shp in ((".self_attn.q_proj", (2048, D)), (".self_attn.k_proj", (1024, D)),
                        (".self_attn.v_proj", (1024, D)), (".self_attn.o_proj", (D, 2048)),
                        (".cross_attn.q_proj", (2048, D)), (".cross_attn.k_proj", (1024, D)),
                        (".cross_attn.v_proj", (1024, D)), (".cross_attn.o_proj", (D, 2048)),
                        (".mlp.gate_proj", (6144, D)), (".mlp.up_proj", (6144, D)), (".mlp.down_proj", (D, 6144))):
            sd[p + nm + ".weight"] = (torch.randn(shp, generator=g) / shp[1] ** 0.5).to(torch.bfloat16)
        for nm in (".self_attn_norm", ".cross_attn_norm", ".mlp_norm"):
            sd[p + nm + ".weight"] = torch.ones(D, dtype=torch.bfloat16)
        for nm in (".self_attn.q_norm", ".self_attn.k_norm", ".cross_attn.q_norm", ".cross_attn.k_norm"):
            sd[p + nm + ".weight"] = torch.ones(128, dtype=torch.bfloat16)
        sd[p + ".scale_shift_table"] = (torch.randn(1, 6, D, generator=g) / D ** 0.5).to(torch.bfloat16)
    for i in range(2, NL):
        for k in [k for k in sd if k.startswith(f"layers.{i % 2}.")]:
            sd[f"layers.{i}." + k.split(".", 2)[2]] = sd[k]
    ref = DiTRef(sd, {"num_hidden_layers": NL, "sliding_window": 128})
    S = T5 // 2
    h0 = torch.randn(2, S, D, generator=g).to(torch.bfloat16)
    tproj = (torch.randn(2, 6, D, generator=g) * 0.1).to(torch.bfloat16)
    enc = torch.randn(2, L5, D, generator=g).to(torch.bfloat16)
    rope = ref.rope(S, torch.bfloat16)
    masks = [ref.mask4d(S, torch.bfloat16, 128), ref.mask4d(S, torch.bfloat16, None)]
    menc = ref.mask4d(max(S, L5), torch.bfloat16, None)[:, :, :S, :L5]
    rng = np.random.default_rng(0)
    lat = lambda: rng.standard_normal((T5, 64)).astype(np.float32)
    slot = dict(xt=lat(), pos=[(lat(), None)], neg=[(lat(), None)], momentum=lat(), has_cfg=True,
                rcfg_mode=None, guidance=np.full(T5, 5.0, np.float32), apg_momentum=-0.75, cfg_rescale=None,
                velocity_scale=np.ones(T5, np.float32), t_curr=0.75, t_next=0.5, step_idx=3, total_steps=8,
                infer_method="ode", noise=None, dec_next=True, dcw=("double", 0.05, 0.02))

    def slot_step():
        h = h0
        for i in range(NL):
            h = ref.layer(i, h, tproj, enc, rope, masks[i % 2], menc)
        OO.step_slot(dict(slot))
        return h
    with torch.no_grad():
        ref.layer(0, h0, tproj, enc, rope, masks[0], menc)  # warm-up
        n, t0 = 0, time.perf_counter()
        while True:
            slot_step()
            n += 1
            el = time.perf_counter() - t0
            if n >= min_steps and (el >= budget_s or (max_steps and n >= max_steps)):
                break
    return {"per_slot_step_s": el / n, "slot_steps": n, "seconds": el, "cores": cores,
            "sample": f"{n} complete slot-steps ({NL} DiT layers of one slot's CFG pair, B=2, 750 tokens, on "
                      f"the CPU restatement of AceStepDiTModel, bit-exact with the reference module, + the CPU "
                      f"ODE-step oracle) in {el:.1f} s on {cores} cores, {el / n:.2f} s each; a tick is {RING} "
                      f"slot-steps, so ticks/s = 1 / ({RING} x seconds per slot-step)"}


def stream_config(world):
    """The config dict of the stream workload, printed identically by both arms."""
    return dict(CONFIG5, parallelism=f"slot-sharded ring x{world} ({RING // world} slots per GPU)",
                prefill_ticks=STEPS5)


def run_stream(args):
    import torch
    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist_mod = dist_init(world)
    from demon_b200 import _build
    if rank == 0 or not (ROOT / "demon_b200" / "libdemon_b200.so").exists():
        _build.build()
    if dist_mod is not None:
        dist_mod.barrier()
    from demon_b200 import _native as nat
    if RING % world:
        raise SystemExit(f"--gpus must divide {RING}")
    dit = build_dit(dev)
    tm_dev = request_templates(dev)
    r = Ring(dit, dev, rank, world, tm_dev)
    stream = torch.cuda.current_stream(dev)
    # prefill: STEPS5 ticks fill the ring with staggered slots; then W warm-up ticks
    for _ in range(STEPS5 + args.warmup):
        r.tick()
    torch.cuda.synchronize()

    def timed(n, on_finished=None, sampler=None):
        if dist_mod is not None:
            dist_mod.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            r.tick(on_finished)
        e1.record(stream)
        torch.cuda.synchronize()
        if dist_mod is not None:
            dist_mod.barrier()
        return max_over_ranks(e0.elapsed_time(e1), dist_mod, dev)

    with ClockSampler(local) as clk:
        ms = timed(args.steps)
    graphed = r.pipe.decoder
    r.pipe.decoder = graphed.decoder          # one eager tick: every launch goes through the C ABI
    try:
        n_launch, per_kind = count_launches(lambda: (r.tick(), torch.cuda.synchronize()))
    finally:
        r.pipe.decoder = graphed
    # end to end: request inputs from pinned host memory, finished latents back to pinned host
    tm_host = request_templates(dev, pin=True)
    r.set_templates(tm_host)
    fin_host = [torch.empty(1, T5, 64, dtype=torch.bfloat16).pin_memory() for _ in range(r.local)]

    def to_host(fin):
        for i, f in enumerate(fin):
            fin_host[i].copy_(f, non_blocking=True)
    for _ in range(2):
        r.tick(to_host)
    e2e_ms = timed(args.steps, to_host)
    r.set_templates(tm_dev)
    status = nat.device_status()
    if not args.legs:  # the timed stream only (the launch-list profile uses this form)
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": args.steps / (ms * 1e-3), "unit": "ticks/s",
                              "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                              "ms_per_step": ms / args.steps, "e2e_ticks_per_s": args.steps / (e2e_ms * 1e-3),
                              "config": stream_config(world), "note": "--no-legs: secondary legs skipped",
                              "device_status": list(status)}), flush=True)
        if dist_mod is not None:
            r.pipe.decoder._graphs.clear()
            dist_mod.barrier()
            dist_mod.destroy_process_group()
        return
    # where a tick's time goes on this rank (then max over ranks per phase)
    tp = tick_phases(r, n=8)
    tp_max = {k: max_over_ranks(v, dist_mod, dev) for k, v in tp.items()}
    fp = forward_phases(dit, dev, B=2 * r.local)
    fp_max = {k: max_over_ranks(v, dist_mod, dev) for k, v in fp["ms"].items()}
    lora_ring = ring_lora_leg(r, dit, dev, dist_mod)
    if rank == 0:
        pk = peaks()
        quant = measure_quantize_big(dev, stream, M=2 * r.local * (T5 // 2))
        odek = measure_ode(dev, stream) if args.ode else None
        lin = linear_leg(dev, stream)
        attn = attention_leg(dev, B=2 * r.local)
        cfg3 = run_config3(dit, dev) if world == 1 else None
        cfg2 = run_config2(dit, dev) if world == 1 else None
        cfg4 = run_config4(dit, dev) if world == 1 else None
        cpu = None
        if world == 1 and args.cpu_seconds > 0:
            c = cpu_stream_sample(args.cpu_seconds)
            cpu = {"value": 1.0 / (RING * c["per_slot_step_s"]), "unit": "ticks/s", "cores": c["cores"],
                   "kind": "port", "sample": c["sample"], "extrapolated": True, "scale_factor": RING}
        achieved = fp["gemm_achieved"]
        fp4_peak = 4.0 * pk.get("bf16_sustained", pk["bf16_tflops"])
        new_bytes = 2 * L5 * 2048 * 2 + T5 * 128 * 2
        line = {
            "metric": METRIC, "value": args.steps / (ms * 1e-3), "unit": "ticks/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "nvfp4 linears (e2m1 x ue4m3 blocks, fp32 accumulate), bf16 elsewhere",
            "data": "synthetic (random-init weights, N(0,1) inputs)",
            "config": stream_config(world),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": fp4_peak, "unit": "TFLOP/s",
                         "frac": achieved / fp4_peak, "traffic": fp["traffic"],
                         "traffic_note": "DRAM bytes of all GEMM launches of one forward: ncu "
                                         "dram__bytes_read+write per launch at M=12000 for each (N, K), scaled "
                                         "by the launch's rows (profiles/traffic.json); covers "
                                         f"{100 * fp['traffic_flops_covered']:.1f} % of the GEMM FLOPs; "
                                         "algorithmic bytes (operands + bf16 outputs) "
                                         f"{fp['alg_bytes'] / 1e9:.2f} GB",
                         "peak_note": "FP4 dense peak taken as 4x the measured sustained bf16 cuBLAS figure "
                                      f"({pk.get('bf16_sustained', pk['bf16_tflops']):.0f} TF/s, of measured: the "
                                      f"GEMMs run inside a long step); nominal 9 PF/s -> frac {achieved / 9000.0:.3f}",
                         "kernel": "demon::gemm_kernel (all NVFP4 GEMMs of one DiT forward at the rank's batch)",
                         "gemm_launches": fp["gemm_launches"], "gemm_ms_per_forward": fp["ms"]["gemm"],
                         "gemm_ms_per_forward_max_over_ranks": fp_max["gemm"], "method": fp["method"]},
            "phases": {"tick_ms": {k: round(v, 4) for k, v in tp.items()},
                       "tick_ms_max_over_ranks": {k: round(v, 4) for k, v in tp_max.items()},
                       "forward_ms": {k: round(v, 4) for k, v in fp["ms"].items()},
                       "forward_ms_max_over_ranks": {k: round(v, 4) for k, v in fp_max.items()},
                       "note": "tick: CUDA events around the graph-replayed forward, the ODE launch, the gather "
                               "and the control broadcast over 8 ticks (collectives include waiting for the "
                               "slowest rank); forward: " + fp["method"]},
            "e2e": {"value": args.steps / (e2e_ms * 1e-3), "unit": "ticks/s",
                    "h2d_bytes_per_step": world * r.k_new * new_bytes,
                    "d2h_bytes_per_step": world * r.k_new * T5 * 64 * 2},
            "gpu_launches": n_launch * args.steps,
            "gpu_launches_per_tick": per_kind,
            "clocks": clk.summary(),
            "device_status": list(status),
            "kernels": {"quantize": dict(quant, peak=pk["hbm_gbs"], frac=quant["achieved"] / pk["hbm_gbs"]),
                        "nvfp4_linear_config1": lin, "attention": attn},
            "secondary": {"lora_through_ring": lora_ring},
        }
        if odek is not None:
            line["kernels"]["ode_step"] = dict(odek, peak=pk["hbm_gbs"], frac=odek["achieved"] / pk["hbm_gbs"])
        for k, v in (("config3_stream", cfg3), ("config2_forward", cfg2), ("config4_hot_lora", cfg4)):
            if v is not None:
                line["secondary"][k] = v
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if dist_mod is not None:
        r.pipe.decoder._graphs.clear()
        dist_mod.barrier()
        dist_mod.destroy_process_group()


def run_reference_stream(args):
    """The reference arm: the reference's CPU path (its DiT forward and ODE step, restated
    bit-exactly) on this host's cores, each step one complete slot-step; ticks/s is
    extrapolated from the measured seconds per slot-step (a tick is 64 slot-steps)."""
    rank, world, _ = env_rank()
    if rank != 0:
        return
    c0 = time.perf_counter()
    cpu_stream_sample(0.0, max_steps=max(1, min(args.warmup, 3)))        # warm-up slot-steps
    c = cpu_stream_sample(150.0, max_steps=args.steps, min_steps=args.steps)
    v = 1.0 / (RING * c["per_slot_step_s"])
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "ticks/s", "n_gpus": args.gpus,
        "steps": c["slot_steps"], "warmup": args.warmup, "ms_per_step": 1e3 / v, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": stream_config(world),
        "extrapolated": True, "scale_factor": RING,
        "sampled": {"slot_steps": c["slot_steps"], "seconds": c["seconds"], "per_slot_step_s": c["per_slot_step_s"],
                    "wall_s_incl_warmup": time.perf_counter() - c0},
        "cpu_baseline": {"value": v, "unit": "ticks/s", "cores": c["cores"], "kind": "port", "sample": c["sample"],
                         "extrapolated": True, "scale_factor": RING},
        "e2e": {"value": v, "unit": "ticks/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_kernel_workload(args):
    """Kernel-level workloads (one GPU), also the commands the ncu summaries under profiles/ use:
    ``gemm``: NVFP4 linears of shapes ``--shape M,N,K[:M,N,K...]`` (inputs quantised and weights
    packed before timing), launched shape by shape in each warm-up and timed pass;
    ``rows``: the 64-slot ODE step, the AdaLN-RMSNorm quantiser on [M, 2048], SiLU*up on
    [M, 12288] and the activation quantiser on [M, 2048] (M = ``--shape`` when it is one
    number, else 12000; the tick's is 96000);
    ``attention``: the DiT's band (window 128), global and cross attention over ``--seqs``
    sequences of 750 tokens (GQA 16/8 x 128, text 256), with ``--vs-cudnn`` also the cuDNN
    kernels on the same inputs;
    ``layer``: the six NVFP4 GEMMs of a DiT layer at M rows (``--shape`` when it is one number,
    else 96000: the tick's) with their epilogues -- q/k/v with head norm + RoPE, o_proj and down
    with the AdaLN gate (one row per 750 tokens) and the residual, the cross-attention q with
    head norm, the cross-attention o with the residual, gate/up with SwiGLU -- each beside the
    same operands without the epilogue, ``--steps`` launches of each replayed from a CUDA graph.
    Prints per-launch times."""
    import torch
    from demon_b200 import _build, _native as nat, nvfp4
    _build.build()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    launches = []
    if args.workload == "gemm":
        for shape in args.shape.split(":"):
            M, N, K = (int(v) for v in shape.split(","))
            x = torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16)
            w = (torch.randn(N, K, generator=g, device=dev) * 0.02).to(torch.bfloat16)
            a, pw = nvfp4.quantize(x), nvfp4.pack_weight(w)
            out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
            launches.append((f"gemm {M}x{N}x{K}", 2.0 * M * N * K,
                             lambda a=a, pw=pw, out=out: nvfp4.gemm(a, pw, out=out)))
            if args.vs_cublaslt:  # the library's block-scaled NVFP4 GEMM on the same packed operands
                fa, fb = a.codes.view(torch.float4_e2m1fn_x2), pw.codes.view(torch.float4_e2m1fn_x2).t()
                sa, sb = a.sf.view(torch.float8_e4m3fn), pw.sf.view(torch.float8_e4m3fn)
                launches.append((f"cublaslt {M}x{N}x{K}", 2.0 * M * N * K,
                                 lambda fa=fa, fb=fb, sa=sa, sb=sb: torch._scaled_mm(
                                     fa, fb, sa, sb, out_dtype=torch.bfloat16)))
    elif args.workload == "layer":
        M, S = (int(args.shape) if args.shape.isdigit() else 96000), 750
        hq, hk = 16, 8

        def wt(n, k):
            return nvfp4.pack_weight((torch.randn(n, k, generator=g, device=dev) * 0.03).to(torch.bfloat16))
        a2 = nvfp4.quantize(torch.randn(M, 2048, generator=g, device=dev).to(torch.bfloat16))
        a6 = nvfp4.quantize(torch.randn(M, 6144, generator=g, device=dev).to(torch.bfloat16))
        wqkv, wo, wd = wt((hq + 2 * hk) * 128, 2048), wt(2048, 2048), wt(2048, 6144)
        wu = nvfp4.interleave_weights(wt(6144, 2048), wt(6144, 2048))
        resid = torch.randn(M, 2048, generator=g, device=dev).to(torch.bfloat16)
        gate = torch.randn((M + S - 1) // S, 2048, generator=g, device=dev).to(torch.bfloat16)
        nw = (1 + 0.1 * torch.randn(128, generator=g, device=dev)).to(torch.bfloat16)
        pos = torch.arange(S, dtype=torch.float32, device=dev)
        inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, device=dev).float() / 128))
        emb = torch.cat([pos[:, None] * inv[None]] * 2, -1)
        rope = (emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16), S, True)  # equal halves, as the DiT's
        o4, o2 = (torch.empty(M, n, dtype=torch.bfloat16, device=dev) for n in (4096, 2048))
        o6 = torch.empty(M, 6144, dtype=torch.bfloat16, device=dev)
        o12 = torch.empty(M, 12288, dtype=torch.bfloat16, device=dev)
        hn_qkv, hn_q = ((hq + hk) * 128, hq * 128, nw, nw, 1e-6), (2048, 2048, nw, None, 1e-6)
        fl = 2.0 * M * 2048
        launches += [
            ("qkv head_norm+rope", fl * 4096, lambda: nvfp4.gemm(a2, wqkv, head_norm=hn_qkv, rope=rope, out=o4)),
            ("qkv plain", fl * 4096, lambda: nvfp4.gemm(a2, wqkv, out=o4)),
            ("o_proj gate+residual", fl * 2048,
             lambda: nvfp4.gemm(a2, wo, residual=resid, gate=gate, gate_rows=S, out=o2)),
            ("o_proj plain", fl * 2048, lambda: nvfp4.gemm(a2, wo, out=o2)),
            ("cross_q head_norm", fl * 2048, lambda: nvfp4.gemm(a2, wo, head_norm=hn_q, out=o2)),
            ("cross_o residual", fl * 2048, lambda: nvfp4.gemm(a2, wo, residual=resid, out=o2)),
            ("gate_up swiglu", fl * 12288, lambda: nvfp4.gemm(a2, wu, silu_mul=True, out=o6)),
            ("gate_up plain", fl * 12288, lambda: nvfp4.gemm(a2, wu, out=o12)),
            ("down gate+residual", fl * 6144,
             lambda: nvfp4.gemm(a6, wd, residual=resid, gate=gate, gate_rows=S, out=o2)),
            ("down plain", fl * 6144, lambda: nvfp4.gemm(a6, wd, out=o2)),
        ]
    elif args.workload == "attention":
        from demon_b200.attention import attention
        B, S, L, hq, hk, D = args.seqs, 750, L5, 16, 8, 128
        qkv = torch.randn(B * S, (hq + 2 * hk) * D, generator=g, device=dev).to(torch.bfloat16)
        ld = qkv.stride(0)
        q = qkv.as_strided((B, S, hq, D), (S * ld, ld, D, 1))
        k = qkv.as_strided((B, S, hk, D), (S * ld, ld, D, 1), hq * D)
        v = qkv.as_strided((B, S, hk, D), (S * ld, ld, D, 1), (hq + hk) * D)
        kvx = torch.randn(B * L, 2 * hk * D, generator=g, device=dev).to(torch.bfloat16)
        lk = kvx.stride(0)
        ck = kvx.as_strided((B, L, hk, D), (L * lk, lk, D, 1))
        cv = kvx.as_strided((B, L, hk, D), (L * lk, lk, D, 1), hk * D)
        qc = torch.randn(B, S, hq, D, generator=g, device=dev).to(torch.bfloat16)
        out = torch.empty(B, S, hq, D, dtype=torch.bfloat16, device=dev)
        n_band = sum(min(i + 128, S - 1) - max(i - 128, 0) + 1 for i in range(S))
        launches += [("attention band", 4.0 * B * hq * n_band * D, lambda: attention(q, k, v, 128, out=out)),
                     ("attention global", 4.0 * B * hq * S * S * D, lambda: attention(q, k, v, out=out)),
                     ("attention cross", 4.0 * B * hq * S * L * D, lambda: attention(qc, ck, cv, out=out))]
        if args.vs_cudnn:
            from torch.nn.attention import SDPBackend, sdpa_kernel
            band = _CudnnBand()

            def sdpa(qq, kk, vv):
                with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
                    return torch.nn.functional.scaled_dot_product_attention(
                        qq.transpose(1, 2), kk.transpose(1, 2), vv.transpose(1, 2), enable_gqa=True)
            launches += [("cudnn band", 4.0 * B * hq * n_band * D, lambda: band(q, k, v, 128)),
                         ("cudnn global", 4.0 * B * hq * S * S * D, lambda: sdpa(q, k, v)),
                         ("cudnn cross", 4.0 * B * hq * S * L * D, lambda: sdpa(qc, ck, cv))]
    else:
        from demon_b200.rowops import adanorm_quantize, silu_mul_quantize
        tick, nbytes, gain = ode_workload(dev, nslots=64, T=1500, seed=0)
        b, nb = tick._stage()
        tick._dev[b][:nb].copy_(tick._host[b][:nb])
        M, D, F = (int(args.shape) if args.shape.isdigit() else 12000), 2048, 6144
        h = torch.randn(M, D, generator=g, device=dev).to(torch.bfloat16)
        w = torch.ones(D, device=dev, dtype=torch.bfloat16)
        nmod = (M + 749) // 750  # one modulation row per 750-token sequence
        sc = torch.ones(nmod, D, device=dev, dtype=torch.bfloat16)
        sh = torch.zeros(nmod, D, device=dev, dtype=torch.bfloat16)
        gu = torch.randn(M, 2 * F, generator=g, device=dev).to(torch.bfloat16)
        launches += [
            ("ode_step", nbytes, lambda: nat.check(nat.load().demon_ode_step(
                tick._dev[b].data_ptr(), len(tick.slots), tick.T, 64, nat.ptr(gain), nat.stream_ptr()))),
            ("adanorm_quantize", M * D * 2.5625 + M * 4, lambda: adanorm_quantize(h, w, 1e-6, sc, sh, 750)),
            ("silu_mul_quantize", M * 2 * F * 2 + M * F * 0.5625 + M * 4, lambda: silu_mul_quantize(gu, F)),
            ("quantize", M * D * 2.5625 + M * 4, lambda: nvfp4.quantize(h)),
        ]
    for _ in range(max(args.warmup, 3)):
        for _, _, f in launches:
            f()
    torch.cuda.synchronize()
    res = {}
    for name, work, f in launches:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if args.workload == "layer":  # replayed from a CUDA graph: no host work between launches
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                for _ in range(args.steps):
                    f()
            gr.replay()
            torch.cuda.synchronize()
            e0.record()
            gr.replay()
            e1.record()
        else:
            e0.record()
            for _ in range(args.steps):
                f()
            e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / args.steps
        flops = args.workload in ("gemm", "attention", "layer")
        unit = "TFLOP/s" if flops else "GB/s"
        res[name] = {"us": us, unit: work / (us * 1e-6) / (1e12 if flops else 1e9)}
    print(json.dumps({"workload": args.workload, "shape": args.shape, "steps": args.steps, "kernels": res,
                      "device_status": list(nat.device_status())}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="stream", choices=["stream", "linear", "gemm", "rows", "attention", "layer"])
    ap.add_argument("--seqs", type=int, default=128, help="sequences of 750 tokens for --workload attention")
    ap.add_argument("--vs-cudnn", action="store_true",
                    help="with --workload attention: also time the cuDNN attention kernels on the same inputs")
    ap.add_argument("--vs-cublaslt", action="store_true",
                    help="with --workload gemm: also time cuBLASLt's NVFP4 GEMM (torch._scaled_mm) on the same operands")
    ap.add_argument("--shape", default="12000,6144,2048", help="M,N,K[:M,N,K...] of --workload gemm")
    ap.add_argument("--cpu-seconds", type=float, default=20.0)
    ap.add_argument("--no-ode", dest="ode", action="store_false", help="skip the ODE-step roofline leg")
    ap.add_argument("--no-legs", dest="legs", action="store_false",
                    help="stream: time the stream and its e2e run only (no phase split, kernel or config legs)")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = {"stream": 20, "linear": 2000}.get(args.workload, 10)
    if args.warmup is None:
        args.warmup = 3 if args.workload == "stream" else 10
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        (run_reference_stream if args.workload == "stream" else run_reference)(args)
        return
    if args.workload in ("gemm", "rows", "attention", "layer"):
        run_kernel_workload(args)
        return
    (run_stream if args.workload == "stream" else run_linear)(args)


if __name__ == "__main__":
    main()
