"""Benchmark of the DEMON hot path on B200 (driver contract: one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload linear]

Workload ``linear``: one NVFP4 linear y = x W^T + b with
x bf16 [1500, 2048] (N(0,1), 1% of channels x20), W [6144, 2048] (N(0, 0.02)),
bias 0.  One step = quantise x (per-row global scale) + block-scaled tcgen05
GEMM with the bias epilogue.  Each step uses a different (x, W, y) buffer set
from a rotation whose footprint exceeds 2x the 126 MB L2, so no step reads
another step's data from L2.  Multi-GPU: one process per GPU, each rank runs the
same per-GPU work (replicas, weak scaling); the timed region is bracketed by a
barrier and synchronize on both sides, and the reported time is the max over
ranks.

``--impl reference`` times the reference's CPU path for the same workload on
this host's cores: the reference's linear is ``nn.Linear`` in bf16
(acestep/models/modeling_acestep_v15_turbo.py:286-289), i.e. torch F.linear.
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
METRIC = "NVFP4 linear TFLOPS (% FP4 peak); DiT stream ticks/sec, depth 8, 1-8 GPUs"


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
    return {"hbm_gbs": hbm, "bf16_tflops": bf16, "fp4_tflops": 4.0 * bf16, "source": src}


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
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
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
# Our path
# ---------------------------------------------------------------------------

def ode_workload(dev, nslots=64, T=1500, seed=0):
    """Config-3 slot features at config-5 scale: 64 slots x T=1500 x 64, CFG modes cycling
    standard / RCFG-initialize (cached negative) / RCFG-self, per-slot guidance U(3,7),
    per-frame velocity_scale / sde_denoise / apg_momentum / cfg_rescale splines in [0, 1.5],
    source latents (SDE-curve path), binary latent mask with 40 % spans, channel gain U(0.8, 1.2).
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
            dec_out=torch.empty(T, D, dtype=bf, device=dev), seed=1000 + i)
        tick.add(st)
        # reads: v_pos, v_neg source, momentum, xt, mask original + noise, source, gain; writes: momentum, xt, dec
        nbytes += elems * 2 * (8 + 3)
    return tick, nbytes, gain


def measure_ode(dev, stream, reps=20):
    """HBM roofline of the fused ODE step: two slot sets (2 x 135 MB > 2x L2) alternated."""
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
                         "kernel": "demon::gemm_kernel<256,4,true,0>", "gemm_us": gemm_avg * 1e3},
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="linear", choices=["linear"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-ode", dest="ode", action="store_false", help="skip the ODE-step roofline leg")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
        return
    run_linear(args)


if __name__ == "__main__":
    main()
