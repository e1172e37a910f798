"""Benchmark of the shift-window hot path: accumulate_uz on the large
int64 configuration: one 8192 x 8192 image,
x fp16 (1, 3, 8192, 8192) ~ U[0,1], R = 10 half-plane table (S = 221),
channel-shared fp16 weights (221, 1, 8192, 8192) = softplus(N(0,1)) x box
mask (14.8e9 weight elements, 29.7 GB), U and Z in fp32.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one accumulate_uz forward over the whole image.  With N > 1
(torchrun, one rank per GPU) the image is split into N row bands with an
R-row halo and mirror-strip exchange over NCCL; the total work is fixed
("strong" scaling).  Metric: pixel-shifts/s = S*B*C*H*W per step / time.

`--impl reference` times the reference algorithm's CPU path (the oracle's
restatement of neural_shift_cuda's PyTorch implementation, all host cores)
on a bounded row band of the same workload; rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B, C, HG, WG, R = 1, 3, 8192, 8192, 10
METRIC = "pixel-shifts/s (accumulate_uz fwd, 8192^2 x3, S=221, fp16 in / fp32 acc)"
UNIT = "pixel-shifts/s"


def halfplane(R):
    rows = [(dx, dy, 1) for dx in range(-R, R + 1) for dy in range(1, R + 1)]
    rows += [(dx, 0, int(dx != 0)) for dx in range(0, R + 1)]
    return rows


ROWS = halfplane(R)
S = len(ROWS)
PIXEL_SHIFTS = S * B * C * HG * WG


def algorithmic_bytes(Hb: int) -> int:
    """Unique bytes of one band launch: weights once (channel-shared, fp16),
    x once (fp16), U and Z once (fp32)."""
    return S * B * Hb * WG * 2 + B * C * Hb * WG * 2 + 2 * B * C * Hb * WG * 4


# ---------------------------------------------------------------------------
# synthetic inputs
# ---------------------------------------------------------------------------

def make_band(row0: int, Hb: int, device, seed: int = 0):
    """x rows [row0, row0+Hb) and the matching rows of every weight plane,
    generated plane by plane on the device (seed depends only on the plane
    and row range, so any band split sees the same global data)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = torch.rand((B, C, HG, WG), generator=g, device=device,
                   dtype=torch.float32)[:, :, row0:row0 + Hb]
    x = x.to(torch.float16).contiguous()
    w = torch.empty((S * B, 1, Hb, WG), dtype=torch.float16, device=device)
    rows = torch.arange(row0, row0 + Hb, device=device)
    cols = torch.arange(WG, device=device)
    for s, (dx, dy, _) in enumerate(ROWS):
        g.manual_seed(seed * 100003 + s + 1)
        plane = torch.randn((HG, WG), generator=g, device=device)[row0:row0 + Hb]
        m = (((rows + dx >= 0) & (rows + dx < HG))[:, None]
             & ((cols + dy >= 0) & (cols + dy < WG))[None, :])
        w[s, 0] = (torch.nn.functional.softplus(plane) * m).to(torch.float16)
        del plane
    return x, w


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------

class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,"
             "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}",
                 f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"),
                stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                 "sw_power_cap"]
        for line in open(self.path):
            f = [v.strip() for v in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": mx, "samples": len(sm),
                "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# CPU reference arm
# ---------------------------------------------------------------------------

def cpu_reference(rows_sample: int = 8, reps: int = 1):
    """Time the reference algorithm on the host: the oracle restatement of
    neural_shift_cuda's PyTorch accumulate_uz (promotion to fp32, per-shift
    circular slices, pairwise tree sum) on a (1, 3, rows_sample, 8192) band
    with all 221 weight planes.  Returns (pixel-shifts/s, description)."""
    from oracle import nsc_oracle as O
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    x = torch.rand(B, C, rows_sample, WG, generator=g).half()
    w = torch.nn.functional.softplus(
        torch.randn(S * B, 1, rows_sample, WG, generator=g)).half()
    w = w.expand(-1, C, -1, -1)  # the reference API takes (S*B, C, H, W)
    sh = torch.tensor(ROWS)
    O.accumulate_uz(x[:, :, :2], w[:, :, :2].contiguous(), sh)  # warm
    t0 = time.perf_counter()
    for _ in range(reps):
        O.accumulate_uz(x, w.contiguous(), sh)
    dt = (time.perf_counter() - t0) / reps
    work = S * B * C * rows_sample * WG
    return work / dt, threads, dt, (
        f"oracle accumulate_uz (torch CPU, {threads} threads) on a "
        f"(1, 3, {rows_sample}, 8192) band, S=221, fp16 inputs promoted to fp32")


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    vals, dts = [], []
    for _ in range(args.warmup):
        cpu_reference(args.ref_rows)
    for _ in range(args.steps):
        v, threads, dt, desc = cpu_reference(args.ref_rows)
        vals.append(v)
        dts.append(dt)
    v = statistics.median(vals)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        # a step is one timed sample (the bounded band); the whole image at
        # the sample's rate is reported beside it, not as the step time
        "ms_per_step": statistics.median(dts) * 1e3,
        "ms_full_workload_at_sample_rate": PIXEL_SHIFTS / v * 1e3,
        "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "accumulate_uz 8192x8192x3 R=10 S=221 (configs[4])",
                   "sample_rows": args.ref_rows},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads,
                         "kind": "port", "sample": desc},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def run_ours(args):
    import torch.distributed as dist
    import neural_shift_cuda_b200 as nsc
    from neural_shift_cuda_b200 import bands

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    row0, Hb = bands.band_rows(HG, world, rank)
    x, w = make_band(row0, Hb, dev)
    sh = torch.tensor(ROWS)
    torch.cuda.synchronize()

    if world == 1:
        def step():
            return nsc.accumulate_uz(x, w, sh)
        launches_per_step = 1
    else:
        # the rank's x band lives in a buffer with R spare rows on each side;
        # the halo exchange fills them in place every step
        x_pad = torch.empty((B, C, Hb + 2 * R, WG), dtype=x.dtype, device=dev)
        x_pad[:, :, R:R + Hb] = x

        def step():
            return bands.accumulate_uz_banded(x_pad, w, sh, HG, padded=True)
        launches_per_step = 2 if R else 1   # edge strips + band forward

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    stream = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    # the clock sampler starts before the warm-up so the GPU does not idle
    # between warm-up and the timed steps
    with ClockSampler(local) as clk:
        torch.cuda.nvtx.range_push("warmup")   # loads NVTX outside the timed steps
        # hold each result until the next step returns, as the timed loop
        # does, so the allocator has both output sets before timing starts
        out = None
        for _ in range(args.warmup):
            out = step()
        torch.cuda.nvtx.range_pop()
        barrier()
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("timed")
        t_start.record(stream)
        for i in range(args.steps):
            ev[i][0].record(stream)
            out = step()
            ev[i][1].record(stream)
        t_end.record(stream)
        torch.cuda.nvtx.range_pop()
        barrier()
    total_ms = t_start.elapsed_time(t_end)
    step_ms = [a.elapsed_time(b) for a, b in ev]
    if world > 1:
        t = torch.tensor([total_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms = total_ms / args.steps
    value = PIXEL_SHIFTS / (ms * 1e-3)

    # kernel-only time of the dominant kernel: with N == 1 the step is one
    # launch of the accumulate kernel, so its event time is the kernel time.
    kern_ms = statistics.median(step_ms)
    alg = algorithmic_bytes(Hb)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    traffic = None
    if world == 1 and HG == 8192:
        # DRAM bytes per launch of this kernel from the committed ncu summary
        try:
            for line in open(os.path.join(ROOT, "profiles",
                                          "accumulate_uz_fwd_8192x8192_S221.md")):
                if line.startswith("dram_bytes_per_launch:"):
                    traffic = int(line.split(":")[1])
        except OSError:
            pass
    achieved = alg / (kern_ms * 1e-3) / 1e9

    # correctness spot check on the benchmark data: U(x = 1) == Z is exact in
    # the kernel's summation order; here check a cheap property of the run.
    U, Z = out
    ok = bool(torch.isfinite(U).all().item() and (Z >= 0).all().item())

    # end-to-end through the public API with host buffers (rank-local band)
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, x, w, sh, world, dev)

    clocks = clk.summary()
    if rank == 0:
        cpu = None
        if not args.no_cpu and world == 1:
            v, threads, dt, desc = cpu_reference(args.ref_rows, reps=3)
            cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                   "sample": desc}
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f16 in, f32 accumulate", "data": "synthetic",
            "config": {"workload": "accumulate_uz 8192x8192x3 R=10 S=221 "
                                   "channel-shared fp16 weights (configs[4])",
                       "B": B, "C": C, "H": HG, "W": WG, "S": S,
                       "parallelism": f"row bands x{world}" if world > 1 else "single GPU",
                       "l2": "inputs (29.7 GB) larger than L2"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak,
                         "unit": "GB/s", "frac": achieved / peak,
                         "traffic": traffic,
                         "traffic_source": ("from profile: dram__bytes_read.sum + "
                                            "dram__bytes_write.sum of one ncu capture of "
                                            "this kernel at this size, committed in "
                                            "profiles/accumulate_uz_fwd_8192x8192_S221.md "
                                            "(not measured in this run)")
                         if traffic is not None else None,
                         "kernel_ms": kern_ms, "algorithmic_bytes": alg,
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)"
                         if peaks else "fallback 6650 GB/s"},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps,
            "step_ms": {"min": min(step_ms), "median": statistics.median(step_ms),
                        "max": max(step_ms), "slowest": step_ms.index(max(step_ms))},
            "clocks": clocks,
            "self_check": {"finite_and_nonnegative_Z": ok},
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_e2e(args, x, w, sh, world, dev):
    """Host buffers -> device -> op -> host, timed per step on the device."""
    import neural_shift_cuda_b200 as nsc
    try:
        xh = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
        wh = torch.empty(w.shape, dtype=w.dtype, pin_memory=True)
        pinned = True
    except RuntimeError:
        xh = torch.empty(x.shape, dtype=x.dtype)
        wh = torch.empty(w.shape, dtype=w.dtype)
        pinned = False
    xh.copy_(x)
    wh.copy_(w)
    Uh = torch.empty(x.shape, dtype=torch.float32, pin_memory=pinned)
    Zh = torch.empty_like(Uh, pin_memory=pinned)
    xd = torch.empty_like(x)
    wd = torch.empty_like(w)
    steps = max(1, min(args.steps, args.e2e_steps))

    # The result of step k travels device -> host on its own stream while
    # step k + 1's inputs travel host -> device (PCIe is full duplex); the
    # timed region ends when the last result is on the host.
    main = torch.cuda.current_stream()
    d2h = torch.cuda.Stream()

    def once():
        xd.copy_(xh, non_blocking=True)
        wd.copy_(wh, non_blocking=True)
        if world == 1:
            U, Z = nsc.accumulate_uz(xd, wd, sh)
        else:
            from neural_shift_cuda_b200 import bands
            U, Z = bands.accumulate_uz_banded(xd, wd, sh, HG)
        d2h.wait_stream(main)
        with torch.cuda.stream(d2h):
            Uh.copy_(U, non_blocking=True)
            Zh.copy_(Z, non_blocking=True)
        U.record_stream(d2h)
        Z.record_stream(d2h)

    once()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        once()
    main.wait_stream(d2h)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return {"value": PIXEL_SHIFTS / (ms * 1e-3), "unit": UNIT,
            "h2d_bytes_per_step": (x.numel() * x.element_size()
                                   + w.numel() * w.element_size()) * world,
            "d2h_bytes_per_step": 2 * Uh.numel() * 4 * world,
            "steps": steps, "pinned": pinned, "ms_per_step": ms}


# ---------------------------------------------------------------------------
# Secondary workloads (BASELINE.json configs[1..3]): one op per step,
# batch-sharded across ranks (images are independent: no collective).
# ---------------------------------------------------------------------------

class OpWorkload:
    """One op of the path on one BASELINE configuration.

    make(dev, b0, nb) -> dict(inputs=[device tensors], run=callable(*inputs)
    -> outputs, launches=int, units=pixel-shifts of the nb images);
    `cpu(nb)` runs the oracle on a bounded slice and returns (units, seconds,
    description)."""

    def __init__(self, name, metric, B, config, dtype, make, cpu):
        self.name, self.metric, self.B = name, metric, B
        self.config, self.dtype, self.make, self.cpu = config, dtype, make, cpu


def _seeded(shape, b0, nb, seed, dev, fn):
    """Rows b0..b0+nb of a batch tensor whose images are seeded one by one,
    so any batch split sees the same data."""
    out = []
    for b in range(b0, b0 + nb):
        g = torch.Generator(device=dev)
        g.manual_seed(seed * 1009 + b)
        out.append(fn(g, shape))
    return torch.stack(out, 0)


def _wl_pair_gather():
    Bt, Cg, Hs, Ws, Rr = 8, 16, 256, 256, 5
    rows = halfplane(Rr)

    def make(dev, b0, nb):
        import neural_shift_cuda_b200 as nsc
        guide = _seeded((Cg, Hs, Ws), b0, nb, 1, dev,
                        lambda g, sh: torch.rand(sh, generator=g, device=dev))
        sh = torch.tensor(rows)
        return dict(inputs=[guide], run=lambda gd: nsc.pair_gather(gd, sh),
                    launches=1, units=len(rows) * nb * 2 * Cg * Hs * Ws)

    def cpu(nb):
        from oracle import nsc_oracle as O
        g = torch.Generator().manual_seed(0)
        guide = torch.rand(nb, Cg, Hs, Ws, generator=g)
        t0 = time.perf_counter()
        O.pair_gather(guide, torch.tensor(rows))
        return (len(rows) * nb * 2 * Cg * Hs * Ws, time.perf_counter() - t0,
                f"oracle pair_gather on {nb} of {Bt} images")

    return OpWorkload(
        "pair_gather", "pixel-shifts/s (pair_gather fwd, NECTR configs[1]: "
        "guide (8,16,256,256) f32, R=5 S=61)", Bt,
        {"workload": "pair_gather fwd, NECTR latent guide (8,16,256,256) f32, "
                     "half-plane R=5 S=61 (configs[1])"},
        "f32 copy", make, cpu)


def _wl_normalized():
    Bt, Cx, Hs, Ws, Rr = 16, 3, 512, 512, 7
    rows = [(dx, dy, 0) for dx in range(-Rr, Rr + 1) for dy in range(-Rr, Rr + 1)]
    Sn = len(rows)

    def make(dev, b0, nb):
        import neural_shift_cuda_b200 as nsc
        x = _seeded((Cx, Hs, Ws), b0, nb, 2, dev,
                    lambda g, sh: torch.rand(sh, generator=g, device=dev)
                    ).to(torch.bfloat16)
        # logits N(0, 3^2), batch-major (B, S, H, W) as the attention
        # produces them, handed over shift-major and channel-broadcast
        lg = _seeded((Sn, Hs, Ws), b0, nb, 3, dev,
                     lambda g, sh: 3.0 * torch.randn(sh, generator=g, device=dev)
                     ).to(torch.bfloat16)
        lg = lg.transpose(0, 1).reshape(Sn * nb, 1, Hs, Ws).contiguous()
        sh = torch.tensor(rows)
        return dict(inputs=[x, lg],
                    run=lambda a, b: nsc.normalized_accumulate_uz(
                        a, b.expand(-1, Cx, -1, -1), sh, log_weights=True,
                        return_log_degree=True, validate=False),
                    launches=1, units=Sn * nb * Cx * Hs * Ws)

    def cpu(nb):
        from oracle import nsc_oracle as O
        g = torch.Generator().manual_seed(0)
        rows_s = 64
        x = torch.rand(1, Cx, rows_s, Ws, generator=g).to(torch.bfloat16)
        lg = (3.0 * torch.randn(Sn, 1, rows_s, Ws, generator=g)).to(torch.bfloat16)
        t0 = time.perf_counter()
        O.normalized_accumulate_uz(x, lg.expand(-1, Cx, -1, -1), torch.tensor(rows),
                                   log_weights=True)
        return (Sn * Cx * rows_s * Ws, time.perf_counter() - t0,
                f"oracle normalized_accumulate_uz (log) on a (1,3,{rows_s},512) band, S={Sn}")

    return OpWorkload(
        "normalized", "pixel-shifts/s (normalized_accumulate_uz fwd, log weights, "
        "GASD configs[2]: x bf16 (16,3,512,512), S=225)", Bt,
        {"workload": "normalized_accumulate_uz fwd, logits N(0,9) bf16 channel-"
                     "shared, full window R=7 S=225, x bf16 (16,3,512,512) (configs[2])"},
        "bf16 in, f32 accumulate", make, cpu)


def _wl_metropolis():
    Bt, Cx, Hs, Ws, Rr = 16, 3, 512, 512, 5
    rows = halfplane(Rr)
    Sm = len(rows)

    def make(dev, b0, nb):
        from neural_shift_cuda_b200.metropolis import metropolis_aggregate
        x = _seeded((Cx, Hs, Ws), b0, nb, 4, dev,
                    lambda g, sh: torch.rand(sh, generator=g, device=dev))
        wh = _seeded((Sm, 1, Hs, Ws), b0, nb, 5, dev,
                     lambda g, sh: torch.sigmoid(torch.randn(sh, generator=g, device=dev)))
        gw = _seeded((Cx, Hs, Ws), b0, nb, 6, dev,
                     lambda g, sh: torch.randn(sh, generator=g, device=dev))
        sh = torch.tensor(rows)

        def run(w, xi, gy):
            w = w.detach().requires_grad_(True)
            xi = xi.detach().requires_grad_(True)
            # one weight channel read for all three image channels, the
            # form the NKD_mp patch passes (its head mix keeps one channel)
            Wx, dh = metropolis_aggregate(w, xi, sh, use_box=True, eps=1e-6)
            gwh, gx = torch.autograd.grad(Wx, (w, xi), gy)
            return Wx, gwh, gx
        return dict(inputs=[wh, x, gw], run=run, launches=2,
                    units=2 * Sm * nb * Cx * Hs * Ws)

    def cpu(nb):
        from oracle import nsc_oracle as O
        g = torch.Generator().manual_seed(0)
        rows_s = 64
        x = torch.rand(1, Cx, rows_s, Ws, generator=g)
        wh = torch.sigmoid(torch.randn(1, Sm, 1, rows_s, Ws, generator=g))
        gy = torch.randn(1, Cx, rows_s, Ws, generator=g)
        t0 = time.perf_counter()
        O.metropolis_aggregate_grad(wh, x, torch.tensor(rows), True, 1e-6, gy,
                                    torch.zeros_like(gy))
        return (2 * Sm * Cx * rows_s * Ws, time.perf_counter() - t0,
                f"oracle metropolis_aggregate fwd+bwd (autograd) on a (1,3,{rows_s},512) band, S={Sm}")

    return OpWorkload(
        "metropolis", "pixel-shifts/s (metropolis_aggregate fwd+bwd, NKD_mp "
        "configs[3]: x f32 (16,3,512,512), S=61)", Bt,
        {"workload": "metropolis_aggregate fwd+bwd, w_half sigmoid(N(0,1)) "
                     "(16,61,1,512,512) f32 broadcast over C=3, use_box, R=5 S=61 "
                     "(configs[3])"},
        "f32", make, cpu)


def _nectr_model(dev, dtype):
    """NECTR model 1 with the benchmark configuration (concat, residual
    depth 2, projection depth 1, latent 16, patch radius 1, window radius 5,
    one channel, blind, exp head), random init (seed 0), NECTR installer
    applied."""
    from types import SimpleNamespace
    from neural_shift_cuda_b200.integration import install_cuda_shift_nectr
    from neural_shift_cuda_b200.integration.nectr_models1 import NECTR_denoiser
    args = SimpleNamespace(model_type="concat", residual_depth=2, proj_depth=1,
                           latent_dim=16, patch_rad=1, output_activation="exp",
                           window_rad=5, in_channel=1, blind=True)
    cls = type("NECTRBench", (NECTR_denoiser,), {})
    install_cuda_shift_nectr(cls)
    torch.manual_seed(0)
    m = cls(args)
    return m.to(device=dev, dtype=dtype).eval()


def _wl_nectr(dtype_name, fused=True):
    Bt, Hs, Ws, Rr = 8, 256, 256, 5
    rows = halfplane(Rr)
    Sn = len(rows)
    dtype = torch.bfloat16 if dtype_name == "bf16" else torch.float32

    def noisy(g, sh, dev):
        return (torch.rand(sh, generator=g, device=dev)
                + (25 / 255) * torch.randn(sh, generator=g, device=dev))

    def make(dev, b0, nb):
        from neural_shift_cuda_b200.integration import nectr_patch as NP
        m = _nectr_model(dev, dtype)
        m.use_nectr_fused = fused
        x = _seeded((1, Hs, Ws), b0, nb, 7, dev,
                    lambda g, sh: noisy(g, sh, dev)).to(dtype)

        def run(xi):
            with torch.no_grad():
                return m(xi)

        def per_kernel(xi):
            """One forward with CUDA events around the two kernels of the
            path (pair_gather, normalized_accumulate_uz): median of 5."""
            names = ({"_forward_fused": []} if fused else
                     {"pair_gather": [], "normalized_accumulate_uz": []})
            sizes = {}
            orig = {k: getattr(NP, k) for k in names}

            def wrap(k):
                def f(*a, **kw):
                    st = torch.cuda.current_stream()
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record(st)
                    out = orig[k](*a, **kw)
                    e1.record(st)
                    names[k].append((e0, e1))
                    sizes[k] = _nbytes([t for t in a if isinstance(t, torch.Tensor)]
                                       ) + _nbytes(out)
                    if k == "_forward_fused":
                        # x and the guide in; the two per-pixel maps written
                        # and read once; D and Z out
                        L1 = m.proj[0][0].out_channels
                        sizes[k] += 2 * 2 * a[2].shape[0] * L1 * Hs * Ws * 4
                    return out
                return f
            try:
                for k in names:
                    setattr(NP, k, wrap(k))
                for _ in range(5):
                    run(xi)
            finally:
                for k in names:
                    setattr(NP, k, orig[k])
            torch.cuda.synchronize()
            res = {}
            for k, evs in names.items():
                ms = statistics.median(a.elapsed_time(b) for a, b in evs)
                res[k] = {"ms": ms, "algorithmic_bytes": sizes[k]}
            # pair_gather's guide input is (B, L, H, W) and its outputs the
            # (S*B, 2L, H, W) pair batch and (S*B, 1, H, W) mask: the sum above
            # counts the guide, pair batch and mask once each; the normalized
            # reduction counts x, the (S*B, 1, H, W) values, D and log_C.
            return res

        return dict(inputs=[x], run=run, launches=1 if fused else 2,
                    units=Sn * nb * 1 * Hs * Ws, per_kernel=per_kernel,
                    dominant="_forward_fused" if fused else "pair_gather")

    def cpu(nb):
        dev = torch.device("cpu")
        m = _nectr_model(dev, torch.float32)
        g = torch.Generator().manual_seed(0)
        x = noisy(g, (1, 1, Hs, Ws), dev)
        t0 = time.perf_counter()
        with torch.no_grad():
            m(x)     # CPU input: the model's own serial forward
        return (Sn * 1 * Hs * Ws, time.perf_counter() - t0,
                f"NECTR_models1 serial forward (the reference model's own "
                f"per-shift loop) on 1 of {Bt} images, fp32, torch CPU")

    return OpWorkload(
        "nectr_" + dtype_name + ("" if fused else "_unfused"),
        f"pixel-shifts/s (NECTR model-1 patched forward, configs[1]: x "
        f"(8,1,256,256) {dtype_name}, latent 16, R=5 S=61)", Bt,
        {"workload": f"NECTR_models1 patched forward ("
                     + ("fused pair gather + weight head + normalized "
                        "accumulation, one kernel" if fused else
                        "pair_gather -> weight head -> normalized_accumulate_uz")
                     + f", log mode), x "
                     f"(8,1,256,256) {dtype_name} U[0,1]+N(0,(25/255)^2), "
                     f"concat, residual_depth 2, proj_depth 1, latent 16, "
                     f"R=5 S=61, random init (configs[1])",
         "unit_definition": "S*B*C*H*W of the aggregation per forward"},
        f"{dtype_name} model, f32 accumulate", make, cpu)


def _wl_accumulate_train():
    """configs[4] forward + backward: one training step of the reduction
    (U, Z from x and the weights; grad_x, grad_w from grad_U, grad_Z)."""
    Hs = Ws = 8192

    def make(dev, b0, nb):
        import neural_shift_cuda_b200 as nsc
        x, w = make_band(0, Hs, dev)
        gU = torch.randn((1, C, Hs, Ws), device=dev)
        gZ = torch.randn((1, C, Hs, Ws), device=dev)
        sh = torch.tensor(ROWS)

        def run(xi, wi, a, b):
            xi = xi.detach().requires_grad_(True)
            wi = wi.detach().requires_grad_(True)
            U, Z = nsc.accumulate_uz(xi, wi, sh)
            gx, gw = torch.autograd.grad((U, Z), (xi, wi), (a, b))
            return U.detach(), Z.detach(), gx, gw
        # forward, grad_w, grad_x (TMA tile kernel + border-band wrap kernel)
        return dict(inputs=[x, w, gU, gZ], run=run, launches=4,
                    units=2 * S * C * Hs * Ws)

    def cpu(nb):
        from oracle import nsc_oracle as O
        g = torch.Generator().manual_seed(0)
        rows_s = 8
        x = torch.rand(1, C, rows_s, Ws, generator=g).half()
        w = torch.nn.functional.softplus(torch.randn(S, 1, rows_s, Ws, generator=g)).half()
        gU = torch.randn(1, C, rows_s, Ws, generator=g)
        gZ = torch.randn(1, C, rows_s, Ws, generator=g)
        sh = torch.tensor(ROWS)
        t0 = time.perf_counter()
        O.accumulate_uz(x, w.expand(-1, C, -1, -1).contiguous(), sh)
        O.accumulate_uz_backward(x, w, gU, gZ, sh)
        return (2 * S * C * rows_s * Ws, time.perf_counter() - t0,
                f"oracle accumulate_uz forward + backward on a (1, 3, {rows_s}, 8192) band, S=221")

    return OpWorkload(
        "accumulate_train", "pixel-shifts/s (accumulate_uz fwd+bwd, 8192^2 x3, S=221, "
        "fp16 in / fp32 acc)", 1,
        {"workload": "accumulate_uz forward + backward, configs[4] shapes (x fp16 "
                     "(1,3,8192,8192), channel-shared fp16 weights (221,1,8192,8192), "
                     "grad_U / grad_Z fp32 N(0,1))"},
        "f16 in, f32 accumulate", make, cpu)


def _wl_normalized_train():
    """configs[2] forward + backward: normalized_accumulate_uz with logits
    that require grad, grad_D N(0, 1)."""
    base = _wl_normalized()
    Bt, Cx, Hs, Ws, Rr = 16, 3, 512, 512, 7
    rows = [(dx, dy, 0) for dx in range(-Rr, Rr + 1) for dy in range(-Rr, Rr + 1)]
    Sn = len(rows)

    def make(dev, b0, nb):
        import neural_shift_cuda_b200 as nsc
        w = base.make(dev, b0, nb)
        x, lg = w["inputs"]
        gD = _seeded((Cx, Hs, Ws), b0, nb, 8, dev,
                     lambda g, sh: torch.randn(sh, generator=g, device=dev))
        sh = torch.tensor(rows)

        def run(a, b, gd):
            b = b.detach().requires_grad_(True)
            a = a.detach().requires_grad_(True)
            # the channel-broadcast (S*B, 1, H, W) form: an expand + slice of the
            # logits would add the autograd scatter/sum of a 3-channel gradient
            D, L = nsc.normalized_accumulate_uz(a, b, sh, log_weights=True,
                                                return_log_degree=True, validate=False)
            gx, gl = torch.autograd.grad(D, (a, b), gd)
            return D.detach(), gx, gl
        return dict(inputs=[x, lg, gD], run=run, launches=2,
                    units=2 * Sn * nb * Cx * Hs * Ws)

    def cpu(nb):
        from oracle import nsc_oracle as O
        g = torch.Generator().manual_seed(0)
        rows_s = 32
        x = torch.rand(1, Cx, rows_s, Ws, generator=g).to(torch.bfloat16)
        lg = (3.0 * torch.randn(Sn, 1, rows_s, Ws, generator=g)).to(torch.bfloat16)
        gD = torch.randn(1, Cx, rows_s, Ws, generator=g)
        t0 = time.perf_counter()
        D, L = O.normalized_accumulate_uz(x, lg.expand(-1, Cx, -1, -1), torch.tensor(rows), True)
        O.normalized_accumulate_uz_backward(x, lg, D, L, gD, torch.zeros_like(gD),
                                            torch.tensor(rows), True)
        return (2 * Sn * Cx * rows_s * Ws, time.perf_counter() - t0,
                f"oracle normalized_accumulate_uz fwd+bwd (log) on a (1,3,{rows_s},512) band, S={Sn}")

    return OpWorkload(
        "normalized_train", "pixel-shifts/s (normalized_accumulate_uz fwd+bwd, log weights, "
        "GASD configs[2]: x bf16 (16,3,512,512), S=225)", Bt,
        {"workload": "normalized_accumulate_uz forward + backward, logits N(0,9) bf16 "
                     "channel-shared, full window R=7 S=225, x bf16 (16,3,512,512), "
                     "grad_D N(0,1) (configs[2])"},
        "bf16 in, f32 accumulate", make, cpu)


WORKLOADS = {"pair_gather": _wl_pair_gather, "accumulate_train": _wl_accumulate_train,
             "normalized_train": _wl_normalized_train, "normalized": _wl_normalized,
             "metropolis": _wl_metropolis,
             "nectr": lambda: _wl_nectr("f32"),
             "nectr_bf16": lambda: _wl_nectr("bf16"),
             "nectr_unfused": lambda: _wl_nectr("f32", fused=False),
             "nectr_bf16_unfused": lambda: _wl_nectr("bf16", fused=False)}


def _nbytes(ts):
    out = 0
    for t in ts:
        if isinstance(t, torch.Tensor):
            out += t.numel() * t.element_size()
        elif isinstance(t, (tuple, list)):
            out += _nbytes(t)
    return out


def run_workload(args, wl):
    """Time one secondary workload: the batch is split across ranks; value =
    pixel-shifts of the whole batch / max-over-ranks time."""
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return
        vals = []
        for i in range(args.warmup + args.steps):
            u, dt, desc = wl.cpu(1)
            if i >= args.warmup:
                vals.append(u / dt)
        v = statistics.median(vals)
        threads = torch.get_num_threads()
        print(json.dumps({
            "impl": "reference", "metric": wl.metric, "value": v, "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": wl.dtype, "data": "synthetic", "config": wl.config,
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads,
                             "kind": "port", "sample": desc},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}), flush=True)
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    nb = wl.B // world + (1 if rank < wl.B % world else 0)
    b0 = rank * (wl.B // world) + min(rank, wl.B % world)
    w = wl.make(dev, b0, nb)
    inputs, run = w["inputs"], w["run"]
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    stream = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        torch.cuda.nvtx.range_push("warmup")
        for _ in range(args.warmup):
            out = run(*inputs)
        torch.cuda.nvtx.range_pop()
        del out
        barrier()
        t0, t1 = (torch.cuda.Event(enable_timing=True),
                  torch.cuda.Event(enable_timing=True))
        torch.cuda.nvtx.range_push("timed")
        t0.record(stream)
        for i in range(args.steps):
            ev[i][0].record(stream)
            out = run(*inputs)
            ev[i][1].record(stream)
            if i + 1 < args.steps:
                del out
        t1.record(stream)
        torch.cuda.nvtx.range_pop()
        barrier()
    total = t0.elapsed_time(t1)
    if world > 1:
        t = torch.tensor([total], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total = float(t.item())
    ms = total / args.steps
    units_all = w["units"] * wl.B // max(nb, 1) if world == 1 else None
    if world > 1:
        u = torch.tensor([float(w["units"])], device=dev, dtype=torch.float64)
        dist.all_reduce(u)
        units_all = u.item()
    step_ms = [a.elapsed_time(b) for a, b in ev]
    step_median = kern_ms = statistics.median(step_ms)
    alg = _nbytes(inputs) + _nbytes(out)
    kernels = None
    roof_note = "step time of all launches of the op (per rank)"
    if "per_kernel" in w:
        kernels = w["per_kernel"](*inputs)
        dom = kernels[w["dominant"]]
        kern_ms, alg = dom["ms"], dom["algorithmic_bytes"]
        roof_note = (f"dominant kernel {w['dominant']}, CUDA events around its "
                     f"call inside the forward (per rank)")
        for k in kernels.values():
            k["achieved_gbs"] = k["algorithmic_bytes"] / (k["ms"] * 1e-3) / 1e9
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    achieved = alg / (kern_ms * 1e-3) / 1e9
    if kernels:
        for k in kernels.values():
            k["frac"] = k["achieved_gbs"] / peak

    e2e = None
    if not args.no_e2e:
        hin = []
        for t in inputs:
            try:
                h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
            except RuntimeError:
                h = torch.empty(t.shape, dtype=t.dtype)
            h.copy_(t)
            hin.append(h)
        outs = [o for o in (out if isinstance(out, (tuple, list)) else [out])]
        hout = [torch.empty(o.shape, dtype=o.dtype, pin_memory=hin[0].is_pinned())
                for o in outs]
        din = [torch.empty_like(t) for t in inputs]

        def once():
            for d, h in zip(din, hin):
                d.copy_(h, non_blocking=True)
            res = run(*din)
            res = res if isinstance(res, (tuple, list)) else [res]
            for h, o in zip(hout, res):
                h.copy_(o, non_blocking=True)
        once()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = max(1, min(args.steps, args.e2e_steps))
        a.record()
        for _ in range(n):
            once()
        b.record()
        torch.cuda.synchronize()
        e_ms = a.elapsed_time(b) / n
        if world > 1:
            t = torch.tensor([e_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e_ms = float(t.item())
        e2e = {"value": units_all / (e_ms * 1e-3), "unit": UNIT,
               "h2d_bytes_per_step": _nbytes(hin) * world,
               "d2h_bytes_per_step": _nbytes(hout) * world, "steps": n,
               "ms_per_step": e_ms}
    clocks = clk.summary()
    if rank == 0:
        cpu = None
        if not args.no_cpu and world == 1:
            torch.set_num_threads(os.cpu_count() or 1)
            wl.cpu(1)
            u, dt, desc = wl.cpu(1)
            cpu = {"value": u / dt, "unit": UNIT, "cores": torch.get_num_threads(),
                   "kind": "port", "sample": desc}
        cfg = dict(wl.config)
        cfg.update({"B": wl.B, "parallelism": f"batch shards x{world}" if world > 1
                    else "single GPU", "l2": "inputs larger than L2" if
                    _nbytes(inputs) > 126e6 else "inputs smaller than L2"})
        print(json.dumps({
            "metric": wl.metric, "value": units_all / (ms * 1e-3), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic",
            "config": cfg,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak,
                         "unit": "GB/s", "frac": achieved / peak, "traffic": None,
                         "kernel_ms": kern_ms, "algorithmic_bytes": alg,
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)"
                         if peaks else "fallback 6650 GB/s",
                         "note": roof_note},
            "kernels": kernels,
            "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": w["launches"] * args.steps,
            "step_ms": {"min": min(step_ms), "median": step_median, "max": max(step_ms)},
            "clocks": clocks}), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ref-rows", type=int, default=32)
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--size", type=int, default=8192,
                    help="image side (8192 is the benchmark; smaller sides "
                         "are for profiling captures only)")
    ap.add_argument("--workload", default="accumulate",
                    choices=["accumulate"] + sorted(WORKLOADS),
                    help="accumulate (configs[4], the headline) or one of the "
                         "secondary op workloads of configs[1..3]")
    args = ap.parse_args()
    if args.workload != "accumulate":
        run_workload(args, WORKLOADS[args.workload]())
        return
    global HG, WG, PIXEL_SHIFTS
    HG = WG = args.size
    PIXEL_SHIFTS = S * B * C * HG * WG
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
