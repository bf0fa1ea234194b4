"""Benchmark of simtgo's hot path on B200: prints ONE JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1)

Headline (value): FIR throughput in Gsamples/s over the whole job. Each GPU
owns 2^28 consecutive outputs of one long signal with 127 taps -- 2^31
samples at 8 GPUs -- and receives its input slice with the 126 preceding
samples duplicated (the halo), so there is no data-path collective
("scaling": "weak"). One step = one simtgo_FIR_shard launch per GPU over
its resident shard. The inputs (1 GiB per buffer) exceed the 126 MB L2, so
no flush is needed between steps.

e2e: the same metric through the C ABI with HOST buffers: every step copies
the shard in from pinned memory, runs the FIR and copies the outputs back.

Also reported: the roofline of the FIR kernel (FP32 FMA-bound at 127 taps),
clocks sampled during the timed region, a CPU baseline (the oracle port on
the host cores, bounded sample), and at N=1 every kernel's achieved HBM
GB/s at its workload size ("kernels"), plus, at every N, the sharded
histogram (with the bins all-reduced), the sharded tile graph and the
sharded tile reductions (block partials all-gathered).

--impl reference times the reference's CPU path (the oracle port of
gpu.RunCPU's FIR; the reference's own generated FIR.cu stages a 320-sample
tile and cannot hold 127 taps) on the same metric, rank 0 only.
"""
from __future__ import annotations

import argparse
import ctypes as C
import datetime
import json
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = ("achieved HBM GB/s (% of B200 peak) per kernel; FIR Gsamples/s at 1/2/4/8 GPU")
TAPS = 127
FIR_LOG2 = 28            # outputs per GPU
HALO = 128               # >= TAPS-1, a multiple of 4 so shard inputs stay 16-byte aligned
P = C.c_void_p


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def fir_taps():
    """127 taps uniform[-1,1], normalised to sum 1 (redrawn while the sum is
    below 0.1 in magnitude)."""
    import numpy as np

    seed = 3
    while True:
        h = np.random.default_rng(seed).uniform(-1, 1, TAPS)
        if abs(h.sum()) >= 0.1:
            return (h / h.sum()).astype(np.float32)
        seed += 1000


def signal(torch, g0, n, device, piece=1 << 26):
    """Samples g0 .. g0+n-1 of one long uniform[-1,1) signal, as a function
    of the global index, so every shard sees the same halo values. Filled
    in pieces so that a 2^31-sample signal needs no more temporary memory
    than a 2^26-sample one."""
    out = torch.empty(n, dtype=torch.float32, device=device)
    for o in range(0, n, piece):
        m = min(piece, n - o)
        g = torch.arange(g0 + o, g0 + o + m, dtype=torch.int64, device=device)
        h = (g * 0x9E3779B1 + 0x7F4A7C15) & 0xFFFFFFFF
        h = (h ^ (h >> 15)) * 0x2C1B3C6D & 0xFFFFFFFF
        h = h ^ (h >> 12)
        v = out[o:o + m]
        v.copy_((h & 0xFFFFFF).to(torch.float32) * (2.0 / 16777216.0) - 1.0)
        v[g < 0] = 0.0
    return out


class Clocks:
    """nvidia-smi sampled every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        self.f.close()

    def summary(self):
        rows = []
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                    rows.append(parts)
        finally:
            os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm = [float(r[1]) for r in rows]
        loaded = [float(r[1]) for r in rows if float(r[3]) > 300] or sm
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": float(rows[0][2]),
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows),
                "reasons": sorted(reasons)}


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def ncu_traffic(name):
    """Per-unit DRAM bytes from a committed ncu summary, or None."""
    p = ROOT / "profiles" / "ncu_traffic.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text()).get(name)
    except (ValueError, OSError):
        return None


# ---------------------------------------------------------------------------
def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    from simtgo_b200 import _lib

    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    L = _lib.load()
    stream = torch.cuda.current_stream()
    sp = P(stream.cuda_stream)
    sms = C.c_int32()
    _lib.check(L.simtgo_device_info(C.byref(sms), None, None))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def events():
        return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    # ---- the FIR shard -----------------------------------------------------
    from simtgo_b200 import shard

    plan = shard.fir_plan(world << args.fir_log2, world, rank, TAPS)
    n, halo = plan.n, plan.halo
    h = torch.from_numpy(fir_taps()).to(dev)
    x = signal(torch, plan.in_lo, plan.in_len, dev)
    y = torch.empty(n, dtype=torch.float32, device=dev)

    def fir_step(yb=y, xb=x):
        rc = L.simtgo_FIR_shard(P(yb.data_ptr()), n, P(xb.data_ptr()), xb.numel(), halo,
                                P(h.data_ptr()), TAPS, sp)
        if rc:
            _lib.check(rc)

    for _ in range(args.warmup):
        fir_step()
    barrier()
    e0, e1 = events()
    with Clocks(local) as clk:
        # Untimed soak so the sampled clocks are the ones this kernel runs
        # at under load (the timed region alone can be shorter than the
        # 200 ms sampling period).
        t_end = time.perf_counter() + args.soak_s
        while time.perf_counter() < t_end:
            for _ in range(16):
                fir_step()
            torch.cuda.synchronize()
        barrier()
        e0.record(stream)
        for _ in range(args.steps):
            fir_step()
        e1.record(stream)
        e1.synchronize()
        barrier()
    ms = e0.elapsed_time(e1)
    ms_max = max_over_ranks(ms)
    clocks = clk.summary()
    _lib.check(L.simtgo_stream_sync(sp))
    value = world * n * args.steps / (ms_max * 1e-3) / 1e9
    launch_ms = ms / args.steps

    # Parity of this rank's whole shard against the oracle (outside the
    # timed region; the oracle on this rank's share of the host cores).
    spot = shard_parity(np, x, y, h, halo, world)

    # ---- e2e: host buffers through the C ABI ----------------------------------
    # simtgo_FIR_shard_host streams the pinned host shard through the GPU in
    # chunks on three streams, so uploads, kernels and downloads overlap.
    xh = torch.empty(x.numel(), dtype=torch.float32, pin_memory=True)
    xh.copy_(x)
    yh = torch.empty(n, dtype=torch.float32, pin_memory=True)
    hh = h.cpu().pin_memory()
    e2e_steps = max(3, min(args.steps, args.e2e_steps))

    def e2e_step():
        rc = L.simtgo_FIR_shard_host(P(yh.data_ptr()), n, P(xh.data_ptr()), xh.numel(), halo,
                                     P(hh.data_ptr()), TAPS, sp)
        if rc:
            _lib.check(rc)

    # Bytes the host form moves per call: each chunk's input with the taps-1
    # samples before it, the taps once per stream, the outputs.
    chunk = 1 << 22
    h2d_bytes = 3 * TAPS * 4
    for o0 in range(0, n, chunk):
        cn = min(chunk, n - o0)
        hj = min(TAPS - 1, halo + o0)
        h2d_bytes += max(0, min(o0 + cn, xh.numel() - halo) - (o0 - hj)) * 4

    for _ in range(2):
        e2e_step()
    barrier()
    e0, e1 = events()
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    e1.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = world * n * e2e_steps / (e2e_ms * 1e-3) / 1e9
    ceiling = copy_ceiling(torch, xh, yh, h2d_bytes, dev, barrier, max_over_ranks, events,
                           e2e_steps)
    del xh, yh

    # ---- roofline of the FIR kernel ---------------------------------------------
    peaks, peak_src = measured_peaks()
    flops = 2.0 * TAPS * n
    achieved_tflops = flops / (launch_ms * 1e-3) / 1e12
    sm_mhz = clocks.get("sm_mhz") or peaks.get("clocks_under_load", {}).get("sm_mhz_median", 1965)
    fp32_peak = sms.value * 128 * 2 * sm_mhz * 1e6 / 1e12
    hbm_gbs = (8.0 * n + 4.0 * halo) / (launch_ms * 1e-3) / 1e9
    traffic = ncu_traffic("FIR_shard_127")
    # At 127 taps the kernel is bound by FP32 FMA issue, not HBM (2*taps
    # FLOPs per 8 bytes): the headline fraction is of the FP32 peak (no
    # measured figure exists for it: SMs x 128 lanes x 2 x the sampled
    # clock); the HBM fraction is the sub-record.
    roofline = {
        "bound": "fp32",
        "achieved": round(achieved_tflops, 2), "peak": round(fp32_peak, 2), "unit": "TFLOP/s",
        "frac": round(achieved_tflops / fp32_peak, 4),
        "peak_source": f"derived: {sms.value} SMs x 128 FP32 lanes x 2 FLOP x {sm_mhz:.0f} MHz "
                       "(the SM clock sampled during the timed region)",
        "algorithmic_flops_per_launch": int(flops),
        "traffic": None if traffic is None else int(traffic * n),
        "traffic_note": "DRAM bytes per launch (ncu dram__bytes_read+write per output x outputs)",
        "kernel_ms": round(launch_ms, 4),
        "hbm": {
            "achieved": round(hbm_gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(hbm_gbs / peaks["hbm_gbs"], 4),
            "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs, copy burst)",
            "algorithmic_bytes_per_launch": int(8 * n + 4 * halo),
        },
    }

    # ---- sharded histogram (bins all-reduced) and sharded tile graph ------------
    sharded = {}
    del x, y
    torch.cuda.empty_cache()
    sharded["fir_strong"] = bench_fir_strong(args, torch, L, dev, sp, rank, world, h, barrier,
                                             max_over_ranks, events)
    sharded["histogram_allreduce"] = bench_histogram(args, torch, L, dev, sp, rank, world,
                                                     barrier, max_over_ranks, events)
    sharded["tile_graph"] = bench_tile(args, torch, np, L, dev, sp, rank, world, barrier,
                                       max_over_ranks, events)
    sharded["tile_reduce"] = bench_tile_reduce(args, torch, L, dev, rank, world, barrier,
                                               max_over_ranks, events)

    kernels = None
    chain = None
    cpu = None
    if world == 1 and not args.skip_kernels:
        chain = bench_signal_chain(args, torch, np, L, dev, sp, events, peaks)
        kernels = bench_kernels(args, torch, np, L, dev, sp, events, peaks)
    if rank == 0 and world == 1 and not args.skip_cpu:
        cpu = cpu_baseline(args, np, seconds=args.cpu_seconds)

    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "Gsamples/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (uniform[-1,1) signal from a counter hash; seeded taps)",
        "config": {
            "workload": f"FIR, 2^{args.fir_log2} outputs per GPU ({world}x2^{args.fir_log2} "
                        f"of one signal), {TAPS} taps normalised to sum 1",
            "taps": TAPS, "samples_per_gpu": n, "total_samples": world * n,
            "halo": "126 preceding samples duplicated into each shard's input (128 staged)",
            "parallelism": f"{world} shards, no data-path collective",
            "l2": "inputs larger than L2 (1 GiB per buffer), no flush",
        },
        "e2e": {"value": round(e2e_value, 3), "unit": "Gsamples/s",
                "h2d_bytes_per_step": world * h2d_bytes,
                "d2h_bytes_per_step": world * n * 4,
                "steps": e2e_steps,
                "path": "simtgo_FIR_shard_host on pinned host buffers: 2^22-output chunks on "
                        "three streams, uploads, kernels and downloads overlapping; bytes summed "
                        "over ranks",
                "copy_ceiling": ceiling,
                "frac_of_copy_ceiling": (round(e2e_value / ceiling["gsamples_per_s"], 4)
                                         if ceiling else None)},
        "gpu_launches": args.steps,
        "gpu_launches_note": "simtgo_FIR_shard kernels per rank inside the timed region",
        "roofline": roofline,
        "clocks": clocks,
        "cpu_baseline": cpu,
        "parity": spot,
        "signal_chain": chain,
        "sharded": sharded,
        "kernels": kernels,
    }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def oracle_module(world):
    """The oracle (test infrastructure: the checker, never the measured
    path) with this rank's share of the host cores."""
    sys.path.insert(0, str(ROOT / "tests"))
    import oracle_lib as O

    O.set_threads(max(1, (os.cpu_count() or 1) // world))
    return O


def shard_parity(np, x, y, h, halo, world):
    """This rank's whole FIR shard against the oracle's fma order, bit for
    bit (every output, not a sample)."""
    O = oracle_module(world)
    xh = x.cpu().numpy()
    got = y.cpu().numpy()
    rc, want = O.fir_shard(xh, halo, h.cpu().numpy(), got.size)
    bad = int(np.count_nonzero(got.view(np.uint32) != want.view(np.uint32))) if rc == 0 else -1
    return {"fir_shard": {"outputs": int(got.size), "bit_exact": rc == 0 and bad == 0,
                          "mismatches": bad,
                          "check": "every output of this rank's shard against the oracle "
                                   "(device fma order), outside the timed region"}}


def copy_ceiling(torch, xh, yh, h2d_bytes, dev, barrier, max_over_ranks, events, steps):
    """What the host link allows for the e2e step: the same bytes as the
    host-memory FIR moves (h2d_bytes up, the outputs down), as pinned
    copies in 2^22-element pieces on two streams (one per direction) so that
    both directions overlap, with no kernel; Gsamples/s of the same n."""
    n = yh.numel()
    up = max(1, h2d_bytes // 4)
    xd = torch.empty(min(up, xh.numel()), dtype=torch.float32, device=dev)
    yd = torch.empty(n, dtype=torch.float32, device=dev)
    s_up, s_dn = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    piece = 1 << 22
    cur = torch.cuda.current_stream(dev)

    def step():
        s_up.wait_stream(cur)
        s_dn.wait_stream(cur)
        with torch.cuda.stream(s_up):
            for o in range(0, xd.numel(), piece):
                xd[o:o + piece].copy_(xh[o:o + piece], non_blocking=True)
        with torch.cuda.stream(s_dn):
            for o in range(0, n, piece):
                yh[o:o + piece].copy_(yd[o:o + piece], non_blocking=True)
        cur.wait_stream(s_up)
        cur.wait_stream(s_dn)

    step()
    barrier()
    e0, e1 = events()
    e0.record(cur)
    for _ in range(steps):
        step()
    e1.record(cur)
    e1.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps)
    world = int(os.environ.get("WORLD_SIZE", 1))
    return {"ms_per_step": round(ms, 4),
            "gsamples_per_s": round(world * n / (ms * 1e-3) / 1e9, 3),
            "h2d_gbs": round(xd.numel() * 4 / (ms * 1e-3) / 1e9, 1),
            "d2h_gbs": round(n * 4 / (ms * 1e-3) / 1e9, 1),
            "how": "pinned host<->device copies of the e2e step's bytes, 2^22-element pieces, "
                   "one stream per direction, no kernel"}


def bench_fir_strong(args, torch, L, dev, sp, rank, world, h, barrier, max_over_ranks, events):
    """Strong scaling: the whole 2^31-sample, 127-tap signal split over the
    ranks (2^31 outputs on one GPU: 16 GiB of input and output)."""
    from simtgo_b200 import _lib, shard

    total = 1 << args.fir_strong_log2
    plan = shard.fir_plan(total, world, rank, TAPS)
    n, halo = plan.n, plan.halo
    x = signal(torch, plan.in_lo, plan.in_len, dev)
    y = torch.empty(n, dtype=torch.float32, device=dev)

    def step():
        rc = L.simtgo_FIR_shard(P(y.data_ptr()), n, P(x.data_ptr()), x.numel(), halo,
                                P(h.data_ptr()), TAPS, sp)
        if rc:
            _lib.check(rc)

    steps = max(5, min(args.steps, 20))
    barrier()
    ms = max_over_ranks(timed(step, steps, args.warmup, torch.cuda.current_stream(), events))
    del x, y
    torch.cuda.empty_cache()
    return {"total_samples": total, "taps": TAPS, "ms_per_step": round(ms, 4),
            "gsamples_per_s": round(total / (ms * 1e-3) / 1e9, 3), "scaling": "strong",
            "steps": steps,
            "workload": f"one 2^{args.fir_strong_log2}-sample signal, {TAPS} taps, split over "
                        f"{world} GPU(s), each shard with its 126 preceding samples"}


def bench_signal_chain(args, torch, np, L, dev, sp, events, peaks):
    """The signal chain on 2^28 interleaved N(0,1) complex samples:
    MagnitudeFast(scale 3) -> Softclip(0.5) -> Quantize(step 0.25, seed
    0x9e3779b9) -> WarpReduceSum of the Softclip output; one step = the
    four launches, with CUDA events between the stages. The first 2^20
    elements of every stage are checked against the oracle afterwards."""
    from simtgo_b200 import _lib

    n = 1 << args.chain_log2
    gen = torch.Generator(device=dev).manual_seed(11)
    z = torch.randn(2 * n, device=dev, generator=gen)
    mag = torch.empty(n, device=dev)
    soft = torch.empty(n, device=dev)
    code = torch.empty(n, dtype=torch.int32, device=dev)
    energy = torch.empty(n, dtype=torch.int64, device=dev)
    clipped = torch.empty(n, dtype=torch.uint8, device=dev)
    sums = torch.empty(n // 32, device=dev)
    G, W = (n + 255) // 256, (n + 127) // 128
    stages = [
        ("MagnitudeFast_interleaved", 12.0, lambda: L.simtgo_MagnitudeFast_interleaved(
            P(mag.data_ptr()), n, P(z.data_ptr()), 2 * n, 3.0, G, 256, sp)),
        ("Softclip", 8.0, lambda: L.simtgo_Softclip(P(soft.data_ptr()), n, P(mag.data_ptr()), n,
                                                    0.5, G, 256, sp)),
        ("Quantize", 17.0, lambda: L.simtgo_Quantize(
            P(code.data_ptr()), n, P(energy.data_ptr()), n, P(clipped.data_ptr()), n,
            P(soft.data_ptr()), n, 0.25, 0x9E3779B9, G, 256, sp)),
        ("WarpReduceSum", 4.125, lambda: L.simtgo_WarpReduceSum(
            P(sums.data_ptr()), n // 32, P(soft.data_ptr()), n, W, 128, sp)),
    ]
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        for _, _, f in stages:
            _lib.check(f())
    torch.cuda.synchronize()
    steps = max(5, min(args.steps, 20))
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(len(stages) + 1)]
          for _ in range(steps)]
    for k in range(steps):
        ev[k][0].record(stream)
        for j, (_, _, f) in enumerate(stages):
            rc = f()
            if rc:
                _lib.check(rc)
            ev[k][j + 1].record(stream)
    ev[-1][-1].synchronize()
    hbm = peaks["hbm_gbs"]
    res = {"elements": n, "steps": steps, "stages": {}}
    total_ms = sum(ev[k][0].elapsed_time(ev[k][-1]) for k in range(steps)) / steps
    for j, (name, bpe, _) in enumerate(stages):
        ms = sum(ev[k][j].elapsed_time(ev[k][j + 1]) for k in range(steps)) / steps
        gbs = bpe * n / (ms * 1e-3) / 1e9
        res["stages"][name] = {"ms": round(ms, 4), "gbs": round(gbs, 1),
                               "frac_hbm": round(gbs / hbm, 4), "bytes_per_element": bpe}
    bpe = sum(b for _, b, _ in stages)
    gbs = bpe * n / (total_ms * 1e-3) / 1e9
    res.update({"ms": round(total_ms, 4), "gbs": round(gbs, 1), "frac_hbm": round(gbs / hbm, 4),
                "bytes_per_element": bpe,
                "gelements_per_s": round(n / (total_ms * 1e-3) / 1e9, 3)})
    # Parity of the first 2^20 elements of every stage (oracle, outside timing).
    O = oracle_module(1)
    m = min(n, 1 << 20)
    g = (m + 255) // 256
    zs = z[: 2 * m].cpu().numpy()
    ok = {}
    rc, w_mag = O.magnitudefast_interleaved(zs, 3.0, g, 256)
    ok["MagnitudeFast_interleaved"] = rc == 0 and np.array_equal(
        mag[:m].cpu().numpy().view(np.uint32), w_mag.view(np.uint32))
    rc, w_soft = O.softclip(w_mag, 0.5, g, 256)
    ok["Softclip"] = rc == 0 and np.array_equal(soft[:m].cpu().numpy().view(np.uint32),
                                                 w_soft.view(np.uint32))
    rc, wc, we, wk = O.quantize(w_soft, 0.25, 0x9E3779B9, g, 256)
    ok["Quantize"] = (rc == 0 and np.array_equal(code[:m].cpu().numpy(), wc)
                      and np.array_equal(energy[:m].cpu().numpy(), we)
                      and np.array_equal(clipped[:m].cpu().numpy(), wk))
    rc, ws = O.warpreducesum(w_soft, m // 32, (m + 127) // 128)
    ok["WarpReduceSum"] = rc == 0 and np.array_equal(sums[: m // 32].cpu().numpy().view(np.uint32),
                                                      ws.view(np.uint32))
    res["parity_first_2^20"] = {k: bool(v) for k, v in ok.items()}
    del z, mag, soft, code, energy, clipped, sums
    torch.cuda.empty_cache()
    return res


def in_turn(fns):
    """One callable that runs fns[0], fns[1], ... in turn, so that
    consecutive launches read different buffers whose total is larger than
    L2: each launch starts with its inputs out of L2, with no flush."""
    state = {"i": 0}

    def run():
        fns[state["i"] % len(fns)]()
        state["i"] += 1

    return run


def timed(fn, steps, warmup, stream, events):
    """Mean ms per launch of fn on stream: `steps` launches back to back
    between two CUDA events, after `warmup` untimed ones."""
    for _ in range(warmup):
        fn()
    import torch

    torch.cuda.synchronize()
    e0, e1 = events()
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / steps


def make_comm(torch, L, dev, rank, world):
    """The library's communicator over the job's ranks (rank 0's NCCL id
    broadcast through torch.distributed)."""
    from simtgo_b200 import _lib

    comm = P()
    uid = C.create_string_buffer(128)
    if world > 1:
        import torch.distributed as dist

        buf = torch.zeros(128, dtype=torch.uint8, device=dev)
        if rank == 0:
            _lib.check(L.simtgo_comm_unique_id(uid))
            buf.copy_(torch.frombuffer(bytearray(uid.raw), dtype=torch.uint8))
        dist.broadcast(buf, 0)
        uid = C.create_string_buffer(bytes(buf.cpu().numpy().tobytes()), 128)
    else:
        _lib.check(L.simtgo_comm_unique_id(uid))
    _lib.check(L.simtgo_comm_init(C.byref(comm), uid, world, rank))
    return comm


def bench_histogram(args, torch, L, dev, sp, rank, world, barrier, max_over_ranks, events):
    """2^28 samples in total, uniform over [0,255], split over the ranks;
    each rank counts its part and the bins are all-reduced (NCCL)."""
    from simtgo_b200 import _lib, shard

    total = 1 << 28
    n = shard.histogram_plan(total, world, rank).n
    gen = torch.Generator(device=dev).manual_seed(4 + rank)
    x = torch.randint(0, 256, (n,), dtype=torch.int32, device=dev, generator=gen)
    bins = torch.zeros(256, dtype=torch.int32, device=dev)
    comm = make_comm(torch, L, dev, rank, world)

    def run(fn, zero=True):
        def step():
            if zero:
                bins.zero_()
            rc = fn(comm, P(bins.data_ptr()), 256, P(x.data_ptr()), n, sp)
            if rc:
                _lib.check(rc)

        barrier()
        ms = max_over_ranks(timed(step, args.steps, args.warmup, torch.cuda.current_stream(),
                                  events))
        _lib.check(L.simtgo_stream_sync(sp))
        return ms, int(bins.sum().item()) == total

    ms, ok = run(L.simtgo_Histogram_allreduce)
    ms_f, ok_f = run(L.simtgo_Histogram_allreduce_fused_overwrite, zero=False)
    # Where the steps' time goes: the zeroing launch alone (the NCCL step's
    # first part), and this rank's count alone (the local kernel, no
    # exchange); the rest of the fused step is the exchange tail and the
    # ranks' skew.
    stream = torch.cuda.current_stream()
    barrier()
    ms_zero = max_over_ranks(timed(lambda: bins.zero_(), args.steps, args.warmup, stream, events))

    def count():
        rc = L.simtgo_Histogram_shard(P(bins.data_ptr()), 256, P(x.data_ptr()), n, sp)
        if rc:
            _lib.check(rc)

    barrier()
    ms_count = max_over_ranks(timed(count, args.steps, args.warmup, stream, events))
    barrier()
    _lib.check(L.simtgo_comm_destroy(comm))
    return {"samples_total": total, "ms_per_step": round(ms, 4),
            "gbs": round(4.0 * total / (ms * 1e-3) / 1e9, 1),
            "gsamples_per_s": round(total / (ms * 1e-3) / 1e9, 2),
            "scaling": "strong", "bins_sum_ok": ok,
            "step": "zero bins; local privatised histogram; NCCL all-reduce of 256 int32",
            "fused": {"ms_per_step": round(ms_f, 4),
                      "gsamples_per_s": round(total / (ms_f * 1e-3) / 1e9, 2),
                      "bins_sum_ok": ok_f,
                      "step": "one kernel: local histogram, then its last block stores the "
                              "counts to every rank over NVLink and sums the ranks' slots "
                              "into bins (simtgo_Histogram_allreduce_fused_overwrite: no "
                              "zeroing launch)"},
            "breakdown": {"zero_ms": round(ms_zero, 4), "local_count_ms": round(ms_count, 4),
                          "fused_exchange_and_skew_ms": round(ms_f - ms_count, 4),
                          "samples_per_rank": n,
                          "how": "each part timed alone with CUDA events, max over ranks; the "
                                 "fused step's exchange is its time less the local count"}}


def twelve(tile, g, a, b, c, h):
    s = tile.Scale(a, 0.5)
    ab = tile.Abs(b)
    q = tile.Sqrt(ab)
    m = tile.Mul(s, q)
    d = tile.Add(m, c)
    f = tile.FIR(s, h)
    y = tile.Hypot(d, f)
    return tile.Mul(y, ab)


def bench_tile(args, torch, np, L, dev, sp, rank, world, barrier, max_over_ranks, events):
    """3 x 2^28 inputs uniform[-4,4] through the 12-node graph, split over
    the ranks (a 32-element halo for the FIR node)."""
    from simtgo_b200 import shard, tile

    total = 1 << args.tile_log2
    plan = shard.tile_plan(total, world, rank, max_taps=31)
    n, halo = plan.n, plan.halo
    gen = torch.Generator(device=dev).manual_seed(6 + rank)
    ins = [torch.rand(n + halo, device=dev, generator=gen) * 8 - 4 for _ in range(3)]
    g = tile.New()
    a, b, c = (g.InputDevice(t[halo:]) for t in ins)
    root = twelve(tile, g, a, b, c, np.full(31, 1 / 31, np.float32))
    out = torch.empty(n, device=dev)
    stream = torch.cuda.current_stream()

    def step():
        root.Run(out, stream, halo=halo)

    # The first run of the graph compiles its specialised kernel (NVRTC);
    # its wall time, compile included, is reported, and the timed steps
    # that follow launch the cached kernel.
    mode, nvrtc, _, launches0, _ = tile.JITInfo()
    t0 = time.perf_counter()
    step()
    torch.cuda.synchronize()
    first_s = time.perf_counter() - t0
    barrier()
    ms = timed(step, args.steps, args.warmup, stream, events)
    ms = max_over_ranks(ms)
    specialised = tile.JITInfo()[3] > launches0
    res = {"elements_total": total, "ms_per_step": round(ms, 4),
           "gbs": round(16.0 * total / (ms * 1e-3) / 1e9, 1),
           "gelements_per_s": round(total / (ms * 1e-3) / 1e9, 2),
           "scaling": "strong", "bytes_per_element": 16,
           "kernel": ("the graph's specialised kernel (its program compiled in as constants "
                      "by NVRTC for sm_100a, cached)" if specialised else
                      "the precompiled interpreter"),
           "first_run_s": round(first_s, 3)}
    if world == 1 and specialised:
        # The same step on the precompiled interpreter, for comparison.
        tile.SetJIT(0)
        ims = timed(step, args.steps, args.warmup, stream, events)
        tile.SetJIT(mode)
        res["interpreter"] = {"ms_per_step": round(ims, 4),
                              "gbs": round(16.0 * total / (ims * 1e-3) / 1e9, 1)}
    # Parity: this rank's first 2^22 outputs (and its halo) against the
    # oracle's node-by-node evaluation, outside the timed region.
    O = oracle_module(world)
    m = min(n, 1 << 22)
    host = [t[: halo + m].cpu().numpy() for t in ins]
    taps = np.full(31, 1 / 31, np.float32)
    nodes = [{"kind": "input", "data": host[0]}, {"kind": "input", "data": host[1]},
             {"kind": "input", "data": host[2]}, {"kind": "scale", "a": 0, "scale": 0.5},
             {"kind": "abs", "a": 1}, {"kind": "sqrt", "a": 4}, {"kind": "mul", "a": 3, "b": 5},
             {"kind": "add", "a": 6, "b": 2}, {"kind": "input", "data": taps},
             {"kind": "fir", "a": 3, "taps": taps}, {"kind": "hypot", "a": 7, "b": 9},
             {"kind": "mul", "a": 10, "b": 4}]
    rc, want = O.tile_eval(nodes, 11, m, halo)
    got = out[:m].cpu().numpy()
    res["parity"] = {"outputs": m, "bit_exact": bool(rc == 0 and np.array_equal(
        got.view(np.uint32), want.view(np.uint32))),
        "check": "this rank's first outputs against the oracle, outside the timed region"}
    if world == 1:
        # Other graphs over the same inputs: what the interpreter costs per
        # kind of node (the twelve-node graph is compute-heavy: a 31-tap
        # window, the exact hypot and a square root per element).
        peak = measured_peaks()[0]["hbm_gbs"]
        graphs = {
            "identity": (lambda: a, 8),
            "add3": (lambda: tile.Add(tile.Add(a, b), c), 16),
            "mul_chain8": (lambda: _chain(tile, a, b, 8), 12),
            "hypot": (lambda: tile.Hypot(a, b), 12),
            "fir31": (lambda: tile.FIR(a, np.full(31, 1 / 31, np.float32)), 8),
        }
        res["graphs"] = {}
        for name, (make, nbytes) in graphs.items():
            r = make()
            gms = timed(lambda: r.Run(out, stream, halo=halo), args.steps, args.warmup, stream,
                        events)
            gbs = nbytes * total / (gms * 1e-3) / 1e9
            res["graphs"][name] = {"ms": round(gms, 4), "gbs": round(gbs, 1),
                                   "frac_hbm": round(gbs / peak, 4), "bytes_per_element": nbytes}
    return res


def bench_tile_reduce(args, torch, L, dev, rank, world, barrier, max_over_ranks, events):
    """Tile reductions over 2^28 uniform[-4,4] samples split over the ranks
    in whole blocks of 2048 (tile.ShardRange): the sum of squares and the
    argmax, each one fused pass over HBM plus, for N > 1, the NCCL
    all-gather of the block partials; every rank ends with the whole
    signal's result."""
    from simtgo_b200 import _lib, tile

    total = 1 << args.tile_log2
    start, n = tile.ShardRange(total, world, rank)
    gen = torch.Generator(device=dev).manual_seed(12 + rank)
    x = torch.rand(n, device=dev, generator=gen) * 8 - 4
    g = tile.New()
    a = g.InputDevice(x)
    comm = make_comm(torch, L, dev, rank, world)
    v = torch.zeros(1, device=dev)
    i = torch.zeros(1, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream()
    peak = measured_peaks()[0]["hbm_gbs"]
    res = {"elements_total": total, "scaling": "strong", "bytes_per_element": 4,
           "split": "whole blocks of 2048 per rank (tile.ShardRange)"}
    # argmax_abs: the peak of |k x| (a chain of two steps, which runs in
    # its own specialised streaming kernel).
    for name, red in (("sum_of_squares", tile.Sum(tile.Mul(a, a))), ("argmax", tile.ArgMax(a)),
                      ("argmax_abs", tile.ArgMax(tile.Abs(tile.Scale(a, -2.0))))):
        barrier()
        ms = max_over_ranks(timed(lambda: red.RunShard(comm, total, v, i, stream=stream),
                                  args.steps, args.warmup, stream, events))
        gbs = 4.0 * total / (ms * 1e-3) / 1e9
        res[name] = {"ms": round(ms, 4), "gbs": round(gbs, 1),
                     "frac_hbm_per_gpu": round(gbs / world / peak, 4),
                     "value": float(v.item()),
                     "index": int(i.item()) if name.startswith("argmax") else None}
    barrier()
    _lib.check(L.simtgo_comm_destroy(comm))
    return res


def _chain(tile, a, b, k):
    r = a
    for _ in range(k):
        r = tile.Mul(r, b)
    return r


def bench_kernels(args, torch, np, L, dev, sp, events, peaks):
    """Each kernel at its workload size, inputs resident and larger than L2,
    timed with CUDA events; GB/s from the algorithmic bytes per unit."""
    stream = torch.cuda.current_stream()
    steps, warm = max(5, min(args.steps, 20)), 3
    hbm = peaks["hbm_gbs"]
    out = {}
    N = 1 << args.kernels_log2
    gen = torch.Generator(device=dev).manual_seed(11)

    def rec(name, ms, nbytes, units, unit_name):
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"ms": round(ms, 4), "gbs": round(gbs, 1), "frac_hbm": round(gbs / hbm, 4),
                     "size": units, "unit": unit_name,
                     "bytes_per_unit": round(nbytes / units, 3)}

    def grid(n, block=256):
        return (n + block - 1) // block

    a = torch.randn(N, device=dev, generator=gen)
    b = torch.randn(N, device=dev, generator=gen)
    c = torch.empty(N, device=dev)
    pa, pb, pc = P(a.data_ptr()), P(b.data_ptr()), P(c.data_ptr())
    G = grid(N)
    rec("VecAdd", timed(lambda: L.simtgo_VecAdd(pc, N, pa, N, pb, N, G, 256, sp), steps, warm,
                        stream, events), 12.0 * N, N, "elements")
    rec("Scale", timed(lambda: L.simtgo_Scale(pc, N, pa, N, 0.75, G, 256, sp), steps, warm,
                       stream, events), 8.0 * N, N, "elements")
    rec("Magnitude", timed(lambda: L.simtgo_Magnitude(pc, N, pa, N, pb, N, G, 256, sp), steps,
                           warm, stream, events), 12.0 * N, N, "elements")
    rec("MagnitudeFast", timed(lambda: L.simtgo_MagnitudeFast(pc, N, pa, N, pb, N, 3.0, G, 256,
                                                              sp), steps, warm, stream, events),
        12.0 * N, N, "elements")
    rec("Softclip", timed(lambda: L.simtgo_Softclip(pc, N, pa, N, 0.5, G, 256, sp), steps, warm,
                          stream, events), 8.0 * N, N, "elements")
    edges = torch.tensor([0.1, 0.25, 0.5, 0.8, 1.2, 1.8, 2.5], device=dev)
    rec("Classify", timed(lambda: L.simtgo_Classify(pc, N, pa, N, P(edges.data_ptr()), 7, G, 256,
                                                    sp), steps, warm, stream, events),
        8.0 * N, N, "elements")
    from simtgo_b200._lib import Shape

    bands = torch.tensor([-0.5, 0.25, 0.0, 0.5, 0.5, 1.0, 1.0, 2.0], device=dev)
    cfg = Shape(0.125, 3, 0.001)
    rec("BandGain", timed(lambda: L.simtgo_BandGain(pc, N, pa, N, P(bands.data_ptr()), 4,
                                                    C.byref(cfg), G, 256, sp), steps, warm,
                          stream, events), 8.0 * N, N, "elements")
    WN = N // 32
    rec("WarpReduceSum", timed(lambda: L.simtgo_WarpReduceSum(pc, WN, pa, N, grid(N, 128), 128,
                                                              sp), steps, warm, stream, events),
        4.125 * N, N, "elements")
    del b
    torch.cuda.empty_cache()
    # Signal chain: interleaved complex -> MagnitudeFast -> Softclip -> Quantize.
    z = torch.randn(2 * N, device=dev, generator=gen)
    rec("MagnitudeFast_interleaved",
        timed(lambda: L.simtgo_MagnitudeFast_interleaved(pc, N, P(z.data_ptr()), 2 * N, 3.0, G,
                                                         256, sp), steps, warm, stream, events),
        12.0 * N, N, "complex samples")
    del z
    torch.cuda.empty_cache()
    code = torch.empty(N, dtype=torch.int32, device=dev)
    energy = torch.empty(N, dtype=torch.int64, device=dev)
    clipped = torch.empty(N, dtype=torch.uint8, device=dev)
    rec("Quantize", timed(lambda: L.simtgo_Quantize(P(code.data_ptr()), N, P(energy.data_ptr()),
                                                    N, P(clipped.data_ptr()), N, pa, N, 0.25,
                                                    0x9E3779B9, G, 256, sp), steps, warm,
                          stream, events), 17.0 * N, N, "elements")
    del code, energy, clipped
    xi = torch.randint(0, 256, (N,), dtype=torch.int32, device=dev, generator=gen)
    bins = torch.zeros(256, dtype=torch.int32, device=dev)
    rec("Histogram", timed(lambda: L.simtgo_Histogram(P(bins.data_ptr()), 256, P(xi.data_ptr()), N,
                                                      G, 256, sp), steps, warm, stream, events),
        4.0 * N, N, "samples (uniform)")
    p = (torch.arange(256, device=dev, dtype=torch.float64) + 1) ** -1.2
    cdf = torch.cumsum(p / p.sum(), 0)
    u = torch.rand(N, device=dev, generator=gen, dtype=torch.float64)
    xi = torch.searchsorted(cdf, u).clamp_(max=255).to(torch.int32)
    del u
    rec("Histogram_zipf", timed(lambda: L.simtgo_Histogram(P(bins.data_ptr()), 256,
                                                           P(xi.data_ptr()), N, G, 256, sp),
                                steps, warm, stream, events), 4.0 * N, N, "samples (Zipf 1.2)")
    # The launch-sized tile (LaunchShared): 4096 bins, uniform samples.
    xi = torch.randint(0, 4096, (N,), dtype=torch.int32, device=dev, generator=gen)
    bins4k = torch.zeros(4096, dtype=torch.int32, device=dev)
    rec("HistogramDyn_4096", timed(lambda: L.simtgo_HistogramDyn(P(bins4k.data_ptr()), 4096,
                                                                 P(xi.data_ptr()), N, 4096, G,
                                                                 256, sp),
                                   steps, warm, stream, events), 4.0 * N, N,
        "samples (4096-bin launch-sized tile)")
    del xi
    torch.cuda.empty_cache()
    # Gray 7680x4320: 133 MB of traffic per image, about the size of L2, so
    # four images are converted in turn (532 MB).
    npx = 7680 * 4320
    imgs = [(torch.empty(npx, dtype=torch.uint8, device=dev),
             torch.randint(0, 256, (3 * npx,), dtype=torch.uint8, device=dev, generator=gen))
            for _ in range(4)]
    rec("Gray", timed(in_turn([
        (lambda lu=lu, rgb=rgb: L.simtgo_Gray(P(lu.data_ptr()), npx, P(rgb.data_ptr()), 3 * npx,
                                              grid(npx), 256, sp)) for lu, rgb in imgs]),
        steps, warm, stream, events), 4.0 * npx, npx,
        "pixels (4 images in turn, 532 MB: inputs larger than L2, no flush)")
    del imgs
    # Transpose 16384^2 (at the default size; T*T = N).
    T = 1 << (args.kernels_log2 // 2)
    rec("Transpose", timed(lambda: L.simtgo_Transpose(pc, T * T, pa, T * T, T, T, T // 16,
                                                      T // 16, 16, 16, sp), steps, warm, stream,
                           events), 8.0 * T * T, T * T, "elements")
    # FIR of the 2^20-sample, 31-tap case: 32 signals filtered in turn
    # (256 MB), so each launch starts with its 8 MB out of L2. A launch is a
    # few microseconds, less than a host-side call from Python, so the 32
    # launches are captured once in a CUDA graph and the graph is replayed:
    # the time is the device's, per launch.
    n20 = 1 << 20
    h31 = torch.rand(31, device=dev, generator=gen)
    h31 /= h31.sum()
    sig = [(torch.empty(n20, device=dev), torch.randn(n20, device=dev, generator=gen))
           for _ in range(32)]

    def fir20(y, x, s):
        rc = L.simtgo_FIR(P(y.data_ptr()), n20, P(x.data_ptr()), n20, P(h31.data_ptr()), 31,
                          n20 // 256, 256, P(s))
        if rc:
            from simtgo_b200 import _lib
            _lib.check(rc)

    for y, x in sig:
        fir20(y, x, stream.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream(dev)
    cap.wait_stream(stream)
    with torch.cuda.graph(graph, stream=cap, capture_error_mode="thread_local"):
        for y, x in sig:
            fir20(y, x, cap.cuda_stream)
    torch.cuda.synchronize()
    rec("FIR_31taps_2^20", timed(graph.replay, max(3, steps // 4), 2, stream, events) / len(sig),
        8.0 * n20, n20,
        "outputs (32 signals in turn, 256 MB: inputs larger than L2, no flush; the 32 "
        "launches replayed as one CUDA graph, time per launch)")
    del graph, sig
    return out


def cpu_baseline(args, np, seconds):
    """The oracle's FIR in gpu.RunCPU's order (fir_shard_runcpu) on every
    host core, over a bounded leading sample of rank 0's shard."""
    sys.path.insert(0, str(ROOT / "tests"))
    import oracle_lib as O

    threads = os.cpu_count() or 1
    O.set_threads(threads)
    h = fir_taps()
    sample = 1 << 22
    x = np.random.default_rng(0).uniform(-1, 1, sample + TAPS).astype(np.float32)
    done, t0 = 0, time.perf_counter()
    while True:
        O.fir_shard(x, 0, h, sample, fused=False)
        done += 1
        dt = time.perf_counter() - t0
        if dt >= seconds:
            break
    value = done * sample / dt / 1e9
    # One core, for scale: the same code on a smaller sample for ~1 s.
    O.set_threads(1)
    one = 1 << 18
    done1, t1 = 0, time.perf_counter()
    while True:
        O.fir_shard(x[: one + TAPS], 0, h, one, fused=False)
        done1 += 1
        dt1 = time.perf_counter() - t1
        if dt1 >= min(1.0, seconds):
            break
    O.set_threads(threads)
    return {"value": round(value, 4), "unit": "Gsamples/s", "cores": threads,
            "kind": "port", "seconds": round(dt, 2),
            "single_core_value": round(done1 * one / dt1 / 1e9, 4),
            "sample": f"{done} x {sample} outputs x {TAPS} taps of the FIR workload (the oracle "
                      "port of gpu.RunCPU's FIR, -O3 -ffp-contract=off, block-parallel pthreads "
                      f"on every host core); single_core_value: {done1} x {one} outputs on one "
                      "thread"}


def run_reference(args):
    """The reference arm: the oracle port of gpu.RunCPU's FIR on the host
    cores, rank 0 only (no GPU work)."""
    import numpy as np

    rank, world, _ = env_rank()
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT / "tests"))
    import oracle_lib as O

    threads = os.cpu_count() or 1
    O.set_threads(threads)
    h = fir_taps()
    x = np.random.default_rng(0).uniform(-1, 1, (1 << 22) + TAPS).astype(np.float32)
    probe = 1 << 16
    t0 = time.perf_counter()
    O.fir_shard(x[: probe + TAPS], 0, h, probe, fused=False)
    dt = time.perf_counter() - t0
    per_step_s = min(2.0, 150.0 / max(1, args.steps + args.warmup))
    sample = int(min(1 << 22, max(probe, probe * per_step_s / max(dt, 1e-6))))
    for _ in range(args.warmup):
        O.fir_shard(x[: sample + TAPS], 0, h, sample, fused=False)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.fir_shard(x[: sample + TAPS], 0, h, sample, fused=False)
    dt = time.perf_counter() - t0
    value = sample * args.steps / dt / 1e9
    kind = "port"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "Gsamples/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"FIR, 2^{args.fir_log2} outputs per GPU, {TAPS} taps "
                               f"(bounded CPU sample of {sample} outputs per step)",
                   "taps": TAPS},
        "cpu_baseline": {"value": round(value, 4), "unit": "Gsamples/s", "cores": threads,
                         "kind": kind,
                         "sample": f"{sample} outputs x {TAPS} taps per step; the reference's "
                                   "generated FIR.cu holds at most 65 taps in its 320-sample "
                                   "tile, so its CPU path for 127 taps is the oracle port of "
                                   "gpu.RunCPU's arithmetic"},
        "e2e": {"value": round(value, 4), "unit": "Gsamples/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--fir-log2", type=int, default=FIR_LOG2)
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--soak-s", type=float, default=1.5)
    ap.add_argument("--tile-log2", type=int, default=28)
    ap.add_argument("--fir-strong-log2", type=int, default=31,
                    help="samples of the strong-scaling FIR signal (31 = the 2^31 x 127 workload)")
    ap.add_argument("--chain-log2", type=int, default=28)
    ap.add_argument("--kernels-log2", type=int, default=28,
                    help="elements per kernel in the per-kernel table (20..28; 28 = the workloads)")
    ap.add_argument("--skip-kernels", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if not 20 <= args.kernels_log2 <= 28:
        ap.error("--kernels-log2 must be within 20..28")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
