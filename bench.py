"""Benchmark: one synthetic 50-block DiT denoising step of Q4_K projections on B200.

Workload (the headline "DiT step" of its metric): d = 5120,
40 heads x 128, FFN 13824, M = 32760 video + 1024 audio = 33784 latent rows, 512 text
rows, 50 blocks of Q4_K weights (11.87 GB) resident in HBM.  Rows are sharded across
N GPUs (strong scaling: total rows fixed) and gathered with an NCCL all-gather at the
end of the step.  The other BASELINE configs are parity-test cases (tests/).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Prints one JSON line on rank 0.  `value` = GEMM TFLOP/s of the whole step (useful
FLOPs of all 33784 rows, text K/V counted once) / device time, max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Q4_K DiT step ms & dequant-GEMM TFLOP/s (GEMV GB/s) at 1/2/4/8 B200 vs host CPU"
UNIT = "TFLOP/s"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# dram__bytes_read.sum + dram__bytes_write.sum per FLOP of one gemm_bf16_pair_kernel fc1 launch
# (8192 rows: 1164.4 + 219.6 MB for 2.319 TFLOP, profiles/gemm_bf16_pair_fc1_m8192.md), scaled to
# the bench's fc1 launch at this rank's rows.
GEMM_TRAFFIC_BYTES_PER_FLOP = (1164.4e6 + 219.6e6) / 2.319e12


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--blocks", type=int, default=50)
    ap.add_argument("--rows", type=int, default=32760 + 1024)
    ap.add_argument("--text-rows", type=int, default=512)
    ap.add_argument("--e2e-steps", type=int, default=4)
    ap.add_argument("--cpu-seconds", type=float, default=8.0, help="target CPU baseline sample time")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the output check (N = 1: sampled rows against the CPU oracle through all "
                         "blocks; N > 1: rank 0 recomputes every other rank's shard and compares bitwise)")
    ap.add_argument("--parity-rows", type=int, default=4)
    ap.add_argument("--no-overlap", action="store_true",
                    help="run each projection as one fh3cuda_gemm_q4k_dev call (no second stream)")
    ap.add_argument("--no-gemv", action="store_true",
                    help="skip the GEMV (1..4 token), q/k norm+rope and attention measurements")
    ap.add_argument("--case", choices=["gemm", "matmul", "gemv", "qk", "attn", "vsa", "norm"], default=None,
                    help="run one kernel's launches on a small case (for ncu) instead of the bench")
    ap.add_argument("--case-rows", type=int, default=8192, help="--case gemm / qk: activation rows")
    ap.add_argument("--case-kn", type=int, nargs=2, default=(5120, 13824), help="--case gemv: in, out")
    ap.add_argument("--case-m", type=int, default=1, help="--case gemv: tokens")
    ap.add_argument("--case-reps", type=int, default=3)
    return ap.parse_args()


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


class Clocks:
    """nvidia-smi sampler for the timed region (SM clock, throttle reasons)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.lines = []
        self.t_region = 0.0

    def start(self):
        """Start sampling and return once the first sample has arrived (nvidia-smi takes a
        while to start), so that a short timed region is sampled too; samples that arrive
        before this returns are not counted."""
        import threading
        self.lines = []
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return

        def read():
            for line in self.proc.stdout:
                self.lines.append((time.time(), line))

        self.reader = threading.Thread(target=read, daemon=True)
        self.reader.start()
        t0 = time.time()
        while not self.lines and self.proc.poll() is None and time.time() - t0 < 5.0:
            time.sleep(0.01)
        self.t_region = time.time()

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait()
        self.reader.join(timeout=5)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for t, line in self.lines:
            if t < self.t_region:
                continue
            f = [c.strip() for c in line.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- CPU legs
def host_cpu() -> dict:
    """CPU model, logical CPUs this process may run on, and the physical cores among them."""
    avail = sorted(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else list(range(os.cpu_count() or 1))
    cores = set()
    for c in avail:
        base = f"/sys/devices/system/cpu/cpu{c}/topology/"
        try:
            with open(base + "physical_package_id") as f:
                pkg = f.read().strip()
            with open(base + "core_id") as f:
                core = f.read().strip()
        except OSError:
            pkg, core = "0", str(c)
        cores.add((pkg, core))
    model = "unknown"
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"model": model, "logical_cpus": len(avail), "physical_cores": len(cores)}


def pin_cpu_threads(n: int) -> int:
    """Give the OpenMP runtime of the CPU legs n threads, whatever the launcher set.

    torch.distributed.run exports OMP_NUM_THREADS=1 to every rank; the reference's fh3_matmul
    (and the oracle) run on the system libgomp, whose thread count is set here both through the
    environment (read when libgomp initialises) and through omp_set_num_threads (which overrides
    it afterwards).  Returns the thread count the oracle library then reports."""
    import ctypes
    os.environ["OMP_NUM_THREADS"] = str(n)
    from oracle import oracle as orc
    o = orc.Oracle()
    if orc.Reference.available():
        orc.Reference()
    try:
        ctypes.CDLL("libgomp.so.1").omp_set_num_threads(n)
    except OSError:
        pass
    return o.num_threads()


def cpu_sample(trunk_block_raw, rows_s: int, text_s: int, threads: int, use_ref: bool, reps: int = 1):
    """Time the reference's fh3_matmul (or the oracle port) on one block's projections.

    Returns (flops, best seconds, kind)."""
    import numpy as np

    from fasth3inc_b200.trunk import D_MODEL, FFN, block_shapes
    from oracle import oracle as orc
    if use_ref and orc.Reference.available():
        impl, kind = orc.Reference(), "reference"
    else:
        impl, kind = orc.Oracle(), "port"
    rng = np.random.default_rng(0)
    xs = {D_MODEL: rng.standard_normal((rows_s, D_MODEL), dtype=np.float32),
          FFN: rng.standard_normal((rows_s, FFN), dtype=np.float32)}
    xt = rng.standard_normal((text_s, D_MODEL), dtype=np.float32)
    flops = 0
    for name, out, inn in block_shapes():
        r = text_s if name == "ckv" else rows_s
        flops += 2 * r * inn * out
    best = None
    for _ in range(reps):
        t0 = time.perf_counter()
        for name, out, inn in block_shapes():
            x = xt if name == "ckv" else xs[inn]
            impl.matmul(12, trunk_block_raw[name], inn, out, x)
        dt = time.perf_counter() - t0
        best = dt if best is None else min(best, dt)
    return flops, best, kind


def host_block_weights(trunk, b: int = 0) -> dict:
    """Download block b's Q4_K bytes (the same weights the GPU uses) for the CPU legs."""
    return {k: w.data.cpu().numpy() for k, w in trunk.blocks[b].w.items()}


def size_cpu_sample(raw, threads, use_ref, target_s):
    rows = 16
    flops, dt, kind = cpu_sample(raw, rows, rows, threads, use_ref)
    rows = int(max(16, min(4096, rows * target_s / max(dt, 1e-3))))
    return rows


# ----------------------------------------------------------------------------- ours
def run_ours(args):
    import torch
    import torch.distributed as dist

    import fasth3inc_b200 as fh3
    from fasth3inc_b200.trunk import (Runner, Trunk, Workspace, block_flops, rows_for_rank, D_MODEL, FFN)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and world > 1:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        os.environ.setdefault("NCCL_NVLS_ENABLE", "1")
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    fh3.init(local)
    M, T = args.rows, args.text_rows
    r0, r1 = rows_for_rank(M, rank, world)
    m_loc = r1 - r0
    t_build = time.time()
    trunk = Trunk(n_blocks=args.blocks, seed=0, device=local).build()
    t_build = time.time() - t_build
    ws = Workspace(m_loc, T, device=local)
    dev = f"cuda:{local}"
    g = torch.Generator(device=dev).manual_seed(1234)
    h_full = torch.randn((M, D_MODEL), device=dev, generator=g)          # seeded N(0,1) latent rows
    text = torch.randn((T, D_MODEL), device=dev, generator=g)
    text_bf = fh3.to_bf16(text)
    h0 = h_full[r0:r1].clone()
    h = h0.clone()
    stream = torch.cuda.current_stream(local)
    runner = Runner(trunk, ws, stream, overlap=not args.no_overlap)
    # gather target: padded equal shards for all_gather_into_tensor
    shard = (M + world - 1) // world
    gather_out = torch.empty((shard * world, D_MODEL), device=dev) if world > 1 else None
    send = torch.empty((shard, D_MODEL), device=dev) if world > 1 else None

    ag_events = None   # (start, end) of each all-gather when recording

    def step():
        h.copy_(h0)  # every step starts from the same latents
        runner.step(h, text_bf)
        if world > 1:
            send[:m_loc].copy_(h)
            if ag_events is not None:
                a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a0.record(stream)
            dist.all_gather_into_tensor(gather_out, send)
            if ag_events is not None:
                a1.record(stream)
                ag_events.append((a0, a1))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    status = fh3.device_status()
    if status != 0:
        raise SystemExit(f"device status {status} after warm-up")

    # timed region
    clocks = Clocks(local)
    clocks.start()  # returns once sampling runs; the barrier then lines the ranks up
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    runner.gemm_events, runner.expand_events, runner.norm_events = [], [], []
    ag_events = []
    runner.launches = 0
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    ms_local = e0.elapsed_time(e1) / args.steps
    def total_ms(evs, tag_prefix=None):
        return sum(a.elapsed_time(b) for a, b, _, t in evs if tag_prefix is None or t.startswith(tag_prefix))
    gemm_ms = total_ms(runner.gemm_events)
    gemm_flops = sum(f for _, _, f, _ in runner.gemm_events)
    ckv_ms = sum(a.elapsed_time(b) for a, b, _, t in runner.gemm_events if t == f"fused:{T}")
    expand_ms = total_ms(runner.expand_events)
    norm_ms = total_ms(runner.norm_events)
    ag_ms = sum(a.elapsed_time(b) for a, b in ag_events)
    launches = runner.launches
    runner.gemm_events = runner.expand_events = runner.norm_events = None
    ag_events = None
    stat = torch.tensor([ms_local, gemm_ms, float(gemm_flops), float(launches), ckv_ms, expand_ms, norm_ms, ag_ms],
                        device=dev, dtype=torch.float64)
    if world > 1:
        mx = stat.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = stat.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
    else:
        mx = sm = stat
    ms = float(mx[0])
    total_flops = args.blocks * block_flops(M, T)   # useful FLOPs of the whole step
    value = total_flops / (ms * 1e-3) / 1e12
    # roofline of the dominant kernel: rank-local GEMM events (max over ranks of time)
    gemm_tflops = float(sm[2]) / world / (float(mx[1]) * 1e-3) / 1e12 if float(mx[1]) > 0 else None

    # ---- end to end through the public API with host buffers
    e2e_val = None
    h_host = torch.empty((m_loc, D_MODEL), dtype=torch.float32, pin_memory=True)
    h_host.copy_(h0.cpu())
    t_host = text.cpu().pin_memory()
    out_host = torch.empty((M if world > 1 else m_loc, D_MODEL), dtype=torch.float32, pin_memory=True)
    h2d = h_host.numel() * 4 + t_host.numel() * 4
    d2h = out_host.numel() * 4 if rank == 0 else 0
    # Inputs double-buffered on the device and copied on a copy stream, so that one step's
    # upload and the previous step's readback run beside the neighbouring steps' compute; every
    # step still copies its own inputs in and its result out inside the timed region, which
    # opens before the first upload and closes after the last readback.
    cs = torch.cuda.Stream(device=dev)
    hb = [h, torch.empty_like(h)]
    tb = [torch.empty_like(text), torch.empty_like(text)]

    def e2e_run(n: int) -> None:
        opened = torch.cuda.Event()
        opened.record(stream)
        cs.wait_event(opened)
        ins, outs = [None] * n, [None] * n

        def upload(i):
            with torch.cuda.stream(cs):
                hb[i % 2].copy_(h_host, non_blocking=True)
                tb[i % 2].copy_(t_host, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(cs)
                ins[i] = ev

        upload(0)
        if n > 1:
            upload(1)
        for i in range(n):
            stream.wait_event(ins[i])
            fh3.to_bf16(tb[i % 2], out=text_bf)
            runner.step(hb[i % 2], text_bf)
            src = hb[i % 2]
            if world > 1:
                if i > 0:
                    stream.wait_event(outs[i - 1])  # the previous readback has left gather_out
                send[:m_loc].copy_(hb[i % 2])
                dist.all_gather_into_tensor(gather_out, send)
                src = gather_out[:M] if rank == 0 else None
            done = torch.cuda.Event()
            done.record(stream)
            cs.wait_event(done)
            with torch.cuda.stream(cs):
                if src is not None:
                    out_host.copy_(src, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(cs)
                outs[i] = ev
            if i + 2 < n:
                upload(i + 2)  # into the buffer this step has finished with (the copy stream is in order)
        stream.wait_event(outs[n - 1])

    e2e_run(1)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    a0 = torch.cuda.Event(enable_timing=True)
    a1 = torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    e2e_run(args.e2e_steps)
    a1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([a0.elapsed_time(a1) / args.e2e_steps], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_val = total_flops / (float(e2e_ms[0]) * 1e-3) / 1e12
    status = fh3.device_status()

    # ---- output check (outside every timed region)
    parity = None
    if not args.no_parity:
        if world > 1:
            parity = {"method": "rank 0 recomputed every other rank's row shard on its own GPU (same launches) and "
                                "compared the all-gathered rows bit for bit", "shards_checked": 0,
                      "bitwise_equal": None}
            if rank == 0:
                ok = True
                for r in range(1, world):
                    a, b = rows_for_rank(M, r, world)
                    hr = h_full[a:b].clone()
                    runner.step(hr, text_bf)
                    ok = ok and bool(torch.equal(hr, gather_out[r * shard:r * shard + (b - a)]))
                    parity["shards_checked"] += 1
                ok = ok and bool(torch.equal(h, gather_out[:m_loc]))
                parity["bitwise_equal"] = ok
                parity["ok"] = ok
        elif rank == 0:
            parity = parity_vs_oracle(fh3, torch, trunk, h0, h, text_bf, args.parity_rows)

    # ---- CPU baseline (rank 0, N = 1 only)
    cpu = None
    hc = host_cpu()
    cpu_threads = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_threads = pin_cpu_threads(hc["physical_cores"])
        raw = host_block_weights(trunk, 0)
        rows_s = size_cpu_sample(raw, cpu_threads, True, args.cpu_seconds)
        f, dt, kind = cpu_sample(raw, rows_s, min(rows_s, T), cpu_threads, True, reps=1)
        cpu = {"value": round(f / dt / 1e12, 5), "unit": UNIT, "cores": cpu_threads, "kind": kind,
               "cpu": hc,
               "sample": f"block 0's 7 Q4_K projections (fh3_matmul, OpenMP, {cpu_threads} threads) on {rows_s} "
                         f"latent rows and {min(rows_s, T)} text rows = {f / 1e9:.1f} GFLOP in {dt:.2f} s; same "
                         f"weights as the GPU"}

    peaks, src = load_peaks()
    gemv = qk = attn = vsa = configs = None
    if rank == 0 and not args.no_gemv:
        hbm = float(peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
        configs = measure_configs(fh3, torch, trunk, text_bf,
                                  float(peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"])), src, cpu_threads)
        gemv = measure_gemv(fh3, torch, hbm, src, cpu_threads=cpu_threads)
        qk = measure_qk_norm_rope(fh3, torch, m_loc, hbm, src)
        attn = measure_attention(fh3, torch, m_loc, float(peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"])),
                                 src)
        vsa = measure_vsa(fh3, torch, m_loc, float(peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"])), src)
    peak = float(peaks.get("bf16_tflops_sustained", PEAKS_FALLBACK["bf16_tflops_sustained"]))
    roof = None
    if gemm_tflops:
        traffic = None
        if GEMM_TRAFFIC_BYTES_PER_FLOP is not None:   # bytes per launch of the fc1 GEMM at this rank's rows
            traffic = int(GEMM_TRAFFIC_BYTES_PER_FLOP * 2 * m_loc * D_MODEL * 2 * FFN)
        roof = {"bound": "tensor", "achieved": round(gemm_tflops, 1), "peak": peak, "unit": "TFLOP/s",
                "frac": round(gemm_tflops / peak, 4), "traffic": traffic,
                "traffic_note": "DRAM bytes of one fc1 gemm_bf16_pair_kernel launch at this rank's rows, scaled "
                                "from an 8192-row ncu capture",
                "achieved_note": "GEMM FLOPs / the GEMM launches' CUDA-event time on the main stream (the "
                                 "Q4_K -> bf16 expansions run beside them on a second stream; their time is "
                                 "in breakdown.expand_ms)",
                "kernel": "gemm_bf16_pair_kernel", "peak_source": f"{src} bf16_tflops_sustained",
                "gemm_share_of_step": round(float(mx[1]) / (ms * args.steps), 4)}
    breakdown = {"unit": "ms per step, max over ranks of each rank's CUDA-event sums",
                 "gemm_ms": round(float(mx[1]) / args.steps, 3),
                 "ckv_gemm_ms": round(float(mx[4]) / args.steps, 3),
                 "expand_ms_side_stream": round(float(mx[5]) / args.steps, 3),
                 "norm_ms": round(float(mx[6]) / args.steps, 3),
                 "allgather_ms": round(float(mx[7]) / args.steps, 3),
                 "rows_per_rank": m_loc,
                 "ms_per_step_x_sm_ghz": round(ms * clk["sm_mhz"] / 1000.0, 2) if clk.get("sm_mhz") else None,
                 "note": "the expansions overlap the GEMMs (second stream); ckv is the 512-text-row K/V "
                         "projection every rank computes; ms_per_step_x_sm_ghz normalises the step by the median "
                         "SM clock seen in the timed region"}
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 2), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded N(0,0.02) weights quantised to Q4_K on the device, N(0,1) fp32 latent rows",
            "config": {"workload": "BASELINE config 5: 50-block synthetic DiT trunk step (Q4_K GEMMs, AdaLN "
                                   "rmsnorm+modulate, SwiGLU and gated-residual epilogues)",
                       "blocks": args.blocks, "rows": M, "text_rows": T, "d_model": D_MODEL, "heads": 40,
                       "head_dim": 128, "ffn": FFN, "weights_gb": round(trunk.weight_bytes / 1e9, 3),
                       "step_gflop": round(total_flops / 1e9, 1), "parallelism": f"rows{world}",
                       "l2": "inputs larger than L2 (11.87 GB of Q4_K weights streamed every step)",
                       "trunk_build_s": round(t_build, 1)},
            "roofline": roof, "breakdown": breakdown, "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_val, 2), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": args.e2e_steps,
                    "method": "every step uploads its latent and text rows from pinned host memory and reads its "
                              "output rows back, on a copy stream beside the neighbouring steps' compute (inputs "
                              "double-buffered on the device); CUDA events from before the first upload to after "
                              "the last readback, max over ranks"},
            "gpu_launches": int(float(mx[3])), "clocks": clk, "device_status": status, "parity": parity,
            "configs": configs, "gemv": gemv, "qk_norm_rope": qk, "attention": attn, "vsa_attention": vsa,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def parity_vs_oracle(fh3, torch, trunk, h0, h, text_bf, n_rows: int) -> dict:
    """Sampled output rows of the bench's own step against the CPU oracle composed in fp32
    through every block (fh3_rmsnorm, fh3_modulate, fh3_matmul, fh3_swiglu, fh3_gate_residual
    restated: src/core/fh3_ops.c:317-585).  Rows are independent in every projection."""
    import numpy as np

    from oracle.oracle import Oracle, rel_fro
    o = Oracle()
    t0 = time.time()
    M, d = h0.shape
    F = trunk.F
    rows = np.unique(np.concatenate([[0, M - 1], np.random.default_rng(7).choice(M, max(0, n_rows - 2),
                                                                              replace=False)]))
    n = len(rows)
    ri = torch.from_numpy(rows).to(h0.device)
    hs = h0.index_select(0, ri).cpu().numpy()
    start = hs.copy()
    ones = np.ones(d, np.float32)

    def norm_mod(x, shift, scale):
        return o.modulate(o.rmsnorm(x, ones, 1e-6), np.tile(shift, (n, 1)), np.tile(scale, (n, 1)))

    for blk in trunk.blocks:
        raw = {k: w.data.cpu().numpy() for k, w in blk.w.items()}
        v = [t.cpu().numpy() for t in (blk.shift1, blk.scale1, blk.gate1, blk.shift_c, blk.scale_c, blk.gate_c,
                                       blk.shift2, blk.scale2, blk.gate2)]

        def mm(name, x, out, inn):
            return o.matmul(12, raw[name], inn, out, x)
        qkv = mm("qkv", norm_mod(hs, v[0], v[1]), 3 * d, d)
        hs = o.gate_residual(hs, np.tile(v[2], (n, 1)), mm("o", qkv[:, 2 * d:], d, d))
        cq = mm("cq", norm_mod(hs, v[3], v[4]), d, d)
        hs = o.gate_residual(hs, np.tile(v[5], (n, 1)), mm("co", cq, d, d))
        g = o.swiglu(mm("fc1", norm_mod(hs, v[6], v[7]), 2 * F, d))
        hs = o.gate_residual(hs, np.tile(v[8], (n, 1)), mm("fc2", g, d, F))
    got = h.index_select(0, ri).cpu().numpy()
    err = rel_fro(got - start, hs - start)
    return {"method": f"{n} sampled rows of the step's output against the CPU oracle composed in fp32 through "
                      f"all {len(trunk.blocks)} blocks (relative Frobenius error of the residual increment)",
            "rows": [int(r) for r in rows], "rel_err": float(f"{err:.3e}"), "tol": 1e-2, "ok": bool(err <= 1e-2),
            "seconds": round(time.time() - t0, 1)}


# ----------------------------------------------------------------------------- GEMV and kernel cases
GEMV_SHAPES = ((5120, 13824), (13824, 5120), (5120, 5120))   # (in, out): fc-up, fc-down, attention proj


def gemv_kernel_name(K: int, N: int, M: int) -> str:
    """The kernel the default GEMV dispatch (csrc/gemv_mma.cu, gemv_mma) picks."""
    if M == 1 and (K // 256) * 2180 <= 227 * 1024:
        return "gemv_i8_kernel"
    if 2 <= M <= 4 and (M == 2 or N > K) and (K // 256) * (768 * M + 128 + 4 * M) <= 227 * 1024:
        return "gemv_i8m_kernel"
    if N <= K or M >= 5:
        return "gemv_tc_kernel (i8 A)" if M <= 5 else "gemv_tc_kernel (f16 A = sc*q) + gemv_xprep_kernel"
    if M <= 2:
        return "gemv_stream_kernel"
    return "gemv_mma_small_kernel" if M <= 4 else "gemv_mma_kernel"


def cpu_gemv_us(K: int, N: int, M: int, reps: int = 5) -> tuple[float, str]:
    """Best-of-reps time of the reference's fh3_matmul (oracle/_ref; the oracle port if it is
    absent) on one M-token GEMV, as benchmarks/bench_matmul.c:76-94 times it."""
    import numpy as np

    from oracle import oracle as orc
    o = orc.Oracle()
    impl, kind = (orc.Reference(), "reference") if orc.Reference.available() else (o, "port")
    raw = o.make_weights(seed=100, stream=9, rows=N, n=K)
    x = np.random.default_rng(M).standard_normal((M, K), dtype=np.float32)
    best = None
    for i in range(reps + 1):
        t0 = time.perf_counter()
        impl.matmul(12, raw, K, N, x)
        dt = time.perf_counter() - t0
        if i > 0:
            best = dt if best is None else min(best, dt)
    return best * 1e6, kind


def measure_gemv(fh3, torch, hbm_gbs: float, peak_src: str, reps: int = 100, cpu_threads=None) -> dict:
    """Device time of back-to-back GEMV calls (1, 4 and 16 tokens) on
    weights larger than L2, with the reference's CPU fh3_matmul timed beside each shape when
    cpu_threads is given (rank 0 at N = 1).

    A sleep kernel holds the stream while the host queues `reps` calls, so the CUDA events
    bracket GPU time only (each call's launches, chained by programmatic dependent launch).
    GB/s counts the algorithmic bytes of one call: Q4_K weights + x + y.  Each entry also
    carries the second fraction the hot-path contract asks for at M = 4 and 16, where a GEMV
    has 3.6 M flop per byte: 2 M K N flop per call against the fp32 CUDA-core FMA rate (the
    rate an fp32 dequantise-and-FMA GEMV is bound by; the kernels here use exact-operand
    tensor-core MMAs instead, so it is a comparison, not their own ceiling)."""
    import math
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    sm_mhz = float(load_peaks()[0].get("sm_max_mhz") or 1965.0)
    fp32_tflops = sms * 128 * 2 * sm_mhz * 1e6 / 1e12
    out = {"unit": "GB/s", "peak": hbm_gbs, "peak_source": f"{peak_src} hbm_gbs", "reps": reps,
           "fp32_core_peak_tflops": round(fp32_tflops, 1),
           "fp32_core_peak_source": f"nominal: {sms} SMs x 128 fp32 lanes x 2 flop x {sm_mhz:.0f} MHz max SM clock",
           "method": "sleep-held stream, CUDA events around back-to-back calls, weights rotated > L2",
           "cpu_threads": cpu_threads,
           "cpu_method": "fh3_matmul on the host, best of 5 calls after one warm-up (bench_matmul.c:76-94)",
           "shapes": []}
    for K, N in GEMV_SHAPES:
        wbytes = N * K // 256 * 144
        nw = max(4, math.ceil(300e6 / wbytes))
        ws = [fh3.make_weights(N, K, seed=100 + i, stream_id=9) for i in range(nw)]
        for M in (1, 4, 16):
            x = torch.randn((M, K), device="cuda")
            y = torch.empty((M, N), device="cuda")
            for i in range(2 * nw):
                fh3.gemv(ws[i % nw], x, out=y)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda._sleep(40_000_000)
            e0.record()
            for i in range(reps):
                fh3.gemv(ws[i % nw], x, out=y)
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1000.0 / reps
            gbs = (wbytes + 4 * M * (K + N)) / us / 1e3
            tflops = 2.0 * M * K * N / us / 1e6
            entry = {"in": K, "out": N, "tokens": M, "kernel": gemv_kernel_name(K, N, M),
                     "us_per_call": round(us, 2), "achieved": round(gbs, 1), "frac": round(gbs / hbm_gbs, 4),
                     "tflops": round(tflops, 2), "fp32_core_frac": round(tflops / fp32_tflops, 4)}
            if cpu_threads:
                cus, kind = cpu_gemv_us(K, N, M)
                entry.update({"cpu_us": round(cus, 1), "cpu_kind": kind})
            out["shapes"].append(entry)
        del ws
        torch.cuda.synchronize()
    return out


def measure_configs(fh3, torch, trunk, text_bf, peak: float, peak_src: str, cpu_threads) -> dict:
    """BASELINE configs 1, 3 and 4 on one GPU, each through the path the library takes for it,
    with weights rotated across the trunk's blocks (more than L2 between repeats):
      1: fh3_matmul drop-in semantics on device buffers (fh3cuda_matmul_dev), W 5120x5120 Q4_K,
         x [256][5120] fp32 -> y fp32 (13.42 GFLOP);
      3: the SwiGLU FFN at M = 4096: x -> bf16, fc1 with the SwiGLU epilogue, fc2 (1.739 TFLOP);
      4: one block's projection set at M = 16384 latent rows + 512 text rows for cross K/V, through
         the trunk runner (prologues, epilogues, overlapped expansion; 12.06 TFLOP).
    The reference's fh3_matmul is timed beside config 1 in full and beside configs 3 and 4 on a row
    sample (rows are independent; the FLOPs scale with the rows), when cpu_threads is given."""
    from fasth3inc_b200.trunk import D_MODEL, FFN, Runner, Workspace, block_flops
    out = {"unit": "TFLOP/s", "peak": peak, "peak_source": f"{peak_src} bf16_tflops", "cpu_threads": cpu_threads}
    blocks = trunk.blocks
    nb = len(blocks)

    def timed(fn, reps):
        fn(0)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(reps):
            fn(i + 1)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    def cpu_rate(pairs):
        """GFLOP/s of the reference's fh3_matmul over [(raw, in, out, x)]"""
        import numpy as np
        from oracle import oracle as orc
        impl = orc.Reference() if orc.Reference.available() else orc.Oracle()
        flops, t0 = 0, time.perf_counter()
        for raw, inn, o, x in pairs:
            impl.matmul(12, raw, inn, o, x)
            flops += 2 * x.shape[0] * inn * o
        return flops / (time.perf_counter() - t0) / 1e9, ("reference" if orc.Reference.available() else "port")

    # config 1
    x1 = torch.randn((256, D_MODEL), device="cuda")
    y1 = torch.empty((256, D_MODEL), device="cuda")
    ms = timed(lambda i: fh3.matmul(blocks[i % nb].w["o"], x1, out=y1), 20)
    f1 = 2 * 256 * D_MODEL * D_MODEL
    c1 = {"workload": "W 5120x5120 Q4_K, x [256][5120] fp32, y = x W^T (fh3cuda_matmul_dev)", "ms": round(ms, 4),
          "achieved": round(f1 / ms / 1e9, 1), "frac": round(f1 / ms / 1e9 / peak, 4)}
    # config 3
    M3 = 4096
    x3 = torch.randn((M3, D_MODEL), device="cuda")
    xb = torch.empty((M3, D_MODEL), dtype=torch.bfloat16, device="cuda")
    g3 = torch.empty((M3, FFN), dtype=torch.bfloat16, device="cuda")
    y3 = torch.empty((M3, D_MODEL), device="cuda")

    # FFNs back to back on the blocks' weights through the trunk runner, as config 4 and the
    # trunk run their projections: each FFN converts x, then fc1 (SwiGLU epilogue) and fc2,
    # every projection's Q4_K -> bf16 expansion on the side stream one projection ahead
    runner3 = Runner(trunk, Workspace(1, 1))

    def ffn_ops(b):
        return [("call", lambda st: fh3.to_bf16(x3, out=xb, stream=st)),
                ("gemm", b.w["fc1"], xb.data_ptr(), D_MODEL, M3, g3.data_ptr(), FFN, fh3.EPI_SWIGLU, None, None),
                ("gemm", b.w["fc2"], g3.data_ptr(), FFN, M3, y3.data_ptr(), D_MODEL, fh3.EPI_F32, None, None)]

    reps3 = 5
    runner3.run(ffn_ops(blocks[0]))
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    runner3.run([op for i in range(reps3) for op in ffn_ops(blocks[(i + 1) % nb])])
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps3
    f3 = 3 * 2 * M3 * D_MODEL * FFN
    c3 = {"workload": "SwiGLU FFN, x [4096][5120] fp32: to bf16, fc1 [up; gate] 27648x5120 with the SwiGLU "
                      "epilogue, fc2 5120x13824; five FFNs on five blocks' weights back to back through the trunk "
                      "runner (each expansion on the side stream one projection ahead; the first one exposed)",
          "ms": round(ms, 3), "achieved": round(f3 / ms / 1e9, 1), "frac": round(f3 / ms / 1e9 / peak, 4)}
    del xb, g3, y3, runner3
    # config 4
    M4, T4 = 16384, text_bf.shape[0]
    ws = Workspace(M4, T4)
    h4 = torch.randn((M4, D_MODEL), device="cuda")
    runner = Runner(trunk, ws)
    ms = timed(lambda i: runner.block(blocks[i % nb], h4, text_bf), 5)
    f4 = block_flops(M4, T4)
    c4 = {"workload": "one block's projection set: QKV/O self-attention and Q/O cross-attention on 16384 latent "
                      "rows, cross K/V on 512 text rows, SwiGLU FFN 13824, AdaLN rmsnorm+modulate prologues",
          "ms": round(ms, 3), "achieved": round(f4 / ms / 1e9, 1), "frac": round(f4 / ms / 1e9 / peak, 4)}
    del ws, h4
    torch.cuda.synchronize()
    if cpu_threads:
        import numpy as np
        rng = np.random.default_rng(3)
        b0 = {k: w.data.cpu().numpy() for k, w in blocks[0].w.items()}
        r, kind = cpu_rate([(b0["o"], D_MODEL, D_MODEL, rng.standard_normal((256, D_MODEL), dtype=np.float32))])
        c1.update({"cpu_ms": round(2 * 256 * D_MODEL * D_MODEL / r / 1e6, 2), "cpu_kind": kind,
                   "cpu_sample": "the full config"})
        s3 = 256
        xs = rng.standard_normal((s3, D_MODEL), dtype=np.float32)
        gs = rng.standard_normal((s3, FFN), dtype=np.float32)
        r, kind = cpu_rate([(b0["fc1"], D_MODEL, 2 * FFN, xs), (b0["fc2"], FFN, D_MODEL, gs)])
        c3.update({"cpu_ms": round(f3 / r / 1e6, 1), "cpu_kind": kind,
                   "cpu_sample": f"fc1 and fc2 on {s3} rows, scaled to 4096 rows"})
        c4.update({"cpu_ms": round(f4 / r / 1e6, 1), "cpu_kind": kind,
                   "cpu_sample": f"the config-3 sample's rate ({s3} rows of fc1 and fc2), scaled to the config's FLOPs"})
    out.update({"config1_gemm_m256": c1, "config3_swiglu_ffn_m4096": c3, "config4_block_m16384": c4})
    return out


def measure_qk_norm_rope(fh3, torch, rows: int, hbm_gbs: float, peak_src: str, reps: int = 20) -> dict:
    """Device time of the fused q/k rmsnorm + rope3 on the q third of a bf16 QKV output of
    `rows` tokens (40 heads x 128, rot 96), bf16 out; algorithmic bytes = q read + q written
    + the cos/sin rows + the norm weights.  The inputs exceed L2."""
    H, D, R = 40, 128, 96
    inner = H * D
    qkv = torch.randn((rows, 3 * inner), device="cuda").to(torch.bfloat16)
    out = torch.empty((rows, inner), dtype=torch.bfloat16, device="cuda")
    w = torch.ones(D, device="cuda")
    ang = torch.rand((rows, R), device="cuda")
    cs, sn = torch.cos(ang), torch.sin(ang)
    for _ in range(3):
        fh3.qk_norm_rope(qkv[:, :inner], w, cs, sn, H, D, R, 1e-6, out=out)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for r in range(reps):
        src = qkv[:, (r % 2) * inner:(r % 2 + 1) * inner]       # q and k alternate
        fh3.qk_norm_rope(src, w, cs, sn, H, D, R, 1e-6, out=out)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / reps
    nbytes = rows * inner * 2 * 2 + rows * R * 4 * 2 + D * 4
    gbs = nbytes / us / 1e3
    del qkv, out
    return {"kernel": "qk_norm_rope_kernel", "rows": rows, "heads": H, "head_dim": D, "rot_dim": R,
            "dtype": "bf16 in, bf16 out", "us_per_launch": round(us, 2), "bound": "hbm", "achieved": round(gbs, 1),
            "unit": "GB/s", "peak": hbm_gbs, "frac": round(gbs / hbm_gbs, 4), "peak_source": f"{peak_src} hbm_gbs",
            "bytes_per_launch": nbytes}


def measure_attention(fh3, torch, rows: int, peak: float, peak_src: str, reps: int = 3) -> dict:
    """Device time of one dense attention over `rows` tokens (40 heads x 128, bf16 q/k/v as
    the thirds of a QKV output, bf16 o); FLOPs = 4 * rows^2 * 40 * 128 (QK^T and PV)."""
    H, D = 40, 128
    inner = H * D
    qkv = torch.randn((rows, 3 * inner), device="cuda").to(torch.bfloat16)
    o = torch.empty((rows, inner), dtype=torch.bfloat16, device="cuda")
    q, k, v = qkv[:, :inner], qkv[:, inner:2 * inner], qkv[:, 2 * inner:]
    fh3.attention(q, k, v, H, out=o)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fh3.attention(q, k, v, H, out=o)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    flops = 4.0 * rows * rows * H * D
    tf = flops / (ms * 1e-3) / 1e12
    del qkv, o
    return {"kernel": "attention_pp_kernel (+ vt_transpose_kernel)", "rows": rows, "heads": H, "head_dim": D,
            "ms_per_launch": round(ms, 3),
            "bound": "tensor", "achieved": round(tf, 1), "unit": "TFLOP/s", "peak": peak, "frac": round(tf / peak, 4),
            "peak_source": f"{peak_src} bf16_tflops", "flop_per_launch": flops,
            "note": "tcgen05, score and output tiles in TMEM; not part of the GEMM-only step"}


def vsa_seq(rows: int):
    """A DiT sequence of `rows` tokens for video sparse attention: 1024 audio tokens then a
    video grid of 30 x 52 latent patches per frame (21 frames, 33,784 rows)."""
    audio = 1024
    frames = max(1, (rows - audio) // (30 * 52))
    v = frames * 30 * 52
    return (audio + v, 0, audio, v, frames, 30, 52)


def measure_vsa(fh3, torch, rows: int, peak: float, peak_src: str, reps: int = 3) -> dict:
    """Device time of one video sparse attention call (fh3_vsa_attention, tile 64, sparsity 0.8,
    with the coarse gate) over a `rows`-token sequence, 40 heads x 128, bf16 q/k/v/gate/o.
    FLOPs = 4 * 128 * sum over heads and query tiles of (query rows x kept keys): the fine
    pass's QK^T and PV over the keys the tile mask keeps (the tile stage is a few GFLOP)."""
    H, D = 40, 128
    inner = H * D
    seq = vsa_seq(rows)
    n = seq[0]
    qkv = torch.randn((n, 3 * inner), device="cuda").to(torch.bfloat16)
    gate = torch.randn((n, inner), device="cuda").to(torch.bfloat16)
    o = torch.empty((n, inner), dtype=torch.bfloat16, device="cuda")
    q, k, v = qkv[:, :inner], qkv[:, inner:2 * inner], qkv[:, 2 * inner:]
    _, mask = fh3.vsa_tiles(q, k, seq, H, D, 64, 0.8)
    nt, npre, nvid = fh3.vsa_num_tiles(seq)
    # tokens per tile from the geometry (prefix runs of 64, then 4x4x4 cells of the grid)
    cnt = [min(64, seq[2] - 64 * a) for a in range(npre)]
    ct, ch, cw = (seq[4] + 3) // 4, (seq[5] + 3) // 4, (seq[6] + 3) // 4
    for c in range(nvid):
        tt, hh, ww = c // (ch * cw), (c // cw) % ch, c % cw
        cnt.append(min(4, seq[4] - 4 * tt) * min(4, seq[5] - 4 * hh) * min(4, seq[6] - 4 * ww))
    cnt_t = torch.tensor(cnt, dtype=torch.float64, device="cuda")
    keys = (mask.double() * cnt_t).sum(dim=2)                 # [H][nt] kept keys per query tile
    flops = float(4.0 * D * (keys * cnt_t).sum().item())
    del mask
    fh3.vsa_attention(q, k, v, gate, seq, H, D, out=o)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fh3.vsa_attention(q, k, v, gate, seq, H, D, out=o)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    tf = flops / (ms * 1e-3) / 1e12
    del qkv, gate, o
    return {"kernel": "vsa_tc64_kernel (+ tile stage, tile-order copies and coarse pass in the timed call)", "rows": n,
            "seq": {"audio": seq[2], "video": seq[3], "grid": list(seq[4:])}, "tiles": nt, "heads": H,
            "head_dim": D, "sparsity": 0.8, "ms_per_call": round(ms, 3), "bound": "tensor",
            "achieved": round(tf, 1), "unit": "TFLOP/s", "peak": peak, "frac": round(tf / peak, 4),
            "peak_source": f"{peak_src} bf16_tflops", "flop_per_call": flops,
            "dense_equivalent_ms": round(4.0 * n * n * H * D / (tf * 1e12) * 1e3, 3),
            "note": "tcgen05 fine pass, TMEM score and output tiles; not part of the GEMM-only step"}


def run_case(args):
    """One kernel's launches on a small case, for ncu (prints a one-line JSON summary)."""
    import torch
    import fasth3inc_b200 as fh3
    from fasth3inc_b200.trunk import D_MODEL, FFN
    fh3.init(0)
    if args.case == "gemm":
        w = fh3.make_weights(2 * FFN, D_MODEL, seed=1, stream_id=1)     # fc1: [up; gate]
        x = fh3.to_bf16(torch.randn((args.case_rows, D_MODEL), device="cuda"))
        y = torch.empty((args.case_rows, FFN), dtype=torch.bfloat16, device="cuda")
        for _ in range(args.case_reps):
            fh3.gemm(w, x, fh3.EPI_SWIGLU, out=y)
        shape = {"rows": args.case_rows, "in": D_MODEL, "out": 2 * FFN, "epilogue": "swiglu"}
    elif args.case == "matmul":
        # BASELINE config 1's drop-in call: fh3cuda_matmul_dev on fp32 rows, W 5120 x 5120 Q4_K
        ws = [fh3.make_weights(D_MODEL, D_MODEL, seed=i, stream_id=3) for i in range(args.case_reps)]
        x = torch.randn((args.case_rows, D_MODEL), device="cuda")
        y = torch.empty((args.case_rows, D_MODEL), device="cuda")
        for w in ws:
            fh3.matmul(w, x, out=y)
        shape = {"rows": args.case_rows, "in": D_MODEL, "out": D_MODEL}
    elif args.case == "attn":
        H, Dh = 40, 128
        qkv = torch.randn((args.case_rows, 3 * H * Dh), device="cuda").to(torch.bfloat16)
        out = torch.empty((args.case_rows, H * Dh), dtype=torch.bfloat16, device="cuda")
        for _ in range(args.case_reps):
            fh3.attention(qkv[:, :H * Dh], qkv[:, H * Dh:2 * H * Dh], qkv[:, 2 * H * Dh:], H, out=out)
        shape = {"rows": args.case_rows, "heads": H, "head_dim": Dh}
    elif args.case == "vsa":
        H, Dh = 40, 128
        seq = vsa_seq(args.case_rows)
        n = seq[0]
        qkv = torch.randn((n, 3 * H * Dh), device="cuda").to(torch.bfloat16)
        gate = torch.randn((n, H * Dh), device="cuda").to(torch.bfloat16)
        out = torch.empty((n, H * Dh), dtype=torch.bfloat16, device="cuda")
        for _ in range(args.case_reps):
            fh3.vsa_attention(qkv[:, :H * Dh], qkv[:, H * Dh:2 * H * Dh], qkv[:, 2 * H * Dh:], gate, seq, H, Dh,
                              out=out)
        shape = {"rows": n, "heads": H, "head_dim": Dh, "grid": list(seq[4:])}
    elif args.case == "norm":
        M = args.case_rows
        h = torch.randn((M, D_MODEL), device="cuda")
        sh, sc = 0.1 * torch.randn(D_MODEL, device="cuda"), 0.1 * torch.randn(D_MODEL, device="cuda")
        a = torch.empty((M, D_MODEL), dtype=torch.bfloat16, device="cuda")
        for _ in range(args.case_reps):
            fh3.rmsnorm_modulate(h, sh, sc, out=a)
        shape = {"rows": M, "dim": D_MODEL}
    elif args.case == "qk":
        H, Dh, R = 40, 128, 96
        qkv = torch.randn((args.case_rows, 3 * H * Dh), device="cuda").to(torch.bfloat16)
        out = torch.empty((args.case_rows, H * Dh), dtype=torch.bfloat16, device="cuda")
        ang = torch.rand((args.case_rows, R), device="cuda")
        for r in range(args.case_reps):
            fh3.qk_norm_rope(qkv[:, (r % 2) * H * Dh:(r % 2 + 1) * H * Dh], torch.ones(Dh, device="cuda"),
                             torch.cos(ang), torch.sin(ang), H, Dh, R, 1e-6, out=out)
        shape = {"rows": args.case_rows, "heads": H, "head_dim": Dh, "rot_dim": R}
    else:
        K, N = args.case_kn
        ws = [fh3.make_weights(N, K, seed=i, stream_id=3) for i in range(args.case_reps)]
        x = torch.randn((args.case_m, K), device="cuda")
        y = torch.empty((args.case_m, N), device="cuda")
        for w in ws:
            fh3.gemv(w, x, out=y)
        shape = {"in": K, "out": N, "tokens": args.case_m}
    torch.cuda.synchronize()
    print(json.dumps({"case": args.case, **shape, "reps": args.case_reps, "status": fh3.device_status()}))


# ----------------------------------------------------------------------------- reference arm
def run_reference(args):
    """The reference's own CPU fh3_matmul (oracle/_ref, else the oracle port) on a bounded sample."""
    import numpy as np

    from fasth3inc_b200.trunk import D_MODEL, FFN, block_flops, block_shapes
    from oracle import oracle as orc
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    hc = host_cpu()
    threads = pin_cpu_threads(hc["physical_cores"])
    o = orc.Oracle()
    raw = {}
    for i, (name, out, inn) in enumerate(block_shapes()):
        raw[name] = o.make_weights(seed=0, stream=i + 1, rows=out, n=inn)
    use_ref = orc.Reference.available()
    rows_s = size_cpu_sample(raw, threads, use_ref, 5.0)
    T = min(rows_s, args.text_rows)
    for _ in range(args.warmup):
        cpu_sample(raw, 16, 16, threads, use_ref)
    times = []
    kind = "reference" if use_ref else "port"
    f = 0
    for _ in range(args.steps):
        f, dt, kind = cpu_sample(raw, rows_s, T, threads, use_ref)
        times.append(dt)
    dt = sum(times) / len(times)
    value = f / dt / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 5), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded N(0,0.02) weights quantised to Q4_K on the host, N(0,1) fp32 rows",
        "config": {"workload": "BASELINE config 5: 50-block synthetic DiT trunk step (bounded sample: one block's "
                               "7 projections)", "blocks": args.blocks, "rows": args.rows,
                   "text_rows": args.text_rows, "sample_rows": rows_s, "sample_text_rows": T,
                   "full_step_gflop": round(args.blocks * block_flops(args.rows, args.text_rows) / 1e9, 1)},
        "cpu_baseline": {"value": round(value, 5), "unit": UNIT, "cores": threads, "kind": kind, "cpu": hc,
                         "sample": f"fh3_matmul (OpenMP, {threads} threads) over block 0's 7 Q4_K projections on "
                                   f"{rows_s} latent + {T} text rows, {f / 1e9:.1f} GFLOP per step"},
        "e2e": {"value": round(value, 5), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.case:
        run_case(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
