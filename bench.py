#!/usr/bin/env python
"""Benchmark of the B200 attention hot path (one JSON line on rank 0).

Workload (every N): configuration 4 -- head-parallel long-context attention,
B=16, T=6144, H=16, D=128, Q/K/V fp32 N(0,1) (seeded synthetic data), causal,
scale 1/sqrt(128), followed by the O projection (Wo 2048x2048, N(0, 0.02)).
With N GPUs rank r owns heads [r*16/N, (r+1)*16/N); per-head outputs are
exchanged token-sliced (by the attention kernel's own NVLink stores, or an NCCL
all-to-all with --exchange nccl) and each rank projects B*T/N tokens.
Total work is fixed, so scaling is "strong".

A step = cast K/V to bf16 (one launch) -> flash attention (reads the fp32 Q rows
and rounds them itself) -> exchange -> O projection.
value      = (attention FLOPs 2*B*H*T^2*D + O-proj FLOPs 2*B*T*d^2) / step time,
             device-resident inputs, CUDA events on the launching stream, max over ranks.
e2e        = the same through host buffers: pinned Q/K/V slices copied in and the
             y slice copied out inside the timed region, batch chunks pipelined
             over a copy-in, a compute and a copy-out stream.
roofline   = the flash kernel (CUDA events around each launch in the timed region)
             against the measured dense bf16 peak.
cpu_baseline / --impl reference = the reference's own flash_attention_forward
             (FlashAttention.cpp, compiled from the reference sources into
             oracle/_ref) plus the O projection through OpenBLAS sgemm, on a bounded
             sample of the same workload (whole batch elements), all host threads.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B, T, H, D, DM = 16, 6144, 16, 128, 2048
SCALE = 1.0 / np.sqrt(128.0)
METRIC = "causal attn TFLOP/s + OLMo-2-1B prefill tok/s, T=512-6144, 1/2/4/8 B200"
F_ATTN = 2.0 * B * H * T * T * D          # causal: 4*B*H*T^2*D / 2
F_OPROJ = 2.0 * B * T * DM * DM
PEAKS_FALLBACK = {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0}


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    except (OSError, ValueError):
        return PEAKS_FALLBACK, "fallback"


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="dt_clocks_", suffix=".csv")
            self.fh = os.fdopen(fd, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", self.gpu_id], stdout=self.fh,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx = float(parts[2])
                    power.append(float(parts[3]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        try:
            os.unlink(self.path)
        except OSError:
            pass
        loaded = [s for s, p in zip(sm, power) if p > 300] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def gpu_id_for(torch, dev) -> str:
    try:
        u = str(torch.cuda.get_device_properties(dev).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            return vis.split(",")[dev]
        return str(dev)


# ---------------------------------------------------------------------------
# CPU: the reference's own flash_attention_forward + OpenBLAS O projection
# ---------------------------------------------------------------------------
def reference_sample(n_batch: int, seed: int = 0):
    """Runs the reference flash on n_batch whole batch elements (all 16 heads,
    T=6144) and their O projection.  Returns (flops, seconds, threads, kind)."""
    import oracle

    ref = oracle.ref_lib()
    kind = "reference"
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((n_batch, T, H, D), dtype=np.float32)
    k = rng.standard_normal((n_batch, T, H, D), dtype=np.float32)
    v = rng.standard_normal((n_batch, T, H, D), dtype=np.float32)
    wo = (0.02 * rng.standard_normal((DM, DM), dtype=np.float32)).astype(np.float32)
    threads = os.cpu_count() or 1
    if ref is not None:
        o, _, _, t_attn = oracle.ref_flash_fwd(q, k, v, SCALE, True, threads=0)
        threads = ref.ref_get_threads()
    else:  # the reference sources were not compiled: time the C restatement instead
        kind = "port"
        oracle.set_threads(0)
        t0 = time.perf_counter()
        o, _, _ = oracle.flash_fwd(q, k, v, SCALE, True)
        t_attn = time.perf_counter() - t0
    oracle.set_threads(0)
    t0 = time.perf_counter()
    oracle.linear(o.reshape(n_batch * T, DM), wo)
    t_proj = time.perf_counter() - t0
    flops = n_batch * (F_ATTN + F_OPROJ) / B
    return flops, t_attn + t_proj, threads, kind


def run_reference(args, rank):
    if rank != 0:
        return
    budget = 150.0  # seconds for the whole --warmup/--steps run
    f1, t1, threads, kind = reference_sample(1, seed=1)  # calibration (counts as a warm-up)
    per_step = budget / max(1, args.warmup + args.steps)
    n_batch = int(max(1, min(B, per_step / max(t1, 1e-3))))
    vals = []
    for i in range(args.warmup + args.steps - 1):
        f, t, threads, kind = reference_sample(n_batch, seed=2 + i)
        if i >= args.warmup - 1:
            vals.append((f, t))
    if not vals:
        vals = [(f1, t1)]
    flops = sum(f for f, _ in vals)
    secs = sum(t for _, t in vals)
    value = flops / secs / 1e12
    sample = f"{n_batch} of {B} batch elements x 16 heads, T={T}, per step"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": len(vals), "warmup": args.warmup, "ms_per_step": 1e3 * secs / len(vals), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config4_head_parallel_attention", "B": B, "T": T, "H": H, "D": D,
                   "sample": sample},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="dirktensor", choices=["dirktensor", "reference"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", default="fused", choices=["fused", "nccl"],
                    help="N>1: fused flash + NVLink stores (default) or an NCCL all-to-all")
    ap.add_argument("--case", default=None, choices=["flash_bf16", "flash_bwd", "layer", "gemm", "prologue", "flash_api", "step4"],
                    help="profiling case for ncu: a few launches of one stage, no timing")
    ap.add_argument("--sweep", action="store_true",
                    help="config-1 sweep (T = 64 ... 6144) and config 4: flash kernel TFLOP/s per shape")
    ap.add_argument("--no-model", action="store_true", help="skip the config-3 full-model measurement")
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--gemm-mnk", default="16384,16384,2048", help="--case gemm: M,N,K")
    ap.add_argument("--seq", type=int, default=4096)
    args = ap.parse_args()
    rank = env_int("RANK", 0)
    world = env_int("WORLD_SIZE", 1)
    local = env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        return run_reference(args, rank)
    if args.case:
        return run_case(args)
    if args.sweep:
        return run_sweep(args)
    if args.warmup < 3:
        args.warmup = 3

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)

    import dirktensor_b200 as dt
    from dirktensor_b200.head_parallel import HeadParallelAttention

    Hl = H // world
    M = B * T
    gen = torch.Generator(device=dev)
    gen.manual_seed(args.seed * 1000 + rank)
    q = torch.randn((B, T, Hl, D), generator=gen, device=dev)
    k = torch.randn((B, T, Hl, D), generator=gen, device=dev)
    v = torch.randn((B, T, Hl, D), generator=gen, device=dev)
    gen.manual_seed(args.seed * 1000 + 999)
    wo = torch.randn((DM, DM), generator=gen, device=dev) * 0.02
    hp = HeadParallelAttention(wo, n_heads=H, head_dim=D, exchange=args.exchange)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident step -------------------------------------------
    for _ in range(args.warmup):
        hp.forward(q, k, v, SCALE, True)
    torch.cuda.synchronize()
    barrier()
    sampler = ClockSampler(gpu_id_for(torch, local)) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    fl_events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                 for _ in range(args.steps)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier()
    e0.record()
    for i in range(args.steps):
        hp.forward(q, k, v, SCALE, True, events=fl_events[i])
    e1.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop() if sampler else None
    dt.check_device_error()
    ms_step = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    ms_flash = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in fl_events))
    flops_step = F_ATTN + F_OPROJ
    value = flops_step / (ms_step * 1e-3) / 1e12

    # ---- end to end through host buffers ----------------------------------
    e2e = bench_e2e(torch, dev, hp, q, k, v, world, max(3, min(args.steps, 10)), barrier, max_over_ranks)
    e2e["value"] = flops_step / (e2e["ms_per_step"] * 1e-3) / 1e12

    # ---- the other exchanges (N > 1) and the head-parallel layer ------------
    # (sub-measurements: a failure is recorded in the line instead of losing it; every rank
    # runs the same steps, so a failure there is normally the same on all ranks)
    variants = None
    if world > 1:
        try:
            variants = bench_exchange_variants(torch, dev, q, k, v, wo, world, args, barrier, max_over_ranks)
        except Exception as e:  # noqa: BLE001
            variants = {"unavailable": f"{type(e).__name__}: {e}"}
    try:
        layers_sharded = bench_layers_sharded(torch, dev, world, args, barrier, max_over_ranks)
    except Exception as e:  # noqa: BLE001
        layers_sharded = {"unavailable": f"{type(e).__name__}: {e}"}

    # ---- config 1 at T=4096 (north-star single-GPU target) ---------------
    t4096 = None
    if world == 1:
        t4096 = bench_t4096(torch, dt, dev, args)

    layers = None
    model3 = model_host = None
    train = None
    prologue = None
    if world == 1:
        layers = bench_layers(torch, dt, dev, args)
        prologue = bench_prologue(torch, dt, dev, args)
        train = bench_train(torch, dt, dev, args)
        if not args.no_model:
            model3, model_host = bench_model(torch, dt, dev, args)

    # ---- CPU baseline (rank 0, N=1) ---------------------------------------
    cpu = None
    cpu_cfg = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        try:
            f1, s1, _, _ = reference_sample(1, seed=7)  # calibration: size the sample to ~10 s
            nb = int(max(1, min(B, 10.0 / max(s1, 1e-3))))
            f, s, threads, kind = reference_sample(nb, seed=8)
            cpu = {"value": f / s / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": kind,
                   "sample": f"{nb} of {B} batch elements (16 heads, T={T}) attention + their O projection",
                   "seconds": s}
        except Exception as e:  # the oracle is optional at run time
            cpu = {"value": None, "unit": "TFLOP/s", "cores": None, "kind": "reference",
                   "sample": f"unavailable: {e}"}
        try:
            cpu_cfg = cpu_baselines(model_host)
        except Exception as e:  # the oracle is optional at run time
            cpu_cfg = {"unavailable": str(e)}
        model_host = None
        if model3 is not None and "config3" in cpu_cfg:
            c3 = cpu_cfg["config3"]
            model3.update({"parity_rel_l2": c3["parity_rel_l2"], "parity_max_abs": c3["parity_max_abs"],
                           "parity_top1": c3["top1_agreement"],
                           "parity_sample": "sequence 0 vs the CPU restatement of OlmoModel::forward"})
        for name, sub in (("config0", (layers or {}).get("config0")), ("config2", (layers or {}).get("config2")),
                          ("config1_t4096", t4096), ("config3", model3)):
            if sub is not None and name in cpu_cfg:
                sub["cpu_baseline"] = cpu_cfg[name]

    peaks, src = load_peaks()
    peak = float(peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"]))
    f_flash_rank = F_ATTN / world
    achieved = f_flash_rank / (ms_flash * 1e-3) / 1e12
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "attn_fwd_traffic.json")
    if os.path.exists(tpath):
        try:
            with open(tpath) as f:
                tj = json.load(f)
            traffic = tj.get("bytes_per_launch_config4", {}).get(str(world))
        except (OSError, ValueError):
            traffic = None

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "config4_head_parallel_attention", "B": B, "T": T, "H": H, "D": D,
                       "d_model": DM, "causal": True,
                       "parallelism": f"head-parallel x{world} + token-sliced exchange ({args.exchange}) + O-proj",
                       "flops_per_step": flops_step,
                       "l2": "inputs larger than L2 (805 MB fp32 per tensor in total)"},
            "prefill_tok_s": M / (ms_step * 1e-3),
            "roofline": {"bound": "tensor", "kernel": "attn_fwd_kernel", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak, "peak_source": f"{src} bf16 burst",
                         "ms_per_launch": ms_flash, "flops_per_launch": f_flash_rank, "traffic": traffic},
            "cpu_baseline": cpu,
            "e2e": e2e,
            # one K+V cast launch + attention (which rounds fp32 Q itself) + O projection; the fused
            # exchange adds its one-thread system fence and the flag barrier kernel
            "gpu_launches": (5 if world > 1 and args.exchange == "fused" else 3) * args.steps,
            "clocks": clocks,
            "config1_t4096": t4096,
            "exchange_variants": variants,
            "layers_sharded": layers_sharded,
            "layers": layers,
            "prologue": prologue,
            "model_config3": model3,
            "training": train,
        }
        print(json.dumps(line), flush=True)
    hp.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def bench_exchange_variants(torch, dev, q, k, v, wo, world, args, barrier, max_over_ranks):
    """N > 1: the config-4 step with the other two exchanges -- the NCCL
    all-to-all of token slices, and the replicated form the task statement
    names (all-gather of every rank's per-head outputs, then every rank
    projects all B*T tokens; its O-projection FLOPs are counted once)."""
    from dirktensor_b200.head_parallel import HeadParallelAttention

    out = {}
    for mode in ("nccl", "allgather"):
        hp = HeadParallelAttention(wo, n_heads=H, head_dim=D, exchange=mode)
        for _ in range(args.warmup):
            hp.forward(q, k, v, SCALE, True)
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            hp.forward(q, k, v, SCALE, True)
        e1.record()
        torch.cuda.synchronize()
        barrier()
        ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
        hp.close()
        out[mode] = {"ms_per_step": ms, "tflops": (F_ATTN + F_OPROJ) / (ms * 1e-3) / 1e12,
                     "received_bytes_per_rank": (world - 1) * B * T * (H // world) * D * 2 // (
                         1 if mode == "allgather" else world)}
    return out


def bench_layers_sharded(torch, dev, world, args, barrier, max_over_ranks):
    """The attention layer (OlmoAttention::forward) head-parallel over the N
    GPUs through the C ABI (dt_attn_create_sharded / dt_attn_forward_sharded on
    the library's own NCCL communicator; in-kernel exchange): config 0 (B=1,
    T=512) and config 2 (B=8, T_max=2048, right-padded, seeded lengths in
    [256, 2048]).  Every rank holds the full input and returns its token slice.
    tok/s counts valid tokens; L2 flushed before every timed forward."""
    from dirktensor_b200.head_parallel import Communicator, ShardedOlmoAttention

    rng = np.random.default_rng(0)
    w = [(0.02 * rng.standard_normal((DM, DM), dtype=np.float32)) for _ in range(4)]
    gains = [(1 + 0.02 * rng.standard_normal(DM, dtype=np.float32)).astype(np.float32) for _ in range(2)]
    comm = Communicator.from_process_group(timeout_ms=120000)
    layer = ShardedOlmoAttention(*w, *gains, comm=comm, exchange="fused")
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    out = {}
    for name, Bl, Tl, lens in [("config0", 1, 512, None),
                               ("config2", 8, 2048, np.random.default_rng(2).integers(256, 2049, 8))]:
        x = torch.from_numpy(rng.standard_normal((Bl, Tl, DM), dtype=np.float32)).to(dev)
        y = torch.empty((Bl * Tl // world, DM), dtype=torch.float32, device=dev)
        lens_t = None if lens is None else torch.as_tensor(lens, dtype=torch.int32, device=dev)
        valid = Bl * Tl if lens is None else int(np.sum(lens))
        seqs = [Tl] * Bl if lens is None else [int(v) for v in lens]
        flops = 2.0 * valid * DM * 8192 + sum(2.0 * H * L * L * D for L in seqs)
        reps = max(3, min(args.steps, 20))
        ts = []
        for i in range(args.warmup + reps):
            flush.fill_(float(i))
            torch.cuda.synchronize()
            barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            layer.forward(x, seq_lens=lens_t, out=y)
            b.record()
            torch.cuda.synchronize()
            if i >= args.warmup:
                ts.append(a.elapsed_time(b))
        ms = max_over_ranks(statistics.median(ts))
        out[name] = {"B": Bl, "T": Tl, "valid_tokens": valid, "ms": ms, "tok_s": valid / (ms * 1e-3),
                     "tflops": flops / (ms * 1e-3) / 1e12, "gpus": world}
    torch.cuda.synchronize()
    barrier()
    layer.close()
    comm.close()
    return out


def bench_e2e(torch, dev, hp, q, k, v, world, steps, barrier, max_over_ranks, chunks=8):
    """The config-4 step end to end through HeadParallelAttention.forward with
    pinned host buffers: every step copies this rank's Q, K, V in and its y
    slice out.  The batch is split into `chunks` groups of batch elements
    (attention never mixes batch elements, so the split is exact), and three
    streams overlap them: chunk c+1's host->device copies and chunk c-1's
    device->host copy run under chunk c's attention and projection.  Every
    chunk has its own device input and output slices; a step's copy into a
    slice waits for the previous step's reader of that slice (events).  The
    events bracket all three streams' work."""
    Bq, Tq, Hl, Dq = q.shape
    if Bq % chunks:
        chunks = 1
    bc = Bq // chunks
    mc = bc * Tq // world  # this rank's tokens of one chunk
    qh, kh, vh = (t.cpu().pin_memory() for t in (q, k, v))
    yh = torch.empty((chunks * mc, DM), dtype=torch.float32).pin_memory()
    qd, kd, vd = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    yd = torch.empty((chunks, mc, DM), dtype=torch.float32, device=dev)
    comp = torch.cuda.current_stream(dev)
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(chunks)]
    ev_out = [torch.cuda.Event() for _ in range(chunks)]
    ev_done = [torch.cuda.Event() for _ in range(chunks)]

    def step():
        for c in range(chunks):
            sl = slice(c * bc, (c + 1) * bc)
            with torch.cuda.stream(h2d):
                h2d.wait_event(ev_out[c])  # the previous step's attention has read these slices
                qd[sl].copy_(qh[sl], non_blocking=True)
                kd[sl].copy_(kh[sl], non_blocking=True)
                vd[sl].copy_(vh[sl], non_blocking=True)
                ev_in[c].record(h2d)
            comp.wait_event(ev_in[c])
            comp.wait_event(ev_done[c])  # the previous step's copy-out of yd[c] is done
            hp.forward(qd[sl], kd[sl], vd[sl], SCALE, True, out=yd[c])
            ev_out[c].record(comp)
            with torch.cuda.stream(d2h):
                d2h.wait_event(ev_out[c])
                yh[c * mc:(c + 1) * mc].copy_(yd[c], non_blocking=True)
                ev_done[c].record(d2h)

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    h2d.wait_event(e0)
    d2h.wait_event(e0)
    for _ in range(steps):
        step()
    comp.wait_event(ev_done[chunks - 1])  # the copy-out stream is in order: its last copy ends the step
    e1.record(comp)
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps)
    h2d_bytes = 3 * q.numel() * 4 * world
    d2h_bytes = yh.numel() * 4 * world
    return {"unit": "TFLOP/s", "ms_per_step": ms, "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": d2h_bytes,
            "pcie_gbs_h2d_per_gpu": 3 * q.numel() * 4 / (ms * 1e-3) / 1e9, "chunks": chunks,
            "api": "HeadParallelAttention.forward over the C ABI, pinned host buffers; "
                   f"{chunks} batch chunks, host->device, compute and device->host on three streams"}


def bench_layers(torch, dt, dev, args):
    """One OLMo-2-1B attention layer (OlmoAttention::forward) on the device:
    config 0 (B=1, T=512) and config 2 (B=8, T_max=2048, right-padded, seeded
    lengths in [256, 2048]).  tok/s counts valid tokens; FLOPs = projections
    2*tokens*2048*8192 + causal attention 2*H*len^2*D per sequence.  L2 is
    flushed before every timed forward."""
    rng = np.random.default_rng(0)
    w = [(0.02 * rng.standard_normal((DM, DM), dtype=np.float32)) for _ in range(4)]
    gains = [(1 + 0.02 * rng.standard_normal(DM, dtype=np.float32)).astype(np.float32) for _ in range(2)]
    attn = dt.OlmoAttention.from_weights(*w, *gains, device=dev.index or 0)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    out = {}
    for name, Bl, Tl, lens in [("config0", 1, 512, None),
                               ("config2", 8, 2048, np.random.default_rng(2).integers(256, 2049, 8))]:
        x = torch.from_numpy(rng.standard_normal((Bl, Tl, DM), dtype=np.float32)).to(dev)
        y = torch.empty_like(x)
        lens_t = None if lens is None else torch.as_tensor(lens, dtype=torch.int32, device=dev)
        valid = Bl * Tl if lens is None else int(np.sum(lens))
        seqs = [Tl] * Bl if lens is None else [int(v) for v in lens]
        flops = 2.0 * valid * DM * 8192 + sum(2.0 * H * L * L * D for L in seqs)
        reps = max(3, min(args.steps, 20))
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        for i in range(args.warmup + reps):
            flush.fill_(float(i))
            torch.cuda._sleep(2_000_000)
            e = ev[i - args.warmup] if i >= args.warmup else None
            if e:
                e[0].record()
            attn.forward(x, seq_lens=lens_t, out=y)
            if e:
                e[1].record()
        torch.cuda.synchronize()
        ms = statistics.median(a.elapsed_time(b) for a, b in ev)
        out[name] = {"B": Bl, "T": Tl, "valid_tokens": valid, "ms": ms, "tok_s": valid / (ms * 1e-3),
                     "tflops": flops / (ms * 1e-3) / 1e12}
    dt.check_device_error()
    attn.close()
    return out


def bench_model(torch, dt, dev, args):
    """Configuration 3: full 16-layer OLMo-2-0425-1B prefill, B=4, T=4096,
    vocab 100352, random weights N(0, 0.02) (two distinct layer weight sets,
    uploaded into 16 separate layers), token ids seeded uniform in [0, 100278).
    FLOPs: 2 * tokens * (16 * (4 d^2 + 3 d * 8192) + 100352 d) for the
    matmuls plus 16 * 2 * B * H * T^2 * D for causal attention.
    Returns (result, host) -- host keeps the weights, ids and the logits of
    sequence 0 for the CPU leg, which runs the same sequence on the host."""
    Bm, Tm, vocab, hidden, nl = 4, 4096, 100352, 8192, 16
    g = torch.Generator(device=dev)
    g.manual_seed(3)

    def rnd(*shape, scale=0.02):
        return (torch.randn(shape, generator=g, device=dev) * scale).cpu().numpy()

    def gain():
        return (1 + torch.randn((DM,), generator=g, device=dev) * 0.02).cpu().numpy()

    base = []
    for _ in range(2):
        base.append({"q_proj": rnd(DM, DM), "k_proj": rnd(DM, DM), "v_proj": rnd(DM, DM), "o_proj": rnd(DM, DM),
                     "q_norm": gain(), "k_norm": gain(), "post_attention_norm": gain(),
                     "gate_proj": rnd(hidden, DM), "up_proj": rnd(hidden, DM), "down_proj": rnd(DM, hidden),
                     "post_feedforward_norm": gain()})
    layers = [base[i % 2] for i in range(nl)]
    embed, final_norm, lm_head = rnd(vocab, DM), gain(), rnd(vocab, DM)
    model = dt.OlmoModel.from_weights(embed, layers, final_norm, lm_head, device=dev.index or 0)
    ids = torch.randint(0, 100278, (Bm, Tm), generator=g, device=dev, dtype=torch.int32)
    logits = torch.empty((Bm, Tm, vocab), dtype=torch.float32, device=dev)
    for _ in range(2):
        model.forward(ids, out=logits)
    torch.cuda.synchronize()
    reps = 3
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        model.forward(ids, out=logits)
    e1.record()
    torch.cuda.synchronize()
    dt.check_device_error()
    ms = e0.elapsed_time(e1) / reps
    tokens = Bm * Tm
    flops = 2.0 * tokens * (nl * (4 * DM * DM + 3 * DM * hidden) + vocab * DM) + nl * 2.0 * Bm * H * Tm * Tm * D
    finite = bool(torch.isfinite(logits).all().item())
    host = {"embed": embed, "layers": layers, "final_norm": final_norm, "lm_head": lm_head,
            "ids0": ids[0:1].cpu().numpy().astype(np.uint32), "logits0": logits[0].cpu().numpy()}
    model.close()
    del logits
    torch.cuda.empty_cache()
    res = {"B": Bm, "T": Tm, "n_layers": nl, "vocab": vocab, "ms": ms, "tok_s": tokens / (ms * 1e-3),
           "tflops": flops / (ms * 1e-3) / 1e12, "flops": flops, "logits_finite": finite,
           "data": "synthetic ids, random N(0,0.02) weights"}
    return res, host


def _median_time(fn, reps=3):
    fn()  # warm-up
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return statistics.median(ts)


def cpu_baselines(model_host=None):
    """The reference's CPU path beside configs 0-3, on the host cores (rank 0,
    N=1): config 1 at T=4096 through the reference's own flash_attention_forward
    compiled from its sources (kind "reference"); configs 0, 2 and 3 through the
    C restatement of OlmoAttention::forward / OlmoModel::forward with OpenBLAS
    sgemm and the restated FlashAttention.cpp loop (kind "port"; the
    reference's OlmoAttention.cpp needs xtensor, which is not installed).  All
    host threads.  Config 3 runs one of the four sequences (the reference's
    saved activations for the whole batch exceed host RAM); its logits are also
    compared with the GPU's logits of that sequence."""
    import oracle

    oracle.set_threads(0)
    cores = os.cpu_count() or 1
    out = {}
    rng = np.random.default_rng(0)
    w = [(0.02 * rng.standard_normal((DM, DM), dtype=np.float32)) for _ in range(4)]
    gains = [(1 + 0.02 * rng.standard_normal(DM, dtype=np.float32)).astype(np.float32) for _ in range(2)]
    # config 0: one layer, B=1, T=512
    x = rng.standard_normal((1, 512, DM), dtype=np.float32)
    s = _median_time(lambda: oracle.attention_layer(x, *w, *gains))
    f = 2.0 * 512 * DM * 8192 + 2.0 * H * 512 * 512 * D
    out["config0"] = {"ms": s * 1e3, "tok_s": 512 / s, "tflops": f / s / 1e12, "cores": cores, "kind": "port",
                      "sample": "whole workload: B=1, T=512 attention layer"}
    # config 1 at T=4096: the reference's own flash_attention_forward
    qq, kk, vv = (rng.standard_normal((1, 4096, H, D), dtype=np.float32) for _ in range(3))
    ref = oracle.ref_lib()
    if ref is not None:
        s = _median_time(lambda: oracle.ref_flash_fwd(qq, kk, vv, SCALE, True, threads=0))
        kind, thr = "reference", ref.ref_get_threads()
    else:
        s = _median_time(lambda: oracle.flash_fwd(qq, kk, vv, SCALE, True))
        kind, thr = "port", cores
    f = 2.0 * H * 4096 * 4096 * D
    out["config1_t4096"] = {"ms": s * 1e3, "tflops": f / s / 1e12, "cores": thr, "kind": kind,
                            "sample": "whole workload: B=1, H=16, T=4096 causal attention"}
    # config 2: B=8 right-padded layer; each sequence at its own length (valid tokens)
    lens = [int(v) for v in np.random.default_rng(2).integers(256, 2049, 8)]
    xs = [rng.standard_normal((1, L, DM), dtype=np.float32) for L in lens]

    def run2():
        for xb in xs:
            oracle.attention_layer(xb, *w, *gains)

    s = _median_time(run2, reps=1)
    valid = sum(lens)
    f = 2.0 * valid * DM * 8192 + sum(2.0 * H * L * L * D for L in lens)
    out["config2"] = {"ms": s * 1e3, "tok_s": valid / s, "tflops": f / s / 1e12, "cores": cores, "kind": "port",
                      "sample": f"whole workload: 8 sequences of lengths {lens}, valid tokens only"}
    # config 3: one sequence of the full model
    if model_host is not None:
        hst = model_host
        t0 = time.perf_counter()
        ref3 = oracle.model_forward(hst["ids0"], hst["embed"], hst["layers"], hst["final_norm"], hst["lm_head"])[0]
        s = time.perf_counter() - t0
        got = hst["logits0"]
        d = got.astype(np.float64) - ref3
        rel = float(np.sqrt(np.sum(d * d) / np.sum(ref3.astype(np.float64) ** 2)))
        top1 = float(np.mean(got.argmax(-1) == ref3.argmax(-1)))
        f = 2.0 * 4096 * (16 * (4 * DM * DM + 3 * DM * 8192) + 100352 * DM) + 16 * 2.0 * H * 4096 * 4096 * D
        out["config3"] = {"ms": s * 1e3, "tok_s": 4096 / s, "tflops": f / s / 1e12, "cores": cores, "kind": "port",
                          "sample": "sequence 0 of the B=4, T=4096 batch (16 layers, vocab 100352), forward only",
                          "parity_rel_l2": rel, "parity_max_abs": float(np.max(np.abs(d))), "top1_agreement": top1}
    return out


def bench_train(torch, dt, dev, args):
    """Training path (OlmoAttention::backward, flash_attention_backward).
    flash_bwd: dt_flash_bwd (fp32 in/out, bf16 casts inside) at config 1
    T=4096 (B=1) and at B=4, T=4096, H=16; algorithmic FLOPs 2.5x the causal
    forward (5 products of the forward's 2), L2 flushed before each call.
    layer: one attention layer forward + backward + SGD step at config 0 (B=1,
    T=512) and at the config-3 layer shape (B=4, T=4096); FLOPs = forward
    (2*tok*2048*8192 + 2*B*H*T^2*D) + backward (2x the projections + 2.5x the
    attention)."""
    out = {}
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    reps = max(3, min(args.steps, 10))
    for name, Bt, Tt in (("flash_bwd_config1_t4096", 1, 4096), ("flash_bwd_b4_t4096", 4, 4096)):
        g = torch.Generator(device=dev)
        g.manual_seed(Tt + Bt)
        q, k, v, do = (torch.randn((Bt, Tt, H, D), generator=g, device=dev) for _ in range(4))
        fwd = dt.flash_attention_forward(q, k, v, SCALE, True)
        ts = []
        for i in range(args.warmup + reps):
            flush.fill_(float(i))
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            dt.flash_attention_backward(do, fwd.output, fwd.softmax_m, fwd.softmax_l, q, k, v, SCALE, True)
            b.record()
            torch.cuda.synchronize()
            if i >= args.warmup:
                ts.append(a.elapsed_time(b))
        dt.check_device_error()
        ms = statistics.median(ts)
        f = 2.5 * 2.0 * Bt * H * Tt * Tt * D
        out[name] = {"B": Bt, "T": Tt, "ms": ms, "flops": f, "tflops": f / (ms * 1e-3) / 1e12,
                     "note": "includes the fp32->bf16 casts of q, k, v and dO"}
    rng = np.random.default_rng(3)
    w = [(0.02 * rng.standard_normal((DM, DM), dtype=np.float32)) for _ in range(4)]
    gains = [(1 + 0.02 * rng.standard_normal(DM, dtype=np.float32)).astype(np.float32) for _ in range(2)]
    attn = dt.OlmoAttention.from_weights(*w, *gains, device=dev.index or 0)
    for name, Bl, Tl in (("layer_train_config0", 1, 512), ("layer_train_b4_t4096", 4, 4096)):
        x = torch.from_numpy(rng.standard_normal((Bl, Tl, DM), dtype=np.float32)).to(dev)
        dy = torch.from_numpy(0.01 * rng.standard_normal((Bl, Tl, DM), dtype=np.float32)).to(dev)
        y, dx = torch.empty_like(x), torch.empty_like(x)
        ts = []
        for i in range(args.warmup + reps):
            flush.fill_(float(i))
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            attn.forward(x, out=y)
            attn.backward(dy, out=dx)
            attn.step(1e-6)
            attn.zero_grad()
            b.record()
            torch.cuda.synchronize()
            if i >= args.warmup:
                ts.append(a.elapsed_time(b))
        dt.check_device_error()
        ms = statistics.median(ts)
        tok = Bl * Tl
        f_proj = 2.0 * tok * DM * 8192
        f_attn = 2.0 * Bl * H * Tl * Tl * D
        f = f_proj + f_attn + 2 * f_proj + 2.5 * f_attn
        out[name] = {"B": Bl, "T": Tl, "ms": ms, "tok_s": tok / (ms * 1e-3), "flops": f,
                     "tflops": f / (ms * 1e-3) / 1e12, "step": "forward + backward + SGD step + zero_grad"}
    attn.close()
    return out


def bench_t4096(torch, dt, dev, args):
    """Config 1 at T=4096 (B=1, H=16): the single-GPU 50%-of-peak target.
    api: flash_attention_forward on fp32 Q, K, V -- the call a
      flash_attention_forward caller makes (dt_flash_fwd: one launch rounds K
      and V to bf16, then the attention kernel, which rounds Q itself);
    kernel: the attention kernel alone on bf16 operands already in HBM.
    Inputs are 32 MB per tensor (< L2), so L2 is flushed (256 MB write) before
    every timed call, outside the events."""
    Tt = 4096
    g = torch.Generator(device=dev)
    g.manual_seed(4096)
    q, k, v = (torch.randn((1, Tt, H, D), generator=g, device=dev) for _ in range(3))
    qb, kb, vb = dt.cast_bf16(q), dt.cast_bf16(k), dt.cast_bf16(v)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    out = torch.empty((1, Tt, H, D), dtype=torch.float32, device=dev)
    m = torch.empty((1, Tt, H), dtype=torch.float32, device=dev)
    l = torch.empty_like(m)

    def timed(fn):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
        for i in range(args.warmup + args.steps):
            flush.fill_(float(i))
            torch.cuda._sleep(1_000_000)  # the GPU is busy while the host queues the call
            e = ev[i - args.warmup] if i >= args.warmup else None
            if e:
                e[0].record()
            fn()
            if e:
                e[1].record()
        torch.cuda.synchronize()
        return statistics.median(a.elapsed_time(b) for a, b in ev)

    ms_api = timed(lambda: dt.flash_attention_forward(q, k, v, SCALE, True))
    ms_flash = timed(lambda: dt.flash_attention_forward_bf16(qb, kb, vb, SCALE, True, out=out, softmax_m=m,
                                                             softmax_l=l))
    dt.check_device_error()
    f = 2.0 * H * Tt * Tt * D
    peaks, src = load_peaks()
    peak = float(peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"]))
    return {"B": 1, "T": Tt, "H": H, "D": D, "flops": f,
            "ms_api": ms_api, "tflops_api": f / (ms_api * 1e-3) / 1e12, "frac_api": f / (ms_api * 1e-3) / 1e12 / peak,
            "api": "flash_attention_forward (dt_flash_fwd: fp32 Q/K/V in, fp32 O/m/l out)",
            "ms_flash": ms_flash, "tflops_flash": f / (ms_flash * 1e-3) / 1e12,
            "frac_flash": f / (ms_flash * 1e-3) / 1e12 / peak, "peak": peak,
            "peak_source": f"{src} bf16 burst", "l2": "flushed (256 MB write) before each call"}


def bench_prologue(torch, dt, dev, args):
    """QK-RMSNorm + RoPE prologue (qk_norm_rope_kernel) at the config-3 layer
    shape (B=4, T=4096: 16384 tokens), HBM-bound: algorithmic bytes per token =
    read q, k, v fp32 (3 * 2048 * 4) + write q, k, v bf16 (3 * 2048 * 2); the
    gains and RoPE tables (L2-resident) are not counted.  L2 flushed before
    each call."""
    Mt, Bp, Tp = 16384, 4, 4096
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    qkv = torch.randn((Mt, 3 * DM), generator=g, device=dev)
    gq = 1 + 0.02 * torch.randn(DM, generator=g, device=dev)
    gk = 1 + 0.02 * torch.randn(DM, generator=g, device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    reps = max(3, min(args.steps, 20))
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for i in range(args.warmup + reps):
        flush.fill_(float(i))
        torch.cuda._sleep(1_000_000)
        e = ev[i - args.warmup] if i >= args.warmup else None
        if e:
            e[0].record()
        dt.qk_norm_rope(qkv[:, :DM], qkv[:, DM:2 * DM], qkv[:, 2 * DM:], gq, gk, Bp, Tp)
        if e:
            e[1].record()
    torch.cuda.synchronize()
    dt.check_device_error()
    ms = statistics.median(a.elapsed_time(b) for a, b in ev)
    nbytes = Mt * 3 * DM * (4 + 2)
    peaks, src = load_peaks()
    hbm = float(peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
    return {"kernel": "qk_norm_rope_loop_kernel", "tokens": Mt, "ms": ms, "bytes": nbytes, "gbs": nbytes / ms / 1e6,
            "peak_gbs": hbm, "frac_hbm": nbytes / ms / 1e6 / hbm, "peak_source": f"{src} HBM copy"}


def run_sweep(args):
    """Flash kernel alone (bf16 operands already in HBM) and with the fp32->bf16
    casts, for config 1 (B=1, H=16, T = 64 ... 6144) and config 4 (B=16, T=6144).
    L2 is flushed (256 MB write) before every timed launch, outside the events,
    and a GPU-side spin before the start event hides the host's launch latency."""
    import torch

    import dirktensor_b200 as dt

    dev = torch.device("cuda:0")
    peaks, src = load_peaks()
    peak = float(peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"]))
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(1)
    rows = []
    for Bs, Ts in [(1, 64), (1, 512), (1, 1024), (1, 2048), (1, 4096), (1, 6144), (16, 6144)]:
        q, k, v = (torch.randn((Bs, Ts, H, D), generator=g, device=dev) for _ in range(3))
        out = torch.empty_like(q)
        reps = max(3, min(args.steps, 20))
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(reps)]
        for i in range(args.warmup + reps):
            flush.fill_(float(i))
            # keep the GPU busy while the host queues the launches below, so the
            # events time the kernels and not the host's launch latency
            torch.cuda._sleep(2_000_000)
            e = ev[i - args.warmup] if i >= args.warmup else None
            if e:
                e[0].record()
            qb, kb, vb = dt.cast_bf16(q), dt.cast_bf16(k), dt.cast_bf16(v)
            if e:
                e[1].record()
            dt.flash_attention_forward_bf16(qb, kb, vb, SCALE, True, out=out)
            if e:
                e[2].record()
        torch.cuda.synchronize()
        ms_flash = statistics.median(a.elapsed_time(b) for _, a, b in ev)
        ms_cast = statistics.median(a.elapsed_time(b) for a, b, _ in ev)
        f = 2.0 * Bs * H * Ts * Ts * D
        rows.append({"B": Bs, "T": Ts, "ms_flash": ms_flash, "tflops_flash": f / ms_flash / 1e9,
                     "frac_flash": f / ms_flash / 1e9 / peak, "ms_cast": ms_cast,
                     "tflops_with_cast": f / (ms_flash + ms_cast) / 1e9})
        del q, k, v, out, qb, kb, vb
    dt.check_device_error()
    # projection GEMMs at the configuration-3 shapes (M = 4 x 4096 tokens)
    grows = []
    for name, M, N, K in [("qkv", 16384, 6144, 2048), ("o_proj", 16384, 2048, 2048), ("mlp_gate_up", 16384, 16384, 2048),
                          ("mlp_down", 16384, 2048, 8192), ("lm_head", 16384, 100352, 2048),
                          ("config0_qkv", 512, 6144, 2048), ("config4_o_proj", 98304, 2048, 2048)]:
        a = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
        b = torch.randn((N, K), generator=g, device=dev).to(torch.bfloat16)
        c = torch.empty((M, N), dtype=torch.float32, device=dev)
        reps = 5
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        for i in range(args.warmup + reps):
            flush.fill_(float(i))
            torch.cuda._sleep(2_000_000)
            e = ev[i - args.warmup] if i >= args.warmup else None
            if e:
                e[0].record()
            dt.gemm_bf16_tn(a, b, out=c)
            if e:
                e[1].record()
        torch.cuda.synchronize()
        ms = statistics.median(x.elapsed_time(y) for x, y in ev)
        f = 2.0 * M * N * K
        grows.append({"gemm": name, "M": M, "N": N, "K": K, "ms": ms, "tflops": f / ms / 1e9,
                      "frac": f / ms / 1e9 / peak})
        del a, b, c
    dt.check_device_error()
    # HBM-bound kernels: the QK-norm/RoPE prologue and the fp32->bf16 cast at the
    # configuration-3 token count; algorithmic bytes = bytes read + bytes written once
    hbm = float(peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
    erows = []
    Mt = 16384
    qkv = torch.randn((Mt, 3 * DM), generator=g, device=dev)
    gq = torch.ones(DM, device=dev)
    reps = 10
    for name in ("qk_norm_rope", "cast_f32_bf16"):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        for i in range(args.warmup + reps):
            flush.fill_(float(i))
            torch.cuda._sleep(2_000_000)
            e = ev[i - args.warmup] if i >= args.warmup else None
            if e:
                e[0].record()
            if name == "qk_norm_rope":
                dt.qk_norm_rope(qkv[:, :DM], qkv[:, DM:2 * DM], qkv[:, 2 * DM:], gq, gq, 4, 4096)
            else:
                dt.cast_bf16(qkv)
            if e:
                e[1].record()
        torch.cuda.synchronize()
        ms = statistics.median(x.elapsed_time(y) for x, y in ev)
        nbytes = Mt * 3 * DM * (4 + 2)  # both kernels read 3*d fp32 and write 3*d bf16 per token
        erows.append({"kernel": name, "tokens": Mt, "ms": ms, "bytes": nbytes, "gbs": nbytes / ms / 1e6,
                      "frac_hbm": nbytes / ms / 1e6 / hbm})
    dt.check_device_error()
    print(json.dumps({"sweep": "flash_fwd causal, H=16, D=128", "peak": peak, "peak_source": f"{src} bf16 burst",
                      "rows": rows, "gemm": grows, "hbm_peak_gbs": hbm, "elementwise": erows}), flush=True)


def run_case(args):
    """Small fixed workloads for ncu captures (one GPU, a few launches)."""
    import torch

    import dirktensor_b200 as dt

    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    Bc, Tc = args.batch, args.seq
    if args.case == "gemm":
        M, N, K = (int(v) for v in args.gemm_mnk.split(","))
        a = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
        b = torch.randn((N, K), generator=g, device=dev).to(torch.bfloat16)
        c = torch.empty((M, N), dtype=torch.float32, device=dev)
        for _ in range(3):
            dt.gemm_bf16_tn(a, b, out=c)
    elif args.case == "flash_bwd":
        q, k, v, do = (torch.randn((Bc, Tc, H, D), generator=g, device=dev) for _ in range(4))
        fwd = dt.flash_attention_forward(q, k, v, SCALE, True)
        for _ in range(3):
            dt.flash_attention_backward(do, fwd.output, fwd.softmax_m, fwd.softmax_l, q, k, v, SCALE, True)
    elif args.case == "step4":
        from dirktensor_b200.head_parallel import HeadParallelAttention

        q, k, v = (torch.randn((B, T, H, D), generator=g, device=dev) for _ in range(3))
        hp = HeadParallelAttention(torch.randn((DM, DM), generator=g, device=dev) * 0.02, n_heads=H, head_dim=D)
        for _ in range(5):
            hp.forward(q, k, v, SCALE, True)
        hp.close()
    elif args.case == "prologue":
        qkv = torch.randn((Bc * Tc, 3 * DM), generator=g, device=dev)
        gq = torch.ones(DM, device=dev)
        for _ in range(3):
            dt.qk_norm_rope(qkv[:, :DM], qkv[:, DM:2 * DM], qkv[:, 2 * DM:], gq, gq, Bc, Tc)
    elif args.case == "flash_api":
        q, k, v = (torch.randn((Bc, Tc, H, D), generator=g, device=dev) for _ in range(3))
        for _ in range(3):
            dt.flash_attention_forward(q, k, v, SCALE, True)
    elif args.case == "flash_bf16":
        q, k, v = (torch.randn((Bc, Tc, H, D), generator=g, device=dev).to(torch.bfloat16) for _ in range(3))
        out = torch.empty((Bc, Tc, H, D), device=dev)
        for _ in range(3):
            dt.flash_attention_forward_bf16(q, k, v, SCALE, True, out=out)
    else:
        rng = np.random.default_rng(0)
        w = [0.02 * rng.standard_normal((DM, DM), dtype=np.float32) for _ in range(4)]
        gains = [np.ones(DM, np.float32), np.ones(DM, np.float32)]
        attn = dt.OlmoAttention.from_weights(*w, *gains)
        x = torch.randn((Bc, Tc, DM), generator=g, device=dev)
        for _ in range(3):
            attn.forward(x)
    torch.cuda.synchronize()
    dt.check_device_error()
    print("ok", args.case, Bc, Tc)


if __name__ == "__main__":
    main()
