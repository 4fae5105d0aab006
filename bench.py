#!/usr/bin/env python
"""Benchmark of the decode-attention hot path (one JSON line on rank 0).

Workload (default, BASELINE configs[3], the north-star call): batch 30720,
seqlen_q 1, seqlen_kv 16, num_heads_q = num_heads_kv = 32, head_dim 256, bf16
Q/K/V in [B,H,S,D] from the seeded generator (synthetic; the reference has no
dataset), fp16 O. One step = one fmha_forward call over the whole batch; with
N GPUs the batch is split into N contiguous shards (strong scaling: total work
fixed), one process per GPU, no collective on the data path.

metric: achieved HBM TB/s = algorithmic bytes per call / device time per call,
with bytes = 2*B*Hq*D (Q) + 4*B*Hkv*S*D (K+V) + 2*B*Hq*D (O), the reference's
own formula (fmha_host.cpp:428-431). ms_per_step is the matching us/call.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--config NAME] [--variant auto|bulk|ldg] [--sweep]

After the timed region each rank checks every row of its output against the
CPU oracle (`parity`), reports every rank's device time (`per_rank_ms`), and,
with N > 1, all-gathers the sharded O over NCCL and checks it (`gather`).

--impl reference times the reference's own CPU implementation of the path
(oracle/_ref: the reference's do_validation compiled from its sources; the
oracle port if that build is absent) on the host cores, on the full batch
every step; under torchrun only rank 0 runs it.

--sweep [--sweep-auto] [--sweep-gb G] prints device-time lines for every
config (small cases of about G GB for ncu captures); --traffic-from CSV turns
the ncu CSV of such a run into profiles/ncu_traffic.json.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    # name: (batch, num_heads_q, num_heads_kv, seqlen_kv, head_dim)
    "flagship": (30720, 32, 32, 16, 256),          # configs[3]; 1..8 GPU scaling
    "h16_d128_s1": (30720, 16, 16, 1, 128),        # configs[0]
    "h16_d128_s16": (30720, 16, 16, 16, 128),      # configs[1]
    "h16_d256_s16": (30720, 16, 16, 16, 256),      # configs[2]
    "gqa_32_16_d256_s16": (30720, 32, 16, 16, 256),
}
for _s in (1, 2, 4, 8, 16):
    for _d in (128, 256):
        for _h in (16, 32):
            CONFIGS.setdefault(f"h{_h}_d{_d}_s{_s}", (30720, _h, _h, _s, _d))
    CONFIGS.setdefault(f"gqa_32_16_d256_s{_s}", (30720, 32, 16, _s, 256))
    CONFIGS.setdefault(f"gqa_32_16_d128_s{_s}", (30720, 32, 16, _s, 128))
    for _hkv in (8, 4):  # 4 and 8 query heads per kv head
        for _d in (128, 256):
            CONFIGS.setdefault(f"gqa_32_{_hkv}_d{_d}_s{_s}", (30720, 32, _hkv, _s, _d))

# The reference's own benchmark table (fmha_host.cpp:511-517): packed varlen
# K/V with Poisson(4) seqlens in [2, 16] (seed 42) -> fmha_forward_varlen.
VARLEN = {f"varlen_h{_h}_d{_d}": (30720, _h, _h, 16, _d) for _h in (16, 32) for _d in (128, 256)}
VARLEN.update({f"varlen_gqa_32_16_d{_d}": (30720, 32, 16, 16, _d) for _d in (128, 256)})
CONFIGS.update(VARLEN)

L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0
METRIC = "decode-attn achieved HBM TB/s (algorithmic bytes / device time per call)"


def algo_bytes(b, hq, hkv, s, d):
    return 2 * b * hq * d + 4 * b * hkv * s * d + 2 * b * hq * d


def algo_flops(b, hq, s, d):
    return 4 * b * hq * s * d  # fmha_host.cpp:413-414


def peak_hbm():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(name):
    """DRAM bytes per launch of the dominant kernel from a committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(p) as f:
            return json.load(f).get(name)
    except (OSError, ValueError):
        return None


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.gpus = set(gpu_indices)
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(prefix="fmha_clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9 or not parts[0].isdigit() or int(parts[0]) not in self.gpus:
                    continue
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1])]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        per_gpu = {}
        for g in sorted({int(r[0]) for r in rows}):
            mine = [r for r in rows if int(r[0]) == g]
            v = [num(r[1]) for r in mine if num(r[1])]
            per_gpu[str(g)] = {"sm_mhz": statistics.median(v) if v else None,
                               "sm_mhz_min": min(v) if v else None,
                               "power_w_max": max(num(r[3]) or 0 for r in mine),
                               "reasons": sorted({names[i] for r in mine for i in range(4)
                                                  if r[5 + i] == "Active"})}
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(num(r[2]) or 0 for r in rows),
                "power_w_max": max(num(r[3]) or 0 for r in rows),
                "reasons": reasons, "samples": len(rows), "per_gpu": per_gpu}


# ---------------------------------------------------------------- reference arm

def run_reference_arm(args, cfg_name, cfg):
    """The reference's own CPU attention (do_validation, fmha_host.cpp:158-284,
    built from the reference sources into oracle/_ref) on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import numpy as np
    from oracle import oracle as O
    b_all, hq, hkv, s, d = cfg
    use_ref = O.ref_available() and hq == hkv
    threads = os.cpu_count() or 1
    if use_ref:
        threads = O.ref().fmha_ref_hardware_threads()
    else:
        O.set_threads(threads)

    def make(nrows):
        q, k, v = O.make_inputs_bhsd(nrows, hq, hkv, s, d, seed=0)
        if use_ref:
            def pack(x):
                return np.ascontiguousarray(
                    x.reshape(nrows, hkv, s, d).transpose(0, 2, 1, 3)).reshape(-1)
            k, v = pack(k), pack(v)
        return q, k, v

    def step(nrows, q, k, v):
        if use_ref:
            sl = np.full(nrows, s, dtype=np.int32)
            O.ref_do_validation(q, k, v, sl, nrows, hq, hkv, d, threads=threads)
        else:
            O.decode_bhsd(q, k, v, nrows, hq, hkv, s, d, want_f32=False)

    # The whole batch every step (the CPU work is linear in rows; timing the
    # full call makes ms_per_step a measurement, not an extrapolation). Only
    # when the host cannot hold the inputs twice over is a contiguous sample
    # used, and the line says so.
    import psutil
    need = 2 * 2 * (b_all * hq * d + 2 * b_all * hkv * s * d) * (2 if use_ref else 1)
    n = b_all
    if psutil.virtual_memory().available < need:
        n = max(1, int(b_all * psutil.virtual_memory().available / need))
    q, k, v = make(n)
    for _ in range(args.warmup):
        step(n, q, k, v)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step(n, q, k, v)
        times.append(time.perf_counter() - t0)
    sec = sum(times) / len(times)
    tbps = algo_bytes(n, hq, hkv, s, d) / sec / 1e12
    kind = "reference" if use_ref else "port"
    sample = (f"{n} of {b_all} batch rows per step (seed 0); "
              + ("reference do_validation (bf16 P) built from fmha_host.cpp, one batch slice "
                 "per thread" if use_ref else "oracle restatement (fp32 P), OpenMP over batch"))
    line = {
        "impl": "reference", "metric": METRIC, "value": round(tbps, 6), "unit": "TB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sec * 1e3, 3),
        "rows_per_step": n,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded bf16 N(0,1) approximation)",
        "config": config_block(cfg_name, cfg, 1),
        "cpu_baseline": {"value": round(tbps, 6), "unit": "TB/s", "cores": threads, "kind": kind,
                         "sample": sample},
        "e2e": {"value": round(tbps, 6), "unit": "TB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def config_block(name, cfg, n_gpus):
    b, hq, hkv, s, d = cfg
    total = algo_bytes(b, hq, hkv, s, d)
    if name in VARLEN:
        return {"workload": f"decode attention {name}: batch={b} seqlen_q=1 seqlen_kv "
                            f"Poisson(4) in [2,{s}] (seed 42, the reference's table) "
                            f"num_heads_q={hq} num_heads_kv={hkv} head_dim={d}",
                "batch": b, "seqlen_q": 1, "max_seqlen_kv": s, "num_heads_q": hq,
                "num_heads_kv": hkv, "head_dim": d,
                "layout": "Q/O [B,H,1,D], K/V packed [sum S_b,Hkv,D] + cu_seqlens_kv",
                "global_batch": b, "parallelism": f"batch-shard x{n_gpus} (no collective)",
                "l2": "inputs larger than L2; no flush"}
    return {"workload": f"decode attention {name}: batch={b} seqlen_q=1 seqlen_kv={s} "
                        f"num_heads_q={hq} num_heads_kv={hkv} head_dim={d}",
            "batch": b, "seqlen_q": 1, "seqlen_kv": s, "num_heads_q": hq, "num_heads_kv": hkv,
            "head_dim": d, "layout": "Q/O [B,H,1,D], K/V [B,Hkv,S,D]",
            "global_batch": b, "parallelism": f"batch-shard x{n_gpus} (no collective)",
            "bytes_per_call": total,
            "l2": f"inputs larger than L2 ({total / 1e9:.2f} GB per call vs 126 MB L2); no flush"
                  if total / n_gpus > 3 * L2_BYTES else "rotating input sets > 3x L2"}


# ---------------------------------------------------------------- our arm

def cpu_baseline_leg(cfg, seconds=10.0):
    """The oracle port (fp32-P restatement of the reference math, OpenMP over
    all host cores) on a bounded sample of the same workload."""
    import numpy as np  # noqa: F401
    from oracle import oracle as O
    b_all, hq, hkv, s, d = cfg
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    n = min(b_all, 128)
    while True:
        q, k, v = O.make_inputs_bhsd(n, hq, hkv, s, d, seed=0)
        t0 = time.perf_counter()
        O.decode_bhsd(q, k, v, n, hq, hkv, s, d, want_f32=False)
        dt = time.perf_counter() - t0
        if dt >= seconds / 4 or n >= b_all:
            break
        n = min(b_all, int(n * max(2.0, seconds / 4 / max(dt, 1e-4))))
    reps, tot = 0, 0.0
    while tot < seconds and reps < 100:
        t0 = time.perf_counter()
        O.decode_bhsd(q, k, v, n, hq, hkv, s, d, want_f32=False)
        tot += time.perf_counter() - t0
        reps += 1
    sec = tot / reps
    return {"value": round(algo_bytes(n, hq, hkv, s, d) / sec / 1e12, 6), "unit": "TB/s",
            "cores": O.threads(), "kind": "port",
            "sample": f"{n} of {b_all} batch rows x {reps} reps ({tot:.1f} s); oracle fp32-P "
                      "restatement, OpenMP over batch rows"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="flagship", choices=sorted(CONFIGS))
    ap.add_argument("--variant", default="auto", choices=["auto", "bulk", "ldg"])
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the all-rows check of the output against the CPU oracle")
    ap.add_argument("--no-gather", action="store_true",
                    help="skip the NCCL all-gather of the sharded output (N > 1)")
    ap.add_argument("--no-clocks", action="store_true",
                    help="skip the nvidia-smi sampler (profiling runs)")
    ap.add_argument("--varlen-uniform", type=int, default=0,
                    help="varlen configs: every row this long instead of Poisson(4) (profiling)")
    ap.add_argument("--varlen-mix", default="",
                    help="varlen configs: rows cycle through these lengths, e.g. 3,4 (profiling)")
    ap.add_argument("--batch", type=int, default=0,
                    help="override the config's batch (small profiling cases only)")
    ap.add_argument("--sweep-gb", type=float, default=0.0,
                    help="--sweep: shrink each config's batch to about this many GB per call "
                         "(never below 3x L2; small cases for ncu captures)")
    ap.add_argument("--traffic-from", default="",
                    help="write profiles/ncu_traffic.json from an ncu CSV of a --sweep-gb run")
    ap.add_argument("--sweep", action="store_true",
                    help="device-time lines for every config and variant (no e2e/cpu)")
    ap.add_argument("--sweep-configs", default="",
                    help="comma-separated config names for --sweep (default: all)")
    ap.add_argument("--sweep-warps", default="8,16",
                    help="bulk consumer-warp counts to try in --sweep")
    ap.add_argument("--sweep-auto", action="store_true",
                    help="--sweep with the library's own per-shape choice only")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    if args.traffic_from:
        return write_traffic_table(args)
    if args.impl == "reference":
        return run_reference_arm(args, args.config, CONFIGS[args.config])

    import torch
    import fmha_b200

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and rank == 0:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    fmha_b200.load()

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if args.sweep:
        names = [x for x in args.sweep_configs.split(",") if x] or sorted(CONFIGS)
        trials = [("ldg", None)] + [("bulk", int(w)) for w in args.sweep_warps.split(",") if w]
        if args.sweep_auto:
            trials = [("auto", None)]
        for name in names:
            cfg_n = CONFIGS[name]
            if args.batch > 0:
                cfg_n = (args.batch,) + tuple(cfg_n[1:])
            elif args.sweep_gb > 0:
                cfg_n = (small_batch(name, args.sweep_gb),) + tuple(cfg_n[1:])
            for var, warps in trials:
                if warps is not None:
                    os.environ["FMHA_BULK_WARPS"] = str(warps)
                if name in VARLEN:
                    if var not in ("ldg", "auto"):
                        continue  # one varlen line
                    r = time_varlen(torch, fmha_b200, cfg_n, world, rank, args, barrier,
                                    max_over_ranks, dev)
                else:
                    r = time_config(torch, fmha_b200, cfg_n, world, rank, args, var,
                                    barrier, max_over_ranks, dev, clocks=False)
                if rank == 0:
                    print(json.dumps({"sweep": name, "variant": var, "warps": warps, **r}),
                          flush=True)
        os.environ.pop("FMHA_BULK_WARPS", None)
        return 0

    cfg = CONFIGS[args.config]
    if args.batch > 0:
        cfg = (args.batch,) + tuple(cfg[1:])
    varlen = args.config in VARLEN
    keep = []
    if varlen:
        # The reference's own table: packed K/V, Poisson(4) seqlens (device time
        # only; the e2e and CPU legs are defined for the dense north-star call).
        r = time_varlen(torch, fmha_b200, cfg, world, rank, args, barrier, max_over_ranks, dev,
                        keep=keep)
        args.no_e2e = args.no_cpu = True
    else:
        r = time_config(torch, fmha_b200, cfg, world, rank, args, args.variant, barrier,
                        max_over_ranks, dev, clocks=not args.no_clocks, keep=keep)
    ranks_ms = per_rank(torch, dist, dev, r["kernel_ms"], world)
    parity = None
    if not args.no_parity:
        parity = parity_leg(torch, dist, dev, keep, cfg, world, rank, varlen)
    gather = None
    if world > 1 and not args.no_gather:
        gather = gather_leg(torch, dist, dev, keep[3], cfg, world, rank)
    del keep
    torch.cuda.empty_cache()
    e2e = None
    if not args.no_e2e:
        e2e = e2e_leg(torch, fmha_b200, cfg, world, rank, args, barrier, max_over_ranks, dev)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline_leg(cfg)
    if rank == 0:
        peak, peak_src = peak_hbm()
        b, hq, hkv, s, d = cfg
        per_launch_bytes = (r["bytes_total"] if varlen else algo_bytes(b, hq, hkv, s, d)) / world
        achieved = per_launch_bytes / (r["kernel_ms"] * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": r["value"], "unit": "TB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
            "us_per_call": round(r["ms_per_step"] * 1e3, 2),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "compute_dtype": "f32 (bf16 in, fp16 out)",
            "data": "synthetic (seeded bf16 N(0,1) approximation, generated on device)",
            "config": config_block(args.config, cfg, world),
            "variant": args.variant,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs, copy bw)"
                         if peak_src == "measured" else "fallback 6.65 TB/s",
                         "traffic": ncu_traffic(args.config),
                         "kernel": "fmha::decode_*_kernel (one launch per step)"},
            "gpu_launches": args.steps,
            "per_rank_ms": ranks_ms,
            "parity": parity,
            "gather": gather,
            "clocks": r["clocks"],
            "e2e": e2e,
            "cpu_baseline": cpu,
            "flops_per_call": algo_flops(b, hq, s, d),
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()
    return 0


def row_bytes(name):
    """Algorithmic bytes of one batch row of a config (varlen: at the mean
    Poisson(4) length in [2, 16], 4.35)."""
    _, hq, hkv, s, d = CONFIGS[name]
    if name in VARLEN:
        return 4 * hq * d + 4 * 4.35 * hkv * d
    return algo_bytes(1, hq, hkv, s, d)


def small_batch(name, gb):
    """A batch for a small profiling case of `name`: about `gb` GB per call,
    at least 3x L2 of traffic, at most the config's own batch."""
    b_all = CONFIGS[name][0]
    want = max(gb * 1e9, 3 * L2_BYTES) / row_bytes(name)
    return int(min(b_all, max(1, math.ceil(want))))


def write_traffic_table(args):
    """profiles/ncu_traffic.json from the ncu CSV of
    `bench.py --sweep --sweep-auto --sweep-gb G --steps K --warmup W` run under
    `ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum,gpu__time_duration.sum`:
    per config, the last captured launch's DRAM bytes, scaled from the small
    batch to the config's full batch by rows (read traffic grows in proportion
    to the rows processed)."""
    import csv
    names = [x for x in args.sweep_configs.split(",") if x] or sorted(CONFIGS)
    per = args.warmup + args.steps
    rows = {}
    with open(args.traffic_from) as f:
        lines = [ln for ln in f if ln.startswith('"')]
    for r in csv.DictReader(lines):
        if "decode" not in r.get("Kernel Name", ""):
            continue
        key = int(r["ID"])
        e = rows.setdefault(key, {"kernel": r["Kernel Name"].split("(")[0]})
        e[r["Metric Name"]] = float(r["Metric Value"].replace(",", ""))
        e[r["Metric Name"] + " unit"] = r["Metric Unit"]
    launches = [rows[k] for k in sorted(rows)]
    if len(launches) != per * len(names):
        raise SystemExit(f"{len(launches)} decode launches in the CSV, expected "
                         f"{per} x {len(names)} configs")
    scale_unit = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}
    table = {"_note": "DRAM bytes (read + write) per full-size launch of each config's "
                      "dominant kernel: ncu dram__bytes_read.sum + dram__bytes_write.sum of a "
                      f"small case (about {args.sweep_gb} GB per call, >= 3x L2), scaled to the "
                      "config's batch by rows processed"}
    for i, name in enumerate(names):
        e = launches[(i + 1) * per - 1]
        rd = e["dram__bytes_read.sum"] * scale_unit[e["dram__bytes_read.sum unit"]]
        wr = e["dram__bytes_write.sum"] * scale_unit[e["dram__bytes_write.sum unit"]]
        b_small = small_batch(name, args.sweep_gb)
        b_all = CONFIGS[name][0]
        table[name] = round((rd + wr) * b_all / b_small)
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    with open(p, "w") as f:
        json.dump(table, f, indent=1, sort_keys=True)
        f.write("\n")
    print(f"wrote {len(table)} configs to {p}")
    return 0


ATOL, RTOL = 2e-3, 1e-2   # the library tolerance, against the fp32-P oracle
PARITY_SLICE_ROWS = 1024


def per_rank(torch, dist, dev, ms, world):
    """Device ms per call of every rank (min / median / max and the list)."""
    vals = [ms]
    if dist is not None:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        out = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(out, t)
        vals = [float(x.item()) for x in out]
    return {"min": round(min(vals), 5), "median": round(statistics.median(vals), 5),
            "max": round(max(vals), 5), "all": [round(v, 5) for v in vals]}


def parity_leg(torch, dist, dev, keep, cfg, world, rank, varlen):
    """Every row of this rank's output against the CPU oracle (the fp32-P
    restatement of the reference's do_validation, fmha_host.cpp:158-284) on
    the same inputs, copied back from the device after the timed region, in
    slices of PARITY_SLICE_ROWS rows. An element passes when |o-r| <= 2e-3 or
    |o-r| <= 1e-2*|r|; a non-finite output fails. Sums over ranks."""
    import numpy as np
    from oracle import oracle as Or
    _, hq, hkv, s, d = cfg
    Q, K, V, O = keep[:4]
    Or.set_threads(max(1, (os.cpu_count() or 1) // world))
    t0 = time.perf_counter()
    qn = hq * d
    b = O.numel() // qn

    def bits(x):
        return x.cpu().view(torch.int16).numpy().view(np.uint16)

    bad, max_abs = 0, 0.0
    for r0 in range(0, b, PARITY_SLICE_ROWS):
        r1 = min(b, r0 + PARITY_SLICE_ROWS)
        q = bits(Q[r0 * qn:r1 * qn])
        if varlen:
            cu = np.asarray(keep[4], dtype=np.int64)
            c0, c1 = int(cu[r0]), int(cu[r1])
            k = bits(K[c0 * hkv * d:c1 * hkv * d])
            v = bits(V[c0 * hkv * d:c1 * hkv * d])
            ref, _ = Or.decode_thd(q, k, v, (cu[r0:r1 + 1] - c0).astype(np.int32), r1 - r0, hq,
                                   hkv, d)
        else:
            kn = hkv * s * d
            k = bits(K[r0 * kn:r1 * kn])
            v = bits(V[r0 * kn:r1 * kn])
            ref, _ = Or.decode_bhsd(q, k, v, r1 - r0, hq, hkv, s, d)
        o = bits(O[r0 * qn:r1 * qn]).view(np.float16).astype(np.float32)
        err = np.abs(o - ref)
        ok = np.isfinite(o) & ((err <= ATOL) | (err <= RTOL * np.abs(ref)))
        bad += int((~ok).sum())
        max_abs = max(max_abs, float(np.nanmax(err)) if err.size else 0.0)
    sec = time.perf_counter() - t0
    rows, elems = b, b * qn
    if dist is not None:
        t = torch.tensor([rows, elems, bad], dtype=torch.int64, device=dev)
        dist.all_reduce(t)
        rows, elems, bad = (int(x) for x in t.tolist())
        m = torch.tensor([max_abs, sec], dtype=torch.float64, device=dev)
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        max_abs, sec = (float(x) for x in m.tolist())
    return {"rows": rows, "elements": elems, "bad": bad, "max_abs": float(f"{max_abs:.3e}"),
            "rule": "|o-r| <= 2e-3 or |o-r| <= 1e-2*|r| vs the fp32-P oracle, every row",
            "check_s": round(sec, 2)}


def gather_leg(torch, dist, dev, O, cfg, world, rank):
    """All-gather of the sharded O over NCCL (fmha_b200.multi.gather_output),
    device-timed, max over ranks, then checked: every rank's slice of the
    gathered tensor must equal that rank's own shard bit for bit (compared
    through two int64 checksums all-gathered from the ranks)."""
    from fmha_b200.multi import gather_output, make_shard
    b_all, hq, hkv, s, d = cfg
    sh = make_shard(b_all, hq, hkv, s, d, world, rank)

    def checksum(x):
        v = x.reshape(-1).view(torch.int16).to(torch.int64)
        w = torch.arange(v.numel(), device=v.device, dtype=torch.int64) % 65521 + 1
        return torch.stack([v.sum(), (v * w).sum()])

    full = gather_output(O, sh)  # warm-up (NCCL communicator set-up)
    del full
    torch.cuda.synchronize(dev)
    dist.barrier()
    stream = torch.cuda.current_stream(dev)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    full = gather_output(O, sh)
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    ms = ev0.elapsed_time(ev1)
    mine = checksum(O)
    sums = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(sums, mine)
    ok = full.numel() == b_all * hq * d
    for r in range(world):
        lo, hi = shard_rows_(b_all, world, r)
        part = full[lo * hq * d:hi * hq * d]
        ok = ok and bool(torch.equal(checksum(part), sums[r]))
    ok = ok and bool(torch.equal(full[sh.o_offset:sh.o_offset + O.numel()].view(torch.int16),
                                 O.view(torch.int16)))
    t = torch.tensor([0 if ok else 1], dtype=torch.int64, device=dev)
    dist.all_reduce(t)
    m = torch.tensor([ms], dtype=torch.float64, device=dev)
    dist.all_reduce(m, op=dist.ReduceOp.MAX)
    ms = float(m.item())
    nbytes = full.numel() * full.element_size()
    del full
    return {"ok": int(t.item()) == 0, "ms": round(ms, 4), "bytes": nbytes,
            "algbw_gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
            "busbw_gbs": round(nbytes * (world - 1) / world / (ms * 1e-3) / 1e9, 1),
            "how": "NCCL all-gather of the fp16 O shards (torch.distributed), max over ranks"}


def shard_rows_(b_all, world, rank):
    from fmha_b200.multi import shard_rows
    return shard_rows(b_all, world, rank)


def shard(b_all, world, rank):
    from fmha_b200.multi import shard_rows
    return shard_rows(b_all, world, rank)


def alloc_inputs(torch, fmha_b200, cfg, lo, hi, dev):
    b_all, hq, hkv, s, d = cfg
    b = hi - lo
    Q = torch.empty(b * hq * d, dtype=torch.bfloat16, device=dev)
    K = torch.empty(b * hkv * s * d, dtype=torch.bfloat16, device=dev)
    V = torch.empty_like(K)
    fmha_b200.fill_normal_bf16(Q, 0, 1, lo * hq * d)
    fmha_b200.fill_normal_bf16(K, 0, 2, lo * hkv * s * d)
    fmha_b200.fill_normal_bf16(V, 0, 3, lo * hkv * s * d)
    O = torch.empty(b * hq * d, dtype=torch.float16, device=dev)
    return Q, K, V, O


def time_config(torch, fmha_b200, cfg, world, rank, args, variant, barrier, max_over_ranks, dev,
                clocks, keep=None):
    """Device time of K back-to-back calls on this rank's shard. When `keep`
    is a list, the first input set and its output (Q, K, V, O) are appended
    to it for the parity and gather checks after timing."""
    b_all, hq, hkv, s, d = cfg
    lo, hi = shard(b_all, world, rank)
    b = hi - lo
    per_call = algo_bytes(b, hq, hkv, s, d)
    nsets = 1 if per_call > 3 * L2_BYTES else math.ceil(3 * L2_BYTES / per_call) + 1
    sets = [alloc_inputs(torch, fmha_b200, cfg, lo, hi, dev) for _ in range(nsets)]
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream

    def call(i):
        Q, K, V, O = sets[i % nsets]
        st = fmha_b200.fmha_forward_ptr(Q, K, V, O, b, hq, hkv, s, d, stream=sh, variant=variant)
        if st != 0:
            raise fmha_b200.FmhaError(st, "fmha_forward")

    for i in range(args.warmup):
        call(i)
    torch.cuda.synchronize(dev)
    sampler = ClockSampler([local_gpu_index(dev, r) for r in range(world)] if rank == 0 else [])
    if clocks and rank == 0:
        sampler.start()
    barrier()
    torch.cuda.synchronize(dev)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i in range(args.steps):
        call(i)
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    clk = None
    if clocks:
        # Too short a timed region for the sampler: every rank keeps the same
        # kernel running (untimed) until ~1 s of load has been sampled, so each
        # GPU's clock record is taken under load.
        t0 = time.perf_counter()
        while (time.perf_counter() - t0) * 1e3 < max(0.0, 1000.0 - ms * args.steps):
            for i in range(50):
                call(i)
            torch.cuda.synchronize(dev)
        if rank == 0:
            clk = sampler.stop()
    if fmha_b200.device_error() != 0:
        raise RuntimeError("device error word set during the timed region")
    ms_max = max_over_ranks(ms)
    total = algo_bytes(b_all, hq, hkv, s, d)
    r = {"value": round(total / (ms_max * 1e-3) / 1e12, 4), "ms_per_step": round(ms_max, 5),
         "kernel_ms": ms, "clocks": clk}
    if keep is not None:
        call(0)  # set 0's O from one more call, outside the timed region
        torch.cuda.synchronize(dev)
        keep.extend(sets[0])
    del sets
    torch.cuda.empty_cache()
    return r


def time_varlen(torch, fmha_b200, cfg, world, rank, args, barrier, max_over_ranks, dev, keep=None):
    """fmha_forward_varlen on the reference's packed layout and seqlens; this
    rank's batch shard. Bytes: Q + K + V (sum of seqlens) + O."""
    import numpy as np
    b_all, hq, hkv, max_s, d = cfg
    sl_all = fmha_b200.seqlens_poisson(b_all, max_s, 42, 4.0)
    if args.varlen_uniform > 0:
        sl_all[:] = args.varlen_uniform
    if args.varlen_mix:
        mix = np.array([int(x) for x in args.varlen_mix.split(",")], dtype=np.int32)
        sl_all[:] = np.resize(mix, b_all)
    lo, hi = shard(b_all, world, rank)
    b = hi - lo
    cu_all = np.concatenate([[0], np.cumsum(sl_all)]).astype(np.int64)
    t0_row, t1_row = int(cu_all[lo]), int(cu_all[hi])
    cu = torch.from_numpy((cu_all[lo:hi + 1] - t0_row).astype(np.int32)).to(dev)
    Q = torch.empty(b * hq * d, dtype=torch.bfloat16, device=dev)
    K = torch.empty((t1_row - t0_row) * hkv * d, dtype=torch.bfloat16, device=dev)
    V = torch.empty_like(K)
    fmha_b200.fill_normal_bf16(Q, 0, 1, lo * hq * d)
    fmha_b200.fill_normal_bf16(K, 0, 2, t0_row * hkv * d)
    fmha_b200.fill_normal_bf16(V, 0, 3, t0_row * hkv * d)
    O = torch.empty(b * hq * d, dtype=torch.float16, device=dev)
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream

    def call():
        st = fmha_b200.fmha_forward_varlen_ptr(Q, K, V, O, cu, b, hq, hkv, max_s, d, 0.0, sh)
        if st != 0:
            raise fmha_b200.FmhaError(st, "fmha_forward_varlen")

    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize(dev)
    barrier()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        call()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    if fmha_b200.device_error() != 0:
        raise RuntimeError("device error word set during the timed region")
    ms = ev0.elapsed_time(ev1) / args.steps
    ms_max = max_over_ranks(ms)
    total_rows = int(cu_all[-1])
    total = 2 * b_all * hq * d + 4 * total_rows * hkv * d + 2 * b_all * hq * d
    if keep is not None:
        keep.extend([Q, K, V, O, cu_all[lo:hi + 1] - t0_row])
    del Q, K, V, O
    torch.cuda.empty_cache()
    return {"value": round(total / (ms_max * 1e-3) / 1e12, 4), "ms_per_step": round(ms_max, 5),
            "kernel_ms": ms, "clocks": None, "mean_seqlen": float(sl_all.mean()),
            "bytes_total": total}


def local_gpu_index(dev, r):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x for x in vis.split(",") if x.strip()]
        if r < len(ids) and ids[r].strip().isdigit():
            return int(ids[r])
    return r


E2E_SLICES = 8


def bind_to_gpu_cpus(dev, local_rank):
    """Binds the calling thread to the CPUs NVML reports as local to this GPU
    (intersected with the CPUs the process may use). Returns (previous
    affinity or None, a short description)."""
    try:
        import pynvml
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(local_gpu_index(dev, local_rank))
        ncpu = os.cpu_count() or 1
        words = pynvml.nvmlDeviceGetCpuAffinity(h, (ncpu + 63) // 64)
        local = {w * 64 + i for w, m in enumerate(words) for i in range(64) if (int(m) >> i) & 1}
        before = os.sched_getaffinity(0)
        cpus = local & before
        if not cpus or cpus == before:
            return None, f"unbound ({len(before)} cpus; NVML-local {len(local)})"
        os.sched_setaffinity(0, cpus)
        return before, f"bound to {len(cpus)} NVML-local cpus of {len(before)}"
    except Exception as e:  # NVML missing or unsupported: leave the thread unbound
        return None, f"unbound ({type(e).__name__})"


def e2e_leg(torch, fmha_b200, cfg, world, rank, args, barrier, max_over_ranks, dev):
    """The same call through the C ABI with HOST buffers: each step copies
    this shard's Q/K/V from pinned host memory to the device, runs
    fmha_forward and copies O back, all inside the timed region."""
    import psutil
    b_all, hq, hkv, s, d = cfg
    lo, hi = shard(b_all, world, rank)
    b = hi - lo
    # Host buffers are pinned from a thread bound to the GPU's NUMA-local
    # cores, so their pages land on the node next to the GPU's PCIe root.
    saved_aff, numa = bind_to_gpu_cpus(dev, int(os.environ.get("LOCAL_RANK", "0")))
    Q, K, V, O = alloc_inputs(torch, fmha_b200, cfg, lo, hi, dev)
    need = 2 * (Q.numel() + K.numel() + V.numel() + O.numel())
    if psutil.virtual_memory().available < 1.5 * need * world:
        return {"value": None, "unit": "TB/s", "note": "not enough host RAM to pin the inputs"}
    hQ = torch.empty_like(Q, device="cpu", pin_memory=True)
    hK = torch.empty_like(K, device="cpu", pin_memory=True)
    hV = torch.empty_like(V, device="cpu", pin_memory=True)
    hO = torch.empty_like(O, device="cpu", pin_memory=True)
    hQ.copy_(Q)
    hK.copy_(K)
    hV.copy_(V)
    stream = torch.cuda.current_stream(dev)
    # The step is pipelined over E2E_SLICES batch slices on three streams:
    # host->device copies of slice i+1 overlap the call on slice i and the
    # device->host copy of slice i-1 (PCIe is full duplex).
    s_in, s_run, s_out = (torch.cuda.Stream(dev) for _ in range(3))
    nsl = max(1, min(E2E_SLICES, b))
    bounds = [b * i // nsl for i in range(nsl + 1)]
    qn, kn = hq * d, hkv * s * d

    def step():
        start = torch.cuda.Event()
        start.record(stream)
        for st_ in (s_in, s_run, s_out):
            st_.wait_event(start)
        last = None
        for i in range(nsl):
            r0, r1 = bounds[i], bounds[i + 1]
            if r1 == r0:
                continue
            with torch.cuda.stream(s_in):
                Q[r0 * qn:r1 * qn].copy_(hQ[r0 * qn:r1 * qn], non_blocking=True)
                K[r0 * kn:r1 * kn].copy_(hK[r0 * kn:r1 * kn], non_blocking=True)
                V[r0 * kn:r1 * kn].copy_(hV[r0 * kn:r1 * kn], non_blocking=True)
                ev_in = torch.cuda.Event()
                ev_in.record(s_in)
            s_run.wait_event(ev_in)
            q0, k0 = r0 * qn * 2, r0 * kn * 2
            st = fmha_b200.fmha_forward_ptr(Q.data_ptr() + q0, K.data_ptr() + k0,
                                            V.data_ptr() + k0, O.data_ptr() + q0, r1 - r0,
                                            hq, hkv, s, d, stream=s_run.cuda_stream)
            if st != 0:
                raise fmha_b200.FmhaError(st, "fmha_forward")
            ev_run = torch.cuda.Event()
            ev_run.record(s_run)
            s_out.wait_event(ev_run)
            with torch.cuda.stream(s_out):
                hO[r0 * qn:r1 * qn].copy_(O[r0 * qn:r1 * qn], non_blocking=True)
                last = torch.cuda.Event()
                last.record(s_out)
        if last is not None:
            stream.wait_event(last)

    step()
    torch.cuda.synchronize(dev)
    barrier()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.e2e_steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    my_ms = ev0.elapsed_time(ev1) / args.e2e_steps
    ms = max_over_ranks(my_ms)
    h2d = 2 * (Q.numel() + K.numel() + V.numel())
    d2h = 2 * O.numel()
    dist_ = None
    if world > 1:
        import torch.distributed as dist_
    ranks = per_rank(torch, dist_, dev, my_ms, world)
    ranks["h2d_gbs_min"] = round(h2d / (ranks["max"] * 1e-3) / 1e9, 1)
    ranks["h2d_gbs_max"] = round(h2d / (ranks["min"] * 1e-3) / 1e9, 1)
    del Q, K, V, O, hQ, hK, hV, hO
    torch.cuda.empty_cache()
    if saved_aff is not None:
        os.sched_setaffinity(0, saved_aff)
    return {"value": round(algo_bytes(b_all, hq, hkv, s, d) / (ms * 1e-3) / 1e12, 5),
            "unit": "TB/s", "ms_per_step": round(ms, 3), "steps": args.e2e_steps,
            "per_rank_ms": ranks, "numa": numa,
            "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
            "note": f"pinned host buffers; each step H2D of Q/K/V, fmha_forward and D2H of O "
                    f"over {nsl} batch slices pipelined on three streams"}


if __name__ == "__main__":
    sys.exit(main())
