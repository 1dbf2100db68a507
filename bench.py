#!/usr/bin/env python3
"""Benchmark of the two trellis hot paths on B200: encode and codes-only scan.

Workload (N=1 default): the 1,000,000-row x 10,000-query flat MIPS scan at
d=128 -- non-negative heavy-tailed integer rows (about 40% zeros, the rest
geometric with mean 20, clipped at 255) cast to f32 and mean-centered by the
base mean, 2 bits per coordinate, trellis memory M=8, top-100 (top-10 is also
reported).  Seeded synthetic data stand in for the public corpora.

One step = one pass of both hot paths over the resident inputs:
  encode   every base row -> codes-only trellis records (the index build),
  scan     every query against every record, per-query top-100 by MIPS score.
`value` is queries/s of the scan phase; `encode.value` is rows/s of the
encode phase; `ms_per_step` covers both.  With N GPUs the base is sharded in
contiguous row ranges (strong scaling: same 1M x 10k job), every rank scans
its shard for all queries; the ranks share one threshold from their
first-pass bounds (one NCCL all-gather), exchange their packed lists by
query slice (all-to-all), merge a slice each on the device and all-gather
the merged slices.

`--impl reference` times the CPU restatement of the reference algorithm
(oracle/, OpenMP over queries, all host threads) on a bounded sample of the
same workload.
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
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

DIM, BITS, MEM = 128, 2, 8
N_BASE, N_QUERY = 1_000_000, 10_000
K_MAIN, K_ALT = 100, 10
FP32_LANES_PER_SM = 128  # FP32 FMA lanes per SM on sm_100
# DRAM bytes (read + write) per launch of the two tensor-core passes at the
# bench workload (1M records x 10k queries), from one ncu capture of the
# dram__bytes_read.sum and dram__bytes_write.sum metrics; pass 1 as if it
# bounded every tile (the bench scales it by the fraction it bounds, and
# both by the records of the shard: the operand rows stream once per pass).
# A measurement, not recomputed at run time.
TC_TRAFFIC_PASS1 = 4 * 135.5e6
TC_TRAFFIC_PASS2 = 328.7e6


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--n-base", type=int, default=N_BASE)
    ap.add_argument("--n-query", type=int, default=N_QUERY)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--workload", choices=["flat", "wide", "ivf", "encode-sweep", "candidates",
                                           "shortlist", "coset"],
                    default="flat",
                    help="flat: the headline 1M x 10k d=128 MIPS step (the default line); the "
                         "others measure the remaining configurations, one JSON line each")
    ap.add_argument("--cell", default=None, metavar="BITS,MEM",
                    help="encode-sweep: run this one cell only (e.g. 2,16)")
    ap.add_argument("--rows", type=int, default=0,
                    help="encode-sweep: rows per cell (0: sized to about a second)")
    ap.add_argument("--tune", action="append", default=[], metavar="KEY=VALUE",
                    help="uv_set_tuning before the run (launch shapes and samples; results "
                         "never depend on them), e.g. --tune tc_hot=1")
    ap.add_argument("--scan", choices=["auto", "exact", "tc"], default="auto",
                    help="auto: tensor-core prefilter where it is built; exact: the CUDA-core "
                         "kernel only; tc: prefilter wherever it is built")
    return ap.parse_args()


# ------------------------------------------------------------------ data ---

def make_data(n_base: int, n_query: int, seed: int = 0):
    """Heavy-tailed integer rows in [0, 255]: P(0) = 0.4, else geometric(1/20)
    clipped at 255; base mean (f64) subtracted from base and queries in f32."""
    rng = np.random.default_rng(seed)
    out = np.empty((n_base + n_query, DIM), np.float32)
    step = 131072
    for a in range(0, n_base + n_query, step):
        b = min(a + step, n_base + n_query)
        zero = rng.random((b - a, DIM)) < 0.4
        geo = np.minimum(rng.geometric(1.0 / 20.0, (b - a, DIM)), 255)
        out[a:b] = np.where(zero, 0, geo).astype(np.float32)
    base, query = out[:n_base], out[n_base:]
    mean = base.mean(axis=0, dtype=np.float64).astype(np.float32)
    base -= mean
    query -= mean
    return base, query


# ---------------------------------------------------------------- clocks ---

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        # the samples go to a private temporary file; the line reports them
        self.path = Path(tempfile.gettempdir()) / f"uvb200_clocks_gpu{gpu_index}_{os.getpid()}.csv"

    def start(self):
        try:
            self.path.parent.mkdir(exist_ok=True)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[4:]))
            except ValueError:
                continue
        if not rows:
            return None
        smax = max(r[1] for r in rows)
        load = [r for r in rows if r[0] > 0.5 * smax] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[2][1:5])
                          if v.strip().lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in load), "sm_max_mhz": smax,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------- reference ---

def run_reference(args, rank: int):
    """CPU restatement of the reference path (oracle/), all host threads."""
    if rank != 0:
        return
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle as O

    threads = O.threads_available()
    base, query = make_data(args.n_base, args.n_query)
    codec = O.Codec(DIM, BITS, MEM)
    t0 = time.time()
    index = codec.encode_batch(base, threads=threads)
    build_s = time.time() - t0
    norms = O.l2_norms(base, threads=threads)
    sample_q = max(threads, 16)
    times = []
    for step in range(args.warmup + args.steps):
        qs = query[(step * sample_q) % len(query):][:sample_q]
        t = time.perf_counter()
        codec.search_topk(index, qs, K_MAIN, norms=norms, threads=threads)
        dt = time.perf_counter() - t
        if step >= args.warmup:
            times.append(dt)
    qps = sample_q * len(times) / sum(times)
    line = {
        "impl": "reference", "metric": METRIC, "value": qps, "unit": "queries/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * sum(times) / len(times), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(args),
        "encode": {"value": args.n_base / build_s, "unit": "rows/s",
                   "note": "one untimed-by-steps build of the full base"},
        "cpu_baseline": {"value": qps, "unit": "queries/s", "cores": threads, "kind": "port",
                         "sample": f"{sample_q} queries x {args.n_base} records per step"},
        "e2e": {"value": qps, "unit": "queries/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ ours ---

METRIC = "flat codes-only MIPS queries/s and encode vectors/s at 1/2/4/8 B200; % HBM roofline"


# kernel families of one step (uv_profile_read names)
SCAN_FAMILIES = ("encode", "prep_queries", "flat_scan", "merge_topk", "tc_prepare", "tc_hot",
                 "tc_pass1", "tc_theta", "tc_bounds", "tc_pass2", "tc_rescore", "topk_pack")


def config_dict(args):
    return {"workload": "flat-mips-1Mx10k-d128", "n_base": args.n_base, "n_query": args.n_query,
            "dim": DIM, "bits": BITS, "mem": MEM, "k": K_MAIN, "metric_space": "mips",
            "parallelism": f"shard{args.gpus}", "l2": "flushed between steps (256 MiB write); "
            "base rows 512 MB > L2"}


def main():
    args = parse()
    if args.workload == "ivf" and int(os.environ.get("WORLD_SIZE", "1")) > 1:
        run_ivf_sharded(args)
        return
    if args.workload != "flat":
        run_secondary(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    import torch

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    from ultravec_ann_b200_loader import load

    uv = load()
    dev = torch.device("cuda", local)

    base_np, query_np = make_data(args.n_base, args.n_query)
    lo, hi = rank * args.n_base // world, (rank + 1) * args.n_base // world
    shard = torch.from_numpy(base_np[lo:hi]).to(dev)
    ids = torch.arange(lo, hi, dtype=torch.int64, device=dev)
    queries = torch.from_numpy(query_np).to(dev)
    nq = queries.shape[0]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    uv.set_tuning("tc_scan", {"auto": 0, "exact": 1, "tc": 2}[args.scan])
    for kv in args.tune:
        key, val = kv.split("=", 1)
        uv.set_tuning(key, int(val))
    codec = uv.Codec(DIM, BITS, MEM, device=local)
    index = uv.Index(codec)
    index.reserve(hi - lo)

    import ultravec_ann_b200.shard as shardlib

    def sharded(qs, k):
        # the flat multi-GPU protocol: first-pass bounds all-gathered into one
        # shared threshold, packed lists, all-to-all of query slices, per-slice
        # k-way merge, all-gather of the merged slices
        return shardlib.sharded_search(
            lambda n: index.search_begin(qs, k, mips=True, n_shards=n), k, dist,
            lambda i, sc: uv.topk_pack(i, sc, device=local),
            lambda p: uv.topk_unpack(p, device=local),
            lambda recv, rows, nl, kin, kk, rs, ls: uv.topk_merge_packed(
                recv, rows, nl, kin, kk, rs, ls, device=local))

    def scan(k):
        if world == 1:
            return index.search(queries, k, mips=True)
        return sharded(queries, k)

    def step(ev=None):
        index.clear()
        if ev:
            ev[0].record()
        index.add(ids, shard)
        if ev:
            ev[1].record()
        if world > 1:
            # the index is built on every rank before any rank searches it:
            # each phase is timed from a common start, so neither carries the
            # ranks' launch skew
            barrier()
        if ev:
            ev[2].record()
        res = scan(K_MAIN)
        if ev:
            ev[3].record()
        return res

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    barrier()

    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    enc_ms, scan_ms = [], []
    last = None
    for _ in range(args.steps):
        flush.fill_(1)
        barrier()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        last = step(ev)
        torch.cuda.synchronize()
        enc_ms.append(ev[0].elapsed_time(ev[1]))
        scan_ms.append(ev[2].elapsed_time(ev[3]))
    barrier()
    clk = clocks.stop() if clocks else None
    # one more step, untimed, with the library's per-launch event hook on:
    # per-kernel device times and the launches of a step (the hook's event
    # records would otherwise sit inside the timed region)
    uv.profile_enable(True)
    flush.fill_(1)
    barrier()
    step()
    torch.cuda.synchronize()
    kern = {name: tuple(v * args.steps for v in uv.profile_read(name)) for name in SCAN_FAMILIES}
    launches_total = uv.profile_read("*")[1] * args.steps
    tc_candidates = uv.profile_read("tc_candidates")[1]
    tc_sample = max(1, uv.profile_read("tc_sample")[1])
    uv.profile_enable(False)
    barrier()

    # top-10 throughput (same index), timed the same way
    for _ in range(2):  # warm-up of the top-10 shape
        scan(K_ALT)
    k10_ms = []
    for _ in range(max(2, args.steps // 2)):
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        scan(K_ALT)
        e1.record()
        torch.cuda.synchronize()
        k10_ms.append(e0.elapsed_time(e1))

    tot = torch.tensor([sum(enc_ms), sum(scan_ms), sum(k10_ms)], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    enc_tot, scan_tot, k10_tot = tot.tolist()

    # End to end through the public API: pinned host queries in, host results
    # out.  At N=1 the host buffers go straight into uv_index_search (the
    # library stages them); with N ranks each rank copies its queries up, scans
    # its shard, and the merged top-k is read back to the host.
    e2e = None
    if not args.no_e2e:
        q_host = torch.from_numpy(query_np).pin_memory()
        # pinned host results for the sharded path (copied back asynchronously)
        o_ids = torch.empty((nq, K_MAIN), dtype=torch.int64).pin_memory()
        o_sc = torch.empty((nq, K_MAIN), dtype=torch.float32).pin_memory()
        e_ms = []
        h2d = d2h = 0
        for s_i in range(args.warmup + max(2, args.steps // 2)):
            barrier()
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record()
            if world == 1:
                h_ids, h_sc = index.search(q_host, K_MAIN, mips=True)
            else:
                out_ids, out_scores = sharded(q_host.to(dev, non_blocking=True), K_MAIN)
                o_ids.copy_(out_ids, non_blocking=True)
                o_sc.copy_(out_scores, non_blocking=True)
                h_ids, h_sc = o_ids, o_sc
            t1.record()
            torch.cuda.synchronize()
            if s_i >= args.warmup:
                e_ms.append(t0.elapsed_time(t1))
            h2d = int(q_host.numel() * 4)
            d2h = int(h_ids.size * 8 + h_sc.size * 4) if world == 1 else \
                int(h_ids.numel() * 8 + h_sc.numel() * 4)
        et = torch.tensor([sum(e_ms)], dtype=torch.float64, device=dev)
        if dist is not None:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        e2e = {"value": nq * len(e_ms) / (et.item() / 1e3), "unit": "queries/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "api": "uv_index_search with host buffers" if world == 1 else
                      "uv_index_search_begin / set_bounds / finish + NCCL all-gather, "
                      "all-to-all and uv_topk_merge_packed, host copies"}

    # CPU baseline: the oracle on a bounded sample, rank 0 at N=1
    cpu = parity = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu, parity = cpu_baseline(index, base_np, query_np, last)

    if rank == 0:
        qps = nq * args.steps / (scan_tot / 1e3)
        rows_s = args.n_base * args.steps / (enc_tot / 1e3)
        n_local = hi - lo
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        peaks = load_peaks()
        smax = peaks.get("sm_max_mhz", 1965.0)
        rec_bytes = 32 + 1 + 4 + 4
        hbm = peaks.get("hbm_gbs", 6650.0)
        flops = 2.0 * nq * n_local * DIM
        hbm_model = {"bytes_per_query": n_local * rec_bytes,
                     "gbs": qps / world * n_local * rec_bytes / 1e9, "peak_gbs": hbm,
                     "frac": qps / world * n_local * rec_bytes / 1e9 / hbm,
                     "note": "streaming model (every query re-reads its shard); >1 means "
                             "on-chip reuse across the query tile"}
        if kern["tc_pass2"][1] > 0:
            # tensor-core prefilter: the dominant kernels are the two fp16 MMA
            # passes, counted per step (one launch of each): pass 2 does the
            # full Q x N x d contraction, pass 1 the one over every S-th tile
            n_t = (n_local + 191) // 192
            frac1 = ((n_t + tc_sample - 1) // tc_sample) / n_t
            flops_step = flops * (1.0 + frac1)
            steps_tc = max(kern["tc_pass2"][1], 1)
            t_step = (kern["tc_pass1"][0] + kern["tc_pass2"][0]) / steps_tc
            achieved = flops_step / (t_step / 1e3) / 1e12
            peak = peaks.get("bf16_tflops", 1590.0)
            roof = {"bound": "tensor", "kernel": "tc_scan_kernel (pass 1 and pass 2 per step)",
                    "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                    "frac": achieved / peak,
                    "traffic": (TC_TRAFFIC_PASS1 * frac1 + TC_TRAFFIC_PASS2) * n_local / 1e6,
                    "peak_source": "bf16_tflops of MEASURED_PEAKS.json (dense f16 and bf16 "
                                   "tensor peaks are equal)" if "bf16_tflops" in peaks
                                   else "fallback 1.59 PFLOP/s",
                    "flops_per_step": flops_step, "ms_per_step": t_step,
                    "pass1_tile_stride": tc_sample, "hbm_model": hbm_model,
                    "candidates_per_query": tc_candidates / nq}
        else:
            scan_k_ms, scan_k_n = kern["flat_scan"]
            avg_scan = scan_k_ms / max(scan_k_n, 1)
            fp32_peak = sms * FP32_LANES_PER_SM * 2 * smax * 1e6 / 1e12
            achieved = flops / (avg_scan / 1e3) / 1e12
            roof = {"bound": "fp32", "kernel": "flat_scan_kernel", "achieved": achieved,
                    "peak": fp32_peak, "unit": "TFLOP/s", "frac": achieved / fp32_peak,
                    "traffic": None,
                    "peak_source": f"nominal {sms} SMs x {FP32_LANES_PER_SM} FMA/clk x 2 x "
                                   f"{smax:.0f} MHz (sm_max_mhz of MEASURED_PEAKS.json)",
                    "flops_per_launch": flops, "avg_launch_ms": avg_scan,
                    "hbm_model": hbm_model}
        line = {
            "metric": METRIC, "value": qps, "unit": "queries/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": (enc_tot + scan_tot) / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_dict(args),
            "encode": {"value": rows_s, "unit": "rows/s", "ms_per_step": enc_tot / args.steps},
            "scan_ms_per_step": scan_tot / args.steps,
            "top10": {"value": nq * len(k10_ms) / (k10_tot / 1e3), "unit": "queries/s"},
            "roofline": roof,
            "kernels_ms": {k: v[0] / args.steps for k, v in kern.items()},
            "kernels_ms_note": "device ms per step of each kernel family (all its launches), "
                               "from one untimed step with the per-launch event hook on",
            "gpu_launches": launches_total,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "parity": parity,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def load_peaks():
    try:
        return json.loads((REPO / "MEASURED_PEAKS.json").read_text())
    except Exception:
        return {}


def cpu_baseline(index, base_np, query_np, last):
    """The oracle (C restatement of the reference CPU path) on a bounded
    sample: scan of a few queries over the full index, all host threads.

    The same sample is the parity check of the measured configuration: the
    oracle's top-100 ids and score bits for those queries, over the GPU's
    1M records, against the GPU's answer for them in the last timed step
    (`last`), and the oracle's encoding of the first 8,192 rows against the
    GPU's records byte for byte (codes, start states, rescale bits)."""
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle as O

    threads = O.threads_available()
    ex = index.export()
    rec = {"codes": ex["codes"], "start": ex["start"], "rescale": ex["rescale"]}
    oc = O.Codec(DIM, BITS, MEM)
    sample = max(16, threads)
    qs = query_np[:sample]
    oc.search_topk(rec, qs[:threads], K_MAIN, norms=ex["norms"], threads=threads)  # warm
    t = time.perf_counter()
    wids, wsc = oc.search_topk(rec, qs, K_MAIN, norms=ex["norms"], threads=threads)
    dt = time.perf_counter() - t
    enc_rows = 8192
    t = time.perf_counter()
    enc = oc.encode_batch(base_np[:enc_rows], threads=threads)
    de = time.perf_counter() - t
    gids = last[0][:sample].cpu().numpy()
    gsc = last[1][:sample].cpu().numpy()
    norms_ok = bool(np.array_equal(ex["norms"].view(np.uint32),
                                   O.l2_norms(base_np, threads=threads).view(np.uint32)))
    parity = {
        "queries": sample, "records": int(len(ex["start"])), "k": K_MAIN,
        "ids_equal": bool(np.array_equal(gids, wids)),
        "scores_bitequal": bool(np.array_equal(gsc.view(np.uint32), wsc.view(np.uint32))),
        "encode_rows": enc_rows,
        "encode_rows_equal": bool(
            np.array_equal(ex["codes"][:enc_rows], enc["codes"])
            and np.array_equal(ex["start"][:enc_rows], enc["start"])
            and np.array_equal(ex["rescale"][:enc_rows].view(np.uint32),
                               enc["rescale"].view(np.uint32))),
        "norms_bitequal": norms_ok,
        "oracle": "C restatement of the reference CPU path (oracle/), same inputs",
    }
    cpu = {"value": sample / dt, "unit": "queries/s", "cores": threads, "kind": "port",
           "sample": f"{sample} queries x {len(ex['start'])} records (scan); encode {enc_rows} "
                     f"rows",
           "encode_rows_s": enc_rows / de}
    return cpu, parity


# ------------------------------------------------------ other workloads ---

def ivf_data(rng, n, nq, d, d_pad):
    """The IVF corpus: 64 unit Gaussian centres + 0.3 N(0,1), renormalized,
    zero-padded from d to d_pad; base rows then queries."""
    c = rng.standard_normal((64, d)).astype(np.float32)
    c /= np.linalg.norm(c, axis=1, keepdims=True)
    x = np.zeros((n + nq, d_pad), np.float32)
    for a in range(0, n + nq, 50_000):
        b = min(a + 50_000, n + nq)
        v = c[rng.integers(0, 64, b - a)] + np.float32(0.3) * \
            rng.standard_normal((b - a, d), dtype=np.float32)
        x[a:b, :d] = v / np.linalg.norm(v, axis=1, keepdims=True)
    return x


def run_ivf_sharded(args):
    """The IVF workload on N GPUs (torchrun, one rank per GPU, NCCL): every
    rank computes the same k-means and assignment, owns the posting lists
    dealt to it by record bytes (shard.ivf_list_owners) and builds an IVF
    index of its rows (global ids); per search, each rank probes its query
    slice, the lists are shared by one all-gather, every rank scans the
    probed lists it owns, and the packed per-rank top-10 lists combine by an
    all-to-all of query slices, device merges and one all-gather
    (shard.ivf_sharded_search).  Device time per search is the max over
    ranks."""
    import datetime

    import torch
    import torch.distributed as dist

    world = int(os.environ["WORLD_SIZE"])
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    from ultravec_ann_b200_loader import load

    uv = load()
    import ultravec_ann_b200.shard as shard

    dev = torch.device("cuda", local)
    n, nq, d, d_pad, nlist = 1_000_000, 10_000, 1536, 2048, 4096
    x = ivf_data(np.random.default_rng(0), n, nq, d, d_pad)
    base = torch.from_numpy(x[:n]).to(dev)
    qs = torch.from_numpy(x[n:]).to(dev)
    del x
    cen = uv.kmeans(base, nlist, seed=42, iters=5, device=local)
    asg = uv.ivf_assign(base, cen, device=local)
    asg_np = asg.cpu().numpy() if hasattr(asg, "cpu") else np.asarray(asg)
    owners = shard.ivf_list_owners(np.bincount(asg_np, minlength=nlist), world)
    rows = shard.ivf_owned_rows(asg_np, owners, rank)
    rows_t = torch.from_numpy(rows).to(dev)
    codec = uv.Codec(d_pad, 2, 8, device=local)
    ivf = uv.IvfIndex(codec, cen, centered=True)
    ivf.build(base.index_select(0, rows_t), assign=asg.index_select(0, rows_t.to(asg.device))
              if hasattr(asg, "index_select") else asg_np[rows],
              ids=rows_t.to(torch.int64))
    del base

    def search(nprobe):
        # the probe split by query slices and shared by one all-gather; every
        # rank scans the probed lists it holds; packed lists, all-to-all of
        # query slices, per-slice merges, all-gather of the merged slices
        return shard.ivf_sharded_search(
            ivf, qs, 10, nprobe, dist,
            lambda i, sc: uv.topk_pack(i, sc, device=local),
            lambda p: uv.topk_unpack(p, device=local),
            lambda recv, rows, nl, kin, kk, rs, ls: uv.topk_merge_packed(
                recv, rows, nl, kin, kk, rs, ls, device=local))

    for nprobe in (1, 4, 16, 64):
        search(nprobe)
        best = float("inf")
        for _ in range(3):
            torch.cuda.synchronize()
            dist.barrier()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            search(nprobe)
            b.record()
            torch.cuda.synchronize()
            t = torch.tensor([a.elapsed_time(b)], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            best = min(best, t.item())
        if rank == 0:
            print(json.dumps({"metric": METRIC, "workload": "ivf-1Mx10k-d2048-nlist4096",
                              "n_gpus": world, "data": "synthetic", "nprobe": nprobe,
                              "value": nq / best * 1e3, "unit": "queries/s",
                              "higher_is_better": True, "scaling": "strong",
                              "queries_s": nq / best * 1e3, "search_ms": best,
                              "centered": True, "k": 10, "bits": 2, "mem": 8,
                              "parallelism": f"lists dealt by bytes over {world} ranks",
                              "rows_per_rank": int(len(rows))}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def _timed(fn, reps):
    """Device time of fn() in ms (CUDA events), best of reps after one warm-up."""
    import torch

    fn()
    best = float("inf")
    for _ in range(reps):
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        best = min(best, a.elapsed_time(b))
    return best


def run_secondary(args):
    """One GPU; prints one JSON line per configuration:
    wide          1M rows, d=960 padded to 1024, x_ij = U[0,1) + 0.5 j / 959,
                  b in {1, 2, 4}, M=8: encode rows/s and 1k-query top-10 MIPS
                  (the tensor-core prefilter with K streamed in chunks)
    ivf           1M rows, d=1536 padded to 2048: 64 unit Gaussian centres +
                  0.3 N(0,1), renormalized; k-means nlist=4096 (seed 42, 5
                  rounds), centered lists, b=2, M=8; 10k-query top-10 at
                  nprobe 1/4/16/64
    encode-sweep  1M rows (a 100k prefix at M=12, 10k at M=16), d=128 N(0,1),
                  b=2, M in {2, 4, 8, 12, 16}: encode rows/s
    candidates    1M rows d=128 N(0,1), b=2, M=8; 10k prepared queries with
                  256 uniformly random candidate positions each (a batched
                  graph-walk expansion): candidates scored per second
    shortlist     the flat workload's rows (1M x 128 heavy-tailed integers,
                  mean-removed), b=2, M=8: IVF nlist=1024 (k-means seed 42, 5
                  rounds), 10k queries top-10 with the 1-bit shortlist
                  (Hamming stage 1) at C in {128, 256, 512}, nprobe in
                  {1, 8, 32, 128}, beside the plain codes scan; and the flat
                  shortlist at C = 512 over all 1M rows (1k queries)
    coset         the coset trellis (E8 cosets, 4-branch Viterbi), N(0,1)
                  rows, b=2: the reference's research cells (d=128 5k rows
                  and d=960 padded to 1024 20k rows, M=16, 500 queries
                  top-10) and a throughput cell (d=128, 200k rows, the
                  default M=12, 1k queries); encode rows/s, queries/s, and
                  the oracle's rates on a bounded sample of each cell"""
    import torch

    from ultravec_ann_b200_loader import load

    uv = load()
    uv.set_tuning("tc_scan", {"auto": 0, "exact": 1, "tc": 2}[args.scan])
    for kv in args.tune:
        key, val = kv.split("=", 1)
        uv.set_tuning(key, int(val))
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(0)

    def emit(workload, extra):
        line = {"metric": METRIC, "workload": workload, "n_gpus": 1, "data": "synthetic"}
        line.update(extra)
        print(json.dumps(line), flush=True)

    if args.workload == "wide":
        run_wide(uv, dev, emit, rng)
    elif args.workload == "ivf":
        run_ivf(uv, dev, emit, rng, args)
    elif args.workload == "shortlist":
        n, nq, nlist = 1_000_000, 10_000, 1024
        base_np, query_np = make_data(n, nq)
        base = torch.from_numpy(base_np).to(dev)
        qs = torch.from_numpy(query_np).to(dev)
        cen = uv.kmeans(base, nlist, seed=42, iters=5)
        codec = uv.Codec(DIM, 2, 8)
        plain = uv.IvfIndex(codec, cen, centered=False)
        plain.build(base)
        arms = {}
        for c in (128, 256, 512):
            arms[c] = uv.IvfIndex(codec, cen, centered=False)
            arms[c].set_shortlist(c)
            arms[c].build(base)
        for nprobe in (1, 8, 32, 128):
            ms = _timed(lambda: plain.search(qs, 10, nprobe), 3)
            ref_ids = plain.search(qs, 10, nprobe)[0].cpu().numpy()
            emit("ivf-shortlist-1Mx10k-d128-nlist1024", {
                "arm": "codes", "nprobe": nprobe, "queries_s": nq / ms * 1e3, "search_ms": ms,
                "k": 10, "bits": 2, "mem": 8})
            for c, sl in arms.items():
                ms = _timed(lambda: sl.search(qs, 10, nprobe), 3)
                ids = sl.search(qs, 10, nprobe)[0].cpu().numpy()
                agree = float(np.mean([len(set(ids[q]) & set(ref_ids[q])) / 10
                                       for q in range(0, nq, 10)]))
                uv.profile_enable(True)
                sl.search(qs, 10, nprobe)
                torch.cuda.synchronize()
                kern = round(uv.profile_read("shortlist")[0], 3)
                uv.profile_enable(False)
                emit("ivf-shortlist-1Mx10k-d128-nlist1024", {
                    "arm": f"shortlist_c{c}", "nprobe": nprobe, "queries_s": nq / ms * 1e3,
                    "search_ms": ms, "kernel_ms": kern, "top10_agreement_with_codes": agree,
                    "k": 10, "bits": 2, "mem": 8})
        flat = uv.Index(codec)
        flat.set_shortlist(512)
        flat.add_batch(base)
        q1k = qs[:1000]
        ms = _timed(lambda: flat.search(q1k, 10), 2)
        emit("flat-shortlist-1Mx1k-d128", {"c": 512, "queries_s": 1000 / ms * 1e3,
                                           "search_ms": ms, "k": 10, "bits": 2, "mem": 8})
    elif args.workload == "candidates":
        n, nq, per_q, d = 1_000_000, 10_000, 256, 128
        base = torch.from_numpy(rng.standard_normal((n, d), dtype=np.float32)).to(dev)
        qs = torch.from_numpy(rng.standard_normal((nq, d), dtype=np.float32)).to(dev)
        codec = uv.Codec(d, 2, 8)
        index = uv.Index(codec)
        index.add_batch(base)
        pos = torch.from_numpy(rng.integers(0, n, nq * per_q).astype(np.int64)).to(dev)
        off = torch.arange(nq + 1, dtype=torch.int64, device=dev) * per_q
        prep_ms = _timed(lambda: index.prepare(qs).close(), 3)
        prep = index.prepare(qs)
        ms = _timed(lambda: prep.score(pos, off), 5)
        uv.profile_enable(True)
        prep.score(pos, off)
        torch.cuda.synchronize()
        kern_ms = uv.profile_read("score_candidates")[0]
        uv.profile_enable(False)
        # algorithmic bytes per candidate: 32 code bytes + start, rescale, rnorm
        # (4 each) + position (8) + score (4)
        per_cand = 32 + 4 + 4 + 4 + 8 + 4
        ncand = nq * per_q
        emit("candidates-1M-d128-10kx256", {
            "candidates_s": ncand / ms * 1e3, "score_ms": ms, "kernel_ms": kern_ms,
            "prepare_ms": prep_ms, "bytes_per_candidate": per_cand,
            "achieved_gbs": ncand * per_cand / (kern_ms * 1e-3) / 1e9, "bits": 2, "mem": 8})
    elif args.workload == "coset":
        sys.path.insert(0, str(REPO / "oracle"))
        import oracle as O  # the CPU oracle: the timed CPU baseline only

        threads = os.cpu_count() or 1
        for name, d, mem, n, nq in (("coset-sift-d128-b2-M16-5k", 128, 16, 5_000, 500),
                                    ("coset-gist-d1024-b2-M16-20k", 1024, 16, 20_000, 500),
                                    ("coset-d128-b2-M12-200k", 128, 12, 200_000, 1000)):
            rows = rng.standard_normal((n + nq, d), dtype=np.float32)
            base = torch.from_numpy(rows[:n]).to(dev)
            qs = torch.from_numpy(rows[n:]).to(dev)
            enc_ms = float("inf")
            for rep in range(3):  # a fresh index each time; the first is warm-up
                ix = uv.CosetIndex(d, 2, mem=mem)
                torch.cuda.synchronize()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                ix.add_batch(base)
                b.record()
                torch.cuda.synchronize()
                if rep > 0:
                    enc_ms = min(enc_ms, a.elapsed_time(b))
            scan_ms = _timed(lambda: ix.search(qs, 10), 3)
            uv.profile_enable(True)
            ix2 = uv.CosetIndex(d, 2, mem=mem)
            ix2.add_batch(base)
            ix2.search(qs, 10)
            torch.cuda.synchronize()
            del ix2
            kern = {f: round(uv.profile_read(f)[0], 3)
                    for f in ("coset_prep", "coset_nearest", "coset_viterbi", "prep_queries",
                              "coset_scan", "merge_topk")}
            uv.profile_enable(False)
            # the oracle on a bounded sample of the same cell
            oc = O.Coset(d, 2, mem=mem)
            ns = 64 if d > 256 else 256
            t0 = time.perf_counter()
            enc = oc.encode_batch(rows[:ns])
            cpu_enc = ns / (time.perf_counter() - t0)
            big = {k: np.concatenate([v] * (n // ns)) for k, v in enc.items()}
            t0 = time.perf_counter()
            oc.search(big, rows[n:n + 16], 10)
            cpu_q = 16 / (time.perf_counter() - t0)
            emit(name, {"bits": 2, "mem": mem, "dim": d, "rows": n, "queries": nq, "k": 10,
                        "encode_rows_s": n / enc_ms * 1e3, "encode_ms": enc_ms,
                        "queries_s": nq / scan_ms * 1e3, "search_ms": scan_ms,
                        "kernels_ms": kern,
                        "cpu_baseline": {"encode_rows_s": cpu_enc, "queries_s": cpu_q,
                                         "cores": threads, "kind": "port",
                                         "sample": f"encode {ns} rows; search 16 queries over "
                                                   f"{(n // ns) * ns} records"}})
            del ix, oc, enc, big
    else:
        run_encode_sweep(uv, dev, emit, args)

def _tc_roofline(uv, flops_full, nq_tiles_flops, peaks):
    """Tensor-pipe roofline of the prefilter passes of the last profiled
    search: pass 2 does the full contraction, pass 1 the one over every S-th
    tile."""
    p1 = uv.profile_read("tc_pass1")
    p2 = uv.profile_read("tc_pass2")
    s_ = max(1, uv.profile_read("tc_sample")[1])
    if p2[1] == 0:
        return None
    flops = flops_full * (1.0 + 1.0 / s_)
    t = (p1[0] + p2[0]) / p2[1]
    peak = peaks.get("bf16_tflops", 1590.0)
    ach = flops / (t / 1e3) / 1e12
    return {"bound": "tensor", "kernel": "tc_wide_kernel (pass 1 and pass 2 per search)",
            "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
            "flops_per_search": flops, "ms_per_search": t, "pass1_tile_stride": s_,
            "peak_source": "bf16_tflops of MEASURED_PEAKS.json" if "bf16_tflops" in peaks
            else "fallback 1.59 PFLOP/s", "traffic": None}


def _e2e_host(fn, q_host, reps=3):
    """Search timed end to end with host buffers (pinned queries in, host
    results out), best of reps after one warm-up, in ms."""
    import torch

    fn(q_host)
    best = float("inf")
    for _ in range(reps):
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn(q_host)
        b.record()
        torch.cuda.synchronize()
        best = min(best, a.elapsed_time(b))
    return best


def run_wide(uv, dev, emit, rng):
    """1M rows, d=960 padded to 1024, x_ij = U[0,1) + 0.5 j / 959, b in {1,
    2, 4}, M=8: encode rows/s and 1k-query top-10 MIPS (the tensor-core
    prefilter with K streamed in chunks), with the oracle's top-10 for 16
    of the queries over the full GPU index and its encoding of 512 rows as
    the parity check and CPU baseline."""
    import torch

    sys.path.insert(0, str(REPO / "oracle"))
    import oracle as O  # the CPU oracle: baseline and checker only

    threads = O.threads_available()
    peaks = load_peaks()
    n, nq, d, d_pad = 1_000_000, 1000, 960, 1024
    x = np.zeros((n + nq, d_pad), np.float32)
    for a in range(0, n + nq, 100_000):
        b = min(a + 100_000, n + nq)
        x[a:b, :d] = rng.random((b - a, d), dtype=np.float32) + \
            np.float32(0.5) * (np.arange(d, dtype=np.float32) / np.float32(959))
    base = torch.from_numpy(x[:n]).to(dev)
    qs = torch.from_numpy(x[n:]).to(dev)
    q_host = torch.from_numpy(x[n:]).pin_memory()
    for bits in (1, 2, 4):
        codec = uv.Codec(d_pad, bits, 8)
        index = uv.Index(codec)
        index.reserve(n)
        enc_ms = _timed(lambda: (index.clear(), index.add_batch(base)), 2)
        clocks = ClockSampler(0)
        clocks.start()
        scan_ms = _timed(lambda: index.search(qs, 10, mips=True), 3)
        clk = clocks.stop()
        uv.profile_enable(True)
        ids, scores = index.search(qs, 10, mips=True)
        torch.cuda.synchronize()
        kern = {f: round(uv.profile_read(f)[0], 3) for f in SCAN_FAMILIES}
        roof = _tc_roofline(uv, 2.0 * nq * n * d_pad, None, peaks)
        launches = uv.profile_read("*")[1]
        uv.profile_enable(False)
        e2e_ms = _e2e_host(lambda q: index.search(q, 10, mips=True), q_host)
        ex = index.export()
        oc = O.Codec(d_pad, bits, 8)
        rec = {"codes": ex["codes"], "start": ex["start"], "rescale": ex["rescale"]}
        sample = max(16, threads)
        t0 = time.perf_counter()
        wids, wsc = oc.search_topk(rec, x[n:n + sample], 10, norms=ex["norms"], threads=threads)
        cpu_q = sample / (time.perf_counter() - t0)
        t0 = time.perf_counter()
        enc = oc.encode_batch(x[:512], threads=threads)
        cpu_enc = 512 / (time.perf_counter() - t0)
        gi, gs = ids[:sample].cpu().numpy(), scores[:sample].cpu().numpy()
        parity = {"queries": sample, "records": n, "k": 10,
                  "ids_equal": bool(np.array_equal(gi, wids)),
                  "scores_bitequal": bool(np.array_equal(gs.view(np.uint32),
                                                         wsc.view(np.uint32))),
                  "encode_rows": 512,
                  "encode_rows_equal": bool(np.array_equal(ex["codes"][:512], enc["codes"])
                                            and np.array_equal(ex["start"][:512],
                                                               enc["start"]))}
        emit("wide-1Mx1k-d1024", {
            "bits": bits, "mem": 8, "value": nq / scan_ms * 1e3, "unit": "queries/s",
            "queries_s": nq / scan_ms * 1e3, "scan_ms": scan_ms,
            "encode_rows_s": n / enc_ms * 1e3, "encode_ms": enc_ms, "k": 10, "mips": True,
            "kernels_ms": kern, "gpu_launches": launches, "roofline": roof,
            "e2e": {"value": nq / e2e_ms * 1e3, "unit": "queries/s",
                    "h2d_bytes_per_step": nq * d_pad * 4, "d2h_bytes_per_step": nq * 10 * 12,
                    "api": "uv_index_search with host buffers"},
            "cpu_baseline": {"value": cpu_q, "unit": "queries/s", "cores": threads,
                             "kind": "port", "sample": f"{sample} queries x {n} records; "
                                                       f"encode 512 rows",
                             "encode_rows_s": cpu_enc},
            "parity": parity, "clocks": clk,
            "l2": "1M records of 137-521 B exceed L2 at b >= 2"})
        del index, codec


def run_ivf(uv, dev, emit, rng, args=None):
    """1M rows, d=1536 padded to 2048: 64 unit Gaussian centres + 0.3 N(0,1),
    renormalized; k-means nlist=4096 (seed 42, 5 rounds), centered lists,
    b=2, M=8; 10k-query top-10 at nprobe 1/4/16/64.  Per nprobe: queries/s,
    the records the probed lists hold per query and the FP32 rate of the list
    scan over them, end to end with host buffers, and the oracle's top-10 for
    16 queries over the GPU's posting lists (parity and CPU baseline)."""
    import torch

    sys.path.insert(0, str(REPO / "oracle"))
    import oracle as O  # the CPU oracle: baseline and checker only

    threads = O.threads_available()
    peaks = load_peaks()
    smax = peaks.get("sm_max_mhz", 1965.0)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    fp32_peak = sms * FP32_LANES_PER_SM * 2 * smax * 1e6
    n, nq, d, d_pad, nlist = 1_000_000, 10_000, 1536, 2048, 4096
    if args is not None and args.n_base != N_BASE:  # a smaller case (profiling)
        n, nq = args.n_base, args.n_query
        nlist = max(256, min(4096, n // 244))
    x = ivf_data(rng, n, nq, d, d_pad)
    base = torch.from_numpy(x[:n]).to(dev)
    qs = torch.from_numpy(x[n:]).to(dev)
    q_np = x[n:].copy()
    del x
    q_host = torch.from_numpy(q_np).pin_memory()
    t0 = time.time()
    cen = uv.kmeans(base, nlist, seed=42, iters=5)
    torch.cuda.synchronize()
    km_s = time.time() - t0
    codec = uv.Codec(d_pad, 2, 8)
    ivf = uv.IvfIndex(codec, cen, centered=True)
    t0 = time.time()
    ivf.build(base)
    torch.cuda.synchronize()
    build_s = time.time() - t0
    del base
    ex = ivf.export()
    sizes = np.diff(ex["list_off"])
    list_stats = {"mean": float(sizes.mean()), "max": int(sizes.max()),
                  "p99": float(np.percentile(sizes, 99)), "empty": int((sizes == 0).sum())}
    cen_np = cen.cpu().numpy() if hasattr(cen, "cpu") else np.asarray(cen)
    oc = O.Codec(d_pad, 2, 8)
    lists = {"codes": ex["codes"], "start": ex["start"], "rescale": ex["rescale"],
             "rnorm": ex["rnorm"]}
    fams = ("prep_queries", "ivf_cosine", "ivf_select", "ivf_bucket", "ivf_pair_qm",
            "ivf_scan", "merge_topk", "ivf_tc_prepare", "ivf_tc_pairs", "ivf_tc_scan",
            "ivf_tc_select")
    kpad = (d_pad + 63) // 64 * 64
    sample = max(16, threads)
    for nprobe in (1, 4, 16, 64):
        clocks = ClockSampler(0)
        clocks.start()
        ms = _timed(lambda: ivf.search(qs, 10, nprobe), 3)
        clk = clocks.stop()
        uv.profile_enable(True)
        ids, scores = ivf.search(qs, 10, nprobe)
        torch.cuda.synchronize()
        kern = {f: round(uv.profile_read(f)[0], 3) for f in fams}
        launches = uv.profile_read("*")[1]
        exact = uv.profile_read("tc_candidates")[1]
        store_full, over_cand = uv.profile_read("ivf_tc_overflow")
        uv.profile_enable(False)
        probed = ivf.probe(qs, nprobe)
        probed = probed.cpu().numpy() if hasattr(probed, "cpu") else np.asarray(probed)
        scanned = float(np.where(probed >= 0, sizes[np.maximum(probed, 0)], 0).sum()) / nq
        flops = 2.0 * scanned * nq * d_pad
        tc_ms = kern["ivf_tc_scan"]
        if tc_ms > 0:
            # tc_ivf_kernel: per item (list, <= 128 pairs, <= 512 records) the
            # range's fp16 record rows and bound constants once, the pairs'
            # fp16 query rows once per 256-record tile
            pairs = np.bincount(probed[probed >= 0].ravel(), minlength=nlist).astype(np.float64)
            ranges = np.maximum(1, np.ceil(sizes / 512.0))
            groups = np.ceil(pairs / 128.0)
            tiles = np.ceil(np.minimum(sizes, 512) / 256.0)
            alg_bytes = float((groups * sizes * (kpad * 2 + 32)).sum()
                              + (pairs * ranges * tiles * kpad * 2).sum())
            roof = {"bound": "hbm", "kernel": "tc_ivf_kernel (IVF list scan, fp16 bounds)",
                    "achieved": alg_bytes / (tc_ms / 1e3) / 1e9,
                    "peak": peaks.get("hbm_gbs"), "unit": "GB/s",
                    "frac": alg_bytes / (tc_ms / 1e3) / 1e9 / peaks["hbm_gbs"]
                    if peaks.get("hbm_gbs") else None,
                    "bytes_per_search": alg_bytes, "scan_ms": tc_ms,
                    "useful_tflops": flops / (tc_ms / 1e3) / 1e12,
                    "tensor_frac_of_bf16_peak": flops / (tc_ms / 1e3) / 1e12
                    / peaks["bf16_tflops"] if peaks.get("bf16_tflops") else None,
                    "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)",
                    "traffic": None}
        else:
            scan_ms = kern["ivf_scan"]
            roof = {"bound": "fp32", "kernel": "chunked_scan_kernel (IVF list scan)",
                    "achieved": flops / (scan_ms / 1e3) / 1e12 if scan_ms > 0 else None,
                    "peak": fp32_peak / 1e12, "unit": "TFLOP/s",
                    "frac": flops / (scan_ms / 1e3) / fp32_peak if scan_ms > 0 else None,
                    "flops_per_search": flops, "scan_ms": scan_ms,
                    "peak_source": f"nominal {sms} SMs x {FP32_LANES_PER_SM} FMA x 2 x "
                                   f"{smax:.0f} MHz", "traffic": None}
        e2e_ms = _e2e_host(lambda q: ivf.search(q, 10, nprobe), q_host)
        t0 = time.perf_counter()
        wids, wsc = oc.ivf_search_topk(cen_np, ex["list_off"], ex["ids"], lists, True,
                                       q_np[:sample], nprobe, 10, threads=threads)
        cpu_q = sample / (time.perf_counter() - t0)
        gi, gs = ids[:sample].cpu().numpy(), scores[:sample].cpu().numpy()
        emit("ivf-1Mx10k-d2048-nlist4096" if n == 1_000_000 and nq == 10_000 else
             f"ivf-{n}x{nq}-d2048-nlist{nlist}", {
            "nprobe": nprobe, "value": nq / ms * 1e3, "unit": "queries/s",
            "queries_s": nq / ms * 1e3, "search_ms": ms, "kmeans_s": km_s,
            "build_s": build_s, "centered": True, "k": 10, "bits": 2, "mem": 8,
            "kernels_ms": kern, "gpu_launches": launches, "list_sizes": list_stats,
            "records_scanned_per_query": scanned,
            "records_scored_exactly_per_query": exact / nq if tc_ms > 0 else scanned,
            "tc_overflow": {"store_full": bool(store_full), "queries_over_candidates":
                            int(over_cand)} if tc_ms > 0 else None,
            "roofline": roof,
            "e2e": {"value": nq / e2e_ms * 1e3, "unit": "queries/s",
                    "h2d_bytes_per_step": nq * d_pad * 4, "d2h_bytes_per_step": nq * 10 * 12,
                    "api": "uv_ivf_search with host buffers"},
            "cpu_baseline": {"value": cpu_q, "unit": "queries/s", "cores": threads,
                             "kind": "port", "sample": f"{sample} queries over the GPU's "
                                                       f"posting lists"},
            "parity": {"queries": sample, "k": 10,
                       "ids_equal": bool(np.array_equal(gi, wids)),
                       "scores_bitequal": bool(np.array_equal(gs.view(np.uint32),
                                                              wsc.view(np.uint32)))},
            "clocks": clk})


def run_encode_sweep(uv, dev, emit, args):
    """The trellis-memory sweep: 1M rows d=128 N(0,1) from seed 1 (a prefix
    where a cell would take more than about a second), b = 2 at M in {2, 4,
    8, 12, 16} and the reference's whole 2-, 3- and 4-bit ladder M = 4..16
    (its encode-cost table).  Per cell: encode rows/s (CUDA events, best of
    two after a warm-up), the FP32/ALU lane operations of the add-compare-
    select against the SMs' issue rate, the direction fidelity of the
    reconstructions, the oracle's rate on a bounded sample with all host
    threads, and that sample's records compared byte for byte."""
    import torch

    sys.path.insert(0, str(REPO / "oracle"))
    import oracle as O  # the CPU oracle: baseline and checker only

    threads = O.threads_available()
    d = 128
    rows = np.random.default_rng(1).standard_normal((1_000_000, d), dtype=np.float32)
    base = torch.from_numpy(rows).to(dev)
    peaks = load_peaks()
    smax = peaks.get("sm_max_mhz", 1965.0)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    cells = [(2, 2)] + [(b, m) for b in (2, 3, 4) for m in (4, 6, 8, 10, 12, 14, 16)]
    if args.cell:
        cells = [tuple(int(v) for v in args.cell.split(","))]
    for bits, mem in cells:
        w = mem + bits
        n = int(min(1_000_000, max(2000, 2e11 / (d * 2 ** w))))
        if args.rows > 0:
            n = min(args.rows, 1_000_000)
        codec = uv.Codec(d, bits, mem)
        index = uv.Index(codec)
        index.reserve(n)
        sub = base[:n]
        clocks = ClockSampler(dev.index if dev.index is not None else 0)
        clocks.start()
        ms = _timed(lambda: (index.clear(), index.add_batch(sub)), 2)
        clk = clocks.stop()
        rate = n / ms * 1e3
        # add-compare-select lane operations per row: a subtract, a multiply
        # and an add per window, a compare-select per extra candidate
        ops = d * (3 * 2 ** w + (2 ** bits - 1) * 2 ** mem)
        lane_peak = sms * FP32_LANES_PER_SM * smax * 1e6
        ex = index.export()
        m = min(n, 2000)
        rec = codec.decode(ex["codes"][:m], ex["start"][:m])
        rec = rec / np.maximum(np.linalg.norm(rec, axis=1, keepdims=True), 1e-30)
        unit = rows[:m] / np.linalg.norm(rows[:m], axis=1, keepdims=True)
        fidelity = float(np.mean(np.sum(rec * unit, axis=1)))
        oc = O.Codec(d, bits, mem)
        n_cpu = int(max(threads, min(4096, 2e9 / (d * 2 ** w))))
        t0 = time.perf_counter()
        enc = oc.encode_batch(rows[:n_cpu], threads=threads)
        cpu_rate = n_cpu / (time.perf_counter() - t0)
        same = bool(np.array_equal(ex["codes"][:n_cpu], enc["codes"])
                    and np.array_equal(ex["start"][:n_cpu], enc["start"])
                    and np.array_equal(ex["rescale"][:n_cpu].view(np.uint32),
                                       enc["rescale"].view(np.uint32)))
        emit("encode-sweep-d128", {
            "bits": bits, "mem": mem, "window_bits": w, "rows": n, "encode_rows_s": rate,
            "encode_ms": ms, "encoder": "staged" if (w > 18 or (w >= 15 and bits > 2) or
                                                     mem < bits) else
                                       ("cluster" if w >= 15 else "resident"),
            "roofline": {"bound": "fp32/alu issue", "lane_ops_per_row": ops,
                         "achieved_lane_ops_s": rate * ops, "peak_lane_ops_s": lane_peak,
                         "frac": rate * ops / lane_peak,
                         "peak_source": f"nominal {sms} SMs x {FP32_LANES_PER_SM} lanes x "
                                        f"{smax:.0f} MHz"},
            "direction_fidelity": fidelity,
            "cpu_baseline": {"value": cpu_rate, "unit": "rows/s", "cores": threads,
                             "kind": "port", "sample": f"{n_cpu} rows"},
            "parity": {"rows": n_cpu, "records_equal": same},
            "clocks": clk})
        del index, codec


if __name__ == "__main__":
    main()
