#!/usr/bin/env python3
"""Quantized paged decode-attention benchmark on B200 (the BASELINE metric).

Default workload: Qwen3-4B-shaped batched decode,
36 layers, 32 query heads, 8 KV heads, head_dim 128, 32 sequences per GPU
with contexts ~U[1024, 8192], page size 16, int8 per-token-per-head KV with
fp16 scale, random page permutation.  One step = every sequence appends one
token and attends over its whole cache in every layer.  Weak scaling: the
global batch is 32 x N sequences, LPT-sharded by sequence (no collective).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2|3]
  python bench.py --impl reference ...   # the reference's own CPU path

Prints one JSON line (rank 0).  Timing: CUDA events on the launching
stream, barrier + synchronize around the timed steps, max over ranks.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "quant paged decode-attn KV GB/s (% HBM peak) and seq-steps/s at 1/2/4/8 B200"
HD = 128


def workload(cfg: int) -> dict:
    if cfg == 2:
        return dict(name="cfg2 Qwen3-4B-shaped batched decode, int8 per-token-head KV + fp16 scale",
                    codec=2, layers=36, H=32, HK=8, P=16, batch=32, lo=1024, hi=8192, seed=2,
                    outliers=0)
    if cfg == 3:
        return dict(name="cfg3 Qwen3-4B-shaped batched decode, 4-bit KV groups of 32 (fp16 range+min), "
                         "1% K outlier channels x8", codec=4, layers=36, H=32, HK=8, P=16, batch=64, lo=4096,
                    hi=16384, seed=3, outliers=10)
    raise SystemExit(f"unknown --config {cfg}")


def kv_bytes(codec: int) -> int:
    return {1: 272, 2: 260, 3: 128, 4: 160}[codec]


def profiled_traffic(cfg: int):
    """DRAM bytes per attention launch (dram__bytes_read + write) from the
    committed ncu capture of the same kernel on this workload's shapes, or
    None when no capture covers the workload."""
    path = os.path.join(ROOT, "profiles", {2: "attn_kernel_q8head_cfg2_full.md"}.get(cfg, ""))
    if not os.path.isfile(path):
        return None
    with open(path) as f:
        for line in f:
            if line.startswith("traffic_bytes_per_launch:"):
                return {"bytes_per_launch": float(line.split(":", 1)[1]), "source": os.path.relpath(path, ROOT)}
    return None


def peaks() -> tuple:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled while the GPU works."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.rows, self.proc, self.thread = gpu, [], None, None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "100"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.perf_counter(), [x.strip() for x in line.split(",")]))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self, t0: float, t1: float):
        rows = [r for t, r in self.rows if t0 <= t <= t1 and len(r) >= 9]
        if not rows:
            return None
        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": num(rows[0][2]),
                "samples": len(rows), "power_w_max": max((num(r[3]) or 0.0) for r in rows),
                "reasons": sorted(reasons)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    return world, rank, local


def global_lengths(wl: dict, n_gpus: int) -> np.ndarray:
    rng = np.random.default_rng(wl["seed"])
    return rng.integers(wl["lo"], wl["hi"] + 1, size=wl["batch"] * n_gpus).astype(np.int32)


# ---------------------------------------------------------------------------
# reference arm: the reference's own CPU code (oracle/_ref), bounded sample
# ---------------------------------------------------------------------------
def reference_rate(wl: dict, lens: np.ndarray, steps: int, warmup: int, layers_sample: int):
    """Decode steps of the reference CPU path on `lens` over the first
    `layers_sample` layers; returns (seq-steps/s scaled to all layers,
    seconds per sampled step, threads, codec name)."""
    import ctypes as C
    from oracle import oracle as O
    R = O.ref()
    if R is None:
        return None
    codec = 1 if wl["codec"] in (1, 2) else 3  # the reference CPU has only its own codecs
    ids = np.ascontiguousarray(lens, dtype=np.int32)
    h = R.qref_batch_create(codec, ids.size, ids.ctypes.data_as(C.POINTER(C.c_int32)), layers_sample,
                            wl["H"], wl["HK"], HD, steps + warmup + 1, wl["seed"])
    if not h:
        return None
    for _ in range(warmup):
        R.qref_batch_step(h, layers_sample)
    t0 = time.perf_counter()
    for _ in range(steps):
        R.qref_batch_step(h, layers_sample)
    dt = (time.perf_counter() - t0) / steps
    R.qref_batch_destroy(h)
    rate = ids.size / (dt * wl["layers"] / layers_sample)
    return rate, dt, int(R.qref_max_threads()), ("q8_b64_f32" if codec == 1 else "tq35_g64")


def run_reference(args, wl, world, rank):
    if rank != 0:
        return 0
    lens = global_lengths(wl, 1)
    layers_sample = 2
    res = reference_rate(wl, lens, max(1, args.steps), max(0, args.warmup), layers_sample)
    if res is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref (the reference CPU library) is not built"}))
        return 0
    rate, dt, threads, cname = res
    sample = (f"{lens.size} sequences, first {layers_sample} of {wl['layers']} layers per step "
              f"(time scaled x{wl['layers'] / layers_sample:g}), reference codec {cname}")
    line = {"metric": METRIC, "value": rate, "unit": "seq-steps/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * dt * wl["layers"] / layers_sample,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": wl["name"], "global_batch": int(lens.size), "layers": wl["layers"],
                       "query_heads": wl["H"], "kv_heads": wl["HK"], "head_dim": HD, "page_tokens": wl["P"],
                       "parallelism": "host cores (OpenMP over sequence x query head)"},
            "cpu_baseline": {"value": rate, "unit": "seq-steps/s", "cores": threads, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": rate, "unit": "seq-steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args, wl, world, rank, local):
    import torch
    import qwanto_b200 as qb
    from qwanto_b200.sharding import balanced_count_shard

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    glens = global_lengths(wl, world)
    mine = balanced_count_shard(glens, world)[rank]
    lens = glens[mine]
    B, L, H, HK, P = len(lens), wl["layers"], wl["H"], wl["HK"], wl["P"]
    K, W = args.steps, args.warmup
    E = args.e2e_steps
    grow = W + K + E + 2
    max_pages = (int(lens.max()) + grow + P - 1) // P + 1
    total_pages = int(sum((int(c) + grow + P - 1) // P for c in lens)) + 8
    pool = qb.KvPool(wl["codec"], L, HK, P, total_pages, B, max_pages, max_query_heads=H,
                     permutation_seed=1000 + rank, device=local)
    mask = None
    if wl["outliers"]:
        mask = np.zeros((L, HK * HD), np.uint8)
        rng = np.random.default_rng(wl["seed"] + 17)
        for layer in range(L):
            mask[layer, rng.choice(HK * HD, wl["outliers"], replace=False)] = 1
    seed = 1000 * wl["seed"] + rank
    pool.prefill_synthetic(list(range(B)), lens.tolist(), seed, mask, stream)
    torch.cuda.synchronize(dev)

    # per-step inputs, generated on the device for each step's positions
    ring = min(W + K, args.ring)
    ids = torch.arange(B, dtype=torch.int32, device=dev)
    Wq, Wkv = H * HD, HK * HD
    q = torch.empty((ring, L, B, Wq), dtype=torch.float32, device=dev)
    k = torch.empty((ring, L, B, Wkv), dtype=torch.float32, device=dev)
    v = torch.empty((ring, L, B, Wkv), dtype=torch.float32, device=dev)
    mask_dev = None if mask is None else torch.tensor(mask, device=dev)
    for s in range(ring):
        pos = torch.tensor(lens + s, dtype=torch.int32, device=dev)
        for layer in range(L):
            mk = None if mask_dev is None else mask_dev[layer]
            qb.generate_rows(q[s, layer], B, Wq, 1, seed, layer, ids, pos, None, stream)
            qb.generate_rows(k[s, layer], B, Wkv, 2, seed, layer, ids, pos, mk, stream)
            qb.generate_rows(v[s, layer], B, Wkv, 3, seed, layer, ids, pos, None, stream)
    out = torch.empty((L, B, Wq), dtype=torch.float32, device=dev)

    ev_a = [[torch.cuda.Event(enable_timing=True) for _ in range(L)] for _ in range(K)]
    ev_b = [[torch.cuda.Event(enable_timing=True) for _ in range(L)] for _ in range(K)]

    def step(s, timed_idx=None):
        # one decode step: grow every sequence by a token, then per layer one
        # launch that quantizes the new K/V into its page and attends
        r = s % ring
        pool.seq_append(B, None, None, stream)
        for layer in range(L):
            if timed_idx is not None:
                ev_a[timed_idx][layer].record(stream)
            pool.decode(layer, B, H, q[r, layer], out[layer], key=k[r, layer], value=v[r, layer], stream=stream)
            if timed_idx is not None:
                ev_b[timed_idx][layer].record(stream)

    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    for s in range(W):
        step(s)
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    launches0 = qb.launch_count()
    t_wall0 = time.perf_counter()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(K):
        step(W + i, i)
    end.record(stream)
    torch.cuda.synchronize(dev)
    launches = qb.launch_count() - launches0
    if world > 1:
        torch.distributed.barrier()
    ms_total = start.elapsed_time(end)
    # keep the GPU busy (attention only, no growth) so the clock samples cover
    # at least ~1.5 s of this workload
    while time.perf_counter() - t_wall0 < 1.5:
        for layer in range(L):
            pool.decode(layer, B, H, q[0, layer], out[layer], stream=stream)
        torch.cuda.synchronize(dev)
    t_wall1 = time.perf_counter()
    status = pool.check()

    attn_ms = [ev_a[i][l].elapsed_time(ev_b[i][l]) for i in range(K) for l in range(L)]
    attn_avg_ms = float(np.mean(attn_ms))

    # ---- e2e through the host-buffer C-ABI entry (copies inside) ----------
    e2e = None
    if E > 0:
        hq = torch.empty((L, B, Wq), dtype=torch.float32).pin_memory()
        hk = torch.empty((L, B, Wkv), dtype=torch.float32).pin_memory()
        hv = torch.empty((L, B, Wkv), dtype=torch.float32).pin_memory()
        ho = torch.empty((L, B, Wq), dtype=torch.float32).pin_memory()
        hq.copy_(q[0])
        hk.copy_(k[0])
        hv.copy_(v[0])
        torch.cuda.synchronize(dev)
        pool.decode_step_host(L, B, H, hq, hk, hv, ho)  # warm the staging buffers
        if world > 1:
            torch.distributed.barrier()
        t0 = time.perf_counter()
        for _ in range(E):
            pool.decode_step_host(L, B, H, hq, hk, hv, ho)
        e2e_s = (time.perf_counter() - t0) / E
        h2d = (hq.numel() + hk.numel() + hv.numel()) * 4
        d2h = ho.numel() * 4
        e2e = [e2e_s, h2d, d2h]
    sampler.stop()

    # ---- reductions over ranks -------------------------------------------
    t_local = torch.tensor([ms_total, attn_avg_ms, e2e[0] if e2e else 0.0], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t_local, op=torch.distributed.ReduceOp.MAX)
    ms_total, attn_avg_max, e2e_s = t_local.tolist()
    ms_step = ms_total / K
    seq_steps_total = B * world
    value = seq_steps_total / (ms_step / 1000.0)

    # algorithmic bytes for the timed steps, this rank: K/V codes and scales
    # of every attended token and of the appended one, the new K/V rows, the
    # Q and O rows and the page-table entries read
    bkv = kv_bytes(wl["codec"])
    step_bytes, attn_bytes = 0.0, 0.0
    for i in range(K):
        c_after = lens + W + i + 1
        per_layer = float(np.sum(c_after * HK * bkv + HK * bkv + 2 * HK * HD * 4 + 2 * H * HD * 4
                                 + np.ceil(c_after / P) * 4))
        step_bytes += L * per_layer
        attn_bytes += L * per_layer  # the fused launch does append + attention
    step_bytes /= K
    attn_bytes_per_launch = attn_bytes / (K * L)
    peak, peak_kind = peaks()
    achieved = attn_bytes_per_launch / (attn_avg_ms / 1000.0) / 1e9
    kv_gbs = step_bytes * world / (ms_step / 1000.0) / 1e9

    line = None
    if rank == 0:
        clocks = sampler.summary(t_wall0 - 0.05, t_wall1 + 0.05)
        # the capture covers one GPU's full cfg batch; other shapes report none
        traffic = profiled_traffic(args.config) if world == 1 and not args.batch else None
        line = {
            "metric": METRIC, "value": value, "unit": "seq-steps/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8" if wl["codec"] in (1, 2) else "u4", "data": "synthetic",
            "config": {"workload": wl["name"], "global_batch": int(B * world), "per_gpu_batch": int(B),
                       "layers": L, "query_heads": H, "kv_heads": HK, "head_dim": HD, "page_tokens": P,
                       "context": f"U[{wl['lo']},{wl['hi']}] (+{W} warmup tokens)",
                       "mean_context": float(lens.mean()), "parallelism": f"sequence-sharded x{world}",
                       "l2": "inputs larger than L2 (KV bytes per step >> 126 MB)"},
            "kv_gbs": kv_gbs, "hbm_frac_per_gpu": kv_gbs / world / peak,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": (traffic or {}).get("bytes_per_launch"),
                         "traffic_source": (traffic or {}).get("source"),
                         "kernel": "attn_kernel (fused quantize-on-append + split-KV decode attention)",
                         "algorithmic_bytes_per_launch": attn_bytes_per_launch,
                         "avg_launch_ms": attn_avg_ms, "avg_launch_ms_max_rank": attn_avg_max},
            "gpu_launches": int(launches), "status_bits": status,
            "clocks": clocks,
        }
        if e2e:
            line["e2e"] = {"value": seq_steps_total / e2e_s, "unit": "seq-steps/s", "h2d_bytes_per_step": e2e[1],
                           "d2h_bytes_per_step": e2e[2], "ms_per_step": e2e_s * 1000.0,
                           "path": "qwn_kv_decode_step_host (pinned host buffers)"}
    pool.close()
    del q, k, v
    torch.cuda.empty_cache()

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res = reference_rate(wl, lens, 2, 1, 2)
        if res:
            rate, dt, threads, cname = res
            line["cpu_baseline"] = {"value": rate, "unit": "seq-steps/s", "cores": threads, "kind": "reference",
                                    "sample": f"{len(lens)} sequences (same lengths), first 2 of {L} layers, "
                                              f"2 timed steps, scaled x{L / 2:g}; reference codec {cname}"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--ring", type=int, default=8, help="distinct input step buffers")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=0, help="override the config's layer count (profiling)")
    ap.add_argument("--batch", type=int, default=0, help="override the per-GPU batch (profiling)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3  # the timing rules want >= 3 warm-up steps
    wl = workload(args.config)
    if args.layers:
        wl["layers"] = args.layers
        wl["name"] += f" [layers overridden to {args.layers}]"
    if args.batch:
        wl["batch"] = args.batch
        wl["name"] += f" [batch overridden to {args.batch}]"
    if args.impl == "reference":
        # CPU only: rank 0 runs the reference, the other ranks exit at once
        return run_reference(args, wl, int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")))
    world, rank, local = dist_setup()
    rc = run_ours(args, wl, world, rank, local)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return rc


if __name__ == "__main__":
    sys.exit(main())
