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
    if cfg == 1:
        return dict(name="cfg1 Qwen2-1.5B-shaped single-layer decode, 1 sequence from 2048 tokens, "
                         "int8 per-token-head KV + fp16 scale", codec=2, layers=1, H=12, HK=2, P=16, batch=1,
                    lo=2048, hi=2048, seed=1, outliers=0, steps=256)
    if cfg == 4:
        return dict(name="cfg4 27B-shaped long-context single sequence, 131072 tokens, page 64, "
                         "int8 per-token-head KV + fp16 scale, split-KV across GPUs", codec=2, layers=1, H=48,
                    HK=8, P=64, batch=1, lo=131072, hi=131072, seed=4, outliers=0, steps=50)
    if cfg == 5:
        return dict(name="cfg5 page-pool churn: 1,048,576 pages x 16 tokens, 256 sequences, append + attend, "
                         "p=0.05 score-based eviction to 2048 tokens + compaction", codec=2, layers=1, H=32, HK=8,
                    P=16, batch=256, lo=2048, hi=4096, seed=5, outliers=0, steps=50, pool_pages=1 << 20,
                    evict_p=0.05, budget=2048)
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
    return {1: 272, 2: 260, 3: 128, 4: 160, 5: 512}[codec]


def dtype_of(codec: int) -> str:
    return {1: "int8", 2: "int8", 3: "u4", 4: "u4", 5: "f16"}[codec]


CODEC_LABEL = {1: "int8 per 64 channels + fp32 scale", 2: "int8 per-token-head KV + fp16 scale",
               3: "TurboQuant 3.5-bit groups of 64", 4: "4-bit KV groups of 32 (fp16 range+min)",
               5: "fp16 KV (the reference's paged pool format)"}


def with_codec(wl: dict, codec: int) -> dict:
    """The workload with another KV codec (--codec): same shapes and inputs."""
    if not codec or codec == wl["codec"]:
        return wl
    wl = dict(wl)
    wl["name"] = wl["name"].split(",")[0] + f", {CODEC_LABEL[codec]} (codec override)"
    wl["codec"] = codec
    return wl


def profiled_traffic(cfg: int):
    """DRAM bytes per attention launch (dram__bytes_read + write) from the
    committed ncu capture of the same kernel on this workload's shapes, or
    None when no capture covers the workload."""
    path = os.path.join(ROOT, "profiles", {2: "attn_kernel_q8head_cfg2_full.md", 3: "attn_kernel_q4_cfg3_full.md",
                                           4: "attn_kernel_q8head_hg2_cfg4_full.md"}.get(cfg, ""))
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
        return self.summary_windows([(t0, t1)])

    def summary_windows(self, windows):
        """Clock summary over the samples taken inside any of the windows."""
        rows = [r for t, r in self.rows if any(a <= t <= b for a, b in windows) and len(r) >= 9]
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


def outlier_masks(wl: dict):
    """[layers][kv_heads*128] K outlier channels (x8) of the workload, or None."""
    if not wl["outliers"]:
        return None
    mask = np.zeros((wl["layers"], wl["HK"] * HD), np.uint8)
    rng = np.random.default_rng(wl["seed"] + 17)
    for layer in range(wl["layers"]):
        mask[layer, rng.choice(wl["HK"] * HD, wl["outliers"], replace=False)] = 1
    return mask


def global_lengths(wl: dict, n_gpus: int) -> np.ndarray:
    rng = np.random.default_rng(wl["seed"])
    return rng.integers(wl["lo"], wl["hi"] + 1, size=wl["batch"] * n_gpus).astype(np.int32)


# ---------------------------------------------------------------------------
# reference arm: the reference's own CPU code (oracle/_ref), bounded sample
# ---------------------------------------------------------------------------
def reference_rate(wl: dict, lens: np.ndarray, steps: int, warmup: int, layers_sample: int, threads: int = 0,
                   budget_s: float = 0.0):
    """Decode steps of the reference CPU path on `lens` over the first
    `layers_sample` layers with `threads` OpenMP threads (0 = every host
    core).  Each step's Q/K/V rows are generated before its timer starts (the
    decoder's projections make them), so a step times the append and the
    attention only.  With budget_s > 0 the timed steps stop early (after at
    least 3) once they would run past budget_s seconds.  Returns (seq-steps/s
    scaled to all layers, seconds per sampled step, threads, codec name,
    timed steps)."""
    import ctypes as C
    from oracle import oracle as O
    R = O.ref()
    if R is None:
        return None
    # the reference CPU has only its own codecs: its Q8 for the int8 codecs,
    # TurboQuant for the low-bit ones, its fp16 paged pool for fp16
    codec = {1: 1, 2: 1, 3: 3, 4: 3, 5: 5}[wl["codec"]]
    # every host core: torchrun sets OMP_NUM_THREADS=1 in its workers, so the
    # thread count is set explicitly (the affinity mask bounds it)
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    R.qref_set_threads(threads if threads > 0 else cores)
    R.qref_batch_prepare.restype = C.c_int
    R.qref_batch_prepare.argtypes = [C.c_void_p]
    ids = np.ascontiguousarray(lens, dtype=np.int32)
    h = R.qref_batch_create(codec, ids.size, ids.ctypes.data_as(C.POINTER(C.c_int32)), layers_sample,
                            wl["H"], wl["HK"], HD, steps + warmup + 1, wl["seed"])
    if not h:
        return None
    for _ in range(warmup):
        R.qref_batch_prepare(h)
        R.qref_batch_step(h, layers_sample)
    total, done = 0.0, 0
    for i in range(steps):
        R.qref_batch_prepare(h)
        t0 = time.perf_counter()
        R.qref_batch_step(h, layers_sample)
        total += time.perf_counter() - t0
        done += 1
        if budget_s > 0 and done >= 3 and total / done * (done + 1) > budget_s:
            break
    dt = total / done
    R.qref_batch_destroy(h)
    rate = ids.size / (dt * wl["layers"] / layers_sample)
    return (rate, dt, int(R.qref_max_threads()), {1: "q8_b64_f32", 3: "tq35_g64", 5: "f16_paged"}[codec], done)


def one_thread_row(wl, lens: np.ndarray, steps: int, unit: str, what: str):
    """The reference CPU path on one thread (the 1-thread row next to the
    all-cores baseline), one sampled layer."""
    res = reference_rate(wl, lens, steps, 0, 1, threads=1)
    if not res:
        return None
    rate, dt, threads, cname, done = res
    return {"value": rate, "unit": unit, "cores": threads, "kind": "reference",
            "sample": f"{what}, first 1 of {wl['layers']} layers, {done} timed step(s) on one thread, "
                      f"scaled x{wl['layers']:g}; reference codec {cname}"}


def run_reference(args, wl, world, rank):
    """The reference's own CPU implementation of the path (oracle/_ref, built
    from the reference sources) on every host core: exactly --steps full
    decode steps of the workload (every sequence, every layer) after
    --warmup untimed ones, unless a step takes so long that the run would
    exceed ~3 minutes, in which case it stops after the steps that fit (at
    least 3) and says so."""
    if rank != 0:
        return 0
    lens = global_lengths(wl, 1)
    t_start = time.perf_counter()
    res = reference_rate(wl, lens, max(1, args.steps), max(0, args.warmup), wl["layers"], budget_s=150.0)
    if res is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref (the reference CPU library) is not built"}))
        return 0
    rate, dt, threads, cname, done = res
    sample = (f"{lens.size} sequences, all {wl['layers']} layers per step, {done} timed step(s) after "
              f"{max(0, args.warmup)} warm-up; Q/K/V rows generated before each step's timer; reference codec {cname}")
    line = {"metric": METRIC, "value": rate, "unit": "seq-steps/s", "n_gpus": world, "steps": done,
            "warmup": args.warmup, "ms_per_step": 1000.0 * dt,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype_of(wl["codec"]),
            "data": "synthetic", "impl": "reference",
            "config": {"workload": wl["name"], "global_batch": int(lens.size), "layers": wl["layers"],
                       "query_heads": wl["H"], "kv_heads": wl["HK"], "head_dim": HD, "page_tokens": wl["P"],
                       "parallelism": "host cores (OpenMP over sequence x query head)"},
            "cpu_baseline": {"value": rate, "unit": "seq-steps/s", "cores": threads, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": rate, "unit": "seq-steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "wall_s": time.perf_counter() - t_start}
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
    mask = outlier_masks(wl)
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

    # events around each step's L attention launches (after its page
    # allocation), none between the launches: consecutive launches overlap
    # (each starts its setup and first tiles while the previous one finishes)
    ev_a = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ev_b = [torch.cuda.Event(enable_timing=True) for _ in range(K)]

    def step(s, timed_idx=None):
        # one decode step: grow every sequence by a token, then per layer one
        # launch that quantizes the new K/V into its page and attends
        r = s % ring
        pool.seq_append(B, None, None, stream)
        if timed_idx is not None:
            ev_a[timed_idx].record(stream)
        for layer in range(L):
            pool.decode(layer, B, H, q[r, layer], out[layer], key=k[r, layer], value=v[r, layer], stream=stream)
        if timed_idx is not None:
            ev_b[timed_idx].record(stream)

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
    while time.perf_counter() - t_wall0 < args.soak_ms / 1000.0:
        for layer in range(L):
            pool.decode(layer, B, H, q[0, layer], out[layer], stream=stream)
        torch.cuda.synchronize(dev)
    t_wall1 = time.perf_counter()
    status = pool.check()

    # average duration of one attention launch over the timed steps
    attn_avg_ms = float(np.mean([ev_a[i].elapsed_time(ev_b[i]) / L for i in range(K)]))

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
        traffic = profiled_traffic(args.config) if world == 1 and not args.batch and not args.codec else None
        line = {
            "metric": METRIC, "value": value, "unit": "seq-steps/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": dtype_of(wl["codec"]), "data": "synthetic",
            "config": {"workload": wl["name"], "global_batch": int(B * world), "per_gpu_batch": int(B),
                       "layers": L, "query_heads": H, "kv_heads": HK, "head_dim": HD, "page_tokens": P,
                       "context": f"U[{wl['lo']},{wl['hi']}] (+{W} warmup tokens)",
                       "mean_context": float(lens.mean()), "parallelism": f"sequence-sharded x{world}",
                       "l2": ("L2-resident (the whole cache is ~1 MB): the HBM fraction is not meaningful"
                              if args.config == 1 else "inputs larger than L2 (KV bytes per step >> 126 MB)")},
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
        ls = min(2, L)
        res = reference_rate(wl, lens, 2 if L > 1 else 20, 1, ls)
        if res:
            rate, dt, threads, cname, _ = res
            line["cpu_baseline"] = {"value": rate, "unit": "seq-steps/s", "cores": threads, "kind": "reference",
                                    "sample": f"{len(lens)} sequences (same lengths), first {ls} of {L} layers, "
                                              f"{2 if L > 1 else 20} timed steps, scaled x{L / ls:g}; "
                                              f"reference codec {cname}"}
            line["cpu_baseline"]["one_thread"] = one_thread_row(wl, lens, 1 if L > 1 else 20, "seq-steps/s",
                                                                f"{len(lens)} sequences")
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def _finish_line(args, wl, world, rank, value, ms_step, attn_bytes, attn_ms, attn_ms_max, launches, status,
                 clocks, extra_config, scaling, e2e=None):
    peak, peak_kind = peaks()
    achieved = attn_bytes / (attn_ms / 1000.0) / 1e9 if attn_ms > 0 else 0.0
    # the committed capture covers the 1-GPU launch of this workload only
    traffic = profiled_traffic(args.config) if world == 1 and not args.codec else None
    line = {
        "metric": METRIC, "value": value, "unit": "seq-steps/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": scaling,
        "vs_baseline": None, "dtype": dtype_of(wl["codec"]), "data": "synthetic",
        "config": dict({"workload": wl["name"], "layers": wl["layers"], "query_heads": wl["H"],
                        "kv_heads": wl["HK"], "head_dim": HD, "page_tokens": wl["P"]}, **extra_config),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": peak_kind, "traffic": (traffic or {}).get("bytes_per_launch"),
                     "traffic_source": (traffic or {}).get("source"), "algorithmic_bytes_per_launch": attn_bytes,
                     "avg_launch_ms": attn_ms, "avg_launch_ms_max_rank": attn_ms_max},
        "gpu_launches": int(launches), "status_bits": status, "clocks": clocks,
    }
    if e2e:
        line["e2e"] = e2e
    return line


def run_split(args, wl, world, rank, local):
    """cfg4: one long sequence.  At N GPUs every rank holds the cache and
    attends its contiguous page-aligned KV range.  Default exchange "p2p":
    qwn_kv_decode_split, whose attention kernel stores each kv head's partial
    (m, l, o) into every rank's exchange buffer over NVLink and merges the
    ranks' partials itself -- one launch per step, no collective.  Exchange
    "nccl": qwn_kv_partial writing o | m | l into one block, an NCCL
    all-gather of the blocks and qwn_kv_merge_partials_packed on every rank.
    The rank owning the tail stores each new token.  Total work is fixed:
    strong scaling."""
    import torch
    import qwanto_b200 as qb
    from qwanto_b200.sharding import kv_ranges

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    H, HK, P, c0 = wl["H"], wl["HK"], wl["P"], wl["lo"]
    K, W = args.steps, args.warmup
    max_pages = (c0 + W + K + 2 + P - 1) // P + 1
    pool = qb.KvPool(wl["codec"], 1, HK, P, max_pages + 4, 1, max_pages, max_query_heads=H, permutation_seed=1000,
                     device=local)
    seed = 1000 * wl["seed"]
    pool.prefill_synthetic([0], [c0], seed, None, stream)
    ids = torch.zeros(1, dtype=torch.int32, device=dev)
    ring = min(W + K, args.ring)
    q = torch.empty((ring, H * HD), dtype=torch.float32, device=dev)
    k = torch.empty((ring, HK * HD), dtype=torch.float32, device=dev)
    v = torch.empty((ring, HK * HD), dtype=torch.float32, device=dev)
    for s in range(ring):
        pos = torch.tensor([c0 + s], dtype=torch.int32, device=dev)
        qb.generate_rows(q[s], 1, H * HD, 1, seed, 0, ids, pos, None, stream)
        qb.generate_rows(k[s], 1, HK * HD, 2, seed, 0, ids, pos, None, stream)
        qb.generate_rows(v[s], 1, HK * HD, 3, seed, 0, ids, pos, None, stream)
    out = torch.empty((H * HD,), dtype=torch.float32, device=dev)
    blk = H * (HD + 2)
    send = torch.empty((blk,), dtype=torch.float32, device=dev)
    recv = torch.empty((world, blk), dtype=torch.float32, device=dev)
    torch.cuda.synchronize(dev)
    if world > 1:
        import torch.distributed as dist
    ev_a = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ev_b = [torch.cuda.Event(enable_timing=True) for _ in range(K)]

    # fixed page ranges of the prefilled context; the last rank owns the tail,
    # where every new token goes
    ranges = kv_ranges(c0, world, P)
    p2p = world > 1 and args.exchange == "p2p"
    ex = None
    if p2p:
        from qwanto_b200.exchange import PeerExchange
        ex = PeerExchange(H, device=local, timeout_ns=2_000_000_000)

    def step(s, i=None):
        r = s % ring
        c = c0 + s + 1  # length after this step's token
        pool.seq_append(1, None, None, stream)
        if i is not None:
            ev_a[i].record(stream)
        if world == 1:
            pool.decode(0, 1, H, q[r], out, key=k[r], value=v[r], stream=stream)
        elif p2p:
            a, b = ranges[rank]
            tail = rank == world - 1
            pool.decode_split(0, H, q[r], out, ex, t_begin=a, t_end=0 if tail else b,
                              key=k[r] if tail else None, value=v[r] if tail else None, stream=stream)
        else:
            a, b = ranges[rank]
            if rank == world - 1:
                b = c
                pool.append(0, 1, k[r], v[r], None, stream)
            pool.partial(0, 1, H, q[r], send[H * HD: H * HD + H], send[H * HD + H:], send[: H * HD],
                         t_begin=a, t_end=b, stream=stream)
            dist.all_gather_into_tensor(recv, send)
            qb.merge_partials_packed(world, H, recv, out, stream)
        if i is not None:
            ev_b[i].record(stream)

    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    for s in range(W):
        step(s)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
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
        dist.barrier()
    ms_total = start.elapsed_time(end)
    attn_ms = float(np.mean([ev_a[i].elapsed_time(ev_b[i]) for i in range(K)]))
    t_local = torch.tensor([ms_total, attn_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t_local, op=dist.ReduceOp.MAX)
    ms_total, attn_max = t_local.tolist()
    ms_step = ms_total / K
    # keep the GPUs on this workload (no growth; the same count on every rank,
    # so the collectives match) until the clock samples cover ~1.5 s
    n_soak = min(100000, int(args.soak_ms / max(ms_step, 1e-3)) + 1) if args.soak_ms > 0 else 0
    for _ in range(n_soak):
        if world == 1:
            pool.decode(0, 1, H, q[0], out, stream=stream)
        elif p2p:
            a, b = ranges[rank]
            pool.decode_split(0, H, q[0], out, ex, t_begin=a, t_end=0 if rank == world - 1 else b, stream=stream)
        else:
            a, b = ranges[rank]
            pool.partial(0, 1, H, q[0], send[H * HD: H * HD + H], send[H * HD + H:], send[: H * HD],
                         t_begin=a, t_end=(c0 + W + K) if rank == world - 1 else b, stream=stream)
            dist.all_gather_into_tensor(recv, send)
            qb.merge_partials_packed(world, H, recv, out, stream)
    torch.cuda.synchronize(dev)
    t_wall1 = time.perf_counter()
    sampler.stop()
    status = pool.check()
    if ex is not None:
        dist.barrier()  # every rank is past its last split call before the buffers go
        ex.close()
    # this rank's algorithmic bytes per step: its KV range, the appended
    # token (tail rank), Q, the exchanged partial blocks and the output
    a, b = ranges[rank]
    if rank == world - 1:
        b = c0 + W + K // 2
    attn_bytes = float((b - a) * HK * kv_bytes(wl["codec"]) + H * HD * 4 * 2 + world * blk * 4
                       + ((b - a) + P - 1) // P * 4)
    line = None
    if rank == 0:
        line = _finish_line(args, wl, world, rank, 1000.0 / ms_step, ms_step, attn_bytes, attn_ms, attn_max,
                            launches, status, sampler.summary(t_wall0 - 0.05, t_wall1 + 0.05),
                            {"global_batch": 1, "context": c0,
                             "parallelism": (f"split-KV x{world}" if world == 1 else
                                             f"split-KV x{world}, (m, l, o) exchanged in-kernel over NVLink peer "
                                             f"stores, {blk * 4} B per rank" if p2p else
                                             f"split-KV x{world} (NCCL all-gather of (m, l, o) blocks, "
                                             f"{blk * 4} B per rank)"),
                             "l2": "inputs larger than L2 (272 MB of KV per layer-step)"}, "strong")
        line["unit"] = "layer-steps/s"
    pool.close()
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            res = reference_rate(wl, np.array([c0], np.int32), 3, 1, 1)
            if res:
                rate, dt, threads, cname, _ = res
                line["cpu_baseline"] = {"value": rate, "unit": "layer-steps/s", "cores": threads, "kind": "reference",
                                        "sample": f"1 sequence of {c0} tokens, 3 timed steps; reference codec {cname}"}
                line["cpu_baseline"]["one_thread"] = one_thread_row(wl, np.array([c0], np.int32), 1, "layer-steps/s",
                                                                    f"1 sequence of {c0} tokens")
        print(json.dumps(line), flush=True)
    return 0


def run_churn(args, wl, world, rank, local):
    """cfg5: a 1,048,576-page pool, 256 sequences per GPU; each step every
    sequence appends a token and attends (page attention mass exported), and
    with probability evict_p (seeded, per sequence-step) a sequence evicts
    its lowest-score pages down to the token budget and compacts.  Sequences
    shard over GPUs (weak scaling)."""
    import torch
    import qwanto_b200 as qb
    from qwanto_b200.sharding import balanced_count_shard

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    glens = global_lengths(wl, world)
    mine = balanced_count_shard(glens, world)[rank]
    lens = glens[mine].astype(np.int64)
    B, H, HK, P = len(lens), wl["H"], wl["HK"], wl["P"]
    K, W = args.steps, args.warmup
    max_pages = (int(lens.max()) + W + K + 2 + P - 1) // P + 1
    pool = qb.KvPool(wl["codec"], 1, HK, P, wl["pool_pages"], B, max_pages, max_query_heads=H,
                     permutation_seed=5000 + rank, device=local)
    seed = 1000 * wl["seed"] + rank
    pool.prefill_synthetic(list(range(B)), lens.tolist(), seed, None, stream)
    ring = min(W + K, args.ring)
    ids = torch.arange(B, dtype=torch.int32, device=dev)
    q = torch.empty((ring, B, H * HD), dtype=torch.float32, device=dev)
    k = torch.empty((ring, B, HK * HD), dtype=torch.float32, device=dev)
    v = torch.empty((ring, B, HK * HD), dtype=torch.float32, device=dev)
    for s in range(ring):
        pos = torch.tensor(lens + s, dtype=torch.int32, device=dev)
        qb.generate_rows(q[s], B, H * HD, 1, seed, 0, ids, pos, None, stream)
        qb.generate_rows(k[s], B, HK * HD, 2, seed, 0, ids, pos, None, stream)
        qb.generate_rows(v[s], B, HK * HD, 3, seed, 0, ids, pos, None, stream)
    out = torch.empty((B, H * HD), dtype=torch.float32, device=dev)
    mass = torch.zeros((B, max_pages), dtype=torch.float32, device=dev)
    rng = np.random.default_rng(wl["seed"] * 7919 + rank)
    flags_host = (rng.random((W + K, B)) < wl["evict_p"]).astype(np.uint8)
    flags = torch.tensor(flags_host, device=dev)
    budget = wl["budget"]
    # host mirror of the lengths (eviction removes whole pages until len <= budget)
    hl = lens.copy()
    attn_bytes_steps = []
    ev_a = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ev_b = [torch.cuda.Event(enable_timing=True) for _ in range(K)]

    def step(s, i=None):
        r = s % ring
        hl[:] += 1
        pool.seq_append(B, None, None, stream)
        if i is not None:
            ev_a[i].record(stream)
            attn_bytes_steps.append(float(np.sum(hl * HK * kv_bytes(wl["codec"]) + HK * kv_bytes(wl["codec"])
                                              + 2 * HK * HD * 4 + 2 * H * HD * 4 + np.ceil(hl / P) * 4)))
        pool.decode(0, B, H, q[r], out, key=k[r], value=v[r], page_mass=mass, stream=stream)
        if i is not None:
            ev_b[i].record(stream)
        pool.evict(B, mass, flags[s], budget, None, stream)
        f = flags_host[s].astype(bool) & (hl > budget)
        hl[f] -= P * ((hl[f] - budget + P - 1) // P)

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
    # keep the GPU on this workload (attention only, no growth or eviction)
    # until the clock samples cover ~1.5 s
    while time.perf_counter() - t_wall0 < args.soak_ms / 1000.0:
        for _ in range(20):
            pool.decode(0, B, H, q[0], out, stream=stream)
        torch.cuda.synchronize(dev)
    t_wall1 = time.perf_counter()
    sampler.stop()
    status = pool.check()
    gpu_lens = pool.lens()[:B]
    lens_match = bool(np.array_equal(gpu_lens.astype(np.int64), hl))
    attn_ms = float(np.mean([ev_a[i].elapsed_time(ev_b[i]) for i in range(K)]))
    t_local = torch.tensor([ms_total, attn_ms], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t_local, op=torch.distributed.ReduceOp.MAX)
    ms_total, attn_max = t_local.tolist()
    ms_step = ms_total / K
    line = None
    if rank == 0:
        line = _finish_line(args, wl, world, rank, B * world / (ms_step / 1000.0), ms_step,
                            float(np.mean(attn_bytes_steps)), attn_ms, attn_max, launches, status,
                            sampler.summary(t_wall0 - 0.05, t_wall1 + 0.05),
                            {"global_batch": int(B * world), "per_gpu_batch": int(B),
                             "pool_pages": wl["pool_pages"], "evict_p": wl["evict_p"], "token_budget": budget,
                             "evictions_timed": int(np.sum(flags_host[W:])),
                             "lengths_match_host_model": lens_match,
                             "parallelism": f"sequence-sharded x{world}",
                             "l2": "inputs larger than L2 (KV bytes per step >> 126 MB)"}, "weak")
        line["roofline"]["kernel"] = "attn_kernel with page-mass export (the eviction launches are in ms_per_step)"
    pool.close()
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            res = reference_rate(wl, lens.astype(np.int32), 2, 1, 1)
            if res:
                rate, dt, threads, cname, _ = res
                line["cpu_baseline"] = {"value": rate, "unit": "seq-steps/s", "cores": threads, "kind": "reference",
                                        "sample": f"{B} sequences (same lengths), append + attend, 2 timed steps, "
                                                  f"no eviction; reference codec {cname}"}
                line["cpu_baseline"]["one_thread"] = one_thread_row(wl, lens.astype(np.int32), 1, "seq-steps/s",
                                                                    f"{B} sequences, append + attend, no eviction")
        print(json.dumps(line), flush=True)
    return 0


def run_gemv(args) -> int:
    """HyperVSQ-2 GEMV / batched GEMM (74-byte blocks of 256 2-bit weights
    times int8 activations), through ABI v1 exactly as qwnrun calls it: this
    library against the reference's own GPU library (oracle/_ref, compiled
    from c/cuda/qwn_hypervsq2_cuda_abi.cu) on the same weights and inputs.
    Times are each library's own kernel events (telemetry gpu_kernel_ms per
    call); outputs are cross-checked.  One JSON line per shape."""
    import ctypes as C
    from qwanto_b200 import _lib
    libs = {"ours": os.path.join(ROOT, "qwanto_b200", "qwn_cuda.so"),
            "reference": os.path.join(ROOT, "oracle", "_ref", "qwn_cuda_ref.so")}
    P = C.POINTER
    loaded = {}
    for name, path in libs.items():
        if not os.path.exists(path):
            continue
        L = C.CDLL(path, mode=os.RTLD_LOCAL)
        for fn, res, argt in (("qwn_cuda_abi_context_create", C.c_int, [P(_lib.ContextOptions), P(_lib.Handle)]),
                              ("qwn_cuda_abi_context_destroy", C.c_int, [P(_lib.Handle)]),
                              ("qwn_cuda_abi_upload_tensor", C.c_int, [P(_lib.Handle), P(_lib.TensorUpload), P(_lib.Handle)]),
                              ("qwn_cuda_abi_release_tensor", C.c_int, [P(_lib.Handle), P(_lib.Handle)]),
                              ("qwn_cuda_abi_hypervsq2_gemm", C.c_int, [P(_lib.Handle), P(_lib.GemmRequest), P(_lib.Telemetry)])):
            getattr(L, fn).restype = res
            getattr(L, fn).argtypes = argt
        loaded[name] = L
    rng = np.random.default_rng(7)
    shapes = [(4096, 4096, 1), (14336, 4096, 1), (4096, 14336, 1), (151936, 4096, 1), (4096, 4096, 8), (14336, 4096, 8)]
    for rows, cols, batch in shapes:
        nblk = (cols + 255) // 256
        w = rng.integers(0, 256, size=(rows, nblk, 74), dtype=np.uint8)
        base = (rng.random((rows, nblk)) * 0.01 + 0.001).astype(np.float16)
        offs = (rng.random((rows, nblk)) * 0.002 - 0.001).astype(np.float16)
        w[:, :, 0:2] = base.view(np.uint8).reshape(rows, nblk, 2)
        w[:, :, 2:4] = offs.view(np.uint8).reshape(rows, nblk, 2)
        wb = np.ascontiguousarray(w.reshape(-1))
        act = rng.integers(-127, 128, size=(batch, cols), dtype=np.int8)
        scales = (rng.random(batch) + 0.5).astype(np.float32)
        line = {"gemv": {"rows": rows, "cols": cols, "batch": batch}, "weight_bytes": int(wb.size)}
        outs = {}
        for name, L in loaded.items():
            o = _lib.init(_lib.ContextOptions())
            o.device_id = 0
            ctx = _lib.init(_lib.Handle())
            if L.qwn_cuda_abi_context_create(C.byref(o), C.byref(ctx)) != 0:
                line[name] = "context_create failed"
                continue
            up = _lib.init(_lib.TensorUpload())
            up.host_data, up.data_bytes, up.dtype, up.rows, up.cols, up.block_bytes = wb.ctypes.data, wb.size, 1, rows, cols, 74
            th = _lib.init(_lib.Handle())
            assert L.qwn_cuda_abi_upload_tensor(C.byref(ctx), C.byref(up), C.byref(th)) == 0
            out = np.zeros((batch, rows), np.float32)
            rq = _lib.init(_lib.GemmRequest())
            rq.tensor, rq.input_q8 = th, act.ctypes.data
            rq.input_scales = scales.ctypes.data_as(C.POINTER(C.c_float))
            rq.output = out.ctypes.data_as(C.POINTER(C.c_float))
            rq.batch, rq.rows, rq.cols, rq.input_mode = batch, rows, cols, 1
            tel = _lib.init(_lib.Telemetry())
            per = []
            n = 10 if wb.size > 50e6 else 60
            for i in range(3):
                assert L.qwn_cuda_abi_hypervsq2_gemm(C.byref(ctx), C.byref(rq), C.byref(tel)) == 0
            # at least n calls and --soak-ms of them, with the clocks sampled meanwhile
            clocks = ClockSampler(0)
            clocks.start()
            time.sleep(0.3)
            w0 = time.perf_counter()
            while len(per) < n or time.perf_counter() - w0 < args.soak_ms / 1000.0:
                before = tel.gpu_kernel_ms
                assert L.qwn_cuda_abi_hypervsq2_gemm(C.byref(ctx), C.byref(rq), C.byref(tel)) == 0
                per.append(tel.gpu_kernel_ms - before)
            w1 = time.perf_counter()
            clocks.stop()
            us = 1000.0 * float(np.median(per))
            moved = wb.size + act.size + 4 * out.size
            line[name] = {"kernel_us": us, "gbs": moved / (us * 1e-6) / 1e9, "calls": len(per),
                          "clocks": clocks.summary(w0, w1)}
            outs[name] = out.copy()
            L.qwn_cuda_abi_release_tensor(C.byref(ctx), C.byref(th))
            L.qwn_cuda_abi_context_destroy(C.byref(ctx))
        if "ours" in outs and "reference" in outs:
            ref = outs["reference"]
            line["max_rel_diff"] = float(np.max(np.abs(outs["ours"] - ref) / (1e-3 + np.abs(ref))))
            line["speedup"] = line["reference"]["kernel_us"] / line["ours"]["kernel_us"]
        print(json.dumps(line), flush=True)
    return 0


def run_abi_kv(args) -> int:
    """cfg1 through ABI v1 exactly as qwnrun's CUDA backend drives its Q8 KV
    cache (c/qwanto_decode.c:1658-1724): per decode step one
    qwn_cuda_abi_kv_cache_append of the token's K/V rows and one
    qwn_cuda_abi_kv_cache_attention of the 12 query heads, host buffers and
    synchronous calls, for this library and for the reference's own GPU
    library (oracle/_ref/qwn_cuda_ref.so, built from
    c/cuda/qwn_hypervsq2_cuda_abi.cu; kernel qwn_q8_attention at :175-223) on
    the same inputs: 2048 tokens prefilled, then 256 timed steps.  Wall time
    per step (the calls return after their results are on the host) and the
    libraries' own kernel time (telemetry); outputs are cross-checked.  One
    JSON line."""
    import ctypes as C
    from qwanto_b200 import _lib
    wl = workload(1)
    H, HK, T0 = wl["H"], wl["HK"], wl["lo"]
    steps = args.steps if args.steps > 0 else wl["steps"]
    libs = {"ours": os.path.join(ROOT, "qwanto_b200", "qwn_cuda.so"),
            "reference_gpu": os.path.join(ROOT, "oracle", "_ref", "qwn_cuda_ref.so")}
    P = C.POINTER
    rng = np.random.default_rng(wl["seed"])
    ch = HK * HD
    keys = rng.standard_normal((T0 + steps, ch)).astype(np.float32)
    vals = rng.standard_normal((T0 + steps, ch)).astype(np.float32)
    qs = rng.standard_normal((steps, H * HD)).astype(np.float32)
    line = {"abi_v1_kv": {"workload": wl["name"], "query_heads": H, "kv_heads": HK, "head_dim": HD,
                          "prefill_tokens": T0, "steps": steps,
                          "path": "qwn_cuda_abi_kv_cache_append + qwn_cuda_abi_kv_cache_attention per step, "
                                  "host buffers, synchronous (qwnrun --backend cuda --kv-cache q8)"}}
    outs = {}
    for name, path in libs.items():
        if not os.path.exists(path):
            line[name] = "not built"
            continue
        L = C.CDLL(path, mode=os.RTLD_LOCAL)
        for fn, argt in (("qwn_cuda_abi_context_create", [P(_lib.ContextOptions), P(_lib.Handle)]),
                         ("qwn_cuda_abi_context_destroy", [P(_lib.Handle)]),
                         ("qwn_cuda_abi_kv_cache_create", [P(_lib.Handle), P(_lib.KvCacheOptions), P(_lib.Handle)]),
                         ("qwn_cuda_abi_kv_cache_destroy", [P(_lib.Handle), P(_lib.Handle)]),
                         ("qwn_cuda_abi_kv_cache_append", [P(_lib.Handle), P(_lib.KvAppendRequest), P(_lib.Telemetry)]),
                         ("qwn_cuda_abi_kv_cache_attention", [P(_lib.Handle), P(_lib.KvAttentionRequest),
                                                              P(_lib.Telemetry)])):
            getattr(L, fn).restype = C.c_int
            getattr(L, fn).argtypes = argt
        o = _lib.init(_lib.ContextOptions())
        ctx = _lib.init(_lib.Handle())
        assert L.qwn_cuda_abi_context_create(C.byref(o), C.byref(ctx)) == 0
        ko = _lib.init(_lib.KvCacheOptions())
        ko.max_tokens, ko.kv_heads, ko.head_dim = T0 + steps + 16, HK, HD
        tel = _lib.init(_lib.Telemetry())
        out = np.zeros(H * HD, np.float32)
        res = np.zeros((steps, H * HD), np.float32)
        # The 256 steps are timed as rounds until --soak-ms of timed steps
        # have passed (at least one round), so that the clock samples fall
        # inside the timed region.  ABI v1 appends only at the cache's end,
        # so every round runs on a fresh cache with the same 2048 tokens
        # prefilled outside the timed windows; every round computes the same
        # outputs.
        clocks = ClockSampler(0)
        clocks.start()
        time.sleep(0.3)
        rounds, timed, windows, kernel_ms = 0, 0.0, [], 0.0
        while rounds == 0 or timed < args.soak_ms / 1000.0:
            cache = _lib.init(_lib.Handle())
            assert L.qwn_cuda_abi_kv_cache_create(C.byref(ctx), C.byref(ko), C.byref(cache)) == 0
            ap = _lib.init(_lib.KvAppendRequest())
            ap.cache, ap.n_channels = cache, ch
            at = _lib.init(_lib.KvAttentionRequest())
            at.cache, at.query_heads, at.kv_heads, at.head_dim, at.scale = cache, H, HK, HD, 1.0 / math.sqrt(HD)
            at.host_output = out.ctypes.data_as(P(C.c_float))
            for t in range(T0):
                ap.host_key = keys[t].ctypes.data_as(P(C.c_float))
                ap.host_value = vals[t].ctypes.data_as(P(C.c_float))
                ap.token = t
                assert L.qwn_cuda_abi_kv_cache_append(C.byref(ctx), C.byref(ap), C.byref(tel)) == 0
            k0 = tel.kv_cache_kernel_ms
            t0 = time.perf_counter()
            for i in range(steps):
                t = T0 + i
                ap.host_key = keys[t].ctypes.data_as(P(C.c_float))
                ap.host_value = vals[t].ctypes.data_as(P(C.c_float))
                ap.token = t
                assert L.qwn_cuda_abi_kv_cache_append(C.byref(ctx), C.byref(ap), C.byref(tel)) == 0
                at.host_query = qs[i].ctypes.data_as(P(C.c_float))
                at.position = t
                assert L.qwn_cuda_abi_kv_cache_attention(C.byref(ctx), C.byref(at), C.byref(tel)) == 0
                res[i] = out
            t1 = time.perf_counter()
            kernel_ms += tel.kv_cache_kernel_ms - k0
            timed += t1 - t0
            windows.append((t0, t1))
            rounds += 1
            L.qwn_cuda_abi_kv_cache_destroy(C.byref(ctx), C.byref(cache))
        clocks.stop()
        wall = timed / (steps * rounds)
        line[name] = {"steps_per_s": 1.0 / wall, "wall_us_per_step": wall * 1e6,
                      "kernel_us_per_step": kernel_ms * 1000.0 / (steps * rounds),
                      "kernel_type": tel.kv_cache_kernel_type.decode(errors="replace"), "rounds": rounds,
                      "clocks": clocks.summary_windows(windows)}
        outs[name] = res
        L.qwn_cuda_abi_context_destroy(C.byref(ctx))
    if len(outs) == 2:
        a, b = outs["ours"], outs["reference_gpu"]
        line["max_abs_diff"] = float(np.abs(a - b).max())
        line["speedup_wall"] = line["ours"]["steps_per_s"] / line["reference_gpu"]["steps_per_s"]
        # (the reference library's telemetry may leave its kernel time at 0)
        rk = line["reference_gpu"]["kernel_us_per_step"]
        line["speedup_kernel"] = rk / max(line["ours"]["kernel_us_per_step"], 1e-9) if rk > 0 else None
    print(json.dumps(line), flush=True)
    return 0


def run_linear(args) -> int:
    """Linear attention (qwn_linear_attention_*): decode over a batch of
    sequences' states and prefill of one long sequence, each timed with CUDA
    events on device buffers, end to end through the host-buffer call, and
    against the reference's own qwanto_linear_attention_decode/prefill
    (oracle/_ref, built from c/qwanto_attention.c) on the host cores.  The
    decode state is larger than L2, so every timed step streams it from HBM.
    One JSON line per workload."""
    import ctypes as C
    import torch
    from qwanto_b200.linear_attention import LinearAttentionState
    peak, peak_kind = peaks()
    ref = None
    try:
        sys.path.insert(0, ROOT)
        from oracle import oracle as _ora
        ref = _ora.ref()
    except Exception:
        ref = None
    fp = lambda a: a.ctypes.data_as(C.POINTER(C.c_float))
    rng = np.random.default_rng(3)
    decay = 0.97
    steps = args.steps or 20
    for name, H, D, T in (("decode: 96 sequences x 32 heads, head_dim 128", 3072, 128, 1),
                          ("decode: 8 sequences x 32 heads, head_dim 64", 256, 64, 1),
                          ("prefill: 1 sequence x 32 heads, head_dim 128, 4096 tokens", 32, 128, 4096),
                          ("prefill: 16 sequences x 32 heads, head_dim 128, 512 tokens", 512, 128, 512)):
        st = LinearAttentionState(H, D)
        ring = 4 if T == 1 else 1
        q, k, v = (torch.randn((ring, T, H, D), device="cuda") * 0.1 for _ in range(3))
        o = torch.empty((ring, T, H, D), device="cuda")
        for i in range(args.warmup):
            st.prefill(q[i % ring], k[i % ring], v[i % ring], decay, T, o[i % ring])
        torch.cuda.synchronize()
        n = steps if T == 1 else max(3, steps // 4)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        # a probe sizes the timed loop so that it lasts at least --soak-ms:
        # the clock samples (every 100 ms) then fall inside the timed region
        ev[0].record()
        for i in range(n):
            st.prefill(q[i % ring], k[i % ring], v[i % ring], decay, T, o[i % ring])
        ev[1].record()
        torch.cuda.synchronize()
        n = max(n, int(args.soak_ms / max(ev[0].elapsed_time(ev[1]) / n, 1e-3)) + 1)
        clocks = ClockSampler(0)
        clocks.start()
        time.sleep(0.3)
        w0 = time.perf_counter()
        ev[0].record()
        for i in range(n):
            st.prefill(q[i % ring], k[i % ring], v[i % ring], decay, T, o[i % ring])
        ev[1].record()
        torch.cuda.synchronize()
        w1 = time.perf_counter()
        clocks.stop()
        us = ev[0].elapsed_time(ev[1]) * 1000.0 / n
        state_bytes = 4 * H * D * D
        moved = 2 * state_bytes + 16 * T * H * D  # state read+write once, q/k/v in, o out
        line = {"linear_attention": name, "n_heads": H, "head_dim": D, "tokens": T, "steps": n,
                "kernel_us": us, "tokens_per_s": T / (us * 1e-6),
                "roofline": {"bound": "hbm", "achieved": moved / (us * 1e-6) / 1e9, "peak": peak, "unit": "GB/s",
                             "frac": moved / (us * 1e-6) / 1e9 / peak, "peak_kind": peak_kind,
                             "algorithmic_bytes": moved},
                "clocks": clocks.summary(w0, w1)}
        # end to end through the host-buffer call (pinned host inputs, output read back)
        hq, hk, hv = (x[0].cpu().pin_memory() for x in (q, k, v))
        ho = torch.empty((T, H, D)).pin_memory()
        e2e_n = 5 if T == 1 else 2
        st.prefill_host(hq.data_ptr(), hk.data_ptr(), hv.data_ptr(), decay, T, ho.data_ptr())
        t0 = time.perf_counter()
        for _ in range(e2e_n):
            st.prefill_host(hq.data_ptr(), hk.data_ptr(), hv.data_ptr(), decay, T, ho.data_ptr())
        e2e_s = (time.perf_counter() - t0) / e2e_n
        line["e2e"] = {"tokens_per_s": T / e2e_s, "ms": e2e_s * 1e3, "h2d_bytes": 12 * T * H * D,
                       "d2h_bytes": 4 * T * H * D}
        st.close()
        if ref is not None and not args.no_cpu_baseline:
            # the reference on the host cores: a bounded sample of the same workload
            rs = _ora.RefLinearState()
            assert ref.qwanto_linear_attention_init(C.byref(rs), H, D) == 0
            nt = 2 if T == 1 else max(4, min(T, int(5e8 / (2 * H * D * D))))
            cq, ck, cv = ((rng.standard_normal((nt, H, D)) * 0.1).astype(np.float32) for _ in range(3))
            co = np.empty((nt, H, D), np.float32)
            t0 = time.perf_counter()
            reps = 0
            while True:
                ref.qwanto_linear_attention_prefill(C.byref(rs), fp(cq), fp(ck), fp(cv), C.c_float(decay), nt, fp(co))
                reps += 1
                if time.perf_counter() - t0 > 3.0:
                    break
            cpu_s = (time.perf_counter() - t0) / (reps * nt)
            ref.qwanto_linear_attention_destroy(C.byref(rs))
            line["cpu_reference"] = {"tokens_per_s": 1.0 / cpu_s, "cores": 1, "kind": "reference",
                                     "sample": f"{reps * nt} token steps of the same shape"}
            line["speedup_kernel"] = line["tokens_per_s"] / line["cpu_reference"]["tokens_per_s"]
            line["speedup_e2e"] = line["e2e"]["tokens_per_s"] / line["cpu_reference"]["tokens_per_s"]
        print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=0, help="timed steps (default 20; cfg1 256, cfg4/5 50)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--ring", type=int, default=8, help="distinct input step buffers")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--gemv", action="store_true",
                    help="time the HyperVSQ-2 GEMV against the reference GPU library instead (one line per shape)")
    ap.add_argument("--codec", type=int, default=0, choices=[0, 1, 2, 3, 4, 5],
                    help="run the config's shapes with another KV codec (5 = fp16, the reference's paged pool)")
    ap.add_argument("--soak-ms", type=float, default=1500.0,
                    help="cfg4/cfg5: keep the GPU on the workload after the timed steps until the clock samples "
                         "cover this long (0 for profiling runs)")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"],
                    help="cfg4 at N>1: partials exchanged in-kernel over NVLink (p2p) or by an NCCL all-gather")
    ap.add_argument("--layers", type=int, default=0, help="override the config's layer count (profiling)")
    ap.add_argument("--batch", type=int, default=0, help="override the per-GPU batch (profiling)")
    ap.add_argument("--abi-kv", action="store_true",
                    help="cfg1 through ABI v1 (qwnrun's CUDA Q8 KV calls): this library vs the reference GPU library")
    ap.add_argument("--linear", action="store_true",
                    help="time linear-attention decode/prefill against the reference CPU code (one line per shape)")
    args = ap.parse_args()
    if args.gemv:
        return run_gemv(args)
    if args.linear:
        return run_linear(args)
    if args.abi_kv:
        return run_abi_kv(args)
    if args.warmup < 3:
        args.warmup = 3  # the timing rules want >= 3 warm-up steps
    wl = with_codec(workload(args.config), args.codec)
    if not args.steps:
        args.steps = wl.get("steps", 20)
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
    if args.config == 4:
        rc = run_split(args, wl, world, rank, local)
    elif args.config == 5:
        rc = run_churn(args, wl, world, rank, local)
    else:
        rc = run_ours(args, wl, world, rank, local)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return rc


if __name__ == "__main__":
    sys.exit(main())
