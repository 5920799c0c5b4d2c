#!/usr/bin/env python
"""Benchmark of the B200 paged KV-cache path (one JSON line on rank 0).

Workload ("isolated paged decode microbench"):
Llama-3-8B attention shape (32 q heads, 8 KV heads, head_dim 128), f16 K/V
~ N(0,1), 64 sequences with context lengths uniform in [512, 4096], 16-token
blocks whose physical ids are randomly interleaved across sequences.  One
step = one append (KvCache::append for 64 tokens, host bookkeeping) + one
fused K/V write and decode-attention launch over every cached block.  Each
block of 16 steps ends with kv_remove back to the starting lengths, so the
per-step work stays that of the configuration.

`value` is device-timed (CUDA events, inputs resident in HBM); `e2e` runs
the same step through the public API from pinned host buffers, copying q/k/v
in and the attention output out every step and reading it on the host.

--impl reference times the reference's CPU path (the C restatement in
oracle/, since the Rust reference cannot be built here) on this host's cores.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "paged decode-attn tokens/s & HBM GB/s vs ~8 TB/s; append/CoW GB/s, 1–8 GPU"
N_HEADS, N_KV_HEADS, HEAD_DIM, BATCH, BLOCK = 32, 8, 128, 64, 16
CTX_LO, CTX_HI = 512, 4096
CYCLE = 16  # steps between kv_remove back to the starting lengths
FALLBACK_HBM_GBS = 6650.0


def rank_info():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def workload(seed: int):
    rng = np.random.default_rng(seed)
    lens = rng.integers(CTX_LO, CTX_HI + 1, BATCH)
    return lens


def step_bytes(lens_now: np.ndarray) -> dict:
    """Algorithmic bytes of one step (one layer) at current lengths `lens_now`
    (after the step's append): K and V of every cached position once, q, out,
    block-table entries, and the appended rows (f16 in, f16 out)."""
    kv_row = N_KV_HEADS * HEAD_DIM * 2  # bytes of one K (or V) row
    attn = int(lens_now.sum()) * kv_row * 2
    q = BATCH * N_HEADS * HEAD_DIM * 2
    out = BATCH * N_HEADS * HEAD_DIM * 2
    tables = int(((lens_now + BLOCK - 1) // BLOCK).sum()) * 4
    append = BATCH * 2 * kv_row * 2  # read f16 input + write f16 cell, K and V
    return {"attn": attn, "q": q, "out": out, "tables": tables, "append": append,
            "total": attn + q + out + tables + append}


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic():
    """DRAM bytes per launch of the attention kernel from the committed ncu
    summary (profiles/paged_attn_c2.md, line 'traffic_bytes_per_launch: N')."""
    p = ROOT / "profiles" / "paged_attn_c2.md"
    try:
        for line in p.read_text().splitlines():
            if line.strip().startswith("traffic_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1].strip()))
    except Exception:
        pass
    return None


class Clocks:
    """nvidia-smi clock / throttle sampling around the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_id: str):
        self.proc = None
        self.path = ROOT / "gpurun_out" / f"clocks_{os.getpid()}.csv"
        try:
            self.path.parent.mkdir(exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "50", "-i", device_id], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def mark(self):
        return time.time()

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        try:
            self.path.unlink()
        except Exception:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        return {"sm_mhz": float(np.median([r[0] for r in rows])), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# our arm


def build_cache(kv_mod, torch, device: int, lens: np.ndarray, seed: int):
    """Fill a cache with the workload: every sequence's context appended in
    16-token pieces in a random interleaving (seed+1), so physical block ids
    are scattered across sequences, then K/V written as f16 N(0,1)."""
    headroom = CYCLE + 1
    n_blocks = int(((lens + headroom + BLOCK - 1) // BLOCK).sum()) + BATCH
    kv = kv_mod.KvCache(1, N_KV_HEADS, HEAD_DIM, n_blocks * BLOCK, n_heads=N_HEADS, max_seqs=BATCH,
                        max_batch=8192, device=device)
    rng = np.random.default_rng(seed + 1)
    pieces = np.repeat(np.arange(BATCH), (lens + BLOCK - 1) // BLOCK)
    rng.shuffle(pieces)
    cur = np.zeros(BATCH, np.int64)
    seqs, pos = [], []
    for s in pieces:
        n = min(BLOCK, int(lens[s] - cur[s]))
        seqs.append(np.full(n, s))
        pos.append(np.arange(cur[s], cur[s] + n))
        cur[s] += n
    seqs = np.concatenate(seqs)
    pos = np.concatenate(pos)
    gen = torch.Generator(device=f"cuda:{device}")
    gen.manual_seed(seed)
    chunk = 8192
    for i in range(0, seqs.size, chunk):
        b, sl = kv.append_batch(seqs[i:i + chunk], pos[i:i + chunk])
        n = b.size
        k = torch.randn((n, N_KV_HEADS * HEAD_DIM), generator=gen, device=f"cuda:{device}", dtype=torch.float16)
        v = torch.randn((n, N_KV_HEADS * HEAD_DIM), generator=gen, device=f"cuda:{device}", dtype=torch.float16)
        kv.write(0, b, sl, k, v)
    torch.cuda.synchronize()
    return kv


class Stepper:
    """One decode step through the public API: append + fused write/attend."""

    def __init__(self, kv, lens, k, v, q, out):
        self.kv, self.lens = kv, lens
        self.seqs = np.arange(BATCH, dtype=np.uint32)
        self.k, self.v, self.q, self.out = k, v, q, out
        self.phase = 0

    def step(self):
        pos = (self.lens + self.phase).astype(np.uint32)
        b, s = self.kv.append_batch(self.seqs, pos)
        self.kv.write_attend(0, b, s, self.k, self.v, self.q, self.seqs, pos, out=self.out)
        lens_now = self.lens + self.phase + 1
        self.phase += 1
        if self.phase == CYCLE:
            for i in range(BATCH):
                self.kv.truncate(i, int(self.lens[i]))  # Backend::kv_remove
            self.phase = 0
        return lens_now


def run_ours(args, rank, world, local):
    import torch
    import torch.distributed as dist

    from langtrain_studio_b200 import kv as kv_mod

    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    seed = 1234 + rank
    lens = workload(seed)
    kv = build_cache(kv_mod, torch, local, lens, seed)
    g = torch.Generator(device=dev)
    g.manual_seed(seed + 7)
    k = torch.randn((BATCH, N_KV_HEADS * HEAD_DIM), generator=g, device=dev, dtype=torch.float16)
    v = torch.randn((BATCH, N_KV_HEADS * HEAD_DIM), generator=g, device=dev, dtype=torch.float16)
    q = torch.randn((BATCH, N_HEADS * HEAD_DIM), generator=g, device=dev, dtype=torch.float16)
    out = torch.empty((BATCH, N_HEADS * HEAD_DIM), device=dev, dtype=torch.float16)
    st = Stepper(kv, lens, k, v, q, out)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---------------- device-resident timed region ----------------
    for _ in range(args.warmup):
        st.step()
    # align to a cycle boundary so every run sees the same phases
    while st.phase != 0:
        st.step()
    try:
        uuid = str(torch.cuda.get_device_properties(local).uuid)
        dev_id = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
    except Exception:
        dev_id = str(local)
    clocks = Clocks(dev_id)
    time.sleep(0.3)
    kv.profile(True)
    launches0 = kv.launch_count()
    total_bytes = 0
    attn_bytes = 0
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        lens_now = st.step()
        b = step_bytes(lens_now)
        total_bytes += b["total"]
        attn_bytes += b["total"]
    e1.record()
    barrier()
    ms = e0.elapsed_time(e1)
    launches = kv.launch_count() - launches0
    attn_ms, attn_n = kv.profile_read()
    kv.profile(False)
    clk = clocks.stop()
    kv.check()
    ms_max = ms
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())
    # ---------------- end-to-end through the public API ----------------
    hq = torch.empty_like(q, device="cpu").pin_memory()
    hk = torch.empty_like(k, device="cpu").pin_memory()
    hv = torch.empty_like(v, device="cpu").pin_memory()
    hout = torch.empty_like(out, device="cpu").pin_memory()
    hq.copy_(q)
    hk.copy_(k)
    hv.copy_(v)
    stream = torch.cuda.current_stream()
    e2e_steps = args.steps

    def e2e_step():
        q.copy_(hq, non_blocking=True)
        k.copy_(hk, non_blocking=True)
        v.copy_(hv, non_blocking=True)
        st.step()
        hout.copy_(out, non_blocking=True)
        stream.synchronize()  # the host reads this step's result
        return float(hout[0, 0])

    for _ in range(max(args.warmup, 1)):
        e2e_step()
    while st.phase != 0:
        e2e_step()
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(e2e_steps):
        e2e_step()
    f1.record()
    barrier()
    e2e_ms = f0.elapsed_time(f1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    h2d = (q.numel() + k.numel() + v.numel()) * 2
    d2h = out.numel() * 2

    result = None
    if rank == 0:
        peak, peak_kind = measured_peak()
        avg_attn_ms = attn_ms / max(attn_n, 1)
        per_launch_bytes = attn_bytes / max(args.steps, 1)
        achieved = per_launch_bytes / (avg_attn_ms * 1e-3) / 1e9
        tokens = BATCH * args.steps * world
        result = {
            "metric": METRIC,
            "value": tokens / (ms_max * 1e-3),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_max / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f16",
            "data": "synthetic: f16 K/V and q ~ N(0,1), seeded; lengths U[512,4096] seeded",
            "config": {
                "workload": "configs[1]: isolated paged decode microbench, Llama-3-8B attention shape, one layer",
                "batch_per_gpu": BATCH, "ctx": f"U[{CTX_LO},{CTX_HI}]", "n_heads": N_HEADS,
                "n_kv_heads": N_KV_HEADS, "head_dim": HEAD_DIM, "block_tokens": BLOCK,
                "step": "append 1 token/seq + fused K/V write + decode attention (f32 softmax/accumulate)",
                "kv_bytes_per_step": int(attn_bytes / max(args.steps, 1)),
                "l2": "inputs larger than L2: ~0.6 GB of K/V read per step vs 126 MB L2",
                "parallelism": f"seq-sharded x{world} (independent pools, no collective)",
            },
            "hbm_gbs": total_bytes / (ms_max * 1e-3) / 1e9 / 1.0 * world,
            "roofline": {
                "bound": "hbm", "kernel": "paged_attn_kernel<128> (fused append + attention)",
                "achieved": achieved, "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                "frac": achieved / peak, "traffic": ncu_traffic(),
                "algorithmic_bytes_per_launch": int(per_launch_bytes), "avg_launch_ms": avg_attn_ms,
            },
            "e2e": {"value": tokens / (e2e_ms * 1e-3) if world == 1 else BATCH * e2e_steps * world / (e2e_ms * 1e-3),
                    "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": int(launches),
            "clocks": clk,
        }
    if world > 1:
        dist.barrier()
        kv.close()
        dist.destroy_process_group()
    else:
        kv.close()
    return result


# ---------------------------------------------------------------------------
# CPU arm (restated reference path)


def cpu_fill(ok_mod, lens, seed):
    n_blocks = int(((lens + CYCLE + 1 + BLOCK - 1) // BLOCK).sum()) + BATCH
    ok = ok_mod.OracleKv(1, N_KV_HEADS * HEAD_DIM, n_blocks * BLOCK, max_seqs=BATCH)
    rng = np.random.default_rng(seed + 1)
    pieces = np.repeat(np.arange(BATCH), (lens + BLOCK - 1) // BLOCK)
    rng.shuffle(pieces)
    cur = np.zeros(BATCH, np.int64)
    seqs, pos = [], []
    for s in pieces:
        n = min(BLOCK, int(lens[s] - cur[s]))
        seqs.append(np.full(n, s))
        pos.append(np.arange(cur[s], cur[s] + n))
        cur[s] += n
    seqs = np.concatenate(seqs)
    pos = np.concatenate(pos)
    drng = np.random.default_rng(seed)
    chunk = 16384
    for i in range(0, seqs.size, chunk):
        rc, done, b, sl = ok.append_batch(seqs[i:i + chunk], pos[i:i + chunk])
        assert rc == 0
        n = b.size
        k = drng.standard_normal((n, N_KV_HEADS * HEAD_DIM), np.float32).astype(np.float16)
        v = drng.standard_normal((n, N_KV_HEADS * HEAD_DIM), np.float32).astype(np.float16)
        ok.write_batch(0, b, sl, k, v)
    return ok


def cpu_run(lens, seed, budget_s, max_steps, threads):
    """Time the restated reference step (append + write + attention over every
    sequence, model.rs:380-476) on `threads` host threads.  Steps run until
    `budget_s` seconds or `max_steps`; returns (tokens/s, steps, seconds)."""
    from oracle import oracle as ok_mod

    ok = cpu_fill(ok_mod, lens, seed)
    rng = np.random.default_rng(seed + 9)
    kin = rng.standard_normal((BATCH, N_KV_HEADS * HEAD_DIM), np.float32)
    vin = rng.standard_normal((BATCH, N_KV_HEADS * HEAD_DIM), np.float32)
    q = rng.standard_normal((BATCH, N_HEADS * HEAD_DIM), np.float32)
    seqs = np.arange(BATCH, dtype=np.uint32)
    phase = 0
    steps = 0
    t0 = time.perf_counter()
    while steps < max_steps:
        pos = (lens + phase).astype(np.uint32)
        rc, done, b, sl = ok.append_batch(seqs, pos)
        assert rc == 0
        ok.write_batch(0, b, sl, kin, vin)
        ok.attend(0, q, seqs, pos, N_HEADS, N_KV_HEADS, HEAD_DIM, n_threads=threads)
        phase += 1
        if phase == CYCLE:
            for i in range(BATCH):
                ok.truncate(i, int(lens[i]))
            phase = 0
        steps += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return BATCH * steps / dt, steps, dt


def cpu_desc():
    try:
        model = [l.split(":", 1)[1].strip() for l in open("/proc/cpuinfo") if l.startswith("model name")][0]
    except Exception:
        model = "unknown CPU"
    return model


def run_reference(args, rank, world):
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    lens = workload(1234)
    # warm-up steps are untimed; each timed step is the full workload (64
    # sequences), bounded to ~60 s in total.
    from oracle import oracle as ok_mod  # noqa: F401  (builds the oracle if needed)

    value, steps, dt = cpu_run(lens, 1234, budget_s=60.0, max_steps=max(args.steps, 1), threads=threads)
    sample = (f"{steps} full steps (64 seqs, one layer: append + f32->f16 write + attention) in {dt:.1f} s, "
              f"{threads} threads on {cpu_desc()}")
    return {
        "impl": "reference",
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": dt * 1e3 / max(steps, 1), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16 storage, f32 arithmetic",
        "data": "synthetic: f16 K/V ~ N(0,1), seeded; lengths U[512,4096] seeded",
        "config": {"workload": "configs[1]: isolated paged decode microbench, Llama-3-8B attention shape, one layer",
                   "batch_per_gpu": BATCH, "ctx": f"U[{CTX_LO},{CTX_HI}]", "n_heads": N_HEADS,
                   "n_kv_heads": N_KV_HEADS, "head_dim": HEAD_DIM, "block_tokens": BLOCK,
                   "implementation": "restated reference CPU path (oracle/lt_oracle.c); the Rust reference is "
                                     "not buildable here"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="CPU-baseline sample budget (rank 0, N=1)")
    args = ap.parse_args()
    rank, world, local = rank_info()
    if args.impl == "reference":
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    res = run_ours(args, rank, world, local)
    if rank == 0 and res is not None:
        if world == 1:
            threads = os.cpu_count() or 1
            value, steps, dt = cpu_run(workload(1234), 1234, budget_s=args.cpu_seconds, max_steps=10 ** 6,
                                       threads=threads)
            res["cpu_baseline"] = {
                "value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                "sample": f"{steps} full steps of the same workload (64 seqs, one layer) in {dt:.1f} s on "
                          f"{threads} threads of {cpu_desc()}; restated reference (oracle/lt_oracle.c)"}
        else:
            res["cpu_baseline"] = None
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
