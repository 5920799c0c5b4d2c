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
import os
import subprocess
import sys
import tempfile
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


def shard_seed(rank: int) -> int:
    """Sequence sharding: every rank owns its own 64 sequences (own lengths,
    own pool, own seed); nothing crosses ranks on the data path."""
    return 1234 + rank


def ensure_pg(world: int, local: int):
    """One NCCL process group for the whole run (every configuration of the
    default line runs in it), with a short timeout so ranks that wait for one
    another end with an error instead of hanging."""
    if world <= 1:
        return
    import datetime

    import torch
    import torch.distributed as dist

    if not dist.is_initialized():
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device(f"cuda:{local}"))


def finish_pg(world: int):
    if world <= 1:
        return
    import torch.distributed as dist

    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


def reduce_max(x: float, device, world: int) -> float:
    """Max over ranks of a per-rank device time (whole-job time of a step)."""
    if world <= 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def fill_plan(lens: np.ndarray, seed: int):
    """(seqs, positions) of the cache fill: each sequence's context in
    16-token pieces, pieces of all sequences randomly interleaved (seed+1) so
    physical block ids are scattered across sequences."""
    rng = np.random.default_rng(seed + 1)
    pieces = np.repeat(np.arange(len(lens)), (lens + BLOCK - 1) // BLOCK)
    rng.shuffle(pieces)
    cur = np.zeros(len(lens), np.int64)
    seqs, pos = [], []
    for s in pieces:
        n = min(BLOCK, int(lens[s] - cur[s]))
        seqs.append(np.full(n, s))
        pos.append(np.arange(cur[s], cur[s] + n))
        cur[s] += n
    return np.concatenate(seqs), np.concatenate(pos)


def workload(seed: int):
    rng = np.random.default_rng(seed)
    lens = rng.integers(CTX_LO, CTX_HI + 1, BATCH)
    return lens


def kv_row_bytes(kv_dim: int, kv_format: str = "f16") -> float:
    """Cached bytes of one K (or V) row: f16 values, or Q8_0 int8 values plus
    one f16 scale per 32."""
    return kv_dim * 2 if kv_format == "f16" else kv_dim * 34 / 32


IO_BYTES = 4  # q, new K/V rows and outputs cross the ABI as f32, the model runner's types (model.rs:393-400)


def step_bytes(lens_now: np.ndarray, kv_format: str = "f16", io_bytes: int = IO_BYTES) -> dict:
    """Algorithmic bytes of one step (one layer) at current lengths `lens_now`
    (after the step's append): K and V of every cached position once, q, out,
    block-table entries, and the appended rows (read in the call's type,
    written in the cached format)."""
    batch = len(lens_now)
    kv_row = kv_row_bytes(N_KV_HEADS * HEAD_DIM, kv_format)  # bytes of one cached K (or V) row
    attn = int(int(lens_now.sum()) * kv_row * 2)
    q = batch * N_HEADS * HEAD_DIM * io_bytes
    out = batch * N_HEADS * HEAD_DIM * io_bytes
    tables = int(((lens_now + BLOCK - 1) // BLOCK).sum()) * 4
    append = int(batch * 2 * (N_KV_HEADS * HEAD_DIM * io_bytes + kv_row))  # read the input row, write the cell
    return {"attn": attn, "q": q, "out": out, "tables": tables, "append": append,
            "total": attn + q + out + tables + append}


def rank_lens(rank: int) -> np.ndarray:
    """Context lengths of a rank's 64 sequences: every rank serves the same
    multiset (configs[1]'s draw), in its own order, so the max over ranks
    measures the system rather than one rank's longer draw."""
    lens = workload(1234)
    return lens if rank == 0 else np.random.default_rng(4321 + rank).permutation(lens)


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(name: str = "paged_attn_c2.md"):
    """DRAM bytes per launch of the attention kernel from a committed ncu
    summary (profiles/<name>, line 'traffic_bytes_per_launch: N')."""
    p = ROOT / "profiles" / name
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
        self.path = Path(tempfile.gettempdir()) / f"lt_bench_clocks_{os.getpid()}.csv"
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


def build_cache(kv_mod, torch, device: int, lens: np.ndarray, seed: int, kv_format: str = "f16"):
    """Fill a cache with the workload: every sequence's context appended in
    16-token pieces in a random interleaving (seed+1), so physical block ids
    are scattered across sequences, then K/V written as f16 N(0,1)."""
    headroom = CYCLE + 1
    n_blocks = int(((lens + headroom + BLOCK - 1) // BLOCK).sum()) + BATCH
    kv = kv_mod.KvCache(1, N_KV_HEADS, HEAD_DIM, n_blocks * BLOCK, n_heads=N_HEADS, max_seqs=BATCH,
                        max_batch=8192, device=device, kv_format=kv_format)
    seqs, pos = fill_plan(lens, seed)
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

    def __init__(self, kv, lens, k, v, q, out, gather: bool = False):
        import ctypes

        import torch

        self.kv, self.lens = kv, lens
        self.seqs = np.arange(len(lens), dtype=np.uint32)
        self.k, self.v, self.q, self.out = k, v, q, out
        self.phase = 0
        self.stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        # head-sharded: the NVLink gather fused into the attention call
        self.attend = kv.write_attend_gather if gather else kv.write_attend

    def step(self, bufs=None, stream=None):
        """bufs: (k, v, q, out) for this step (default: those given at
        construction); stream: a ctypes stream handle (default: the current
        stream at construction)."""
        k, v, q, out = bufs if bufs is not None else (self.k, self.v, self.q, self.out)
        stream = stream if stream is not None else self.stream
        pos = (self.lens + self.phase).astype(np.uint32)
        b, s = self.kv.append_batch(self.seqs, pos, stream=stream)
        self.attend(0, b, s, k, v, q, self.seqs, pos, out=out, stream=stream)
        lens_now = self.lens + self.phase + 1
        self.phase += 1
        if self.phase == CYCLE:
            for i in range(len(self.lens)):
                self.kv.truncate(i, int(self.lens[i]))  # Backend::kv_remove
            self.phase = 0
        return lens_now


def c2_config(world: int, kv_format: str = "f16") -> dict:
    """The `config` of the configs[1] line; both arms print the same dict."""
    lens = workload(1234)
    b = step_bytes(lens + 1, kv_format)
    return {
        "workload": "configs[1]: isolated paged decode microbench, Llama-3-8B attention shape, one layer",
        "batch_per_gpu": BATCH, "ctx": f"U[{CTX_LO},{CTX_HI}]", "n_heads": N_HEADS,
        "n_kv_heads": N_KV_HEADS, "head_dim": HEAD_DIM, "block_tokens": BLOCK,
        "kv_format": kv_format,
        "step": "append 1 token/seq + fused K/V write + decode attention (f32 softmax/accumulate); q, new K/V rows "
                "and outputs in f32, the model runner's types (model.rs:393-400)"
                + ("; K/V cached as Q8_0 (int8 + f16 scale per 32 values)" if kv_format == "q8_0" else ""),
        "kv_bytes_per_step": b["attn"],
        "l2": "inputs larger than L2: ~%.1f GB of K/V read per step vs 126 MB L2" % (b["attn"] / 1e9),
        "parallelism": f"seq-sharded x{world} (independent pools, no collective); every rank serves the same "
                       "multiset of context lengths",
    }


def run_ours(args, rank, world, local):
    import ctypes

    import torch
    import torch.distributed as dist

    from langtrain_studio_b200 import kv as kv_mod

    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    ensure_pg(world, local)
    seed = shard_seed(rank)
    lens = rank_lens(rank)
    kv = build_cache(kv_mod, torch, local, lens, seed, args.kv_format)
    g = torch.Generator(device=dev)
    g.manual_seed(seed + 7)
    # A step's q, new K and new V rows live in one f32 buffer (the model
    # runner's types), so the end-to-end path moves them with one
    # host->device copy; two such buffers (and two outputs) for the
    # pipelined end-to-end loop.
    kvd, qd = N_KV_HEADS * HEAD_DIM, N_HEADS * HEAD_DIM
    width = 2 * kvd + qd
    packed = [torch.randn((BATCH, width), generator=g, device=dev, dtype=torch.float32) for _ in range(2)]

    def split(p):
        flat = p.view(-1)
        return (flat[: BATCH * kvd].view(BATCH, kvd), flat[BATCH * kvd: 2 * BATCH * kvd].view(BATCH, kvd),
                flat[2 * BATCH * kvd:].view(BATCH, qd))

    outs = [torch.empty((BATCH, qd), device=dev, dtype=torch.float32) for _ in range(2)]
    bufs = [split(packed[i]) + (outs[i],) for i in range(2)]
    st = Stepper(kv, lens, *bufs[0])

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
    clocks = Clocks(device_uuid(torch, local))
    time.sleep(0.3)
    kv.profile(True)
    launches0 = kv.launch_count()
    total_bytes = 0
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        lens_now = st.step()
        total_bytes += step_bytes(lens_now, args.kv_format)["total"]
    e1.record()
    barrier()
    ms = e0.elapsed_time(e1)
    launches = kv.launch_count() - launches0
    attn_ms, attn_n = kv.profile_read()
    kv.profile(False)
    clk = clocks.stop()
    kv.check()
    ms_max = reduce_max(ms, dev, world)

    # ---------------- end-to-end through the public API ----------------
    # Every step copies its inputs from pinned host memory and reads its
    # result back on the host.  The copies run on their own streams against
    # double buffers: step t+1's inputs land while step t computes, and the
    # host reads step t's result while step t+1 computes.
    hin = torch.empty((BATCH, width), dtype=torch.float32).pin_memory()
    hin.copy_(packed[0].cpu())
    hout = [torch.empty((BATCH, qd), dtype=torch.float32).pin_memory() for _ in range(2)]
    hout_np = [h.numpy() for h in hout]  # the same pinned bytes, read without a torch call
    s_comp, s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    comp_ptr = ctypes.c_void_p(s_comp.cuda_stream)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def e2e_run(n):
        """n pipelined steps, from host inputs to host results; returns the
        last result the host read."""
        with torch.cuda.stream(s_in):
            s_in.wait_stream(s_comp)
            packed[0].copy_(hin, non_blocking=True)
            ev_in[0].record(s_in)
        last = 0.0
        for t in range(n):
            i = t & 1
            s_comp.wait_event(ev_in[i])  # this step's inputs have landed
            if t >= 2:
                s_comp.wait_event(ev_out[i])  # step t-2's result has left this output buffer
            st.step(bufs[i], comp_ptr)
            ev_comp[i].record(s_comp)
            if t + 1 < n:  # step t+1's inputs, once step t-1 has consumed that buffer
                with torch.cuda.stream(s_in):
                    if t >= 1:
                        s_in.wait_event(ev_comp[i ^ 1])
                    packed[i ^ 1].copy_(hin, non_blocking=True)
                    ev_in[i ^ 1].record(s_in)
            with torch.cuda.stream(s_out):  # step t's result to the host
                s_out.wait_event(ev_comp[i])
                hout[i].copy_(outs[i], non_blocking=True)
                ev_out[i].record(s_out)
            if t >= 1:  # the host reads step t-1's result
                ev_out[i ^ 1].synchronize()
                last = float(hout_np[i ^ 1][0, 0])
        ev_out[(n - 1) & 1].synchronize()
        last = float(hout_np[(n - 1) & 1][0, 0])
        s_comp.wait_stream(s_out)
        return last

    e2e_run(max(args.warmup, 2))
    while st.phase != 0:
        st.step(bufs[0], comp_ptr)
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(s_comp)
    e2e_run(args.steps)
    f1.record(s_comp)
    f1.synchronize()
    barrier()
    e2e_ms = reduce_max(f0.elapsed_time(f1), dev, world)
    h2d = hin.numel() * 4
    d2h = outs[0].numel() * 4
    kv.check()

    result = None
    if rank == 0:
        q8 = args.kv_format == "q8_0"
        peak, peak_kind = measured_peak()
        avg_attn_ms = attn_ms / max(attn_n, 1)
        per_launch_bytes = total_bytes / max(args.steps, 1)
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
            "data": "synthetic: f16 K/V ~ N(0,1), f32 q and new rows ~ N(0,1), seeded; lengths U[512,4096] seeded",
            "config": c2_config(world, args.kv_format),
            "hbm_gbs": total_bytes / (ms_max * 1e-3) / 1e9 * world,
            "roofline": {
                "bound": "hbm",
                "kernel": "paged_attn_kernel<128, %s> (fused append + attention)" % ("q8" if q8 else "f16"),
                "achieved": achieved, "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                "frac": achieved / peak,
                "traffic": ncu_traffic("paged_attn_q8_c2.md" if q8 else "paged_attn_c2.md"),
                "algorithmic_bytes_per_launch": int(per_launch_bytes), "avg_launch_ms": avg_attn_ms,
            },
            "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "how": "KvCache.append_batch + KvCache.write_attend per step; inputs copied from pinned host "
                           "memory and results read back on the host every step, double-buffered on copy "
                           "streams"},
            "gpu_launches": int(launches),
            "clocks": clk,
        }
    kv.close()
    return result


def device_uuid(torch, local: int) -> str:
    try:
        uuid = str(torch.cuda.get_device_properties(local).uuid)
        return uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
    except Exception:
        return str(local)


# ---------------------------------------------------------------------------
# further configurations; run with
# --config c3 / c4-batch / c4-head.  The driver's default line is configs[1].


def _json_common(args, world, metric_value, unit, ms_step, config):
    return {"metric": METRIC, "value": metric_value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic: f16 K/V and q ~ N(0,1), seeded",
            "config": config}


def run_c3(args, rank, world, local):
    """configs[2], prefix-sharing stress: one 2048-token source, 256 sequences
    made with share(src, s, 2047) (the scheduler's cap = len-1 rule), whose
    first append at position 2047 copies the shared partial block (256
    copy-on-write copies in one plan launch), a distinct 256-token suffix
    each, then decode steps of append + fused write/attention over all 256.
    Shared blocks are counted once for the unique-byte roofline."""
    import torch

    from langtrain_studio_b200 import kv as kv_mod

    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    n_seq, prefix, suffix = 256, 2048, 256
    hq, hkv, d = 32, 8, 128
    kvd = hkv * d
    steps, warm = args.steps, args.warmup
    total_dec = steps + warm
    per_seq_blocks = 1 + (suffix + total_dec + 2 + BLOCK - 1) // BLOCK
    n_blocks = prefix // BLOCK + n_seq * per_seq_blocks + 8
    kv = kv_mod.KvCache(1, hkv, d, n_blocks * BLOCK, n_heads=hq, max_seqs=n_seq + 1, max_batch=8192, device=local)
    g = torch.Generator(device=dev)
    g.manual_seed(shard_seed(rank))
    rnd = lambda n: torch.randn((n, kvd), generator=g, device=dev, dtype=torch.float16)
    b, s = kv.append_batch(np.zeros(prefix, np.uint32), np.arange(prefix))
    kv.write(0, b, s, rnd(prefix), rnd(prefix))
    seqs = np.arange(1, n_seq + 1, dtype=np.uint32)
    for i in seqs:
        kv.share(0, int(i), prefix - 1)
    kv.flush()
    torch.cuda.synchronize()
    # divergence: 256 copy-on-write copies of the shared partial block
    c0, c1, c2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    launches0 = kv.launch_count()
    kv.profile(True)  # times the plan launch alone (after its upload)
    c0.record()
    b, s = kv.append_batch(seqs, np.full(n_seq, prefix - 1))  # host bookkeeping: 256 allocations + plan
    c1.record()
    kv.flush()  # the plan: one upload + one apply_plan launch moving 256 blocks
    c2.record()
    torch.cuda.synchronize()
    cow_ms = c0.elapsed_time(c2)
    cow_dev_ms = c1.elapsed_time(c2)
    cow_kernel_ms, cow_kernel_n, cow_blocks, cow_entries = kv.profile_read_plan()
    kv.profile(False)
    cow_launches = kv.launch_count() - launches0
    cow_bytes = n_seq * kvd * 2 * BLOCK * 2 * 2  # K+V block, read + write
    kv.write(0, b, s, rnd(n_seq), rnd(n_seq))
    # distinct suffixes; the K/V write kernel (append of prompt rows,
    # kv.rs:123-131) timed alone: the table entries go first with a flush
    pos = np.arange(prefix, prefix + suffix)
    kv.profile(True)
    for i0 in range(0, n_seq, 32):
        ss = np.repeat(seqs[i0:i0 + 32], suffix)
        pp = np.tile(pos, len(seqs[i0:i0 + 32]))
        b, s = kv.append_batch(ss, pp)
        kv.write(0, b, s, rnd(ss.size), rnd(ss.size))
    w_ms, w_n, w_rows, w_in = kv.profile_read_write()
    kv.profile(False)
    w_bytes = w_in + w_rows * kvd * 2 * 2  # input rows read + f16 cells written, K and V
    lens = np.full(n_seq, prefix + suffix, np.int64)
    k, v = rnd(n_seq), rnd(n_seq)
    q = torch.randn((n_seq, hq * d), generator=g, device=dev, dtype=torch.float16)
    out = torch.empty_like(q)
    shared_blocks = (prefix - 1) // BLOCK  # blocks 0..126 stay shared after the copy

    def step():
        pos = lens.astype(np.uint32)
        b, s = kv.append_batch(seqs, pos)
        kv.write_attend(0, b, s, k, v, q, seqs, pos, out=out)
        lens[:] += 1

    for _ in range(warm):
        step()
    torch.cuda.synchronize()
    kv.profile(True)
    l0 = kv.launch_count()
    uniq = logical = 0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        lens_now = lens + 1
        row = kvd * 2 * 2  # K+V bytes of one position
        logical += int(lens_now.sum()) * row
        uniq += shared_blocks * BLOCK * row + int((lens_now - shared_blocks * BLOCK).sum()) * row
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = reduce_max(e0.elapsed_time(e1), dev, world)
    attn_ms, attn_n = kv.profile_read()
    kv.check()
    extra = n_seq * hq * d * 2 * 2 + n_seq * 2 * kvd * 2 * 2  # q, out, appended rows
    peak, kind = measured_peak()
    per_launch_u = uniq / steps + extra
    achieved = per_launch_u / (attn_ms / attn_n * 1e-3) / 1e9
    res = _json_common(args, world, n_seq * steps * world / (ms * 1e-3), "tokens/s", ms / steps, {
        "workload": "configs[2]: prefix-sharing stress, 256 seqs sharing a 2048-token prefix (share(src, s, 2047)), "
                    "256-token distinct suffixes, decode steps, Llama-3-8B attention shape, one layer"
                    + (f"; an independent replica on each of {world} GPUs" if world > 1 else ""),
        "n_heads": hq, "n_kv_heads": hkv, "head_dim": d, "block_tokens": BLOCK,
        "context_at_start": prefix + suffix})
    res.update({
        "hbm_gbs_unique": (uniq + extra * steps) / (ms * 1e-3) / 1e9,
        "hbm_gbs_logical": (logical + extra * steps) / (ms * 1e-3) / 1e9,
        "roofline": {"bound": "hbm", "kernel": "prefix_attn_kernel<128> (tcgen05, shared prefix) + paged_attn_kernel<128> "
                                                "(own blocks); unique bytes",
                     "achieved": achieved, "peak": peak, "peak_kind": kind, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "algorithmic_bytes_per_launch": int(per_launch_u),
                     "logical_bytes_per_launch": int(logical / steps + extra), "avg_launch_ms": attn_ms / attn_n},
        "cow": {"copies": n_seq, "bytes": cow_bytes, "ms": cow_ms, "gbs": cow_bytes / (cow_ms * 1e-3) / 1e9,
                "plan_ms": cow_dev_ms, "plan_gbs": cow_bytes / (cow_dev_ms * 1e-3) / 1e9, "launches": cow_launches,
                "kernel_ms": cow_kernel_ms, "kernel_gbs": cow_bytes / (cow_kernel_ms * 1e-3) / 1e9,
                "kernel_launches": cow_kernel_n, "kernel_blocks_copied": cow_blocks,
                "kernel_frac_of_peak": cow_bytes / (cow_kernel_ms * 1e-3) / 1e9 / peak,
                "note": "ms/gbs include the host bookkeeping of the 256 appends; plan_* the upload + copy launch; "
                        "kernel_* the apply_plan_kernel launch alone (CUDA events after the upload); bytes: a K+V "
                        "block read and written per copy"},
        "append": {"kernel": "kv_write_kernel<128> (f16 rows in, swizzled f16 cells out)", "rows": w_rows,
                   "launches": w_n, "bytes": w_bytes, "kernel_ms": w_ms,
                   "kernel_gbs": w_bytes / (w_ms * 1e-3) / 1e9,
                   "kernel_frac_of_peak": w_bytes / (w_ms * 1e-3) / 1e9 / peak,
                   "note": "the 256-token suffix rows of 32 sequences per lt_kv_write call (8192 rows, 32 MiB "
                           "read + 32 MiB written), the kernel alone (CUDA events after the cells' upload); decode "
                           "appends are fused into the attention launch"},
        "gpu_launches": kv.launch_count() - l0,
    })
    kv.close()
    return res


def run_prefill(args, rank, world, local):
    """Chunked prefill attention (the reference's prefill chunks,
    scheduler.rs:388-407): 4 sequences with 2048 cached tokens each take a
    256-token prompt chunk per step -- append, K/V write, and causal attention
    of all 1024 chunk tokens in one call (token at position p attends [0, p]).
    The tokens of a sequence share its first 128 blocks, which the tensor-core
    prefix pass attends once per group; the stream-K launch covers each
    token's own blocks.  Each step ends with kv_remove back to 2048 tokens, so
    every step does the same work.  Llama-3-8B attention shape, one layer."""
    import torch

    from langtrain_studio_b200 import kv as kv_mod

    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    n_seq, ctx, chunk = 4, 2048, 256
    hq, hkv, d = 32, 8, 128
    kvd = hkv * d
    n_blocks = n_seq * ((ctx + chunk + BLOCK - 1) // BLOCK) + 8
    kv = kv_mod.KvCache(1, hkv, d, n_blocks * BLOCK, n_heads=hq, max_seqs=n_seq, max_batch=8192, device=local)
    g = torch.Generator(device=dev)
    g.manual_seed(shard_seed(rank))
    rnd = lambda n, w=kvd: torch.randn((n, w), generator=g, device=dev, dtype=torch.float16)
    for sq in range(n_seq):
        b, s = kv.append_batch(np.full(ctx, sq), np.arange(ctx))
        kv.write(0, b, s, rnd(ctx), rnd(ctx))
    seqs = np.repeat(np.arange(n_seq, dtype=np.uint32), chunk)
    pos = np.tile(np.arange(ctx, ctx + chunk, dtype=np.uint32), n_seq)
    n = seqs.size
    k, v, q = rnd(n), rnd(n), rnd(n, hq * d)
    out = torch.empty_like(q)

    def step():
        b, s = kv.append_batch(seqs, pos)
        kv.write(0, b, s, k, v)
        kv.attend(0, q, seqs, pos, out=out)
        for sq in range(n_seq):
            kv.truncate(sq, ctx)  # Backend::kv_remove back to the cached context

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    casc0 = kv.cascade_launches()
    kv.profile(True)
    l0 = kv.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = reduce_max(e0.elapsed_time(e1), dev, world)
    attn_ms, attn_n = kv.profile_read()
    kv.check()
    flops = float(((pos.astype(np.int64) + 1) * hq * d * 4).sum())  # S = QK^T and O = PV, 2 flop per MAC
    uniq = n_seq * (ctx + chunk) * kvd * 2 * 2 + n * (hq * d * 2 * 2 + kvd * 2 * 2)  # K/V once, q, out, new rows
    tf = flops / (attn_ms / attn_n * 1e-3) / 1e12
    with open(ROOT / "MEASURED_PEAKS.json") as f:
        peaks = json.load(f)
    peak_tf = float(peaks.get("bf16_tflops", 1590.0))
    res = _json_common(args, world, n * args.steps * world / (ms * 1e-3), "tokens/s", ms / args.steps, {
        "workload": "chunked prefill: 4 seqs x 2048 cached tokens, a 256-token chunk each per step, "
                    "causal attention of the 1024 chunk tokens in one call, Llama-3-8B attention shape, one layer",
        "n_heads": hq, "n_kv_heads": hkv, "head_dim": d, "block_tokens": BLOCK})
    res.update({
        "roofline": {"bound": "tensor", "kernel": "prefix_attn_kernel<128> (tcgen05) + paged_attn_kernel<128>",
                     "achieved": tf, "peak": peak_tf, "peak_kind": "measured (cuBLAS bf16 GEMM, burst)",
                     "unit": "TFLOP/s", "frac": tf / peak_tf, "traffic": None,
                     "algorithmic_flops_per_launch": flops,
                     "note": "q and P enter the tensor cores as f16 value + f16 residual, so the MMAs carry "
                             "2x these FLOPs",
                     "avg_launch_ms": attn_ms / attn_n},
        "hbm_gbs_unique": uniq / (attn_ms / attn_n * 1e-3) / 1e9,
        "cascade_launches_per_step": (kv.cascade_launches() - casc0) / max(args.steps, 1),
        "gpu_launches": kv.launch_count() - l0,
    })
    kv.close()
    return res


def run_c4(args, rank, world, local, mode):
    """configs[3], long-context decode at the Llama-3-70B attention shape (64 q
    heads, 8 KV heads, head_dim 128): 16 sequences of 32768 tokens.
      batch: sequences sharded across ranks (16/N each), no collective;
      head:  KV heads sharded across ranks (8/N each), bookkeeping replicated,
             the per-head attention outputs gathered every step: by default
             inside the attention call (NVLink peer stores, lt_kv_*_gather),
             with --gather nccl by a separate NCCL all-gather + permute."""
    import datetime

    import torch
    import torch.distributed as dist

    from langtrain_studio_b200 import kv as kv_mod

    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    ensure_pg(world, local)
    B, L, hq, hkv, d = 16, 32768, 64, 8, 128
    # --emulate-ranks R on one GPU: the work of one rank of an R-GPU run (no
    # collective), to time the per-rank launch that R GPUs would each run
    split = world if world > 1 else max(1, getattr(args, "emulate_ranks", 1))
    if mode == "batch":
        assert B % split == 0
        n_seq, my_hkv, my_hq = B // split, hkv, hq
    else:
        assert hkv % split == 0
        n_seq, my_hkv, my_hq = B, hkv // split, hq // split
    kvd = my_hkv * d
    n_blocks = n_seq * ((L + CYCLE + 1 + BLOCK - 1) // BLOCK) + 8
    kv = kv_mod.KvCache(1, my_hkv, d, n_blocks * BLOCK, n_heads=my_hq, max_seqs=n_seq, max_batch=8192, device=local,
                        kv_format=args.kv_format)
    g = torch.Generator(device=dev)
    g.manual_seed(shard_seed(rank))
    chunk = 8192
    for sq in range(n_seq):
        for p0 in range(0, L, chunk):
            b, s = kv.append_batch(np.full(chunk, sq), np.arange(p0, p0 + chunk))
            kv.write(0, b, s, torch.randn((chunk, kvd), generator=g, device=dev, dtype=torch.float16),
                     torch.randn((chunk, kvd), generator=g, device=dev, dtype=torch.float16))
    lens = np.full(n_seq, L, np.int64)
    seqs = np.arange(n_seq, dtype=np.uint32)
    k = torch.randn((n_seq, kvd), generator=g, device=dev, dtype=torch.float16)
    v = torch.randn((n_seq, kvd), generator=g, device=dev, dtype=torch.float16)
    q = torch.randn((n_seq, my_hq * d), generator=g, device=dev, dtype=torch.float16)
    out = torch.empty_like(q)
    comm = None
    peer = mode == "head" and world > 1 and args.gather == "peer"
    if mode == "head" and world > 1 and not peer:
        uid = [kv_mod.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = kv_mod.NcclComm(world, uid[0], rank, local)
        gathered = torch.empty((world, n_seq, my_hq * d), device=dev, dtype=torch.float16)
        full = torch.empty((n_seq, world * my_hq * d), device=dev, dtype=torch.float16)
    if peer:
        kv_mod.setup_peer_gather(kv, rank, world, max_tokens=n_seq)
        out = torch.empty((n_seq, world * my_hq * d), device=dev, dtype=torch.float16)
    st = Stepper(kv, lens, k, v, q, out, gather=peer)

    def step():
        lens_now = st.step()
        if comm is not None:  # NCCL all-gather + permute to [seq][all heads * D]
            kv_mod.gather_heads(kv, out, comm, out=full, gathered=gathered, stream=st.stream)
        return lens_now

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    while st.phase != 0:
        step()
    kv.profile(True)
    l0 = kv.launch_count()
    byts = 0
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        lens_now = step()
        row = kv_row_bytes(kvd, args.kv_format)
        byts += int(int(lens_now.sum()) * row * 2 + n_seq * (my_hq * d * 2 * 2 + 2 * (kvd * 2 + row)))
    e1.record()
    barrier()
    ms = reduce_max(e0.elapsed_time(e1), dev, world)
    attn_ms, attn_n = kv.profile_read()
    kv.check()
    peak, kind = measured_peak()
    achieved = byts / args.steps / (attn_ms / attn_n * 1e-3) / 1e9
    res = None
    if rank == 0:
        res = _json_common(args, world, B * args.steps / (ms * 1e-3), "tokens/s", ms / args.steps, {
            "workload": f"configs[3]: long-context decode, Llama-3-70B attention shape, 16 seqs x 32768 tokens, "
                        f"{mode}-sharded x{world}, one layer",
            "n_heads": hq, "n_kv_heads": hkv, "head_dim": d, "block_tokens": BLOCK, "kv_format": args.kv_format,
            "per_rank": {"seqs": n_seq, "kv_heads": my_hkv, "q_heads": my_hq},
            "emulated_ranks": split if world == 1 else None,
            "collective": ("lt_kv_write_attend_gather: outputs stored to every rank over NVLink by the attention "
                           "kernel, flag wait + copy" if peer else
                           "lt_kv_gather_heads: NCCL all-gather of [seqs, q_heads*D] f16 per step + permute")
            if mode == "head" and world > 1 else "none"})
        res["scaling"] = "strong" if mode == "head" else "weak"
        res["hbm_gbs_per_gpu"] = byts / args.steps / (ms / args.steps * 1e-3) / 1e9
        res["roofline"] = {"bound": "hbm", "kernel": "paged_attn_kernel<128> (rank 0)",
                           "achieved": achieved, "peak": peak, "peak_kind": kind, "unit": "GB/s",
                           "frac": achieved / peak, "traffic": None,
                           "algorithmic_bytes_per_launch": int(byts / args.steps), "avg_launch_ms": attn_ms / attn_n}
        res["gpu_launches"] = kv.launch_count() - l0
    if world > 1:
        if peer:
            kv.peer_close()  # every rank unmaps the others' buffers before any is freed
        dist.barrier()
        if comm is not None:
            comm.close()
    kv.close()
    return res


class Arrivals:
    """The configs[4] request process: Poisson(lam) arrivals per step, prompt
    lengths log-uniform in [lo, hi], output lengths uniform in [olo, ohi]."""

    def __init__(self, lam, seed, lo=64, hi=8192, olo=16, ohi=512):
        self.rng = np.random.default_rng(seed)
        self.lam, self.lo, self.hi, self.olo, self.ohi = lam, lo, hi, olo, ohi

    def step(self):
        out = []
        for _ in range(self.rng.poisson(self.lam)):
            prompt = int(np.exp(self.rng.uniform(np.log(self.lo), np.log(self.hi))))
            out.append((prompt, int(self.rng.integers(self.olo, self.ohi + 1))))
        return out


PREFILL_CHUNK = 256


def run_c5(args, rank, world, local):
    """continuous-batching churn, Llama-3-8B attention shape, one
    layer; arrivals Poisson(32/N) per rank and step (sequence-sharded), prompts
    log-uniform in [64, 8192], outputs U[16, 512], block pool at 60 % of the
    peak demand of an uncapped dry run.  The scheduler policy runs in the
    native driver (lt_sched): admission, LRU eviction, preemption, chunked
    prefill, retire, compaction every step."""
    import datetime

    import torch
    import torch.distributed as dist

    from langtrain_studio_b200 import kv as kv_mod
    from langtrain_studio_b200.sched import Scheduler

    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    ensure_pg(world, local)
    lam = args.c5_rate / world
    seed = shard_seed(rank)
    hq, hkv, d = 32, 8, 128
    # uncapped dry run of the same arrival/length process: peak blocks held by running sequences
    dry = Arrivals(lam, seed + 101)
    live, peak = [], 0
    for _ in range(args.warmup + args.steps):
        for prompt, out_len in dry.step():
            live.append([prompt, prompt + out_len, 0])
        nxt = []
        for r in live:  # [prompt, total, n_past]
            r[2] = min(r[2] + PREFILL_CHUNK, r[0]) if r[2] < r[0] else r[2] + 1
            if r[2] < r[1]:
                nxt.append(r)
        live = nxt
        peak = max(peak, sum((r[2] + BLOCK - 1) // BLOCK for r in live))
    pool = max(int(0.6 * peak), 64)
    n_slots = 16384
    max_blocks = (8192 + 512 + 2 * BLOCK) // BLOCK
    kv = kv_mod.KvCache(1, hkv, d, pool * BLOCK, n_heads=hq, max_seqs=n_slots, max_batch=1 << 17,
                        max_blocks_per_seq=max_blocks, device=local)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    kv_src = torch.randn((1 << 17, hkv * d), generator=g, device=dev, dtype=torch.float16)
    q_src = torch.randn((n_slots, hq * d), generator=g, device=dev, dtype=torch.float16)
    out = torch.empty((n_slots, hq * d), device=dev, dtype=torch.float16)
    sched = Scheduler(kv, n_slots)
    arrivals = Arrivals(lam, seed + 101)

    def step():
        for prompt, out_len in arrivals.step():
            sched.submit(prompt, out_len)
        sched.step(kv_src, q_src, out)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s0 = sched.stats
    kv.profile(True)
    l0 = kv.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    if world > 1:
        dist.barrier()
    ms = reduce_max(e0.elapsed_time(e1), dev, world)
    attn_ms, attn_n = kv.profile_read()
    plan_ms, plan_n, plan_blocks, plan_entries = kv.profile_read_plan()
    kv.check()
    s1 = sched.stats
    delta = {k: s1[k] - s0[k] for k in s1}
    tot = torch.tensor([float(delta["decode_tokens"]), float(delta["prefill_tokens"]), float(delta["moved_blocks"])],
                       device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(tot)
    res = None
    if rank == 0:
        moved_bytes = tot[2].item() * hkv * d * 2 * BLOCK * 2 * 2  # K+V block, read + write
        res = _json_common(args, world, tot[0].item() / (ms * 1e-3), "tokens/s", ms / args.steps, {
            "workload": "configs[4]: continuous-batching churn, Llama-3-8B attention shape, one layer, "
                        f"Poisson({args.c5_rate:g}) arrivals/step over {world} rank(s), prompts log-U[64,8192], "
                        "outputs U[16,512], pool 60% of peak demand, compaction every step",
            "n_heads": hq, "n_kv_heads": hkv, "head_dim": d, "block_tokens": BLOCK,
            "pool_blocks_per_rank": pool, "parallelism": f"seq-sharded x{world}"})
        res.update({
            "decode_tokens_per_s": tot[0].item() / (ms * 1e-3),
            "prefill_tokens_per_s": tot[1].item() / (ms * 1e-3),
            "rank0": {"steps": args.steps, "decode": delta["decode_tokens"], "prefill": delta["prefill_tokens"],
                      "admitted": delta["admitted"], "finished": delta["finished"], "evicted": delta["evicted"],
                      "preempted": delta["preempted"], "moved_blocks": delta["moved_blocks"],
                      "running_at_end": s1["running"], "queued_at_end": s1["queued"],
                      "attn_ms_per_step": attn_ms / max(attn_n, 1), "host_wall_ms_per_step": wall * 1e3 / args.steps},
            "compaction_gb_moved_per_s": moved_bytes / (ms * 1e-3) / 1e9,
            "plan_kernel": {"kernel": "apply_plan_kernel (compaction moves + block-table entries), rank 0",
                            "launches": plan_n, "ms_per_step": plan_ms / args.steps, "blocks_copied": plan_blocks,
                            "table_entries": plan_entries,
                            "gbs": (plan_blocks * hkv * d * 2 * BLOCK * 2 * 2 + plan_entries * 8)
                            / max(plan_ms * 1e-3, 1e-12) / 1e9},
            "mean_context_per_decode_token": delta["attended_positions"] / max(delta["decode_tokens"], 1),
            "gpu_launches": kv.launch_count() - l0,
        })
        # Rank 0's decode attention launches: K+V rows of every attended
        # position, q and out rows, and the fused append (source read + row write).
        kvd = hkv * d
        attn_bytes = (delta["attended_positions"] * kvd * 2 * 2 + delta["decode_tokens"] * hq * d * 2 * 2
                      + delta["decode_tokens"] * kvd * 2 * 2 * 2)
        if attn_n:
            per_launch = attn_bytes / attn_n
            achieved = per_launch / (attn_ms / attn_n * 1e-3) / 1e9
            peak, kind = measured_peak()
            res["roofline"] = {"bound": "hbm", "kernel": "paged_attn_kernel<128> (fused append + decode attention, "
                                                          "rank 0)",
                               "achieved": achieved, "peak": peak, "peak_kind": kind, "unit": "GB/s",
                               "frac": achieved / peak, "traffic": None,
                               "algorithmic_bytes_per_launch": int(per_launch), "avg_launch_ms": attn_ms / attn_n}
    sched.close()
    if world > 1:
        dist.barrier()
    kv.close()
    return res


# ---------------------------------------------------------------------------
# CPU arm (restated reference path)


# ---------------------------------------------------------------------------
# the end-to-end Llama decode (--config c1)

C1_SHAPE = dict(n_layers=22, dim=2048, n_heads=32, n_kv_heads=4, head_dim=64, ffn_dim=5632, vocab=32000)
C1_SEQS, C1_PROMPT, C1_SHARED = 4, 128, 64


def c1_prompts(vocab: int, seed: int = 0) -> np.ndarray:
    """4 uniform-random prompts of 128 ids whose first 64 are shared."""
    rng = np.random.default_rng(seed)
    common = rng.integers(0, vocab, C1_SHARED)
    return np.stack([np.concatenate([common, rng.integers(0, vocab, C1_PROMPT - C1_SHARED)])
                     for _ in range(C1_SEQS)]).astype(np.int32)


def run_c1(args, rank, world, local):
    """configs[0] on the device: random-init Llama (22 layers, hidden 2048,
    32/4 heads, head_dim 64, FFN 5632, vocab 32000, Q8_0), 4 sequences whose
    128-token prompts share their first 64 tokens (sequence 0 prefilled,
    share(0, s, 64), the suffixes prefilled in one batch), then greedy decode
    steps of 4 tokens.  value: decode steps queued back to back on the device
    (forward + argmax, token ids not fed back: the work does not depend on
    them); e2e: the greedy loop through lt_llama_step_greedy, host ids in and
    out every step.  Roofline: the Q8_0 matmul kernel against HBM."""
    import torch
    import torch.distributed as dist

    from langtrain_studio_b200 import llama as LL

    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    ensure_pg(world, local)
    seed = shard_seed(rank)
    model = LL.Llama(**C1_SHAPE, max_batch=256, device=local)
    model.load(LL.random_weights(model, seed=seed))
    steps, warm = args.steps, args.warmup
    e2e_steps = steps
    n_prof = min(steps, 100)
    per_seq = C1_PROMPT + warm + 2 * steps + n_prof + 2 * BLOCK  # positions every sequence reaches
    kv = model.kv_cache(C1_SEQS * per_seq, C1_SEQS)
    prompts = c1_prompts(model.vocab, seed)
    seqs = np.arange(C1_SEQS, dtype=np.uint32)
    first = model.step_greedy(kv, prompts[0], np.zeros(C1_PROMPT), np.arange(C1_PROMPT), [C1_PROMPT - 1])
    for s_ in range(1, C1_SEQS):
        kv.share(0, s_, C1_SHARED)
    m = C1_PROMPT - C1_SHARED
    rest = model.step_greedy(kv, prompts[1:, C1_SHARED:].reshape(-1), np.repeat(seqs[1:], m),
                             np.tile(np.arange(C1_SHARED, C1_PROMPT), C1_SEQS - 1),
                             [(i + 1) * m - 1 for i in range(C1_SEQS - 1)])
    cur = np.concatenate([first, rest]).astype(np.int32)
    pos = C1_PROMPT
    logits = torch.empty((C1_SEQS, model.vocab), dtype=torch.float32, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def queued_step():
        nonlocal pos
        model.forward(kv, cur, seqs, np.full(C1_SEQS, pos), seqs, logits=logits)
        LL.argmax_rows(logits)
        pos += 1

    for _ in range(warm):
        queued_step()
    try:
        uuid = str(torch.cuda.get_device_properties(local).uuid)
        dev_id = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
    except Exception:
        dev_id = str(local)
    clocks = Clocks(dev_id)
    time.sleep(0.3)
    l0 = model.launch_count() + kv.launch_count()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        queued_step()
    e1.record()
    barrier()
    ms = e0.elapsed_time(e1)
    launches = model.launch_count() + kv.launch_count() - l0 + steps  # + one argmax per step
    clk = clocks.stop()
    ms_max = reduce_max(ms, dev, world)
    # matmul roofline: the same steps with an event pair around each matmul
    model.profile(True)
    mm_ms = mm_n = mm_bytes = 0
    for _ in range(n_prof):
        queued_step()
        a, b_, c_ = model.profile_read()
        mm_ms, mm_n, mm_bytes = mm_ms + a, mm_n + b_, mm_bytes + c_
    model.profile(False)
    # e2e: the greedy loop, ids to the host and back every step
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        cur = model.step_greedy(kv, cur, seqs, np.full(C1_SEQS, pos), seqs)
        pos += 1
    barrier()
    e2e_ms = reduce_max((time.perf_counter() - t0) * 1e3, dev, world)
    result = None
    if rank == 0:
        peak, peak_kind = measured_peak()
        tokens = C1_SEQS * steps * world
        achieved = mm_bytes / (mm_ms * 1e-3) / 1e9
        result = _json_common(args, world, tokens / (ms_max * 1e-3), "tokens/s", ms_max / steps, {
            "workload": "configs[0]: end-to-end greedy decode, random-init Llama 22 layers / hidden 2048 / 32 q, "
                        "4 KV heads / head_dim 64 / FFN 5632 / vocab 32000, Q8_0 weights; 4 sequences, 128-token "
                        "prompts with the first 64 shared via share(0, s, 64)",
            "batch_per_gpu": C1_SEQS, "parallelism": f"replicas x{world} (independent models and caches)",
            "context_at_start": C1_PROMPT, "l2": "inputs larger than L2: 1.16 GB of weights read per step"})
        result.update({
            "dtype": "int8 x int8 -> int32 (Q8_0 matmuls), f32 elsewhere, f16 KV",
            "data": "synthetic: random-init Q8_0 weights (seeded), uniform-random prompt ids (seeded)",
            "roofline": {"bound": "hbm",
                         "kernel": ("decode_kernel<64> (persistent: every layer's matmuls, norms, RoPE, K/V append "
                                    "and attention, the output matrix and the pick in one launch per step)"
                                    if model.persistent_available() else
                                    "q8_gemv_kernel (all projections and the output matrix)"),
                         "achieved": achieved, "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": None,
                         "algorithmic_bytes_per_launch": int(mm_bytes / max(mm_n, 1)),
                         "avg_launch_ms": mm_ms / max(mm_n, 1), "launches_per_step": mm_n / max(n_prof, 1),
                         "matmul_ms_per_step": mm_ms / max(n_prof, 1)},
            "e2e": {"value": C1_SEQS * e2e_steps * world / (e2e_ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": 256 * 8 + C1_SEQS * (C1_SHAPE["head_dim"] // 2) * 8,
                    "d2h_bytes_per_step": C1_SEQS * 4},
            "gpu_launches": int(launches),
            "clocks": clk,
        })
    if world > 1:
        dist.barrier()
    kv.close()
    model.close()
    return result


def cpu_run_c1(budget_s: float, threads: int, seed: int = 0):
    """The restated reference forward (oracle/lt_model.c) on `threads` host
    threads: prefill as configs[0] (untimed), then greedy decode steps of 4
    tokens until `budget_s`.  Returns (tokens/s, steps, seconds)."""
    from oracle import model as om

    model = om.OracleModel(**{k: C1_SHAPE[k] for k in ("dim", "n_layers", "n_heads", "n_kv_heads", "head_dim",
                                                        "ffn_dim", "vocab")}, seed=seed)
    kv = model.oracle_kv(C1_SEQS * 1024, C1_SEQS)
    prompts = c1_prompts(model.vocab, seed)
    lg = model.forward(kv, prompts[0], np.zeros(C1_PROMPT), np.arange(C1_PROMPT), [C1_PROMPT - 1], threads)
    first = model.argmax(lg)
    for s_ in range(1, C1_SEQS):
        kv.share(0, s_, C1_SHARED)
    m = C1_PROMPT - C1_SHARED
    lg = model.forward(kv, prompts[1:, C1_SHARED:].reshape(-1), np.repeat(np.arange(1, C1_SEQS), m),
                       np.tile(np.arange(C1_SHARED, C1_PROMPT), C1_SEQS - 1),
                       [(i + 1) * m - 1 for i in range(C1_SEQS - 1)], threads)
    cur = np.concatenate([first, model.argmax(lg)])
    pos, steps = C1_PROMPT, 0
    t0 = time.perf_counter()
    while steps < 1000 - C1_PROMPT:
        lg = model.forward(kv, cur, np.arange(C1_SEQS), np.full(C1_SEQS, pos), np.arange(C1_SEQS), threads)
        cur = model.argmax(lg)
        pos += 1
        steps += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return C1_SEQS * steps / dt, steps, dt


def cpu_fill(ok_mod, lens, seed, kv_format="f16"):
    n_blocks = int(((lens + CYCLE + 1 + BLOCK - 1) // BLOCK).sum()) + BATCH
    ok = ok_mod.OracleKv(1, N_KV_HEADS * HEAD_DIM, n_blocks * BLOCK, max_seqs=BATCH, kv_format=kv_format)
    seqs, pos = fill_plan(lens, seed)
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


def cpu_run(lens, seed, budget_s, max_steps, threads, kv_format="f16"):
    """Time the restated reference step (append + write + attention over every
    sequence, model.rs:380-476) on `threads` host threads.  Steps run until
    `budget_s` seconds or `max_steps`; returns (tokens/s, steps, seconds)."""
    from oracle import oracle as ok_mod

    ok = cpu_fill(ok_mod, lens, seed, kv_format)
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


def cpu_run_c3(budget_s: float, threads: int, max_steps: int = 64):
    """configs[2] on the restated reference path: a 2048-token source, 256
    sequences made by share(src, s, 2047), their first appends (256
    copy-on-write copies), 256 distinct suffix tokens each, then timed decode
    steps (append + f32 write + attention of all 256) until `budget_s`.  The
    reference attends every token over its whole context (model.rs:431-476),
    shared blocks included.  Returns (tokens/s, steps, seconds)."""
    from oracle import oracle as ok_mod

    n_seq, prefix, suffix = 256, 2048, 256
    kvd = N_KV_HEADS * HEAD_DIM
    per_seq_blocks = 1 + (suffix + max_steps + 2 + BLOCK - 1) // BLOCK
    n_blocks = prefix // BLOCK + n_seq * per_seq_blocks + 8
    ok = ok_mod.OracleKv(1, kvd, n_blocks * BLOCK, max_seqs=n_seq + 1)
    rng = np.random.default_rng(1234)
    rows = lambda n: rng.standard_normal((n, kvd), np.float32).astype(np.float16)  # noqa: E731

    def put(seqs, pos):
        rc, done, b, sl = ok.append_batch(seqs, pos)
        assert rc == 0
        ok.write_batch(0, b, sl, rows(b.size), rows(b.size))

    put(np.zeros(prefix, np.uint32), np.arange(prefix))
    seqs = np.arange(1, n_seq + 1, dtype=np.uint32)
    for i in seqs:
        ok.share(0, int(i), prefix - 1)
    put(seqs, np.full(n_seq, prefix - 1))
    for i0 in range(0, n_seq, 32):
        ss = seqs[i0:i0 + 32]
        put(np.repeat(ss, suffix), np.tile(np.arange(prefix, prefix + suffix), ss.size))
    lens = np.full(n_seq, prefix + suffix, np.int64)
    kin = rng.standard_normal((n_seq, kvd), np.float32)
    vin = rng.standard_normal((n_seq, kvd), np.float32)
    q = rng.standard_normal((n_seq, N_HEADS * HEAD_DIM), np.float32)
    steps = 0
    t0 = time.perf_counter()
    while steps < max_steps:
        pos = lens.astype(np.uint32)
        rc, done, b, sl = ok.append_batch(seqs, pos)
        assert rc == 0
        ok.write_batch(0, b, sl, kin, vin)
        ok.attend(0, q, seqs, pos, N_HEADS, N_KV_HEADS, HEAD_DIM, n_threads=threads)
        lens += 1
        steps += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return n_seq * steps / dt, steps, dt


def cpu_run_c4(budget_s: float, threads: int, max_steps: int = 64):
    """configs[3] (16 x 32768, 64 q / 8 KV heads) on the restated reference
    path: the cache filled in 8192-token appends (rows tiled from one
    8192-row N(0,1) draw: the arithmetic per position is the same for any
    values), then timed decode steps of append + f32 write + attention, with
    kv_remove back to 32768 every 16 steps.  Returns (tokens/s, steps, s)."""
    from oracle import oracle as ok_mod

    B, L, hq, hkv, d = 16, 32768, 64, 8, 128
    kvd = hkv * d
    n_blocks = B * ((L + CYCLE + 1 + BLOCK - 1) // BLOCK) + 8
    ok = ok_mod.OracleKv(1, kvd, n_blocks * BLOCK, max_seqs=B)
    rng = np.random.default_rng(1234)
    chunk = 8192
    kc = rng.standard_normal((chunk, kvd), np.float32).astype(np.float16)
    vc = rng.standard_normal((chunk, kvd), np.float32).astype(np.float16)
    for sq in range(B):
        for p0 in range(0, L, chunk):
            rc, done, b, sl = ok.append_batch(np.full(chunk, sq), np.arange(p0, p0 + chunk))
            assert rc == 0
            ok.write_batch(0, b, sl, kc, vc)
    kin = rng.standard_normal((B, kvd), np.float32)
    vin = rng.standard_normal((B, kvd), np.float32)
    q = rng.standard_normal((B, hq * d), np.float32)
    seqs = np.arange(B, dtype=np.uint32)
    phase = steps = 0
    t0 = time.perf_counter()
    while steps < max_steps:
        pos = np.full(B, L + phase, np.uint32)
        rc, done, b, sl = ok.append_batch(seqs, pos)
        assert rc == 0
        ok.write_batch(0, b, sl, kin, vin)
        ok.attend(0, q, seqs, pos, hq, hkv, d, n_threads=threads)
        phase += 1
        if phase == CYCLE:
            for sq in range(B):
                ok.truncate(sq, L)
            phase = 0
        steps += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return B * steps / dt, steps, dt


def cpu_run_prefill(budget_s: float, threads: int, max_steps: int = 16):
    """The chunked-prefill line on the restated reference path: 4 sequences
    of 2048 cached tokens, each step a 256-token chunk per sequence (append +
    f32 write + causal attention of the 1024 chunk tokens), then kv_remove
    back to 2048.  Returns (prompt tokens/s, steps, seconds)."""
    from oracle import oracle as ok_mod

    n_seq, ctx, chunk = 4, 2048, 256
    kvd = N_KV_HEADS * HEAD_DIM
    n_blocks = n_seq * ((ctx + chunk + BLOCK - 1) // BLOCK) + 8
    ok = ok_mod.OracleKv(1, kvd, n_blocks * BLOCK, max_seqs=n_seq)
    rng = np.random.default_rng(1234)
    for sq in range(n_seq):
        rc, done, b, sl = ok.append_batch(np.full(ctx, sq), np.arange(ctx))
        assert rc == 0
        ok.write_batch(0, b, sl, rng.standard_normal((ctx, kvd), np.float32).astype(np.float16),
                       rng.standard_normal((ctx, kvd), np.float32).astype(np.float16))
    seqs = np.repeat(np.arange(n_seq, dtype=np.uint32), chunk)
    pos = np.tile(np.arange(ctx, ctx + chunk, dtype=np.uint32), n_seq)
    n = seqs.size
    kin = rng.standard_normal((n, kvd), np.float32)
    vin = rng.standard_normal((n, kvd), np.float32)
    q = rng.standard_normal((n, N_HEADS * HEAD_DIM), np.float32)
    steps = 0
    t0 = time.perf_counter()
    while steps < max_steps:
        rc, done, b, sl = ok.append_batch(seqs, pos)
        assert rc == 0
        ok.write_batch(0, b, sl, kin, vin)
        ok.attend(0, q, seqs, pos, N_HEADS, N_KV_HEADS, HEAD_DIM, n_threads=threads)
        for sq in range(n_seq):
            ok.truncate(sq, ctx)
        steps += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return n * steps / dt, steps, dt


def cpu_desc():
    try:
        model = [l.split(":", 1)[1].strip() for l in open("/proc/cpuinfo") if l.startswith("model name")][0]
    except Exception:
        model = "unknown CPU"
    return model


def _sub_args(args, **kw):
    ns = argparse.Namespace(**vars(args))
    ns.__dict__.update(kw)
    return ns


# The other configurations of BASELINE.json, run after the headline in the
# same process at step counts that keep the whole line within a few minutes:
# key -> (runner, CPU-baseline leg for rank 0 at N = 1).
def _sub_q8(args, rank, world, local):
    return run_ours(_sub_args(args, kv_format="q8_0"), rank, world, local)


def _sub_c3(args, rank, world, local):
    return run_c3(_sub_args(args, steps=32, warmup=5), rank, world, local)


def _sub_c4(mode):
    return lambda args, rank, world, local: run_c4(_sub_args(args, steps=32, warmup=16), rank, world, local, mode)


def _sub_c5(args, rank, world, local):
    return run_c5(_sub_args(args, steps=60, warmup=500 if world == 1 else 400), rank, world, local)


def _sub_c1(args, rank, world, local):
    return run_c1(_sub_args(args, steps=32, warmup=8), rank, world, local)


def _sub_prefill(args, rank, world, local):
    return run_prefill(_sub_args(args, steps=20, warmup=3), rank, world, local)


def _cpu_leg(name, res, budget, threads):
    """cpu_baseline of one sub-configuration: the restated reference path on
    a bounded sample of the same workload."""
    how = f"{threads} threads of {cpu_desc()}"
    if name == "q8":
        v, n, dt = cpu_run(workload(1234), 1234, budget, 10 ** 6, threads, kv_format="q8_0")
        sample = f"{n} full steps (64 seqs, one layer, Q8_0 cache) in {dt:.1f} s on {how}"
    elif name == "c3":
        v, n, dt = cpu_run_c3(budget, threads)
        sample = (f"{n} decode steps of all 256 sequences after the untimed build (prefix, 256 shares and "
                  f"copy-on-write copies, suffixes) in {dt:.1f} s on {how}")
    elif name == "c4_batch":
        v, n, dt = cpu_run_c4(budget, threads)
        sample = f"{n} decode steps of all 16 sequences (32768 tokens, 64/8 heads) in {dt:.1f} s on {how}"
    elif name == "c5":
        ctx = int(round(res["mean_context_per_decode_token"]))
        lens = np.full(BATCH, max(ctx - 8, 1), np.int64)  # a 16-step cycle attends lens + 1 .. lens + 16
        v, n, dt = cpu_run(lens, 1234, budget, 10 ** 6, threads)
        sample = (f"{n} steps of 64 decode tokens at the GPU run's mean attended context per decode token "
                  f"({ctx} positions; the churn's prefill chunks are not timed) in {dt:.1f} s on {how}")
    elif name == "c1":
        v, n, dt = cpu_run_c1(budget, threads)
        sample = f"{n} greedy decode steps of 4 tokens after an untimed prefill, {dt:.1f} s on {how}"
    elif name == "prefill":
        v, n, dt = cpu_run_prefill(budget, threads)
        sample = f"{n} steps of 4 x 256 prompt tokens over 2048 cached tokens in {dt:.1f} s on {how}"
    else:
        return None
    return {"value": v, "unit": res.get("unit", "tokens/s"), "cores": threads, "kind": "port",
            "sample": sample + "; restated reference (oracle/)"}


SUB_RUNNERS = {"q8": _sub_q8, "c3": _sub_c3, "c4_batch": _sub_c4("batch"), "c4_head": _sub_c4("head"),
               "c5": _sub_c5, "prefill": _sub_prefill, "c1": _sub_c1}


def run_subconfigs(args, rank, world, local) -> dict:
    """Every other configuration, one after the other on every rank (the same
    collective calls in the same order), each summarised under its key.
    c4_head is the KV-head-sharded long-context mode; on one GPU it is the
    same launch as c4_batch and is left out."""
    import torch

    names = list(SUB_RUNNERS) if args.sub == "all" else [n for n in args.sub.split(",") if n]
    out = {}
    threads = os.cpu_count() or 1
    for name in names:
        if name not in SUB_RUNNERS or (name == "c4_head" and world == 1):
            continue
        t0 = time.perf_counter()
        try:
            res = SUB_RUNNERS[name](args, rank, world, local)
        except Exception as e:  # recorded, and the other configurations still run
            res = {"error": f"{type(e).__name__}: {e}"}
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        if rank != 0 or res is None:
            continue
        res = {k: v for k, v in res.items() if k not in ("metric", "higher_is_better", "vs_baseline")}
        res["gpu_run_s"] = round(time.perf_counter() - t0, 2)
        res["cpu_baseline"] = None
        if world == 1 and args.cpu_seconds > 0 and "error" not in res:
            try:
                res["cpu_baseline"] = _cpu_leg(name, res, min(args.cpu_seconds, 8.0), threads)
            except Exception as e:
                res["cpu_baseline"] = {"error": f"{type(e).__name__}: {e}"}
        out[name] = res
    return out


def run_reference(args, rank, world):
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    if args.config == "c1":
        value, steps, dt = cpu_run_c1(60.0, threads)
        sample = (f"{steps} greedy decode steps of 4 tokens after an untimed prefill, {dt:.1f} s on {threads} "
                  f"threads of {cpu_desc()}; restated reference forward (oracle/lt_model.c)")
        return {
            "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": steps, "warmup": 0, "ms_per_step": dt * 1e3 / max(steps, 1), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8 x int8 -> int32 (Q8_0 matmuls), f32, f16 KV",
            "data": "synthetic: random-init Q8_0 weights (seeded), uniform-random prompt ids (seeded)",
            "config": {"workload": "configs[0]: end-to-end greedy decode, random-init Llama (22 layers, Q8_0), "
                                   "4 sequences, 64 shared prompt tokens", "batch_per_gpu": C1_SEQS,
                       "implementation": "restated reference CPU forward (oracle/lt_model.c); the Rust reference "
                                         "is not buildable here"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
    lens = workload(1234)
    # warm-up steps are untimed; each timed step is the full workload (64
    # sequences), bounded to ~60 s in total.
    from oracle import oracle as ok_mod  # noqa: F401  (builds the oracle if needed)

    if args.warmup > 0:
        cpu_run(lens, 1234, budget_s=30.0, max_steps=args.warmup, threads=threads)  # untimed warm-up
    value, steps, dt = cpu_run(lens, 1234, budget_s=60.0, max_steps=max(args.steps, 1), threads=threads)
    sample = (f"{steps} full steps (64 seqs, one layer: append + f32->f16 write + attention) in {dt:.1f} s, "
              f"{threads} threads on {cpu_desc()}")
    return {
        "impl": "reference",
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": dt * 1e3 / max(steps, 1), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16 storage, f32 arithmetic",
        "data": "synthetic: f16 K/V ~ N(0,1), f32 q and new rows ~ N(0,1), seeded; lengths U[512,4096] seeded",
        "config": c2_config(world, "f16"),
        "implementation": "restated reference CPU path (oracle/lt_oracle.c); the Rust reference is not buildable "
                          "here",
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=["c1", "c2", "c3", "c4-batch", "c4-head", "c5", "prefill"], default="c2",
                    help="c2: configs[1] (default, the headline); c1: configs[0]; c3: configs[2]; "
                         "c4-*: configs[3]; c5: configs[4]; prefill: chunked prefill attention")
    ap.add_argument("--sub", default="all",
                    help="c2: the other configurations to run after the headline and report under their keys "
                         "(comma-separated from %s; 'all' or 'none')" % ",".join(SUB_RUNNERS))
    ap.add_argument("--c5-rate", type=float, default=32.0, help="c5: mean arrivals per step over the whole job")
    ap.add_argument("--gather", choices=["peer", "nccl"], default="peer",
                    help="c4-head: gather the sharded heads inside the attention call over NVLink (peer) or with "
                         "a separate NCCL all-gather (nccl)")
    ap.add_argument("--emulate-ranks", type=int, default=1,
                    help="c4-*: on one GPU, run the per-rank work of an R-GPU run (sequences or KV heads / R)")
    ap.add_argument("--kv-format", choices=["f16", "q8_0"], default="f16",
                    help="c2 / c4-*: cached K/V format (f16: the reference's; q8_0: int8 + f16 scale per 32)")
    ap.add_argument("--cpu-seconds", type=float, default=15.0,
                    help="CPU-baseline sample budget in seconds (rank 0, N=1); 0 skips it")
    args = ap.parse_args()
    rank, world, local = rank_info()
    if args.impl == "reference":
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    if args.config != "c2":
        runners = {"c1": run_c1, "c3": run_c3, "prefill": run_prefill, "c5": run_c5,
                   "c4-batch": lambda a, r, w, lo: run_c4(a, r, w, lo, "batch"),
                   "c4-head": lambda a, r, w, lo: run_c4(a, r, w, lo, "head")}
        res = runners[args.config](args, rank, world, local)
        if rank == 0 and res is not None and args.config == "c1":
            res["cpu_baseline"] = None
            if world == 1 and args.cpu_seconds > 0:
                res["cpu_baseline"] = _cpu_leg("c1", res, args.cpu_seconds, os.cpu_count() or 1)
        finish_pg(world)
        if rank == 0 and res is not None:
            print(json.dumps(res), flush=True)
        return
    res = run_ours(args, rank, world, local)
    if rank == 0 and res is not None:
        if world == 1 and args.cpu_seconds > 0:
            threads = os.cpu_count() or 1
            value, steps, dt = cpu_run(workload(1234), 1234, budget_s=args.cpu_seconds, max_steps=10 ** 6,
                                       threads=threads, kv_format=args.kv_format)
            res["cpu_baseline"] = {
                "value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                "sample": f"{steps} full steps of the same workload (64 seqs, one layer, {args.kv_format} cache) "
                          f"in {dt:.1f} s on {threads} threads of {cpu_desc()}; restated reference "
                          f"(oracle/lt_oracle.c)"}
        else:
            res["cpu_baseline"] = None
    if args.sub != "none":
        subs = run_subconfigs(args, rank, world, local)
        if rank == 0 and res is not None:
            res["configs"] = subs
    finish_pg(world)
    if rank == 0 and res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
