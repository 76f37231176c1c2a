"""Benchmark of the paged-KV hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload default|decode_bf16|decode_int8|decode_fp32|longctx|migrate|
                                config1|prefill|prefill_int8|cow] [--tq T]

Default line (BASELINE config 2 as the headline): Llama-3-8B-shaped bf16 decode attention,
32 query heads over 8 KV heads, head_dim 128, block 16, 64 sequences with context lengths
U[512, 8192] per GPU, pages a random permutation of the pool.  One step = one decode
attention launch over the batch.  At N GPUs each rank decodes its own 64-sequence batch
with the same lengths and page tables as every other rank (its own q/K/V values):
sequences are independent units, no collective on the data path, weak scaling.  The same
line carries the other BASELINE configs, measured in the same run:
  config1      config 1 through the legacy synchronous symbol paged_attention_launch
  decode_int8  config 3: int8 KV with per-(page, head) scales
  longctx      config 5: KV heads sharded over the N GPUs (8/N each), strong scaling
  migrate      config 4 (N >= 2): prefill ranks [0, N/2) push KV blocks to decode ranks
               [N/2, N) over NVLink, checked bit for bit by block checksums

--workload X runs one of these alone (one JSON line), or decode_fp32, prefill /
prefill_int8 (multi-query causal attention, T query tokens per sequence over config 2's
bf16 or config 3's int8 pool), cow (prompt-cache copy-on-write block copy inside one
GPU's pool, config 4's block layout).

--impl reference times the reference's own CPU algorithm for the same workload and the
same aggregate work (N batches at N GPUs): the C restatement in oracle/ (the reference is
Java; no JDK exists here), on all host threads.
"""
from __future__ import annotations

import argparse
import copy
import json
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "paged-decode attn tokens/s + HBM GB/s vs 8 TB/s; KV migration GB/s vs NVLink"
L2_BYTES = 126 * 1024 * 1024


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="default",
                    choices=["default", "decode_bf16", "decode_int8", "decode_fp32", "longctx", "migrate",
                             "config1", "prefill", "prefill_int8", "cow"])
    ap.add_argument("--tq", type=int, default=4, help="prefill: query tokens per sequence")
    ap.add_argument("--seed", type=int, default=2024)
    ap.add_argument("--gather", action="store_true", help="longctx: all-gather head-sharded outputs")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--seqs", type=int, default=0,
                    help="with --workload: sequences per batch instead of the BASELINE config's "
                         "(a smaller case for profiling; the line's config reports it)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def traffic_per_launch(workload, algorithmic=None):
    """ncu dram bytes (read + write) per launch of the dominant kernel, from the committed
    summary: its per-launch figure, or its traffic-to-algorithmic ratio times this launch's
    algorithmic bytes (for a workload captured on a smaller case)."""
    p = os.path.join(ROOT, "profiles", f"ncu_{workload}.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        try:
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].split()[0])
            if line.startswith("traffic_ratio_to_algorithmic:") and algorithmic:
                return float(line.split(":", 1)[1].split()[0]) * float(algorithmic)
        except ValueError:
            return None
    return None


# ------------------------------------------------------------------ workloads

BATCH_OVERRIDE = {}  # workload -> sequences (--seqs: smaller cases for ncu captures)


def decode_shape(workload):
    if workload == "longctx":
        sh = dict(hq=64, hkv=8, d=128, bs=16, batch=256, lo=4096, hi=131072, dist="loguniform")
    else:
        sh = dict(hq=32, hkv=8, d=128, bs=16, batch=64, lo=512, hi=8192, dist="uniform")
    sh["batch"] = BATCH_OVERRIDE.get(workload, sh["batch"])
    return sh


def context_lengths(shape, rng):
    import numpy as np
    if shape["dist"] == "uniform":
        return rng.integers(shape["lo"], shape["hi"] + 1, shape["batch"]).astype(np.int32)
    u = rng.uniform(math.log(shape["lo"]), math.log(shape["hi"]), shape["batch"])
    return np.exp(u).astype(np.int32)


class DecodeBatch:
    """Synthetic decode batch resident in HBM: pool, tables, q, output."""

    def __init__(self, workload, seed, device, head_lo=0, head_hi=None, value_seed=None):
        """seed draws the context lengths and the page tables (the same on every rank, so
        every rank has the same work); value_seed (default: seed) draws q, K and V."""
        import numpy as np
        import torch
        sh = decode_shape(workload)
        self.workload = workload
        self.sh = sh
        rng = np.random.default_rng(seed)
        self.ctx_np = context_lengths(sh, rng)
        B, BS, D = sh["batch"], sh["bs"], sh["d"]
        hkv_all = sh["hkv"]
        head_hi = hkv_all if head_hi is None else head_hi
        self.hkv = head_hi - head_lo
        self.hq = sh["hq"] // hkv_all * self.hkv
        need = (self.ctx_np + BS - 1) // BS
        self.nb = int(need.sum())
        perm = rng.permutation(self.nb).astype(np.int32)
        self.maxb = int(need.max())
        bt = np.zeros((B, self.maxb), np.int32)
        off = 0
        for s in range(B):
            bt[s, :need[s]] = perm[off:off + need[s]]
            off += need[s]
        self.bt_np = bt
        self.device = device
        g = torch.Generator(device=device).manual_seed(seed if value_seed is None else value_seed)
        kv_dt = {"decode_fp32": torch.float32}.get(workload, torch.bfloat16)
        q_dt = torch.float32 if workload == "decode_fp32" else torch.bfloat16
        std = 1.0 if workload == "decode_fp32" else 0.5
        shape = (self.nb, self.hkv, BS, D)
        self.k = self._randn(shape, std, kv_dt, g)
        self.v = self._randn(shape, std, kv_dt, g)
        self.k_scales = self.v_scales = None
        self.scale_strides = (0, 0, 0)
        if workload == "decode_int8":
            self.k, self.k_scales = self._quant_pages(self.k)
            self.v, self.v_scales = self._quant_pages(self.v)
            self.scale_strides = (self.hkv, 1, 0)
        self.q = (torch.randn((B, self.hq, D), generator=g, device=device) * 1.0).to(q_dt)
        self.bt = torch.from_numpy(bt).to(device)
        self.ctx = torch.from_numpy(self.ctx_np).to(device)
        self.out = torch.empty_like(self.q)
        self.kv_elem = self.k.element_size()
        self.q_elem = self.q.element_size()

    @staticmethod
    def _randn(shape, std, dt, g):
        import torch
        t = torch.empty(shape, dtype=dt, device=g.device)
        flat = t.view(-1)
        step = 1 << 28
        for i in range(0, flat.numel(), step):
            n = min(step, flat.numel() - i)
            flat[i:i + n] = (torch.randn(n, generator=g, device=g.device) * std).to(dt)
        return t

    @staticmethod
    def _quant_pages(x):
        """Per-(page, kv-head) symmetric int8 of bf16 values: scale = max|x|/127."""
        import torch
        nb = x.shape[0]
        q = torch.empty(x.shape, dtype=torch.int8, device=x.device)
        sc = torch.empty(x.shape[:2], dtype=torch.float32, device=x.device)
        step = 1 << 14
        for i in range(0, nb, step):
            xs = x[i:i + step].float()
            amax = xs.abs().amax(dim=(2, 3))
            s = torch.where(amax == 0, torch.ones_like(amax), amax / 127.0)
            q[i:i + step] = torch.clamp(torch.floor(xs / s[:, :, None, None] + 0.5), -127, 127).to(torch.int8)
            sc[i:i + step] = s
        return q, sc

    def algorithmic_bytes(self):
        """Bytes one decode step must move: every context token's K and V row of each
        kv-head, the scales, q, out, the used block-table entries and the lengths."""
        return decode_alg_bytes(self.sh, self.ctx_np, self.hkv, self.kv_elem, self.q_elem,
                                self.q.numel(), self.k_scales is not None)

    def run(self, out=None, q=None, bt=None, ctx=None, stream=None, workspace=None):
        from gollek_b200 import ops
        return ops.paged_attention(q if q is not None else self.q, self.k, self.v,
                                   bt if bt is not None else self.bt,
                                   ctx if ctx is not None else self.ctx,
                                   num_kv_heads=self.hkv, block_size=self.sh["bs"],
                                   num_blocks=self.nb, k_scales=self.k_scales,
                                   v_scales=self.v_scales, scale_strides=self.scale_strides,
                                   out=out if out is not None else self.out, stream=stream,
                                   workspace=workspace)


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while the timed region runs."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown", 0x1: "gpu_idle",
               0x2: "applications_clocks_setting"}

    def __init__(self, index, period=0.002):
        self.index, self.period = index, period
        self.samples, self.reasons = [], 0
        self._stop = threading.Event()
        self.ok = False
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.ok = False

    def _loop(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    nv.nvmlDeviceGetCurrentClocksThrottleReasons
                self.reasons |= fn(self.h)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._loop, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"], "samples": 0}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples)}


# ------------------------------------------------------------------ distributed

def dist_setup(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ------------------------------------------------------------------ CPU baseline

def cpu_decode_baseline(batch, seconds, threads=None, q=None, tq=1, max_seqs=None):
    """The reference's CPU algorithm (oracle restatement of PagedAttentionVectorAPI) on
    fp32 copies of the same values, all host threads.  q/tq: a multi-query step
    ([S, tq, Hq, D] queries at each sequence's last tq positions).

    Bounded sample: the first n sequences of the batch, n doubled until one call takes
    about a third of `seconds`; only their pages are gathered to the host.  The step time
    is scaled to the whole batch by context tokens (the work is linear in them)."""
    import numpy as np
    import torch
    from oracle import oracle as O
    threads = threads or host_cores()
    qa = (batch.q if q is None else q)
    bt_all, ctx_all = batch.bt_np, batch.ctx_np
    bs = batch.sh["bs"]
    B = len(ctx_all)
    n_cap = B if max_seqs is None else max_seqs
    # host memory: at most ~3 GB of gathered fp32 K and V pages in the sample
    page_f32 = batch.hkv * bs * batch.sh["d"] * 4 * 2
    cum = np.cumsum((ctx_all + bs - 1) // bs) * page_f32
    n_cap = max(1, min(n_cap, int(np.searchsorted(cum, 3e9, side="right"))))
    scale = 1.0 / math.sqrt(batch.sh["d"])

    def sample(n):
        need = (ctx_all[:n] + bs - 1) // bs
        pages = np.concatenate([bt_all[i, :need[i]] for i in range(n)]).astype(np.int64)
        remap = np.zeros_like(bt_all[:n])
        off = 0
        for i in range(n):
            remap[i, :need[i]] = np.arange(off, off + need[i], dtype=np.int32)
            off += need[i]
        idx = torch.from_numpy(pages).to(batch.k.device)
        qs = qa[:n].float().cpu().numpy()
        if qs.ndim == 3:
            qs = qs[:, None]
        if batch.k_scales is not None:
            k = batch.k.index_select(0, idx).cpu().numpy()
            v = batch.v.index_select(0, idx).cpu().numpy()
            ks = np.repeat(batch.k_scales.index_select(0, idx).cpu().numpy()[:, :, None], bs, axis=2)
            vs = np.repeat(batch.v_scales.index_select(0, idx).cpu().numpy()[:, :, None], bs, axis=2)
            st = O.INT8
        else:
            k = batch.k.index_select(0, idx).float().cpu().numpy()
            v = batch.v.index_select(0, idx).float().cpu().numpy()
            ks = vs = None
            st = O.FP32
        return qs, k, v, remap, ctx_all[:n].copy(), ks, vs, st

    def call(smp):
        qs, k, v, bt, ctx, ks, vs, st = smp
        O.a2_compute(qs, k, v, bt, ctx, scale, storage=st, num_kv_heads=batch.hkv, block_size=bs,
                     k_scale=ks, v_scale=vs, threads=threads)

    n = 1
    while True:
        smp = sample(n)
        t0 = time.perf_counter()
        call(smp)
        dt = time.perf_counter() - t0
        if n >= n_cap or dt > seconds / 3:
            break
        n = min(n_cap, n * 2)
    reps, total, t_start = 0, 0.0, time.perf_counter()
    while time.perf_counter() - t_start < seconds and reps < 1000:
        t0 = time.perf_counter()
        call(smp)
        total += time.perf_counter() - t0
        reps += 1
    frac = float(ctx_all[:n].sum()) / float(ctx_all.sum())
    t_step = (total / reps) / frac
    return {"value": B * tq / t_step, "unit": "tokens/s" if tq == 1 else "query tokens/s",
            "cores": int(threads), "kind": "port",
            "sample": f"{n} of {B} sequences ({frac:.1%} of the batch's context tokens, "
                      f"{batch.hkv} kv heads), {reps} repetitions, {total:.1f} s; scaled to the "
                      f"full batch by context tokens; oracle/oracle.c a2 (PagedAttentionVectorAPI "
                      f"restatement), fp32 values, OpenMP over (sequence, q-head)",
            "seconds_per_step": t_step, "per_seq_s": (total / reps) / n}


# ------------------------------------------------------------------ decode bench

def host_cores() -> int:
    """Host threads this process may use (the CPU arms use all of them, whatever
    OMP_NUM_THREADS a launcher set)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def decode_config(workload, world, ctx_np, alg_bytes, hkv_per_gpu):
    """The `config` dict of a decode line -- the same for our arm and the reference arm."""
    sh = decode_shape(workload)
    tok = int(ctx_np.sum())
    shard = workload == "longctx"
    return {
        "workload": WORKLOAD_NAMES[workload],
        "batch_per_gpu": sh["batch"],
        "num_q_heads": sh["hq"], "num_kv_heads": sh["hkv"], "head_dim": sh["d"],
        "block_size": sh["bs"], "context": f"{sh['dist']}[{sh['lo']},{sh['hi']}]",
        "context_tokens_per_gpu": tok,
        "context_tokens_total": tok if shard else tok * world,
        "kv_heads_per_gpu": hkv_per_gpu,
        "parallelism": (f"kv-head shard x{world}" if shard
                        else f"independent batches x{world} (same lengths and tables on every rank)"),
        "l2": f"no flush: {alg_bytes / 1e9:.2f} GB of KV per step per GPU > 126 MB L2",
    }


def bench_decode(args, world, rank, local, workload=None, steps=None, cpu=True):
    """One decode workload; returns its JSON line (a dict) on rank 0, None elsewhere."""
    import numpy as np
    import torch
    from gollek_b200 import ops
    workload = workload or args.workload
    steps = steps or args.steps
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if workload == "longctx":
        from gollek_b200.sharding import kv_head_shard
        lo, hi = kv_head_shard(decode_shape("longctx")["hkv"], world, rank)
        batch = DecodeBatch("longctx", args.seed, dev, head_lo=lo, head_hi=hi)
    else:
        # every rank: the same lengths and page tables (equal work), its own values
        batch = DecodeBatch(workload, args.seed, dev, value_seed=args.seed + rank)
    stream = torch.cuda.current_stream(dev)
    gather_buf = None
    if workload == "longctx" and args.gather and world > 1:
        gather_buf = torch.empty((world,) + tuple(batch.out.shape), dtype=batch.out.dtype, device=dev)

    def step():
        batch.run()
        if gather_buf is not None:
            import torch.distributed as dist
            dist.all_gather_into_tensor(gather_buf, batch.out)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    t_ms = e0.elapsed_time(e1)
    t_ms_max = max_over_ranks(t_ms, world)
    B = len(batch.ctx_np)
    launches = steps * (1 + (1 if gather_buf is not None else 0))

    # ---------------- e2e: host buffers in, host result out, through the C ABI
    from gollek_b200 import _lib
    B, Hq, D = batch.q.shape
    append = workload in ("decode_bf16", "decode_fp32", "longctx")
    # The step's host inputs sit in one pinned staging block (q, tables, lengths and, with
    # the append, the new K/V rows and their positions), so a step moves them with one
    # H2D copy; the output comes back with one D2H copy.
    parts = [("q", batch.q.cpu()), ("bt", batch.bt.cpu()), ("ctx", batch.ctx.cpu())]
    if append:
        g = torch.Generator().manual_seed(args.seed + 7 + rank)
        kv_dt = batch.k.dtype
        parts += [("k_new", torch.randn((B, batch.hkv, D), generator=g).to(kv_dt)),
                  ("v_new", torch.randn((B, batch.hkv, D), generator=g).to(kv_dt)),
                  ("pos", (batch.ctx.cpu() - 1).to(torch.int32))]
    offs, total = {}, 0
    for name, t in parts:
        offs[name] = total
        total += (t.numel() * t.element_size() + 255) // 256 * 256
    h_stage = torch.empty(total, dtype=torch.uint8).pin_memory()
    d_stage = torch.empty(total, dtype=torch.uint8, device=dev)

    def view(buf, name, like):
        n = like.numel() * like.element_size()
        return buf[offs[name]:offs[name] + n].view(like.dtype).view(like.shape)

    for name, t in parts:
        view(h_stage, name, t).copy_(t)
    hout_pin = torch.empty(batch.out.shape, dtype=batch.out.dtype).pin_memory()
    ws_e2e = torch.zeros(_lib.load().gollek_paged_attention_workspace_size(B, Hq, batch.hkv, D),
                         dtype=torch.uint8, device=dev)

    # The steps run as a double-buffered pipeline, the way a serving loop overlaps its
    # transfers with compute: step k's inputs go up on a copy stream (into staging buffer
    # k % 2) while step k-1 decodes, and step k's output comes down on a second copy
    # stream while step k+1 decodes.  Every step still copies its own inputs in and its
    # own result out; the append and the decode of consecutive steps stay in order on the
    # compute stream.
    s_comp = stream
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    d_stages = [d_stage, torch.empty_like(d_stage)]
    dv = [{name: view(buf, name, t) for name, t in parts} for buf in d_stages]
    outs = [batch.out, torch.empty_like(batch.out)]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def pipe_step(k, after=None):
        b = k % 2
        dd = dv[b]
        with torch.cuda.stream(s_in):
            if after is not None:
                s_in.wait_event(after)
            if k >= 2:
                s_in.wait_event(ev_used[b])  # step k-2's decode has read this staging buffer
            d_stages[b].copy_(h_stage, non_blocking=True)
            ev_in[b].record(s_in)
        s_comp.wait_event(ev_in[b])
        if k >= 2:
            s_comp.wait_event(ev_out[b])  # step k-2's output has been copied out
        if append:
            ops.kv_append(dd["k_new"], dd["v_new"], dd["pos"], dd["bt"], batch.k, batch.v,
                          block_size=batch.sh["bs"], num_blocks=batch.nb, stream=s_comp)
        batch.run(out=outs[b], q=dd["q"], bt=dd["bt"], ctx=dd["ctx"], workspace=ws_e2e, stream=s_comp)
        ev_used[b].record(s_comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_used[b])
            hout_pin.copy_(outs[b], non_blocking=True)
            ev_out[b].record(s_out)

    graph_note = ("double-buffered pipeline on 3 streams: H2D of step k+1 and D2H of step k-1 "
                  "overlap the decode of step k")
    e2e_steps = max(1, min(steps, 100))
    for k in range(max(2, args.warmup)):
        pipe_step(k)
    torch.cuda.synchronize()
    barrier(world)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    f0.record(s_comp)
    for k in range(e2e_steps):
        pipe_step(k, after=f0 if k == 0 else None)
    s_comp.wait_event(ev_out[(e2e_steps - 1) % 2])
    f1.record(s_comp)
    torch.cuda.synchronize()
    wall = time.perf_counter() - w0
    barrier(world)
    e2e_ms = max_over_ranks(f0.elapsed_time(f1), world)
    h2d = h_stage.numel()
    d2h = hout_pin.numel() * hout_pin.element_size()

    if workload == "longctx":
        total_seqs = B  # every rank processes all sequences for its heads
    else:
        total_seqs = B * world
    value = total_seqs * steps / (t_ms_max / 1e3)
    e2e_value = total_seqs * e2e_steps / (e2e_ms / 1e3)

    # roofline of the decode kernel (this rank's launch; the slowest rank's rate)
    alg = batch.algorithmic_bytes()
    per_launch_s = (t_ms / 1e3) / steps
    achieved = alg / per_launch_s / 1e9
    achieved_min = -max_over_ranks(-achieved, world)
    alg_total = sum_over_ranks(float(alg), world)
    peak, peak_kind = peaks()
    traffic = traffic_per_launch(workload, alg)

    cpu_line = None
    if cpu and rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_line = cpu_decode_baseline(batch, args.cpu_seconds)
        cpu_line.pop("per_seq_s", None)
        cpu_line.pop("seconds_per_step", None)

    clocks = clk.summary()
    ctx_np = batch.ctx_np
    hkv = batch.hkv
    del batch, d_stages, dv, outs, ws_e2e, d_stage, gather_buf
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": args.warmup,
        "ms_per_step": t_ms_max / steps,
        "higher_is_better": True,
        "scaling": "strong" if workload == "longctx" else "weak",
        "vs_baseline": None,
        "dtype": {"decode_fp32": "f32", "decode_int8": "int8 KV, bf16 q/out, f32 accumulate"}
        .get(workload, "bf16 KV/q/out, f32 accumulate"),
        "data": "synthetic (seeded; BASELINE shapes and distributions)",
        "config": decode_config(workload, world, ctx_np, alg, hkv),
        "hbm_gbs": achieved_min,
        "hbm_gbs_aggregate": alg_total * steps / (t_ms_max / 1e3) / 1e9,
        "context_tokens_per_s": float(ctx_np.sum()) * (world if workload != "longctx" else 1)
        * steps / (t_ms_max / 1e3),
        "roofline": {"bound": "hbm", "achieved": achieved_min, "peak": peak, "unit": "GB/s",
                     "frac": achieved_min / peak, "traffic": traffic,
                     "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})",
                     "algorithmic_bytes_per_launch": alg,
                     "achieved_is": "the slowest rank's algorithmic bytes per launch / its launch time",
                     "kernel": "decode_tma_kernel"},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                "wall_s": wall,
                "path": "pinned host staging block (q, tables, lengths, new K/V rows) -> one H2D -> "
                        "gollek_kv_append -> gollek_paged_attention_v2 -> one D2H of out"
                        if append else
                        "pinned host staging block (q, tables, lengths) -> one H2D -> "
                        "gollek_paged_attention_v2 -> one D2H of out",
                "gpu_launches_per_step": 2 if append else 1,
                "execution": graph_note},
        "gpu_launches": launches,
        "clocks": clocks,
        "cpu_baseline": cpu_line,
    }
    if workload == "longctx":
        line["limiter"] = ("no exchange inside attention (KV-head shards are independent); each "
                           "GPU streams its heads' pages, so strong scaling follows per-GPU HBM "
                           "time, and the head split is exact (every head has the same tokens)")
    elif world > 1:
        line["limiter"] = ("none across GPUs: independent batches with equal work; NCCL carries "
                           "only the barrier and the timing all-reduce")
    return line


# ------------------------------------------------------------------ migration bench

def migrate_plan(seed, world):
    """Requests, their prefill (source) rank and block counts; config 4 shapes."""
    import numpy as np

    from gollek_b200.sharding import assign_requests
    rng = np.random.default_rng(seed)
    lens = np.exp(rng.uniform(math.log(2048), math.log(32768), 64)).astype(np.int64)
    nsrc = max(1, world // 2)
    src_rank = np.array(assign_requests(64, world))
    blocks = (lens + 15) // 16
    return lens, src_rank, blocks, nsrc


NVLINK_NOMINAL_GBS = 900.0   # NVLink 5, per direction per GPU (NVIDIA's B200 figure)
NVLINK_PEER_COPY_GBS = 770.0  # peer copy per direction measured on this pool of B200s


def bench_migrate(args, world, rank, local, steps=None):
    """Config 4 migration; returns its JSON line (a dict) on rank 0, None elsewhere."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from gollek_b200 import _lib, ops
    if world < 2:
        raise SystemExit("migrate needs --gpus >= 2 (prefill ranks push to decode ranks)")
    steps = steps or args.steps
    dev = torch.device("cuda", local)
    L, H, BS, D = 32, 8, 16, 128
    bpb = BS * H * D * 2  # bytes per (block, layer), bf16: 32 KiB
    blk = L * bpb         # one block, all layers: 1 MiB, per K and per V
    lens, src_rank, blocks, nsrc = migrate_plan(args.seed, world)
    from gollek_b200.sharding import migration_peer
    is_src, peer = migration_peer(world, rank)
    mine = np.where(src_rank == (rank if is_src else peer))[0]
    nblk = int(blocks[mine].sum())
    rng = np.random.default_rng(args.seed + 100 + (rank if is_src else peer))
    # prefill pool: requests' blocks at permuted positions; decode pool: random free list
    pool_blocks = nblk + 64
    src_ids = rng.permutation(pool_blocks)[:nblk].astype(np.int32)
    dst_ids = rng.permutation(pool_blocks)[:nblk].astype(np.int32)
    k = torch.empty(pool_blocks * blk, dtype=torch.uint8, device=dev)
    v = torch.empty_like(k)
    if is_src:
        g = torch.Generator(device=dev).manual_seed(args.seed + rank)
        for t in (k, v):
            fl = t.view(torch.bfloat16)
            step = 1 << 28
            for i in range(0, fl.numel(), step):
                n = min(step, fl.numel() - i)
                fl[i:i + n] = torch.randn(n, generator=g, device=dev).to(torch.bfloat16)
    else:
        k.zero_()
        v.zero_()
    # exchange the decode pools' IPC handles
    import ctypes
    lib = _lib.load()
    hk = (ctypes.c_char * 64)()
    hv = (ctypes.c_char * 64)()
    ok_, ov_ = ctypes.c_longlong(0), ctypes.c_longlong(0)
    if not is_src:
        _lib.check(lib.gollek_ipc_get_handle(ctypes.c_void_p(k.data_ptr()), hk, ctypes.byref(ok_)))
        _lib.check(lib.gollek_ipc_get_handle(ctypes.c_void_p(v.data_ptr()), hv, ctypes.byref(ov_)))
    handles = [None] * world
    dist.all_gather_object(handles, (bytes(hk), bytes(hv), ok_.value, ov_.value) if not is_src else None)
    torch.cuda.synchronize()
    dk_ptr = dv_ptr = None
    if is_src:
        hk_b, hv_b, off_k, off_v = handles[peer]
        pk, pv = ctypes.c_void_p(), ctypes.c_void_p()
        _lib.check(lib.gollek_ipc_open_handle(hk_b, ctypes.byref(pk)))
        _lib.check(lib.gollek_ipc_open_handle(hv_b, ctypes.byref(pv)))
        base_k, base_v = pk.value, pv.value
        dk_ptr, dv_ptr = base_k + off_k, base_v + off_v
    s_ids = torch.from_numpy(src_ids).to(dev)
    d_ids = torch.from_numpy(dst_ids).to(dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        if is_src:
            ops.kv_migrate(k, v, None, None, s_ids, d_ids, src_block_stride=blk, dst_block_stride=blk,
                           bytes_per_block=blk, device=local, dst_k_ptr=dk_ptr, dst_v_ptr=dv_ptr,
                           src_num_blocks=pool_blocks, dst_num_blocks=pool_blocks)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    t_ms = e0.elapsed_time(e1) if is_src else 0.0
    t_max = max_over_ranks(t_ms, world)
    # every source rank's own link rate; the slowest one bounds the step
    my_bytes = float(nblk * blk * 2) if is_src else 0.0
    link_gbs = my_bytes * steps / (t_ms / 1e3) / 1e9 if is_src and t_ms > 0 else float("inf")
    link_min = -max_over_ranks(-link_gbs, world)
    status_bits = ops.device_status(local, clear=True)
    bad = max_over_ranks(float(status_bits), world)
    # verification: per-block checksums on both sides must agree (bit-exact copy)
    ids = s_ids if is_src else d_ids
    ck = ops.block_checksums(k, ids, block_stride=blk, bytes_per_block=blk).cpu().numpy()
    cv = ops.block_checksums(v, ids, block_stride=blk, bytes_per_block=blk).cpu().numpy()
    gathered = [None] * world
    dist.all_gather_object(gathered, (ck, cv))
    ok = all(np.array_equal(gathered[r][0], gathered[r + nsrc][0]) and
             np.array_equal(gathered[r][1], gathered[r + nsrc][1]) for r in range(nsrc))
    bytes_total = int(blocks.sum()) * blk * 2
    if is_src:
        lib.gollek_ipc_close_handle(ctypes.c_void_p(base_k))
        lib.gollek_ipc_close_handle(ctypes.c_void_p(base_v))
    clocks = clk.summary()
    del k, v, s_ids, d_ids
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    barrier(world)
    if rank != 0:
        return None
    gbs = bytes_total * steps / (t_max / 1e3) / 1e9
    peak = NVLINK_NOMINAL_GBS * nsrc
    return {
        "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": t_max / steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "u8 (bf16 KV bytes)",
        "data": "synthetic (seeded; BASELINE config 4 shapes)",
        "config": {"workload": "config4_prefill_to_decode_migration", "layers": L,
                   "kv_heads": H, "head_dim": D, "block_size": BS, "requests": 64,
                   "prompt": "loguniform[2048,32768]", "blocks": int(blocks.sum()),
                   "bytes_per_step": bytes_total, "sources": nsrc, "destinations": nsrc,
                   "parallelism": f"{nsrc} prefill ranks -> {nsrc} decode ranks, NVLink P2P push "
                                  "(plain 16-byte peer stores through a CUDA-IPC mapping)",
                   "l2": f"no flush: {bytes_total / nsrc / 1e9:.1f} GB moved per source per step"},
        "bit_exact": bool(ok) and bad == 0,
        "roofline": {"bound": "nvlink", "achieved": gbs, "peak": peak, "unit": "GB/s",
                     "frac": gbs / peak, "traffic": None,
                     "peak_source": f"NVLink 5 nominal {NVLINK_NOMINAL_GBS:.0f} GB/s per direction "
                                    f"x {nsrc} source GPU(s)",
                     "frac_of_measured_peer_copy": gbs / (NVLINK_PEER_COPY_GBS * nsrc),
                     "measured_peer_copy_source": f"{NVLINK_PEER_COPY_GBS:.0f} GB/s per direction: "
                                                  "the peer copy measured on this pool of B200s",
                     "slowest_source_gbs": link_min,
                     "kernel": "kv_migrate_kernel_v16"},
        "limiter": "each source GPU's NVLink egress (one destination per source, plain peer stores)",
        "gpu_launches": steps * nsrc, "clocks": clocks,
        "cpu_baseline": None,
    }


def config1_case(seed):
    """fp32 MHA decode, 4 sequences of {37, 128, 301, 512} tokens, 8 heads,
    head_dim 64, block 16, a seeded permutation of a 256-block pool, N(0, 1) values, scale 1/8."""
    import numpy as np
    rng = np.random.default_rng(seed)
    ctx = np.array([37, 128, 301, 512], np.int32)
    perm = rng.permutation(256).astype(np.int32)
    bt = np.zeros((4, 32), np.int32)
    off = 0
    for s, c in enumerate(ctx):
        n = (int(c) + 15) // 16
        bt[s, :n] = perm[off:off + n]
        off += n
    q = rng.standard_normal((4, 8, 64)).astype(np.float32)
    k = rng.standard_normal((256, 8, 16, 64)).astype(np.float32)
    v = rng.standard_normal((256, 8, 16, 64)).astype(np.float32)
    alg = int(ctx.sum()) * 8 * 64 * 4 * 2 + q.nbytes * 2 + bt.size * 4 + ctx.nbytes
    return q, k, v, bt, ctx, 0.125, alg


def cpu_config1_baseline(seed, seconds=10.0):
    """PagedAttentionCpuFallback.execute (the reference's fp32 CPU path, single-threaded as
    in Java) restated in oracle/oracle.c, on config 1."""
    from oracle import oracle as O
    q, k, v, bt, ctx, scale, _ = config1_case(seed)
    O.a1_execute(q, k, v, bt, ctx, scale)
    reps, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        O.a1_execute(q, k, v, bt, ctx, scale)
        reps += 1
    el = time.perf_counter() - t0
    return {"value": 4 * reps / el, "unit": "tokens/s", "cores": 1, "kind": "port",
            "seconds_per_step": el / reps,
            "sample": f"the whole config 1 batch, {reps} repetitions in {el:.1f} s; oracle/oracle.c "
                      "oracle_a1_execute (PagedAttentionCpuFallback restatement), one thread"}


def bench_config1(args, world, rank, local, steps=None):
    """BASELINE config 1 through the legacy synchronous symbol paged_attention_launch (the
    reference's FFM entry point): latency-bound at 4 sequences, reported as tokens/s with
    the GB/s of its 4 MB step."""
    import torch
    from gollek_b200 import ops
    steps = steps or args.steps
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    q, k, v, bt, ctx, scale, alg = config1_case(args.seed)
    dq, dk, dv = (torch.from_numpy(x).to(dev) for x in (q, k, v))
    dbt, dctx = torch.from_numpy(bt).to(dev), torch.from_numpy(ctx).to(dev)
    out = torch.empty_like(dq)
    per_thread = torch.cuda.ExternalStream(2, device=dev)  # cudaStreamPerThread, the symbol's stream

    def step():
        ops.paged_attention_launch(out, dq, dk, dv, dbt, dctx, scale)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(per_thread)
        for _ in range(steps):
            step()
        e1.record(per_thread)
        torch.cuda.synchronize()
    t_ms = max_over_ranks(e0.elapsed_time(e1), world)
    # e2e: pinned host q, tables, lengths -> H2D -> the legacy call -> D2H of out
    hq, hbt, hctx = (torch.from_numpy(x).pin_memory() for x in (q, bt, ctx))
    hout = torch.empty_like(out, device="cpu").pin_memory()
    e2e_steps = max(1, min(steps, 200))
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(per_thread)
    for _ in range(e2e_steps):
        with torch.cuda.stream(per_thread):
            dq.copy_(hq, non_blocking=True)
            dbt.copy_(hbt, non_blocking=True)
            dctx.copy_(hctx, non_blocking=True)
        step()
        with torch.cuda.stream(per_thread):
            hout.copy_(out, non_blocking=True)
    f1.record(per_thread)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(f0.elapsed_time(f1), world)
    del dq, dk, dv, dbt, dctx, out
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    per_s = t_ms / 1e3 / steps
    gbs = alg / per_s / 1e9
    peak, peak_kind = peaks()
    cpu = None if args.no_cpu_baseline or world > 1 else cpu_config1_baseline(
        args.seed, seconds=min(10.0, args.cpu_seconds))
    if cpu:
        cpu.pop("seconds_per_step", None)
    return {
        "metric": METRIC, "value": 4 * world / per_s, "unit": "tokens/s", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": t_ms / steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; BASELINE config 1)",
        "config": {"workload": "config1_fp32_mha_decode_legacy_symbol", "batch_per_gpu": 4,
                   "num_heads": 8, "head_dim": 64, "block_size": 16, "context": "{37,128,301,512}",
                   "pool_blocks": 256, "entry_point": "paged_attention_launch (synchronous)",
                   "l2": "4 MB step: L2-resident after the first call (latency-bound size)"},
        "hbm_gbs": gbs,
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                     "traffic": None, "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})",
                     "algorithmic_bytes_per_launch": alg, "kernel": "decode_tma_kernel<float,64,1,...>",
                     "note": "latency-bound: 4 sequences, each call synchronises its stream"},
        "e2e": {"value": 4 * world * e2e_steps / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": q.nbytes + bt.nbytes + ctx.nbytes, "d2h_bytes_per_step": q.nbytes,
                "steps": e2e_steps,
                "path": "pinned host q/tables/lengths -> H2D -> paged_attention_launch -> D2H out"},
        "gpu_launches": steps, "clocks": clk.summary(), "cpu_baseline": cpu,
    }


def cpu_migrate_baseline(seed, seconds=3.0, sample_blocks=128):
    """The reference's migration loop (transferKvToDecodePartition: per (block, layer)
    copyFrom of 32 KiB slices, PD/PrefillDecodeDisaggService.java:415-429) restated in
    oracle/oracle.c, timed single-threaded on host memory over a bounded sample of config
    4's blocks (1 MiB per block for each of K and V) into a permuted destination layout."""
    import numpy as np
    from oracle import oracle as O
    L, bpb = 32, 16 * 8 * 128 * 2
    rng = np.random.default_rng(seed)
    n = sample_blocks
    src_k = np.frombuffer(rng.bytes(n * L * bpb), dtype=np.uint8).copy()
    src_v = np.frombuffer(rng.bytes(n * L * bpb), dtype=np.uint8).copy()
    dst_k, dst_v = np.zeros_like(src_k), np.zeros_like(src_v)
    src = np.arange(n, dtype=np.int32)
    dst = rng.permutation(n).astype(np.int32)
    O.migrate(src_k, src_v, dst_k, dst_v, src, dst, L, bpb)  # warm the pages
    reps, t0 = 0, time.perf_counter()
    while True:
        moved = O.migrate(src_k, src_v, dst_k, dst_v, src, dst, L, bpb)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    gbs = moved * reps / el / 1e9
    return {"value": gbs, "unit": "GB/s", "cores": 1, "kind": "port", "seconds_per_step": el / reps,
            "sample": f"{n} blocks x 32 layers x 32 KiB for K and V ({moved / 2**30:.2f} GiB), "
                      f"{reps} repetitions in {el:.1f} s, host memory to host memory; "
                      "oracle/oracle.c oracle_migrate, the reference's sequential copy loop"}


# ------------------------------------------------------------------ multi-query and CoW benches

def timed_steps(step, args, world, local, stream):
    """Warm-up, then args.steps steps between CUDA events on `stream` (barrier and
    synchronize on both sides); returns (this rank's ms, max over ranks, clock summary)."""
    import torch
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    t_ms = e0.elapsed_time(e1)
    return t_ms, max_over_ranks(t_ms, world), clk.summary()


def bench_prefill(args, world, rank, local):
    """Multi-query paged attention (gollek_paged_attention_prefill; the reference's
    PagedAttentionVectorAPI.compute with seqLenQ > 1): config 2's batch and pool with
    --tq query tokens per sequence at its last positions, causal -- speculative
    verification or a short prefill chunk.  value = query tokens/s.  The roofline
    numerator counts each context token's K/V once per step (what a kernel reading every
    page once must move); the kernel reads a sequence's pages once per query, the repeats
    of adjacent queries largely served from L2, so traffic shows how much reaches HBM."""
    import torch
    from gollek_b200 import _lib, ops
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    int8 = args.workload == "prefill_int8"
    batch = DecodeBatch("decode_int8" if int8 else "decode_bf16", args.seed, dev, value_seed=args.seed + rank)
    B, Hq, D = batch.q.shape
    Tq = args.tq
    g = torch.Generator(device=dev).manual_seed(args.seed + 11 + rank)
    q = torch.randn((B, Tq, Hq, D), generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    lib = _lib.load()
    ws = torch.zeros(lib.gollek_paged_attention_prefill_workspace_size(B, Tq, Hq, batch.hkv, D),
                     dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def run(qd, od, bt, ctx):
        ops.paged_attention_prefill(qd, batch.k, batch.v, bt, ctx, num_kv_heads=batch.hkv,
                                    k_scales=batch.k_scales, v_scales=batch.v_scales,
                                    scale_strides=batch.scale_strides,
                                    block_size=batch.sh["bs"], num_blocks=batch.nb, causal=True,
                                    out=od, workspace=ws, stream=stream)

    t_ms, t_max, clocks = timed_steps(lambda: run(q, out, batch.bt, batch.ctx), args, world, local,
                                      stream)
    # e2e: q, tables and lengths from pinned host memory, output back to pinned host memory
    hq_ = q.cpu().pin_memory()
    hbt, hctx = batch.bt.cpu().pin_memory(), batch.ctx.cpu().pin_memory()
    hout = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    dq, dbt, dctx = torch.empty_like(q), torch.empty_like(batch.bt), torch.empty_like(batch.ctx)

    def e2e_step():
        dq.copy_(hq_, non_blocking=True)
        dbt.copy_(hbt, non_blocking=True)
        dctx.copy_(hctx, non_blocking=True)
        run(dq, out, dbt, dctx)
        hout.copy_(out, non_blocking=True)

    class _E2E:
        steps, warmup = max(1, min(args.steps, 100)), args.warmup
    e_ms, e_max, _ = timed_steps(e2e_step, _E2E, world, local, stream)
    h2d = sum(t.numel() * t.element_size() for t in (hq_, hbt, hctx))
    d2h = hout.numel() * hout.element_size()

    # queries sharing one pass over the pages (the library's rule for causal calls with
    # head_dim 128 and no window: F * G <= 16 rows for bf16 KV, or 32 / 64 with bf16 q
    # on the tensor-memory kernel (GOLLEK_PREFILL_TC=0: not), <= 8 for int8 KV;
    # GOLLEK_PREFILL_FOLD=0 turns folding off)
    G = Hq // batch.hkv
    fold = 1
    tc_rows = not int8 and os.environ.get("GOLLEK_PREFILL_TC", "1") != "0"
    if os.environ.get("GOLLEK_PREFILL_FOLD", "1") != "0":
        f = 64
        while f > 1:
            if Tq % f == 0 and (f * G <= (8 if int8 else 16) or (tc_rows and f * G in (32, 64))):
                fold = f
                break
            f >>= 1
    halves = os.environ.get("GOLLEK_PREFILL_TC_HALVES", "1") != "0"
    kernel = (f"prefill_tc_kernel (tcgen05; the folded rows are the MMA rows; {2 if halves else 1} "
              "warp(s) per 32 rows)" if fold * G in (32, 64)
              else "decode_tma_kernel (queries folded into the MMA rows)" if fold > 1
              else "decode_tma_kernel (per-query decode sequences)")
    kv_once = batch.algorithmic_bytes() - 2 * batch.q.numel() * batch.q_elem
    alg = kv_once + 2 * q.numel() * q.element_size()
    achieved = alg / ((t_ms / 1e3) / args.steps) / 1e9
    achieved_min = -max_over_ranks(-achieved, world)
    peak, peak_kind = peaks()
    value = B * Tq * world * args.steps / (t_max / 1e3)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_decode_baseline(batch, args.cpu_seconds, q=q, tq=Tq)
        cpu.pop("per_seq_s", None)
        cpu.pop("seconds_per_step", None)
    if rank != 0:
        return None
    sh = batch.sh
    return {
        "metric": METRIC, "value": value, "unit": "query tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_max / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 KV, bf16 q/out, f32 accumulate" if int8 else "bf16 KV/q/out, f32 accumulate",
        "data": "synthetic (seeded; config 3 shapes)" if int8 else "synthetic (seeded; config 2 shapes)",
        "config": {"workload": f"multi_query_causal_tq{Tq}_{'config3' if int8 else 'config2'}_pool",
                   "batch_per_gpu": B,
                   "queries_per_seq": Tq, "queries_per_page_pass": fold, "num_q_heads": sh["hq"], "num_kv_heads": sh["hkv"],
                   "head_dim": sh["d"], "block_size": sh["bs"],
                   "context": f"{sh['dist']}[{sh['lo']},{sh['hi']}]",
                   "parallelism": f"independent batches x{world}",
                   "l2": f"no flush: {kv_once / 1e9:.2f} GB of KV per step per GPU > 126 MB L2"},
        "roofline": {"bound": "hbm", "achieved": achieved_min, "peak": peak, "unit": "GB/s",
                     "frac": achieved_min / peak,
                     "traffic": traffic_per_launch(f"prefill{'_int8' if int8 else ''}_tq{Tq}"),
                     "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})",
                     "algorithmic_bytes_per_launch": alg,
                     "note": "numerator counts each page once per step (page-once ideal); "
                             f"the kernel reads a page once per {fold} queries",
                     "kernel": kernel},
        "e2e": {"value": B * Tq * world * _E2E.steps / (e_max / 1e3), "unit": "query tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": _E2E.steps,
                "path": "pinned q, tables, lengths -> H2D -> gollek_paged_attention_prefill "
                        "-> D2H of out, serialised on one stream"},
        "gpu_launches": 2 * args.steps, "clocks": clocks, "cpu_baseline": cpu,
    }


def bench_cow(args, world, rank, local):
    """Prompt-cache copy-on-write block copy (the per-(block, layer) copy of
    optimization/gollek-plugin-prompt-cache PagedKVCacheManagerExtension.java:170-180):
    gollek_kv_migrate with source and destination in one GPU's pool.  Config 4's block
    layout (32 layers x 32 KiB per block, 1 MiB per block for each of K and V); each step
    copies the blocks of a quarter of config 4's requests to a permuted set of free
    blocks of the same pool.  value = GB/s copied; the HBM roofline counts the bytes read
    plus the bytes written, like the measured copy peak."""
    import numpy as np
    import torch
    from gollek_b200 import ops
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    L, H, BS, D = 32, 8, 16, 128
    blk = L * BS * H * D * 2
    lens, src_rank, blocks, _ = migrate_plan(args.seed, 8)
    nblk = int(blocks[src_rank == 0].sum())
    rng = np.random.default_rng(args.seed + 300 + rank)
    pool_blocks = 2 * nblk + 64
    perm = rng.permutation(pool_blocks).astype(np.int32)
    src_ids, dst_ids = perm[:nblk], perm[nblk:2 * nblk]
    k = torch.empty(pool_blocks * blk, dtype=torch.uint8, device=dev)
    v = torch.empty_like(k)
    gen = torch.Generator(device=dev).manual_seed(args.seed + rank)
    for t in (k, v):
        fl = t.view(torch.bfloat16)
        step_n = 1 << 28
        for i in range(0, fl.numel(), step_n):
            n = min(step_n, fl.numel() - i)
            fl[i:i + n] = torch.randn(n, generator=gen, device=dev).to(torch.bfloat16)
    s_ids, d_ids = torch.from_numpy(src_ids).to(dev), torch.from_numpy(dst_ids).to(dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        ops.kv_migrate(k, v, k, v, s_ids, d_ids, src_block_stride=blk, dst_block_stride=blk,
                       bytes_per_block=blk, device=local)

    t_ms, t_max, clocks = timed_steps(step, args, world, local, stream)
    same = all(torch.equal(ops.block_checksums(p, s_ids, block_stride=blk, bytes_per_block=blk),
                           ops.block_checksums(p, d_ids, block_stride=blk, bytes_per_block=blk))
               for p in (k, v))
    ok = -max_over_ranks(-float(same), world) > 0.5
    copied = nblk * blk * 2
    gbs = copied / ((t_ms / 1e3) / args.steps) / 1e9
    gbs_min = -max_over_ranks(-gbs, world)
    peak, peak_kind = peaks()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_migrate_baseline(args.seed)
        cpu.pop("seconds_per_step")
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": copied * world * args.steps / (t_max / 1e3) / 1e9,
            "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": t_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u8 (bf16 KV bytes)",
            "data": "synthetic (seeded; config 4 block layout)",
            "config": {"workload": "prompt_cache_cow_block_copy_config4_layout", "layers": L,
                       "kv_heads": H, "head_dim": D, "block_size": BS, "blocks_per_step": nblk,
                       "bytes_copied_per_step": copied,
                       "parallelism": f"independent pools x{world}",
                       "l2": f"no flush: {copied / 1e9:.1f} GB copied per step > 126 MB L2"},
            "bit_exact": bool(ok),
            "roofline": {"bound": "hbm", "achieved": 2 * gbs_min, "peak": peak, "unit": "GB/s",
                         "frac": 2 * gbs_min / peak, "traffic": None,
                         "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind}); achieved "
                                        "counts read + write bytes",
                         "kernel": "kv_migrate_kernel_v16"},
            "gpu_launches": args.steps, "clocks": clocks, "cpu_baseline": cpu,
        }), flush=True)


# ------------------------------------------------------------------ reference arm

def bench_reference(args):
    """The reference's CPU decode algorithm on the host cores (rank 0 only)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np
    from oracle import oracle as O
    if args.workload == "config1":
        r = cpu_config1_baseline(args.seed, seconds=max(1.0, min(20.0, 0.5 * args.steps)))
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": r["value"], "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["seconds_per_step"] * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 (reference CPU path)", "data": "synthetic (seeded; BASELINE config 1)",
            "config": {"workload": "config1_fp32_mha_decode_legacy_symbol", "batch_per_gpu": 4,
                       "num_heads": 8, "head_dim": 64, "block_size": 16, "context": "{37,128,301,512}"},
            "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": r["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
              flush=True)
        return
    if args.workload == "migrate":
        r = cpu_migrate_baseline(args.seed, seconds=max(1.0, min(20.0, 2.0 * args.steps)))
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": r["value"], "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["seconds_per_step"] * 1e3,
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "u8 (bf16 KV bytes)",
            "data": "synthetic (seeded; BASELINE config 4 shapes)",
            "config": {"workload": "config4_prefill_to_decode_migration", "layers": 32, "kv_heads": 8,
                       "head_dim": 128, "block_size": 16},
            "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": r["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
              flush=True)
        return

    class HostBatch:
        pass

    import torch
    threads = host_cores()
    torch.set_num_threads(threads)
    workload = "decode_bf16" if args.workload == "default" else args.workload
    sh = decode_shape(workload)
    # the GPU arm's lengths and page tables (the same seed), values drawn on the host
    rng = np.random.default_rng(args.seed)
    ctx = context_lengths(sh, rng)
    B, BS, D = sh["batch"], sh["bs"], sh["d"]
    need = (ctx + BS - 1) // BS
    nb = int(need.sum())
    perm = rng.permutation(nb).astype(np.int32)
    bt = np.zeros((B, int(need.max())), np.int32)
    off = 0
    for s_ in range(B):
        bt[s_, :need[s_]] = perm[off:off + need[s_]]
        off += need[s_]
    hkv = sh["hkv"]
    if workload == "longctx":
        hkv = max(1, hkv // max(world, 1))
    hq = sh["hq"] // sh["hkv"] * hkv
    g = torch.Generator().manual_seed(args.seed)
    std = 1.0 if workload == "decode_fp32" else 0.5
    to = torch.float32 if workload == "decode_fp32" else torch.bfloat16
    elem = 4 if to == torch.float32 else 2
    # The sample is drawn from the first sequences, so the host pool holds only their
    # pages (at most ~1.5 GB of K and V: config 5's whole pool would not fit in reason).
    page_bytes = hkv * BS * D * elem * 2
    cum = np.cumsum(need) * page_bytes
    max_seqs = max(1, int(np.searchsorted(cum, 1.5e9, side="right")))
    max_seqs = min(B, max_seqs)
    nb_host = int(need[:max_seqs].sum())
    perm_h = rng.permutation(nb_host).astype(np.int32)
    bt = np.zeros_like(bt)
    off = 0
    for s_ in range(max_seqs):
        bt[s_, :need[s_]] = perm_h[off:off + need[s_]]
        off += need[s_]
    hb = HostBatch()
    hb.sh, hb.hkv, hb.ctx_np, hb.bt_np = sh, hkv, ctx, bt
    # values rounded to bf16 as on the GPU arm (fp32 stays fp32)
    hb.q = torch.randn((B, hq, D), generator=g).to(to)
    hb.k = (torch.randn((nb_host, hkv, BS, D), generator=g) * std).to(to)
    hb.v = (torch.randn((nb_host, hkv, BS, D), generator=g) * std).to(to)
    hb.k_scales = hb.v_scales = None
    if workload == "decode_int8":
        hb.k, hb.k_scales = DecodeBatch._quant_pages(hb.k)
        hb.v, hb.v_scales = DecodeBatch._quant_pages(hb.v)
    kv_elem = hb.k.element_size()
    alg = decode_alg_bytes(sh, ctx, hkv, kv_elem, hb.q.element_size(), hb.q.numel(),
                           hb.k_scales is not None)
    per_step_budget = max(1.0, args.cpu_seconds / max(1, args.steps + args.warmup))
    r = cpu_decode_baseline(hb, per_step_budget * (args.steps + args.warmup), threads=threads,
                            max_seqs=max_seqs)
    # The GPU arm decodes one batch per GPU per step (KV-head shards of one batch for
    # config 5).  The reference arm does the same aggregate work on the host: N batches
    # of the same lengths (so N times one batch's time), or config 5's whole batch.
    n_batches = 1 if workload == "longctx" else world
    t_step = r["seconds_per_step"] * n_batches
    if workload == "longctx":
        t_step = r["seconds_per_step"] * (sh["hkv"] // hkv)  # every head shard, one after another
    value = B * n_batches / t_step
    sample = (r["sample"] + f"; one step = {n_batches} batch(es) of these lengths"
              if workload != "longctx" else r["sample"] + "; one step = all kv-head shards")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t_step * 1e3, "higher_is_better": True,
        "scaling": "strong" if workload == "longctx" else "weak", "vs_baseline": None,
        "dtype": "f32 (reference CPU path)", "data": "synthetic (seeded; same shapes as ours)",
        "config": decode_config(workload, world, ctx, alg, hkv),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": r["cores"],
                         "kind": r["kind"], "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def decode_alg_bytes(sh, ctx_np, hkv, kv_elem, q_elem, q_numel, scales):
    """Bytes one decode step must move (see DecodeBatch.algorithmic_bytes)."""
    tok = int(ctx_np.sum())
    kv = tok * hkv * sh["d"] * kv_elem * 2
    pages = int(((ctx_np + sh["bs"] - 1) // sh["bs"]).sum())
    sc = pages * hkv * 4 * 2 if scales else 0
    return kv + sc + 2 * q_numel * q_elem + pages * 4 + len(ctx_np) * 4


WORKLOAD_NAMES = {"decode_bf16": "config2_llama3_8b_bf16_gqa_decode",
                  "decode_int8": "config3_int8_kv_decode",
                  "decode_fp32": "fp32_gqa_decode",
                  "longctx": "config5_llama3_70b_longctx_kvhead_sharded"}


SUB_DROP = ("metric", "n_gpus", "higher_is_better", "vs_baseline", "data")


def bench_default(args, world, rank, local):
    """The default line: BASELINE config 2 as the headline, with the other BASELINE configs
    measured in the same run as sub-objects -- config 1 through the legacy symbol, config 3
    (int8 KV), config 5 (KV heads sharded over the N GPUs, strong scaling), multi-query
    attention with 16 queries per sequence on config 2's pool and, at N >= 2, config 4
    (prefill ranks push KV blocks to decode ranks over NVLink)."""
    head = bench_decode(args, world, rank, local, "decode_bf16")
    subs = {"config1": bench_config1(args, world, rank, local),
            "decode_int8": bench_decode(args, world, rank, local, "decode_int8"),
            "longctx": bench_decode(args, world, rank, local, "longctx")}
    # multi-query attention (16 causal queries per sequence on config 2's pool): one pass
    # over the pages on the tcgen05 kernel (64 folded rows per kv head)
    pa = copy.copy(args)
    pa.workload, pa.tq, pa.no_cpu_baseline = "prefill", 16, True
    subs["prefill_tq16"] = bench_prefill(pa, world, rank, local)
    if world >= 2 and world % 2 == 0:
        subs["migrate"] = bench_migrate(args, world, rank, local, steps=min(args.steps, 20))
    else:
        subs["migrate"] = {"skipped": "config 4 needs an even number of GPUs >= 2 "
                                      "(prefill ranks push to decode ranks)"}
    if rank != 0:
        return None
    for name, sub in subs.items():
        head[name] = {k: v for k, v in sub.items() if k not in SUB_DROP}
    return head


def main():
    args = parse()
    if args.impl == "reference":
        bench_reference(args)
        return
    if args.seqs > 0 and args.workload != "default":
        BATCH_OVERRIDE[args.workload] = args.seqs
    world, rank, local = dist_setup(args)
    try:
        if args.workload == "default":
            line = bench_default(args, world, rank, local)
        elif args.workload == "migrate":
            line = bench_migrate(args, world, rank, local)
        elif args.workload == "config1":
            line = bench_config1(args, world, rank, local)
        elif args.workload in ("prefill", "prefill_int8"):
            line = bench_prefill(args, world, rank, local)
        elif args.workload == "cow":
            line = bench_cow(args, world, rank, local)
        else:
            line = bench_decode(args, world, rank, local)
        if rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
