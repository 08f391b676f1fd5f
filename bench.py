"""Paged decode benchmark: KV append + paged GQA decode over every layer of one
decode step, on 1..N B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 70b|7b|prefill|churn]
                    [--impl ours|reference] [--kv fp16|fp8] [--gather p2p|p2p-wait|nccl]
                    [--no-e2e] [--no-cpu-baseline]

Workloads (synthetic, seeded; fp16 K/V/Q drawn from N(0, 0.5^2)):
  70b  Llama-2-70B-shaped GQA decode: 64 query heads, 8 KV heads, head dim 128,
       80 layers, batch 64, context lengths lognormal (median 2048, sigma 0.6)
       clipped to [256, 8192], 16-token pages in a random block table.  At N
       GPUs each rank holds 8/N KV heads (and their 64/N query heads) of every
       sequence; each layer's output is all-gathered inside the decode kernel
       itself (peer stores into every rank's receive buffer over NVLink, one
       flag per rank and layer; --gather nccl uses an NCCL all-gather on a side
       stream instead).
  7b   Llama-2-7B decode: 32/32 heads, head dim 128, 32 layers, batch 32,
       contexts uniform in [128, 4096], pool 1.2x the tokens; sequences are
       sharded across ranks (no collective).
  prefill, churn: chunked prefill and long-context paged churn (one GPU).

One step = for every layer one planned-decode launch (vk_decode_run): the new
token's K/V appended into its page, paged attention over the whole context with
the split units merged in the same launch, and the gather when sharded; the
host plan is built and uploaded once per step, and the layers run as one CUDA
graph with programmatic dependent launch between them.  Timed with CUDA events
between barriers, max over ranks.  Rank 0 prints one JSON line.  --impl
reference times the reference's CPU attention (oracle port) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np
from typing import List

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "paged decode-attn tokens/s & HBM GB/s (% of B200 peak) at 1/2/4/8 B200"
PAGE = 16


# ----------------------------------------------------------------------------- workload

def workload(name: str):
    if name == "70b":
        rng = np.random.Generator(np.random.PCG64(2048))
        B, sigma = 64, 0.6
        ctx = np.clip(np.round(np.exp(rng.normal(math.log(2048), sigma, B))), 256, 8192).astype(np.int64)
        return dict(name="llama2-70b-gqa-decode", B=B, Hq=64, Hkv=8, D=128, L=80, ctx=ctx, shard="head",
                    desc="Llama-2-70B GQA decode: B=64, Hq=64, Hkv=8, D=128, L=80, 16-token pages, "
                         "ctx lognormal(median 2048, sigma 0.6) clipped [256, 8192], random block table",
                    sigma=sigma, seed=2048)
    if name == "prefill":
        rng = np.random.Generator(np.random.PCG64(8192))
        B = 8
        ctx = rng.integers(0, 4097, B).astype(np.int64)  # cached prefix before the chunk
        return dict(name="llama2-7b-chunked-prefill", B=B, Hq=32, Hkv=32, D=128, L=32, T=2048, ctx=ctx,
                    shard="seq",
                    desc="Llama-2-7B chunked prefill: 8 sequences x 2048-token chunk appended into 16-token "
                         "pages over cached prefixes U[0, 4096], Hq=Hkv=32, D=128, L=32, random block table",
                    seed=8192)
    if name == "churn":
        rng = np.random.Generator(np.random.PCG64(32768))
        B = 256
        ctx = rng.integers(1024, 32769, B).astype(np.int64)
        return dict(name="long-context-churn", B=B, Hq=32, Hkv=32, D=128, L=1, ctx=ctx, shard="seq",
                    rate=16, steps=200, capacity=0.7, seed=32768,
                    desc="Long-context paged churn, Llama-2-7B head shapes (32/32, D=128), 1 layer: 256 "
                         "sequences arriving Poisson(16)/step, contexts U[1k, 32k], pool 70% of demand, "
                         "LRU swap to pinned host and back, compaction by page copy every 25 steps, 200 decode steps")
    if name == "70b-wo":
        wl = workload("70b")
        wl["desc"] = wl["desc"] + "; then wo (8192 x 8192 fp16 per layer) fused with its reduce-scatter"
        wl["name"] = "llama2-70b-gqa-decode-wo"
        return wl
    if name == "7b":
        rng = np.random.Generator(np.random.PCG64(4096))
        B = 32
        ctx = rng.integers(128, 4097, B).astype(np.int64)
        return dict(name="llama2-7b-decode", B=B, Hq=32, Hkv=32, D=128, L=32, ctx=ctx, shard="seq",
                    desc="Llama-2-7B decode: B=32, Hq=Hkv=32, D=128, L=32, 16-token pages, "
                         "ctx uniform [128, 4096], pool 1.2x tokens, random block table",
                    seed=4096)
    raise SystemExit("unknown config " + name)


def layout(ctx, seed, slack=1.2):
    """Random physical pages for contexts ctx (+1 appended token each)."""
    rng = np.random.Generator(np.random.PCG64(seed + 1))
    lens = ctx + 1
    need = (lens + PAGE - 1) // PAGE
    num_pages = int(math.ceil(slack * need.sum()))
    perm = rng.permutation(num_pages).astype(np.int32)
    width = int(need.max())
    bt = np.full((len(ctx), width), -1, np.int32)
    off = 0
    for b, k in enumerate(need):
        bt[b, :k] = perm[off:off + k]
        off += k
    return bt, num_pages


def algorithmic_bytes(ctx, Hq, Hkv, D, kv_format="fp16"):
    """Bytes one layer of one step must move (counted once): K/V read, new K/V
    read (fp16) + write (page format), Q read + O write, block-table reads.
    FP8 pages hold 2*D code bytes + 8 scale bytes per (token, head)."""
    lens = ctx + 1
    row = 2 * D * 2 if kv_format == "fp16" else 2 * D + 8
    kv = int((lens * Hkv * row).sum())
    new = len(ctx) * Hkv * (2 * D * 2 + row)
    qo = len(ctx) * 2 * Hq * D * 2
    table = int((4 * ((lens + PAGE - 1) // PAGE)).sum())
    return dict(decode=kv + qo + table, append=new, total=kv + new + qo + table)


def workload_config(wl, kv_format, world):
    """The `config` object of both arms' JSON lines: what the workload is, not
    how an arm runs it (that goes under `run`), so the two arms' lines carry
    the same config at every N."""
    ab = algorithmic_bytes(wl["ctx"], wl["Hq"], wl["Hkv"], wl["D"], kv_format)
    return {"workload": wl["desc"], "kv_format": kv_format,
            "shard": wl["shard"] if world > 1 else "none",
            "l2": "inputs larger than L2: %.1f GB of K/V read per step" % (ab["decode"] * wl["L"] / 1e9),
            "context_tokens": int((wl["ctx"] + 1).sum())}


def fill_fp8(pool, D, dev, gen):
    """Fills an FP8 pool with e4m3 codes of N(0, 0.5^2) rows at the scale of
    their quantisation (max|x| ~ 1.4 over 128 values), every code finite."""
    import torch
    blocks = pool.block_view().view(-1, pool.block_bytes)
    codes_b = 2 * PAGE * D
    for s in range(0, blocks.shape[0], 1 << 16):
        part = blocks[s:s + (1 << 16)]
        x = torch.randn(part.shape[0], codes_b, device=dev, generator=gen) * (0.5 * 448.0 / 1.4)
        part[:, :codes_b].copy_(x.clamp_(-448.0, 448.0).to(torch.float8_e4m3fn).view(torch.uint8))
        sc = torch.full((part.shape[0], 2 * PAGE), 1.4 / 448.0, device=dev, dtype=torch.float32)
        part[:, codes_b:].copy_(sc.view(torch.uint8))


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# DRAM traffic per launch (dram__bytes_read.sum + dram__bytes_write.sum) from
# the committed ncu captures, for the workloads they were taken on.
NCU_DECODE_70B_BYTES = 591.055360e6 + 4.537344e6   # profiles/planned_decode_kernel_70b-one-layer_full.md
NCU_PREFILL_2SEQ_BYTES = 189.434624e6 + 8.898816e6  # profiles/prefill_tc_kernel_small-case_full.md


def prefill_tile_reads(ctx, T, rows=256, keys=128):
    """K/V tiles the tcgen05 prefill reads per head: one pass over the keys of
    each 256-row CTA (keys up to the CTA's last row)."""
    n = 0
    for p in np.asarray(ctx).tolist():
        for q0 in range(0, T, rows):
            n += (p + min(T, q0 + rows) + keys - 1) // keys
    return n


# ----------------------------------------------------------------------------- clocks

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            self.path = "/tmp/vk_clocks_%d_%d.csv" % (os.getpid(), self.device)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), "--query-gpu=" + self.FIELDS,
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- cpu baseline

def cpu_decode_sample(wl, bt, ctx, Hkv, Hq, seqs, nthreads, host_pages=None):
    """Times the oracle port of the reference's golden attention (decode row,
    block-table gather) on one layer of the given sequences.  Returns seconds."""
    import oracle
    D = wl["D"]
    lens = (ctx + 1).astype(np.int32)
    sub_bt = bt[seqs]
    need = (lens[seqs] + PAGE - 1) // PAGE
    # compact host pool holding only the sampled sequences' pages of one layer
    n_pages = int(need.sum())
    g = oracle.Geom(1, Hkv, D, PAGE, n_pages)
    rng = np.random.Generator(np.random.PCG64(99))
    if host_pages is None:
        pool = (rng.standard_normal(g.pool_shape(), dtype=np.float32) * 0.5).astype(np.float16)
    else:
        pool = host_pages
    cbt = np.full((len(seqs), sub_bt.shape[1]), -1, np.int32)
    off = 0
    for i, k in enumerate(need):
        cbt[i, :k] = np.arange(off, off + k, dtype=np.int32)
        off += k
    q = (rng.standard_normal((len(seqs), Hq, D), dtype=np.float32) * 0.5).astype(np.float16)
    t0 = time.perf_counter()
    oracle.decode_paged(pool.view(np.uint16), g, 0, q.view(np.uint16), cbt, lens[seqs], nthreads=nthreads)
    return time.perf_counter() - t0


def run_reference_arm(args, wl):
    """The reference's CPU implementation of the path (oracle port of its golden
    cpu_attention, decode row over the paged gather) on all host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    ctx = wl["ctx"]
    bt, _ = layout(ctx, wl["seed"])
    threads = os.cpu_count() or 1
    # bounded sample per step: one layer of a quarter of the sequences (all heads)
    rng = np.random.Generator(np.random.PCG64(7))
    seqs = np.sort(rng.choice(wl["B"], max(1, wl["B"] // 4), replace=False))
    frac = float((ctx[seqs] + 1).sum()) / float((ctx + 1).sum())
    times = []
    for i in range(args.warmup + args.steps):
        t = cpu_decode_sample(wl, bt, ctx, wl["Hkv"], wl["Hq"], seqs, threads)
        if i >= args.warmup:
            times.append(t)
    sample_s = statistics.median(times)
    step_s = sample_s / frac * wl["L"]  # the whole step, extrapolated from the sample
    value = wl["B"] / step_s
    sample = ("1 of %d layers, %d of %d sequences (all %d heads) per step, %.2f s measured per sample; "
              "tokens/s extrapolated x%d layers / %.3f of the tokens"
              % (wl["L"], len(seqs), wl["B"], wl["Hq"], sample_s, wl["L"], frac))
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup,
            # what was timed: one bounded sample per step (the full step would
            # take ms_per_step_extrapolated)
            "ms_per_step": sample_s * 1e3, "ms_per_step_kind": "measured sample (see extrapolated)",
            "extrapolated": {"layers": wl["L"], "token_frac": frac, "sample_ms": sample_s * 1e3,
                             "ms_per_step_extrapolated": step_s * 1e3,
                             "value_is": "B / ms_per_step_extrapolated"},
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,0.5^2) fp16 K/V/Q, random block tables)",
            "config": workload_config(wl, args.kv, args.gpus),
            "run": {"threads": threads, "code": "oracle port of the reference's golden cpu_attention "
                                                 "(decode row over the paged gather)"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU arm

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="70b", choices=["70b", "7b", "prefill", "churn", "70b-wo"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--path", default="planned", choices=["planned", "split"],
                    help="planned: one persistent launch per layer (append+decode+merge fused); "
                         "split: vk_append + vk_decode (split grid + merge kernel)")
    ap.add_argument("--pps", type=int, default=0, help="override decode pages per split (0 = auto)")
    ap.add_argument("--eager", action="store_true", help="launch every layer from Python instead of a CUDA graph")
    ap.add_argument("--no-early-start", action="store_true",
                    help="launch each layer's decode only after the previous one completes")
    ap.add_argument("--gather", default="p2p", choices=["p2p", "p2p-wait", "nccl"],
                    help="head-sharded output allgather: peer stores fused into the decode, overlapping the "
                         "next layer (p2p) or waited for before the next layer reads its inputs (p2p-wait); "
                         "or NCCL on a side stream")
    ap.add_argument("--kv", default="fp16", choices=["fp16", "fp8"],
                    help="page format of the decode configs: fp16, or e4m3 codes with an fp32 scale per row")
    ap.add_argument("--layers", type=int, default=0, help="profiling aid: use only this many layers")
    ap.add_argument("--batch", type=int, default=0, help="profiling aid: use only the first B sequences")
    ap.add_argument("--share-of", type=int, default=0,
                    help="profiling aid: run rank 0's KV-head share of an N-GPU run alone on one GPU")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    wl = workload(args.config)
    if args.layers:
        wl["L"] = args.layers
        wl["desc"] += " [profiling case: %d layers]" % args.layers
    if args.share_of > 1:
        wl["desc"] += " [profiling case: rank 0's KV-head share of %d GPUs, alone on one GPU]" % args.share_of
    if args.batch:
        wl["B"] = args.batch
        wl["ctx"] = wl["ctx"][:args.batch]
        wl["desc"] += " [profiling case: first %d sequences]" % args.batch
    if args.impl == "reference":
        return run_reference_arm(args, wl)
    if args.config == "prefill":
        return run_prefill(args, wl)
    if args.config == "70b-wo":
        return run_attn_wo(args, wl)
    if args.config == "churn":
        if args.kv != "fp16":
            raise SystemExit("--kv fp8 applies to the decode configs (70b, 7b) and prefill, not churn")
        return run_churn(args, wl)

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit("WORLD_SIZE %d != --gpus %d" % (world, args.gpus))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))

    import vulcan_b200 as vk

    B, Hq, Hkv, D, L = wl["B"], wl["Hq"], wl["Hkv"], wl["D"], wl["L"]
    ctx_all = wl["ctx"]
    bt_all, num_pages_all = layout(ctx_all, wl["seed"])
    from vulcan_b200.shard import head_shard, seq_shard
    if wl["shard"] == "head":
        sh = head_shard(Hkv, Hq, args.share_of if (args.share_of > 1 and world == 1) else world, rank)
        hkv_l, hq_l = sh.num_kv_heads, sh.num_q_heads
        seqs = np.arange(B)
        ctx, bt, num_pages = ctx_all, bt_all, num_pages_all
    else:
        seqs = seq_shard(ctx_all + 1, world)[rank]
        hkv_l, hq_l = Hkv, Hq
        ctx = ctx_all[seqs]
        bt, num_pages = layout(ctx, wl["seed"] + 17 * rank)
    Bl = len(seqs)
    lens = (ctx + 1).astype(np.int32)
    max_len = int(lens.max())

    # --- pool and inputs on the device
    pool = vk.PagedKVPool(L, hkv_l, D, num_pages, own_memory=False, zero=False, kv_format=args.kv)
    if args.pps:
        pool.set_split(args.pps)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1000 + rank)
    if args.kv == "fp16":
        flat = pool.storage.view(torch.float16)
        chunk = 1 << 28
        for s in range(0, flat.numel(), chunk):
            part = flat[s:s + chunk]
            part.copy_(torch.randn(part.shape, device=dev, generator=gen) * 0.5)
    else:
        fill_fp8(pool, D, dev, gen)
    bt_d = torch.from_numpy(bt).to(dev)
    pos_d = torch.from_numpy(ctx.astype(np.int32)).to(dev)
    lens_d = torch.from_numpy(lens).to(dev)
    q = (torch.randn(L, Bl, hq_l, D, device=dev, generator=gen) * 0.5).half()
    kn = (torch.randn(L, Bl, 1, hkv_l, D, device=dev, generator=gen) * 0.5).half()
    vn = (torch.randn(L, Bl, 1, hkv_l, D, device=dev, generator=gen) * 0.5).half()
    out = torch.empty(L, Bl, hq_l, D, device=dev, dtype=torch.float16)
    ws = pool.workspace(Bl, hq_l, max_len)
    lens_host = lens.tolist()
    kn3 = kn.view(L, Bl, hkv_l, D)
    vn3 = vn.view(L, Bl, hkv_l, D)
    plan_ws = torch.empty(pool.plan(lens_host, hq_l).workspace.numel() + 4096, dtype=torch.uint8, device=dev)
    gathered = None
    comm = None
    gat = None
    if world > 1 and wl["shard"] == "head":
        if args.gather.startswith("p2p") and args.path == "planned":
            # receive buffers of every layer on every rank, written by the decode;
            # 2L slots so that alternate steps of the e2e run use alternate halves
            gat = vk.Gather(rank, world, Bl * hq_l * D * 2, slots=2 * L, device=dev)
            gat.exchange()
        else:
            gathered = torch.empty(L, world, Bl, hq_l, D, device=dev, dtype=torch.float16)
            comm = torch.cuda.Stream(device=dev)
    compute = torch.cuda.current_stream(dev)
    merge_launched = 1 if pool.workspace_size(Bl, hq_l, max_len) > 0 else 0
    launches_per_step = (L * (2 + merge_launched) if args.path == "split" else L) + (1 if gat is not None else 0)

    use_graph = not args.eager
    plan_keep = {}

    def new_plan():
        """Host plan for this step (every layer shares the lengths), uploaded in stream order."""
        if args.path == "planned":
            p_ = pool.plan(lens_host, hq_l, workspace=plan_ws)
            if not args.no_early_start:
                p_.set_early_start(True)  # layers are back to back: overlap each launch's start
            if gat is not None:
                p_.set_gather(gat, slot_base=0, wait_prev=args.gather == "p2p-wait")
            p_.upload()
            plan_keep["plan"] = p_

    def layers(events=None):
        plan = plan_keep.get("plan")
        cur = torch.cuda.current_stream(dev)
        for l in range(L):
            if args.path == "split":
                pool.append(l, kn[l], vn[l], bt_d, pos_d)
            if events is not None:
                events[l][0].record(cur)
            if args.path == "split":
                pool.decode(l, q[l], bt_d, lens_d, max_len, out=out[l], workspace=ws)
            else:
                plan.run(l, q[l], bt_d, out=None if gat is not None else out[l], k_new=kn3[l], v_new=vn3[l])
            if events is not None:
                events[l][1].record(cur)
            if gathered is not None:
                ev = torch.cuda.Event()
                ev.record(cur)
                comm.wait_event(ev)
                with torch.cuda.stream(comm):
                    dist.all_gather_into_tensor(gathered[l].view(-1), out[l].view(-1))
        if gathered is not None:
            cur.wait_stream(comm)
        if gat is not None:
            plan.gather_wait(L - 1)  # signal the last layer's slot, wait for every rank's

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        new_plan()
        layers()
    pool.check()  # no device errors during warm-up
    if gat is not None:
        gat.check()
    barrier()

    graph = None
    per_layer_events = True
    if use_graph:
        # the whole L-layer step as one CUDA graph; timing events are graph nodes
        layer_events = [(torch.cuda.Event(enable_timing=True, external=True),
                         torch.cuda.Event(enable_timing=True, external=True)) for _ in range(L)]
        graph = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream(device=dev)
        cap.wait_stream(compute)
        # Event nodes between launches would break the early-start edges; with
        # early start the per-launch time is the step time over the layers.
        per_layer_events = args.path == "split" or args.no_early_start
        with torch.cuda.graph(graph, stream=cap):
            layers(layer_events if per_layer_events else None)
        compute.wait_stream(cap)
        new_plan()
        graph.replay()
        pool.check()

        def step():
            new_plan()
            graph.replay()
    else:
        layer_events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                        for _ in range(L)]

        def step():
            new_plan()
            layers(layer_events)
    barrier()

    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        t_start.record(compute)
        for _ in range(args.steps):
            step()
        t_end.record(compute)
        barrier()
    ms_total = t_start.elapsed_time(t_end)
    if world > 1:
        t = torch.tensor([ms_total], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
    ms_step = ms_total / args.steps
    dec_avg_ms = ms_step / L
    dec_src = "step time / layers (launches back to back, early start)"
    if not use_graph or per_layer_events:
        try:  # per-launch durations of the last timed step
            dec_ms = [a.elapsed_time(b) for a, b in layer_events]
            dec_avg_ms = sum(dec_ms) / len(dec_ms)
            dec_src = "CUDA events around each decode launch of the last timed step"
        except RuntimeError:
            dec_src = "step time / layers (events unavailable)"
    clocks = clk.summary()

    # --- each decode launch timed alone: one more step launched eagerly, no
    # early start, CUDA events around every launch (median over the layers)
    iso_ms = None
    if args.path == "planned":
        p_iso = pool.plan(lens_host, hq_l, workspace=plan_ws)
        p_iso.upload()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(L)]
        barrier()
        for l in range(L):
            evs[l][0].record(compute)
            p_iso.run(l, q[l], bt_d, out=out[l], k_new=kn3[l], v_new=vn3[l])
            evs[l][1].record(compute)
        barrier()
        iso_ms = statistics.median(a.elapsed_time(b) for a, b in evs)
        if world > 1:
            t = torch.tensor([iso_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            iso_ms = float(t.item())
        pool.check()

    # --- DRAM traffic per launch from the committed ncu capture (70B, 1 GPU, planned)
    traffic, traffic_src = None, None
    if (args.config == "70b" and world == 1 and args.path == "planned" and not args.layers and not args.batch
            and args.kv == "fp16"):
        traffic = NCU_DECODE_70B_BYTES
        traffic_src = "ncu capture of one launch: profiles/planned_decode_kernel_70b-one-layer_full.md"

    # --- algorithmic bytes (this rank's share) and roofline of the decode launch
    ab_local = algorithmic_bytes(ctx, hq_l, hkv_l, D, args.kv)
    peak, peak_kind = measured_peaks()
    achieved = ab_local["decode"] / (dec_avg_ms * 1e-3) / 1e9
    ab_job = algorithmic_bytes(ctx_all, Hq, Hkv, D, args.kv)
    job_gbs = ab_job["total"] * L / (ms_step * 1e-3) / 1e9
    tokens_s = B / (ms_step * 1e-3)

    # --- end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, pool, L, Bl, hq_l, hkv_l, D, bt_d, pos_d, lens_d, max_len, ws, dev, world,
                      gathered, comm, lens_host, plan_ws, use_graph, gat)
        e2e["value"] = B / (e2e.pop("ms_step") * 1e-3)

    # --- CPU baseline (rank 0 at N=1 only): oracle port, 1 thread, bounded sample
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rng = np.random.Generator(np.random.PCG64(5))
        sample = np.sort(rng.choice(Bl, max(1, Bl // 8), replace=False))
        frac = float(lens[sample].sum()) / float(lens.sum())
        t_cpu = cpu_decode_sample(wl, bt, ctx, hkv_l, hq_l, sample, 1)
        step_cpu = t_cpu / frac * L
        cpu = {"value": B / step_cpu, "unit": "tokens/s", "cores": 1, "kind": "port",
               "sample": "oracle port of the reference's golden attention, 1 thread: 1 of %d layers, "
                         "%d of %d sequences (all heads); extrapolated x%d layers / %.3f of the tokens "
                         "(%.1f s measured)" % (L, len(sample), Bl, L, frac, t_cpu)}

    if rank == 0:
        line = {
            "metric": METRIC, "value": tokens_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "f16" if args.kv == "fp16" else "e4m3 K/V pages (fp32 scale per 128-value row), f16 Q/O, f32 accumulation",
            "data": "synthetic (seeded N(0,0.5^2) fp16 K/V/Q, random block tables)",
            "config": workload_config(wl, args.kv, world),
            "run": {"parallelism": ("kv-head shard x%d + %s" % (world, "allgather fused into the decode "
                                                                      "(peer stores over NVLink, flag per layer)"
                                                                      + (", each layer waits for the previous "
                                                                         "layer's gather" if args.gather == "p2p-wait"
                                                                         else "")
                                                                      if gat is not None else "NCCL allgather")
                                       if wl["shard"] == "head" else "sequence shard x%d" % world)
                                      if world > 1 else "single GPU",
                       "decode_path": args.path,
                       "launch": "CUDA graph of the %d-layer step" % L if use_graph else "eager",
                       "pages_per_split": pool.pages_per_split(Bl, max_len) if args.path == "split" else None,
                       "plan_workers": pool.plan(lens_host, hq_l).workers if args.path == "planned" else None},
            "hbm_gbs": job_gbs / world,
            "hbm_frac_of_peak": job_gbs / world / peak,
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "traffic_source": traffic_src,
                         "kernel": ("vk_decode_run (planned: append + decode + merge in one launch)"
                                    if args.path == "planned" else "vk_decode (split grid + merge)"),
                         "peak_source": peak_kind, "launch_ms": dec_avg_ms, "launch_timing": dec_src,
                         "launch_ms_alone": iso_ms,
                         "frac_alone": (ab_local["decode"] / (iso_ms * 1e-3) / 1e9 / peak) if iso_ms else None,
                         "alone_timing": "median over the layers of one more step launched eagerly without early "
                                         "start, CUDA events around each launch" if iso_ms else None,
                         "algorithmic_bytes_per_launch": ab_local["decode"]},
            "cpu_baseline": cpu,
            "e2e": e2e,
        }
        print(json.dumps(line), flush=True)
    pool.check()
    if gat is not None:
        gat.check()
    del graph
    if gat is not None:
        gat.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_churn(args, wl):
    """Config 5 on one GPU through vulcan_b200.scheduler: arrivals, LRU swap-out
    to a pinned host arena, swap-in, one decode launch per step (planned, fused
    append) over the resident sequences, compaction by page copy.  Swaps run on a
    side stream and are timed with CUDA events on it; decode and copies on the
    compute stream."""
    import torch
    import vulcan_b200 as vk
    from vulcan_b200.scheduler import PagedKVScheduler
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    H, D, steps = wl["Hq"], wl["D"], wl["steps"]
    ctx = wl["ctx"]
    need = int(((ctx + steps + 15) // 16).sum())
    num_pages = int(wl["capacity"] * need)
    pool = vk.PagedKVPool(1, H, D, num_pages, zero=False)
    g = torch.Generator(device=dev)
    g.manual_seed(9)
    flat = pool.storage.view(torch.float16)
    for s0 in range(0, flat.numel(), 1 << 28):
        part = flat[s0:s0 + (1 << 28)]
        part.copy_(torch.randn(part.shape, device=dev, generator=g) * 0.5)
    host_slots = need - num_pages + 2048
    host = torch.empty(host_slots * pool.page_bytes, dtype=torch.uint8, pin_memory=True)
    swap_stream = torch.cuda.Stream(device=dev)
    compute = torch.cuda.current_stream(dev)
    swap_events = {"out": [], "in": []}

    def on_swap(kind, pages, fn):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        swap_stream.wait_stream(compute)  # pages leaving were last written on the compute stream
        e0.record(swap_stream)
        r = fn()
        e1.record(swap_stream)
        swap_events[kind].append((e0, e1, pages))
        return r

    sched = PagedKVScheduler(pool, host_buffer=host, host_slots=host_slots, swap_stream=swap_stream,
                             on_swap=on_swap)
    rng = np.random.Generator(np.random.PCG64(wl["seed"] + 1))
    arrivals = rng.poisson(wl["rate"], steps)
    kq = (torch.randn(wl["B"], H, D, device=dev, generator=g) * 0.5).half()
    kn = (torch.randn(wl["B"], H, D, device=dev, generator=g) * 0.5).half()
    plan_ws = torch.empty(64 << 20, dtype=torch.uint8, device=dev)
    copy_events = []
    dec_events = []
    decoded = 0
    dec_bytes = 0
    next_sid = 0
    pending: List[int] = []

    def copy_fn(src, dst):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        src_d = torch.tensor(src, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
        dst_d = torch.tensor(dst, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
        e0.record(compute)
        pool.copy_pages(src_d, dst_d)
        e1.record(compute)
        copy_events.append((e0, e1, len(src)))

    torch.cuda.synchronize(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    wall0 = time.perf_counter()
    t0.record(compute)
    for step in range(steps):
        for _ in range(int(arrivals[step])):
            if next_sid < wl["B"]:
                pending.append(next_sid)
                next_sid += 1
        protect = set()
        for _ in range(4):  # bring back the longest-waiting swapped sequences
            if not sched.swapped:
                break
            sid = next(iter(sched.swapped))
            if not sched.restore(sid, protect=protect):
                break
            protect.add(sid)
        while pending:
            sid = pending[0]
            if not sched.admit(sid, int(ctx[sid])):
                break
            pending.pop(0)
            protect.add(sid)
        active = sched.resident_ids()
        active = [sid for sid in active if sched.grow(sid, protect=protect)]
        active = [sid for sid in active if sched.seqs[sid].resident]
        if step % 25 == 24:
            compute.wait_stream(swap_stream)
            sched.compact(copy_fn=copy_fn)
        if not active:
            continue
        bt = torch.from_numpy(sched.block_table(active)).to(dev, non_blocking=True)
        lens = sched.lengths(active)
        compute.wait_stream(swap_stream)  # restored pages in, evicted pages out
        plan = pool.plan(lens.tolist(), H, workspace=plan_ws)
        plan.upload()
        idx = torch.tensor(active, device=dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(compute)
        plan.run(0, kq[idx], bt, k_new=kn[idx], v_new=kn[idx])
        e1.record(compute)
        dec_events.append((e0, e1))
        decoded += len(active)
        dec_bytes += algorithmic_bytes(lens.astype(np.int64) - 1, H, H, D)["total"]
    compute.wait_stream(swap_stream)
    t1.record(compute)
    torch.cuda.synchronize(dev)
    wall = time.perf_counter() - wall0
    pool.check()
    ms = t0.elapsed_time(t1)
    dec_ms = sum(a.elapsed_time(b) for a, b in dec_events)
    res = {"metric": "long-context churn: decode tokens/s and swap / copy GB/s", "value": decoded / (ms * 1e-3),
           "unit": "tokens/s", "n_gpus": 1, "steps": steps, "warmup": 0, "ms_per_step": ms / steps,
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
           "data": "synthetic (seeded)", "config": {"workload": wl["desc"], "pool_pages": num_pages,
                                                   "demand_pages": need, "host_slots": host_slots,
                                                   "page_bytes": pool.page_bytes},
           "decode": {"tokens": decoded, "ms": dec_ms, "hbm_gbs": dec_bytes / (dec_ms * 1e-3) / 1e9},
           "wall_s": wall}
    for kind in ("out", "in"):
        ev = swap_events[kind]
        tms = sum(a.elapsed_time(b) for a, b, _ in ev)
        byt = sum(n for _, _, n in ev) * pool.page_bytes
        res["swap_" + kind] = {"calls": len(ev), "bytes": byt, "ms": tms,
                               "gbs": byt / (tms * 1e-3) / 1e9 if tms > 0 else None}
    cms = sum(a.elapsed_time(b) for a, b, _ in copy_events)
    cby = sum(n for _, _, n in copy_events) * pool.page_bytes * 2
    res["copy"] = {"calls": len(copy_events), "pages": sum(n for _, _, n in copy_events), "ms": cms,
                   "gbs_read_plus_write": cby / (cms * 1e-3) / 1e9 if cms > 0 else None}
    res["scheduler"] = dict(sched.stats)
    print(json.dumps(res), flush=True)


def prefill_flops(ctx, T, Hq, D):
    """Attention FLOPs of one layer: QK^T and PV, 2 FLOPs per multiply-add, over
    the causal (query, key) pairs of each chunk (prefix keys + lower triangle)."""
    pairs = sum(int(T * c + T * (T + 1) // 2) for c in ctx)
    return 4 * D * Hq * pairs


def run_attn_wo(args, wl):
    """Attention + output projection of the 70B decode step (row 8f.3): per layer
    the planned decode of this rank's KV heads (fused append), then the wo
    projection of its attention output fused with the reduce-scatter over output
    features (vk_oproj: tcgen05 GEMM tile by tile, partials stored into the
    owning rank over NVLink).  Eager launches (the projection is a cooperative
    launch); a second pass times the projection launches alone for its
    roofline: weights + x + y through HBM, and the partials that cross NVLink."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    import vulcan_b200 as vk
    from vulcan_b200.shard import head_shard
    B, Hq, Hkv, D, L = wl["B"], wl["Hq"], wl["Hkv"], wl["D"], wl["L"]
    hidden = Hq * D
    ctx = wl["ctx"]
    bt, num_pages = layout(ctx, wl["seed"])
    sh = head_shard(Hkv, Hq, world, rank)
    hkv_l, hq_l = sh.num_kv_heads, sh.num_q_heads
    k_local = hq_l * D
    lens = (ctx + 1).astype(np.int32)
    pool = vk.PagedKVPool(L, hkv_l, D, num_pages, own_memory=False, zero=False)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1000 + rank)
    flat = pool.storage.view(torch.float16)
    for s0 in range(0, flat.numel(), 1 << 28):
        part = flat[s0:s0 + (1 << 28)]
        part.copy_(torch.randn(part.shape, device=dev, generator=gen) * 0.5)
    bt_d = torch.from_numpy(bt).to(dev)
    q = (torch.randn(L, B, hq_l, D, device=dev, generator=gen) * 0.5).half()
    kn = (torch.randn(L, B, hkv_l, D, device=dev, generator=gen) * 0.5).half()
    vn = (torch.randn(L, B, hkv_l, D, device=dev, generator=gen) * 0.5).half()
    # this rank's rows of wo per layer, packed once (as at model load)
    w_t = [vk.OutputProjection.pack_weight_t16((torch.randn(hidden, k_local, device=dev, generator=gen) * 0.02).half())
           for _ in range(L)]
    att = torch.empty(L, B, hq_l, D, device=dev, dtype=torch.float16)
    y = torch.empty(L, B, hidden // world, device=dev, dtype=torch.float16)
    op = vk.OutputProjection(rank, world, B, k_local, hidden, device=dev)
    if world > 1:
        op.exchange()
    lens_host = lens.tolist()
    plan_ws = torch.empty(pool.plan(lens_host, hq_l).workspace.numel() + 4096, dtype=torch.uint8, device=dev)
    keep = {}

    def new_plan():
        p_ = pool.plan(lens_host, hq_l, workspace=plan_ws)
        p_.set_early_start(True)
        p_.upload()
        keep["plan"] = p_

    def layers():
        p_ = keep["plan"]
        for l in range(L):
            p_.run(l, q[l], bt_d, out=att[l], k_new=kn[l], v_new=vn[l])
            op.run(att[l].view(B, k_local), w_t[l], y=y[l])

    graph = None
    if not args.eager:
        # the L-layer step as one CUDA graph (the projection keeps its run
        # number on the device, so replays are valid)
        try:
            new_plan()
            layers()
            torch.cuda.synchronize(dev)
            g_ = torch.cuda.CUDAGraph()
            cap = torch.cuda.Stream(device=dev)
            cap.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.graph(g_, stream=cap):
                layers()
            torch.cuda.current_stream(dev).wait_stream(cap)
            graph = g_
        except Exception as exc:  # capture refused: launch eagerly
            print("graph capture failed (%s); eager launches" % exc, file=sys.stderr)
            graph = None

    def step():
        new_plan()
        if graph is not None:
            graph.replay()
        else:
            layers()

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step()
    barrier()
    op.check()
    pool.check()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        t0.record()
        for _ in range(args.steps):
            step()
        t1.record()
        barrier()
    ms = t0.elapsed_time(t1) / args.steps
    clocks = clk.summary()
    # the projection alone: all layers' projections back to back (each with its
    # own weights, so every launch streams its 8192 x k_local weights from HBM)
    barrier()
    t0.record()
    for _ in range(2):
        for l in range(L):
            op.run(att[l].view(B, k_local), w_t[l], y=y[l])
    t1.record()
    barrier()
    op_ms = t0.elapsed_time(t1) / (2 * L)
    op.check()
    pool.check()
    if world > 1:
        t = torch.tensor([ms, op_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, op_ms = float(t[0]), float(t[1])
    hbm_peak, peak_kind = measured_peaks()
    peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if peak_kind == "measured" else {}
    tflops_peak = float(peaks.get("bf16_tflops", 1590.0))
    hbm_b = hidden * k_local * 2 + B * k_local * 2 + B * (hidden // world) * 2  # weights + x + y
    nvl_b = B * hidden * 4 * (world - 1) // world  # fp32 partials leaving this rank
    flops = 2.0 * B * k_local * hidden
    t_hbm = hbm_b / (hbm_peak * 1e9)
    t_tc = flops / (tflops_peak * 1e12)
    t_nvl = nvl_b / 770e9
    target = max(t_hbm, t_tc, t_nvl)
    bound = "hbm" if target == t_hbm else ("tensor" if target == t_tc else "nvlink")
    ab = algorithmic_bytes(ctx, hq_l, hkv_l, D)
    if rank == 0:
        line = {"metric": "attention + wo step tokens/s (70B decode, head-sharded, wo fused with its reduce-scatter)",
                "value": B / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f16 (fp32 accumulation, fp32 partial sums)",
                "data": "synthetic (seeded N(0,0.5^2) K/V/Q, wo ~ N(0, 0.02^2))",
                "config": workload_config(wl, "fp16", world),
                "run": {"launch": ("CUDA graph of" if graph is not None else "eager:") +
                           " per layer vk_decode_run (early start) + vk_oproj_run (cooperative); projection "
                           "launch time from 2L projections back to back",
                        "oproj_splits": op.splits, "oproj_ctas": (hidden // 128) * op.splits},
                "per_layer_us": ms * 1e3 / L,
                "step_hbm_gbs": (ab["total"] + hbm_b) * L / (ms * 1e-3) / 1e9,
                "gpu_launches": 2 * L * args.steps, "clocks": clocks,
                "roofline": {"kernel": "oproj_kernel (tcgen05 GEMM + reduce-scatter over NVLink)",
                             "bound": bound, "launch_us": op_ms * 1e3,
                             "target_us": target * 1e6, "frac": target / (op_ms * 1e-3),
                             "hbm_bytes": hbm_b, "hbm_gbs": hbm_b / (op_ms * 1e-3) / 1e9, "hbm_peak": hbm_peak,
                             "nvlink_bytes_out": nvl_b, "flops": flops, "tensor_tflops": flops / (op_ms * 1e-3) / 1e12,
                             "peak_source": peak_kind + " (NVLink: 770 GB/s measured peer copy)"}}
        print(json.dumps(line), flush=True)
    op.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_prefill(args, wl):
    """Config 4: per layer, append the 2048-token chunks (K1) then causal prefill
    attention over prefix + chunk (K3); one CUDA graph per step of L layers.
    Sequences are sharded over ranks (no collective)."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    import vulcan_b200 as vk
    B, H, D, L, T = wl["B"], wl["Hq"], wl["D"], wl["L"], wl["T"]
    seqs = np.arange(B)[rank::world]
    ctx = wl["ctx"][seqs]
    Bl = len(seqs)
    bt, num_pages = layout(ctx + T - 1, wl["seed"] + rank, slack=1.0)
    pool = vk.PagedKVPool(L, H, D, num_pages, zero=False, kv_format=args.kv)
    gen = torch.Generator(device=dev)
    gen.manual_seed(5 + rank)
    if args.kv == "fp16":
        flat = pool.storage.view(torch.float16)
        for s0 in range(0, flat.numel(), 1 << 28):
            part = flat[s0:s0 + (1 << 28)]
            part.copy_(torch.randn(part.shape, device=dev, generator=gen) * 0.5)
    else:
        fill_fp8(pool, D, dev, gen)
    bt_d = torch.from_numpy(bt).to(dev)
    pos_d = torch.from_numpy(ctx.astype(np.int32)).to(dev)
    q = (torch.randn(Bl, T, H, D, device=dev, generator=gen) * 0.5).half()
    kn = (torch.randn(Bl, T, H, D, device=dev, generator=gen) * 0.5).half()
    vn = (torch.randn(Bl, T, H, D, device=dev, generator=gen) * 0.5).half()
    out = torch.empty_like(q)
    compute = torch.cuda.current_stream(dev)
    ev = [(torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True))
          for _ in range(L)]

    def layers(record):
        cur = torch.cuda.current_stream(dev)
        for l in range(L):
            pool.append(l, kn, vn, bt_d, pos_d)
            if record:
                ev[l][0].record(cur)
            pool.prefill(l, q, bt_d, pos_d, out=out)
            if record:
                ev[l][1].record(cur)

    for _ in range(args.warmup):
        layers(False)
    pool.check()
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream(device=dev)
    cap.wait_stream(compute)
    with torch.cuda.graph(graph, stream=cap):
        layers(True)
    compute.wait_stream(cap)
    graph.replay()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        t0.record(compute)
        for _ in range(args.steps):
            graph.replay()
        t1.record(compute)
        torch.cuda.synchronize(dev)
    pool.check()
    ms = t0.elapsed_time(t1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    launch_ms = sum(a.elapsed_time(b) for a, b in ev) / L
    flops_local = prefill_flops(ctx, T, H, D)
    flops_job = prefill_flops(wl["ctx"], T, H, D)
    # ncu traffic of the 2-sequence capture scaled by the K/V tiles this launch reads
    full_wl = workload("prefill")
    traffic, traffic_src = None, None
    if args.kv == "fp16":
        traffic = NCU_PREFILL_2SEQ_BYTES * prefill_tile_reads(ctx, T) / prefill_tile_reads(full_wl["ctx"][:2], T)
        traffic_src = ("ncu capture of the first 2 sequences (1 layer), scaled by K/V tiles read: "
                       "profiles/prefill_tc_kernel_small-case_full.md")
    peak_t = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["bf16_tflops"] \
        if os.path.exists(os.path.join(ROOT, "MEASURED_PEAKS.json")) else 1590.0
    achieved = flops_local / (launch_ms * 1e-3) / 1e12
    if rank == 0:
        line = {"metric": "chunked prefill (append + causal attention) tokens/s and TFLOP/s",
                "value": B * T / (ms_step * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None,
                "dtype": "f16" if args.kv == "fp16" else "e4m3 K/V pages (fp32 scale per row), f16 MMA, f32 accumulation",
                "data": "synthetic (seeded N(0,0.5^2) fp16)",
                "config": {"workload": wl["desc"], "kv_format": args.kv,
                           "kernel": ("tcgen05 kernel with FP8-to-fp16 converter warps" if args.kv == "fp8" else
                                      "tcgen05 kernel" if wl["D"] == 128 else "mma.sync kernel"),
                           "launch": "CUDA graph of the %d-layer step" % L,
                           "shard": "sequence x%d" % world if world > 1 else "none"},
                "attn_tflops": flops_job * L / (ms_step * 1e-3) / 1e12,
                "gpu_launches": 2 * L * args.steps, "clocks": clk.summary(),
                "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_t, "unit": "TFLOP/s",
                             "frac": achieved / peak_t, "traffic": traffic, "traffic_source": traffic_src,
                             "kernel": "vk_prefill",
                             "launch_ms": launch_ms, "flops_per_launch": flops_local}}
        print(json.dumps(line), flush=True)
    del graph
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_e2e(args, pool, L, Bl, hq_l, hkv_l, D, bt_d, pos_d, lens_d, max_len, ws, dev, world, gathered, comm,
            lens_host, plan_ws, use_graph, gat=None):
    """Same step through the public API with host buffers: each layer's q/k/v is
    copied from pinned host memory to the device on a copy stream (they stand
    in for the projections a model computes on the device), and every layer's
    attention output (this rank's heads) is copied back to pinned host memory
    on a second copy stream, plus the last layer's all-gathered output when
    heads are sharded, all inside the timed region.  The layers run in chunks
    of growing size (1, 2, 4, 8, 16, ..., the last layer alone): a chunk's
    inputs are copied while the previous chunk runs, its kernels run back to
    back with early start, and its outputs are copied back after its last
    kernel, so only the first layer's inputs and the last layer's output are
    not hidden.  (NCCL all-gather: one layer at a time, double buffered.)  At
    N=1 the step is one CUDA graph."""
    import torch
    import torch.distributed as dist
    g = torch.Generator()
    g.manual_seed(77)
    hq = (torch.randn(L, Bl, hq_l, D, generator=g) * 0.5).half().pin_memory()
    hk = (torch.randn(L, Bl, hkv_l, D, generator=g) * 0.5).half().pin_memory()
    hv = (torch.randn(L, Bl, hkv_l, D, generator=g) * 0.5).half().pin_memory()
    gathered_host = gathered is not None or gat is not None
    out_shape = (world, Bl, hq_l, D) if gathered_host else (Bl, hq_l, D)
    hout = torch.empty(out_shape, dtype=torch.float16).pin_memory()
    hout_layers = torch.empty(L, Bl, hq_l, D, dtype=torch.float16).pin_memory()  # every layer, own heads
    chunked = gathered is None  # NCCL all-gather keeps one layer at a time
    nbuf = L if chunked else 2
    # one device tensor per input / output across the buffered layers, so a
    # chunk's copies are one copy per tensor
    dq = torch.empty(nbuf, Bl, hq_l, D, device=dev, dtype=torch.float16)
    dk = torch.empty(nbuf, Bl, hkv_l, D, device=dev, dtype=torch.float16)
    dv = torch.empty(nbuf, Bl, hkv_l, D, device=dev, dtype=torch.float16)
    douts = torch.empty(nbuf, Bl, hq_l, D, device=dev, dtype=torch.float16)
    h2d = torch.cuda.Stream(device=dev)
    d2h = torch.cuda.Stream(device=dev)
    compute = torch.cuda.current_stream(dev)
    from vulcan_b200.shard import GatherSchedule
    sched = GatherSchedule(L, slots=2 * L)  # the receive buffer holds 2L slots
    h2d_bytes = (hq.numel() + hk.numel() + hv.numel()) * 2
    d2h_bytes = hout_layers.numel() * 2 + (hout.numel() * 2 if gathered_host else 0)
    plan_keep = {}

    chunks = []  # (first layer, layers): growing sizes, the last layer alone
    c0, size = 0, 1
    while c0 < L:
        n = min(size, L - c0)
        chunks.append((c0, n))
        c0 += n
        size = min(2 * size, 16)
    if chunks[-1][1] > 1:
        f, n = chunks.pop()
        chunks += [(f, n - 1), (L - 1, 1)]

    def new_plan(parity=0):
        if args.path == "planned":
            p_ = pool.plan(lens_host, hq_l, workspace=plan_ws)
            if chunked and not args.no_early_start:
                p_.set_early_start(True)  # the layers of a chunk are back to back
            if gat is not None:
                # alternate steps write alternate halves of the 2L slots, so a
                # slot is rewritten only after every rank's copies of it are done
                p_.set_gather(gat, slot_base=sched.slot_base(parity + 1), wait_prev=args.gather == "p2p-wait")
            p_.upload()
            plan_keep["plan"] = p_

    def run_layer(plan, l, s):
        if plan is None:
            pool.append(l, dk[s].view(Bl, 1, hkv_l, D), dv[s].view(Bl, 1, hkv_l, D), bt_d, pos_d)
            pool.decode(l, dq[s], bt_d, lens_d, max_len, out=douts[s], workspace=ws)
        else:
            plan.run(l, dq[s], bt_d, out=None if gat is not None else douts[s], k_new=dk[s], v_new=dv[s])

    def layers_chunked(parity=0):
        base = sched.slot_base(parity + 1)
        cur = torch.cuda.current_stream(dev)
        plan = plan_keep.get("plan")
        h2d.wait_stream(cur)  # the previous step's kernels have read every input buffer
        d2h.wait_stream(cur)
        loaded = []
        with torch.cuda.stream(h2d):
            for c0, n in chunks:
                dq[c0:c0 + n].copy_(hq[c0:c0 + n], non_blocking=True)
                dk[c0:c0 + n].copy_(hk[c0:c0 + n], non_blocking=True)
                dv[c0:c0 + n].copy_(hv[c0:c0 + n], non_blocking=True)
                e = torch.cuda.Event()
                e.record(h2d)
                loaded.append(e)
        for ci, (c0, n) in enumerate(chunks):
            cur.wait_event(loaded[ci])
            for l in range(c0, c0 + n):
                run_layer(plan, l, l)
            fe = torch.cuda.Event()
            fe.record(cur)
            d2h.wait_event(fe)
            with torch.cuda.stream(d2h):
                if gat is None:
                    hout_layers[c0:c0 + n].copy_(douts[c0:c0 + n], non_blocking=True)
                for l in range(c0, c0 + n) if gat is not None else ():
                    hout_layers[l].copy_(gat.view(base + l, Bl, hq_l, D)[gat.rank], non_blocking=True)
                    if l == L - 1:
                        plan.gather_wait(l, stream=d2h)  # every rank's slices of the step
                        hout.copy_(gat.view(base + l, Bl, hq_l, D), non_blocking=True)
        cur.wait_stream(d2h)  # outputs read before the next step rewrites them
        cur.wait_stream(h2d)

    def layers(parity=0):
        if chunked:
            return layers_chunked(parity)
        base = sched.slot_base(parity + 1)
        cur = torch.cuda.current_stream(dev)
        plan = plan_keep.get("plan")
        h2d.wait_stream(cur)
        d2h.wait_stream(cur)
        loaded = [None] * nbuf
        freed = [None] * nbuf
        outdone = [None] * nbuf

        def load(l):
            s = l % nbuf
            with torch.cuda.stream(h2d):
                if freed[s] is not None:
                    h2d.wait_event(freed[s])
                dq[s].copy_(hq[l], non_blocking=True)
                dk[s].copy_(hk[l], non_blocking=True)
                dv[s].copy_(hv[l], non_blocking=True)
                e = torch.cuda.Event()
                e.record(h2d)
                loaded[s] = e

        load(0)
        for l in range(L):
            s = l % nbuf
            if l + 1 < L:
                load(l + 1)
            cur.wait_event(loaded[s])
            if outdone[s] is not None:
                cur.wait_event(outdone[s])
            run_layer(plan, l, s)
            fe = torch.cuda.Event()
            fe.record(cur)
            freed[s] = fe
            last = l == L - 1
            if gat is not None:
                # this rank's own slice of the layer's slot (written by its run)
                d2h.wait_event(fe)
                with torch.cuda.stream(d2h):
                    hout_layers[l].copy_(gat.view(base + l, Bl, hq_l, D)[gat.rank], non_blocking=True)
                    if last:
                        # wait for every rank's slices of the last layer (ranks
                        # raise their flags in layer order, so this covers the
                        # step), then read the whole slot
                        plan.gather_wait(l, stream=d2h)
                        hout.copy_(gat.view(base + l, Bl, hq_l, D), non_blocking=True)
            else:
                if gathered_host:
                    comm.wait_event(fe)
                    with torch.cuda.stream(comm):
                        dist.all_gather_into_tensor(gathered[l].view(-1), douts[s].view(-1))
                        ge = torch.cuda.Event()
                        ge.record(comm)
                    d2h.wait_event(ge)  # the all-gather has read douts[s]
                else:
                    d2h.wait_event(fe)
                with torch.cuda.stream(d2h):
                    hout_layers[l].copy_(douts[s], non_blocking=True)
                    if gathered_host and last:
                        hout.copy_(gathered[l], non_blocking=True)
                    od = torch.cuda.Event()
                    od.record(d2h)
                    outdone[s] = od  # douts[s] may be rewritten after this
        cur.wait_stream(d2h)
        cur.wait_stream(h2d)

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    counter = [0]
    for _ in range(args.warmup):
        par = counter[0] % 2
        counter[0] += 1
        new_plan(par)
        layers(par)
    barrier()
    graph = None
    graphs = []
    per_layer_events = True
    if use_graph:
        for par in ((0, 1) if gat is not None else (0,)):
            g_ = torch.cuda.CUDAGraph()
            cap = torch.cuda.Stream(device=dev)
            cap.wait_stream(compute)
            new_plan(par)
            with torch.cuda.graph(g_, stream=cap):
                layers(par)
            compute.wait_stream(cap)
            graphs.append(g_)

        def step():
            par = counter[0] % len(graphs)
            counter[0] += 1
            new_plan(par)
            graphs[par].replay()
    else:
        def step():
            par = counter[0] % 2
            counter[0] += 1
            new_plan(par)
            layers(par)
    step()
    barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(compute)
    for _ in range(args.steps):
        step()
    t1.record(compute)
    barrier()
    ms = t0.elapsed_time(t1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    del graph, graphs
    return {"ms_step": ms / args.steps, "unit": "tokens/s", "h2d_bytes_per_step": int(h2d_bytes),
            "d2h_bytes_per_step": int(d2h_bytes),
            "path": "PagedKVPool / DecodePlan (C ABI): every layer's q, k, v from pinned host memory; every "
                    "layer's attention output (this rank's heads) back to pinned host memory" +
                    (", and the last layer's all-gathered output" if gathered_host else "") +
                    "; H2D and D2H on copy streams inside the timed region" +
                    ("; layers in chunks of %s, each chunk's copies overlapping the previous chunk's kernels, "
                     "early start within a chunk" % "/".join(str(n) for _, n in chunks) if chunked else
                     "; one layer at a time, double buffered") +
                    ("; CUDA graph per step" if use_graph else "")}


if __name__ == "__main__":
    main()
