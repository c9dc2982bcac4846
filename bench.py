"""Benchmark of the OomLlama GQA attention step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-secondary]

Headline workload (the causal-prefill configuration of the metric): one
Qwen2.5-7B-shaped layer, 28 q / 4 kv heads, head_dim 128, 4096 new tokens,
bf16 Q/K/V ~N(0,1), interleaved RoPE theta=1e6, causal.  One step = K-A
(RoPE of Q and K + append of K/V into the paged bf16 cache) + K-C (tcgen05
causal prefill) for one sequence per GPU (weak scaling: N GPUs process N
independent sequences).  Metric: algorithmic causal FLOPs
4*d*Hq*S(S+1)/2 per sequence / step time (TFLOP/s).

Secondary lines in the same JSON object ("decode"): split-KV decode HBM GB/s
and tokens/s for the Llama-3-8B long-context shape (32q/8kv, batch 8, 32768
context, bf16, sharded by kv-head group across GPUs) and the batched
Qwen2.5-7B decode (batch 64, context U[1024, 8192], shuffled 16-token pages;
with more GPUs than kv heads the context is split and the partial (O, lse)
are all-gathered over NCCL and merged).

--impl reference times the oracle's restatement of the reference's scalar
f32 CPU attention (src/oom_inference.rs:240-272) on the host's cores over a
bounded sample of the same workload.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

S_PREFILL, HQ, HKV, D = 4096, 28, 4, 128
PREFILL_FLOPS = 4 * D * HQ * S_PREFILL * (S_PREFILL + 1) // 2   # 120,288,444,416 per sequence
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# a device-side sleep (about 25 us) queued before a start event: the host enqueues the launches
# meanwhile, so the event pairs bracket device work, not host launch latency (used for the per-stage
# split of a split-context decode step; a kernel's own time comes from a CUDA graph of its launches)
GPU_SLEEP_CYCLES = 50_000
ENQUEUE_SLEEP_CYCLES = 4_000_000  # about 2 ms at 1.9 GHz: covers the host enqueue of a timed decode loop
L2_BYTES = 126 * 1024 * 1024  # B200 L2: timed loops rotate inputs past it
SPEC_PEAKS = {"hbm_gbs": 7700.0, "bf16_tflops": 2250.0}  # nominal B200 (HGX HBM3e; dense bf16), for context
# dram__bytes_read.sum + dram__bytes_write.sum per launch from one ncu capture
# of each kernel on these workloads: the 4096-token causal prefill and the
# 8 x 32768-token Llama-3 decode.
NCU_TRAFFIC_BYTES = {"prefill_bf16_kernel": 37_828_608 + 7_362_048, "decode_bf16_kernel": 1_074_328_000 + 5_611_008}


SECTIONS = ("prefill", "decode-llama", "decode-qwen", "c1", "q8", "layer", "repack", "model")


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--only", default="", help="comma-separated subset of: " + ", ".join(SECTIONS) +
                   " (\"decode\" = both decode configurations); default all")
    p.add_argument("--no-secondary", action="store_true", help="the headline prefill only")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


def sections(args):
    if args.no_secondary:
        return {"prefill"}
    if not args.only:
        return set(SECTIONS)
    out = set()
    for name in args.only.split(","):
        name = name.strip()
        if name == "decode":
            out |= {"decode-llama", "decode-qwen"}
        elif name in SECTIONS:
            out.add(name)
        elif name:
            raise SystemExit(f"--only: unknown section {name!r}")
    return out


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            pk = json.load(f)
        return {k: float(pk[k]) for k in FALLBACK_PEAKS}, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


# ---------------------------------------------------------------- distributed
class Dist:
    def __init__(self, gpus):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = False
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist
            torch.cuda.set_device(self.local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                    device_id=torch.device(f"cuda:{self.local}"))
            self.pg = True

    def barrier(self):
        if self.pg:
            import torch
            import torch.distributed as dist
            dist.barrier(device_ids=[self.local])
            torch.cuda.synchronize()

    def max(self, x: float) -> float:
        if not self.pg:
            return x
        import torch
        import torch.distributed as dist
        t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{self.local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum(self, x: float) -> float:
        if not self.pg:
            return x
        import torch
        import torch.distributed as dist
        t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{self.local}")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    def close(self):
        if self.pg:
            import torch.distributed as dist
            dist.destroy_process_group()


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
        return False

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() in ("active", "1", "yes"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- prefill (headline)
def block_flops(blocks, n_heads, s=S_PREFILL):
    """Algorithmic causal FLOPs of the 256-row query blocks `blocks` ([lo, hi) ranges) for n_heads
    q heads: query row i sees i + 1 keys, 4 * d FLOPs per (row, key)."""
    f = 0
    for lo, hi in blocks:
        r0, r1 = 256 * lo, min(s, 256 * hi)
        f += (r1 * (r1 + 1) - r0 * (r0 + 1)) // 2
    return 4 * D * n_heads * f


def bench_prefill(args, dist_, torch, strong):
    """One C2 prefill step per GPU.  strong: the ranks share ONE sequence (PrefillShardPlan: kv-head
    groups, then zig-zag query blocks); otherwise every rank runs its own whole sequence."""
    from oomllama_b200 import TurboConfig, TurboEngine
    from oomllama_b200.shard import PrefillShardPlan
    dev = torch.cuda.current_device()
    W, r = dist_.world, dist_.rank
    plan = PrefillShardPlan(HQ, HKV, W if strong else 1, r if strong else 0)
    hq, hkv = len(plan.q_heads), len(plan.kv_heads)
    blocks = plan.blocks(S_PREFILL)
    rank_flops = block_flops(blocks, hq)
    cfg = TurboConfig(n_layers=1, hidden_size=hq * D, n_heads=hq, n_kv_heads=hkv, max_seq_len=S_PREFILL,
                      max_seqs=1, kv_dtype="bf16", rope_variant="interleaved", rope_theta=1e6)
    eng = TurboEngine(cfg, device=dev)
    n_sets = 4  # 4 x 37.7 MB of Q/K/V inputs (whole heads) > 126 MB L2, rotated between steps
    g = torch.Generator(device="cuda").manual_seed(1 + (plan.group if strong else r))
    sets = []
    for _ in range(n_sets):
        q = torch.randn(S_PREFILL, hq * D, generator=g, device="cuda").to(torch.bfloat16)
        k = torch.randn(S_PREFILL, hkv * D, generator=g, device="cuda").to(torch.bfloat16)
        v = torch.randn(S_PREFILL, hkv * D, generator=g, device="cuda").to(torch.bfloat16)
        sets.append((q, k, v))
    out = torch.empty(S_PREFILL, hq, D, dtype=torch.float32, device="cuda")
    pf_stream = torch.cuda.current_stream()

    def step(i, ev=None, qkv=None, o=None):
        q, k, v = sets[i % n_sets] if qkv is None else qkv
        eng.reset()
        qr = eng.rope_append(0, [0], q, k, v, q_out_dtype=torch.bfloat16)
        eng.prefill(0, 0, qr, out=out if o is None else o, blocks=blocks)
        return qr

    for i in range(args.warmup):
        step(i)
    eng.sync()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def load_for(seconds):
        # untimed steps around the timed region so the 200 ms clock sampler
        # sees this kernel's clocks under load
        end = time.perf_counter() + seconds
        i = 0
        while time.perf_counter() < end:
            step(i)
            i += 1
            if i % 32 == 0:
                torch.cuda.synchronize()
        torch.cuda.synchronize()

    # one CUDA graph per input set holds a whole step (K-A then K-C; the positions are fixed at
    # capture, so every replay appends at the same slots and does the same work)
    side = torch.cuda.Stream()
    graphs = []
    with torch.cuda.stream(side):
        step(0)
        for i in range(n_sets):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=side):
                step(i)
            graphs.append(gr)
    torch.cuda.synchronize()
    for i in range(max(3, args.warmup)):
        graphs[i % n_sets].replay()
    with ClockSampler(dev) as clk:
        load_for(0.7)
        dist_.barrier()
        torch.cuda.synchronize()
        t0.record()
        for i in range(args.steps):
            graphs[i % n_sets].replay()
        t1.record()
        torch.cuda.synchronize()
        dist_.barrier()
        # the prefill kernel alone: a CUDA graph of back-to-back launches over each set's rotated q (the
        # cache holds the last set's K/V; every launch does the step's work), CUDA events on its stream
        qrs = [step(i).clone() for i in range(n_sets)]
        with torch.cuda.stream(side):
            kg = torch.cuda.CUDAGraph()
            with torch.cuda.graph(kg, stream=side):
                for i in range(n_sets):
                    eng.prefill(0, 0, qrs[i], out=out, blocks=blocks)
        torch.cuda.synchronize()
        kg.replay()
        ka, kb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ka.record()
        for _ in range(args.steps):
            kg.replay()
        kb.record()
        torch.cuda.synchronize()
        load_for(0.5)
    eng.sync()
    del graphs, kg
    ms = t0.elapsed_time(t1) / args.steps
    kern_ms = ka.elapsed_time(kb) / (args.steps * n_sets)
    ms_max = dist_.max(ms)
    kern_max = dist_.max(kern_ms)

    # e2e through the public API with pinned host buffers.  Every step copies this rank's Q/K/V
    # host->device, runs RoPE/append + prefill, and copies the f32 attention rows of its query
    # blocks device->host.  Like a serving loop, the copies run on their own streams and overlap the
    # neighbouring steps' compute (inputs and outputs double-buffered on both sides).
    rows = [(256 * lo, min(S_PREFILL, 256 * hi)) for lo, hi in blocks]
    hq_ = [tuple(t.cpu().pin_memory() for t in s_) for s_ in sets[:2]]
    ho = [torch.empty(S_PREFILL, hq, D, dtype=torch.float32).pin_memory() for _ in range(2)]
    dq = [[torch.empty_like(t) for t in sets[0]] for _ in range(2)]
    dout = [torch.empty(S_PREFILL, hq, D, dtype=torch.float32, device="cuda") for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    s_comp = pf_stream
    ev = lambda: torch.cuda.Event()  # noqa: E731
    in_ready, in_free = [ev(), ev()], [ev(), ev()]
    out_ready, out_free = [ev(), ev()], [ev(), ev()]
    for e_ in in_free + out_free:
        e_.record(s_comp)

    def e2e_step(i):
        b = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(in_free[b])
            for d_, h_ in zip(dq[b], hq_[i % 2]):
                d_.copy_(h_, non_blocking=True)
            in_ready[b].record(s_in)
        s_comp.wait_event(in_ready[b])
        s_comp.wait_event(out_free[b])
        step(i, qkv=dq[b], o=dout[b])
        in_free[b].record(s_comp)
        out_ready[b].record(s_comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(out_ready[b])
            for a_, z_ in rows:
                ho[b][a_:z_].copy_(dout[b][a_:z_], non_blocking=True)
            out_free[b].record(s_out)

    for i in range(3):
        e2e_step(i)
    torch.cuda.synchronize()
    e_steps = max(4, args.steps)
    dist_.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(s_in)
    for i in range(e_steps):
        e2e_step(i)
    b.record(s_out)
    torch.cuda.synchronize()
    dist_.barrier()
    e2e_ms = dist_.max(a.elapsed_time(b) / e_steps)
    h2d = sum(t.numel() * t.element_size() for t in hq_[0])
    d2h = sum((z_ - a_) * hq * D * 4 for a_, z_ in rows)
    eng.close()
    return {
        "ms": ms_max, "kernel_ms": kern_max, "kernel_ms_local": kern_ms, "clocks": clk.summary(), "e2e_ms": e2e_ms,
        "h2d": dist_.sum(h2d), "d2h": dist_.sum(d2h), "launches_per_step": 2, "rank_flops": rank_flops,
        "heads": hq, "blocks": blocks,
    }


# ---------------------------------------------------------------- decode (secondary)
def f64_attention(q, k, v, scale):
    """Float64 restatement of one decode row for the in-bench parity check: q [hq, d], k, v
    [hkv, L, d]; q head h reads kv head h // (hq / hkv); softmax(scale * K q) V per head."""
    hq, hkv = q.shape[0], k.shape[0]
    grp = hq // hkv
    out = np.empty_like(q, dtype=np.float64)
    for h in range(hq):
        kk, vv = k[h // grp].astype(np.float64), v[h // grp].astype(np.float64)
        s_ = kk @ q[h].astype(np.float64) * scale
        p = np.exp(s_ - s_.max())
        out[h] = p @ vv / p.sum()
    return out


def bench_decode(args, dist_, torch, name):
    """Split-KV decode.  llama: 32q/8kv, batch 8, 32768 context, split-half theta=5e5, sharded by
    kv-head group (strong scaling: the same 8 x 32768 work at every N).  qwen-batched: 28q/4kv, batch
    64, context U[1024,8192], shuffled pages; beyond 4 GPUs each context is split in world/4 slices,
    and one step is the packed decode, ONE all-gather of the group's (O, lse) partials over NCCL and
    the merge.  After timing, rank-local parity of sampled rows (every local q head) against a
    float64 restatement over the whole context (slices gathered from the group)."""
    from oomllama_b200 import TurboConfig, TurboEngine
    from oomllama_b200.shard import DecodeShardPlan, SplitContextDecoder, new_group_comms
    dev = torch.cuda.current_device()
    W, r = dist_.world, dist_.rank
    if name == "llama-32k":
        hq, hkv, B, variant, theta = 32, 8, 8, "split_half", 5e5
        lens = [32768] * B
    else:
        hq, hkv, B, variant, theta = 28, 4, 64, "interleaved", 1e6
        lens = np.random.default_rng(2).integers(1024, 8193, size=B).tolist()
        lens = [L + 1 for L in lens]  # cached tokens + the new one
    plan = DecodeShardPlan(hq, hkv, W, r)
    ctx_split = plan.ctx_split
    l_hkv, l_hq = len(plan.kv_heads), len(plan.q_heads)
    slices = [plan.context_slice(L) for L in lens]  # this rank's slice of every sequence: whole pages
    local = [b - a for a, b in slices]
    n_pages = sum(-(-x // 16) for x in local)
    # timed steps rotate over enough layers of cache that a rank's working set
    # exceeds 1.5x the L2 (126 MB): a layer is read again only after the others
    rank_bytes = sum(local) * l_hkv * D * 2 * 2
    n_layers = max(1, min(8, -(-int(1.5 * L2_BYTES) // max(1, rank_bytes))))
    cfg = TurboConfig(n_layers=n_layers, hidden_size=0, n_heads=l_hq, n_kv_heads=l_hkv, max_seq_len=max(lens) + 16,
                      max_seqs=B, n_pages=max(1, n_pages), kv_dtype="bf16", rope_variant=variant, rope_theta=theta)
    eng = TurboEngine(cfg, device=dev, assign_pages=False)
    perm = np.random.default_rng(3 + r).permutation(max(1, n_pages))
    tables, o = [], 0
    for s in range(B):
        np_s = -(-local[s] // 16)
        tables.append(perm[o:o + np_s])
        eng.set_block_table(s, tables[s].tolist())
        o += np_s
        for layer in range(n_layers):
            eng.set_seq_len(layer, s, local[s])
    kp, vp = eng.kv_pool()
    g = torch.Generator(device="cuda").manual_seed(11 + r)
    kp.normal_(generator=g)
    vp.normal_(generator=g)
    kp[:, -1].zero_()
    vp[:, -1].zero_()  # the null page stays zero
    # the query is the same on every rank of a group (its heads, seeded by the group)
    gq = torch.Generator(device="cuda").manual_seed(101 + plan.group)
    q = torch.randn(B, l_hq, D, generator=gq, device="cuda")
    comm = None
    if dist_.pg:
        import torch.distributed as tdist
        comm = new_group_comms(plan, tdist)[plan.group]  # every rank creates every group, in order
    dec = SplitContextDecoder(eng, plan, tdist if dist_.pg else None, comm)
    seqs = list(range(B))
    merge = ctx_split > 1
    stream = torch.cuda.current_stream()

    def step(ev=None, layer=0):
        if ev is not None:
            # the GPU sleeps while the host enqueues the step, so the events bracket device work only
            torch.cuda._sleep(GPU_SLEEP_CYCLES)
            ev[0].record(stream)
        if not merge:
            out = eng.decode(layer, seqs, q)
            if ev is not None:
                ev[1].record(stream)
            return out
        packed, gathered, out = dec.buffers(B, l_hq, q.device)
        eng.decode_packed(layer, seqs, q, out=packed)
        if ev is not None:
            ev[1].record(stream)
        from oomllama_b200.shard import gather_packed
        gather_packed(packed, plan, tdist, comm, out=gathered)
        if ev is not None:
            ev[2].record(stream)
        eng.merge_packed(gathered, ctx_split, out=out.view(B * l_hq, D))
        if ev is not None:
            ev[3].record(stream)
        return out

    steps = max(5, args.steps)
    for i in range(max(args.warmup, n_layers)):
        step(layer=i % n_layers)
    eng.sync()
    mk = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    evs = [(mk(), mk(), mk(), mk()) if merge else (mk(), mk()) for _ in range(steps)]
    t0, t1 = mk(), mk()
    dist_.barrier()
    # The GPU sleeps while the host enqueues every timed step (each is up to
    # three host calls, one of them an NCCL all-gather), so the events bracket
    # back-to-back device work, as a captured serving loop would run it.
    torch.cuda._sleep(ENQUEUE_SLEEP_CYCLES)
    t0.record(stream)
    for i in range(steps):
        step(layer=i % n_layers)
    t1.record(stream)
    torch.cuda.synchronize()
    dist_.barrier()
    ms = dist_.max(t0.elapsed_time(t1) / steps)
    # the decode kernel alone: a CUDA graph of back-to-back launches on this rank
    side = torch.cuda.Stream()
    packed = dec.buffers(B, l_hq, q.device)[0] if merge else None
    kl = [i % n_layers for i in range(4)]
    with torch.cuda.stream(side):
        for layer in kl[:2]:
            eng.decode_packed(layer, seqs, q, out=packed) if merge else eng.decode(layer, seqs, q)
        kg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(kg, stream=side):
            for layer in kl:
                eng.decode_packed(layer, seqs, q, out=packed) if merge else eng.decode(layer, seqs, q)
    torch.cuda.synchronize()
    kg.replay()
    ka, kb = mk(), mk()
    ka.record(stream)
    for _ in range(steps):
        kg.replay()
    kb.record(stream)
    torch.cuda.synchronize()
    kern_local = ka.elapsed_time(kb) / (4 * steps)
    del kg
    # the all-gather and merge stages of a split-context step: CUDA events around each (eager steps)
    coll_ms = merge_ms = 0.0
    if merge:
        dist_.barrier()
        for i in range(steps):
            step(evs[i], layer=i % n_layers)
        torch.cuda.synchronize()
        coll_ms = sum(e[1].elapsed_time(e[2]) for e in evs) / steps
        merge_ms = sum(e[2].elapsed_time(e[3]) for e in evs) / steps
    dist_.barrier()
    eng.sync()
    kern_max = dist_.max(kern_local)
    local_bytes = sum(local) * l_hkv * D * 2 * 2
    total_bytes = sum(lens) * hkv * D * 2 * 2

    # parity: sampled rows, every local q head, over the whole context
    out = step()
    torch.cuda.synchronize()
    scale = 1.0 / math.sqrt(D)
    rows = np.random.default_rng(17).choice(B, size=min(3, B), replace=False)
    worst, worst_rel = 0.0, 0.0
    for z in rows:
        pg = torch.from_numpy(tables[z].astype(np.int64)).cuda()
        kr = kp[0].index_select(0, pg).permute(1, 0, 2, 3).reshape(l_hkv, -1, D)[:, :local[z]]
        vr = vp[0].index_select(0, pg).permute(1, 0, 2, 3).reshape(l_hkv, -1, D)[:, :local[z]]
        if merge:  # the group's slices of this row, in slice order
            import torch.distributed as tdist
            cap = max(plan.slice_of(lens[z], s_)[1] - plan.slice_of(lens[z], s_)[0] for s_ in range(ctx_split))
            pad_k = torch.zeros(l_hkv, cap, D, dtype=kr.dtype, device="cuda")
            pad_v = torch.zeros_like(pad_k)
            pad_k[:, :local[z]] = kr
            pad_v[:, :local[z]] = vr
            gk = [torch.empty_like(pad_k) for _ in range(ctx_split)]
            gv = [torch.empty_like(pad_v) for _ in range(ctx_split)]
            tdist.all_gather(gk, pad_k, group=comm)
            tdist.all_gather(gv, pad_v, group=comm)
            n_s = [plan.slice_of(lens[z], s_)[1] - plan.slice_of(lens[z], s_)[0] for s_ in range(ctx_split)]
            kr = torch.cat([gk[s_][:, :n_s[s_]] for s_ in range(ctx_split)], dim=1)
            vr = torch.cat([gv[s_][:, :n_s[s_]] for s_ in range(ctx_split)], dim=1)
        ref = f64_attention(q[z].cpu().numpy(), kr.float().cpu().numpy(), vr.float().cpu().numpy(), scale)
        got = out[z].double().cpu().numpy()
        worst = max(worst, float(np.abs(got - ref).max()))
        worst_rel = max(worst_rel, float(np.linalg.norm(got - ref) / np.linalg.norm(ref)))
    worst, worst_rel = dist_.max(worst), dist_.max(worst_rel)
    eng.close()
    return {"ms": ms, "kernel_ms": kern_max, "kern_local_ms": kern_local, "coll_ms": dist_.max(coll_ms),
            "merge_ms": dist_.max(merge_ms), "local_bytes": local_bytes, "total_bytes": total_bytes, "batch": B,
            "merge": merge, "lens_sum": sum(lens), "parity_max_abs": worst, "parity_rel": worst_rel,
            "parity_ok": bool(worst <= 2e-3 and worst_rel <= 1e-2), "cache_layers": n_layers}


# ---------------------------------------------------------------- Q8 linear (K-E, secondary)
Q8_LAYER = (("qkv", 4608, 3584), ("o_proj", 3584, 3584), ("gate_up", 37888, 3584), ("down", 3584, 18944))


def bench_q8(args, dist_, torch, T):
    """One Qwen2.5-7B layer's linears from GPU-resident Q8 weights (qkv fused 4608x3584, o_proj 3584x3584,
    gate+up fused 37888x3584, down 3584x18944) for T decode tokens: the weights a decode step streams
    (src/oomllama.rs:425-439 dequantises and uploads them per call instead).  Two layers' weights
    (466 MB) rotate, so no matrix is L2-resident when it is read."""
    from oomllama_b200 import Q8Matrix, TurboConfig, TurboEngine
    dev = torch.cuda.current_device()
    eng = TurboEngine(TurboConfig(n_layers=1, hidden_size=0, n_heads=8, n_kv_heads=1, max_seq_len=16, max_seqs=1,
                                  kv_dtype="bf16"), device=dev)
    g = torch.Generator(device="cuda").manual_seed(21 + dist_.rank)
    layers = []
    for _ in range(2):
        mats = []
        for _, rows, cols in Q8_LAYER:
            nb = (rows * cols + 255) // 256
            q = torch.randint(0, 256, (rows * cols,), dtype=torch.uint8, device="cuda", generator=g)
            mats.append(Q8Matrix(q, torch.rand(nb, device="cuda", generator=g) * 1e-3,
                                 -torch.rand(nb, device="cuda", generator=g) * 0.1, rows, cols))
        layers.append(mats)
    xs = {cols: torch.randn(T, cols, device="cuda", generator=g) for _, _, cols in Q8_LAYER}
    ys = {rows: torch.empty(T, rows, device="cuda") for _, rows, _ in Q8_LAYER}
    byts = sum(r * c + 8 * ((r * c + 255) // 256) + 4 * T * (r + c) for _, r, c in Q8_LAYER)

    def step(i):
        for (name, rows, cols), w in zip(Q8_LAYER, layers[i % 2]):
            eng.q8_linear(w, xs[cols], out=ys[rows])

    # a decode step is replayed as a CUDA graph (8 launches: x split + linear per matrix), so the
    # measurement is the kernels and their dependencies, not the Python host loop
    side = torch.cuda.Stream()
    graphs = []
    with torch.cuda.stream(side):
        for i in range(max(2, args.warmup)):
            step(i)  # grows the library's scratch before capture
        for i in range(2):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=side):
                step(i)
            graphs.append(gr)
    torch.cuda.synchronize()
    eng.sync()
    for i in range(args.warmup):
        graphs[i % 2].replay()
    steps = max(10, args.steps)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist_.barrier()
    torch.cuda.synchronize()
    t0.record()
    for i in range(steps):
        graphs[i % 2].replay()
    t1.record()
    torch.cuda.synchronize()
    dist_.barrier()
    eng.sync()
    ms = dist_.max(t0.elapsed_time(t1) / steps)
    del graphs
    eng.close()
    del layers
    return ms, byts


def bench_layer_q8(args, dist_, torch, B, ctx_len=2048):
    """One Qwen2.5-7B decoder layer's decode step on resident Q8 weights (oomattn_decoder_layer_q8:
    RMSNorm, QKV + bias, RoPE + append, split-KV attention over ctx_len cached bf16 tokens, o_proj +
    residual, RMSNorm, gated MLP + residual) for B sequences, replayed as a CUDA graph."""
    from oomllama_b200 import Q8DecoderLayer, Q8Matrix, TurboConfig, TurboEngine
    dev = torch.cuda.current_device()
    H, hq, hkv, inter = 3584, 28, 4, 18944
    pages_per = -(-(ctx_len + 1) // 16)
    cfg = TurboConfig(n_layers=1, hidden_size=H, n_heads=hq, n_kv_heads=hkv, max_seq_len=ctx_len + 16, max_seqs=B,
                      n_pages=B * pages_per, kv_dtype="bf16", rope_variant="interleaved", rope_theta=1e6)
    eng = TurboEngine(cfg, device=dev, assign_pages=False)
    perm = np.random.default_rng(7 + dist_.rank).permutation(B * pages_per)
    for b in range(B):
        eng.set_block_table(b, perm[b * pages_per:(b + 1) * pages_per].tolist())
        eng.set_seq_len(0, b, ctx_len)
    g = torch.Generator(device="cuda").manual_seed(31 + dist_.rank)
    kp, vp = eng.kv_pool()
    kp.normal_(generator=g)
    vp.normal_(generator=g)
    kp[:, -1].zero_()
    vp[:, -1].zero_()

    def mat(rows, cols):
        nb = (rows * cols + 255) // 256
        q = torch.randint(0, 256, (rows * cols,), dtype=torch.uint8, device="cuda", generator=g)
        return Q8Matrix(q, torch.rand(nb, device="cuda", generator=g) * 2e-4,
                        -torch.rand(nb, device="cuda", generator=g) * 0.02, rows, cols)

    w = Q8DecoderLayer(q=mat(hq * D, H), k=mat(hkv * D, H), v=mat(hkv * D, H), o=mat(H, hq * D), gate=mat(inter, H),
                       up=mat(inter, H), down=mat(H, inter), input_norm=torch.ones(H, device="cuda"),
                       post_norm=torch.ones(H, device="cuda"), eps=1e-6,
                       bq=torch.zeros(hq * D, device="cuda"), bk=torch.zeros(hkv * D, device="cuda"),
                       bv=torch.zeros(hkv * D, device="cuda"))
    x = torch.randn(B, H, device="cuda", generator=g)
    out = torch.empty_like(x)
    seqs = list(range(B))
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        for _ in range(2):  # grows the scratch; each call appends at the next slot
            eng.decoder_layer_q8(0, seqs, x, w, out=out)
        for b in range(B):
            eng.set_seq_len(0, b, ctx_len)  # replays then overwrite slot ctx_len: the same work every step
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=side):
            eng.decoder_layer_q8(0, seqs, x, w, out=out)
    torch.cuda.synchronize()
    eng.sync()
    for _ in range(max(3, args.warmup)):
        gr.replay()
    steps = max(10, args.steps)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist_.barrier()
    torch.cuda.synchronize()
    t0.record()
    for _ in range(steps):
        gr.replay()
    t1.record()
    torch.cuda.synchronize()
    dist_.barrier()
    eng.sync()
    ms = dist_.max(t0.elapsed_time(t1) / steps)
    wbytes = sum(r * c + 8 * ((r * c + 255) // 256) for r, c in
                 [(hq * D, H), (hkv * D, H), (hkv * D, H), (H, hq * D), (inter, H), (inter, H), (H, inter)])
    kvbytes = B * (ctx_len + 1) * hkv * D * 2 * 2
    del gr
    eng.close()
    return ms, wbytes + kvbytes


def bench_c1(args, dist_, torch, n_sets=4, cached=512):
    """C1: one Qwen2.5-7B layer's f32 attention step for one sequence with 512 cached tokens:
    K-A GEMV over f32 Wq/Wk/Wv (66 MB) + bias + interleaved RoPE + append at slot 512, then the
    f32 K-B decode over 513 tokens.  n_sets layers, each with its own weights and cache, rotate so
    the 4 x 68 MB working set exceeds L2; replayed as a CUDA graph (slot 512 rewritten every step)."""
    from oomllama_b200 import TurboConfig, TurboEngine
    dev = torch.cuda.current_device()
    H, hq, hkv = 3584, 28, 4
    cfg = TurboConfig(n_layers=n_sets, hidden_size=H, n_heads=hq, n_kv_heads=hkv, max_seq_len=cached + 16,
                      max_seqs=1, kv_dtype="f32", rope_variant="interleaved", rope_theta=1e6)
    eng = TurboEngine(cfg, device=dev)
    g = torch.Generator(device="cuda").manual_seed(0 + dist_.rank)
    ws = []
    for l in range(n_sets):
        eng.kv_write(l, 0, torch.randn(cached, hkv, D, device="cuda", generator=g),
                     torch.randn(cached, hkv, D, device="cuda", generator=g))
        ws.append([torch.randn(n * D, H, device="cuda", generator=g) * 0.02 for n in (hq, hkv, hkv)])
    bq, bk, bv = (torch.zeros(n * D, device="cuda") for n in (hq, hkv, hkv))
    x = torch.randn(1, H, device="cuda", generator=g)
    out = torch.empty(1, hq, D, device="cuda")
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        for l in range(n_sets):  # warm the scratch on this stream
            q = eng.qkv_rope_append(l, [0], x, *ws[l], bq, bk, bv)
            eng.decode(l, [0], q, out=out)
            eng.set_seq_len(l, 0, cached)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=side):
            for l in range(n_sets):
                q = eng.qkv_rope_append(l, [0], x, *ws[l], bq, bk, bv)
                eng.decode(l, [0], q, out=out)
    torch.cuda.synchronize()
    eng.sync()
    for _ in range(max(3, args.warmup)):
        gr.replay()
    reps = max(10, args.steps)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist_.barrier()
    torch.cuda.synchronize()
    t0.record()
    for _ in range(reps):
        gr.replay()
    t1.record()
    torch.cuda.synchronize()
    dist_.barrier()
    eng.sync()
    ms = dist_.max(t0.elapsed_time(t1) / (reps * n_sets))
    L = cached + 1
    byts = ((hq + 2 * hkv) * D * H * 4 + (hq + 2 * hkv) * D * 4 + H * 4  # weights, biases, x
            + 2 * hkv * L * D * 4 + 2 * hkv * D * 4 + 2 * hq * D * 4)  # K/V read, K/V append, q and O
    del gr
    eng.close()
    return ms, byts


def cpu_c1_sample(threads=None, reps=5):
    """The oracle's f32 layer attention (QKV matvec + bias + interleaved RoPE + append + GQA
    attention, oomllama_turbo.rs:618-723 up to o_proj) for the C1 shape; returns (tok/s, threads)."""
    from oracle import oracle as O
    O.build()
    nt = O.set_threads(O.host_cores() if threads is None else threads)
    rng = np.random.default_rng(0)
    H, hq, hkv, P = 3584, 28, 4, 512
    x = rng.standard_normal((1, 1, H), dtype=np.float32)
    wq, wk, wv = (rng.standard_normal((n * D, H), dtype=np.float32) * np.float32(0.02) for n in (hq, hkv, hkv))
    kc = rng.standard_normal((1, hkv, P, D), dtype=np.float32)
    vc = rng.standard_normal((1, hkv, P, D), dtype=np.float32)
    cos_t, sin_t = O.rope_table(1e6, D, P + 1)
    best = 1e30
    for _ in range(reps):
        t = time.perf_counter()
        O.layer_attention(x, wq, wk, wv, None, None, None, hq, hkv, kc, vc, cos_t, sin_t, O.ROPE_INTERLEAVED)
        best = min(best, time.perf_counter() - t)
    return 1.0 / best, nt


def q8_random_matrix(torch, rows, cols, g, std=0.02, chunk=1 << 26):
    """A Q8 matrix of weights ~N(0, std) quantised on the device the way the .oom writer does
    (src/gguf2oom.rs:719-770: per 256-value block min, scale = range / 255, q = round((v - min) / scale));
    rows * cols must be a multiple of 256."""
    from oomllama_b200 import Q8Matrix
    n = rows * cols
    q = torch.empty(n, dtype=torch.uint8, device="cuda")
    scale = torch.empty(n // 256, device="cuda")
    mn = torch.empty(n // 256, device="cuda")
    for o in range(0, n, chunk):
        m = min(chunk, n - o)
        v = (torch.randn(m, device="cuda", generator=g) * std).view(-1, 256)
        lo, hi = v.min(1).values, v.max(1).values
        sc = (hi - lo) / 255.0
        sc = torch.where((hi - lo).abs() < 1e-9, torch.zeros_like(sc), sc)
        qq = torch.where(sc[:, None] > 0, torch.floor((v - lo[:, None]) / sc[:, None].clamp_min(1e-30) + 0.5),
                         torch.zeros_like(v)).clamp_(0, 255)
        q[o:o + m] = qq.view(-1).to(torch.uint8)
        scale[o // 256:(o + m) // 256] = sc
        mn[o // 256:(o + m) // 256] = lo
    return Q8Matrix(q, scale, mn, rows, cols)


def bench_model_q8(args, dist_, torch, B=16, prompt=2048, gen=256, n_layers=28):
    """The whole Qwen2.5-7B-shaped model on resident Q8 weights: the prompt of B sequences x `prompt` random
    token ids through oomattn_prefill_step_q8 (every layer's projections on the tensor cores, K-A append,
    K-C causal attention; timed separately), then `gen` greedy steps of oomattn_decode_step_q8 (embedding, 28
    decoder layers, final RMSNorm, LM head 152064 x 3584, argmax; each step's ids feed the next on the device
    and are copied to pinned host memory) over the cache the prefill wrote."""
    from oomllama_b200 import Q8DecoderLayer, Q8Model, TurboConfig, TurboEngine
    dev = torch.cuda.current_device()
    H, hq, hkv, inter, vocab = 3584, 28, 4, 18944, 152064
    cap = prompt + gen + 8
    pages_per = -(-cap // 16)
    cfg = TurboConfig(n_layers=n_layers, hidden_size=H, n_heads=hq, n_kv_heads=hkv, max_seq_len=cap, max_seqs=B,
                      n_pages=B * pages_per, kv_dtype="bf16", rope_variant="interleaved", rope_theta=1e6)
    eng = TurboEngine(cfg, device=dev, assign_pages=False)
    perm = np.random.default_rng(9 + dist_.rank).permutation(B * pages_per)
    for b in range(B):
        eng.set_block_table(b, perm[b * pages_per:(b + 1) * pages_per].tolist())
    g = torch.Generator(device="cuda").manual_seed(4 + dist_.rank)
    bias = lambda n: torch.randn(n, device="cuda", generator=g) * 0.02  # noqa: E731
    layers = [Q8DecoderLayer(q=q8_random_matrix(torch, hq * D, H, g), k=q8_random_matrix(torch, hkv * D, H, g),
                             v=q8_random_matrix(torch, hkv * D, H, g), o=q8_random_matrix(torch, H, hq * D, g),
                             gate=q8_random_matrix(torch, inter, H, g), up=q8_random_matrix(torch, inter, H, g),
                             down=q8_random_matrix(torch, H, inter, g), input_norm=torch.ones(H, device="cuda"),
                             post_norm=torch.ones(H, device="cuda"), eps=1e-6, bq=bias(hq * D), bk=bias(hkv * D),
                             bv=bias(hkv * D)) for _ in range(n_layers)]
    model = Q8Model(layers=layers, embed=q8_random_matrix(torch, vocab, H, g),
                    lm_head=q8_random_matrix(torch, vocab, H, g), final_norm=torch.ones(H, device="cuda"), eps=1e-6)
    seqs = list(range(B))
    prompt_ids = torch.randint(0, vocab, (B, prompt), dtype=torch.int32, device="cuda", generator=g)
    tokens = torch.empty(B, dtype=torch.int32, device="cuda")
    out_host = torch.empty(gen, B, dtype=torch.int32).pin_memory()
    stream = torch.cuda.current_stream()
    mk = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731

    def run_prefill():
        eng.reset()
        eng.prefill_step_q8(model, seqs, prompt_ids, next_tokens=tokens)

    run_prefill()  # warm-up: grows the scratch
    eng.sync()
    dist_.barrier()
    p0, p1 = mk(), mk()
    p0.record(stream)
    run_prefill()
    p1.record(stream)
    torch.cuda.synchronize()
    eng.sync()
    prefill_ms = dist_.max(p0.elapsed_time(p1))
    first = tokens.clone()
    # decode warm-up, then the timed chain from the prefill's state
    for _ in range(max(3, args.warmup)):
        eng.decode_step_q8(model, seqs, tokens, next_tokens=tokens)
    eng.sync()
    for l in range(n_layers):
        for b in range(B):
            eng.set_seq_len(l, b, prompt)
    tokens.copy_(first)
    t0, t1 = mk(), mk()
    dist_.barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev) as clk:
        t0.record(stream)
        for i in range(gen):
            eng.decode_step_q8(model, seqs, tokens, next_tokens=tokens)
            out_host[i].copy_(tokens, non_blocking=True)
        t1.record(stream)
        torch.cuda.synchronize()
    clocks = clk.summary()
    dist_.barrier()
    eng.sync()
    ms = dist_.max(t0.elapsed_time(t1))
    ids = out_host.numpy()
    lens_ok = all(eng.seq_len(l, b) == prompt + gen for l in (0, n_layers - 1) for b in range(B))
    wbytes = sum(m.rows * m.cols + 8 * (m.rows * m.cols // 256) for lay in layers
                 for m in (lay.q, lay.k, lay.v, lay.o, lay.gate, lay.up, lay.down))
    wbytes += vocab * H + 8 * (vocab * H // 256)  # LM head (the embedding reads B rows)
    kv_per_step = sum(B * (prompt + i + 1) * hkv * D * 2 * 2 * n_layers for i in range(gen)) / gen
    layer_params = sum(m.rows * m.cols for m in (layers[0].q, layers[0].k, layers[0].v, layers[0].o, layers[0].gate,
                                                 layers[0].up, layers[0].down))
    prefill_flops = 2.0 * B * prompt * layer_params * n_layers + \
        n_layers * B * 4.0 * D * hq * prompt * (prompt + 1) / 2 + 2.0 * B * vocab * H
    eng.close()
    return {"ms": ms, "ids": ids, "lens_ok": lens_ok, "weight_bytes": wbytes, "kv_bytes_per_step": kv_per_step,
            "clocks": clocks, "prefill_ms": prefill_ms, "prefill_flops": prefill_flops}


def synthetic_q8_stream(rows, cols, seed=6):
    """A valid .oom Q8 block stream of rows*cols values (a multiple of 256): per block
    [f32 scale][f32 min][u32 256][256 random bytes] (src/gguf2oom.rs:782-829 layout)."""
    n = rows * cols
    nb = n // 256
    rng = np.random.default_rng(seed)
    blk = np.empty((nb, 268), np.uint8)
    blk[:, 0:4] = (rng.random(nb, dtype=np.float32) * 1e-3).view(np.uint8).reshape(nb, 4)
    blk[:, 4:8] = (-rng.random(nb, dtype=np.float32) * 0.05).view(np.uint8).reshape(nb, 4)
    blk[:, 8:12] = np.frombuffer(np.uint32(256).tobytes(), np.uint8)
    blk[:, 12:] = rng.integers(0, 256, (nb, 256), dtype=np.uint8)
    return blk.reshape(-1)


def bench_oom_repack(args, dist_, torch, rows=18944, cols=3584):
    """The .oom loader path for one Qwen2.5-7B gate matrix (Q8, 67.9 M values, a 70.5 MB block stream):
    the device repack from a resident stream (oomattn_q8_repack), and end to end from pinned host memory
    (one H2D copy + the repack).  Returns (device ms, e2e ms, stream bytes, device bytes moved)."""
    from oomllama_b200 import TurboConfig, TurboEngine
    dev = torch.cuda.current_device()
    eng = TurboEngine(TurboConfig(n_layers=1, hidden_size=0, n_heads=8, n_kv_heads=1, max_seq_len=16, max_seqs=1),
                      device=dev)
    host = torch.from_numpy(synthetic_q8_stream(rows, cols)).pin_memory()
    n = rows * cols
    d_stream = host.to("cuda")
    w = eng.q8_repack(d_stream, n, rows, cols)  # allocates the outputs once
    for _ in range(3):
        eng.q8_repack(d_stream, n, rows, cols)
    eng.sync()
    reps = max(10, args.steps)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist_.barrier()
    torch.cuda.synchronize()
    t0.record()
    for _ in range(reps):
        eng.q8_repack(d_stream, n, rows, cols)
    t1.record()
    torch.cuda.synchronize()
    ms = dist_.max(t0.elapsed_time(t1) / reps)
    t0.record()
    for _ in range(reps):
        d_stream.copy_(host, non_blocking=True)
        eng.q8_repack(d_stream, n, rows, cols)
    t1.record()
    torch.cuda.synchronize()
    e2e_ms = dist_.max(t0.elapsed_time(t1) / reps)
    eng.sync()
    byts = host.numel()
    moved = byts + n + 8 * (n // 256)
    del w
    eng.close()
    return ms, e2e_ms, byts, moved


def cpu_oom_sample(rows=2048, cols=3584):
    """The reference's loader work on the host for a sample of the same stream: the block walk that
    dequantises to f32 (OomLoader::dequantize_tensor_into, src/quant.rs:431-463; the oracle's restatement),
    and this library's host unpack (oomattn_q8_unpack).  Returns GB/s of stream bytes for each."""
    from oracle import oracle as O
    from oomllama_b200 import q8_unpack
    O.build()
    s = synthetic_q8_stream(rows, cols)
    n = rows * cols
    t = time.perf_counter()
    O.q8_dequantize(s, n)
    deq = s.size / (time.perf_counter() - t) / 1e9
    t = time.perf_counter()
    q8_unpack(s, n)
    unp = s.size / (time.perf_counter() - t) / 1e9
    return deq, unp


def cpu_q8_sample(T, rows_per_matrix=64):
    """The oracle's Q8 dequantise + matvec (src/quant.rs:201-224, src/oom_inference.rs:168-180) on
    rows_per_matrix rows of each matrix of the layer; returns GB/s of algorithmic bytes and threads."""
    from oracle import oracle as O
    O.build()
    nt = O.set_threads(O.host_cores())
    rng = np.random.default_rng(5)
    total_bytes, total_s = 0, 0.0
    for _, rows, cols in Q8_LAYER:
        w = (rng.standard_normal((rows_per_matrix, cols)) * 0.02).astype(np.float32)
        stream = O.q8_quantize(w)
        x = rng.standard_normal((T, cols)).astype(np.float32)
        t = time.perf_counter()
        wd = O.q8_dequantize(stream, w.size).reshape(w.shape)
        O.linear(x, wd)
        total_s += time.perf_counter() - t
        total_bytes += w.size + 8 * ((w.size + 255) // 256) + 4 * T * (rows_per_matrix + cols)
    return total_bytes / total_s / 1e9, nt


# ---------------------------------------------------------------- CPU baseline (oracle port)
def cpu_prefill_sample(seconds_budget=8.0, threads=None):
    """Time the oracle's scalar causal attention (oom_inference.rs:240-272 per
    (query row, head)) on a sample of (row, head) pairs of the 4096-token
    prefill; returns (TFLOP/s, threads, description)."""
    from oracle import oracle as O
    O.build()
    rng = np.random.default_rng(0)
    q = rng.standard_normal((S_PREFILL, HQ, D), dtype=np.float32)
    k = rng.standard_normal((HKV, S_PREFILL, D), dtype=np.float32)
    v = rng.standard_normal((HKV, S_PREFILL, D), dtype=np.float32)
    nt = O.set_threads(O.host_cores() if threads is None else threads)
    n_pairs = 64 * nt
    while True:
        rows = rng.integers(0, S_PREFILL, n_pairs).astype(np.int32)
        heads = rng.integers(0, HQ, n_pairs).astype(np.int32)
        t = time.perf_counter()
        O.gqa_attention_rows(q, k, v, rows, heads, causal=True)
        dt = time.perf_counter() - t
        flops = float(np.sum(4.0 * D * (rows.astype(np.float64) + 1)))
        if dt > 1.0 or n_pairs > 4096 * nt:
            break
        n_pairs = int(n_pairs * min(8.0, max(2.0, seconds_budget / 4 / max(dt, 1e-3))))
    return flops / dt / 1e12, nt, f"{n_pairs} random (query row, head) pairs of the 4096-token causal prefill"


def reference_arm(args):
    """--impl reference: the oracle port of the reference's CPU attention, all host threads."""
    dist_ = Dist(args.gpus)
    if dist_.rank != 0:
        dist_.close()
        return
    from oracle import oracle as O
    O.build()
    nt = O.set_threads(O.host_cores())
    rng = np.random.default_rng(0)
    q = rng.standard_normal((S_PREFILL, HQ, D), dtype=np.float32)
    k = rng.standard_normal((HKV, S_PREFILL, D), dtype=np.float32)
    v = rng.standard_normal((HKV, S_PREFILL, D), dtype=np.float32)
    n_pairs = 48 * nt
    vals = []
    for i in range(args.warmup + args.steps):
        rows = rng.integers(0, S_PREFILL, n_pairs).astype(np.int32)
        heads = rng.integers(0, HQ, n_pairs).astype(np.int32)
        t = time.perf_counter()
        O.gqa_attention_rows(q, k, v, rows, heads, causal=True)
        dt = time.perf_counter() - t
        if i >= args.warmup:
            vals.append((float(np.sum(4.0 * D * (rows + 1.0))), dt))
    flops = sum(f for f, _ in vals)
    secs = sum(t for _, t in vals)
    value = flops / secs / 1e12
    ms_step = secs / len(vals) * 1e3
    line = {
        "impl": "reference", "metric": "prefill-attn TFLOPS (causal GQA 28q/4kv d128, S=4096)",
        "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic ~N(0,1), seeded", "config": workload_config(args.gpus),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": nt, "kind": "port",
                         "sample": f"{n_pairs} random (query row, head) pairs per step of the 4096-token causal "
                                   f"prefill (oracle/attn_ref.c restating src/oom_inference.rs:240-272)"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    dist_.close()


def workload_config(n):
    return {"workload": "causal prefill, Qwen2.5-7B GQA 28q/4kv d128, one sequence of 4096 tokens, bf16 Q/K/V "
                        "~N(0,1), interleaved RoPE theta=1e6, paged bf16 KV cache (16-token pages)",
            "sequences": 1, "seq_len": S_PREFILL,
            "parallelism": "1 GPU" if n == 1 else
            f"one sequence over {n} GPUs: kv-head groups" + (", zig-zag 256-row query blocks" if n > HKV else ""),
            "l2": "inputs rotated over 4 sets of 37.7 MB (> 126 MB L2)"}


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    import torch
    dist_ = Dist(args.gpus)
    torch.cuda.set_device(dist_.local)
    from oomllama_b200 import _lib
    _lib.load()  # fail loudly when the library is missing
    only = sections(args)
    peaks, peak_src = load_peaks()
    W = dist_.world
    line = {"metric": "prefill-attn TFLOPS (causal GQA 28q/4kv d128, S=4096)", "value": None, "unit": "TFLOP/s",
            "n_gpus": W, "steps": args.steps, "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic ~N(0,1), seeded",
            "config": workload_config(W)}
    summary = {}
    if "prefill" in only:
        pf = bench_prefill(args, dist_, torch, strong=True)
        achieved = pf["rank_flops"] / (pf["kernel_ms"] * 1e-3) / 1e12
        timed_s = pf["ms"] * args.steps * 1e-3
        peak_key = "bf16_tflops_sustained" if timed_s > 1.0 else "bf16_tflops"
        line.update({
            "value": PREFILL_FLOPS / (pf["ms"] * 1e-3) / 1e12, "ms_per_step": pf["ms"],
            "roofline": {"bound": "tensor", "kernel": "prefill_bf16_kernel", "achieved": achieved,
                         "peak": peaks[peak_key], "unit": "TFLOP/s", "frac": achieved / peaks[peak_key],
                         "frac_of_spec": achieved / SPEC_PEAKS["bf16_tflops"],
                         "peak_source": f"{peak_src} {peak_key}",
                         "traffic": NCU_TRAFFIC_BYTES["prefill_bf16_kernel"] if W == 1 else None,
                         "algorithmic_flops_per_launch": pf["rank_flops"], "heads_per_gpu": pf["heads"],
                         "query_blocks_per_gpu": pf["blocks"]},
            "e2e": {"value": PREFILL_FLOPS / (pf["e2e_ms"] * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": pf["h2d"], "d2h_bytes_per_step": pf["d2h"],
                    "api": "TurboEngine.rope_append + TurboEngine.prefill (C ABI) from pinned host buffers"},
            "gpu_launches": pf["launches_per_step"] * args.steps,
            "clocks": pf["clocks"],
        })
        summary["prefill"] = {"tflops": round(line["value"], 1), "kernel_us": round(pf["kernel_ms"] * 1e3, 1),
                              "frac": round(line["roofline"]["frac"], 4)}
        if W > 1:
            wk = bench_prefill(args, dist_, torch, strong=False)
            line["weak_scaling"] = {
                "value": W * PREFILL_FLOPS / (wk["ms"] * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": wk["ms"],
                "kernel_ms": wk["kernel_ms"], "sequences": W, "parallelism": f"one whole sequence per GPU x{W}"}
            summary["prefill"]["weak_tflops"] = round(line["weak_scaling"]["value"], 1)
    dec = {}
    for name in ("llama-32k", "qwen-batched"):
        if ("decode-llama" if name == "llama-32k" else "decode-qwen") not in only:
            continue
        r = bench_decode(args, dist_, torch, name)
        gbs = r["total_bytes"] / (r["ms"] * 1e-3) / 1e9
        kern_gbs = r["local_bytes"] / (r["kernel_ms"] * 1e-3) / 1e9
        dec[name] = {
            "hbm_gbs": gbs, "tok_s": r["batch"] / (r["ms"] * 1e-3), "ms_per_step": r["ms"],
            "bytes_per_step": r["total_bytes"], "split_context_merge": r["merge"], "scaling": "strong",
            "l2": f"steps rotate over {r['cache_layers']} cache layers (a rank's share x layers > 1.5 x 126 MB L2); "
                  "the GPU sleeps while the host enqueues the timed loop",
            "stages_ms": {"decode_kernel": r["kernel_ms"], "all_gather": r["coll_ms"], "merge": r["merge_ms"]},
            "roofline": {"bound": "hbm", "kernel": "decode_bf16_kernel", "achieved": kern_gbs,
                         "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": kern_gbs / peaks["hbm_gbs"],
                         "frac_of_spec": kern_gbs / SPEC_PEAKS["hbm_gbs"],
                         "traffic": NCU_TRAFFIC_BYTES["decode_bf16_kernel"] if name == "llama-32k" and W == 1
                         else None},
            "parity": {"ok": r["parity_ok"], "max_abs": r["parity_max_abs"], "rel": r["parity_rel"],
                       "against": "float64 restatement, 3 sampled rows x every q head, whole context"},
        }
        summary["decode_" + ("c4" if name == "llama-32k" else "c3")] = {
            "gbs": round(gbs, 1), "tok_s": round(dec[name]["tok_s"], 1), "step_us": round(r["ms"] * 1e3, 1),
            "kern_us": round(r["kernel_ms"] * 1e3, 1), "coll_us": round(r["coll_ms"] * 1e3, 1),
            "merge_us": round(r["merge_ms"] * 1e3, 1), "frac_gpu": round(dec[name]["roofline"]["frac"], 4),
            "parity_ok": r["parity_ok"]}
    if dec:
        line["decode"] = dec
        if line["value"] is None:  # a decode-only run: its first configuration is the line's metric
            first = next(iter(dec.values()))
            line.update({"metric": "decode-attn HBM GB/s", "value": first["hbm_gbs"], "unit": "GB/s",
                         "ms_per_step": first["ms_per_step"], "roofline": first["roofline"]})
    if "c1" in only:
        ms, byts = bench_c1(args, dist_, torch)
        gbs = byts / (ms * 1e-3) / 1e9
        line["c1_decode_f32"] = {
            "workload": "one Qwen2.5-7B layer's f32 attention step, B=1, 512 cached + 1 new: K-A GEMV over f32 "
                        "Wq/Wk/Wv (66 MB) + bias + interleaved RoPE + append, then f32 K-B decode",
            "tok_s": W / (ms * 1e-3), "ms_per_step": ms, "bytes_per_step": byts, "hbm_gbs": W * gbs,
            "roofline": {"bound": "hbm", "kernel": "qkv_gemv_rope_append_kernel + decode_f32_kernel",
                         "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": gbs / peaks["hbm_gbs"],
                         "frac_of_spec": gbs / SPEC_PEAKS["hbm_gbs"], "traffic": None},
            "l2": "4 layers' weights and caches rotate (4 x 68 MB > 126 MB L2)",
        }
        summary["c1"] = {"step_us": round(ms * 1e3, 1), "frac": round(gbs / peaks["hbm_gbs"], 4)}
        if dist_.rank == 0 and W == 1 and not args.no_cpu_baseline:
            v, nt = cpu_c1_sample()
            line["c1_decode_f32"]["cpu_baseline"] = {
                "value": v, "unit": "tok/s", "cores": nt, "kind": "port",
                "sample": "the whole C1 step: oracle QKV matvec + RoPE + append + GQA attention, best of 5"}
    if "q8" in only:
        q8 = {}
        for T in (1, 8, 16):
            ms, byts = bench_q8(args, dist_, torch, T)
            gbs = W * byts / (ms * 1e-3) / 1e9
            q8[f"qwen7b-layer-T{T}"] = {
                "hbm_gbs": gbs, "ms_per_step": ms, "bytes_per_step": byts, "tokens": T,
                "linears": [f"{n} {r_}x{c}" for n, r_, c in Q8_LAYER],
                "roofline": {"bound": "hbm", "kernel": "q8_linear_kernel (with q8_prep_x_kernel)",
                             "achieved": gbs / W, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                             "frac": gbs / W / peaks["hbm_gbs"], "traffic": None},
            }
            if dist_.rank == 0 and W == 1 and not args.no_cpu_baseline:
                v, nt = cpu_q8_sample(T)
                q8[f"qwen7b-layer-T{T}"]["cpu_baseline"] = {
                    "value": v, "unit": "GB/s", "cores": nt, "kind": "port",
                    "sample": "64 rows of each linear: oracle Q8 dequantise + matvec"}
        line["q8_linear"] = q8
        summary["q8_frac"] = {k.split("-")[-1]: round(v["roofline"]["frac"], 3) for k, v in q8.items()}
    if "layer" in only:
        lay = {}
        for B in (1, 16):
            ms, byts = bench_layer_q8(args, dist_, torch, B)
            lay[f"qwen7b-B{B}-ctx2048"] = {
                "ms_per_step": ms, "tok_s_per_layer": W * B / (ms * 1e-3),
                "tok_s_28_layers": W * B / (28 * ms * 1e-3), "hbm_gbs": W * byts / (ms * 1e-3) / 1e9,
                "bytes_per_step": byts,
                "note": "decode step of one decoder layer (no embedding / LM head); tok_s_28_layers = B / (28 x step)",
                "roofline": {"bound": "hbm", "kernel": "decoder layer (K-E, K-A, K-B, RMSNorm)",
                             "achieved": byts / (ms * 1e-3) / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                             "frac": byts / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"], "traffic": None},
            }
        line["decoder_layer_q8"] = lay
    if "repack" in only:
        ms, e2e_ms, sb, moved = bench_oom_repack(args, dist_, torch)
        rp = {
            "workload": "device repack of a Qwen2.5-7B gate matrix's .oom Q8 block stream (18944 x 3584, 70.5 MB)",
            "stream_gbs": W * sb / (ms * 1e-3) / 1e9, "ms": ms,
            "roofline": {"bound": "hbm", "kernel": "q8_repack_kernel", "achieved": moved / (ms * 1e-3) / 1e9,
                         "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": moved / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"], "traffic": None,
                         "algorithmic_bytes": moved},
            "e2e": {"value": W * sb / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s of stream", "h2d_bytes_per_step": sb,
                    "d2h_bytes_per_step": 0, "api": "H2D copy from pinned memory + TurboEngine.q8_repack"},
        }
        if dist_.rank == 0 and W == 1 and not args.no_cpu_baseline:
            deq, unp = cpu_oom_sample()
            rp["cpu_baseline"] = {"value": deq, "unit": "GB/s of stream", "cores": 1, "kind": "port",
                                  "sample": "2048 x 3584 of the same stream: the oracle's block walk to f32",
                                  "host_unpack_gbs": unp}
        line["oom_repack"] = rp
    if "model" in only:
        B, P, G = 16, 2048, 256
        r = bench_model_q8(args, dist_, torch, B, P, G)
        step_ms = r["ms"] / G
        step_bytes = r["weight_bytes"] + r["kv_bytes_per_step"]
        line["model_q8"] = {
            "workload": f"Qwen2.5-7B-shaped 28 layers, Q8 weights ~N(0,0.02), B={B}, prompt {P}, {G} greedy steps",
            "tok_s": W * B * G / (r["ms"] * 1e-3), "decode_ms": r["ms"], "ms_per_step": step_ms,
            "bytes_per_step": step_bytes, "hbm_gbs": step_bytes / (step_ms * 1e-3) / 1e9,
            "frac_of_hbm": step_bytes / (step_ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
            "prefill": {"tok_s": W * B * P / (r["prefill_ms"] * 1e-3), "ms": r["prefill_ms"],
                        "tflops": r["prefill_flops"] / (r["prefill_ms"] * 1e-3) / 1e12,
                        "frac_of_bf16_peak": r["prefill_flops"] / (r["prefill_ms"] * 1e-3) / 1e12 /
                        peaks["bf16_tflops_sustained"],
                        "api": "TurboEngine.prefill_step_q8: 16 x 2048 random prompt ids, all 28 layers"},
            "prompt": "random token ids run through the model's prefill; decode attends over the KV it wrote",
            "api": "TurboEngine.decode_step_q8 per step, ids copied to pinned host memory each step",
            "distinct_ids": int(len(np.unique(r["ids"]))), "lens_ok": r["lens_ok"], "clocks": r["clocks"],
            "cpu_baseline": None,
            "cpu_baseline_note": "not run: the full-size CPU reference model is infeasible on the host",
        }
        summary["model_q8"] = {"tok_s": round(line["model_q8"]["tok_s"], 1),
                               "frac": round(line["model_q8"]["frac_of_hbm"], 4),
                               "prefill_tok_s": round(line["model_q8"]["prefill"]["tok_s"], 1)}
    if "prefill" in only and dist_.rank == 0 and W == 1 and not args.no_cpu_baseline:
        v, nt, desc = cpu_prefill_sample()
        v1, _, desc1 = cpu_prefill_sample(seconds_budget=3.0, threads=1)
        line["cpu_baseline"] = {"value": v, "unit": "TFLOP/s", "cores": nt, "kind": "port", "sample": desc,
                                "single_thread": {"value": v1, "cores": 1, "sample": desc1}}
    # the compact summary goes last: a reader that keeps only the end of the line still sees the
    # decode half of the metric and the per-stage split
    line["summary"] = summary
    if dist_.rank == 0:
        print(json.dumps(line))
    dist_.close()


if __name__ == "__main__":
    main()
