"""Decode-attention benchmark of the InnerQ hot path on B200.

    python bench.py [--gpus N --steps K --warmup W]            # this framework
    python bench.py --impl reference [--steps K --warmup W]     # reference CPU path

Workload (the metric's configuration): Llama-3-8B attention
shape — 32 layers, 32 query / 8 KV heads, head_dim 128 — batch 32, context
32768, 4-bit InnerQ cache (K channel groups of 32, symmetric, normalised, flush
1; V token groups of 32, symmetric, flush 32; 32 sink + 96 recent fp16 tokens).
K = N(0,1) x exp(N(0,1)) per channel, V = N(0,1), q = N(0,1), fp16, seeded.

One step = one decode token through all 32 layers: append the new K/V token
(quantize-and-pack) and run the fused decode attention per layer.  With N
GPUs the 8 KV heads (and their query heads) are partitioned across ranks.  By
default the scaling is weak: the global batch is 32 x N, so every GPU holds
the one-GPU workload's 256 (sequence, KV head) pairs and the attention path
has no exchange; `--scaling strong` splits the 32-sequence workload itself and
all-gathers the KV-head shards' outputs over NCCL once per step.

`value` is algorithmic HBM bytes per step (packed codes + scales + fp16 sink /
recent + normalisation factor + q + out, summed over all ranks) / time.
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
import types

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode attn HBM GB/s (4-bit QK^T+AV, Llama-3-8B attention shape)"
D = 128
NOMINAL_HBM_GBS = 8000.0  # B200 HBM3e, nominal (DGX figure)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--ctx", type=int, default=None)
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--hq", type=int, default=None)
    ap.add_argument("--hkv", type=int, default=8)
    ap.add_argument("--kbits", type=int, default=None)
    ap.add_argument("--vbits", type=int, default=None)
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"],
                    help="weak (default): every GPU keeps the one-GPU workload's (sequence, KV "
                         "head) pairs, the global batch grows with the GPU count and the KV heads "
                         "are partitioned (no exchange on the attention path); strong: the "
                         "one-GPU workload itself is split, and the KV-head shards' outputs are "
                         "all-gathered once per step")
    ap.add_argument("--ctx-shards", type=int, default=1,
                    help="context chunks per KV-head shard (N GPUs = head shards x ctx shards): "
                         "each rank stores one chunk of the context, the split partials are "
                         "all-gathered within the chunk group and log-sum-exp merged per layer")
    ap.add_argument("--group", type=int, default=32)
    ap.add_argument("--v-layout", default="tokens", choices=["tokens", "channels"],
                    help="value groups over tokens (InnerQ default) or over channels "
                         "(groups along head_dim for K and V)")
    ap.add_argument("--mode", default="symmetric", choices=["symmetric", "asymmetric"],
                    help="quantisation mode of both K and V")
    ap.add_argument("--no-graph", action="store_true",
                    help="launch every kernel from the host each step instead of replaying the "
                         "recorded decode step (CUDA graph, cache graph mode)")
    ap.add_argument("--only", default=None,
                    help="sweep: run only the rows whose name contains this text (=NAME: exactly)")
    ap.add_argument("--sweep-ctx", type=int, default=None,
                    help="sweep: override the context of the selected rows (small profiling cases)")
    ap.add_argument("--sweep-batch", type=int, default=None,
                    help="sweep: override the batch of the selected rows")
    ap.add_argument("--sweep-hkv", type=int, default=None,
                    help="sweep: KV heads of the selected rows (a KV-head shard of a larger model)")
    ap.add_argument("--split-scan", default=None,
                    help="sweep: comma-separated split counts to time (0 = the planner's), "
                         "attention only, one JSON line per count")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--workload", default="c1", choices=["c1", "c3", "c4", "sweep"],
                    help="c1: decode attention over a 32-layer cache (default); "
                         "c4: the same over the 70B-shaped 80-layer 2-bit cache (B 8, Hq 64, "
                         "131072 tokens); "
                         "c3: full decode step of a random-init Llama-3-8B-shaped model; "
                         "sweep: the C1/C2/C4 attention and append grid, one JSON line per "
                         "configuration (not the one-line bench contract)")
    a = ap.parse_args()
    # BASELINE config 1 (C1) and config 4 (C4); C3 keeps its own defaults
    defaults = {"c4": dict(batch=8, ctx=131072, layers=80, hq=64, kbits=2, vbits=2)}.get(
        a.workload, dict(batch=32, ctx=32768, layers=32, hq=32, kbits=4, vbits=4))
    for k_, v_ in defaults.items():
        if getattr(a, k_) is None:
            setattr(a, k_, v_)
    return a


def metric_name(a):
    """The C1 line keeps BASELINE's metric name; other workloads say their shape."""
    if a.workload == "c4":
        return f"decode attn HBM GB/s ({a.kbits}/{a.vbits}-bit QK^T+AV, 70B attention shape)"
    if (a.kbits, a.vbits) != (4, 4):
        return f"decode attn HBM GB/s ({a.kbits}/{a.vbits}-bit QK^T+AV, Llama-3-8B attention shape)"
    return METRIC


def cache_kw(a):
    vtok = getattr(a, "v_layout", "tokens") == "tokens"
    mode = getattr(a, "mode", "symmetric")
    return dict(k_bits=a.kbits, v_bits=a.vbits, key_group_size=a.group, value_group_size=a.group,
                key_flush_size=1, value_flush_size=max(32, a.group) if vtok else 32,
                key_w_sink=32, value_w_sink=32, key_w_recent=96, value_w_recent=96,
                key_normalize=True, key_quantize_over_token=False, value_quantize_over_token=vtok,
                key_quantize_mode=mode, value_quantize_mode=mode)


def side_bytes(n_q, n_sink, n_recent, bits, group, over_token, asym=False, norm=False):
    """Algorithmic bytes one (b, kv-head) reads for one side."""
    z = 2 if asym else 1
    if over_token:
        b = n_q * bits * D // 8 + (n_q // group) * D * 2 * z
    else:
        b = n_q * (bits * D // 8 + (D // group) * 2 * z)
    b += (n_sink + n_recent) * D * 2
    if norm:
        b += D * 2
    return b


def layer_bytes(layer, B, Hkv, Hq, graph_steps=None):
    """Algorithmic bytes one attention launch reads and writes; graph_steps:
    the layer is in graph mode, that many steps after its step-0 state."""
    k, v = layer.key_side, layer.value_side
    (knq, knr), (vnq, vnr) = ((k.n_q, k.n_recent), (v.n_q, v.n_recent)) if graph_steps is None else \
        (k.state_after(graph_steps), v.state_after(graph_steps))
    per_bh = side_bytes(knq, k.n_sink, knr, k.bits, k.group, k.over_token, k.mode == 1, k.normalize) \
        + side_bytes(vnq, v.n_sink, vnr, v.bits, v.group, v.over_token, v.mode == 1)
    if getattr(v, "zp", None) is not None and v.over_token:
        # hybrid values: the asymmetric (bits-1)-bit set, its scales and zeros, the mask
        per_bh += vnq * (v.bits - 1) * D // 8 + (vnq // v.group) * (D * 2 * 2 + 16)
    return B * Hkv * per_bh + 2 * B * Hq * D * 2


# --------------------------------------------------------------- clocks ---
class NvmlClockSampler:
    """SM clock and clock-event reasons of one GPU read through NVML, in a
    burst taken while the GPU executes the timed region: the host enqueues
    every step of the region first and samples afterwards, so no launch waits
    behind an NVML call (polling during the launches, from nvidia-smi or from
    a thread, delayed the ranks' launches by milliseconds per sample on
    multi-GPU boxes)."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, torch_device, enabled=True):
        self.dev = torch_device
        self.enabled = enabled
        self.samples = []
        self.h = None

    def _handle(self, N):
        import torch
        try:
            uuid = str(torch.cuda.get_device_properties(self.dev).uuid)
            return N.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:
            return N.nvmlDeviceGetHandleByIndex(self.dev.index or 0)

    def start(self):
        """Before the region: open NVML (nothing is sampled yet)."""
        if not self.enabled:
            return
        import pynvml as N
        N.nvmlInit()
        self.N = N
        self.h = self._handle(N)
        self.max_mhz = float(N.nvmlDeviceGetMaxClockInfo(self.h, N.NVML_CLOCK_SM))

    def burst(self, region_ms_estimate, n=5):
        """After the region's launches are enqueued: n samples spread over
        20-60% of the region's expected duration."""
        if self.h is None:
            return
        N = self.N
        # let the other ranks finish enqueueing their steps first
        time.sleep(0.2 * region_ms_estimate / 1000.0)
        gap = max(0.5, 0.4 * region_ms_estimate / n) / 1000.0
        for _ in range(n):
            sm = float(N.nvmlDeviceGetClockInfo(self.h, N.NVML_CLOCK_SM))
            r = N.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            self.samples.append((sm, [name for name, attr in self.REASONS if r & getattr(N, attr)]))
            time.sleep(gap)

    def stop(self):
        if not self.samples:
            return None
        reasons = sorted({n for _, rs in self.samples for n in rs})
        return {"sm_mhz": statistics.median([s for s, _ in self.samples]), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples),
                "source": "NVML, sampled while the GPU ran the enqueued timed region"}


def clock_sampler(torch_device, local, period_ms=20, enabled=True):
    """NVML bursts when pynvml is importable, else nvidia-smi polling."""
    try:
        import pynvml  # noqa: F401
        return NvmlClockSampler(torch_device, enabled)
    except ImportError:
        return ClockSampler(local, period_ms, enabled)


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index, period_ms=20, enabled=True):
        self.gpu = gpu_index
        self.period = period_ms
        self.enabled = enabled
        self.proc = None
        self.f = None
        self.skip = 0

    def start(self):
        """Start sampling every `period_ms` and return once the first sample is
        in, so that a short timed region that follows is covered."""
        if not self.enabled:
            return
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", str(self.period)],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return
        t_end = time.time() + 5.0
        while time.time() < t_end and os.path.getsize(self.f.name) == 0 and self.proc.poll() is None:
            time.sleep(0.01)
        self.skip = sum(1 for _ in open(self.f.name))  # samples taken before the region

    def burst(self, region_ms_estimate, n=5):
        """Polling runs on its own; nothing to do after the enqueue."""

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        # samples inside the timed region; the last one before it (taken under
        # the same load, just after warm-up) when the region was shorter than
        # the sampling period
        inside = rows[self.skip:] if len(rows) > self.skip else rows[-1:]
        rows = inside
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [x.strip() for x in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
            except ValueError:
                continue
            for n, val in zip(names, r[5:9]):
                if val.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------- CPU reference ---
def cpu_reference_sample(a, seconds=None, steps=None, warmup=0, budget_s=150.0):
    """The reference's decode step on the host cores: the torch restatement of
    cache.py's update (append, flush, quantize, cat, dequantize the whole
    store in fp32, cast) and the Hugging Face sdpa consumer, torch running on
    every host core (torch.set_num_threads(os.cpu_count())).  Sample = one
    layer of the benchmark's configuration; the batch is the benchmark's
    unless host memory or the time budget (`budget_s` for warm-up + timed
    steps, estimated from a batch-1 probe) needs a smaller one, in which case
    the sample says so.  Returns (GB/s of the same algorithmic bytes as the
    GPU metric, threads, sample description, seconds per step)."""
    import torch

    from oracle.torch_ref import TorchRefLayer, consumer_attention
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    kw = cache_kw(a)
    S = a.ctx
    gen = torch.Generator().manual_seed(0)

    def make(b):
        layer = TorchRefLayer(**kw)
        k = torch.randn((b, a.hkv, S - 1, D), generator=gen)
        k *= torch.exp(torch.randn(D, generator=gen))
        v = torch.randn((b, a.hkv, S - 1, D), generator=gen)
        layer.update(k.half(), v.half())
        del k, v
        q = torch.randn((b, a.hq, 1, D), generator=gen).half()
        new = torch.randn((b, a.hkv, 1, D), generator=gen).half()
        return layer, q, new

    def step(layer, q, new):
        K, V = layer.update(new, new)
        return consumer_attention(q, K, V)

    # batch-1 probe: per-step time scales with the batch
    layer, q, new = make(1)
    step(layer, q, new)
    t0 = time.perf_counter()
    step(layer, q, new)
    t1 = time.perf_counter() - t0
    del layer
    n_steps = (steps if steps is not None else 2) + warmup
    # host bytes per (batch row): fp16 inputs, int32 codes, fp16 signs, fp32
    # dequantization, the cast and the repeated KV heads, K and V
    per_row = a.hkv * S * D * (2 + 4 + 2 + 4 + 4 + 2 * (a.hq // a.hkv)) * 2
    try:
        import psutil
        avail = psutil.virtual_memory().available
    except ImportError:
        avail = 16 << 30
    B = a.batch
    while B > 1 and (per_row * B > 0.4 * avail or t1 * B * n_steps > budget_s):
        B //= 2
    layer, q, new = make(B)
    for _ in range(warmup):
        step(layer, q, new)
    times = []
    t_end = time.perf_counter() + (seconds or 1e9)
    n = 0
    while True:
        t0 = time.perf_counter()
        step(layer, q, new)
        times.append(time.perf_counter() - t0)
        n += 1
        if (steps is not None and n >= steps) or (steps is None and time.perf_counter() > t_end):
            break
    k0, v0 = layer.k, layer.v
    per_bh = side_bytes(k0.codes.shape[2], k0.sink.shape[2], k0.recent.shape[2], a.kbits, a.group,
                        False, kw["key_quantize_mode"] == "asymmetric", norm=True) \
        + side_bytes(v0.codes.shape[2], v0.sink.shape[2], v0.recent.shape[2], a.vbits, a.group,
                     kw["value_quantize_over_token"], kw["value_quantize_mode"] == "asymmetric")
    nbytes = B * a.hkv * per_bh + 2 * B * a.hq * D * 2
    t = statistics.median(times)
    why = "" if B == a.batch else f" (batch {a.batch} reduced to fit host memory / the time budget)"
    sample = (f"torch restatement of the reference decode step (cache.py update + sdpa consumer), "
              f"1 layer, batch {B}{why}, {a.hkv} kv heads x {a.hq // a.hkv} q heads, context {S}, "
              f"{len(times)} steps; torch on {cores} threads")
    return nbytes / t / 1e9, cores, sample, t


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    gbs, cores, sample, t = cpu_reference_sample(a, steps=a.steps, warmup=a.warmup)
    line = {
        "impl": "reference", "metric": metric_name(a), "value": round(gbs, 4), "unit": "GB/s",
        "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(t * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp16",
        "data": "synthetic",
        "config": {"workload": (f"C4: 70B attention shape, {a.kbits}/{a.vbits}-bit InnerQ cache, "
                                "decode step" if a.workload == "c4" else
                                f"C1: Llama-3-8B attention shape, {a.kbits}/{a.vbits}-bit InnerQ "
                                "cache, decode step"),
                   "batch": a.batch, "context": a.ctx, "layers": a.layers, "q_heads": a.hq,
                   "kv_heads": a.hkv, "reference_sample": sample},
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------- ours ---
def run_ours(a):
    import torch
    import torch.distributed as dist

    from innerq_b200 import _lib
    from innerq_b200.cache import InnerqDynamicLayer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    from innerq_b200.sharding import ContextMerge, HeadGather, head_shard
    from innerq_b200.attention import build_args, plan
    CS = a.ctx_shards
    if CS < 1 or world % CS:
        raise SystemExit(f"--ctx-shards {CS} does not divide {world} ranks")
    HS = world // CS
    hs, cs = divmod(rank, CS)     # this rank: KV-head shard hs, context chunk cs
    last = cs == CS - 1           # the chunk that holds the recent window and takes the appends
    h_lo, h_hi = head_shard(a.hkv, HS, hs)
    hkv, hq = h_hi - h_lo, (h_hi - h_lo) * (a.hq // a.hkv)
    # weak scaling: the global batch grows with the head shards, so each rank
    # holds as many (sequence, KV head) pairs as the one-GPU workload
    B_global = a.batch * (HS if a.scaling == "weak" else 1)
    B, L = B_global, a.layers
    kw = cache_kw(a)
    ctx_group = None
    if CS > 1:
        for i in range(HS):  # every rank takes part in creating every group
            grp = dist.new_group(list(range(i * CS, (i + 1) * CS)))
            if i == hs:
                ctx_group = grp
        # chunk cs of the T = ctx-1 prefill tokens: the sink on chunk 0, the
        # recent window on the last chunk, the packed part of every chunk a
        # whole number of value groups
        T, G = a.ctx - 1, max(32, a.group)
        ns = kw["key_w_sink"]
        cuts = [0] + [ns + ((T - ns) * c // CS) // G * G for c in range(1, CS)] + [T]
        t_lo, t_hi = cuts[cs], cuts[cs + 1]
        if cs > 0:
            kw.update(key_w_sink=0, value_w_sink=0)
        if not last:
            kw.update(key_w_recent=0, value_w_recent=0)
    else:
        t_lo, t_hi = 0, a.ctx - 1
    conf = types.SimpleNamespace(_attn_implementation="innerq", **kw)

    # ---- build the resident cache: prefill this rank's tokens per layer
    layers = []
    g = torch.Generator(device=dev)
    for li in range(L):
        g.manual_seed(1000 * li + rank)
        k = torch.randn((B, hkv, t_hi - t_lo, D), device=dev, generator=g)
        k *= torch.exp(torch.randn(D, device=dev, generator=g))
        k = k.half()
        v = torch.randn((B, hkv, t_hi - t_lo, D), device=dev, generator=g).half()
        layer = InnerqDynamicLayer(conf, li)
        layer.update(k, v)
        del k, v
        layers.append(layer)
    torch.cuda.synchronize()

    NPOOL = 8
    g.manual_seed(7 + rank)
    qs = torch.randn((NPOOL, L, B, hq, 1, D), device=dev, generator=g).half()
    ks = torch.randn((NPOOL, L, B, hkv, 1, D), device=dev, generator=g).half()
    vs = torch.randn((NPOOL, L, B, hkv, 1, D), device=dev, generator=g).half()
    out = torch.empty((L, B, hq, D), device=dev, dtype=torch.float16)
    # the one collective per step: the KV-head shards' outputs gathered into a
    # buffer allocated here, once
    head_group = None
    if HS > 1 and CS > 1:
        for j in range(CS):
            grp = dist.new_group(list(range(j, world, CS)))
            if j == cs:
                head_group = grp
    gather = HeadGather(out, head_group) if (HS > 1 and a.scaling == "strong") else None
    merges = None
    if CS > 1:
        # the same split count on every rank of a chunk group (the largest any
        # rank's planner picks), so the gathered partials blocks line up
        ns_loc = plan(build_args(qs[0][0], layers[0].key_side, layers[0].value_side))[1]
        t_ = torch.tensor([ns_loc], device=dev)
        dist.all_reduce(t_, op=dist.ReduceOp.MAX)
        n_splits_ctx = int(t_.item())
        merges = [ContextMerge(B, hq, n_splits_ctx, dev, ctx_group) for _ in range(L)]

    def attend(li, layer, q):
        if merges is None:
            layer.attend(q, out=out[li])
        else:  # this chunk's partials, one all-gather in the chunk group, one merge
            mg = merges[li]
            layer.attend_partials(q, mg.po, mg.pm, mg.pl)
            mg(out[li])

    def step(i, q=None, k=None, v=None):
        q = qs[i % NPOOL] if q is None else q
        k = ks[i % NPOOL] if k is None else k
        v = vs[i % NPOOL] if v is None else v
        for li, layer in enumerate(layers):
            if last:
                layer.update(k[li], v[li])
            attend(li, layer, q[li])
        if gather is not None:
            gather()  # [L, B, Hq, D] across the KV-head shards

    gsteps = [None]  # graph-mode steps replayed so far (None: eager)

    def bytes_now():
        # the step about to run: appends one token (last chunk), then attends
        n = None if (gsteps[0] is None or not last) else gsteps[0] + 1
        return sum(layer_bytes(l, B, hkv, hq, n) for l in layers)

    def sync_all():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    def sum_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return t.item()

    for i in range(max(3, a.warmup)):
        step(i)
    stream = torch.cuda.current_stream()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    # ---- kernel roofline: attention launches alone (query prep + attention +
    #      merge), eager, before the cache enters graph mode
    sync_all()
    ev0.record(stream)
    reps = 3
    for r in range(reps):
        for li, layer in enumerate(layers):
            if merges is None:
                layer.attend(qs[0][li], out=out[li])
            else:
                layer.attend_partials(qs[0][li], merges[li].po, merges[li].pm, merges[li].pl)
    ev1.record(stream)
    torch.cuda.synchronize()
    per_launch_ms = ev0.elapsed_time(ev1) / (reps * L)
    per_launch_bytes = sum(layer_bytes(l, B, hkv, hq) for l in layers) / L
    achieved = per_launch_bytes / (per_launch_ms * 1e-3) / 1e9

    # ---- launch mode: the decode step launched from the host each step
    #      (eager), or recorded once in a CUDA graph (cache graph mode: the
    #      per-step state comes from a device counter) and replayed.  A few
    #      timed steps of each decide (max over ranks, same choice on every
    #      rank): replay wins where host time per layer exceeds device time
    #      (small batches, many GPUs), eager where the device is the bound.
    graph = None
    per_step_launches = None
    q_in, k_in, v_in = torch.empty_like(qs[0]), torch.empty_like(ks[0]), torch.empty_like(vs[0])
    trial = 3

    def time_steps(fn, i0):
        sync_all()
        ev0.record(stream)
        for i in range(trial):
            fn(i0 + i)
        ev1.record(stream)
        sync_all()
        return max_over_ranks(ev0.elapsed_time(ev1)) / trial

    mode_ms = {"eager": time_steps(step, max(3, a.warmup))}
    eager_step = step
    if not a.no_graph:
        gstep = torch.zeros(1, dtype=torch.int64, device=dev)
        for layer in layers if last else ():  # the other chunks do not change
            layer.graph_begin(gstep, 2 * max(3, a.warmup) + 2 * a.steps + 2 * trial + 4)
        n0 = _lib.launch_count[0]
        cs = torch.cuda.Stream(dev)
        cs.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(cs):
            with torch.cuda.graph(graph, stream=cs):
                gstep.add_(1)
                for li, layer in enumerate(layers):
                    if last:
                        layer.update(k_in[li], v_in[li])
                    attend(li, layer, q_in[li])
        torch.cuda.current_stream().wait_stream(cs)
        per_step_launches = _lib.launch_count[0] - n0
        gsteps[0] = 0

        def graph_step(i, q=None, k=None, v=None):
            q_in.copy_(qs[i % NPOOL] if q is None else q)
            k_in.copy_(ks[i % NPOOL] if k is None else k)
            v_in.copy_(vs[i % NPOOL] if v is None else v)
            graph.replay()
            gsteps[0] += 1
            if gather is not None:
                gather()  # the one collective per step stays outside the recording

        for i in range(max(3, a.warmup)):
            graph_step(i)
        mode_ms["graph"] = time_steps(graph_step, 0)
        if mode_ms["graph"] < mode_ms["eager"]:
            step = graph_step
        else:  # leave graph mode: the host takes the state back
            torch.cuda.synchronize()
            for layer in layers if last else ():
                layer.graph_end(gsteps[0])
            graph, gsteps[0], per_step_launches = None, None, None
            step = eager_step

    # ---- device-resident timed region (rank 0 samples its GPU's clocks)
    sampler = clock_sampler(dev, local, period_ms=20, enabled=rank == 0 and
                            os.environ.get("INNERQ_BENCH_CLOCKS", "1") != "0")
    nbytes = 0
    sync_all()
    sampler.start()
    launches0 = _lib.launch_count[0]
    torch.cuda.nvtx.range_push("timed")  # profiling handle (ncu --nvtx-include timed/)
    ev0.record(stream)
    for i in range(a.steps):
        nbytes += bytes_now()
        step(i)
    ev1.record(stream)
    torch.cuda.nvtx.range_pop()
    # the region is enqueued: sample the clocks while the GPU runs it
    sampler.burst(a.steps * min(mode_ms.values()))
    sync_all()
    clocks = sampler.stop()
    launches = _lib.launch_count[0] - launches0 if graph is None else per_step_launches * a.steps
    ms = max_over_ranks(ev0.elapsed_time(ev1)) / a.steps
    total_bytes = sum_over_ranks(nbytes / a.steps)
    value = total_bytes / (ms * 1e-3) / 1e9

    # ---- the per-step all-gather alone (its share of the step)
    gather_ms = None
    if gather is not None:
        sync_all()
        ev0.record(stream)
        for i in range(a.steps):
            gather()
        ev1.record(stream)
        sync_all()
        gather_ms = max_over_ranks(ev0.elapsed_time(ev1)) / a.steps

    # ---- end to end through the public API with host buffers
    qh = qs[0].cpu().pin_memory()
    kh = ks[0].cpu().pin_memory()
    vh = vs[0].cpu().pin_memory()
    outh = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    qd, kd, vd = torch.empty_like(qs[0]), torch.empty_like(ks[0]), torch.empty_like(vs[0])
    sync_all()
    e2e_bytes = 0
    ev0.record(stream)
    for i in range(a.steps):
        e2e_bytes += bytes_now()
        qd.copy_(qh, non_blocking=True)
        kd.copy_(kh, non_blocking=True)
        vd.copy_(vh, non_blocking=True)
        step(i, qd, kd, vd)
        outh.copy_(out, non_blocking=True)
    ev1.record(stream)
    sync_all()
    e2e_ms = max_over_ranks(ev0.elapsed_time(ev1)) / a.steps
    e2e_value = sum_over_ranks(e2e_bytes / a.steps) / (e2e_ms * 1e-3) / 1e9
    h2d = (qh.numel() + kh.numel() + vh.numel()) * 2 * world
    d2h = outh.numel() * 2 * world

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        gbs, cores, sample, _ = cpu_reference_sample(a, seconds=a.cpu_seconds, warmup=1)
        cpu = {"value": round(gbs, 4), "unit": "GB/s", "cores": cores, "kind": "port",
               "sample": sample}

    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    traffic = None
    try:
        # DRAM bytes per algorithmic byte from an ncu capture of the same
        # kernel configuration (keyed by workload), scaled to this launch
        tr = json.load(open(os.path.join(ROOT, "profiles", "decode_attn_traffic.json")))
        key = a.workload if (a.kbits, a.vbits, a.v_layout, a.mode) == (
            (2, 2) if a.workload == "c4" else (4, 4)) + ("tokens", "symmetric") else None
        ratio = tr.get("by_workload", {}).get(key) if key else None
        if ratio is None and key == "c1":
            ratio = tr["dram_bytes_per_algorithmic_byte"]
        traffic = None if ratio is None else round(ratio * per_launch_bytes)
    except (OSError, KeyError, ValueError):
        pass

    if rank == 0:
        line = {
            "metric": metric_name(a), "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": a.steps, "warmup": max(3, a.warmup), "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": a.scaling, "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic (seeded N(0,1) K with exp(N(0,1)) channel outliers, N(0,1) V and q)",
            "config": {
                "workload": ("C4: decode step over an 80-layer 70B-shaped (64 q / 8 kv heads) "
                             f"{a.kbits}/{a.vbits}-bit InnerQ cache" if a.workload == "c4" else
                             "C1: decode step over a 32-layer Llama-3-8B-shaped "
                             f"{a.kbits}/{a.vbits}-bit InnerQ cache"),
                "batch": B, "context": a.ctx, "layers": L, "q_heads": a.hq, "kv_heads": a.hkv,
                "head_dim": D, "k_bits": a.kbits, "v_bits": a.vbits, "group": a.group,
                "v_groups_over": a.v_layout, "mode": a.mode,
                "parallelism": (f"kv-head shards x{HS}" + (f", context chunks x{CS} (split partials "
                                "all-gathered and merged per layer)" if CS > 1 else "")
                                + (f"; weak scaling: global batch {B} = {a.batch} x {HS} head shards, "
                                   f"{B * hkv} (sequence, KV head) pairs per GPU"
                                   if a.scaling == "weak" and HS > 1 else "")
                                + ("; KV-head outputs all-gathered once per step"
                                   if gather is not None else "")),
                "step": "eager launches" if graph is None else "recorded once (CUDA graph), replayed",
                "step_trial_ms": {k_: round(v_, 3) for k_, v_ in mode_ms.items()},
                "l2": f"inputs larger than L2 ({total_bytes / 1e9:.1f} GB of cache read per step)",
                "us_per_layer": round(ms * 1e3 / L, 2),
                "allgather_ms_per_step": None if gather_ms is None else round(gather_ms, 4),
                "allgather_share": None if gather_ms is None else round(gather_ms / ms, 4),
            },
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": traffic,
                         "kernel": "decode_attn_kernel (+ lse_merge)",
                         "per_launch_bytes": int(per_launch_bytes),
                         "per_launch_us": round(per_launch_ms * 1e3, 2),
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)",
                         "frac_of_nominal": round(achieved / NOMINAL_HBM_GBS, 4),
                         "value_frac_of_measured": round(value / world / peak, 4),
                         "value_frac_of_nominal": round(value / world / NOMINAL_HBM_GBS, 4)},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4)},
            "gpu_launches": launches,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    # release the recorded step (it holds NCCL work in the context-chunk mode)
    # and the communicator buffers before the process group goes
    graph = gather = merges = None
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_c3(a):
    """full decode step of a random-init Llama-3-8B-shaped
    model (32 layers, hidden 4096, 32 q / 8 kv heads, head_dim 128, vocab
    128256, bf16 weights N(0, 0.02)) with a 4-bit InnerQ cache, batch 16,
    context 8192, token ids uniform over the vocabulary; reports tokens/s.
    The cache is pre-filled synthetically (per-layer random K/V through the
    cache's own prefill path) instead of running a prompt through the model."""
    import torch
    from transformers import LlamaConfig

    from innerq_b200 import _lib
    from innerq_b200.cache import DynamicCache
    from innerq_b200.models import InnerqLlamaForCausalLM

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, S = a.batch if a.batch != 32 else 16, a.ctx if a.ctx != 32768 else 8192
    qcfg = cache_kw(a)
    cfg = LlamaConfig(num_hidden_layers=32, hidden_size=4096, intermediate_size=14336,
                      num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                      vocab_size=128256, max_position_embeddings=S + 1024, rope_theta=500000.0,
                      torch_dtype=torch.bfloat16, **qcfg)
    torch.manual_seed(0)
    with torch.device(dev):
        model = InnerqLlamaForCausalLM(cfg).to(torch.bfloat16)
    with torch.no_grad():
        for p in model.parameters():
            p.normal_(0.0, 0.02)
    model.eval()
    cache = DynamicCache(config=model.config.get_text_config(decoder=True))
    g = torch.Generator(device=dev).manual_seed(1)
    for layer in cache.layers:
        k = (torch.randn((B, 8, S - 1, 128), device=dev, generator=g)
             * torch.exp(torch.randn(128, device=dev, generator=g))).bfloat16()
        v = torch.randn((B, 8, S - 1, 128), device=dev, generator=g).bfloat16()
        layer.update(k, v)
        del k, v
    ids = torch.randint(0, cfg.vocab_size, (a.steps + 2 * max(3, a.warmup) + 8, B, 1), device=dev,
                        generator=g)
    pos0 = S - 1

    def step(i):
        pos = torch.full((B, 1), pos0 + i, device=dev, dtype=torch.long)
        out = model(input_ids=ids[i], past_key_values=cache, position_ids=pos, use_cache=True)
        return out.logits

    with torch.no_grad():
        for i in range(max(3, a.warmup)):
            step(i)
        torch.cuda.synchronize()
        per_step_launches = None
        if not a.no_graph:
            # record one decode step of the whole model (cache in graph mode) and
            # replay it: token ids and positions go into the recorded step's inputs
            ids_in = torch.empty((B, 1), dtype=torch.long, device=dev)
            pos_in = torch.empty((B, 1), dtype=torch.long, device=dev)
            cache.graph_begin(2 * max(3, a.warmup) + a.steps + 4)
            n0 = _lib.launch_count[0]
            cs = torch.cuda.Stream(dev)
            cs.wait_stream(torch.cuda.current_stream())
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(cs):
                with torch.cuda.graph(graph, stream=cs):
                    cache.graph_advance()
                    logits_out = model(input_ids=ids_in, past_key_values=cache, position_ids=pos_in,
                                       use_cache=True).logits
            torch.cuda.current_stream().wait_stream(cs)
            per_step_launches = _lib.launch_count[0] - n0

            def step(i):  # noqa: F811 - the recorded step
                ids_in.copy_(ids[i])
                pos_in.fill_(pos0 + i)
                graph.replay()
                return logits_out

            for i in range(max(3, a.warmup)):
                step(max(3, a.warmup) + i)
            torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        sampler = clock_sampler(dev, 0)
        sampler.start()
        n0 = _lib.launch_count[0]
        i0 = max(3, a.warmup) * (1 if per_step_launches is None else 2)
        e0.record()
        for i in range(a.steps):
            step(i0 + i)
        e1.record()
        sampler.burst(a.steps * 7.0)  # ~7-8 ms per replayed step
        torch.cuda.synchronize()
        clocks = sampler.stop()
        ours = _lib.launch_count[0] - n0 if per_step_launches is None else per_step_launches * a.steps
    ms = e0.elapsed_time(e1) / a.steps
    cpu = None
    if not a.no_cpu_baseline:
        del model, cache
        torch.cuda.empty_cache()
        cpu = c3_cpu_baseline(a, B, S, qcfg)
    line = {
        "metric": "decode tokens/s (Llama-3-8B-shaped, 4-bit InnerQ cache)", "value": round(B / (ms * 1e-3), 1),
        "unit": "tokens/s", "n_gpus": 1, "steps": a.steps, "warmup": max(3, a.warmup),
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (random-init weights N(0,0.02), uniform token ids, synthetic cache)",
        "config": {"workload": "C3: full decode step, random-init Llama-3-8B shape", "batch": B,
                   "context": S, "layers": 32, "k_bits": a.kbits, "v_bits": a.vbits,
                   "step": "eager" if a.no_graph else "recorded once (CUDA graph), replayed"},
        "gpu_launches": ours, "clocks": clocks, "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


def c3_cpu_baseline(a, B, S, qcfg, steps=2):
    """C3 on the host cores: the same random-init model shape decoding through
    the reference's cache restated in torch (oracle/torch_ref.py, dequantize
    of the whole cache every layer) and Hugging Face sdpa, torch on every
    core.  A 32-layer step does not fit the time budget, so 1- and 2-layer
    models are timed and the step is extrapolated: t(32) = t(1) + 31 (t(2) - t(1))."""
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM

    from oracle.torch_ref import ref_cache
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    g = torch.Generator().manual_seed(1)
    t = {}
    for L in (1, 2):
        cfg = LlamaConfig(num_hidden_layers=L, hidden_size=4096, intermediate_size=14336,
                          num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                          vocab_size=128256, max_position_embeddings=S + 1024, rope_theta=500000.0)
        torch.manual_seed(0)
        model = LlamaForCausalLM(cfg).to(torch.bfloat16).eval()
        with torch.no_grad():
            for p in model.parameters():
                p.normal_(0.0, 0.02)
        cache = ref_cache(L, **qcfg)
        for layer in cache.layers:
            k = (torch.randn((B, 8, S - 1, 128), generator=g)
                 * torch.exp(torch.randn(128, generator=g))).bfloat16()
            v = torch.randn((B, 8, S - 1, 128), generator=g).bfloat16()
            layer.update(k, v)
            del k, v
        ids = torch.randint(0, cfg.vocab_size, (steps + 1, B, 1), generator=g)
        times = []
        with torch.no_grad():
            for i in range(steps + 1):
                pos = torch.full((B, 1), S - 1 + i, dtype=torch.long)
                t0 = time.perf_counter()
                model(input_ids=ids[i], past_key_values=cache, position_ids=pos, use_cache=True)
                if i:  # the first step warms up
                    times.append(time.perf_counter() - t0)
        t[L] = statistics.median(times)
        del model, cache
    t32 = t[1] + 31 * (t[2] - t[1])
    return {"value": round(B / t32, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": (f"random-init Llama-3-8B-shaped model, batch {B}, context {S}, bf16, the "
                       "reference cache restated in torch (oracle/torch_ref.py) + HF sdpa; 1- and "
                       f"2-layer models timed ({t[1]:.2f} s, {t[2]:.2f} s per step, {steps} steps "
                       f"each), 32-layer step extrapolated as t1 + 31 (t2 - t1); torch on {cores} threads")}


SWEEP = [
    # (name, B, Hq, context, bits, group, v_layout, mode)
    ("C1", 1, 32, 32768, 4, 32, "tokens", "symmetric"),
    ("C1", 8, 32, 32768, 4, 32, "tokens", "symmetric"),
    ("C1", 32, 32, 32768, 4, 32, "tokens", "symmetric"),
    ("C1 BASELINE-literal", 32, 32, 32768, 4, 32, "channels", "symmetric"),
    ("C1 asym", 32, 32, 32768, 4, 32, "tokens", "asymmetric"),
] + [("C2", 16, 32, ctx, bits, g, "tokens", "symmetric")
     for bits in (2, 3) for ctx in (4096, 16384, 65536) for g in (32, 64, 128)] + [
    ("C2 BASELINE-literal", 16, 32, 16384, 2, 32, "channels", "symmetric"),
    ("C2 BASELINE-literal", 16, 32, 16384, 3, 32, "channels", "symmetric"),
    ("C2 asym", 16, 32, 16384, 2, 32, "tokens", "asymmetric"),
    ("C4 (1 GPU, 4 layers)", 8, 64, 131072, 2, 32, "tokens", "symmetric"),
    # the innerq_hybrid preset (scripts/run_lmeval.sh:133-151): 3-bit K, 2-bit hybrid V
    ("C1 innerq_hybrid", 32, 32, 32768, (3, 2), 32, "tokens", "hybrid"),
    # the kivi preset (scripts/run_lmeval.sh:54-72): 2-bit asymmetric keys
    # grouped over tokens, 2-bit asymmetric values grouped over channels
    ("C1 kivi", 32, 32, 32768, 2, 32, "channels", "kivi"),
]


def run_sweep(a):
    """Fused decode attention (query prep + attention + merge, replayed from a
    CUDA graph so batch-1 launches are not host bound) and the append kernels
    over the BASELINE configurations; one JSON line per configuration.
    Several independent layer caches rotate so each launch reads HBM, not L2."""
    import torch

    from innerq_b200.attention import decode_attention
    from innerq_b200.cache import InnerqDynamicLayer
    from innerq_b200.store import PackedSide
    from innerq_b200 import _lib

    dev = torch.device("cuda", 0)
    peak = float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))).get("hbm_gbs", 6650.0)) \
        if os.path.exists(os.path.join(ROOT, "MEASURED_PEAKS.json")) else 6650.0
    done = set()
    for name, B, hq, ctx, bits, group, vlay, mode in SWEEP:
        if a.only is not None and (name != a.only[1:] if a.only.startswith("=") else a.only not in name):
            continue
        ctx = a.sweep_ctx or ctx
        B = a.sweep_batch or B
        key = (name, B, hq, ctx, bits, group, vlay, mode)
        if key in done:
            continue
        done.add(key)
        kb_, vb_ = bits if isinstance(bits, tuple) else (bits, bits)
        a2 = types.SimpleNamespace(kbits=kb_, vbits=vb_, group=group, v_layout=vlay,
                                   mode="symmetric" if mode in ("hybrid", "kivi") else mode)
        kw = cache_kw(a2)
        if mode == "hybrid":
            kw["value_quantize_mode"] = "hybrid"
        if mode == "kivi":
            kw.update(key_quantize_over_token=True, value_quantize_over_token=False,
                      key_quantize_mode="asymmetric", value_quantize_mode="asymmetric",
                      key_flush_size=32, value_flush_size=1, key_w_sink=0, value_w_sink=0,
                      key_w_recent=128, value_w_recent=128, key_normalize=False)
        bits = kb_
        hkv = a.sweep_hkv or 8
        hq = hq * hkv // 8
        per_layer = B * hkv * ctx * ((kb_ + vb_) * 16 + 16)
        nl = max(4, min(8, int(1.2e9 // per_layer) + 1))
        g = torch.Generator(device=dev)
        g.manual_seed(0)
        layers = []
        for _ in range(nl):
            layer = InnerqDynamicLayer(types.SimpleNamespace(**kw), 0)
            k = torch.randn((B, hkv, ctx, D), device=dev, generator=g)
            k *= torch.exp(torch.randn(D, device=dev, generator=g))
            k = k.half()
            v = torch.randn((B, hkv, ctx, D), device=dev, generator=g).half()
            layer.update(k, v)
            del k, v
            layers.append(layer)
        q = torch.randn((B, hq, 1, D), device=dev, generator=g).half()
        outs = [torch.empty((B, hq, D), dtype=q.dtype, device=dev) for _ in layers]
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        nb = layer_bytes(layers[0], B, hkv, hq)

        def time_attn(n_splits):
            for l, o in zip(layers, outs):
                decode_attention(q, l.key_side, l.value_side, out=o, n_splits=n_splits)
            torch.cuda.synchronize()
            reps = 4
            st = torch.cuda.Stream(dev)
            with torch.cuda.stream(st):
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=st):
                    for _ in range(reps):
                        for l, o in zip(layers, outs):
                            decode_attention(q, l.key_side, l.value_side, out=o, n_splits=n_splits)
            torch.cuda.synchronize()
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize()
            e0.record()
            for _ in range(5):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            return e0.elapsed_time(e1) * 1e3 / (5 * reps * nl)

        if a.split_scan:
            from innerq_b200.attention import build_args, plan
            for ns in [int(x) for x in a.split_scan.split(",")]:
                eff = plan(build_args(q, layers[0].key_side, layers[0].value_side, n_splits=ns))[1]
                us = time_attn(ns)
                print(json.dumps({"config": name, "batch": B, "q_heads": hq, "kv_heads": hkv,
                                  "context": ctx, "bits": bits, "n_splits": ns, "splits_used": eff,
                                  "attn_us": round(us, 2), "attn_GBs": round(nb / us / 1e3, 1)}),
                      flush=True)
            del layers, outs
            torch.cuda.empty_cache()
            continue
        us = time_attn(0)
        del layers, outs
        torch.cuda.empty_cache()
        # append: one K token (channel groups) and one 4096-token chunk
        side = PackedSide(_lib.ROLE_K, bits, group, _lib.SYM if mode == "symmetric" else _lib.ASYM,
                          False, 0, 0, 1)
        # two chunks used in turn: together larger than L2
        xs = [torch.randn((B, hkv, 4096, D), device=dev, generator=g).half() for _ in range(2)]
        x = xs[0]
        n_rep = 8
        side.prefill(x[:, :, :1])
        side.reserve(4096 * (n_rep + 2))
        torch.cuda.synchronize()
        e0.record()
        for i in range(20):
            side._quantize(x[:, :, i:i + 1])
        e1.record()
        torch.cuda.synchronize()
        us_tok = e0.elapsed_time(e1) * 1e3 / 20
        # chunk launches back to back (the host runs ahead of the GPU, so
        # launch overhead is not timed); mean per chunk
        side.n_q = 0
        side._quantize(xs[1])
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("chunk")  # profiling handle (ncu --nvtx-include chunk/)
        e0.record()
        for i in range(n_rep):
            side._quantize(xs[i % 2])
        e1.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        us_chunk = e0.elapsed_time(e1) * 1e3 / n_rep
        # keys with the normalisation factor (innerq_base), set by the first chunk
        nside = PackedSide(_lib.ROLE_K, bits, group, _lib.SYM if mode == "symmetric" else _lib.ASYM,
                           False, 0, 0, 1, normalize=True)
        nside.prefill(xs[1])
        nside.reserve(4096 * (n_rep + 2))
        torch.cuda.synchronize()
        e0.record()
        for i in range(n_rep):
            nside._quantize(xs[i % 2])
        e1.record()
        torch.cuda.synchronize()
        us_chunk_n = e0.elapsed_time(e1) * 1e3 / n_rep
        del nside
        # the same chunks as values (token groups, the InnerQ V layout)
        vside = PackedSide(_lib.ROLE_V, bits, group, _lib.SYM if mode == "symmetric" else _lib.ASYM,
                           True, 0, 0, max(32, group))
        vside.prefill(x[:, :, :max(32, group)])
        vside.reserve(4096 * (n_rep + 2))
        vside.n_q = 0
        vside._quantize(xs[1])
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("chunk_v")
        e0.record()
        for i in range(n_rep):
            vside._quantize(xs[i % 2])
        e1.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        us_chunk_v = e0.elapsed_time(e1) * 1e3 / n_rep
        del side, vside, x, xs
        torch.cuda.empty_cache()
        print(json.dumps({
            "config": name, "batch": B, "q_heads": hq, "kv_heads": hkv, "context": ctx,
            "bits": bits, "group": group, "v_groups_over": vlay, "mode": mode,
            "attn_us": round(us, 1), "attn_GBs": round(nb / us / 1e3, 1),
            "frac_of_measured_hbm": round(nb / us / 1e3 / peak, 3), "bytes_per_launch": nb,
            "append_1_token_us": round(us_tok, 1), "append_4096_chunk_us": round(us_chunk, 1),
            "chunk_read_GBs": round(B * hkv * 4096 * D * 2 / us_chunk / 1e3, 1),
            "append_4096_chunk_v_us": round(us_chunk_v, 1),
            "append_4096_chunk_knorm_us": round(us_chunk_n, 1),
            "chunk_v_read_GBs": round(B * hkv * 4096 * D * 2 / us_chunk_v / 1e3, 1)}), flush=True)


def main():
    a = parse()
    if a.workload == "c3" and a.impl != "reference":
        run_c3(a)
        return
    if a.workload == "sweep":
        run_sweep(a)
        return
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
