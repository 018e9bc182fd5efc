"""Benchmark: MoE FFN layer at Qwen3-30B-A3B shape on B200.

One step = one call of the MoE layer (router -> top-k -> dispatch -> grouped
Q4_K gate/up + SwiGLU -> grouped Q6_K down -> combine) on a batch of B tokens.
Weights: 48 layers of configs[1] (d=2048, 128 experts top-8, ff=768, Q4_K
gate/up + Q6_K down from N(0, 0.02), F32 router N(0, 0.02)) made on the GPU
with this library's quantizer; step i runs layer i % 48, so the 18.8 GB of
weights stream from HBM (inputs larger than L2; no step reuses another's
weights from L2). Activations: f32 N(0, 1), a pool of distinct batches.

  value   tokens/s over all ranks, device-timed (CUDA events, max over ranks)
  e2e     same metric through the host-pointer C ABI call kc_moe_ffn (pinned
          host h in, host out back), wall-clock around synchronous calls
  roofline  dominant kernel's algorithmic HBM bytes / its event-timed
            duration vs MEASURED_PEAKS.json's copy bandwidth
  cpu_baseline  the CPU oracle (C++ AVX2 restatement of Kestrel's path) on a
                bounded sample of the same workload, all host threads

--config c2 / c4 measure the other single-layer configs the same way
(Mixtral-8x7B shape; Qwen3-235B-A22B shape with Zipf-skewed routing).

--impl reference times the oracle alone (the reference's CPU arithmetic) on
the same config. Multi-GPU (torchrun, N ranks): expert parallelism -- rank r
holds experts [r*E/N, (r+1)*E/N) of every layer and a copy of the router, routes
its own B tokens, and exchanges token rows and result rows with NCCL inside
each layer call (weak scaling: N*B tokens per step).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# The single-layer configs of the benchmark list: c1 (the headline), c2 and c4.
# `layers`: distinct layers rotated so that no step finds its weights in L2.
CONFIGS = {
    "c1": dict(name="qwen3-30b-a3b-moe-layer", d=2048, E=128, k=8, ff=768, layers=48, batch=16,
               sweep=[1, 16, 128, 512], zipf=False),
    "c2": dict(name="mixtral-8x7b-moe-layer", d=4096, E=8, k=2, ff=14336, layers=8, batch=1,
               sweep=[1, 512, 2048, 4096], zipf=False),
    "c4": dict(name="qwen3-235b-a22b-moe-layer-zipf", d=4096, E=128, k=8, ff=1536, layers=8, batch=64,
               sweep=[1, 64, 2048], zipf=True),
}
CFG = dict(CONFIGS["c1"])
# Tokens per rank and call reserved for the peer-memory exchange (multi-GPU):
# the headline batch by default (--ep-tokens); larger calls use NCCL.


def bytes_per_expert() -> int:
    """Q4_K gate + up and Q6_K down of one expert (c1: 3,059,712 B)."""
    return 2 * CFG["ff"] * (CFG["d"] // 256) * 144 + CFG["d"] * (CFG["ff"] // 256) * 210


def router_bytes() -> int:
    return CFG["E"] * CFG["d"] * 4


def zipf_router_column(rng, E, d):
    """configs[4]'s skew: router column 0 holds beta_e = -1.2 ln(1 + rank(e))
    sigma_logit for a seeded rank permutation; with input feature 0 set to 1
    this adds beta_e to expert e's logit (popularity ~ Zipf s=1.2)."""
    rank = rng.permutation(E)
    return (-1.2 * np.log1p(rank) * 0.02 * np.sqrt(d)).astype(np.float32)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def bf16_peak_tflops() -> float:
    """Measured dense bf16 GEMM throughput (burst), else the pool's fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"])
    except Exception:
        return 1590.0


def algorithmic_bytes(ids: np.ndarray, B: int, block=None) -> dict:
    """Per call: distinct routed experts x bytes/expert + router + x in/out, and
    the split of expert bytes between the int8 (<4 rows) and f32 paths. ids are
    the selections of every token the experts see; with an expert block only
    that block's experts count (the weights this rank streams)."""
    d, ff = CFG["d"], CFG["ff"]
    cnt = np.bincount(ids.reshape(-1), minlength=CFG["E"])
    if block is not None:
        cnt = cnt[block.first:block.first + block.count]
    small = int(((cnt >= 1) & (cnt <= 3)).sum())
    large = int((cnt >= 4).sum())
    gate_up = 2 * ff * (d // 256) * 144
    down = d * (ff // 256) * 210
    return dict(total=(small + large) * bytes_per_expert() + router_bytes() + B * d * 4 * 2,
                gate_up_int8=small * gate_up, down_int8=small * down, gate_up_f32=large * gate_up,
                down_f32=large * down, router=router_bytes(), experts=small + large)


class ClockSampler:
    """SM clock and clock-event reasons sampled during the timed region: NVML
    read from a thread about every millisecond (the timed region can be a few
    ms), else nvidia-smi every 100 ms. Reads only; changes no setting."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits (nvml.h): sw_power_cap 0x4, hw_slowdown 0x8,
    # sw_thermal_slowdown 0x20, hw_thermal_slowdown 0x40.
    REASON_BITS = (("sw_power_cap", 0x4), ("hw_slowdown", 0x8), ("sw_thermal_slowdown", 0x20),
                   ("hw_thermal_slowdown", 0x40))

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.path = None
        self.thread = None
        self.samples = []
        self.max_mhz = None
        self.stop = False

    def _poll(self, nv, hnd):
        while not self.stop:
            try:
                sm = nv.nvmlDeviceGetClockInfo(hnd, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksThrottleReasons(hnd)
                self.samples.append((sm, rs))
            except Exception:
                break
            time.sleep(0.001)

    def __enter__(self):
        # A short switch interval lets the polling thread run while the main
        # thread launches the timed steps (restored on exit).
        self.switch = sys.getswitchinterval()
        sys.setswitchinterval(0.0002)
        try:
            import pynvml as nv
            import torch
            nv.nvmlInit()
            # NVML numbers the machine's GPUs and ignores CUDA_VISIBLE_DEVICES:
            # open this process's GPU by its PCI bus id.
            hnd = None
            try:
                p = torch.cuda.get_device_properties(self.gpu)
                bus = "%08x:%02x:%02x.0" % (p.pci_domain_id, p.pci_bus_id, p.pci_device_id)
                hnd = nv.nvmlDeviceGetHandleByPciBusId_v2(bus)
            except Exception:
                hnd = None
            if hnd is None:
                hnd = nv.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(hnd, nv.NVML_CLOCK_SM)
            import threading
            self.thread = threading.Thread(target=self._poll, args=(nv, hnd), daemon=True)
            self.thread.start()
            return self
        except Exception:
            self.thread = None
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.15)
        return self

    def __exit__(self, *a):
        sys.setswitchinterval(self.switch)
        if self.thread:
            self.stop = True
            self.thread.join(timeout=5)
        if self.proc:
            self.proc.terminate()
            self.proc.wait(timeout=5)

    def summary(self):
        if self.thread is not None:
            if not self.samples:
                return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"], "samples": 0,
                        "source": "nvml"}
            reasons = sorted({n for _, rs in self.samples for n, bit in self.REASON_BITS if rs & bit})
            out = {"sm_mhz": statistics.median(float(sm) for sm, _ in self.samples),
                   "sm_max_mhz": float(self.max_mhz) if self.max_mhz else None, "reasons": reasons,
                   "samples": len(self.samples), "source": "nvml"}
            if len(self.samples) < 10:
                out["note"] = "fewer than 10 samples: the median is unreliable"
            return out
        rows = []
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        except Exception:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "source": "nvidia-smi"}


# ----------------------------------------------------------------------------
def make_layers(ctx, torch, n_layers, seed=0, block=None):
    """configs[1] weights on the GPU: N(0, 0.02) quantised to Q4_K / Q6_K by
    kc_quantize_dev, uploaded with kc_upload_experts (device source). With an
    expert block (expert parallelism) only that block is generated; the router
    is the same on every rank."""
    from kestrel_b200 import ggml as G
    E, d, ff, k = CFG["E"], CFG["d"], CFG["ff"], CFG["k"]
    first, n_loc = (0, E) if block is None else (block.first, block.count)
    g = torch.Generator(device="cuda").manual_seed(seed + first)
    gr = torch.Generator(device="cuda").manual_seed(seed + 777)
    bufs = {n: torch.empty((rows, G.bytes_for(t, cols)), dtype=torch.uint8, device="cuda")
            for n, t, rows, cols in (("gate", G.Q4_K, n_loc * ff, d), ("up", G.Q4_K, n_loc * ff, d),
                                     ("down", G.Q6_K, n_loc * d, ff))}
    x = torch.empty((n_loc * ff, d), dtype=torch.float32, device="cuda")
    for layer in range(n_layers):
        for n, t in (("gate", G.Q4_K), ("up", G.Q4_K), ("down", G.Q6_K)):
            xv = x.view(n_loc * d, ff) if n == "down" else x
            xv.normal_(0.0, 0.02, generator=g)
            ctx.quantize_dev(t, xv, bufs[n])
        router = torch.empty((E, d), dtype=torch.float32, device="cuda").normal_(0.0, 0.02, generator=gr)
        if CFG["zipf"]:
            router[:, 0] = torch.from_numpy(zipf_router_column(np.random.default_rng(layer), E, d)).cuda()
        ctx.upload_experts(layer, E, d, ff, G.Q4_K, bufs["gate"], G.Q4_K, bufs["up"], G.Q6_K, bufs["down"],
                           first_expert=first, n_local=n_loc)
        ctx.upload_router(layer, router, k)
        if layer == 0:
            host0 = {n: b.cpu().numpy() for n, b in bufs.items()}
            host0["router"] = router.cpu().numpy()
    del x, bufs
    torch.cuda.empty_cache()
    return host0


def physical_cores() -> int:
    """Physical cores of the host (the reference sizes its thread pool by
    physical cores); logical CPUs if psutil cannot tell."""
    try:
        import psutil
        n = psutil.cpu_count(logical=False)
        if n:
            return int(n)
    except Exception:
        pass
    return os.cpu_count() or 1


def cpu_oracle_rate(layer_w, B, budget_s, threads, seed=5, min_calls=2):
    """The oracle's moe_ffn (C++ restatement of Kestrel's AVX2 path) on one
    layer, B tokens per call, `threads` threads, repeated until `budget_s`
    seconds have elapsed. Returns (tokens/s, calls, seconds, weight GB/s),
    the GB/s by the GPU arm's algorithmic byte count."""
    import oracle
    from kestrel_b200 import ggml as G
    oracle.set_threads(threads)
    rng = np.random.default_rng(seed)
    calls, tokens, nbytes, t0 = 0, 0, 0, time.perf_counter()
    while True:
        h = rng.standard_normal((B, CFG["d"]), dtype=np.float32)
        if CFG["zipf"]:
            h[:, 0] = 1.0
        _, ids, _ = oracle.moe_ffn(h, layer_w["router"], CFG["k"], G.Q4_K, layer_w["gate"], G.Q4_K, layer_w["up"],
                                   G.Q6_K, layer_w["down"], CFG["ff"])
        nbytes += algorithmic_bytes(ids, B)["total"]
        calls += 1
        tokens += B
        el = time.perf_counter() - t0
        if el >= budget_s and calls >= min_calls:
            return tokens / el, calls, el, nbytes / el / 1e9


# The reference's published CPU figure for the same weight format: a Q4_K
# gemv at 9.19 GB/s on 4 cores (benchmarks/README.md of the reference).
CPU_ANCHOR = "reference's published Q4_K gemv: 9.19 GB/s on 4 cores"


def cpu_baseline_both(layer_w, B, budget_s):
    """The D4 baseline: all physical cores and one thread, each with its
    weight GB/s (same byte formula as the GPU arm)."""
    phys = physical_cores()
    rate, calls, el, gbs = cpu_oracle_rate(layer_w, B, budget_s, phys)
    r1, c1, e1, g1 = cpu_oracle_rate(layer_w, B, budget_s / 2, 1, min_calls=1)
    return {"value": rate, "unit": "tokens/s", "cores": phys, "kind": "port", "gbs": gbs,
            "one_thread": {"value": r1, "unit": "tokens/s", "gbs": g1, "sample": f"{c1} calls ({e1:.1f} s)"},
            "logical_cpus": os.cpu_count(), "anchor": CPU_ANCHOR,
            "sample": f"{calls} calls of layer 0 at B={B} ({el:.1f} s) on {phys} physical cores, oracle "
                      f"restatement of Kestrel's AVX2 path; weights numpy-quantized from other seeds than the "
                      f"GPU arm's (same shapes and rules)"}


def host_layer_numpy(seed=0):
    """One configs[1] layer generated on the CPU (numpy quantizer, threads)."""
    from concurrent.futures import ThreadPoolExecutor

    from kestrel_b200 import ggml as G
    E, d, ff = CFG["E"], CFG["d"], CFG["ff"]

    def mat(name, t, rows, cols, s):
        out = np.empty((rows, G.bytes_for(t, cols)), np.uint8)
        step = 4096

        def part(r0):
            rng = np.random.default_rng([s, r0])
            x = rng.standard_normal((min(step, rows - r0), cols), dtype=np.float32) * np.float32(0.02)
            out[r0:r0 + x.shape[0]] = G.quantize(t, x)

        with ThreadPoolExecutor(os.cpu_count() or 4) as ex:
            list(ex.map(part, range(0, rows, step)))
        return out

    w = {"gate": mat("gate", G.Q4_K, E * ff, d, seed * 10 + 1), "up": mat("up", G.Q4_K, E * ff, d, seed * 10 + 2),
         "down": mat("down", G.Q6_K, E * d, ff, seed * 10 + 3)}
    w["router"] = (np.random.default_rng(seed * 10 + 4).standard_normal((E, d), dtype=np.float32) *
                   np.float32(0.02))
    if CFG["zipf"]:
        w["router"][:, 0] = zipf_router_column(np.random.default_rng(0), E, d)
    return w


# ----------------------------------------------------------------------------
def run_reference(args):
    """--impl reference: the reference's CPU arithmetic (the oracle restatement;
    the Rust reference cannot be built in this image) on the same config."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = physical_cores()
    w = host_layer_numpy()
    B = args.batch
    for _ in range(args.warmup):
        cpu_oracle_rate(w, B, 0.0, threads)
    times, gbs = [], []
    for i in range(args.steps):
        r, c, e, g = cpu_oracle_rate(w, B, 0.0, threads, seed=100 + i)
        times.append(e / c)
        gbs.append(g)
    ms = 1e3 * sum(times) / len(times)
    value = B / (ms / 1e3)
    line = {
        "metric": "moe_layer_tokens_per_s", "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8xq4k/f32", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": CFG["name"], "batch_tokens": B, "d_model": CFG["d"], "experts": CFG["E"],
                   "top_k": CFG["k"], "expert_ff": CFG["ff"], "quant": "Q4_K gate/up + Q6_K down"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "gbs": sum(gbs) / len(gbs), "logical_cpus": os.cpu_count(), "anchor": CPU_ANCHOR,
                         "sample": f"{args.steps} calls of one layer at B={B} on {threads} physical cores "
                                   f"(oracle restatement of Kestrel's AVX2 path; Rust reference not buildable "
                                   f"here)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def timed_steps(torch, ctx, hs, outs, n_layers, B, steps, stream, issue=None):
    """Device time (ms) of `steps` layer calls, CUDA events on the library's
    stream. issue (optional dict): the host time spent issuing the calls (the
    loop before the end event's wait) and the kernels they launched."""
    from kestrel_b200.cuda import kernel_launches
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    n0 = kernel_launches()
    start.record(stream)
    t0 = time.perf_counter()
    for i in range(steps):
        ctx.moe_ffn_dev(i % n_layers, hs[i % len(hs)], outs[i % len(outs)], n_tok=B)
    t1 = time.perf_counter()
    end.record(stream)
    end.synchronize()
    if issue is not None:
        issue["host_s"] = t1 - t0
        issue["launches"] = kernel_launches() - n0
    return start.elapsed_time(end)


def run_ours(args):
    import torch
    import torch.distributed as dist
    from kestrel_b200.cuda import Context

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    ctx = Context(local)
    block = None
    if world > 1:
        from kestrel_b200 import ep
        block = ep.expert_block(CFG["E"], world, rank)
        ep.join(ctx, rank, world)
    # A dedicated (non-default) stream shared by torch and the library, so the
    # CUDA events bracket the library's kernels.
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    n_layers = args.layers
    host0 = make_layers(ctx, torch, n_layers, seed=0, block=block)
    if world > 1:
        # Calls of up to --ep-tokens tokens per rank (the headline batch by
        # default) exchange rows through NVLink peer memory; larger ones (the
        # sweep's prefill sizes) go through NCCL. The owner's expert pipeline
        # runs over the reserved capacity of every source, so the reservation
        # is the batch served (16 against 64 tokens on 2 GPUs: 168.2 against
        # 170.3 us per step).
        ctx.ep_reserve(args.ep_tokens)
    B = args.batch
    batches = sorted(set([B] + args.sweep))
    ctx.reserve(max(batches))
    d = CFG["d"]
    g = torch.Generator(device="cuda").manual_seed(1234 + rank)
    pool = {b: [torch.randn((b, d), generator=g, device="cuda") for _ in range(16)] for b in batches}
    if CFG["zipf"]:
        for b in batches:
            for t in pool[b]:
                t[:, 0] = 1.0
    outs = {b: [torch.empty((b, d), device="cuda") for _ in range(2)] for b in batches}

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def all_ids(ids_dev):
        """Selections of every rank's tokens (what this rank's experts see)."""
        if world == 1:
            return ids_dev.cpu().numpy()
        parts = [torch.empty_like(ids_dev) for _ in range(world)]
        dist.all_gather(parts, ids_dev)
        return torch.cat(parts).cpu().numpy()

    # Warm-up, then the timed region at the headline batch.
    timed_steps(torch, ctx, pool[B], outs[B], n_layers, B, args.warmup, stream)
    barrier()
    torch.cuda.synchronize()
    issue = {}
    with ClockSampler(local) as clk:
        ms_total = timed_steps(torch, ctx, pool[B], outs[B], n_layers, B, args.steps, stream, issue)
    torch.cuda.synchronize()
    barrier()
    ms_total = max_over_ranks(ms_total)
    ms_step = ms_total / args.steps
    value = world * B * args.steps / (ms_total / 1e3)
    clocks = clk.summary()

    # Profiling pass (separate from the timed region): per-stage event times and
    # the routed experts of every call -> algorithmic bytes per stage.
    hbm_peak, peak_kind = peaks()
    bf16_peak = bf16_peak_tflops()
    prof_steps = max(args.steps, 16)
    ids_dev = torch.empty((B, CFG["k"]), dtype=torch.int32, device="cuda")
    ctx.profile_read()
    ctx.profile_enable(True)
    byte_acc = {}
    for i in range(prof_steps):
        ctx.moe_ffn_dev(i % n_layers, pool[B][i % 16], outs[B][0], ids_dev, None, n_tok=B)
        ab = algorithmic_bytes(all_ids(ids_dev), B, block)
        for kk, v in ab.items():
            byte_acc[kk] = byte_acc.get(kk, 0) + v
    stages = ctx.profile_read()
    ctx.profile_enable(False)
    stage_bytes = {"gate_up_int8": byte_acc["gate_up_int8"], "down_int8": byte_acc["down_int8"],
                   "gate_up_f32": byte_acc["gate_up_f32"], "down_f32": byte_acc["down_f32"],
                   "router_logits": byte_acc["router"]}
    # Dominant kernel stage among those that stream weights (the exchange and
    # small metadata stages move no weight bytes).
    dom = max((s for s in stages if s in stage_bytes and stages[s][1]), key=lambda s: stages[s][0])
    dom_ms, dom_calls = stages[dom]
    dom_bytes = stage_bytes.get(dom, 0)
    achieved = (dom_bytes / dom_calls) / (dom_ms / dom_calls / 1e3) / 1e9 if dom_ms > 0 and dom_calls else 0.0
    # DRAM traffic of the dominant kernel per launch: ncu's dram read+write of the
    # same kernel on the profile_layer B=16 case, as a ratio to that launch's
    # algorithmic bytes (profiles/decode_kernel_c1_b16.md), scaled to this
    # launch's algorithmic bytes. Traffic grows with the experts served.
    traffic_ratio = {"gate_up_int8": 1.036, "down_int8": 1.033}
    traffic = (dom_bytes / dom_calls) * traffic_ratio[dom] if dom in traffic_ratio and dom_calls else None
    traffic_src = ("ncu dram read+write / algorithmic bytes of this kernel on the B=16 profile case "
                   "(profiles/decode_kernel_c1_b16.md), times this launch's algorithmic bytes"
                   if traffic is not None else None)
    layer_bytes = byte_acc["total"] / prof_steps
    layer_gbs = layer_bytes / (ms_step / 1e3) / 1e9
    stage_report = {s: {"ms_per_call": (v[0] / v[1]) if v[1] else 0.0,
                        "share": v[0] / max(1e-9, sum(x[0] for x in stages.values())),
                        "gbs": (stage_bytes[s] / v[1]) / (v[0] / v[1] / 1e3) / 1e9
                        if s in stage_bytes and v[0] > 0 else None}
                    for s, v in stages.items() if v[1]}

    # Sweep of the other batch sizes (device-timed, short).
    sweep = {}
    for b in batches:
        steps_b = max(8, args.steps // 2)
        timed_steps(torch, ctx, pool[b], outs[b], n_layers, b, 3, stream)
        barrier()
        ms_b = max_over_ranks(timed_steps(torch, ctx, pool[b], outs[b], n_layers, b, steps_b, stream))
        ids_b = torch.empty((b, CFG["k"]), dtype=torch.int32, device="cuda")
        tot = 0
        for i in range(4):
            ctx.moe_ffn_dev(i % n_layers, pool[b][i], outs[b][0], ids_b, None, n_tok=b)
            tot += algorithmic_bytes(all_ids(ids_b), b, block)["total"]
        per_ms = ms_b / steps_b
        flops = 2.0 * b * CFG["k"] * 3 * CFG["d"] * CFG["ff"]  # routed experts' products of one rank's batch
        sweep[str(b)] = {"ms_per_step": per_ms, "tokens_per_s": world * b / (per_ms / 1e3),
                         "hbm_gbs": (tot / 4) / (per_ms / 1e3) / 1e9,
                         "hbm_frac": (tot / 4) / (per_ms / 1e3) / 1e9 / hbm_peak,
                         "tflops": flops / (per_ms / 1e3) / 1e12,
                         "tensor_frac": flops / (per_ms / 1e3) / 1e12 / bf16_peak}

    # End to end through the host-pointer C ABI call (pinned buffers).
    hp = [torch.randn((B, d), generator=torch.Generator().manual_seed(i)).pin_memory().numpy()
          for i in range(4)]
    if CFG["zipf"]:
        for a in hp:
            a[:, 0] = 1.0
    # The result comes back into a pinned buffer; the top-k ids / weights are
    # not read back (the layer output is the step's result).
    hout = torch.empty((B, d), dtype=torch.float32).pin_memory().numpy()
    e2e_steps = max(4, args.steps // 2)
    for i in range(3):
        ctx.moe_ffn(i % n_layers, hp[i % 4], out=hout, topk=False)
    barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        ctx.moe_ffn(i % n_layers, hp[i % 4], out=hout, topk=False)
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e_value = world * B * e2e_steps / e2e_s

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_both(host0, B, args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": "moe_layer_tokens_per_s", "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8xq4k/f32", "data": "synthetic",
            "config": {"workload": CFG["name"], "batch_tokens": B, "d_model": CFG["d"], "experts": CFG["E"],
                       "top_k": CFG["k"], "expert_ff": CFG["ff"], "quant": "Q4_K gate/up + Q6_K down",
                       "layers_rotated": n_layers,
                       "l2": f"inputs larger than L2 ({n_layers} distinct layers, "
                             f"{n_layers * CFG['E'] * bytes_per_expert() / 1e9:.1f} GB of expert weights)",
                       "parallelism": f"ep{world}" if world > 1 else "single",
                       "experts_per_gpu": CFG["E"] // world},
            "layer_hbm": {"bytes_per_step": layer_bytes, "gbs": layer_gbs, "frac": layer_gbs / hbm_peak,
                          "peak": hbm_peak, "peak_kind": peak_kind},
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak, "traffic": traffic, "traffic_source": traffic_src,
                         "peak_kind": peak_kind},
            "stages": stage_report,
            "sweep": sweep,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": B * d * 4,
                    "d2h_bytes_per_step": B * d * 4},
            # this library's kernel launches in the timed region (kc_kernel_launches before and
            # after; NCCL's own kernels are not counted), and the host time spent issuing the
            # timed calls (all of them are asynchronous): below the device time per call, the
            # call is bound by the GPU, not by the host issuing it.
            "gpu_launches": issue["launches"],
            "host_issue_us_per_call": issue["host_s"] / args.steps * 1e6,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c1",
                    help="c1: Qwen3-30B-A3B layer (headline); c2: Mixtral-8x7B layer; c4: Qwen3-235B-A22B "
                         "layer with Zipf-skewed routing")
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--sweep", type=lambda s: [int(x) for x in s.split(",") if x], default=None)
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ep-tokens", type=int, default=None,
                    help="tokens per rank and call reserved for the peer-memory exchange (multi-GPU)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    CFG.update(CONFIGS[args.config])
    args.batch = CFG["batch"] if args.batch is None else args.batch
    args.sweep = CFG["sweep"] if args.sweep is None else args.sweep
    args.layers = CFG["layers"] if args.layers is None else args.layers
    args.ep_tokens = args.batch if args.ep_tokens is None else args.ep_tokens
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
