#!/usr/bin/env python
"""Benchmark of the grouped FP8 x MXFP4 MoE GEMM (m_grouped_fp8_fp4_gemm_nt_contiguous).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c1|c2|c3|c4|c2u|c3u|c4u] [--impl ours|reference]

Workloads (seeded synthetic data with the configs' shapes and distributions,
consumer_deep_gemm.synthetic; weights transformed once at load and resident):

* N = 1, default c1: one step = one call of the public API on the decode FC1
  batch (E=256, K=N=4096, 64 tokens x top-8, 222 active experts), the HBM-bound
  case the metric is quoted on.  --config c2/c3 run the prefill shapes.
* N > 1 (launched by torchrun), default: every rank serves its own c1-sized
  decode batch (rank-seeded tokens and routing); the 256 experts are sharded
  over the ranks (expert parallelism).  One step = quantise the rank's tokens,
  exchange per-expert counts and dispatch the routed rows to the experts'
  owners (NCCL all-to-all), run the grouped GEMM on the local experts, return
  the rows (all-to-all) and combine them per token.  Weak scaling: per-rank
  tokens fixed, the expert weights divided.
* --config c4: the full expert-parallel MoE layer (FC1 -> SiLU-mul + requant ->
  FC2), 32768 tokens x top-8 split over the ranks, E=256, hidden 4096,
  intermediate 2048.  Strong scaling; reported in TFLOP/s.
* --config c2u / c3u / c4u: c2, c3 and c4 with power-of-two (UE8M0) activation scales,
  the format DeepGEMM's SM100 path quantises to (c4u: the layer quantises that way).

One JSON line on rank 0.  `value` = algorithmic bytes (or FLOPs for c4) of the
whole job per step / device time of K steps (max over ranks).  Algorithmic bytes
count routed rows of A and their scales, the weights and scales of experts that
receive rows, and routed rows of D; padding-row zeros are not counted.  `e2e`
times the same steps with the per-step inputs copied from pinned host memory and
the result copied back.  `roofline` relates the tensor-core GEMM kernels' own
duration (CUDA events the library records around them) to the measured HBM copy
bandwidth (or 2x the measured BF16 GEMM rate for c4).
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "consumer-deepgemm_b200"))
sys.path.insert(0, HERE)

import torch  # noqa: E402

METRIC = "grouped FP8×FP4 MoE GEMM TFLOPS and HBM GB/s vs roofline at 1/2/4/8 B200"
DTYPE = "fp8e4m3 x e2m1 -> fp32 acc -> bf16"
# library kernels per GEMM call on the CTA-pair path: cdg_prep_kernel, cdg_gemm_pair_kernel<16,4>,
# <32,2>, cdg_gemm_planes_kernel, cdg_gemm_direct_kernel, cdg_generic_kernel
GEMM_LAUNCHES = 6
# DRAM bytes (read + write) of one GEMM call's dominant kernel per workload, from the ncu
# captures summarised under profiles/ (absent: no capture of the current kernels yet).
NCU_TRAFFIC = {
    "c1": 2.008183e9 + 0.223044e9,  # cdg_gemm_pair_kernel<16, 4>: profiles/cdg_gemm_pair_kernel16_c1_decode.md
    "c2": 1.427530e9 + 0.654704e9,  # cdg_gemm_planes_kernel: profiles/cdg_gemm_planes_kernel_c2_prefill.md
    "c2u": 1.281316e9 + 0.648415e9,  # cdg_gemm_direct_kernel: profiles/cdg_gemm_direct_kernel_c2u_prefill.md
}
# per EP step on top of the GEMM kernels: dispatch (quantise + pack), permute, return (or unpermute), combine
EP_LAUNCHES = 4


def gemm_bytes(rows, e_act, n, k):
    return rows * k + rows * (k // 128) * 4 + e_act * n * k // 2 + e_act * n * k // 32 + rows * n * 2


def algorithmic(inp):
    """(bytes, flops, active experts) of one GEMM call on routed rows and active experts only."""
    cfg = inp["cfg"]
    ids = inp["m_indices"]
    e_act = int(torch.unique(ids[ids >= 0]).numel())
    r = inp["rows"]
    return gemm_bytes(r, e_act, cfg.n, cfg.k), 2 * r * cfg.n * cfg.k, e_act


def measured_peaks():
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples every 50 ms while the benchmark runs; stop(window)
    reports the samples taken inside the timed region (host wall-clock window of Timed.run,
    widened by one sampling period), else the samples under load."""

    FIELDS = ("timestamp,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    PERIOD_MS = 50

    def __init__(self, device_index: int):
        self.proc = None
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            sel = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-i", sel,
                 "-lms", str(self.PERIOD_MS)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self, window=None):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = []
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((float(f[1]), float(f[2]), float(f[3]), float(f[4]), f[5:9], ts))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        chosen, where = [], "timed region"
        if window is not None:
            pad = self.PERIOD_MS / 1000.0
            chosen = [r for r in rows if window[0] - pad <= r[5] <= window[1] + pad]
        if not chosen:
            chosen, where = [r for r in rows if r[3] >= 50] or rows, "samples under load (none in the timed region)"
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in chosen for i, v in enumerate(r[4]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in chosen), "sm_max_mhz": max(r[1] for r in rows),
                "samples": len(chosen), "sampled": where, "reasons": reasons}


def cpu_port_sample(inp, budget_s: float = 4.0, calls: int = 3, warmup: int = 0):
    """Time the CPU oracle (the reference's dequant + matmul restated) on a bounded sample.

    The sample is the routed rows of the first few active experts, grown until
    one call takes about `budget_s`.  Returns ({"GB/s": .., "TFLOP/s": ..}, cores,
    description), rates of the median call.
    """
    from oracle import cdg_oracle as oracle

    torch.set_num_threads(os.cpu_count() or 1)
    cfg = inp["cfg"]
    ids = inp["m_indices"].cpu()
    experts = torch.unique(ids[ids >= 0])
    a, sa = inp["a"].cpu(), inp["sa"].cpu()

    def run(n_exp):
        sel = experts[:n_exp]
        rows = torch.isin(ids, sel).nonzero().flatten()
        sub = torch.full((int(experts.max()) + 1,), -1, dtype=torch.int32)
        sub[sel] = torch.arange(sel.numel(), dtype=torch.int32)
        b = inp["b"][sel.to(inp["b"].device)].cpu()
        sb = inp["sb"][sel.to(inp["sb"].device)].cpu()
        d = torch.empty(rows.numel(), cfg.n, dtype=torch.bfloat16)
        t0 = time.perf_counter()
        oracle.m_grouped_fp8_fp4_gemm_nt_contiguous((a[rows], sa[rows]), (b, sb), d, sub[ids[rows].long()])
        return time.perf_counter() - t0, gemm_bytes(rows.numel(), sel.numel(), cfg.n, cfg.k), rows.numel()

    dt, _, _ = run(1)
    n_exp = max(1, min(int(experts.numel()), int(budget_s / max(dt, 1e-3))))
    for _ in range(warmup):
        run(n_exp)
    times = []
    for _ in range(max(1, calls)):
        dt, nbytes, r = run(n_exp)
        times.append(dt)
    dt = statistics.median(times)
    desc = (f"{cfg.name}: {r} routed rows of {n_exp} of {experts.numel()} active experts, "
            f"median of {len(times)} calls ({dt:.2f} s each), torch CPU threads={torch.get_num_threads()}")
    rates = {"GB/s": nbytes / dt / 1e9, "TFLOP/s": 2.0 * r * cfg.n * cfg.k / dt / 1e12}
    return rates, torch.get_num_threads(), desc


def run_reference(args):
    """The reference's CPU path (oracle port) on rank 0: each step is a bounded sample."""
    from consumer_deep_gemm import synthetic

    if int(os.environ.get("RANK", "0")) != 0:
        return
    cfg_name = args.config if args.config in ("c1", "c2", "c3") else "c1"
    inp = synthetic.make_inputs(synthetic.CONFIGS[cfg_name], device="cpu", seed=0,
                                weight_device="cuda" if torch.cuda.is_available() else "cpu")
    # K timed samples after W warm-up ones, about 60 s of CPU work in all
    rates, cores, desc = cpu_port_sample(inp, budget_s=max(0.2, 60.0 / max(1, args.steps + args.warmup)),
                                         calls=args.steps, warmup=args.warmup)
    unit = "GB/s" if cfg_name == "c1" else "TFLOP/s"  # the unit of our arm's line for this workload
    v = rates[unit]
    line = {
        "metric": METRIC, "impl": "reference", "value": v, "unit": unit, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": DTYPE, "data": "synthetic",
        "config": {"workload": cfg_name, "parallelism": "cpu"},
        "cpu_baseline": {"value": v, "unit": unit, "cores": cores, "kind": "port", "sample": desc},
        "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


class Timed:
    """Device time of K steps (CUDA events on the current stream) and of the GEMM kernels inside them."""

    def __init__(self, dev, steps):
        from consumer_deep_gemm import native

        self.ext = native.require()
        self.stream = torch.cuda.current_stream(dev)
        self.kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                    for _ in range(steps)]
        for s, e in self.kev:  # materialise the raw event handles
            s.record(self.stream)
            e.record(self.stream)
        torch.cuda.synchronize(dev)

    def run(self, step, steps, with_kernel_events=True):
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        wall0 = time.time()
        t0.record(self.stream)
        for i in range(steps):
            if with_kernel_events:
                self.ext.set_profile_events(self.kev[i][0].cuda_event, self.kev[i][1].cuda_event)
            step()
        self.ext.set_profile_events(0, 0)
        t1.record(self.stream)
        torch.cuda.synchronize()
        self.window = (wall0, time.time())  # host wall-clock span holding the timed device work
        ms = t0.elapsed_time(t1) / steps
        kms = statistics.fmean(s.elapsed_time(e) for s, e in self.kev[:steps]) if with_kernel_events else None
        return ms, kms


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default=None, choices=["c1", "c2", "c3", "c4", "c4u", "c2u", "c3u"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    assert args.warmup >= 3, "at least 3 warm-up steps"
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        if args.config in ("c4", "c4u"):
            line = bench_layer(args, dev, world, rank, dist)
        elif world > 1:
            line = bench_ep_decode(args, dev, world, rank, dist)
        else:
            line = bench_gemm(args, dev, args.config or "c1")
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if dist:
            dist.barrier()
            dist.destroy_process_group()


def _max_over_ranks(dist, dev, *vals):
    if dist is None:
        return vals
    t = torch.tensor(vals, device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return tuple(t.tolist())


def _sum_over_ranks(dist, dev, val):
    if dist is None:
        return val
    t = torch.tensor([val], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t.item()


def bench_gemm(args, dev, cfg_name):
    """N = 1: the public GEMM on one config."""
    import consumer_deep_gemm as cdg
    from consumer_deep_gemm import synthetic

    cfg = synthetic.CONFIGS[cfg_name]
    inp = synthetic.make_inputs(cfg, device=dev, seed=0)
    a, sa, b, sb, ids = inp["a"], inp["sa"], inp["b"], inp["sb"], inp["m_indices"]
    atoms = cdg.transform_sf_into_required_layout(sb, num_groups=b.shape[0], recipe=(1, 32))
    d = torch.empty(a.shape[0], b.shape[1], dtype=torch.bfloat16, device=dev)
    nbytes, flops, e_act = algorithmic(inp)

    def call():
        cdg.m_grouped_fp8_fp4_gemm_nt_contiguous((a, sa), (b, atoms), d, ids, recipe_a=(1, 128), recipe_b=(1, 32))

    sampler = ClockSampler(dev.index)
    for _ in range(args.warmup):
        call()
    timer = Timed(dev, args.steps)
    ms, kernel_ms = timer.run(call, args.steps)
    timed_window = timer.window

    # End to end: every step uploads its inputs from pinned host memory, runs the public call
    # and reads its result D back.  Two buffer sets and two copy streams let step i's upload
    # and step i-1's download overlap each other and the GEMM (the copy engines of the two
    # directions are separate); events order each buffer's reuse.
    h_a, h_sa, h_ids = a.cpu().pin_memory(), sa.cpu().pin_memory(), ids.cpu().pin_memory()
    h_d = [torch.empty(d.shape, dtype=d.dtype).pin_memory() for _ in range(2)]
    a2 = [torch.empty_like(a) for _ in range(2)]
    sa2 = [torch.empty_like(sa) for _ in range(2)]
    ids2 = [torch.empty_like(ids) for _ in range(2)]
    d2 = [d, torch.empty_like(d)]
    comp = torch.cuda.current_stream(dev)
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]    # inputs of the buffer set landed
    ev_used = [torch.cuda.Event() for _ in range(2)]  # its GEMM done (inputs free, result ready)
    ev_out = [torch.cuda.Event() for _ in range(2)]   # its result read back (D free)
    e2e_i = [0]

    def e2e_call():
        p = e2e_i[0] & 1
        e2e_i[0] += 1
        up.wait_event(ev_used[p])
        with torch.cuda.stream(up):
            a2[p].copy_(h_a, non_blocking=True)
            sa2[p].copy_(h_sa, non_blocking=True)
            ids2[p].copy_(h_ids, non_blocking=True)
        ev_in[p].record(up)
        comp.wait_event(ev_in[p])
        comp.wait_event(ev_out[p])
        cdg.m_grouped_fp8_fp4_gemm_nt_contiguous((a2[p], sa2[p]), (b, atoms), d2[p], ids2[p], recipe_a=(1, 128),
                                                 recipe_b=(1, 32))
        ev_used[p].record(comp)
        down.wait_event(ev_used[p])
        with torch.cuda.stream(down):
            h_d[p].copy_(d2[p], non_blocking=True)
        ev_out[p].record(down)

    def e2e_steps(n):
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        t0.record(comp)
        up.wait_event(t0)
        for _ in range(n):
            e2e_call()
        comp.wait_event(ev_out[0])
        comp.wait_event(ev_out[1])
        t1.record(comp)
        torch.cuda.synchronize(dev)
        return t0.elapsed_time(t1) / n

    e2e_steps(args.warmup)
    e2e_ms = e2e_steps(args.steps)
    clocks = sampler.stop(timed_window)
    hbm_peak, bf16_peak, peak_src = measured_peaks()
    achieved_gbs = nbytes / (kernel_ms * 1e-3) / 1e9
    achieved_tf = flops / (kernel_ms * 1e-3) / 1e12
    hbm_roof = {"bound": "hbm", "achieved": achieved_gbs, "peak": hbm_peak, "unit": "GB/s",
                "frac": achieved_gbs / hbm_peak, "traffic": NCU_TRAFFIC.get(cfg.name),
                "peak_source": peak_src, "kernel_ms": kernel_ms, "algorithmic_bytes": nbytes}
    # dense FP8 (kind::mxf8f6f4) runs at twice the BF16 rate: the denominator is twice the
    # measured cuBLAS BF16 burst rate
    tensor_roof = {"bound": "tensor", "achieved": achieved_tf, "peak": 2 * bf16_peak, "unit": "TFLOP/s",
                   "frac": achieved_tf / (2 * bf16_peak), "traffic": NCU_TRAFFIC.get(cfg.name),
                   "peak_source": peak_src + " (2 x BF16 GEMM burst)", "kernel_ms": kernel_ms,
                   "algorithmic_flops": flops}
    hbm_bound = cfg.name == "c1"  # decode is HBM-bound; the prefill shapes are tensor-bound
    line = {
        "metric": METRIC,
        "value": nbytes / (ms * 1e-3) / 1e9 if hbm_bound else flops / (ms * 1e-3) / 1e12,
        "unit": "GB/s" if hbm_bound else "TFLOP/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": DTYPE, "data": "synthetic",
        "config": {"workload": cfg.name, "experts": cfg.num_experts, "k": cfg.k, "n": cfg.n,
                   "routed_rows": inp["rows"], "m_pad": inp["m_pad"], "active_experts": e_act,
                   "parallelism": "single", "l2": "inputs larger than L2 (weights %.2f GB)" % (b.numel() / 1e9)},
        "tflops": flops / (ms * 1e-3) / 1e12,
        "gbs": nbytes / (ms * 1e-3) / 1e9,
        "roofline": hbm_roof if hbm_bound else tensor_roof,
        "roofline_other": tensor_roof if hbm_bound else hbm_roof,
        "e2e": {"value": (nbytes / (e2e_ms * 1e-3) / 1e9) if hbm_bound else flops / (e2e_ms * 1e-3) / 1e12,
                "unit": "GB/s" if hbm_bound else "TFLOP/s",
                "h2d_bytes_per_step": h_a.numel() + h_sa.numel() * 4 + h_ids.numel() * h_ids.element_size(),
                "d2h_bytes_per_step": h_d[0].numel() * 2, "ms_per_step": e2e_ms,
                "copies": "step i's upload overlaps step i-1's download (two buffer sets, two copy streams)"},
        "gpu_launches": GEMM_LAUNCHES * args.steps,
        "clocks": clocks,
    }
    if not args.no_cpu_baseline:
        rates, cores, desc = cpu_port_sample(inp)
        line["cpu_baseline"] = {"value": rates[line["unit"]], "unit": line["unit"], "cores": cores, "kind": "port",
                                "sample": desc}
    return line


def _ep_inputs(cfg, dev, rank, world, tokens, seed_base=0):
    """A rank's tokens, routing and its shard of the expert weights."""
    from consumer_deep_gemm import synthetic

    g = torch.Generator().manual_seed(seed_base + rank)
    x = torch.randn(tokens, cfg.k, generator=g).to(torch.bfloat16)
    ids = torch.rand(tokens, cfg.num_experts, generator=g).topk(cfg.topk, dim=1).indices.to(torch.int32)
    w = torch.rand(tokens, cfg.topk, generator=g)
    w = w / w.sum(1, keepdim=True)
    e_loc = cfg.num_experts // world
    b, sb = synthetic.make_weights(e_loc, cfg.n, cfg.k, dev, seed=100 + rank)
    return x.to(dev), ids.to(dev), w.to(dev), b, sb


def _local_gemm_work(counts, n, k):
    """Algorithmic (bytes, flops) of a local grouped GEMM given per-local-expert received row counts."""
    rows = int(counts.sum())
    e_act = int((counts > 0).sum())
    return gemm_bytes(rows, e_act, n, k), 2 * rows * n * k


def _global_counts(ids, num_experts, dev, dist):
    counts = torch.zeros(num_experts, dtype=torch.int32, device=dev)
    counts.index_add_(0, ids.flatten().long(), torch.ones(ids.numel(), dtype=torch.int32, device=dev))
    if dist:
        dist.all_reduce(counts)
    return counts


def bench_ep_decode(args, dev, world, rank, dist):
    """N > 1: every rank a c1 decode batch, experts sharded, NCCL dispatch/combine around the GEMM."""
    from consumer_deep_gemm import synthetic
    from consumer_deep_gemm.moe import MoELayer

    cfg = synthetic.CONFIGS["c1"]
    x, ids, w, b, sb = _ep_inputs(cfg, dev, rank, world, cfg.tokens)
    # fixed per-destination capacity, rows moved by the library's peer-memory stores over
    # NVLink: no host synchronisation and no collective on the data path
    layer = MoELayer(b, sb, num_experts=cfg.num_experts, group=dist.group.WORLD, max_tokens_per_rank=cfg.tokens,
                     exchange=os.environ.get("CDG_EP_EXCHANGE", "p2p"))
    e_loc = cfg.num_experts // world
    mine = _global_counts(ids, cfg.num_experts, dev, dist)[rank * e_loc:(rank + 1) * e_loc].cpu()
    local_bytes, local_flops = _local_gemm_work(mine, cfg.n, cfg.k)
    job_bytes = _sum_over_ranks(dist, dev, local_bytes)
    job_flops = _sum_over_ranks(dist, dev, local_flops)

    def step():
        layer(x, ids, w)

    sampler = ClockSampler(dev.index)
    for _ in range(args.warmup):
        step()
    # the GEMM kernels' device time, from eager steps with per-step events
    timer = Timed(dev, args.steps)
    dist.barrier()
    torch.cuda.synchronize(dev)
    _, kernel_ms = timer.run(step, args.steps)
    dist.barrier()
    # the step itself: one CUDA graph per rank (peer exchange: no host value per step)
    use_graph = layer.exchange == "p2p"
    if use_graph:
        graph, _ = layer.capture(x, ids, w)
        step = graph.replay
        for _ in range(args.warmup):
            step()
    dist.barrier()
    torch.cuda.synchronize(dev)
    ms, _ = timer.run(step, args.steps, with_kernel_events=False)
    timed_window = timer.window
    dist.barrier()

    h_x, h_ids, h_w = x.cpu().pin_memory(), ids.cpu().pin_memory(), w.cpu().pin_memory()
    h_y = torch.empty(x.shape[0], cfg.n, dtype=torch.bfloat16).pin_memory()
    x2, ids2, w2 = torch.empty_like(x), torch.empty_like(ids), torch.empty_like(w)
    x2.copy_(x)
    ids2.copy_(ids)
    w2.copy_(w)
    if use_graph:
        e2e_graph, y2 = layer.capture(x2, ids2, w2)

    def e2e_step():
        x2.copy_(h_x, non_blocking=True)
        ids2.copy_(h_ids, non_blocking=True)
        w2.copy_(h_w, non_blocking=True)
        if use_graph:
            e2e_graph.replay()
            h_y.copy_(y2, non_blocking=True)
        else:
            h_y.copy_(layer(x2, ids2, w2), non_blocking=True)
    for _ in range(args.warmup):
        e2e_step()
    dist.barrier()
    torch.cuda.synchronize(dev)
    e2e_ms, _ = timer.run(e2e_step, args.steps, with_kernel_events=False)
    clocks = sampler.stop(timed_window)
    ms, e2e_ms, kernel_ms = _max_over_ranks(dist, dev, ms, e2e_ms, kernel_ms)
    torch.cuda.synchronize(dev)
    dist.barrier()
    layer.close()  # after every rank's last forward
    hbm_peak, _, peak_src = measured_peaks()
    achieved = local_bytes / (kernel_ms * 1e-3) / 1e9
    return {
        "metric": METRIC, "value": job_bytes / (ms * 1e-3) / 1e9, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": DTYPE, "data": "synthetic",
        "config": {"workload": "c1-ep", "experts": cfg.num_experts, "k": cfg.k, "n": cfg.n,
                   "tokens_per_rank": cfg.tokens, "topk": cfg.topk, "parallelism": f"ep{world}",
                   "step": "quant, count all-to-all, dispatch all-to-all, grouped GEMM on local experts, "
                           "return all-to-all, weighted combine",
                   "exchange": "fixed capacity per destination (tokens*topk rows), no host synchronisation; "
                               + ("peer-memory stores over NVLink, step replayed as one CUDA graph per rank"
                                  if layer.exchange == "p2p" else "NCCL all-to-all"),
                   "l2": "weights per rank larger than L2"},
        "tflops": job_flops / (ms * 1e-3) / 1e12,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "traffic": None, "peak_source": peak_src,
                     "kernel_ms": kernel_ms, "algorithmic_bytes": local_bytes, "note": "rank 0's GEMM kernels"},
        "e2e": {"value": job_bytes / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": h_x.numel() * 2 + h_ids.numel() * 4 + h_w.numel() * 4,
                "d2h_bytes_per_step": h_y.numel() * 2, "ms_per_step": e2e_ms},
        "gpu_launches": (GEMM_LAUNCHES + EP_LAUNCHES) * args.steps,
        "clocks": clocks,
    }


def bench_layer(args, dev, world, rank, dist):
    """--config c4: the full expert-parallel MoE layer, 32768 tokens split over the ranks.
    --config c4u: the same layer quantising its activations with power-of-two (UE8M0) scales."""
    from consumer_deep_gemm import synthetic
    from consumer_deep_gemm.moe import MoELayer

    c1 = synthetic.CONFIGS["c4_fc1"]
    c2 = synthetic.CONFIGS["c4_fc2"]
    tokens = c1.tokens // world
    x, ids, w, b1, s1 = _ep_inputs(c1, dev, rank, world, tokens)
    b2, s2 = synthetic.make_weights(c1.num_experts // world, c2.n, c2.k, dev, seed=200 + rank)
    ue8m0 = args.config == "c4u"
    layer = MoELayer(b1, s1, b2, s2, num_experts=c1.num_experts, group=dist.group.WORLD if dist else None,
                     ue8m0=ue8m0)
    e_loc = c1.num_experts // world
    mine = _global_counts(ids, c1.num_experts, dev, dist)[rank * e_loc:(rank + 1) * e_loc].cpu()
    _, f_fc1 = _local_gemm_work(mine, c1.n, c1.k)
    _, f_fc2 = _local_gemm_work(mine, c2.n, c2.k)
    job_flops = _sum_over_ranks(dist, dev, f_fc1 + f_fc2)

    def step():
        layer(x, ids, w)

    sampler = ClockSampler(dev.index)
    for _ in range(args.warmup):
        step()
    timer = Timed(dev, args.steps)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    # the library's profile events bracket the last GEMM call of a step (FC2)
    ms, fc2_ms = timer.run(step, args.steps)
    clocks = sampler.stop(timer.window)
    ms, fc2_ms = _max_over_ranks(dist, dev, ms, fc2_ms)
    _, bf16_peak, peak_src = measured_peaks()
    fp8_peak = 2 * bf16_peak
    achieved = f_fc2 / (fc2_ms * 1e-3) / 1e12
    return {
        "metric": METRIC, "value": job_flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": DTYPE, "data": "synthetic",
        "config": {"workload": args.config, "experts": c1.num_experts, "hidden": c1.k, "intermediate": c2.k,
                   "tokens": c1.tokens, "topk": c1.topk, "parallelism": f"ep{world}",
                   "activation_scales": "ue8m0 (power of two)" if ue8m0 else "fp32 1x128"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": fp8_peak, "unit": "TFLOP/s",
                     "frac": achieved / fp8_peak, "traffic": None, "kernel": "FC2 GEMM kernels (rank 0)",
                     "peak_source": f"2 x {peak_src} bf16 GEMM rate (dense FP8:BF16 = 2:1)"},
        "gpu_launches": (2 * GEMM_LAUNCHES + EP_LAUNCHES + 1) * args.steps,
        "clocks": clocks,
    }


if __name__ == "__main__":
    main()
