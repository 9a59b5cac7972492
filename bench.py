#!/usr/bin/env python
"""Benchmark of the grouped FP8 x MXFP4 MoE GEMM (m_grouped_fp8_fp4_gemm_nt_contiguous).

One step = one call of the public API on one batch of a benchmark config
(default c1: the decode FC1 shape E=256, K=N=4096, 64 tokens x top-8, the
HBM-bound case the metric is quoted on).  Inputs are seeded synthetic data with
the config's shapes and distributions (consumer_deep_gemm.synthetic); weights
are transformed once (weight-load time) and stay resident, as in serving.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c1|c2|c3] [--impl ours|reference]

Prints one JSON line on rank 0.  `value` is the algorithmic HBM throughput (GB/s;
bytes of the routed rows of A and their scales, the weights and scales of the
experts that receive rows, and the routed rows of D) of the whole job divided
by the device time of K steps (max over ranks).  `e2e` times the same calls
with the step's inputs copied from pinned host memory and D copied back inside
the timed region.  `roofline` relates the tensor-core GEMM kernels' own duration
(CUDA events recorded by the library around them) to the measured HBM copy
bandwidth.  With --gpus N > 1 every rank runs its own batch (rank-seeded
routing) on its own GPU: weak scaling, no collective on the data path.
"""

from __future__ import annotations

import argparse
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
# cdg_prep_kernel, cdg_gemm_kernel<16>, cdg_gemm_kernel<32>, cdg_gemm_kernel<128>, cdg_generic_kernel
LAUNCHES_PER_CALL = 5


def algorithmic(inp):
    """(bytes, flops) of one call counted on routed rows and active experts only."""
    cfg = inp["cfg"]
    ids = inp["m_indices"]
    r = inp["rows"]
    e_act = int(torch.unique(ids[ids >= 0]).numel())
    n, k = cfg.n, cfg.k
    nbytes = r * k + r * (k // 128) * 4 + e_act * n * k // 2 + e_act * n * k // 32 + r * n * 2
    return nbytes, 2 * r * n * k, e_act


def measured_peaks():
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples every 200 ms while the benchmark runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.proc = None
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            sel = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-i", sel,
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
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
            if len(f) < 8:
                continue
            try:
                rows.append((float(f[0]), float(f[1]), float(f[2]), float(f[3]), f[4:8]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        loaded = [r for r in rows if r[3] >= 50] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i, v in enumerate(r[4]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "samples": len(loaded), "reasons": reasons}


def cpu_port_sample(inp, budget_s: float = 4.0):
    """Time the CPU oracle (the reference's dequant + matmul restated) on a bounded sample.

    The sample is the routed rows of the first few active experts, grown until
    one call takes about `budget_s`.  Returns (GB/s, cores, description).
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
        sub = torch.full((experts.max().item() + 1,), -1, dtype=torch.int32)
        sub[sel] = torch.arange(sel.numel(), dtype=torch.int32)
        b = inp["b"][sel.to(inp["b"].device)].cpu()
        sb = inp["sb"][sel.to(inp["sb"].device)].cpu()
        d = torch.empty(rows.numel(), cfg.n, dtype=torch.bfloat16)
        t0 = time.perf_counter()
        oracle.m_grouped_fp8_fp4_gemm_nt_contiguous((a[rows], sa[rows]), (b, sb), d, sub[ids[rows].long()])
        dt = time.perf_counter() - t0
        r = rows.numel()
        k, n = cfg.k, cfg.n
        nbytes = r * k + r * (k // 128) * 4 + sel.numel() * n * k // 2 + sel.numel() * n * k // 32 + r * n * 2
        return dt, nbytes, r

    n_exp = 1
    dt, _, _ = run(n_exp)
    n_exp = max(1, min(int(experts.numel()), int(budget_s / max(dt, 1e-3))))
    times = []
    for _ in range(3):
        dt, nbytes, r = run(n_exp)
        times.append(dt)
    dt = statistics.median(times)
    desc = (f"{cfg.name}: {r} routed rows of {n_exp} of {experts.numel()} active experts, "
            f"median of 3 calls ({dt:.2f} s each), torch CPU threads={torch.get_num_threads()}")
    return nbytes / dt / 1e9, torch.get_num_threads(), desc


def run_reference(args, cfg_name):
    """The reference's CPU path (oracle port) on rank 0: each step is a bounded sample."""
    from consumer_deep_gemm import synthetic

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    inp = synthetic.make_inputs(synthetic.CONFIGS[cfg_name], device="cpu", seed=0,
                                weight_device="cuda" if torch.cuda.is_available() else "cpu")
    gbs, cores, desc = cpu_port_sample(inp, budget_s=max(1.0, 20.0 / max(1, args.steps)))
    line = {
        "metric": METRIC, "impl": "reference", "value": gbs, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp8e4m3 x e2m1 -> fp32 acc -> bf16", "data": "synthetic",
        "config": {"workload": cfg_name, "parallelism": "cpu"},
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": cores, "kind": "port", "sample": desc},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c1", choices=["c1", "c2", "c3"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args, args.config)
        return

    import consumer_deep_gemm as cdg
    from consumer_deep_gemm import native, synthetic

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    assert args.warmup >= 3, "at least 3 warm-up steps"

    cfg = synthetic.CONFIGS[args.config]
    inp = synthetic.make_inputs(cfg, device=dev, seed=rank)
    a, sa, b, sb, ids = inp["a"], inp["sa"], inp["b"], inp["sb"], inp["m_indices"]
    atoms = cdg.transform_sf_into_required_layout(sb, num_groups=b.shape[0], recipe=(1, 32))
    d = torch.empty(a.shape[0], b.shape[1], dtype=torch.bfloat16, device=dev)
    nbytes, flops, e_act = algorithmic(inp)
    ext = native.require()

    def call():
        cdg.m_grouped_fp8_fp4_gemm_nt_contiguous((a, sa), (b, atoms), d, ids, recipe_a=(1, 128), recipe_b=(1, 32))

    stream = torch.cuda.current_stream(dev)
    sampler = ClockSampler(local)
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize(dev)

    # ---------------------------------------------------------------- device-resident timing
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for s, e in kev:  # materialise the raw event handles
        s.record(stream)
        e.record(stream)
    torch.cuda.synchronize(dev)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps):
        ext.set_profile_events(kev[i][0].cuda_event, kev[i][1].cuda_event)
        call()
    ext.set_profile_events(0, 0)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    if dist:
        dist.barrier()
    ms = t0.elapsed_time(t1) / args.steps
    kernel_ms = statistics.fmean(s.elapsed_time(e) for s, e in kev)

    # ---------------------------------------------------------------- end to end from pinned host memory
    h_a, h_sa, h_ids = a.cpu().pin_memory(), sa.cpu().pin_memory(), ids.cpu().pin_memory()
    h_d = torch.empty(d.shape, dtype=d.dtype).pin_memory()
    a2, sa2, ids2 = torch.empty_like(a), torch.empty_like(sa), torch.empty_like(ids)

    def e2e_call():
        a2.copy_(h_a, non_blocking=True)
        sa2.copy_(h_sa, non_blocking=True)
        ids2.copy_(h_ids, non_blocking=True)
        cdg.m_grouped_fp8_fp4_gemm_nt_contiguous((a2, sa2), (b, atoms), d, ids2, recipe_a=(1, 128), recipe_b=(1, 32))
        h_d.copy_(d, non_blocking=True)

    for _ in range(args.warmup):
        e2e_call()
    torch.cuda.synchronize(dev)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    t0.record(stream)
    for _ in range(args.steps):
        e2e_call()
    t1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = t0.elapsed_time(t1) / args.steps
    clocks = sampler.stop()
    h2d = h_a.numel() * h_a.element_size() + h_sa.numel() * 4 + h_ids.numel() * h_ids.element_size()
    d2h = h_d.numel() * h_d.element_size()

    # max over ranks of the device times
    if dist:
        t = torch.tensor([ms, e2e_ms, kernel_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms, kernel_ms = t.tolist()
    if rank != 0:
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return

    hbm_peak, _, peak_src = measured_peaks()
    gbs = nbytes * world / (ms * 1e-3) / 1e9
    achieved = nbytes / (kernel_ms * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp8e4m3 x e2m1 -> fp32 acc -> bf16", "data": "synthetic",
        "config": {"workload": cfg.name, "experts": cfg.num_experts, "k": cfg.k, "n": cfg.n,
                   "routed_rows": inp["rows"], "m_pad": inp["m_pad"], "active_experts": e_act,
                   "parallelism": f"replicas{world}" if world > 1 else "single",
                   "l2": "inputs larger than L2 (weights %.2f GB)" % (b.numel() / 1e9)},
        "tflops": flops * world / (ms * 1e-3) / 1e12,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "traffic": None, "peak_source": peak_src,
                     "kernel_ms": kernel_ms, "algorithmic_bytes": nbytes},
        "e2e": {"value": nbytes * world / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
        "gpu_launches": LAUNCHES_PER_CALL * args.steps,
        "clocks": clocks,
    }
    if world == 1 and not args.no_cpu_baseline:
        v, cores, desc = cpu_port_sample(inp)
        line["cpu_baseline"] = {"value": v, "unit": "GB/s", "cores": cores, "kind": "port", "sample": desc}
    print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
