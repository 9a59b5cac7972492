#!/usr/bin/env python
"""Benchmark of the grouped FP8 x MXFP4 MoE GEMM (m_grouped_fp8_fp4_gemm_nt_contiguous).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c4|c4u|c1|c2|c3|c2u|c3u|c1-ep]
                    [--impl ours|reference]

Workloads (seeded synthetic data with the configs' shapes and distributions,
consumer_deep_gemm.synthetic; weights transformed once at load and resident):

* default, any N (N > 1 launched by torchrun): c4, the expert-parallel MoE layer
  FC1 -> SiLU-mul + FP8 requant -> FC2 around two grouped GEMMs, 32768 tokens x top-8
  split evenly over the ranks, E=256 experts sharded over the ranks, hidden 4096,
  intermediate 2048.  One step = one forward of the layer: on one rank the tokens are
  quantised straight into the contiguous layout; on N ranks the library's peer-memory
  exchange moves the rows over NVLink (dispatch and return stores straight into the
  other GPUs' windows, no collective and no host synchronisation on the data path).
  Strong scaling: the whole job is fixed, value = its FLOPs / step time (max over ranks).
  At N = 1 the line also carries `workloads`: the GEMM alone on c1 (decode, HBM-bound),
  c2 and c3 (prefill, tensor-bound), each with its own time, roofline and CPU baseline.
* --config c1|c2|c3|c2u|c3u (N = 1): the public GEMM call alone on that config.
* --config c4u: c4 with power-of-two (UE8M0) activation scales.
* --config c1-ep: each rank a c1-sized decode batch (64 tokens x top-8, FC1 only), experts
  sharded; weak scaling, GB/s.

One JSON line on rank 0.  `value` = algorithmic FLOPs (bytes for the decode configs) of the
whole job per step / device time of K steps (CUDA events, max over ranks).  `e2e` times the
same steps through the public API with the step's inputs copied from pinned host memory and
its result copied back.  `roofline` relates the dominant kernel's own time (CUDA events the
library records around its tensor-core kernels) to the measured peaks.  `parity` compares
sampled output rows with a float32 reference of the same computation (below), outside the
timed region; a failed check fails the run.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import sys
import threading
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
# library kernels of one layer step besides its two GEMM calls: one rank: count, quantise into
# the layout, SiLU-mul requant, unpermute + combine; N ranks: dispatch, permute, SiLU-mul
# requant, return, combine
LAYER_LAUNCHES = {True: 4, False: 5}
# DRAM bytes (read + write) of one GEMM call's dominant kernel per workload, from the ncu
# captures summarised under profiles/ (absent: no capture of the current kernels yet).
NCU_TRAFFIC = {
    "c1": 2.008183e9 + 0.223044e9,  # cdg_gemm_pair_kernel<16, 4>: profiles/cdg_gemm_pair_kernel16_c1_decode.md
    "c2": 1.427530e9 + 0.654704e9,  # cdg_gemm_planes_kernel: profiles/cdg_gemm_planes_kernel_c2_prefill.md
    "c2u": 1.281316e9 + 0.648415e9,  # cdg_gemm_direct_kernel: profiles/cdg_gemm_direct_kernel_c2u_prefill.md
    "c3": 3.371419e9 + 1.185789e9,  # cdg_gemm_planes_kernel: profiles/cdg_gemm_planes_kernel_c3_prefill.md
}
LAYER_TOL = 1e-2  # end-to-end layer tolerance (normwise and per-row L2), see parity_layer


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
    """(HBM GB/s, BF16 TFLOP/s burst, BF16 TFLOP/s sustained, source)."""
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return (float(p["hbm_gbs"]), float(p["bf16_tflops"]), float(p.get("bf16_tflops_sustained", 0.0)) or None,
                "measured")
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


# ------------------------------------------------------------------------------------ clocks
_REASON_BITS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
                0x80: "hw_power_brake_slowdown"}


def _nvml_reader(device_index: int):
    """A function returning (sm_mhz, max_sm_mhz, power_w, util_pct, reasons_mask) of the CUDA
    device `device_index` through NVML (matched by UUID), or None when NVML is unavailable."""
    try:
        import pynvml

        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(device_index).uuid)
        h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)

        def read():
            return (pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM), max_mhz,
                    pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0, pynvml.nvmlDeviceGetUtilizationRates(h).gpu,
                    int(reasons(h)))
        read()
        return read
    except Exception:
        return None


class ClockSampler:
    """SM clock, power and clock-event reasons sampled every 20 ms (NVML, read only) by a
    background thread while the benchmark runs; stop(window) reports the samples taken inside
    the timed region (host wall-clock window of the timed steps, widened by one period), else
    the samples under load."""

    PERIOD_S = 0.02

    def __init__(self, device_index: int | None = None, reader=None):
        self.samples = []  # (t, sm_mhz, max_mhz, power_w, util, reasons_mask)
        self.reader = reader if reader is not None else (_nvml_reader(device_index) if device_index is not None
                                                          else None)
        self._stop = threading.Event()
        self.thread = None
        if self.reader is not None:
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append((time.time(), *self.reader()))
            except Exception:
                pass
            self._stop.wait(self.PERIOD_S)

    def stop(self, window=None):
        self._stop.set()
        if self.thread is not None:
            self.thread.join(timeout=2)
        rows = list(self.samples)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        chosen, where = [], "timed region"
        if window is not None:
            pad = self.PERIOD_S
            chosen = [r for r in rows if window[0] - pad <= r[0] <= window[1] + pad]
        if not chosen:
            chosen, where = [r for r in rows if r[4] >= 50] or rows, "samples under load (none in the timed region)"
        reasons = sorted({name for r in chosen for bit, name in _REASON_BITS.items() if r[5] & bit})
        return {"sm_mhz": statistics.median(r[1] for r in chosen), "sm_max_mhz": max(r[2] for r in rows),
                "power_w_max": max(r[3] for r in chosen), "samples": len(chosen), "sampled": where,
                "reasons": reasons}


# ------------------------------------------------------------------------------------ CPU baselines
_REF_PKG = os.path.join(HERE, "baseline", "_ref", "consumer_deep_gemm")
_REF_MATH = os.path.join(HERE, "baseline", "_ref", "deep_gemm", "utils", "math.py")
_CPU_IMPL = None


def cpu_impl():
    """The CPU implementation of the path that the CPU baselines and the reference arm time.

    When the reference is installed under baseline/_ref (pip --target, pure Python), its own
    CPU path is loaded from there under private module names, so that it cannot collide with
    this repository's package of the same name: the GEMM is the reference's dequant + FP32 mm
    per active expert, `_m_grouped_fp8_fp4_dequant_mm_nt` (consumer_deep_gemm/gemm.py:411-464;
    its public entry, gemm.py:467-470, needs Triton and a GPU), and the activation quantisation
    is its `per_block_cast_to_fp8` (deep_gemm/utils/math.py:21-37); kind "reference".  Without
    the install, the oracle's restatement of the same functions; kind "port".
    Returns {"gemm": fn(a, b, d, m_indices), "quant": fn(x) -> (fp8, scale), "kind": ...}.
    """
    global _CPU_IMPL
    if _CPU_IMPL is not None:
        return _CPU_IMPL
    why = "no reference install under baseline/_ref"
    if os.path.isfile(os.path.join(_REF_PKG, "gemm.py")) and os.path.isfile(_REF_MATH):
        try:
            import importlib.util

            spec = importlib.util.spec_from_file_location("_cdg_reference", os.path.join(_REF_PKG, "__init__.py"),
                                                          submodule_search_locations=[_REF_PKG])
            pkg = importlib.util.module_from_spec(spec)
            sys.modules[spec.name] = pkg
            spec.loader.exec_module(pkg)
            mspec = importlib.util.spec_from_file_location("_cdg_reference_math", _REF_MATH)
            rmath = importlib.util.module_from_spec(mspec)
            mspec.loader.exec_module(rmath)
            _CPU_IMPL = {"gemm": pkg.gemm._m_grouped_fp8_fp4_dequant_mm_nt, "quant": rmath.per_block_cast_to_fp8,
                         "kind": "reference"}
            return _CPU_IMPL
        except Exception as e:  # a broken install falls back to the port, and the line says why
            sys.modules.pop("_cdg_reference", None)
            why = f"baseline/_ref failed to import ({type(e).__name__}: {e})"
    from deep_gemm.utils.math import per_block_cast_to_fp8
    from oracle import cdg_oracle as oracle

    _CPU_IMPL = {"gemm": oracle.m_grouped_fp8_fp4_gemm_nt_contiguous, "quant": per_block_cast_to_fp8,
                 "kind": "port", "why": why}
    return _CPU_IMPL


def _impl_name(impl):
    return ("reference's own _m_grouped_fp8_fp4_dequant_mm_nt (baseline/_ref)" if impl["kind"] == "reference"
            else f"oracle port of the reference's GEMM ({impl['why']})")


def cpu_port_sample(inp, budget_s: float = 4.0, calls: int = 3, warmup: int = 0):
    """Time the CPU implementation (`cpu_impl`) of the GEMM on a bounded sample.

    The sample is the routed rows of the first few active experts, grown until
    one call takes about `budget_s`.  Returns ({"GB/s": .., "TFLOP/s": ..}, cores,
    description), rates of the median call.
    """
    impl = cpu_impl()
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
        impl["gemm"]((a[rows], sa[rows]), (b, sb), d, sub[ids[rows].long()])
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
    desc = (f"{cfg.name}: {r} routed rows of {n_exp} of {experts.numel()} active experts through the "
            f"{_impl_name(impl)}, median of {len(times)} calls ({dt:.2f} s each), "
            f"torch CPU threads={torch.get_num_threads()}")
    rates = {"GB/s": nbytes / dt / 1e9, "TFLOP/s": 2.0 * r * cfg.n * cfg.k / dt / 1e12}
    return rates, torch.get_num_threads(), desc


def cpu_layer_sample(x, ids, w1, s1, w2, s2, ue8m0=False, budget_s: float = 4.0, calls: int = 3, warmup: int = 0):
    """Time the CPU implementation (`cpu_impl`) of the MoE layer (its grouped GEMM for FC1 and
    FC2, its 1x128 quantisation and a torch SiLU-mul between them) on the first tokens of a
    batch, grown until one call takes about `budget_s`.  Weights are fetched per call for the
    experts the sample touches.  Returns (TFLOP/s of the median call, cores, description)."""
    impl = cpu_impl()
    torch.set_num_threads(os.cpu_count() or 1)
    I2, H = w1.shape[1], x.shape[1]
    inter = w2.shape[2] * 2
    ids = ids.cpu()

    def quant(v):
        return _quant_pow2(v) if ue8m0 else impl["quant"](v.float())

    def run(n_tok):
        tids = ids[:n_tok]
        experts = torch.unique(tids.flatten())
        sel = experts.to(w1.device)
        b1, b1s, b2, b2s = w1[sel].cpu(), s1[sel].cpu(), w2[sel].cpu(), s2[sel].cpu()
        local = torch.searchsorted(experts, tids.flatten())
        order = torch.argsort(local, stable=True)
        rows_tok = (torch.arange(n_tok).repeat_interleave(tids.shape[1]))[order]
        m_idx = local[order].to(torch.int32)
        xs = x[:n_tok].cpu()
        t0 = time.perf_counter()
        q, s = quant(xs)
        h = torch.empty(rows_tok.numel(), I2, dtype=torch.bfloat16)
        impl["gemm"]((q[rows_tok], s[rows_tok]), (b1, b1s), h, m_idx)
        v = torch.nn.functional.silu(h[:, :inter].float()) * h[:, inter:].float()
        q2, s2_ = quant(v)
        y = torch.empty(rows_tok.numel(), H, dtype=torch.bfloat16)
        impl["gemm"]((q2, s2_), (b2, b2s), y, m_idx)
        dt = time.perf_counter() - t0
        return dt, rows_tok.numel(), experts.numel()

    dt, _, _ = run(1)
    n_tok = max(1, min(x.shape[0], int(budget_s / max(dt, 1e-3))))
    for _ in range(warmup):
        run(n_tok)
    times = []
    for _ in range(max(1, calls)):
        dt, rows, n_exp = run(n_tok)
        times.append(dt)
    dt = statistics.median(times)
    flops = 2.0 * rows * (I2 * H + H * inter)
    desc = (f"c4 layer: {n_tok} tokens ({rows} routed rows over {n_exp} experts), FC1 + SiLU-mul requant + FC2 "
            f"with the {_impl_name(impl)}, median of {len(times)} calls ({dt:.2f} s each), "
            f"torch CPU threads={torch.get_num_threads()}")
    return flops / dt / 1e12, torch.get_num_threads(), desc


def _layer_inputs(dev, rank, world, ue8m0=False):
    """A rank's c4 tokens, routing and shard of the FC1 / FC2 expert weights."""
    from consumer_deep_gemm import synthetic

    c1 = synthetic.CONFIGS["c4_fc1"]
    c2 = synthetic.CONFIGS["c4_fc2"]
    tokens = c1.tokens // world
    x, ids, w, b1, s1 = _ep_inputs(c1, dev, rank, world, tokens)
    b2, s2 = synthetic.make_weights(c1.num_experts // world, c2.n, c2.k, dev, seed=200 + rank)
    return c1, c2, x, ids, w, b1, s1, b2, s2


def run_reference(args):
    """The reference's CPU path (`cpu_impl`: its own code from baseline/_ref when installed, else
    the oracle port) on rank 0, with all host threads: each step is a bounded sample."""
    from consumer_deep_gemm import synthetic

    if int(os.environ.get("RANK", "0")) != 0:
        return
    cfg_name = args.config or "c4"
    # K timed samples after W warm-up ones, about 60 s of CPU work in all
    budget = max(0.2, 60.0 / max(1, args.steps + args.warmup))
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    if cfg_name in ("c4", "c4u"):
        # the whole job's tokens and routing, as rank 0 of a one-rank run draws them
        _, _, x, ids, _, b1, s1, b2, s2 = _layer_inputs(dev, 0, 1)
        v, cores, desc = cpu_layer_sample(x, ids, b1, s1, b2, s2, ue8m0=cfg_name == "c4u", budget_s=budget,
                                          calls=args.steps, warmup=args.warmup)
        unit = "TFLOP/s"
        scaling = "strong"
    else:
        base = cfg_name if cfg_name in ("c1", "c2", "c3", "c2u", "c3u") else "c1"
        inp = synthetic.make_inputs(synthetic.CONFIGS[base], device="cpu", seed=0, weight_device=dev)
        rates, cores, desc = cpu_port_sample(inp, budget_s=budget, calls=args.steps, warmup=args.warmup)
        unit = "GB/s" if base == "c1" else "TFLOP/s"  # the unit of our arm's line for this workload
        v = rates[unit]
        scaling = "weak"
    line = {
        "metric": METRIC, "impl": "reference", "value": v, "unit": unit, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": scaling,
        "vs_baseline": None, "dtype": DTYPE, "data": "synthetic",
        "config": {"workload": cfg_name, "parallelism": "cpu"},
        "cpu_baseline": {"value": v, "unit": unit, "cores": cores, "kind": cpu_impl()["kind"], "sample": desc},
        "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------ checker
# Float32 reference of the layer for a few sampled tokens (the parity key of the layer's line).
# It follows the reference's arithmetic: activations dequantised as bf16(bf16(e4m3) *
# bf16(scale)) per 128 columns, E2M1 weights times 2^(s-127) rounded to BF16, FP32 products
# rounded to BF16, SiLU-mul in FP32 then the same 1x128 quantisation, the top-k sum in FP32.
# tests/test_bench_layer_reference.py pins it against the oracle-based CPU reference layer.
_E2M1 = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0)


def _deq_weight(b, s):
    """packed e2m1 [N, K/2] (low nibble = even k) + UE8M0 [N, K/32] -> BF16 [N, K]."""
    t = torch.tensor(_E2M1, dtype=torch.float32, device=b.device)
    v = torch.stack((t[(b & 15).long()], t[(b >> 4).long()]), -1).flatten(-2)
    sc = torch.exp2(s.float() - 127.0)
    return (v.view(v.shape[0], -1, 32) * sc.unsqueeze(-1)).view(v.shape[0], -1).to(torch.bfloat16)


def _deq_act(q, s):
    m, k = q.shape
    return (q.view(m, k // 128, 128).to(torch.bfloat16) * s.to(torch.bfloat16).unsqueeze(-1)).view(m, k)


def _quant_pow2(x):
    """1x128 e4m3 with power-of-two scales: amax/448 (amax >= 1e-12) rounded up to a power of two."""
    m, k = x.shape
    xv = x.float().view(m, k // 128, 128)
    s = xv.abs().amax(dim=2).clamp(min=1e-12) / 448.0
    mant, ex = torch.frexp(s)
    s2 = torch.where(mant == 0.5, s, torch.ldexp(torch.ones_like(s), ex))
    return (xv / s2.unsqueeze(-1)).to(torch.float8_e4m3fn).view(m, k), s2


def layer_reference(x, ids, w, b1, s1, b2, s2, ue8m0=False):
    """y [T, H] BF16 of the MoE layer for tokens x [T, H] with global expert ids [T, k] and
    weights [T, k]; b1/s1, b2/s2 are all experts' packed weights and row-major UE8M0 scales."""
    from deep_gemm.utils.math import per_block_cast_to_fp8

    def quant(v):
        return _quant_pow2(v) if ue8m0 else per_block_cast_to_fp8(v.float())

    inter = b2.shape[2] * 2
    q, s = quant(x)
    xa = _deq_act(q, s).float()
    y = torch.zeros(x.shape[0], b2.shape[1], dtype=torch.float32, device=x.device)
    for e in torch.unique(ids.flatten()).tolist():
        tok, slot = (ids == e).nonzero(as_tuple=True)
        h = (xa[tok] @ _deq_weight(b1[e], s1[e]).float().t()).to(torch.bfloat16)
        v = torch.nn.functional.silu(h[:, :inter].float()) * h[:, inter:].float()
        q2, sc2 = quant(v)
        o = (_deq_act(q2, sc2).float() @ _deq_weight(b2[e], s2[e]).float().t()).to(torch.bfloat16)
        y.index_put_((tok,), w[tok, slot].float().unsqueeze(1) * o.float(), accumulate=True)
    return y.to(torch.bfloat16)


def _row_errors(out, ref):
    o, r = out.float(), ref.float()
    nw = ((o - r).abs().max() / r.abs().max().clamp(min=1e-30)).item()
    rl2 = ((o - r).norm(dim=1) / r.norm(dim=1).clamp(min=1e-30)).max().item()
    return nw, rl2


def parity_layer(dist, dev, world, rank, x, ids, w, y, b1, s1, b2, s2, ue8m0):
    """Compare sampled tokens of every rank's output with layer_reference (on rank 0).

    Every rank contributes max(2, 16 // N) seeded tokens; rank 0 gathers them, their outputs
    and all ranks' expert weights, and checks max |y - ref| / max |ref| and the per-row
    relative L2 against LAYER_TOL.  The two GEMMs meet 2e-3 per row each (tests); end to
    end the bound is looser because the e4m3 requantisation between them turns last-bit
    differences of FC1 into whole e4m3 steps of single FC2 inputs.
    """
    per = max(2, 16 // world)
    g = torch.Generator().manual_seed(1234 + rank)
    pick = torch.randperm(x.shape[0], generator=g)[:per].to(dev)
    mine = [x[pick], ids[pick].to(torch.int64), w[pick].float(), y[pick]]
    if dist is not None:
        gathered = []
        for t in mine:
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t.contiguous())
            gathered.append(torch.cat(parts))
        weights = []
        for t in (b1, s1, b2, s2):
            out = torch.empty((world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=dev)
            dist.all_gather_into_tensor(out, t.contiguous())
            weights.append(out)
    else:
        gathered, weights = mine, [b1, s1, b2, s2]
    result = None
    if rank == 0:
        xs, idss, ws, ys = gathered
        ref = layer_reference(xs, idss, ws, *weights, ue8m0=ue8m0)
        nw, rl2 = _row_errors(ys, ref)
        e_loc = weights[0].shape[0] // world
        covered = len(set((idss // e_loc).flatten().tolist()))
        result = {"normwise": nw, "row_l2": rl2, "rows": int(xs.shape[0]), "ranks_sampled": world,
                  "ranks_covered_by_routing": covered, "tolerance": LAYER_TOL,
                  "reference": "float32 layer reference (bench.layer_reference) on the GPU",
                  "ok": bool(nw <= LAYER_TOL and rl2 <= LAYER_TOL and covered == world)}
    del weights
    torch.cuda.empty_cache()
    return result


# ------------------------------------------------------------------------------------ timing
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


class PhaseTimer:
    """Per-phase device time of eager layer steps (MoELayer.on_phase), and the FC1 GEMM's
    tensor-core kernels alone (the library's profile events around that one call)."""

    def __init__(self, layer, steps):
        from consumer_deep_gemm import native

        self.ext = native.require()
        self.layer = layer
        self.steps = steps
        self.marks = [[] for _ in range(steps)]
        self.fc1 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                    for _ in range(steps)]
        for s, e in self.fc1:  # materialise the raw event handles the library records
            s.record()
            e.record()
        torch.cuda.synchronize()
        self.i = 0

    def _hook(self, name):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self.marks[self.i].append((name, ev))
        if name in ("dispatch", "permute") and not (name == "dispatch" and self.layer.world > 1):
            s, e = self.fc1[self.i]
            self.ext.set_profile_events(s.cuda_event, e.cuda_event)  # around the next GEMM call: FC1
        elif name == "fc1":
            self.ext.set_profile_events(0, 0)

    def run(self, step):
        self.layer.on_phase = self._hook
        try:
            for self.i in range(self.steps):
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                self.marks[self.i].append(("start", ev))
                step()
        finally:
            self.layer.on_phase = None
            self.ext.set_profile_events(0, 0)
        torch.cuda.synchronize()
        phases = {}
        for m in self.marks:
            for (_, a), (name, b) in zip(m[:-1], m[1:]):
                phases.setdefault(name, []).append(a.elapsed_time(b))
        fc1_ms = statistics.fmean(s.elapsed_time(e) for s, e in self.fc1)
        return {k: statistics.fmean(v) for k, v in phases.items()}, fc1_ms


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default=None, choices=["c1", "c2", "c3", "c4", "c4u", "c2u", "c3u", "c1-ep"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-workloads", action="store_true", help="N = 1 default: skip the GEMM-alone workloads")
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
    ok = True
    try:
        cfg = args.config or "c4"
        if cfg in ("c4", "c4u"):
            line = bench_layer(args, dev, world, rank, dist, cfg)
            if world == 1 and args.config is None and not args.no_workloads:
                torch.cuda.empty_cache()
                line["workloads"] = {}
                for c in ("c1", "c2", "c3"):
                    sub = bench_gemm(args, dev, c)
                    line["workloads"][c] = {k: sub[k] for k in ("value", "unit", "ms_per_step", "roofline",
                                                                "roofline_other", "config", "cpu_baseline", "e2e",
                                                                "clocks", "gpu_launches") if k in sub}
                    torch.cuda.empty_cache()
        elif cfg == "c1-ep":
            line = bench_ep_decode(args, dev, world, rank, dist)
        else:
            if world > 1:
                raise SystemExit("--config c1/c2/c3/c2u/c3u run on one GPU; use c4, c4u or c1-ep with --gpus N")
            line = bench_gemm(args, dev, cfg)
        if rank == 0:
            print(json.dumps(line), flush=True)
            ok = (line.get("parity") or {}).get("ok", True)
    finally:
        if dist:
            dist.barrier()
            dist.destroy_process_group()
    if not ok:
        print("parity check failed", file=sys.stderr, flush=True)
        sys.exit(1)


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


def _barrier(dist, dev):
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)


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
    hbm_peak, bf16_peak, _, peak_src = measured_peaks()
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
                   "algorithmic_flops": flops,
                   # FP32 activation scales: two e4m3 planes per activation on the tensor cores
                   "mma_planes": 1 if cfg.ue8m0_scales else 2,
                   "issued_frac": achieved_tf * (1 if cfg.ue8m0_scales else 2) / (2 * bf16_peak)}
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
        rates, cores, desc = cpu_port_sample(inp, budget_s=3.0)
        line["cpu_baseline"] = {"value": rates[line["unit"]], "unit": line["unit"], "cores": cores,
                                "kind": cpu_impl()["kind"],
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


def _e2e_layer(layer, x, ids, w, dev, steps, warmup):
    """End to end through the layer's public forward: every step uploads its tokens, routing and
    routing weights from pinned host memory and reads the output rows back; two buffer sets and
    two copy streams overlap step i's upload and step i-1's download with the compute."""
    h_in = [t.cpu().pin_memory() for t in (x, ids, w)]
    h_y = [torch.empty(x.shape[0], layer.out_dim, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    bufs = [[torch.empty_like(t) for t in (x, ids, w)] for _ in range(2)]
    comp = torch.cuda.current_stream(dev)
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    i = [0]

    def step():
        p = i[0] & 1
        i[0] += 1
        up.wait_event(ev_used[p])
        with torch.cuda.stream(up):
            for dst, src in zip(bufs[p], h_in):
                dst.copy_(src, non_blocking=True)
        ev_in[p].record(up)
        comp.wait_event(ev_in[p])
        comp.wait_event(ev_out[p])
        y = layer(*bufs[p])
        ev_used[p].record(comp)
        down.wait_event(ev_used[p])
        with torch.cuda.stream(down):
            h_y[p].copy_(y, non_blocking=True)
        y.record_stream(down)
        ev_out[p].record(down)

    def finish():
        comp.wait_event(ev_out[0])
        comp.wait_event(ev_out[1])

    for _ in range(warmup):
        step()
    finish()
    torch.cuda.synchronize(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(comp)
    up.wait_event(t0)
    for _ in range(steps):
        step()
    finish()  # the last step's download is inside the timed region
    t1.record(comp)
    torch.cuda.synchronize(dev)
    return t0.elapsed_time(t1) / steps, sum(t.numel() * t.element_size() for t in h_in), h_y[0].numel() * 2


def bench_layer(args, dev, world, rank, dist, cfg_name):
    """c4 / c4u: the MoE layer, 32768 tokens split over the ranks, experts sharded."""
    from consumer_deep_gemm.moe import MoELayer

    ue8m0 = cfg_name == "c4u"
    c1, c2, x, ids, w, b1, s1, b2, s2 = _layer_inputs(dev, rank, world)
    tokens = x.shape[0]
    exchange = "p2p" if world > 1 else "nccl"
    layer = MoELayer(b1, s1, b2, s2, num_experts=c1.num_experts, group=dist.group.WORLD if dist else None,
                     ue8m0=ue8m0, max_tokens_per_rank=tokens if world > 1 else None, exchange=exchange)
    e_loc = c1.num_experts // world
    mine = _global_counts(ids, c1.num_experts, dev, dist)[rank * e_loc:(rank + 1) * e_loc].cpu()
    _, f_fc1 = _local_gemm_work(mine, c1.n, c1.k)
    _, f_fc2 = _local_gemm_work(mine, c2.n, c2.k)
    job_flops = _sum_over_ranks(dist, dev, f_fc1 + f_fc2)

    sampler = ClockSampler(dev.index)
    for _ in range(args.warmup):
        layer(x, ids, w)
    # per-phase split of eager steps, and the FC1 GEMM's tensor-core kernels alone
    _barrier(dist, dev)
    phases, fc1_ms = PhaseTimer(layer, args.steps).run(lambda: layer(x, ids, w))
    # the timed steps: the layer's forward captured once in a CUDA graph and replayed (no host
    # synchronisation in the forward at any N: one rank computes its layout on the device, N
    # ranks exchange through the peer-memory windows)
    graph, y = layer.capture(x, ids, w)
    for _ in range(args.warmup):
        graph.replay()
    timer = Timed(dev, args.steps)
    _barrier(dist, dev)
    ms, _ = timer.run(graph.replay, args.steps, with_kernel_events=False)
    timed_window = timer.window
    # end to end through the public forward, host copies included
    _barrier(dist, dev)
    e2e_ms, h2d, d2h = _e2e_layer(layer, x, ids, w, dev, args.steps, args.warmup)
    clocks = sampler.stop(timed_window)
    _barrier(dist, dev)
    graph.replay()  # the checked output: one more replay on the resident inputs
    torch.cuda.synchronize(dev)
    status = layer.status()
    parity = parity_layer(dist, dev, world, rank, x, ids, w, y, b1, s1, b2, s2, ue8m0)
    del graph
    ms, e2e_ms, fc1_ms, st_max = _max_over_ranks(dist, dev, ms, e2e_ms, fc1_ms, float(status))
    names = list(phases)
    phase_max = dict(zip(names, _max_over_ranks(dist, dev, *[phases[k] for k in names])))
    _barrier(dist, dev)
    layer.close()  # after every rank's last forward
    if parity is not None:
        parity["device_status"] = int(st_max)
        parity["ok"] = parity["ok"] and st_max == 0
    _, bf16_peak, bf16_sus, peak_src = measured_peaks()
    fp8_peak = 2 * bf16_peak
    achieved = f_fc1 / (fc1_ms * 1e-3) / 1e12
    step_desc = ("quantise into the layout, FC1, SiLU-mul + requant, FC2, unpermute + combine" if world == 1 else
                 "dispatch (quantise + store into the owners' windows), permute, FC1, SiLU-mul + requant, "
                 "FC2 (its epilogue stores each row into its source's window), combine")
    return {
        "metric": METRIC, "value": job_flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": DTYPE, "data": "synthetic",
        "config": {"workload": cfg_name, "experts": c1.num_experts, "hidden": c1.k, "intermediate": c2.k,
                   "tokens": c1.tokens, "tokens_per_rank": tokens, "topk": c1.topk, "parallelism": f"ep{world}",
                   "activation_scales": "ue8m0 (power of two)" if ue8m0 else "fp32 1x128",
                   "step": step_desc,
                   "exchange": "none (one rank)" if world == 1 else
                   "peer-memory stores over NVLink into fixed-capacity windows (tokens_per_rank x topk rows per "
                   "source), release/acquire flags; no collective, no host synchronisation",
                   "timed": "the forward captured in one CUDA graph per rank, replayed",
                   "l2": "inputs larger than L2 (weights %.2f GB per rank)" % ((b1.numel() + b2.numel()) / 1e9)},
        "phases_ms": phase_max,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": fp8_peak, "unit": "TFLOP/s",
                     "frac": achieved / fp8_peak, "traffic": None, "kernel": "FC1 GEMM's tensor-core kernels",
                     "kernel_ms": fc1_ms, "algorithmic_flops": f_fc1,
                     "peak_source": f"2 x {peak_src} BF16 GEMM burst (dense FP8:BF16 = 2:1)",
                     "frac_of_sustained": (achieved / (2 * bf16_sus)) if bf16_sus else None,
                     # with FP32 activation scales the tensor cores multiply two e4m3 planes (hi, lo)
                     # per activation, twice the algorithmic MMA work: the plane path's ceiling is
                     # half the FP8 peak; issued = what the tensor pipe actually executed
                     "mma_planes": 1 if ue8m0 else 2,
                     "issued_frac": achieved * (1 if ue8m0 else 2) / fp8_peak,
                     "issued_frac_of_sustained": (achieved * (1 if ue8m0 else 2) / (2 * bf16_sus)) if bf16_sus
                     else None},
        "e2e": {"value": job_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                "copies": "per rank: its tokens, routing and weights up, its output rows down; step i's upload "
                          "overlaps step i-1's download (two buffer sets, two copy streams)"},
        "parity": parity,
        "gpu_launches": (2 * GEMM_LAUNCHES + LAYER_LAUNCHES[world == 1]) * args.steps,
        "clocks": clocks,
        **({"cpu_baseline": _layer_cpu_baseline(x, ids, b1, s1, b2, s2, ue8m0)}
           if (world == 1 and rank == 0 and not args.no_cpu_baseline) else {}),
    }


def _layer_cpu_baseline(x, ids, b1, s1, b2, s2, ue8m0):
    v, cores, desc = cpu_layer_sample(x, ids, b1, s1, b2, s2, ue8m0=ue8m0, budget_s=3.0)
    return {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": cpu_impl()["kind"], "sample": desc}


def bench_ep_decode(args, dev, world, rank, dist):
    """--config c1-ep: every rank a c1 decode batch, experts sharded, FC1 only."""
    from consumer_deep_gemm import synthetic
    from consumer_deep_gemm.moe import MoELayer

    cfg = synthetic.CONFIGS["c1"]
    x, ids, w, b, sb = _ep_inputs(cfg, dev, rank, world, cfg.tokens)
    layer = MoELayer(b, sb, num_experts=cfg.num_experts, group=dist.group.WORLD if dist else None,
                     max_tokens_per_rank=cfg.tokens if world > 1 else None, exchange="p2p" if world > 1 else "nccl")
    e_loc = cfg.num_experts // world
    mine = _global_counts(ids, cfg.num_experts, dev, dist)[rank * e_loc:(rank + 1) * e_loc].cpu()
    local_bytes, local_flops = _local_gemm_work(mine, cfg.n, cfg.k)
    job_bytes = _sum_over_ranks(dist, dev, local_bytes)
    job_flops = _sum_over_ranks(dist, dev, local_flops)

    sampler = ClockSampler(dev.index)
    for _ in range(args.warmup):
        layer(x, ids, w)
    _barrier(dist, dev)
    phases, kernel_ms = PhaseTimer(layer, args.steps).run(lambda: layer(x, ids, w))
    graph, _ = layer.capture(x, ids, w)
    for _ in range(args.warmup):
        graph.replay()
    timer = Timed(dev, args.steps)
    _barrier(dist, dev)
    ms, _ = timer.run(graph.replay, args.steps, with_kernel_events=False)
    timed_window = timer.window
    _barrier(dist, dev)
    _barrier(dist, dev)
    e2e_ms, h2d, d2h = _e2e_layer(layer, x, ids, w, dev, args.steps, args.warmup)
    clocks = sampler.stop(timed_window)
    status = layer.status()
    del graph
    ms, e2e_ms, kernel_ms, st_max = _max_over_ranks(dist, dev, ms, e2e_ms, kernel_ms, float(status))
    names = list(phases)
    phase_max = dict(zip(names, _max_over_ranks(dist, dev, *[phases[k] for k in names])))
    _barrier(dist, dev)
    layer.close()
    hbm_peak, _, _, peak_src = measured_peaks()
    achieved = local_bytes / (kernel_ms * 1e-3) / 1e9
    return {
        "metric": METRIC, "value": job_bytes / (ms * 1e-3) / 1e9, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": DTYPE, "data": "synthetic",
        "config": {"workload": "c1-ep", "experts": cfg.num_experts, "k": cfg.k, "n": cfg.n,
                   "tokens_per_rank": cfg.tokens, "topk": cfg.topk, "parallelism": f"ep{world}",
                   "step": ("quantise into the layout, FC1, unpermute + combine" if world == 1 else
                            "dispatch (quantise + store into the owners' windows), permute, FC1, return (store "
                            "into the sources' windows), combine"),
                   "exchange": "none (one rank)" if world == 1 else
                   "peer-memory stores over NVLink into fixed-capacity windows, release/acquire flags; no "
                   "collective, no host synchronisation",
                   "timed": "the forward captured in one CUDA graph per rank, replayed",
                   "l2": "weights per rank larger than L2"},
        "tflops": job_flops / (ms * 1e-3) / 1e12,
        "phases_ms": phase_max,
        "device_status": int(st_max),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "traffic": None, "peak_source": peak_src,
                     "kernel_ms": kernel_ms, "algorithmic_bytes": local_bytes, "note": "rank 0's GEMM kernels"},
        "e2e": {"value": job_bytes / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
        "gpu_launches": (GEMM_LAUNCHES + LAYER_LAUNCHES[world == 1] - 1) * args.steps,
        "clocks": clocks,
    }


if __name__ == "__main__":
    main()
