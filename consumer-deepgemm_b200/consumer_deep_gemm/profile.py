"""Per-call timing of the public entry points: ``CDG_PROFILE=1`` (reference:
consumer_deep_gemm/__init__.py:58-114).

With ``CDG_PROFILE=1`` in the environment at import time, every public function in
``TARGETS`` is wrapped; a summary table (calls, total and average time per function)
is printed every ``CDG_PROFILE_INTERVAL`` calls (default 10).

The reference brackets each call with ``torch.cuda.synchronize()`` and a host clock,
which serialises the caller with the GPU.  Here a call records two CUDA events on the
current stream and returns at once; the events are resolved when a table is printed
(the only synchronisation, on the last event).  Without a GPU (or when the call's
tensors are not on one) the host clock around the call is used instead.
"""

from __future__ import annotations

import functools
import os
import sys
import time
from collections import defaultdict

import torch

TARGETS = (
    "m_grouped_fp8_fp4_gemm_nt_contiguous",
    "m_grouped_fp8_fp4_gemm_nt_masked",
    "transform_sf_into_required_layout",
    "transform_weights_for_mega_moe",
)


class Profiler:
    def __init__(self, interval: int = 10, out=None):
        self.interval = max(1, int(interval))
        self.out = out or sys.stdout
        self.calls = 0
        self.host = defaultdict(lambda: [0, 0.0])  # name -> [calls, seconds] (host-timed calls)
        self.pending = []                          # (name, start event, end event), unresolved
        self.device = defaultdict(lambda: [0, 0.0])  # name -> [calls, seconds] (resolved events)

    def wrap(self, fn, name: str):
        @functools.wraps(fn)
        def wrapper(*args, **kwargs):
            use_events = torch.cuda.is_available() and _on_gpu(args, kwargs)
            if use_events:
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record()
                result = fn(*args, **kwargs)
                end.record()
                self.pending.append((name, start, end))
            else:
                t0 = time.perf_counter()
                result = fn(*args, **kwargs)
                stats = self.host[name]
                stats[0] += 1
                stats[1] += time.perf_counter() - t0
            self.calls += 1
            if self.calls % self.interval == 0:
                self.report()
            return result

        return wrapper

    def resolve(self):
        if self.pending:
            self.pending[-1][2].synchronize()
            for name, start, end in self.pending:
                stats = self.device[name]
                stats[0] += 1
                stats[1] += start.elapsed_time(end) * 1e-3
            self.pending.clear()

    def stats(self) -> dict:
        """{name: (calls, total seconds)} over every call so far."""
        self.resolve()
        merged = defaultdict(lambda: [0, 0.0])
        for table in (self.host, self.device):
            for name, (c, t) in table.items():
                merged[name][0] += c
                merged[name][1] += t
        return {k: (v[0], v[1]) for k, v in merged.items()}

    def report(self):
        stats = self.stats()
        print(f"\n=== CDG Profile ({self.calls} calls) ===", file=self.out)
        for name, (c, t) in sorted(stats.items(), key=lambda kv: -kv[1][1]):
            if c:
                print(f"  {name:50s}  calls={c:6d}  total={t:8.4f}s  avg={t / c * 1e3:8.3f}ms", file=self.out)
        print(f"  {'TOTAL':50s}  calls={sum(c for c, _ in stats.values()):6d}  "
              f"total={sum(t for _, t in stats.values()):8.4f}s\n", file=self.out)


def _on_gpu(args, kwargs) -> bool:
    def first_tensor(v):
        if isinstance(v, torch.Tensor):
            return v
        if isinstance(v, (tuple, list)):
            for x in v:
                t = first_tensor(x)
                if t is not None:
                    return t
        return None

    for v in list(args) + list(kwargs.values()):
        t = first_tensor(v)
        if t is not None:
            return t.is_cuda
    return False


def install(module, names=TARGETS, interval: int | None = None, out=None) -> Profiler:
    """Wrap `module`'s functions `names` with a new Profiler and return it."""
    if interval is None:
        interval = int(os.environ.get("CDG_PROFILE_INTERVAL", "10"))
    prof = Profiler(interval, out)
    for name in names:
        fn = getattr(module, name, None)
        if callable(fn):
            setattr(module, name, prof.wrap(fn, name))
    return prof
