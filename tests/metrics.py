"""Error measures used by the parity tests (tolerances are stated in each test)."""

import torch

# Floating-point tolerance of the grouped GEMM against the reference's output:
# max |out - ref| / max |ref| over the routed rows, and per-row relative L2.
TOL_NORMWISE = 1e-2
TOL_ROW_L2 = 2e-3


def errors(out: torch.Tensor, ref: torch.Tensor, rows=None):
    """(normwise max relative error, max per-row relative L2) over `rows` (default all)."""
    # computed where `out` lies (full-size GPU outputs stay on the GPU)
    o = out.detach().float()
    r = ref.detach().float().to(o.device)
    if rows is not None:
        rows = rows.to(o.device) if isinstance(rows, torch.Tensor) else rows
        o, r = o[rows], r[rows]
    if r.numel() == 0:
        return 0.0, 0.0
    scale = r.abs().max().clamp(min=1e-30)
    normwise = ((o - r).abs().max() / scale).item()
    num = (o - r).norm(dim=1)
    den = r.norm(dim=1)
    nz = den > 0
    row_l2 = (num[nz] / den[nz]).max().item() if bool(nz.any()) else float(num.max())
    return normwise, row_l2
