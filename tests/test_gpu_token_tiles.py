"""GPU parity of the wide-block paths on hand-made routings (CTA-pair path, N % 256 == 0).

Wide blocks with FP32 activation scales run the plane kernel on token tiles: the prep
kernel joins the consecutive wide blocks of one expert into runs and cuts each run into
tiles of at most 112 rows, which may cross block boundaries; the last block of an expert
that spans several blocks joins the wide class whatever its row count.  With power-of-two
scales the same blocks run the direct-class kernel on tiles of at most 224 rows (a tile may
then touch three blocks).  The cases below cover runs of one to five blocks, tiles crossing
one or two block boundaries, runs that end one row into a block, experts without rows, odd
numbers of 128-wide K steps (a partial pipeline stage and a partial scale-atom stage) and a
masked layout whose groups span blocks.  All
outputs are compared with the CPU oracle over every row, with the golden cases'
tolerances; rows outside every group must be exact zeros.
"""

import pytest
import torch

import cabi
from deep_gemm.utils.math import per_block_cast_to_fp8
from consumer_deep_gemm import synthetic
from metrics import TOL_NORMWISE, TOL_ROW_L2, errors
from oracle import cdg_oracle as oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _contiguous(counts, k, pow2, seed):
    """Contiguous layout (groups padded to 128 rows) with the given rows per expert."""
    g = torch.Generator().manual_seed(seed)
    ids = []
    for e, n in enumerate(counts):
        pad = (n + 127) // 128 * 128
        ids += [e] * n + [-1] * (pad - n)
    ids = torch.tensor(ids, dtype=torch.int32)
    m = ids.numel()
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).float()
    a, sa = per_block_cast_to_fp8(x)
    if pow2:
        sa = torch.exp2(torch.ceil(torch.log2(sa)))
        a = (x.view(m, k // 128, 128) / sa.unsqueeze(-1)).view(m, k).to(torch.float8_e4m3fn)
    a.view(torch.uint8)[ids < 0] = 0
    sa[ids < 0] = 1.0
    return a, sa, ids


def _check(a, sa, b, sb, ids, masked=False):
    m, n = a.shape[0], b.shape[1]
    ref = torch.empty(m, n, dtype=torch.bfloat16)
    if masked:
        oracle.m_grouped_fp8_fp4_gemm_nt_masked((a, sa), (b, sb), ref, ids)
        rows = torch.zeros(m, dtype=torch.bool)
        seg = m // b.shape[0]
        for gi, c in enumerate(ids.tolist()):
            rows[gi * seg:gi * seg + min(c, seg)] = True
    else:
        oracle.m_grouped_fp8_fp4_gemm_nt_contiguous((a, sa), (b, sb), ref, ids)
        rows = ids >= 0
    d = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=DEV)
    ws = cabi.gemm(a.to(DEV), sa.to(DEV), b.to(DEV), sb.to(DEV), d, ids.to(DEV), masked=masked)
    torch.cuda.synchronize()
    out = d.cpu()
    assert not torch.isnan(out).any(), "rows left unwritten"
    assert bool((out[~rows] == 0).all()), "rows outside every group must be zero"
    nw, rl2 = errors(out, ref, rows)
    assert nw <= TOL_NORMWISE and rl2 <= TOL_ROW_L2, (nw, rl2)
    return cabi.block_classes(ws)


@pytest.mark.parametrize("k", [384, 640, 1024], ids=["k384", "k640", "k1024"])
@pytest.mark.parametrize("pow2", [False, True], ids=["planes", "direct"])
def test_runs_across_blocks(k, pow2):
    # rows per expert: three blocks (tiles cross both block boundaries), two blocks ending one
    # row into the second, one wide block, a tail of 5 rows after a full block, no rows, one row
    counts = [300, 129, 40, 133, 0, 1]
    a, sa, ids = _contiguous(counts, k, pow2, seed=k)
    b, sb = synthetic.make_weights(len(counts), 512, k, "cpu", seed=3)
    cls = _check(a, sa, b, sb, ids)
    if pow2:
        assert cls["wide_direct"] >= 6 and cls["wide"] == 0, cls
    else:
        # the tail blocks (1 and 5 rows) of multi-block experts are wide too
        assert cls["wide"] == 8 and cls["wide_direct"] == 0, cls


@pytest.mark.parametrize("k", [512, 1152], ids=["k512", "k1152"])
@pytest.mark.parametrize("pow2", [False, True], ids=["planes", "direct"])
def test_long_runs(k, pow2):
    # five blocks of one expert (direct tiles of 224 rows: the middle one touches three blocks),
    # then runs of 449 and 257 rows
    counts = [640, 449, 257]
    a, sa, ids = _contiguous(counts, k, pow2, seed=k + 1)
    b, sb = synthetic.make_weights(len(counts), 256, k, "cpu", seed=4)
    cls = _check(a, sa, b, sb, ids)
    assert cls["wide_direct" if pow2 else "wide"] == 5 + 4 + 3, cls


@pytest.mark.parametrize("pow2", [False, True], ids=["planes", "direct"])
def test_masked_groups_span_blocks(pow2):
    # masked layout: 3 groups of 300 rows each (blocks of 128, 128 and 44 rows per group)
    e, seg, k = 3, 300, 512
    counts = torch.tensor([300, 200, 129], dtype=torch.int32)
    g = torch.Generator().manual_seed(11)
    x = torch.randn(e * seg, k, generator=g).to(torch.bfloat16).float()
    a, sa = per_block_cast_to_fp8(x)
    if pow2:
        sa = torch.exp2(torch.ceil(torch.log2(sa)))
        a = (x.view(e * seg, k // 128, 128) / sa.unsqueeze(-1)).view(e * seg, k).to(torch.float8_e4m3fn)
    b, sb = synthetic.make_weights(e, 256, k, "cpu", seed=5)
    cls = _check(a, sa, b, sb, counts, masked=True)
    assert cls["wide_direct" if pow2 else "wide"] >= 6, cls


@pytest.mark.parametrize("k", [512, 1152], ids=["k512", "k1152"])
def test_direct_and_plane_blocks_within_one_expert(k):
    # power-of-two scales everywhere except one row of expert 0's second block and one row of
    # expert 1's last block: those blocks take the plane kernel, which splits the experts'
    # runs of direct blocks around them (direct | planes | direct, and direct ... | planes)
    counts = [384, 300, 200]
    a, sa, ids = _contiguous(counts, k, True, seed=k + 7)
    for r in (128 + 5, 384 + 256 + 10):  # rows in expert 0's block 1 and expert 1's block 2
        sa[r, 0] *= 1.5
    b, sb = synthetic.make_weights(len(counts), 256, k, "cpu", seed=6)
    cls = _check(a, sa, b, sb, ids)
    # expert 0: blocks 0, 2 direct, 1 planes; expert 1: blocks 0, 1 direct, 2 planes (tail of 44
    # rows); expert 2: two direct blocks (the 72-row tail joins the wide class)
    assert cls["wide"] == 2 and cls["wide_direct"] == 2 + 2 + 2, cls
