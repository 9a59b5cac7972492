"""GPU checks of the MoE-layer kernels and of the layer itself (through the torch binding).

Tolerances:
  * FP8 row quantisation: bit-exact against per_block_cast_to_fp8 (deep_gemm/utils/math.py:21-37),
    and, with power-of-two (UE8M0) scales, against moe_ref.cast_to_fp8_pow2.
  * SiLU-mul + requant: scales within 1e-6 relative; e4m3 codes equal except where the device's
    fast exponential, reciprocal and per-block reciprocal scale and the CPU's arithmetic land on
    opposite sides of an e4m3 rounding point (at most 1 in 1000 codes, each within one e4m3 step).
  * Dispatch / permute / unpermute: exact (bytes).
  * Layer stages, each fed the device's own input of that stage: FC1 and FC2 within the
    GEMM's tolerances (max |d - ref| / max |ref| <= 1e-2, per-row relative L2 <= 2e-3) against
    the oracle; SiLU-mul + requant as above; the top-k combine within 2e-3 per row.
  * Whole layer end to end: max |y - ref| / max |ref| <= 1e-2 and per-row relative L2 <= 1e-2
    against the CPU reference layer.  The 2e-3 bound of a single GEMM cannot hold end to end:
    FC1's outputs agree with the reference's to ~1e-3, i.e. differ in the last BF16 bit for a
    fraction of elements, and the e4m3 requantisation between the GEMMs turns each such
    difference at a rounding boundary into a whole e4m3 step (2^-3 relative) of one FC2 input.
  * A peer wait that nobody satisfies gives up within its configured limit and is reported.
"""

import os
import subprocess
import sys

import pytest
import torch

from moe_ref import TorchRefOps, cast_to_fp8_pow2, make_layer_inputs, row_bytes

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ext():
    from consumer_deep_gemm import native

    return native.require()


def test_quant_fp8_rows_bit_exact():
    from deep_gemm.utils.math import per_block_cast_to_fp8

    g = torch.Generator().manual_seed(1)
    x = (torch.randn(300, 1024, generator=g) * torch.rand(300, 1, generator=g) * 10).to(torch.bfloat16)
    x[7] = 0  # all-zero row: amax clamps at 1e-12
    q, s = _ext().quant_fp8_rows(x.to(DEV))
    rq, rs = per_block_cast_to_fp8(x.float())
    assert torch.equal(q.cpu().view(torch.uint8), rq.view(torch.uint8))
    assert torch.equal(s.cpu(), rs)


def test_quant_fp8_rows_pow2_bit_exact():
    g = torch.Generator().manual_seed(11)
    x = (torch.randn(300, 1024, generator=g) * torch.rand(300, 1, generator=g) * 10).to(torch.bfloat16)
    x[7] = 0  # all-zero row: amax clamps at 1e-12
    x[9, :128] = 448.0 * 2.0 ** -3  # amax / 448 exactly a power of two: kept, not doubled
    q, s = _ext().quant_fp8_rows(x.to(DEV), ue8m0=True)
    rq, rs = cast_to_fp8_pow2(x)
    assert torch.equal(q.cpu().view(torch.uint8), rq.view(torch.uint8))
    assert torch.equal(s.cpu(), rs)
    assert float(rs[9, 0]) == 2.0 ** -3
    mant, _ = torch.frexp(s.cpu())
    assert bool((mant == 0.5).all()), "every scale is a power of two"


@pytest.mark.parametrize("ue8m0", [False, True], ids=["fp32", "ue8m0"])
@pytest.mark.parametrize("inter,offset", [(512, 0), (640, 0), (384, 0), (640, 4), (384, 1)],
                         ids=["i512", "i640", "i384", "i640_8byte", "i384_unaligned"])
def test_silu_mul_quant_matches_reference(ue8m0, inter, offset):
    # rows 16-byte aligned: four 128-column blocks per warp, eight lanes each (640 and 384: a
    # partial group); a view 4 columns in (8-byte aligned): the 8-byte path; a view one column
    # in: one block per warp with 2-byte loads
    g = torch.Generator().manual_seed(2)
    h = torch.randn(200, 2 * inter, generator=g).to(torch.bfloat16)
    if offset == 0:
        hd = h.to(DEV)
    else:
        hd = torch.zeros(200, 2 * inter + 8, dtype=torch.bfloat16, device=DEV)
        hd[:, offset:offset + 2 * inter] = h.to(DEV)
        hd = hd[:, offset:offset + 2 * inter]
    q, s = _ext().silu_mul_quant(hd, None, ue8m0)
    rq, rs = TorchRefOps().act(h, None, ue8m0)
    assert torch.allclose(s.cpu(), rs, rtol=1e-6, atol=0)
    a, b = q.cpu().view(torch.uint8).to(torch.int32), rq.view(torch.uint8).to(torch.int32)
    diff = (a != b)
    assert diff.float().mean().item() <= 1e-3
    assert ((a - b).abs()[diff] <= 1).all()


def test_dispatch_and_permute_are_exact():
    C = _ext()
    T, H, k, E = 64, 512, 4, 16
    g = torch.Generator().manual_seed(3)
    xq = torch.randint(0, 256, (T, H), dtype=torch.uint8, generator=g).to(DEV).view(torch.float8_e4m3fn)
    xs = torch.rand(T, H // 128, generator=g).to(DEV)
    ids = torch.rand(T, E, generator=g).topk(k, dim=1).indices.to(torch.int32)
    ids[3, 1] = -1  # a masked slot
    counts = C.ep_count(ids.to(DEV), E).cpu()
    ref_counts = torch.bincount(ids[ids >= 0].long(), minlength=E)
    assert torch.equal(counts.long(), ref_counts)
    rows = int(counts.sum())
    sent, send_index = C.ep_pack(xq, xs, ids.to(DEV), E, 1, torch.zeros(1, dtype=torch.int64, device=DEV), rows)
    nkb = H // 128
    assert sent.shape == (rows, C.ep_row_bytes(H)) and C.ep_row_bytes(H) == row_bytes(H)
    sent_h = sent.cpu()
    si = send_index.cpu()
    assert int(si[3 * k + 1]) == -1 and int((si >= 0).sum()) == rows
    flat = ids.flatten()
    xq_h, xs_h = xq.cpu().view(torch.uint8), xs.cpu()
    row_e = sent_h[:, H + 4 * nkb:H + 4 * nkb + 4].contiguous().view(torch.int32).flatten()
    for i in range(T * k):
        if si[i] >= 0:
            r = int(si[i])
            assert torch.equal(sent_h[r, :H], xq_h[i // k])
            assert torch.equal(sent_h[r, H:H + 4 * nkb].contiguous().view(torch.float32), xs_h[i // k])
            assert int(row_e[r]) == int(flat[i])
    aligned = (ref_counts + 127) // 128 * 128
    off = (torch.cumsum(aligned, 0) - aligned).to(DEV)
    m_pad = int(aligned.sum())
    a, sa, mi, pos = C.ep_permute(sent, H, E, off, m_pad)
    pos, mi = pos.cpu().long(), mi.cpu()
    assert torch.equal(a.cpu().view(torch.uint8)[pos], sent_h[:, :H])
    assert torch.equal(sa.cpu()[pos], sent_h[:, H:H + 4 * nkb].contiguous().view(torch.float32))
    assert torch.equal(mi[pos], row_e)
    assert int((mi >= 0).sum()) == rows
    for e in range(E):
        seg = mi[int(off[e]):int(off[e]) + int(aligned[e])]
        assert int((seg == e).sum()) == int(ref_counts[e]) and bool((seg[: int(ref_counts[e])] == e).all())
    y = torch.randn(m_pad, H, generator=g).to(torch.bfloat16).to(DEV)
    pos32 = pos.to(torch.int32).to(DEV)
    back = C.ep_unpermute(y, pos32)
    assert torch.equal(back.cpu().view(torch.int16), y.cpu()[pos].view(torch.int16))
    # weighted top-k sum: the fused unpermute + combine gives the same bits as the two steps,
    # and both agree with the CPU reference (FP32 sums in slot order)
    w = torch.rand(T, k, generator=g)
    w = (w / w.sum(1, keepdim=True)).to(DEV)
    y1 = C.ep_combine(back, send_index, w)
    y2 = C.ep_unpermute_combine(y, pos32, send_index, w)
    assert torch.equal(y1.view(torch.int16), y2.view(torch.int16))
    ref = TorchRefOps().combine(back.cpu(), si, w.cpu()).float()
    assert (y1.cpu().float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item()


def test_combine_scalar_path_matches_vector_path():
    """Rows whose length is not a multiple of 8 take the per-element path; on the same
    values its columns equal the 16-byte path's, bit for bit."""
    C = _ext()
    T, k, R, H = 40, 3, 90, 520
    g = torch.Generator().manual_seed(9)
    rows = torch.randn(R, H, generator=g).to(torch.bfloat16).to(DEV)
    send_index = torch.randint(-1, R, (T * k,), generator=g, dtype=torch.int32).to(DEV)
    w = torch.rand(T, k, generator=g).to(DEV)
    y_vec = C.ep_combine(rows, send_index, w)                       # H % 8 == 0: 16-byte path
    y_sc = C.ep_combine(rows[:, :H - 4].contiguous(), send_index, w)  # 516 columns: per element
    assert torch.equal(y_vec[:, :H - 4].view(torch.int16), y_sc.view(torch.int16))


@pytest.mark.parametrize("ue8m0", [False, True], ids=["fp32", "ue8m0"])
@pytest.mark.parametrize("xdtype", [torch.bfloat16, torch.float32], ids=["bf16", "f32"])
def test_quant_dispatch_local_exact(ue8m0, xdtype):
    """One rank: quantise straight into the contiguous layout; the rows land in any order within
    an expert's region, so each slot's row is compared with the reference's row of that slot."""
    C = _ext()
    T, H, k, E = 300, 512, 4, 12
    g = torch.Generator().manual_seed(8)
    x = torch.randn(T, H, generator=g).to(xdtype)
    ids = torch.rand(T, E, generator=g).topk(k, dim=1).indices.to(torch.int32)
    ids[5, 2] = -1  # a skipped slot
    ids[6, 0] = E   # out of range: skipped too
    counts = torch.bincount(ids[(ids >= 0) & (ids < E)].long(), minlength=E)
    aligned = (counts + 127) // 128 * 128
    off = torch.cumsum(aligned, 0) - aligned
    m_pad = int(aligned.sum())
    a, sa, mi, pos, si = C.ep_quant_dispatch_local(x.to(DEV), ids.to(DEV), E, off.to(DEV), m_pad, ue8m0)
    ra, rsa, rmi, rpos, rsi = TorchRefOps().quant_dispatch_local(x, ids, E, off, m_pad, ue8m0)
    a, sa, mi, pos, si = a.cpu().view(torch.uint8), sa.cpu(), mi.cpu(), pos.cpu(), si.cpu()
    assert torch.equal(si, rsi) and torch.equal(pos < 0, rpos < 0)
    ok = pos >= 0
    assert torch.equal(a[pos[ok].long()], ra.view(torch.uint8)[rpos[ok].long()])
    assert torch.equal(sa[pos[ok].long()], rsa[rpos[ok].long()])
    assert torch.equal(mi[pos[ok].long()], rmi[rpos[ok].long()])
    assert torch.equal(torch.sort(mi).values, torch.sort(rmi).values)  # same groups, same padding
    assert len(set(pos[ok].tolist())) == int(ok.sum())  # every slot its own row


@pytest.mark.parametrize("ue8m0", [False, True], ids=["fp32", "ue8m0"])
def test_fixed_capacity_pack_and_permute_exact(ue8m0):
    """Fused quant+pack into fixed-capacity regions, then the receive-side permute: bytes."""
    C = _ext()
    T, H, k, E, ranks = 40, 512, 2, 8, 2
    g = torch.Generator().manual_seed(5)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    ids = torch.rand(T, E, generator=g).topk(k, dim=1).indices.to(torch.int32)
    ids[7, 0] = -1  # a skipped slot
    cap = T * k
    sent, si = C.ep_quant_pack_fixed(x.to(DEV), ids.to(DEV), E, ranks, cap, ue8m0)
    ref_sent, ref_si = TorchRefOps().quant_pack_fixed(x, ids, E, ranks, cap, ue8m0)
    sent, si = sent.cpu(), si.cpu()
    nkb = H // 128
    payload = H + 4 * nkb + 4
    for d in range(ranks):  # headers: per-local-expert counts
        assert torch.equal(sent[d * (cap + 1), :4 * (E // ranks)], ref_sent[d * (cap + 1), :4 * (E // ranks)])
    assert torch.equal(si < 0, ref_si < 0)
    for i in range(T * k):  # same row content wherever the atomics placed it
        if si[i] >= 0:
            assert int(si[i]) // (cap + 1) == int(ref_si[i]) // (cap + 1)
            assert torch.equal(sent[int(si[i]), :payload], ref_sent[int(ref_si[i]), :payload])
    # the receive side of rank 0 sees region 0 of both ranks' buffers; here one buffer stands for both
    e_loc = E // ranks
    recv = torch.cat([sent[:cap + 1], sent[:cap + 1]])
    m_pad = (ranks * cap + 127 * e_loc + 127) // 128 * 128
    a, sa, mi, pos = C.ep_permute_fixed(recv.to(DEV), H, e_loc, ranks, cap, m_pad)
    ra, rsa, rmi, rpos = TorchRefOps().permute_fixed(recv, H, e_loc, ranks, cap, m_pad)
    a, sa, mi, pos = a.cpu(), sa.cpu(), mi.cpu(), pos.cpu()
    assert torch.equal(pos < 0, rpos < 0)
    valid = (pos >= 0).nonzero().flatten()
    assert torch.equal(a.view(torch.uint8)[pos[valid].long()], recv[valid, :H])
    assert torch.equal(sa[pos[valid].long()], recv[valid, H:H + 4 * nkb].contiguous().view(torch.float32))
    assert torch.equal(torch.sort(mi).values, torch.sort(rmi).values)  # same group sizes and offsets
    assert torch.equal(mi >= 0, rmi >= 0)


@pytest.mark.parametrize("ue8m0", [False, True], ids=["fp32", "ue8m0"])
def test_layer_single_gpu_matches_cpu_reference(ue8m0):
    # with ue8m0 the activations carry power-of-two scales and both GEMMs' wide blocks take the
    # direct class: 1000 tokens x top-2 over 8 experts give each expert a run of two blocks
    from consumer_deep_gemm.moe import MoELayer
    from metrics import errors

    cfg = dict(tokens=1000 if ue8m0 else 96, experts=8, hidden=512, inter=256, topk=2)
    x, ids, w, w1, w1s, w2, w2s = make_layer_inputs(**cfg)
    y_ref = MoELayer(w1, w1s, w2, w2s, num_experts=cfg["experts"], ops=TorchRefOps(), ue8m0=ue8m0)(x, ids, w)
    layer = MoELayer(w1.to(DEV), w1s.to(DEV), w2.to(DEV), w2s.to(DEV), num_experts=cfg["experts"], ue8m0=ue8m0)
    y = layer(x.to(DEV), ids.to(DEV), w.to(DEV))
    y2 = layer(x.to(DEV), ids.to(DEV), w.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16)), "repeat runs differ"
    nw, rl2 = errors(y.cpu(), y_ref)
    assert nw <= 1e-2 and rl2 <= 1e-2, (nw, rl2)


class _RecordingOps:
    """NativeOps that keep every stage's inputs and outputs of one forward."""

    def __init__(self):
        from consumer_deep_gemm.moe import NativeOps

        self.inner = NativeOps()
        self.rec = {"gemm": []}

    def __getattr__(self, name):
        return getattr(self.inner, name)

    def quant_dispatch_local(self, *args, **kw):
        out = self.inner.quant_dispatch_local(*args, **kw)
        self.rec["dispatch"] = out
        return out

    def gemm(self, a, sa, w, w_sf, m_indices, skip_ungrouped=False):
        d = self.inner.gemm(a, sa, w, w_sf, m_indices, skip_ungrouped)
        self.rec["gemm"].append((a, sa, m_indices, d))
        return d

    def act(self, h, m_indices, ue8m0=False):
        out = self.inner.act(h, m_indices, ue8m0)
        self.rec["act"] = (h, m_indices, out)
        return out

    def unpermute_combine(self, y, perm_pos, send_index, topk_w):
        out = self.inner.unpermute_combine(y, perm_pos, send_index, topk_w)
        self.rec["combine"] = (y, perm_pos, send_index, topk_w, out)
        return out


@pytest.mark.parametrize("ue8m0", [False, True], ids=["fp32", "ue8m0"])
def test_layer_stages_match_reference_at_gemm_tolerance(ue8m0):
    """Each stage of the one-GPU layer against the reference of that stage, on the device's own
    input to it: the GEMMs meet the single-GEMM bound (per-row L2 <= 2e-3)."""
    from consumer_deep_gemm.moe import MoELayer
    from metrics import TOL_NORMWISE, TOL_ROW_L2, errors
    from oracle import cdg_oracle as oracle

    cfg = dict(tokens=1000 if ue8m0 else 96, experts=8, hidden=512, inter=256, topk=2)
    x, ids, w, w1, w1s, w2, w2s = make_layer_inputs(**cfg)
    ops = _RecordingOps()
    layer = MoELayer(w1.to(DEV), w1s.to(DEV), w2.to(DEV), w2s.to(DEV), num_experts=cfg["experts"], ops=ops,
                     ue8m0=ue8m0, planes=False)  # the row form: its stage inputs are the oracle's inputs
    layer(x.to(DEV), ids.to(DEV), w.to(DEV))
    torch.cuda.synchronize()
    ref_ops = TorchRefOps()
    for (a, sa, mi, d), (wt, ws) in zip(ops.rec["gemm"], ((w1, w1s), (w2, w2s))):
        ref = torch.empty(d.shape, dtype=torch.bfloat16)
        oracle.m_grouped_fp8_fp4_gemm_nt_contiguous((a.cpu(), sa.cpu()), (wt, ws), ref, mi.cpu())
        rows = mi.cpu() >= 0
        nw, rl2 = errors(d.cpu(), ref, rows)
        assert nw <= TOL_NORMWISE and rl2 <= TOL_ROW_L2, ("gemm", nw, rl2)
    h, mi, (q, s) = ops.rec["act"]
    rows = mi.cpu() >= 0
    rq, rs = ref_ops.act(h.cpu()[rows], None, ue8m0)
    assert torch.allclose(s.cpu()[rows], rs, rtol=1e-6, atol=0)
    qa, qb = q.cpu()[rows].view(torch.uint8).to(torch.int32), rq.view(torch.uint8).to(torch.int32)
    diff = qa != qb
    assert diff.float().mean().item() <= 1e-3 and bool(((qa - qb).abs()[diff] <= 1).all())
    y2, pos, si, tw, out = ops.rec["combine"]
    ref_y = ref_ops.unpermute_combine(y2.cpu(), pos.cpu(), si.cpu(), tw.cpu())
    nw, rl2 = errors(out.cpu(), ref_y)
    assert nw <= TOL_NORMWISE and rl2 <= TOL_ROW_L2, ("combine", nw, rl2)


def test_peer_wait_runs_out_and_context_stays_usable():
    """Bounded waits on other ranks' flags, on one GPU: a window whose flags nobody raises.

    With the wait limit at 10 ms, the permute step gives up (it places no row: every
    m_indices and ret_slot entry stays -1), the combine step gives up (its output rows are zeros), the
    window's status word and the library's device record report CDG_ERR_DEVICE_TIMEOUT with
    the permute's wait code, and the context keeps working: a GEMM afterwards matches the
    reference.  Nothing here faults or hangs: every wait has its limit."""
    import consumer_deep_gemm as cdg
    from conftest import load_gemm_case
    from metrics import TOL_NORMWISE, TOL_ROW_L2, errors

    C = _ext()
    ranks, T, topk, H, e_loc = 2, 16, 2, 512, 4
    cap = T * topk
    cdg.read_device_status(True)  # start from a clean record
    own, _ = C.ep_window_create(C.ep_window_bytes(ranks, T, topk, H))
    try:
        C.ep_set_wait_timeout_ns(10_000_000)
        like = torch.zeros(1, device=DEV)
        m_pad = (ranks * cap + 127 * e_loc + 127) // 128 * 128
        a, sa, mi, ret_slot, _ = C.ep_permute_p2p(own, ranks, T, topk, H, e_loc, m_pad, like)
        send_index = torch.arange(T * topk, dtype=torch.int32, device=DEV)
        tw = torch.full((T, topk), 0.5, device=DEV)
        y = C.ep_combine_p2p(own, send_index, tw, ranks, T, H)
        torch.cuda.synchronize()
        assert C.ep_window_status(own) == 6
        st, where = cdg.read_device_status(True)
        assert st == 6 and (where >> 28) == 8, (st, hex(where))
        assert bool((ret_slot == -1).all()) and bool((mi == -1).all())
        assert bool((y.float() == 0).all())
        assert cdg.read_device_status(True) == (0, 0)
    finally:
        C.ep_set_wait_timeout_ns(0)
        C.ep_window_close(own, False)
    c = load_gemm_case("c0")
    dev = [t.to(DEV) for t in (c["a"], c["sa"], c["b"], c["sb"], c["m_indices"])]
    d = torch.empty(c["d"].shape, dtype=torch.bfloat16, device=DEV)
    cdg.m_grouped_fp8_fp4_gemm_nt_contiguous((dev[0], dev[1]), (dev[2], dev[3]), d, dev[4])
    torch.cuda.synchronize()
    pad = c["m_indices"] < 0
    nw, rl2 = errors(d.cpu(), c["d"], ~pad)
    assert nw <= TOL_NORMWISE and rl2 <= TOL_ROW_L2
    assert cdg.read_device_status(True) == (0, 0)


def _free_port() -> int:
    import socket

    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_layer_expert_parallel_two_gpus():
    here = os.path.dirname(os.path.abspath(__file__))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), os.path.join(here, "ep_gpu_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "300"] + cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    for mode in ("split_sizes", "fixed_capacity", "peer_memory", "peer_memory_ue8m0", "peer_memory_return_kernel"):
        assert f"EP_OK {mode}" in r.stdout, r.stdout[-3000:]


@pytest.mark.parametrize("ue8m0,planes,fused", [(False, False, False), (False, True, False), (True, False, False),
                                                (False, False, True), (False, True, True), (True, False, True)],
                         ids=["fp32", "fp32_planes", "ue8m0", "fp32_fused", "fp32_planes_fused", "ue8m0_fused"])
def test_peer_exchange_two_ranks_on_one_gpu(ue8m0, planes, fused):
    """The peer-memory exchange kernels for two ranks whose windows both live on this GPU.

    Each step runs rank 0's and rank 1's calls in order on one stream (dispatch, dispatch,
    permute, permute, GEMMs, return, return, combine, combine), so every flag a wait looks
    for was raised by an earlier launch: no kernel waits on one running beside it.  Fused
    return: FC2 stores its rows into the windows through the permute's row table; rank 1's
    flags are then raised by a return call with no rows and rank 0's by its own combine
    (whose wait finds rank 1's flag already up).  Three steps (both window parities and a
    reuse); the gathered outputs equal the one-GPU layer's (per-row relative L2 <= 1e-3)
    and no wait gave up."""
    import consumer_deep_gemm as cdg
    from consumer_deep_gemm.layout import transform_sf_into_required_layout
    from consumer_deep_gemm.moe import MoELayer, NativeOps
    from metrics import errors

    C = _ext()
    ranks, tpr, E, H, inter, topk = 2, 96, 8, 512, 256, 4
    x, ids, w, w1, w1s, w2, w2s = (t.to(DEV) for t in make_layer_inputs(ranks * tpr, E, H, inter, topk, seed=3))
    ids[5, 1] = -1  # a slot routed nowhere
    y_ref = MoELayer(w1, w1s, w2, w2s, num_experts=E, ue8m0=ue8m0)(x, ids, w)
    e_loc = E // ranks
    cdg.read_device_status(True)
    own = [C.ep_window_create(C.ep_window_bytes(ranks, tpr, topk, H))[0] for _ in range(ranks)]
    peers = torch.tensor(own, dtype=torch.int64, device=DEV)
    ops = NativeOps()
    shard = [(w1[r * e_loc:(r + 1) * e_loc].contiguous(), transform_sf_into_required_layout(w1s[r * e_loc:(r + 1) * e_loc]),
              w2[r * e_loc:(r + 1) * e_loc].contiguous(), transform_sf_into_required_layout(w2s[r * e_loc:(r + 1) * e_loc]))
             for r in range(ranks)]
    tok = [slice(r * tpr, (r + 1) * tpr) for r in range(ranks)]
    m_pad = (ranks * tpr * topk + 127 * e_loc + 127) // 128 * 128
    try:
        for step in range(3):
            si = [C.ep_dispatch_p2p(x[tok[r]], ids[tok[r]].contiguous(), E, ranks, tpr, peers, own[r], r, ue8m0)
                  for r in range(ranks)]
            permute = C.ep_permute_p2p_planes if planes else C.ep_permute_p2p
            placed = [permute(own[r], ranks, tpr, topk, H, e_loc, m_pad, x, peers if fused else None)
                      for r in range(ranks)]
            outs = []
            for r in range(ranks):
                a, sa, mi, _, ret_rows = placed[r]  # planes form: (planes, row exponents, ...)
                d_rows = ret_rows if fused else None
                if fused:
                    # placed rows have an address, the rest none
                    assert bool(((ret_rows != 0) == (mi >= 0)).all())
                b1, s1, b2, s2 = shard[r]
                if planes:
                    h = ops.gemm_planes(a, sa, b1, s1, mi, skip_ungrouped=True)
                    pl, rexp = ops.act_planes(h, mi)
                    outs.append(ops.gemm_planes(pl, rexp, b2, s2, mi, skip_ungrouped=True, d_rows=d_rows))
                else:
                    h = ops.gemm(a, sa, b1, s1, mi, skip_ungrouped=True)
                    aq, asc = ops.act(h, mi, ue8m0)
                    outs.append(ops.gemm(aq, asc, b2, s2, mi, skip_ungrouped=True, d_rows=d_rows))
            no_rows = torch.empty(0, H, dtype=torch.bfloat16, device=DEV)
            if fused:
                assert all(o is None for o in outs)
                C.ep_return_p2p(no_rows, placed[1][3], ranks, tpr, topk, peers, own[1], 1)  # flags only
            else:
                for r in range(ranks):
                    C.ep_return_p2p(outs[r], placed[r][3], ranks, tpr, topk, peers, own[r], r)
            y = torch.cat([C.ep_combine_p2p(own[r], si[r], w[tok[r]].float().contiguous(), ranks, tpr, H,
                                            peers if (fused and r == 0) else None, r)
                           for r in range(ranks)])
            torch.cuda.synchronize()
            nw, rl2 = errors(y, y_ref)
            assert nw <= 1e-3 and rl2 <= 1e-3, (step, nw, rl2)
            # every slot of a routed token was placed exactly once over the two ranks
            n_rows = sum(int((p[2] >= 0).sum()) for p in placed)
            assert n_rows == int((ids >= 0).sum()), (n_rows, int((ids >= 0).sum()))
        for r in range(ranks):
            assert C.ep_window_status(own[r]) == 0
        assert cdg.read_device_status(True) == (0, 0)
    finally:
        for p in own:
            C.ep_window_close(p, False)


def test_count_offsets_match_host_layout():
    """cdg_ep_count_offsets: per-expert counts and the 128-aligned group starts, on the device."""
    C = _ext()
    g = torch.Generator().manual_seed(13)
    for T, k, E in ((4096, 8, 256), (37, 3, 10), (0, 2, 5)):
        ids = torch.rand(T, E, generator=g).topk(k, dim=1).indices.to(torch.int32) if T else \
            torch.empty(0, k, dtype=torch.int32)
        if T:
            ids[0, 0] = -1
            ids[1, 0] = E  # outside [0, E): not counted
        cnt, off = C.ep_count_offsets(ids.to(DEV), E)
        ref = torch.bincount(ids[(ids >= 0) & (ids < E)].long(), minlength=E)
        aligned = (ref + 127) // 128 * 128
        assert torch.equal(cnt.cpu().long(), ref)
        assert torch.equal(off.cpu(), torch.cumsum(aligned, 0) - aligned)


def test_layer_planes_form_equals_rows_form():
    """FP32 activation scales: the layer's quantising steps writing the GEMMs' activation planes
    (the default) give the bits of the layer on e4m3 rows and scales."""
    from consumer_deep_gemm.moe import MoELayer

    cfg = dict(tokens=700, experts=8, hidden=512, inter=256, topk=2)
    x, ids, w, w1, w1s, w2, w2s = (t.to(DEV) for t in make_layer_inputs(**cfg))
    ids[3, 0] = -1
    rows = MoELayer(w1, w1s, w2, w2s, num_experts=cfg["experts"], planes=False)
    pl = MoELayer(w1, w1s, w2, w2s, num_experts=cfg["experts"])
    assert pl.planes and not rows.planes
    y_rows = rows(x, ids, w)
    y_pl = pl(x, ids, w)
    torch.cuda.synchronize()
    assert torch.equal(y_pl.view(torch.int16), y_rows.view(torch.int16))


def test_silu_mul_planes_equal_split_of_rows_form():
    """cdg_silu_mul_quant_planes writes the split the GEMM would make of cdg_silu_mul_quant_fp8's
    codes and scales; rows with a negative m_indices entry are left out."""
    import test_gpu_parity as gp

    C = _ext()
    g = torch.Generator().manual_seed(17)
    h = torch.randn(384, 2 * 640, generator=g).to(torch.bfloat16).to(DEV)
    mi = torch.zeros(384, dtype=torch.int32, device=DEV)
    mi[250:] = -1
    q, s = C.silu_mul_quant(h, mi, False)
    planes, rexp = C.silu_mul_quant_planes(h, mi)
    ref_planes, ref_exp = gp._torch_planes(q[:250], s[:250])
    assert torch.equal(planes[:, :250], ref_planes) and torch.equal(rexp[:250], ref_exp)
