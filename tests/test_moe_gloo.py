"""Expert-parallel exchange logic over two gloo ranks on CPU (no GPU).

Each rank owns half of the experts and half of the tokens; the gathered EP
output must equal the single-process layer computed with the same CPU ops.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

CFG = dict(tokens=24, experts=8, hidden=256, inter=128, topk=2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, fixed=False):
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    for p in (os.path.join(os.path.dirname(here), "consumer-deepgemm_b200"), os.path.dirname(here), here):
        sys.path.insert(0, p)
    import torch.distributed as dist

    from consumer_deep_gemm.moe import MoELayer
    from moe_ref import TorchRefOps, make_layer_inputs

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _run(rank, world, q, fixed)
    except Exception as exc:  # report instead of leaving the parent waiting
        q.put((rank, repr(exc)))
        raise
    finally:
        dist.destroy_process_group()


def _run(rank, world, q, fixed=False):
    import torch.distributed as dist

    from consumer_deep_gemm.moe import MoELayer
    from moe_ref import TorchRefOps, make_layer_inputs

    if True:
        x, ids, w, w1, w1s, w2, w2s = make_layer_inputs(**CFG)
        e_loc = CFG["experts"] // world
        sl = slice(rank * e_loc, (rank + 1) * e_loc)
        tpr = CFG["tokens"] // world
        layer = MoELayer(w1[sl], w1s[sl], w2[sl], w2s[sl], num_experts=CFG["experts"], group=dist.group.WORLD,
                         ops=TorchRefOps(), max_tokens_per_rank=tpr if fixed else None)
        ts = slice(rank * tpr, (rank + 1) * tpr)
        y = layer(x[ts], ids[ts], w[ts])
        q.put((rank, y))


@pytest.mark.parametrize("fixed", [False, True], ids=["split_sizes", "fixed_capacity"])
def test_ep_two_ranks_matches_single_process(fixed):
    from consumer_deep_gemm.moe import MoELayer
    from moe_ref import TorchRefOps, make_layer_inputs

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, fixed)) for r in range(2)]
    for p in procs:
        p.start()
    outs = dict(q.get(timeout=120) for _ in procs)
    for r, v in outs.items():
        assert isinstance(v, torch.Tensor), f"rank {r} failed: {v}"
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    y_ep = torch.cat([outs[0], outs[1]])
    x, ids, w, w1, w1s, w2, w2s = make_layer_inputs(**CFG)
    y_ref = MoELayer(w1, w1s, w2, w2s, num_experts=CFG["experts"], ops=TorchRefOps())(x, ids, w)
    assert torch.equal(y_ep.view(torch.int16), y_ref.view(torch.int16))
    assert y_ref.abs().max() > 0


def test_single_process_layer_composition():
    """world 1 with the reference ops equals a direct per-(token, slot) evaluation."""
    from consumer_deep_gemm.moe import MoELayer
    from deep_gemm.utils.math import per_block_cast_to_fp8
    from moe_ref import TorchRefOps, make_layer_inputs
    from oracle import cdg_oracle as oracle

    x, ids, w, w1, w1s, w2, w2s = make_layer_inputs(**CFG)
    y = MoELayer(w1, w1s, w2, w2s, num_experts=CFG["experts"], ops=TorchRefOps())(x, ids, w)
    xq, xs = per_block_cast_to_fp8(x.float())
    t = 5
    acc = torch.zeros(CFG["hidden"])
    for j in range(CFG["topk"]):
        e = int(ids[t, j])
        h = torch.empty(1, 2 * CFG["inter"], dtype=torch.bfloat16)
        oracle.m_grouped_fp8_fp4_gemm_nt_contiguous((xq[t:t + 1], xs[t:t + 1]), (w1[e], w1s[e]), h)
        g, u = h[:, :CFG["inter"]].float(), h[:, CFG["inter"]:].float()
        aq, asc = per_block_cast_to_fp8(torch.nn.functional.silu(g) * u)
        o = torch.empty(1, CFG["hidden"], dtype=torch.bfloat16)
        oracle.m_grouped_fp8_fp4_gemm_nt_contiguous((aq, asc), (w2[e], w2s[e]), o)
        acc += w[t, j] * o[0].float()
    assert torch.equal(y[t].view(torch.int16), acc.to(torch.bfloat16).view(torch.int16))


def test_pow2_quant_recipe():
    """The power-of-two (UE8M0) activation recipe of the reference ops: every scale is
    2^ceil(log2(amax / 448)), the codes stay within e4m3's range and dequantise to x within
    e4m3 precision; the layer over it stays close to the FP32-scale layer."""
    from consumer_deep_gemm.moe import MoELayer
    from metrics import errors
    from moe_ref import TorchRefOps, cast_to_fp8_pow2, make_layer_inputs

    g = torch.Generator().manual_seed(4)
    x = torch.randn(64, 512, generator=g) * torch.rand(64, 1, generator=g) * 100
    q, s = cast_to_fp8_pow2(x)
    amax = x.view(64, 4, 128).abs().amax(2).clamp(min=1e-12)
    assert torch.equal(s, torch.exp2(torch.ceil(torch.log2(amax / 448.0))))
    mant, _ = torch.frexp(s)
    assert bool((mant == 0.5).all())
    deq = q.float().view(64, 4, 128) * s.unsqueeze(-1)
    assert float(q.float().abs().max()) <= 448.0
    assert bool(((deq - x.view(64, 4, 128)).abs() <= x.view(64, 4, 128).abs() / 16 + s.unsqueeze(-1) * 2 ** -9).all())

    xs, ids, w, w1, w1s, w2, w2s = make_layer_inputs(**CFG)
    y32 = MoELayer(w1, w1s, w2, w2s, num_experts=CFG["experts"], ops=TorchRefOps())(xs, ids, w)
    y2 = MoELayer(w1, w1s, w2, w2s, num_experts=CFG["experts"], ops=TorchRefOps(), ue8m0=True)(xs, ids, w)
    nw, rl2 = errors(y2, y32)
    assert nw <= 0.1 and rl2 <= 0.1, (nw, rl2)
