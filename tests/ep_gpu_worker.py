"""Worker of the 2-GPU expert-parallel test (launched by torchrun from test_gpu_moe.py).

Each rank builds the same layer inputs, keeps its half of the experts and of the
tokens, runs the EP layer, and rank 0 compares the gathered output
  * with the CPU reference layer (moe_ref.TorchRefOps: the oracle GEMM and the reference
    quantisation steps): max |y - ref| / max |ref| <= 1e-2 and per-row relative L2 <= 1e-2,
    the end-to-end layer tolerance (see test_gpu_moe.py), and
  * with the single-GPU layer (all experts on one GPU): per-row relative L2 <= 1e-3.
Every layer also reports no device wait that gave up (MoELayer.status()).
"""

import datetime
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
for p in (os.path.join(os.path.dirname(HERE), "consumer-deepgemm_b200"), os.path.dirname(HERE), HERE):
    sys.path.insert(0, p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from consumer_deep_gemm.moe import MoELayer  # noqa: E402
from metrics import errors  # noqa: E402
from moe_ref import TorchRefOps, make_layer_inputs  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    cfg = dict(tokens=256, experts=16, hidden=1024, inter=512, topk=4)
    x, ids, w, w1, w1s, w2, w2s = (t.to(dev) for t in make_layer_inputs(**cfg))
    e_loc = cfg["experts"] // world
    sl = slice(rank * e_loc, (rank + 1) * e_loc)
    tpr = cfg["tokens"] // world
    ts = slice(rank * tpr, (rank + 1) * tpr)
    y_ref = {u: MoELayer(w1, w1s, w2, w2s, num_experts=cfg["experts"], ue8m0=u)(x, ids, w) if rank == 0 else None
             for u in (False, True)}
    y_cpu = {u: MoELayer(w1.cpu(), w1s.cpu(), w2.cpu(), w2s.cpu(), num_experts=cfg["experts"], ops=TorchRefOps(),
                         ue8m0=u)(x.cpu(), ids.cpu(), w.cpu()) if rank == 0 else None
             for u in (False, True)}
    # split-size exchange (one host sync), fixed-capacity NCCL exchange (none), and the
    # library's peer-memory exchange (no collective), three forwards each (window parities);
    # the peer-memory exchange also with power-of-two activation scales, and with FC2 writing a
    # local buffer that a separate kernel returns (instead of storing into the windows itself)
    for mode, max_tok, exchange, ue8m0, fused in (("split_sizes", None, "nccl", False, True),
                                                  ("fixed_capacity", tpr, "nccl", False, True),
                                                  ("peer_memory", tpr, "p2p", False, True),
                                                  ("peer_memory_ue8m0", tpr, "p2p", True, True),
                                                  ("peer_memory_return_kernel", tpr, "p2p", False, False)):
        y_one = y_ref[ue8m0]
        layer = MoELayer(w1[sl], w1s[sl], w2[sl], w2s[sl], num_experts=cfg["experts"], group=dist.group.WORLD,
                         max_tokens_per_rank=max_tok, exchange=exchange, ue8m0=ue8m0, fused_return=fused)
        for it in range(3):
            y = layer(x[ts], ids[ts], w[ts])
            parts = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(parts, y)
            if rank == 0:
                nw, rl2 = errors(torch.cat(parts), y_one)
                assert nw <= 1e-3 and rl2 <= 1e-3, (mode, it, nw, rl2)
                nwc, rl2c = errors(torch.cat(parts), y_cpu[ue8m0])
                assert nwc <= 1e-2 and rl2c <= 1e-2, (mode, it, "cpu reference", nwc, rl2c)
        if exchange == "p2p":
            # the same step as a CUDA graph, replayed
            xs, idss, ws = x[ts].clone(), ids[ts].clone(), w[ts].clone()
            graph, y_g = layer.capture(xs, idss, ws)
            for it in range(3):
                graph.replay()
                parts = [torch.empty_like(y_g) for _ in range(world)]
                dist.all_gather(parts, y_g)
                if rank == 0:
                    nw, rl2 = errors(torch.cat(parts), y_one)
                    assert nw <= 1e-3 and rl2 <= 1e-3, ("graph", it, nw, rl2)
            torch.cuda.synchronize()
            del graph
        assert layer.status() == 0, "a device wait gave up"
        dist.barrier()
        layer.close()
        if rank == 0:
            print("EP_OK", mode, nw, rl2, flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
