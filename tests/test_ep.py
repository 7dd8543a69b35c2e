"""Expert parallelism: the dispatch / expert / return / combine path.

* GPU (emulated ranks on one device): N ranks, each owning 64/N experts and a
  replica of the shared expert, reproduce the single-GPU layer's output for
  every rank's tokens (same kernels on the same operands: bit-identical).
* CPU (gloo, world size 2): the all-to-all bookkeeping of the distributed
  forward with a stand-in expert function.
"""
import os

import numpy as np
import pytest
import torch


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_emulated_matches_single_gpu(cuda, world):
    from franken_ocr_b200 import synth
    from franken_ocr_b200.ep import EpMoeRank, emulated_forward
    from franken_ocr_b200.moe import MoeLayer

    W = synth.moe_layer(55, shared_inter=1792)
    full = MoeLayer(W, max_tokens=64)
    ranks = [EpMoeRank(W, r, world, max_tokens=64) for r in range(world)]
    xs, idxs, ws, want = [], [], [], []
    for r in range(world):
        x = synth.hidden_states(900 + r, 64)
        i, w = synth.zipf_routing(900 + r, 64)
        xs.append(torch.from_numpy(x).cuda())
        idxs.append(torch.from_numpy(i).cuda())
        ws.append(torch.from_numpy(w).cuda())
        want.append(full.forward(x, i, w))
    ys = emulated_forward(ranks, xs, idxs, ws)
    torch.cuda.synchronize()
    for r in range(world):
        got = ys[r].cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want[r].view(np.uint32)), f"rank {r}"
    for rk in ranks:
        rk.close()
    full.close()


def _gloo_worker(rank, world, port, q):
    """The equal-split all-to-all exchange pattern EpMoeRank.forward uses:
    rank r's block d (rows [d*C, (d+1)*C)) must arrive as block r of rank d."""
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        C, H = 3, 4
        send = torch.stack([torch.full((C, H), float(100 * rank + d)) for d in range(world)]).view(-1, H)
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send)
        want = torch.stack([torch.full((C, H), float(100 * s + rank)) for s in range(world)]).view(-1, H)
        q.put((rank, bool(torch.equal(recv, want))))
    finally:
        dist.destroy_process_group()


def test_ep_exchange_gloo_two_ranks():
    import socket

    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    res = dict(q.get(timeout=5) for _ in range(2))
    assert res == {0: True, 1: True}
