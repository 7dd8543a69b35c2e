"""Expert parallelism (focr_ep_*) and the vocab-parallel top-1 all-gather.

* GPU, one device: ranks that share the GPU run phase by phase from one
  stream (focr_ep_connect_local), worlds 1/2/4/8, several consecutive steps;
  every rank's output is bit-identical to the single-GPU layer's for its
  tokens (same kernels on the same operands).  A world-1 communicator checks
  the NCCL bootstrap and the top-1 all-gather.
* GPU, several devices (skipped on one): one process per GPU over NCCL
  (focr_comm_create + focr_ep_connect_comm), bit-identical to one GPU, and
  the vocab-parallel argmax equal to the unsharded head's.
* CPU (gloo, world size 2): the dispatch / return / combine bookkeeping,
  restated on the host (oracle.ep_dispatch_layout), with the oracle's expert
  as the owner's computation, equals the single-rank oracle layer.
"""
import os
import socket

import numpy as np
import pytest
import torch


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(world, T, seed):
    from franken_ocr_b200 import synth

    out = []
    for r in range(world):
        x = synth.hidden_states(seed + r, T)
        i, w = synth.zipf_routing(seed + r, T)
        out.append((x, i, w))
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_ep_ranks_on_one_gpu_match_single_gpu(cuda, world):
    from franken_ocr_b200 import synth
    from franken_ocr_b200.ep import EpMoe, emulated_forward
    from franken_ocr_b200.moe import MoeLayer

    W = synth.moe_layer(55, shared_inter=1792)
    full = MoeLayer(W, max_tokens=64)
    ranks = [EpMoe(W, r, world, max_tokens=64) for r in range(world)]
    EpMoe.connect_local(ranks)
    for step in range(3):
        T = [64, 17, 1][step]
        ins = _inputs(world, T, 900 + 10 * step)
        want = [full.forward(x, i, w) for x, i, w in ins]
        ys = emulated_forward(ranks, *[[torch.from_numpy(a[k]).cuda() for a in ins] for k in range(3)])
        torch.cuda.synchronize()
        for r in range(world):
            got = ys[r].cpu().numpy()
            assert np.array_equal(got.view(np.uint32), want[r].view(np.uint32)), (step, r)
    assert all(rk.status() == 0 for rk in ranks)
    for rk in ranks:
        rk.close()
    full.close()


@pytest.mark.gpu
def test_ep_world1_over_nccl_and_top1_allgather(cuda):
    from franken_ocr_b200 import synth
    from franken_ocr_b200.ep import Comm, EpMoe, nccl_unique_id
    from franken_ocr_b200.moe import MoeLayer

    comm = Comm(nccl_unique_id(), 0, 1)
    W = synth.moe_layer(56, shared_inter=1792)
    full = MoeLayer(W, max_tokens=64)
    ep = EpMoe(W, 0, 1, max_tokens=64)
    ep.connect_comm(comm)
    x, i, w = _inputs(1, 64, 77)[0]
    y = ep.forward(*(torch.from_numpy(a).cuda() for a in (x, i, w)))
    yd, idd, wd = ep.decode(torch.from_numpy(x).cuda())
    want = full.forward(x, i, w)
    want_d, want_i, _ = full.decode(x)
    torch.cuda.synchronize()
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert np.array_equal(idd.cpu().numpy(), want_i)
    assert np.array_equal(yd.cpu().numpy().view(np.uint32), want_d.view(np.uint32))
    assert ep.status() == 0
    # top-1 all-gather over one rank: ties keep the lowest index, NaN skipped
    bv = torch.tensor([1.0, float("nan"), 2.0], device="cuda")
    bi = torch.tensor([5, 7, -1], dtype=torch.int32, device="cuda")
    tok, val = comm.top1_allgather(bv, bi)
    assert tok.tolist() == [5, 0, 0]
    assert val[0].item() == 1.0
    ep.close()
    full.close()
    comm.close()


def _mp_worker(rank, world, port, uid, q):
    """One GPU per process: EP forward over NCCL-bootstrapped peer memory and
    the vocab-parallel argmax, checked against this GPU's single-layer run."""
    try:
        import torch.distributed as dist

        torch.cuda.set_device(rank)
        from franken_ocr_b200 import synth
        from franken_ocr_b200.ep import Comm, EpMoe
        from franken_ocr_b200.lmhead import LmHeadShard
        from franken_ocr_b200.moe import MoeLayer

        comm = Comm(uid, rank, world)
        W = synth.moe_layer(57, shared_inter=1792)
        ep = EpMoe(W, rank, world, max_tokens=64)
        ep.connect_comm(comm)
        full = MoeLayer(W, max_tokens=64)
        ok = True
        for step in range(4):
            x, i, w = _inputs(world, 64 - 21 * step, 300 + 10 * step)[rank]
            y = ep.forward(*(torch.from_numpy(a).cuda() for a in (x, i, w)))
            want = full.forward(x, i, w)
            torch.cuda.synchronize()
            ok &= bool(np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32)))
        ok &= ep.status() == 0
        # vocab parallel: rank r holds rows [r*V/world, (r+1)*V/world)
        V, H = 4096, 1280
        g = np.random.default_rng(5)
        lw = g.integers(-127, 128, (V, H), dtype=np.int8)
        ls = g.uniform(0.001, 0.02, V).astype(np.float32)
        xs = g.standard_normal((3, H), dtype=np.float32)
        n = V // world
        shard = LmHeadShard(lw[rank * n:(rank + 1) * n], ls[rank * n:(rank + 1) * n],
                            row_begin=rank * n, max_tokens=3)
        bv, bi, _ = shard.top1(torch.from_numpy(xs).cuda())
        tok, _ = comm.top1_allgather(bv, bi)
        whole = LmHeadShard(lw, ls, 0, max_tokens=3)
        _, wi, _ = whole.top1(xs)
        ok &= tok.cpu().tolist() == [int(v) for v in wi]
        ep.close()
        comm.close()
        q.put((rank, ok))
    except Exception as exc:  # report, never hang the parent
        q.put((rank, f"{type(exc).__name__}: {exc}"))


@pytest.mark.gpu
def test_ep_multi_gpu_over_nccl(cuda):
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least two GPUs")
    import torch.multiprocessing as mp

    from franken_ocr_b200.ep import nccl_unique_id

    world = min(n, 8)
    uid = nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_mp_worker, args=(r, world, _port(), uid, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, ok = q.get(timeout=300)
        res[r] = ok
    for p in procs:
        p.join(60)
    assert res == {r: True for r in range(world)}, res


def _gloo_worker(rank, world, port, q):
    """Host restatement of the EP bookkeeping over gloo: rows to owners by
    ep_dispatch_layout, the owner's oracle expert, partials back, slot-order
    combine; compared with the single-rank oracle layer."""
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from franken_ocr_b200 import synth
        from oracle import oracle as O

        H, I, E, K, S, T = 128, 64, 8, 3, 128, 5
        W = synth.moe_layer(41, hidden=H, inter=I, n_experts=E, topk=K, shared_inter=S)
        el = E // world
        cap = T * K
        g = np.random.default_rng(100 + rank)
        x = g.standard_normal((T, H), dtype=np.float32)
        idx = np.stack([g.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
        w = g.uniform(0.05, 0.5, (T, K)).astype(np.float32)
        rows, sends = O.ep_dispatch_layout(idx, el, world, cap)
        # dispatch: [owner][cap] rows + (expert, weight) meta, plus counts
        sx = torch.zeros((world * cap, H))
        sm = torch.full((world * cap, 2), -1.0)
        for d in range(world):
            for pos, b in sends[d]:
                sx[d * cap + pos] = torch.from_numpy(x[b // K])
                sm[d * cap + pos] = torch.tensor([float(idx.flat[b]), float(w.flat[b])])
        rx, rm = torch.empty_like(sx), torch.empty_like(sm)
        dist.all_to_all_single(rx, sx)
        dist.all_to_all_single(rm, sm)
        # owner: p = expert(x) * w for each received row
        A = W.arrays
        part = torch.zeros((world * cap, H))
        for r in range(world * cap):
            e = int(rm[r, 0])
            if e < 0:
                continue
            assert e // el == rank
            y = O.expert_i8(rx[r].numpy(), A["gate_w"][e], A["gate_s"][e], A["up_w"][e],
                            A["up_s"][e], A["down_w"][e], A["down_s"][e])
            part[r] = torch.from_numpy(y * np.float32(rm[r, 1].item()))
        back = torch.empty_like(part)
        dist.all_to_all_single(back, part)
        bk = back.numpy()
        y = np.zeros((T, H), np.float32)
        for t in range(T):
            o = np.zeros(H, np.float32)
            for j in range(K):
                rr = rows[t * K + j]
                o = o + (bk[rr] if rr >= 0 else np.float32(0))
            s = O.expert_i8(x[t], A["sh_gate_w"], A["sh_gate_s"], A["sh_up_w"], A["sh_up_s"],
                            A["sh_down_w"], A["sh_down_s"])
            y[t] = o + s
        want = O.MoeOracle(W).forward(x, idx, w)
        q.put((rank, bool(np.array_equal(y.view(np.uint32), want.view(np.uint32)))))
    except Exception as exc:
        q.put((rank, f"{type(exc).__name__}: {exc}"))
    finally:
        dist.destroy_process_group()


def test_ep_bookkeeping_gloo_two_ranks():
    import torch.multiprocessing as mp

    port = _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(60)
    assert res == {0: True, 1: True}, res


def test_ep_dispatch_layout_positions():
    from oracle import oracle as O

    idx = np.array([[0, 5], [4, 1], [-1, 7]], np.int32)   # e_local 4: owners 0,1 | 1,0 | -,1
    rows, sends = O.ep_dispatch_layout(idx, 4, 2, 6)
    assert rows.tolist() == [0, 6, 7, 1, -1, 8]
    assert sends == [[(0, 0), (1, 3)], [(0, 1), (1, 2), (2, 5)]]
