"""Expert parallelism over real GPUs: two processes, one GPU each (skipped when fewer than
two GPUs are visible).

* The layer (questwend_b200.expert_parallel.moe_layer with the CUDA backend), two layers
  chained, with NCCL's all-reduce and with the peer-memory all-reduce (qwb_ep_comm): both
  ranks end with the same output for all tokens, matching the fused single-GPU layer
  (qwb_moe_ffn) applied twice within 1e-5 normalized RMS.
* The peer-memory all-reduce alone, eager, replayed from a CUDA graph, and three calls
  back to back in one graph (each launched while the previous one still runs), message
  sizes 16 B to 1 MB: every rank gets exactly the float32 sum in rank order.
* Its bounded wait: a rank that never joins the call leaves the other rank's kernel to
  give up after 5 s with QWB_DEVERR_TIMEOUT in the status block (no fault, no hang).
NVLS is off (NCCL_NVLS_ENABLE=0) and the peer all-reduce uses plain peer stores."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle as O
import _data as D

pytestmark = pytest.mark.gpu

H, F, E, K_USED, T = 2048, 768, 32, 8, 8


def _weights():
    r = D.rng(90)
    router_w = (r.standard_normal((E, H), dtype=np.float32) * 0.02).astype(np.float32)
    norm_w = (1.0 + 0.1 * r.standard_normal(H)).astype(np.float32)
    x = D.acts((T, H), seed=91)
    return router_w, norm_w, x, D.weights(O.Q4_K, E, F, H, seed=92), D.weights(O.Q4_K, E, F, H, seed=93), \
        D.weights(O.Q6_K, E, H, F, seed=94)


def _rank_main(rank, world, port, q, use_comm=False):
    import datetime

    import torch.distributed as dist

    import questwend_b200 as qwb
    from questwend_b200.expert_parallel import ExpertShard, moe_layer, shard_range
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    router_w, norm_w, x, gate, up, down = _weights()
    lo, n = shard_range(E, world, rank)
    rg, rd = O.row_size(O.Q4_K, H) * F, O.row_size(O.Q6_K, F) * H
    shard = ExpertShard(qwb.QTensor.from_bytes(gate[lo * rg:(lo + n) * rg], O.Q4_K, (H, F, n)),
                        qwb.QTensor.from_bytes(up[lo * rg:(lo + n) * rg], O.Q4_K, (H, F, n)),
                        qwb.QTensor.from_bytes(down[lo * rd:(lo + n) * rd], O.Q6_K, (F, H, n)), lo, n)
    y = torch.from_numpy(x).cuda()
    rw, nw = torch.from_numpy(router_w).cuda(), torch.from_numpy(norm_w).cuda()
    comm = None
    if use_comm:
        from questwend_b200.expert_parallel import PeerAllReduce
        comm = PeerAllReduce(max_bytes=T * H * 4)
    for _ in range(2):
        y, sel, _ = moe_layer(y, rw, shard, K_USED, norm_w=nw, comm=comm)
    torch.cuda.synchronize()
    flags, _, _ = qwb.read_status()
    q.put((rank, y.cpu().numpy(), sel.cpu().numpy(), flags))
    dist.barrier()
    if comm is not None:
        comm.close()
    dist.destroy_process_group()


def _spawn(target, extra=()):
    here = os.path.dirname(os.path.abspath(__file__))
    os.environ["PYTHONPATH"] = os.pathsep.join([os.path.dirname(here), here, os.environ.get("PYTHONPATH", "")])
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, 2, port, q) + tuple(extra)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        item = q.get(timeout=300)
        res[item[0]] = item[1:]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


@pytest.mark.parametrize("use_comm", [False, True])
def test_two_gpus_match_fused_layer(use_comm):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    res = _spawn(_rank_main, (use_comm,))
    assert res[0][2] == 0 and res[1][2] == 0
    assert np.array_equal(res[0][0], res[1][0]) and np.array_equal(res[0][1], res[1][1])

    import questwend_b200 as qwb
    router_w, norm_w, x, gate, up, down = _weights()
    y = torch.from_numpy(x).cuda()
    G = qwb.QTensor.from_bytes(gate, O.Q4_K, (H, F, E))
    U = qwb.QTensor.from_bytes(up, O.Q4_K, (H, F, E))
    Dn = qwb.QTensor.from_bytes(down, O.Q6_K, (F, H, E))
    for _ in range(2):
        y, sel, _ = qwb.moe_ffn(y, torch.from_numpy(router_w).cuda(), G, U, Dn, K_USED, residual=y,
                                norm_w=torch.from_numpy(norm_w).cuda())
        y = y.clone()
    assert (res[0][1] == sel.cpu().numpy()).all()
    e = O.nrmse(res[0][0], y.cpu().numpy())
    assert e <= 1e-5, (e, O.max_abs_rel(res[0][0], y.cpu().numpy()))


def _allreduce_main(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    import questwend_b200 as qwb
    from questwend_b200.expert_parallel import PeerAllReduce
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    comm = PeerAllReduce(max_bytes=1 << 20)
    results = []
    for n in (4, 4096, 16384, 262144):
        x = torch.from_numpy(np.random.default_rng(1000 * rank + n).standard_normal(n, dtype=np.float32)).cuda()
        y = x.clone()
        comm.all_reduce(y)
        # the same call captured in a graph and replayed three times (the sum grows)
        z = x.clone()
        g = torch.cuda.CUDAGraph()
        cs = torch.cuda.Stream()
        cs.wait_stream(torch.cuda.current_stream())
        torch.cuda.synchronize()
        dist.barrier()
        with torch.cuda.stream(cs):
            with torch.cuda.graph(g, stream=cs):
                comm.all_reduce(z)
        zs = []
        for _ in range(3):
            z.copy_(x)
            g.replay()
            torch.cuda.synchronize()
            zs.append(z.cpu().numpy().copy())
        del g
        # three calls back to back in one graph (each launched while the previous one runs)
        ws = [x.clone() for _ in range(3)]
        g = torch.cuda.CUDAGraph()
        torch.cuda.synchronize()
        dist.barrier()
        with torch.cuda.stream(cs):
            with torch.cuda.graph(g, stream=cs):
                for w_ in ws:
                    comm.all_reduce(w_)
        for _ in range(2):
            for w_ in ws:
                w_.copy_(x)
            g.replay()
            torch.cuda.synchronize()
            zs.extend(w_.cpu().numpy().copy() for w_ in ws)
        del g
        results.append((n, y.cpu().numpy(), zs))
    torch.cuda.synchronize()
    flags, _, _ = qwb.read_status()
    q.put((rank, results, flags))
    dist.barrier()
    comm.close()
    dist.destroy_process_group()


def test_peer_allreduce_exact_rank_order_sum():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    res = _spawn(_allreduce_main)
    assert res[0][1] == 0 and res[1][1] == 0
    for (n, y0, zs0), (_, y1, zs1) in zip(res[0][0], res[1][0]):
        xs = [np.random.default_rng(1000 * r + n).standard_normal(n, dtype=np.float32) for r in range(2)]
        want = xs[0] + xs[1]  # float32, rank order
        assert np.array_equal(y0.view(np.uint32), want.view(np.uint32)), n
        assert np.array_equal(y1.view(np.uint32), want.view(np.uint32)), n
        for z in zs0 + zs1:
            assert np.array_equal(z.view(np.uint32), want.view(np.uint32)), n


def _timeout_main(rank, world, port, q):
    import datetime
    import time

    import torch.distributed as dist

    import questwend_b200 as qwb
    from questwend_b200.expert_parallel import PeerAllReduce
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    comm = PeerAllReduce(max_bytes=1 << 16)
    qwb.read_status()
    t0 = time.time()
    if rank == 0:
        # rank 1 never joins this call: rank 0's kernel gives up after its bounded wait
        x = torch.ones(1024, device="cuda")
        comm.all_reduce(x)
        torch.cuda.synchronize()
    elapsed = time.time() - t0
    flags, bad, _ = qwb.read_status()
    q.put((rank, flags, elapsed))
    dist.barrier()
    comm.close()
    dist.destroy_process_group()


def test_peer_allreduce_bounded_wait_reports_timeout():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    res = _spawn(_timeout_main)
    QWB_DEVERR_TIMEOUT = 0x4
    assert res[0][0] & QWB_DEVERR_TIMEOUT, res
    assert 4.0 < res[0][1] < 60.0, res
    assert res[1][0] == 0
