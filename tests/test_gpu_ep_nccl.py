"""Expert parallelism over real GPUs: two processes, one GPU each, one NCCL all-reduce per
layer (questwend_b200.expert_parallel.moe_layer with the CUDA backend), two layers
chained.  Both ranks must end with the same output for all tokens, matching the fused
single-GPU layer (qwb_moe_ffn) applied twice within 1e-5 normalized RMS.  Skipped when
fewer than two GPUs are visible."""
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


def _rank_main(rank, world, port, q):
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
    for _ in range(2):
        y, sel, _ = moe_layer(y, rw, shard, K_USED, norm_w=nw)
    torch.cuda.synchronize()
    flags, _, _ = qwb.read_status()
    q.put((rank, y.cpu().numpy(), sel.cpu().numpy(), flags))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gpus_match_fused_layer():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    here = os.path.dirname(os.path.abspath(__file__))
    os.environ["PYTHONPATH"] = os.pathsep.join([os.path.dirname(here), here, os.environ.get("PYTHONPATH", "")])
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rank, out, sel, flags = q.get(timeout=300)
        res[rank] = (out, sel, flags)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
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
