"""Expert parallelism: partition and exchange logic on CPU ranks (gloo, world sizes 2 and 4).

questwend_b200.expert_parallel.moe_layer runs unchanged on 2 or 4 CPU processes with a test
backend whose compute step is the CPU oracle (rms_norm, router top-k over all tokens,
mul_mat_id on the rank's expert range, swiglu, masked weighted sum, residual on rank 0).
After the layer's one all-reduce every rank must hold the same output for all tokens,
equal to a one-rank run of the same backend over all experts up to f32 summation order
(1e-6 normalized RMS), and that one-rank run must match the oracle's own build_moe layer
(1e-4).  Two layers are chained, so the second routes on the all-reduced output.  No GPU
is involved."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle as O
import _data as D

H, F, E, K_USED, T_RANK = 1024, 256, 8, 2, 3


class OracleBackend:
    """The compute step of the expert-parallel layer on the CPU oracle (which quantizes the
    activations inside mul_mat_id, exactly as the reference CPU backend does)."""

    def layer(self, x, router_w, shard, n_used, norm_w, norm_eps, residual, out=None):
        xn = O.rms_norm_mul(x.numpy(), norm_w.numpy(), norm_eps)
        logits = (xn.astype(np.float64) @ router_w.numpy().astype(np.float64).T).astype(np.float32)
        sel, w = O.route(logits, n_used)
        T = xn.shape[0]
        local = (sel >= shard.lo) & (sel < shard.lo + shard.n)
        ids = np.where(local, sel - shard.lo, 0).astype(np.int32)
        g, rc = O.mul_mat_id(O.Q4_K, shard.gate, H, F, shard.n, xn[:, None, :], ids)
        assert rc == 0
        u, rc = O.mul_mat_id(O.Q4_K, shard.up, H, F, shard.n, xn[:, None, :], ids)
        assert rc == 0
        act = (g / (1.0 + np.exp(-g)) * u).astype(np.float32)
        dn, rc = O.mul_mat_id(O.Q6_K, shard.down, F, H, shard.n, act, ids)
        assert rc == 0
        part = np.zeros((T, H), dtype=np.float32)
        for j in range(sel.shape[1]):
            part += np.where(local[:, j:j + 1], w[:, j:j + 1] * dn[:, j, :], 0.0).astype(np.float32)
        if residual is not None:
            part += residual.numpy()
        return torch.from_numpy(part), torch.from_numpy(sel), torch.from_numpy(w)


def _inputs(world):
    r = D.rng(11)
    x = r.standard_normal((world * T_RANK, H), dtype=np.float32)
    router_w = (r.standard_normal((E, H), dtype=np.float32) * 0.02).astype(np.float32)
    norm_w = (1.0 + 0.1 * r.standard_normal(H)).astype(np.float32)
    gate = D.weights(O.Q4_K, E, F, H, seed=12)
    up = D.weights(O.Q4_K, E, F, H, seed=13)
    down = D.weights(O.Q6_K, E, H, F, seed=14)
    return x, router_w, norm_w, gate, up, down


def _shard(gate, up, down, lo, n):
    from questwend_b200.expert_parallel import ExpertShard
    rg, rd = O.row_size(O.Q4_K, H) * F, O.row_size(O.Q6_K, F) * H
    return ExpertShard(gate[lo * rg:(lo + n) * rg], up[lo * rg:(lo + n) * rg], down[lo * rd:(lo + n) * rd], lo, n)


def _rank_main(rank, world, port, q):
    import torch.distributed as dist

    from questwend_b200.expert_parallel import moe_layer, shard_range
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    x, router_w, norm_w, gate, up, down = _inputs(world)
    lo, n = shard_range(E, world, rank)
    shard = _shard(gate, up, down, lo, n)
    y = torch.from_numpy(x)
    sels = []
    for _ in range(2):
        y, sel, _ = moe_layer(y, torch.from_numpy(router_w), shard, K_USED, norm_w=torch.from_numpy(norm_w),
                              backend=OracleBackend())
        sels.append(sel.numpy())
    q.put((rank, y.numpy(), sels))
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_cpu_ranks_match_one_rank_and_oracle(world):
    here = os.path.dirname(os.path.abspath(__file__))
    os.environ["PYTHONPATH"] = os.pathsep.join([os.path.dirname(here), here, os.environ.get("PYTHONPATH", "")])
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, out, sels = q.get(timeout=180)
        res[rank] = (out, sels)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # every rank holds the same output (the all-reduce leaves identical sums) and routing
    for r in range(1, world):
        assert np.array_equal(res[r][0], res[0][0])
        assert all(np.array_equal(a, b) for a, b in zip(res[r][1], res[0][1]))

    # one rank, all experts: same backend, no exchange, two chained layers
    x, router_w, norm_w, gate, up, down = _inputs(world)
    bk = OracleBackend()
    full = _shard(gate, up, down, 0, E)
    y = torch.from_numpy(x)
    layer_in = []
    for layer in range(2):
        layer_in.append(y.numpy())
        y, sel, _ = bk.layer(y, torch.from_numpy(router_w), full, K_USED, torch.from_numpy(norm_w), 1e-6, y)
        assert (res[0][1][layer] == sel.numpy()).all()
    single = y.numpy()
    assert O.nrmse(res[0][0], single) <= 1e-6, O.nrmse(res[0][0], single)

    # and the backend itself is build_moe: the oracle's own layer, on the last layer's input
    want = O.moe_layer(layer_in[1], router_w, O.Q4_K, gate, up, O.Q6_K, down, F, E, K_USED, norm_w=norm_w)
    assert O.nrmse(single - layer_in[1], want["out"]) <= 1e-4


def test_shard_range_partitions_experts():
    from questwend_b200.expert_parallel import shard_range
    for E_, world in ((128, 8), (128, 3), (10, 4), (7, 7)):
        spans = [shard_range(E_, world, r) for r in range(world)]
        assert spans[0][0] == 0
        for (lo, n), (lo2, _) in zip(spans, spans[1:]):
            assert lo + n == lo2
        assert spans[-1][0] + spans[-1][1] == E_
        assert max(n for _, n in spans) - min(n for _, n in spans) <= 1
