"""Expert parallelism: partition and exchange logic on CPU ranks (gloo, world sizes 2 and 4).

questwend_b200.expert_parallel.moe_layer runs unchanged on 2 or 4 CPU processes with a test
backend whose compute steps are the CPU oracle (rms_norm, router top-k, mul_mat_id on the
rank's expert range, swiglu, masked weighted sum).  The outputs of the ranks must
equal a one-rank run of the same backend over all tokens and all experts up to f32
summation order (1e-6 normalized RMS), and that one-rank run must match the oracle's own
build_moe layer (1e-4).  No GPU is involved."""
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
    """Compute steps of the expert-parallel layer on the CPU oracle.  The 'packed rows'
    exchanged between ranks are the normalised f32 rows (the oracle quantizes inside
    mul_mat_id, exactly as the reference CPU backend does)."""

    def prepare(self, x, router_w, n_used, norm_w, norm_eps, act_type):
        xn = O.rms_norm_mul(x.numpy(), norm_w.numpy(), norm_eps)
        logits = (xn.astype(np.float64) @ router_w.numpy().astype(np.float64).T).astype(np.float32)
        sel, w = O.route(logits, n_used)
        return torch.from_numpy(xn), torch.from_numpy(sel), torch.from_numpy(w)

    def experts(self, xq, selected, weights, shard, n_expert):
        x = xq.numpy()
        sel = selected.numpy()
        w = weights.numpy()
        T = x.shape[0]
        local = (sel >= shard.lo) & (sel < shard.lo + shard.n)
        ids = np.where(local, sel - shard.lo, 0).astype(np.int32)
        g, rc = O.mul_mat_id(O.Q4_K, shard.gate, H, F, shard.n, x[:, None, :], ids)
        assert rc == 0
        u, rc = O.mul_mat_id(O.Q4_K, shard.up, H, F, shard.n, x[:, None, :], ids)
        assert rc == 0
        act = (g / (1.0 + np.exp(-g)) * u).astype(np.float32)
        dn, rc = O.mul_mat_id(O.Q6_K, shard.down, F, H, shard.n, act, ids)
        assert rc == 0
        out = np.zeros((T, H), dtype=np.float32)
        for j in range(sel.shape[1]):
            out += np.where(local[:, j:j + 1], w[:, j:j + 1] * dn[:, j, :], 0.0).astype(np.float32)
        return torch.from_numpy(out)


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
    xs = torch.from_numpy(x[rank * T_RANK:(rank + 1) * T_RANK].copy())
    out, sel, w = moe_layer(xs, torch.from_numpy(router_w), _shard(gate, up, down, lo, n), K_USED, E,
                            norm_w=torch.from_numpy(norm_w), backend=OracleBackend())
    q.put((rank, out.numpy(), sel.numpy()))
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
        rank, out, sel = q.get(timeout=180)
        res[rank] = (out, sel)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ep_out = np.concatenate([res[r][0] for r in range(world)])
    ep_sel = np.concatenate([res[r][1] for r in range(world)])

    # one rank, all experts: same backend, no exchange
    x, router_w, norm_w, gate, up, down = _inputs(world)
    bk = OracleBackend()
    xn, sel, w = bk.prepare(torch.from_numpy(x), torch.from_numpy(router_w), K_USED, torch.from_numpy(norm_w), 1e-6, 0)
    single = bk.experts(xn, sel, w, _shard(gate, up, down, 0, E), E).numpy() + x
    assert (ep_sel == sel.numpy()).all()
    assert O.nrmse(ep_out, single) <= 1e-6, O.nrmse(ep_out, single)

    # and the backend itself is build_moe: the oracle's own layer
    want = O.moe_layer(x, router_w, O.Q4_K, gate, up, O.Q6_K, down, F, E, K_USED, norm_w=norm_w)
    assert (want["selected"] == sel.numpy()).all()
    assert O.nrmse(single - x, want["out"]) <= 1e-4


def test_shard_range_partitions_experts():
    from questwend_b200.expert_parallel import shard_range
    for E_, world in ((128, 8), (128, 3), (10, 4), (7, 7)):
        spans = [shard_range(E_, world, r) for r in range(world)]
        assert spans[0][0] == 0
        for (lo, n), (lo2, _) in zip(spans, spans[1:]):
            assert lo + n == lo2
        assert spans[-1][0] + spans[-1][1] == E_
        assert max(n for _, n in spans) - min(n for _, n in spans) <= 1
