"""CPU: the multi-GPU row-sharding plan and the verification gather, run as
world_size-2 gloo ranks.  The oracle stands in for the GPU forward."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import sharding


def test_zigzag_plan_covers_rows_and_balances_cost():
    for T in (1, 7, 512, 32768):
        for world in (1, 2, 4, 8):
            plan = sharding.zigzag_plan(T, world)
            rows = sorted(t for r in plan for b in r for t in range(b.start, b.stop))
            assert rows == list(range(T))
            if T >= 64 * world:
                cost = [sharding.causal_pairs(r) for r in plan]
                assert max(cost) / min(cost) < 1.05
                sizes = [sum(b.stop - b.start for b in r) for r in plan]
                assert max(sizes) - min(sizes) <= 2
    assert sharding.causal_pairs([sharding.RowBlock(0, 4)]) == 10
    assert sharding.causal_pairs([sharding.RowBlock(2, 6)], T_k=4) == 3 + 4 + 4 + 4


def _oracle_forward(q_idx, k_idx, w_idx, Q, K, V, top_k, q_row0=0):
    import dsa_oracle as o
    # the oracle wants full-length query tensors; pad rows before q_row0
    pad = lambda x: torch.cat([torch.zeros((x.shape[0], q_row0) + x.shape[2:]), x], 1)
    rows = slice(q_row0, q_row0 + Q.shape[1])
    Tk = K.shape[1]
    qf, wf, Qf = pad(q_idx), pad(w_idx), pad(Q)
    qf = torch.cat([qf, torch.zeros((qf.shape[0], Tk - qf.shape[1]) + qf.shape[2:])], 1)
    wf = torch.cat([wf, torch.zeros((wf.shape[0], Tk - wf.shape[1]) + wf.shape[2:])], 1)
    Qf = torch.cat([Qf, torch.zeros((Qf.shape[0], Tk - Qf.shape[1]) + Qf.shape[2:])], 1)
    return o.dsa_attention(qf, k_idx, wf, Qf, K, V, top_k, rows=rows)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import dsa_oracle as o
        T = 96
        args = o.make_inputs(2, T, 4, 16, 2, 16, 16)
        plan = sharding.zigzag_plan(T, world)
        local = sharding.forward_rows(_oracle_forward, *args, 12, plan[rank])
        full = sharding.gather_rows(local, plan)
        if rank == 0:
            whole = o.dsa_attention(*args, 12)
            q.put(float((full - whole).abs().max()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2])
def test_sharded_forward_gathers_to_whole(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert q.get(timeout=5) < 1e-6
