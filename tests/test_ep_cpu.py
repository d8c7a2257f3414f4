"""Expert-parallel exchange logic on CPU: plan_exchange and exchange_rows with gloo ranks.

The CUDA stages need a GPU; the row exchange between them is plain torch.distributed and is
checked here end to end with 2 and 3 gloo ranks: every row reaches the segment of the expert
it was routed to, and the reverse exchange puts it back where it came from.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from velvetoptimizer_b200.ep import TILE_ROWS, exchange_rows, plan_exchange


def test_plan_exchange_layout():
    # rank 1 of 2, E = 4 (2 local): send counts per global expert, recv counts [src, local e]
    send = [3, 0, 5, 2]
    recv = np.array([[4, 1], [5, 2]])
    p = plan_exchange(send, recv)
    assert p.send_offsets.tolist() == [0, 3, 3, 8, 10]
    assert p.seg_offsets.tolist() == [0, 128, 256]           # 9 -> 128, 3 -> 128
    assert p.recv_offsets.tolist() == [[0, 128], [4, 129]]
    assert p.recv_rows == 256 and p.tile_expert.tolist() == [0, 1]
    big = plan_exchange([0] * 4, np.array([[200, 0], [100, 0]]))
    assert big.tile_expert.tolist() == [0, 0, 0] and big.recv_rows == 3 * TILE_ROWS


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, E, K, T, H, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        El = E // world
        rng = np.random.default_rng(100 + rank)
        idx = np.stack([rng.choice(E, K, replace=False) for _ in range(T)])
        # send layout: expert-major, tokens ascending (what vmoe_ep_route writes)
        order = np.lexsort((np.repeat(np.arange(T), K), idx.reshape(-1)))
        flat_e = idx.reshape(-1)[order]
        flat_t = np.repeat(np.arange(T), K)[order]
        counts = np.bincount(idx.reshape(-1), minlength=E)
        # a row encodes (source rank, token, expert) so its journey can be checked
        send = torch.zeros((T * K, H))
        send[:, 0] = rank
        send[:, 1] = torch.from_numpy(flat_t).float()
        send[:, 2] = torch.from_numpy(flat_e).float()
        recv_counts = torch.empty(world * El, dtype=torch.int64)
        dist.all_to_all_single(recv_counts, torch.from_numpy(counts).long())
        plan = plan_exchange(counts, recv_counts.numpy().reshape(world, El))
        recv = torch.full((plan.recv_rows, H), -1.0)
        exchange_rows(send, recv, plan, rank, world)
        # every received row belongs to one of my experts, in its segment, padding untouched
        for e in range(El):
            lo, hi = plan.seg_offsets[e], plan.seg_offsets[e + 1]
            n = int(plan.recv_counts[:, e].sum())
            seg = recv[lo:hi]
            assert (seg[:n, 2] == rank * El + e).all()
            assert (seg[n:, 0] == -1).all()
            # chunk order: by source rank, tokens ascending within a source
            for s in range(world):
                a = plan.recv_offsets[s, e]
                c = plan.recv_counts[s, e]
                assert (recv[a:a + c, 0] == s).all()
                assert (torch.diff(recv[a:a + c, 1]) > 0).all()
        # the expert stage: add 1000 * (my rank + 1) to column 3, then send back
        y = recv.clone()
        y[:, 3] = 1000.0 * (rank + 1)
        back = torch.zeros_like(send)
        exchange_rows(y, back, plan, rank, world, reverse=True)
        assert torch.equal(back[:, :3], send[:, :3])
        owner = torch.from_numpy(flat_e // El).float()
        assert torch.equal(back[:, 3], 1000.0 * (owner + 1))
        q.put((rank, "ok"))
    except Exception as ex:  # report to the parent
        q.put((rank, repr(ex)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,E,K,T", [(2, 8, 2, 50), (3, 6, 3, 37)])
def test_exchange_round_trip_gloo(world, E, K, T):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, E, K, T, 8, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert all(v == "ok" for v in results.values()), results
