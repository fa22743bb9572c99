"""Expert-parallel exchange logic on CPU gloo ranks (world size 2 and 4).

The decomposition of cti_b200.ep - route locally, dispatch into expert
(= destination rank) order, exchange counts and rows, run the local experts
over (source rank, local expert) groups, send back, combine at the source -
must reproduce the single-process reference layer.  Here the exchange code
is the product's own (cti_b200.ep helpers over torch.distributed / gloo) and
the compute steps are the CPU oracle, so the test needs no GPU.
"""
import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(D, E, F, T, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, D, generator=g)
    wg = torch.randn(E, D, generator=g) * 0.1
    bg = torch.randn(E, generator=g) * 0.5
    w1 = torch.randn(E, F, D, generator=g) * 0.05
    b1 = torch.randn(E, F, generator=g) * 0.05
    w2 = torch.randn(E, D, F, generator=g) * 0.05
    b2 = torch.randn(E, D, generator=g) * 0.05
    return x, wg, bg, w1, b1, w2, b2


def _worker(rank, world, port, splits, seed):
    sys.path.insert(0, str(ROOT))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        import cti_b200.ep as ep
        from oracle import moe_ref as mr

        torch.set_num_threads(1)
        D, E, F = 32, 8, 64
        T = sum(splits)
        x, wg, bg, w1, b1, w2, b2 = _problem(D, E, F, T, seed)
        lo = sum(splits[:rank])
        xl = x[lo:lo + splits[rank]]
        # 1-2: route and dispatch the local tokens (oracle restatement).
        g = mr.gate_ref(xl, wg, bg, renorm=True, tie_lower_id=True)
        offsets, sorted_token, perm_inv = mr.expert_segments(g.idx, E)
        xperm = xl[sorted_token]
        counts = offsets[1:] - offsets[:-1]
        # 3: exchange counts and rows (product code).
        recv_counts = ep.exchange_counts(counts, world)
        send_splits = ep.rank_send_counts(counts, world)
        recv_splits = recv_counts.sum(dim=1).tolist()
        assert sum(send_splits) == 2 * splits[rank]
        rows = ep.exchange_rows(xperm, send_splits, recv_splits)
        offs = ep.received_group_offsets(recv_counts)
        # 4: local experts over (source rank, local expert) groups.
        El = E // world
        y_local = torch.empty_like(rows)
        for grp in range(world * El):
            a, b = int(offs[grp]), int(offs[grp + 1])
            if b > a:
                e = rank * El + grp % El
                y_local[a:b] = mr.expert_ref(rows[a:b], w1[e], b1[e], w2[e], b2[e], "gelu")
        # 5: back to the source rank; 6: combine.
        y = ep.exchange_rows(y_local, recv_splits, send_splits)
        out = (g.score[:, :1] * y[perm_inv[:, 0]] + g.score[:, 1:] * y[perm_inv[:, 1]])
        ref, _ = mr.smoe_ref(x, wg, bg, w1, b1, w2, b2, act="gelu", renorm=True)
        torch.testing.assert_close(out, ref[lo:lo + splits[rank]], rtol=1e-5, atol=1e-6)
        # Every rank receives exactly the routes addressed to its experts.
        full_g = mr.gate_ref(x, wg, bg, renorm=True, tie_lower_id=True)
        mine = ((full_g.idx // El) == rank).sum().item()
        assert rows.shape[0] == mine
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("splits", [[40, 56], [0, 37], [25, 0, 31, 12]])
def test_expert_parallel_exchange_matches_single_process_layer(splits):
    world = len(splits)
    mp.spawn(_worker, args=(world, _free_port(), splits, 7), nprocs=world, join=True)


def test_send_counts_follow_contiguous_expert_blocks():
    import cti_b200.ep as ep

    counts = torch.tensor([3, 0, 5, 1, 2, 2, 0, 7])
    assert ep.rank_send_counts(counts, 2) == [9, 11]
    assert ep.rank_send_counts(counts, 4) == [3, 6, 4, 7]
    offs = ep.received_group_offsets(torch.tensor([[1, 2], [0, 4]]))
    assert offs.tolist() == [0, 1, 3, 3, 7]
