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


def test_balanced_placement_evens_out_zipf_load():
    sys.path.insert(0, str(ROOT))
    import cti_b200.ep as ep
    from cti_b200 import synth

    E = 64
    p = torch.softmax(synth.zipf_router_bias(E, 1.2, seed=0), 0)
    for world in (2, 4, 8):
        place = ep.balanced_placement(p.tolist(), world)
        assert sorted(place) == list(range(E))
        per = E // world
        for r in range(world):
            assert place[r * per:(r + 1) * per] == sorted(place[r * per:(r + 1) * per])
        loads = [float(p[place[r * per:(r + 1) * per]].sum()) for r in range(world)]
        contiguous = [float(p[r * per:(r + 1) * per].sum()) for r in range(world)]
        assert max(loads) <= max(contiguous) + 1e-12
        # LPT bound: max load <= mean + the largest single expert.
        assert max(loads) <= 1.0 / world + float(p.max()) + 1e-12
    with pytest.raises(ValueError):
        ep.balanced_placement([1.0] * 6, 4)


def test_replicated_placement_splits_the_hot_expert():
    sys.path.insert(0, str(ROOT))
    import cti_b200.ep as ep

    load = [47.0, 29.0, 13.0, 5.0, 3.0, 1.0, 1.0, 1.0]
    for world, extra in ((2, 1), (4, 1), (4, 3)):
        S = len(load) // world + extra
        pl = ep.balanced_placement(load, world, S)
        assert len(pl) == world * S and set(pl) == set(range(len(load)))
        n_rep, rep_idx = ep.replica_tables(pl, len(load))
        assert sum(n_rep) == world * S and n_rep[0] > 1
        rank_load = [sum(load[e] / n_rep[e] for e in pl[q * S:(q + 1) * S]) for q in range(world)]
        plain = ep.balanced_placement(load, world)
        plain_load = [sum(load[e] for e in plain[q * (len(load) // world):(q + 1) * (len(load) // world)])
                      for q in range(world)]
        # LPT bound, and at 4 ranks a real gain over the plain placement
        # (at 2 ranks the hot expert is already below half of the load).
        assert max(rank_load) <= sum(load) / world + max(load[e] / n_rep[e] for e in pl) + 1e-9
        if world > 2:
            assert max(rank_load) < max(plain_load)
        # replica shares of a segment cover it exactly, in order
        for c in (0, 1, 7, 100):
            n = n_rep[0]
            parts = [ep.replica_chunk(c, n, i) for i in range(n)]
            assert sum(sz for _, sz in parts) == c
            assert all(parts[i][0] + parts[i][1] == parts[i + 1][0] for i in range(n - 1))


def _layer_worker(rank, world, port, splits, overlap, balanced, extra=0):
    """ExpertParallelSMoE.forward itself on gloo ranks: its compute stages
    (router, dispatch, expert FFN, combine - CUDA kernels in the product)
    are replaced by the CPU oracle, everything else is the product code."""
    sys.path.insert(0, str(ROOT))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        import types

        import cti_b200.ep as ep
        from cti_b200 import ops as real_ops
        from oracle import moe_ref as mr

        torch.set_num_threads(1)
        D, E, F = 32, 8, 64
        T = sum(splits)
        x, wg, bg, w1, b1, w2, b2 = _problem(D, E, F, T, 11)

        def router(x2, wg_, bg_, renorm=True):
            g = mr.gate_ref(x2, wg_, bg_, renorm=renorm, tie_lower_id=True)
            return real_ops.RouterOut(g.idx.int(), g.score.float(), None, None)

        def dispatch(x2, r, n):
            offsets, sorted_token, perm_inv = mr.expert_segments(r.idx2.long(), n)
            return real_ops.DispatchOut(offsets.int(), perm_inv.int(), sorted_token.int(),
                                        x2[sorted_token.long()])

        def combine(y, perm_inv, gate2):
            pi = perm_inv.long()
            return gate2[:, :1] * y[pi[:, 0]] + gate2[:, 1:] * y[pi[:, 1]]

        fake = types.SimpleNamespace(router=router, dispatch=dispatch, combine=combine)
        orig_ops, orig_prep = ep.ops, ep._prepare_x
        ep.ops, ep._prepare_x = fake, lambda t: t.contiguous()
        try:
            placement = None
            if balanced:
                placement = ep.balanced_placement(torch.softmax(bg, 0).tolist(), world,
                                                  E // world + extra)
            m = ep.ExpertParallelSMoE(D, F, E, placement=placement)
            m.load_weights(wg, bg, w1, b1, w2, b2)
            m.prepare_for_inference()

            def ffn_rows(rows, offs, first=0):
                y = torch.empty_like(rows)
                o = offs.long().tolist()
                for grp in range(len(o) - 1):
                    if o[grp + 1] > o[grp]:
                        ex = m.experts[first + grp % (m.local_experts - first)]
                        y[o[grp]:o[grp + 1]] = mr.expert_ref(
                            rows[o[grp]:o[grp + 1]], ex.fc1.weight, ex.fc1.bias,
                            ex.fc2.weight, ex.fc2.bias, "gelu")
                return y

            m._expert_ffn = ffn_rows
            m._ffn_into = lambda rows, offs, out, first_expert=0: out.copy_(
                ffn_rows(rows, offs, first_expert))
            lo = sum(splits[:rank])
            marks = []
            out, aux = m(x[lo:lo + splits[rank]], mark=marks.append, overlap=overlap)
        finally:
            ep.ops, ep._prepare_x = orig_ops, orig_prep
        assert aux is None
        assert marks == ["router", "dispatch", "exchange", "experts", "exchange_back", "combine"]
        ref, _ = mr.smoe_ref(x, wg, bg, w1, b1, w2, b2, act="gelu", renorm=True)
        torch.testing.assert_close(out, ref[lo:lo + splits[rank]], rtol=1e-5, atol=1e-6)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("splits,overlap,balanced,extra", [
    ([40, 56], True, False, 0), ([40, 56], True, True, 0), ([0, 37], True, True, 0),
    ([25, 0, 31, 12], True, True, 0), ([25, 9, 31, 12], False, False, 0),
    ([40, 56], True, True, 2), ([25, 0, 31, 12], True, True, 1), ([30, 30, 30, 30], True, True, 3)])
def test_expert_parallel_layer_forward_on_gloo(splits, overlap, balanced, extra):
    """extra > 0: extra slots per rank, i.e. replicated experts whose rows
    are split over several ranks."""
    world = len(splits)
    mp.spawn(_layer_worker, args=(world, _free_port(), splits, overlap, balanced, extra),
             nprocs=world, join=True)


def test_dispatch_layout_runs():
    sys.path.insert(0, str(ROOT))
    import cti_b200.ep as ep

    # no replicas: one run per rank, dispatch order = the ranks' experts
    slots, order, runs = ep.dispatch_layout([3, 0, 2, 1], 4, 2)
    assert sorted(slots[:2]) == [0, 3] and sorted(slots[2:]) == [1, 2]
    assert order == slots and runs == [[(0, 2)], [(0, 2)]]
    # expert 0 replicated on both ranks: rank 0 keeps it last among its
    # primaries, rank 1 holds the second share as an extra replica
    slots, order, runs = ep.dispatch_layout([0, 1, 2, 0, 3, 4], 5, 2)
    assert slots[:3] == [1, 2, 0] and order[:3] == [1, 2, 0]
    assert runs[0] == [(0, 3)]           # 1, 2 and share 0 of expert 0 are adjacent
    assert len(runs[1]) == 2             # share 1 of expert 0, then experts 3, 4
