"""Expert-parallel Top-2 MoE across the ranks of a process group.

The reference runs on one GPU and has no torch.distributed anywhere; this is
the multi-GPU form of the same layer for the large-expert configuration
(d_model 1024, 64 experts, d_ff 4096).  Every rank holds its own slice of the
packed tokens and S expert slots; an expert may hold several slots on
different ranks (replicas), which splits its rows between them.

Per forward, on every rank:
  1. route the local tokens with the full fp32 router (stage 1), whose rows
     are stored in dispatch order (``dispatch_layout``): each rank's experts
     are consecutive;
  2. dispatch them into that order (stage 2), so the rows for one
     destination are a few contiguous runs (one without replicas);
  3. exchange the per-slot row counts (all_to_all_single; one host read of
     all counts gives the splits), then the rows, point to point, all peers
     in one NCCL group;
  4. run the local experts over the rows this rank routed to itself (while
     the rows travel) and over the received rows, grouped as (source rank,
     local slot) - group g uses local slot g % S;
  5. send the expert outputs back in two all-peer groups that overlap the
     remaining compute, straight into the expert-ordered output buffer;
  6. combine them with the gates at the source rank (stage 4).
Gates and token ids never leave their rank.

The exchange code is plain torch.distributed and runs on any backend (gloo
on CPU in the tests, NCCL over NVLink on GPUs); the compute steps call the
sm_100a kernels.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn

from . import ops
from .moe import Expert, TopKGate, _prepare_x


# ---------------------------------------------------------------------------
# exchange helpers (device agnostic)
# ---------------------------------------------------------------------------
def rank_send_counts(expert_counts: torch.Tensor, world: int) -> list[int]:
    """Rows this rank sends to each destination: its per-expert counts summed
    over each destination's contiguous block of experts."""
    E = expert_counts.numel()
    return expert_counts.view(world, E // world).sum(dim=1).tolist()


def exchange_counts(expert_counts: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """all_to_all of the [E] per-expert counts: returns recv [world, E/world],
    row q = how many rows source rank q sends to each of this rank's experts."""
    E = expert_counts.numel()
    send = expert_counts.to(torch.int64).contiguous()
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return recv.view(world, E // world)


def exchange_rows(send: torch.Tensor, send_splits: list[int], recv_splits: list[int],
                  group=None) -> torch.Tensor:
    """all_to_all of row blocks with uneven splits (rows, not bytes)."""
    recv = send.new_empty((sum(recv_splits),) + tuple(send.shape[1:]))
    dist.all_to_all_single(recv, send.contiguous(), output_split_sizes=recv_splits,
                           input_split_sizes=send_splits, group=group)
    return recv


def _prefix(splits: list[int]) -> list[int]:
    out = [0]
    for v in splits:
        out.append(out[-1] + int(v))
    return out


def split_views(t: torch.Tensor, splits: list[int]) -> list[torch.Tensor]:
    """Consecutive row blocks of t (views, no copies)."""
    o = _prefix(splits)
    return [t[o[q]:o[q + 1]] for q in range(len(splits))]


def post_exchange(send_blocks: list[torch.Tensor], recv_blocks: list[torch.Tensor], me: int,
                  group=None) -> list:
    """Point-to-point exchange of row blocks with every peer: block q of
    send_blocks goes to rank q and block q of recv_blocks is filled by rank
    q.  The block for this rank itself is skipped, and so is every empty
    block (both sides know the sizes).  Returns the pending requests; their
    wait() orders the caller's stream after the transfer."""
    p2p = []
    for q in range(len(send_blocks)):
        if q == me:
            continue
        peer = _global(group, q)
        if recv_blocks[q].shape[0] > 0:
            p2p.append(dist.P2POp(dist.irecv, recv_blocks[q], peer, group))
        if send_blocks[q].shape[0] > 0:
            p2p.append(dist.P2POp(dist.isend, send_blocks[q].contiguous(), peer, group))
    return dist.batch_isend_irecv(p2p) if p2p else []


def post_pair(send: torch.Tensor, dst: int, recv: torch.Tensor, src: int, group=None) -> list:
    """One pipeline step: send rows to rank dst and receive rows from rank
    src in one NCCL group (either side skipped when it has no rows).
    Returns the pending requests."""
    p2p = []
    if recv.shape[0] > 0:
        p2p.append(dist.P2POp(dist.irecv, recv, _global(group, src), group))
    if send.shape[0] > 0:
        p2p.append(dist.P2POp(dist.isend, send, _global(group, dst), group))
    return dist.batch_isend_irecv(p2p) if p2p else []


def _global(group, q: int) -> int:
    return dist.get_global_rank(group, q) if group is not None else q


def _balanced_cut(sizes: list[int]) -> int:
    """Group boundary k (0..len) that splits sum(sizes) closest to half."""
    total, acc, best, best_k = sum(sizes), 0, None, 0
    for k in range(len(sizes) + 1):
        gap = abs(2 * acc - total)
        if best is None or gap < best:
            best, best_k = gap, k
        if k < len(sizes):
            acc += sizes[k]
    return best_k


def received_group_offsets(recv_counts: torch.Tensor) -> torch.Tensor:
    """Group offsets [R*El + 1] of the received rows, which arrive ordered by
    source rank, then by local expert (the senders' expert order)."""
    flat = recv_counts.reshape(-1).to(torch.int64)
    offs = torch.zeros(flat.numel() + 1, dtype=torch.int64, device=flat.device)
    offs[1:] = torch.cumsum(flat, 0)
    return offs


def balanced_placement(expert_load, world: int, slots_per_rank: int | None = None) -> list[int]:
    """Expert placement that evens out the rows each rank computes.

    expert_load[e] = expected rows of expert e (e.g. routing counts of a
    calibration batch).  Every rank gets ``slots_per_rank`` slots (default
    E / world, i.e. no replication).  With more slots than experts, the
    spare slots become replicas: each goes to the expert with the largest
    load per replica, and an expert's rows are split evenly over its
    replicas.  Replicas are then packed heaviest first onto the rank with the
    least load that has a free slot and does not hold that expert yet
    (longest processing time first), and pairwise swaps then lower the
    busiest rank's load while they can.  Returns the slot list: slot
    q*slots_per_rank + j is rank q's local slot j, holding the returned
    expert id; each rank's experts in ascending id order."""
    load = [float(v) for v in expert_load]
    E = len(load)
    S = E // world if slots_per_rank is None else int(slots_per_rank)
    if S * world < E or (slots_per_rank is None and E % world):
        raise ValueError("need at least num_experts slots in total, divisible by the ranks")
    n = [1] * E
    for _ in range(S * world - E):
        e = max(range(E), key=lambda i: (load[i] / n[i], -i))
        n[e] += 1
    reps = sorted(((load[e] / n[e], e) for e in range(E) for _ in range(n[e])),
                  key=lambda t: (-t[0], t[1]))
    bins = [[] for _ in range(world)]
    tot = [0.0] * world
    for w, e in reps:
        free = [q for q in range(world) if len(bins[q]) < S]
        fresh = [q for q in free if e not in bins[q]]
        r = min(fresh or free, key=lambda q: (tot[q], q))
        bins[r].append(e)
        tot[r] += w
    # Pairwise swaps between the busiest rank and the others while they
    # lower the larger of the two loads (bounded; never doubles an expert up).
    share = [load[e] / n[e] for e in range(E)]
    for _ in range(4 * E * world):
        qm = max(range(world), key=lambda q: (tot[q], -q))
        best = None
        for q in range(world):
            if q == qm:
                continue
            for a in set(bins[qm]):
                for b in set(bins[q]):
                    delta = share[a] - share[b]
                    if delta <= 0 or a in bins[q] or b in bins[qm]:
                        continue
                    new_max = max(tot[qm] - delta, tot[q] + delta)
                    if new_max < tot[qm] - 1e-12 and (best is None or new_max < best[0]):
                        best = (new_max, q, a, b, delta)
        if best is None:
            break
        _, q, a, b, delta = best
        bins[qm].remove(a)
        bins[qm].append(b)
        bins[q].remove(b)
        bins[q].append(a)
        tot[qm] -= delta
        tot[q] += delta
    return [e for b in bins for e in sorted(b)]


def dispatch_layout(placement: list[int], num_experts: int, world: int):
    """Orders a slot list for the exchange.

    Returns (slots, order, runs):
      * slots: the same experts per rank, each rank's slots reordered so that
        its primary experts (first occurrence in rank order) come first -
        replicated primaries last among them - then its extra replicas;
      * order: the dispatch order of the experts (order[p] = expert at
        position p): the ranks' primaries in rank and slot order.  The router
        rows are stored in this order, so the rows one rank sends to another
        are few contiguous ranges of the dispatched rows;
      * runs[q]: rank q's slots as maximal intervals [j0, j1) whose replica
        shares are adjacent in the dispatched rows (each expert's segment is
        split into its replicas' shares in replica order) - one
        point-to-point transfer per run and peer, the same structure on the
        sending and the receiving side."""
    E = num_experts
    S = len(placement) // world
    seen, primary = set(), []
    for k, e in enumerate(placement):
        primary.append(e not in seen)
        seen.add(e)
    count = {}
    for e in placement:
        count[e] = count.get(e, 0) + 1
    slots = []
    for q in range(world):
        ks = range(q * S, (q + 1) * S)
        ks = sorted(ks, key=lambda k: (not primary[k], primary[k] and count[placement[k]] > 1,
                                       placement[k]))
        slots += [placement[k] for k in ks]
    # primaries keep their rank after the reorder (first occurrence per expert)
    order, seen = [], set()
    for e in slots:
        if e not in seen:
            order.append(e)
            seen.add(e)
    if len(order) != E:
        raise ValueError("every expert needs at least one slot")
    n_rep, rep_idx = replica_tables(slots, E)
    pos = {e: p for p, e in enumerate(order)}
    first = [0] * E  # index of each expert's first share in the sequence of shares
    acc = 0
    for e in order:
        first[e] = acc
        acc += n_rep[e]
    seq = [first[e] + i for e, i in zip(slots, rep_idx)]
    runs = []
    for q in range(world):
        rq, j0 = [], 0
        for j in range(1, S + 1):
            if j == S or seq[q * S + j] != seq[q * S + j - 1] + 1:
                rq.append((j0, j))
                j0 = j
        runs.append(rq)
    return slots, order, runs


def replica_tables(placement: list[int], num_experts: int):
    """For a slot list: n_rep[e] (replicas of expert e) and, per slot, its
    replica index among the slots holding the same expert (slot order)."""
    n_rep = [0] * num_experts
    rep_idx = []
    for e in placement:
        rep_idx.append(n_rep[e])
        n_rep[e] += 1
    if min(n_rep) < 1:
        raise ValueError("every expert needs at least one slot")
    return n_rep, rep_idx


def replica_chunk(count: int, n: int, i: int) -> tuple[int, int]:
    """(start, size) of replica i's share of an expert segment of `count`
    rows split over n replicas: the first count % n shares get one row more."""
    q, rem = divmod(count, n)
    return i * q + min(i, rem), q + (1 if i < rem else 0)


class ExpertParallelSMoE(nn.Module):
    """Top-2 MoE whose experts are sharded, and optionally replicated, across a
    process group.

    ``placement`` is a slot list of world * S entries: rank q's local slot j
    holds expert placement[q*S + j] (default: contiguous blocks of E/world
    experts, no replication).  An expert may hold several slots; its rows
    are then split evenly over them (``replica_chunk``), which is how one
    expert that draws half of the routes stops bounding the whole layer.
    ``experts`` holds this rank's S slots; ``gate`` is the full router,
    replicated on every rank, in expert order - routing, gates and outputs
    are the reference layer's whatever the placement.
    ``load_global_state_dict`` takes the state dict of a full ``SMoE``."""

    def __init__(self, d_model: int, dim_ff: int, num_experts: int, group=None,
                 activation: str = "gelu", renormalize: bool = True, placement=None):
        super().__init__()
        self.group = group
        distributed = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if distributed else 1
        self.rank = dist.get_rank(group) if distributed else 0
        E = num_experts
        if placement is None:
            if E % self.world != 0:
                raise ValueError("num_experts must be divisible by the number of ranks")
            placement = list(range(E))
        placement = [int(e) for e in placement]
        if len(placement) % self.world or any(not 0 <= e < E for e in placement):
            raise ValueError("placement must list world * S expert ids")
        self.num_experts = E
        self.placement, self.order, self.runs = dispatch_layout(placement, E, self.world)
        self.slots_per_rank = len(placement) // self.world
        self.local_experts = self.slots_per_rank
        self.n_rep, self.rep_idx = replica_tables(self.placement, E)
        self.position = [0] * E  # dispatch position of each expert
        for p, e in enumerate(self.order):
            self.position[e] = p
        self.d_model = d_model
        self.dim_ff = dim_ff
        self.activation = activation
        self.gate = TopKGate(d_model, E, renormalize=renormalize)
        self.experts = nn.ModuleList(
            [Expert(d_model, dim_ff, activation) for _ in range(self.slots_per_rank)])
        self._ready = False

    def _owned(self) -> list[int]:
        S = self.slots_per_rank
        return self.placement[self.rank * S:(self.rank + 1) * S]

    @property
    def contiguous(self) -> bool:
        """True when every rank's slots form one run (no replicas): each
        rank's rows are one block of the dispatched rows."""
        return len(self.placement) == self.num_experts and all(len(r) == 1 for r in self.runs)

    @torch.no_grad()
    def load_global_state_dict(self, sd: dict) -> None:
        order = torch.tensor(self.order)
        self.gate.w_g.weight.copy_(sd["gate.w_g.weight"][order])
        self.gate.w_g.bias.copy_(sd["gate.w_g.bias"][order])
        for j, e in enumerate(self._owned()):
            ex = self.experts[j]
            ex.fc1.weight.copy_(sd[f"experts.{e}.fc1.weight"])
            ex.fc1.bias.copy_(sd[f"experts.{e}.fc1.bias"])
            ex.fc2.weight.copy_(sd[f"experts.{e}.fc2.weight"])
            ex.fc2.bias.copy_(sd[f"experts.{e}.fc2.bias"])
        self._ready = False

    @torch.no_grad()
    def load_weights(self, wg, bg, w1, b1, w2, b2) -> None:
        """Global weights in the reference layout (w1 [E, F, D], w2 [E, D, F]);
        keeps the experts of this rank's slots.  The router rows are stored in
        dispatch order, so the router's outputs are dispatch positions."""
        order = torch.tensor(self.order, device=wg.device)
        self.gate.w_g.weight.copy_(wg[order])
        self.gate.w_g.bias.copy_(bg[order])
        for j, e in enumerate(self._owned()):
            ex = self.experts[j]
            ex.fc1.weight.copy_(w1[e])
            ex.fc1.bias.copy_(b1[e])
            ex.fc2.weight.copy_(w2[e])
            ex.fc2.bias.copy_(b2[e])
        self._ready = False

    @torch.no_grad()
    def prepare_for_inference(self) -> None:
        dev = self.gate.w_g.weight.device
        self._w1 = torch.stack([e.fc1.weight for e in self.experts]).to(dev, torch.bfloat16).contiguous()
        self._b1 = torch.stack([e.fc1.bias for e in self.experts]).to(dev, torch.float32).contiguous()
        self._w2 = torch.stack([e.fc2.weight for e in self.experts]).to(dev, torch.bfloat16).contiguous()
        self._b2 = torch.stack([e.fc2.bias for e in self.experts]).to(dev, torch.float32).contiguous()
        self._wg, self._bg = self.gate.router_weights()
        self._slot_pos = torch.tensor([self.position[e] for e in self.placement],
                                      dtype=torch.int64, device=dev)
        self._slot_nrep = torch.tensor([self.n_rep[e] for e in self.placement], dtype=torch.int64,
                                       device=dev)
        self._slot_rep = torch.tensor(self.rep_idx, dtype=torch.int64, device=dev)
        self._ready = True

    def _ffn_into(self, rows: torch.Tensor, offs: torch.Tensor, out: torch.Tensor,
                  first_expert: int = 0) -> None:
        """Expert FFN of the row groups ``offs`` into ``out``; group g uses
        local slot first_expert + g (modulo the local slots)."""
        if rows.shape[0] == 0:
            return
        offs = offs.to(torch.int32)
        w1, b1 = self._w1[first_expert:], self._b1[first_expert:]
        w2, b2 = self._w2[first_expert:], self._b2[first_expert:]
        if self.d_model in (128, 256) and self.dim_ff <= 1024:
            ops.expert_ffn_fused(rows, w1, b1, w2, b2, offs, act=self.activation, out=out)
            return
        h = ops.grouped_gemm(rows, w1, b1, offs, act=self.activation)
        ops.grouped_gemm(h, w2, b2, offs, act="none", out=out)

    def _expert_ffn(self, rows: torch.Tensor, group_offsets: torch.Tensor) -> torch.Tensor:
        out = torch.empty_like(rows)
        self._ffn_into(rows, group_offsets, out)
        return out

    def slot_counts(self, expert_counts: torch.Tensor) -> torch.Tensor:
        """Rows this rank sends to every slot [world * S] (int64, on the
        device): each expert's count (indexed by dispatch position) split
        over its replicas."""
        c = expert_counts.to(torch.int64)[self._slot_pos]
        n = self._slot_nrep
        return c // n + (self._slot_rep < c % n).to(torch.int64)

    @torch.no_grad()
    def forward(self, x: torch.Tensor, mark=None, overlap: bool = True):
        """x [..., D] bf16 (this rank's tokens) -> (out like x, None).

        With ``overlap`` the rows exchange is point-to-point per peer and
        slot and runs while the local experts compute the rows this rank
        routed to its own slots; the results for the peers go back the same
        way and land directly in the expert-ordered output buffer.  Without
        it (contiguous placement only) the exchange is two plain all_to_all
        calls around one expert pass.

        ``mark(name)``, when given, is called after each stage is enqueued
        (router, dispatch, exchange, experts, exchange_back, combine); the
        benchmark uses it to record CUDA events between stages."""
        shape = x.shape
        x2 = _prepare_x(x).reshape(-1, shape[-1])
        if not self._ready:
            self.prepare_for_inference()
        mark = mark or (lambda name: None)
        E, R, S = self.num_experts, self.world, self.slots_per_rank
        r = ops.router(x2, self._wg, self._bg, renorm=self.gate.renormalize)
        mark("router")
        d = ops.dispatch(x2, r, E)
        mark("dispatch")
        if R == 1 and self.contiguous:
            mark("exchange")
            y = self._expert_ffn(d.xperm, d.offsets) if d.xperm.shape[0] > 0 else d.xperm
            mark("experts")
            mark("exchange_back")
        else:
            counts = d.offsets[1:] - d.offsets[:-1]
            send = self.slot_counts(counts)
            recv = torch.empty_like(send)
            if R > 1:
                dist.all_to_all_single(recv, send, group=self.group)
            else:
                recv.copy_(send)
            # The row splits must be known on the host (one read of all counts).
            both = torch.cat([counts.to(torch.int64), send, recv]).cpu()
            counts_h = both[:E].tolist()
            send_h = both[E:E + R * S].view(R, S).tolist()
            recv_h = both[E + R * S:].view(R, S).tolist()
            if not overlap:
                if not self.contiguous:
                    raise ValueError("the all_to_all exchange needs the contiguous placement")
                send_splits = [sum(v) for v in send_h]
                recv_splits = [sum(v) for v in recv_h]
                rows = exchange_rows(d.xperm, send_splits, recv_splits, self.group)
                mark("exchange")
                y_local = (self._expert_ffn(rows, received_group_offsets(recv.view(R, S)))
                           if rows.shape[0] > 0 else rows)
                mark("experts")
                y = exchange_rows(y_local, recv_splits, send_splits, self.group)
                mark("exchange_back")
            else:
                y = self._forward_overlapped(d, counts_h, send, recv, send_h, recv_h, mark)
        out = ops.combine(y, d.perm_inv, r.gate2)
        mark("combine")
        return out.reshape(shape), None

    def _send_ranges(self, counts_h: list[int], send_h: list[list[int]]):
        """(start, size) in the expert-ordered rows of what goes to each
        (rank, slot): the slot's replica share of its expert's segment."""
        off = _prefix(counts_h)
        S = self.slots_per_rank
        out = []
        for q in range(self.world):
            row = []
            for j in range(S):
                k = q * S + j
                e = self.placement[k]
                p = self.position[e]
                st, sz = replica_chunk(counts_h[p], self.n_rep[e], self.rep_idx[k])
                assert sz == send_h[q][j]
                row.append((off[p] + st, sz))
            out.append(row)
        return out

    def _forward_overlapped(self, d, counts_h, send, recv, send_h, recv_h, mark):
        """The exchange around the experts, overlapped with their compute.

        Transfers are point-to-point, one op per non-empty run of slot shares
        (``dispatch_layout``; a single run per peer without replicas).  All
        outbound rows go in ONE NCCL group over every peer, so all NVSwitch
        links carry their share at once; meanwhile the experts compute the
        first half of the rows this rank routed to its own slots (no transfer
        needed).  Then the received blocks are computed, and their results go
        back in two all-peer groups: the first while the second half of the
        blocks is computed, the second while the other half of the own rows
        is.  Returned rows land directly in the expert-ordered output buffer.
        Every rank posts the same groups in the same order, so the ops of
        each pair of ranks match one to one."""
        R, S, me, D = self.world, self.slots_per_rank, self.rank, self.d_model
        ranges = self._send_ranges(counts_h, send_h)
        blk = [sum(recv_h[q]) if q != me else 0 for q in range(R)]
        bo = _prefix(blk)
        rows = d.xperm.new_empty((bo[-1], D))
        y_remote = torch.empty_like(rows)
        y = torch.empty_like(d.xperm)
        recv_counts = recv.view(R, S)

        def run_views(buf, base, sizes, q):
            # one view per run of q's slots: contiguous in buf from `base`
            o = _prefix(sizes)
            return [buf[base + o[j0]:base + o[j1]] for j0, j1 in self.runs[q]]

        def send_views(q):
            # one view per run of q's slots in the dispatched rows
            return [d.xperm[ranges[q][j0][0]:ranges[q][j0][0] + sum(n for _, n in ranges[q][j0:j1])]
                    for j0, j1 in self.runs[q]]

        def post_all(pairs):
            """One NCCL group over several peers: pairs of (sends, dst, recvs, src)."""
            p2p = []
            for sends, dst, recvs, src in pairs:
                for v in recvs:
                    if v.shape[0] > 0:
                        p2p.append(dist.P2POp(dist.irecv, v, _global(self.group, src), self.group))
                for v in sends:
                    if v.shape[0] > 0:
                        p2p.append(dist.P2POp(dist.isend, v, _global(self.group, dst), self.group))
            return dist.batch_isend_irecv(p2p) if p2p else []

        # All outbound rows in one group: every peer link carries its share at
        # the same time (NVSwitch gives each pair full bandwidth).
        steps = list(range(1, R))
        arrivals = post_all([(send_views((me + s) % R), (me + s) % R,
                              run_views(rows, bo[(me - s) % R], recv_h[(me - s) % R], me),
                              (me - s) % R) for s in steps])
        mark("exchange")
        # Own slots: gathered into one block unless they are already one.
        own = ranges[me]
        own_sizes = [n for _, n in own]
        contiguous_own = all(own[j][0] + own[j][1] == own[j + 1][0] for j in range(S - 1))
        if contiguous_own:
            own_rows = d.xperm[own[0][0]:own[0][0] + sum(own_sizes)]
            own_out = y[own[0][0]:own[0][0] + sum(own_sizes)]
        else:
            own_rows = torch.cat([d.xperm[a:a + n] for a, n in own]) if sum(own_sizes) else \
                d.xperm[:0]
            own_out = torch.empty_like(own_rows)
        own_offs = torch.zeros(S + 1, dtype=torch.int64, device=rows.device)
        own_offs[1:] = torch.cumsum(send.view(R, S)[me], 0)
        cut = _balanced_cut(own_sizes)
        o_own = _prefix(own_sizes)
        self._ffn_into(own_rows[:o_own[cut]], own_offs[:cut + 1], own_out[:o_own[cut]])
        for w in arrivals:
            w.wait()
        # Remote blocks; their results go back in two groups, the first while
        # the second half of the blocks is computed.
        returns = []
        half = (len(steps) + 1) // 2
        for part in (steps[:half], steps[half:]):
            for s_ in part:
                src = (me - s_) % R
                b = slice(bo[src], bo[src + 1])
                self._ffn_into(rows[b], received_group_offsets(recv_counts[src:src + 1]),
                               y_remote[b])
            returns += post_all([
                (run_views(y_remote, bo[(me - s_) % R], recv_h[(me - s_) % R], me), (me - s_) % R,
                 [y[ranges[(me + s_) % R][j0][0]:ranges[(me + s_) % R][j0][0] +
                    sum(n for _, n in ranges[(me + s_) % R][j0:j1])]
                  for j0, j1 in self.runs[(me + s_) % R]], (me + s_) % R)
                for s_ in part])
        self._ffn_into(own_rows[o_own[cut]:], own_offs[cut:] - own_offs[cut],
                       own_out[o_own[cut]:], first_expert=cut)
        if not contiguous_own:
            for (a, n), o in zip(own, o_own[:-1]):
                if n:
                    y[a:a + n].copy_(own_out[o:o + n])
        mark("experts")
        for w in returns:
            w.wait()
        mark("exchange_back")
        return y
