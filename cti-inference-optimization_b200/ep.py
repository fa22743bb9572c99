"""Expert-parallel Top-2 MoE across the ranks of a process group.

The reference is single-GPU (SURVEY: no torch.distributed anywhere); this is
the new multi-GPU form of the same layer for the large-expert configuration
(d_model 1024, 64 experts, d_ff 4096): rank r owns experts
[r*E/R, (r+1)*E/R) and its own slice of the packed tokens.

Per forward, on every rank:
  1. route the local tokens with the full fp32 router (stage 1);
  2. dispatch them into expert order (stage 2).  Experts are contiguous per
     rank, so expert order is destination-rank order and the dispatched rows
     form one contiguous segment per destination;
  3. exchange the per-expert row counts (all_to_all_single of int32 counts),
     then the rows themselves (all_to_all_single with uneven splits, NCCL
     over NVLink on GPUs);
  4. run the local experts over the received rows, grouped as (source rank,
     local expert) - group g uses local weight g % (E/R);
  5. send the expert outputs back along the reverse splits;
  6. combine them with the gates at the source rank (stage 4).
Gates and token ids never leave their rank.

The exchange helpers below are plain torch.distributed code and run on any
backend (gloo on CPU in the tests, NCCL on GPUs); the compute steps call the
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


def balanced_placement(expert_load, world: int) -> list[int]:
    """Expert placement that evens out the rows each rank computes.

    expert_load[e] = expected rows of expert e (e.g. routing counts of a
    calibration batch).  Experts are taken heaviest first and each goes to
    the rank with the least load that still has a free slot (longest
    processing time first).  Returns the placement as a slot list: slot s
    holds expert placement[s], and rank r owns slots [r*E/R, (r+1)*E/R),
    each rank's experts in ascending id order."""
    load = [float(v) for v in expert_load]
    E = len(load)
    if E % world:
        raise ValueError("num_experts must be divisible by the number of ranks")
    per = E // world
    bins = [[] for _ in range(world)]
    tot = [0.0] * world
    for e in sorted(range(E), key=lambda i: (-load[i], i)):
        r = min((q for q in range(world) if len(bins[q]) < per), key=lambda q: (tot[q], q))
        bins[r].append(e)
        tot[r] += load[e]
    return [e for b in bins for e in sorted(b)]


class ExpertParallelSMoE(nn.Module):
    """Top-2 MoE whose experts are sharded across a process group.

    ``experts`` holds only this rank's E/R experts: local index j is global
    expert placement[rank*E/R + j] (identity placement by default, i.e.
    contiguous blocks of experts).  ``gate`` is the full router, replicated,
    with its rows stored in slot order, so the router's outputs are slots and
    every rank's slots are contiguous: dispatch in slot order is dispatch in
    destination order.  Routing, gates and outputs are those of the reference
    layer whatever the placement; only when the 2nd and 3rd logits of a token
    are exactly equal can the tie go to a different expert than the lower id.
    ``load_global_state_dict`` takes the state dict of a full ``SMoE``."""

    def __init__(self, d_model: int, dim_ff: int, num_experts: int, group=None,
                 activation: str = "gelu", renormalize: bool = True, placement=None):
        super().__init__()
        self.group = group
        distributed = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if distributed else 1
        self.rank = dist.get_rank(group) if distributed else 0
        if num_experts % self.world != 0:
            raise ValueError("num_experts must be divisible by the number of ranks")
        self.num_experts = num_experts
        self.local_experts = num_experts // self.world
        self.placement = list(range(num_experts)) if placement is None else [int(e) for e in placement]
        if sorted(self.placement) != list(range(num_experts)):
            raise ValueError("placement must be a permutation of the expert ids")
        self.d_model = d_model
        self.dim_ff = dim_ff
        self.activation = activation
        self.gate = TopKGate(d_model, num_experts, renormalize=renormalize)
        self.experts = nn.ModuleList(
            [Expert(d_model, dim_ff, activation) for _ in range(self.local_experts)])
        self._ready = False

    def _owned(self) -> list[int]:
        base = self.rank * self.local_experts
        return self.placement[base:base + self.local_experts]

    @torch.no_grad()
    def load_global_state_dict(self, sd: dict) -> None:
        slots = torch.tensor(self.placement)
        self.gate.w_g.weight.copy_(sd["gate.w_g.weight"][slots])
        self.gate.w_g.bias.copy_(sd["gate.w_g.bias"][slots])
        for j, e in enumerate(self._owned()):
            ex = self.experts[j]
            ex.fc1.weight.copy_(sd[f"experts.{e}.fc1.weight"])
            ex.fc1.bias.copy_(sd[f"experts.{e}.fc1.bias"])
            ex.fc2.weight.copy_(sd[f"experts.{e}.fc2.weight"])
            ex.fc2.bias.copy_(sd[f"experts.{e}.fc2.bias"])
        self._ready = False

    @torch.no_grad()
    def prepare_for_inference(self) -> None:
        dev = self.gate.w_g.weight.device
        self._w1 = torch.stack([e.fc1.weight for e in self.experts]).to(dev, torch.bfloat16).contiguous()
        self._b1 = torch.stack([e.fc1.bias for e in self.experts]).to(dev, torch.float32).contiguous()
        self._w2 = torch.stack([e.fc2.weight for e in self.experts]).to(dev, torch.bfloat16).contiguous()
        self._b2 = torch.stack([e.fc2.bias for e in self.experts]).to(dev, torch.float32).contiguous()
        self._wg, self._bg = self.gate.router_weights()
        self._ready = True

    def _expert_ffn(self, rows: torch.Tensor, group_offsets: torch.Tensor) -> torch.Tensor:
        offs = group_offsets.to(torch.int32)
        if self.d_model in (128, 256) and self.dim_ff <= 1024:
            return ops.expert_ffn_fused(rows, self._w1, self._b1, self._w2, self._b2, offs,
                                        act=self.activation)
        h = ops.grouped_gemm(rows, self._w1, self._b1, offs, act=self.activation)
        return ops.grouped_gemm(h, self._w2, self._b2, offs, act="none")

    @torch.no_grad()
    def load_weights(self, wg, bg, w1, b1, w2, b2) -> None:
        """Global weights in the reference layout (w1 [E, F, D], w2 [E, D, F]);
        keeps this rank's experts."""
        slots = torch.tensor(self.placement, device=wg.device)
        self.gate.w_g.weight.copy_(wg[slots])
        self.gate.w_g.bias.copy_(bg[slots])
        for j, e in enumerate(self._owned()):
            ex = self.experts[j]
            ex.fc1.weight.copy_(w1[e])
            ex.fc1.bias.copy_(b1[e])
            ex.fc2.weight.copy_(w2[e])
            ex.fc2.bias.copy_(b2[e])
        self._ready = False

    def _ffn_into(self, rows: torch.Tensor, offs: torch.Tensor, out: torch.Tensor,
                  first_expert: int = 0) -> None:
        """Expert FFN of the row groups ``offs`` into ``out``; group g uses
        local expert first_expert + g (modulo the local experts)."""
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

    @torch.no_grad()
    def forward(self, x: torch.Tensor, mark=None, overlap: bool = True):
        """x [..., D] bf16 (this rank's tokens) -> (out like x, None).

        With ``overlap`` the rows exchange is point-to-point per peer and
        runs while the local experts compute the rows this rank routed to
        itself; the results for the peers go back the same way and land
        directly in the expert-ordered output buffer.  Without it the
        exchange is two plain all_to_all calls around one expert pass.

        ``mark(name)``, when given, is called after each stage is enqueued
        (router, dispatch, exchange, experts, exchange_back, combine); the
        benchmark uses it to record CUDA events between stages."""
        shape = x.shape
        x2 = _prepare_x(x).reshape(-1, shape[-1])
        if not self._ready:
            self.prepare_for_inference()
        mark = mark or (lambda name: None)
        E, R, El, me = self.num_experts, self.world, self.local_experts, self.rank
        r = ops.router(x2, self._wg, self._bg, renorm=self.gate.renormalize)
        mark("router")
        d = ops.dispatch(x2, r, E)
        mark("dispatch")
        if R == 1:
            mark("exchange")
            y = self._expert_ffn(d.xperm, d.offsets) if d.xperm.shape[0] > 0 else d.xperm
            mark("experts")
            mark("exchange_back")
        else:
            counts = d.offsets[1:] - d.offsets[:-1]
            recv_counts = exchange_counts(counts, R, self.group)
            # The row splits must be known on the host.
            both = torch.cat([counts.to(torch.int64), recv_counts.reshape(-1)]).cpu()
            counts_h, recv_h = both[:E], both[E:].view(R, El)
            send_splits = counts_h.view(R, El).sum(dim=1).tolist()
            recv_splits = recv_h.sum(dim=1).tolist()
            if not overlap:
                rows = exchange_rows(d.xperm, send_splits, recv_splits, self.group)
                mark("exchange")
                y_local = (self._expert_ffn(rows, received_group_offsets(recv_counts))
                           if rows.shape[0] > 0 else rows)
                mark("experts")
                y = exchange_rows(y_local, recv_splits, send_splits, self.group)
                mark("exchange_back")
            else:
                y = self._forward_overlapped(d, recv_counts, send_splits, recv_splits,
                                             counts_h, mark)
        out = ops.combine(y, d.perm_inv, r.gate2)
        mark("combine")
        return out.reshape(shape), None

    def _forward_overlapped(self, d, recv_counts, send_splits, recv_splits, counts_h, mark):
        """Shift-ordered pipeline over the peers.  Step s (1 <= s < R) sends
        to rank me+s and receives from rank me-s, so every pair of ranks
        meets in the same step.  All row transfers are posted first; the
        experts then work through the received blocks in step order, and
        each block's results are posted back to their source as soon as
        they are computed, so the return of block s overlaps the compute of
        block s+1.  The rows this rank routed to itself need no transfer:
        half of them are computed while the first blocks arrive, the other
        half while the last results travel back."""
        R, El, me = self.world, self.local_experts, self.rank
        so, ro = _prefix(send_splits), _prefix(recv_splits)
        rows = d.xperm.new_empty((ro[-1], self.d_model))
        y_remote = torch.empty_like(rows)
        y = torch.empty_like(d.xperm)
        send_blk = split_views(d.xperm, send_splits)
        recv_blk = split_views(rows, recv_splits)
        arrivals = {}
        for step in range(1, R):
            dst, src = (me + step) % R, (me - step) % R
            arrivals[step] = post_pair(send_blk[dst], dst, recv_blk[src], src, self.group)
        mark("exchange")
        # Own rows, split at an expert boundary into two halves by rows.
        own = counts_h[me * El:(me + 1) * El].tolist()
        cut = _balanced_cut(own)
        base = so[me]
        o_own = _prefix(own)
        self_offs = d.offsets[me * El:(me + 1) * El + 1] - d.offsets[me * El]
        self._ffn_into(d.xperm[base:base + o_own[cut]], self_offs[:cut + 1],
                       y[base:base + o_own[cut]])
        returns = []
        for step in range(1, R):
            dst, src = (me + step) % R, (me - step) % R
            for w in arrivals[step]:
                w.wait()
            blk = slice(ro[src], ro[src + 1])
            self._ffn_into(rows[blk], received_group_offsets(recv_counts[src:src + 1]),
                           y_remote[blk])
            returns.append(post_pair(y_remote[blk], src, y[so[dst]:so[dst + 1]], dst, self.group))
        self._ffn_into(d.xperm[base + o_own[cut]:base + o_own[-1]],
                       self_offs[cut:] - self_offs[cut], y[base + o_own[cut]:base + o_own[-1]],
                       first_expert=cut)
        mark("experts")
        for ws in returns:
            for w in ws:
                w.wait()
        mark("exchange_back")
        return y
