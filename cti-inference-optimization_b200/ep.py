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


def received_group_offsets(recv_counts: torch.Tensor) -> torch.Tensor:
    """Group offsets [R*El + 1] of the received rows, which arrive ordered by
    source rank, then by local expert (the senders' expert order)."""
    flat = recv_counts.reshape(-1).to(torch.int64)
    offs = torch.zeros(flat.numel() + 1, dtype=torch.int64, device=flat.device)
    offs[1:] = torch.cumsum(flat, 0)
    return offs


class ExpertParallelSMoE(nn.Module):
    """Top-2 MoE whose experts are sharded across a process group.

    ``experts`` holds only this rank's E/R experts (local index j is global
    expert rank*E/R + j); ``gate`` is the full router, replicated.
    ``load_global_state_dict`` takes the state dict of a full ``SMoE``."""

    def __init__(self, d_model: int, dim_ff: int, num_experts: int, group=None,
                 activation: str = "gelu", renormalize: bool = True):
        super().__init__()
        self.group = group
        distributed = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if distributed else 1
        self.rank = dist.get_rank(group) if distributed else 0
        if num_experts % self.world != 0:
            raise ValueError("num_experts must be divisible by the number of ranks")
        self.num_experts = num_experts
        self.local_experts = num_experts // self.world
        self.d_model = d_model
        self.dim_ff = dim_ff
        self.activation = activation
        self.gate = TopKGate(d_model, num_experts, renormalize=renormalize)
        self.experts = nn.ModuleList(
            [Expert(d_model, dim_ff, activation) for _ in range(self.local_experts)])
        self._ready = False

    @torch.no_grad()
    def load_global_state_dict(self, sd: dict) -> None:
        self.gate.w_g.weight.copy_(sd["gate.w_g.weight"])
        self.gate.w_g.bias.copy_(sd["gate.w_g.bias"])
        base = self.rank * self.local_experts
        for j, ex in enumerate(self.experts):
            for name in ("fc1.weight", "fc1.bias", "fc2.weight", "fc2.bias"):
                getattr(getattr(ex, name.split(".")[0]), name.split(".")[1]).copy_(
                    sd[f"experts.{base + j}.{name}"])
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
        self.gate.w_g.weight.copy_(wg)
        self.gate.w_g.bias.copy_(bg)
        base = self.rank * self.local_experts
        for j, ex in enumerate(self.experts):
            ex.fc1.weight.copy_(w1[base + j])
            ex.fc1.bias.copy_(b1[base + j])
            ex.fc2.weight.copy_(w2[base + j])
            ex.fc2.bias.copy_(b2[base + j])
        self._ready = False

    @torch.no_grad()
    def forward(self, x: torch.Tensor, mark=None):
        """x [..., D] bf16 (this rank's tokens) -> (out like x, None).

        ``mark(name)``, when given, is called after each stage is enqueued
        (router, dispatch, exchange, experts, exchange_back, combine); the
        benchmark uses it to record CUDA events between stages."""
        shape = x.shape
        x2 = _prepare_x(x).reshape(-1, shape[-1])
        if not self._ready:
            self.prepare_for_inference()
        mark = mark or (lambda name: None)
        E, R = self.num_experts, self.world
        r = ops.router(x2, self._wg, self._bg, renorm=self.gate.renormalize)
        mark("router")
        d = ops.dispatch(x2, r, E)
        mark("dispatch")
        if R > 1:
            counts = d.offsets[1:] - d.offsets[:-1]
            recv_counts = exchange_counts(counts, R, self.group)
            # The row splits must be known on the host (uneven all_to_all).
            both = torch.cat([counts.to(torch.int64), recv_counts.reshape(-1)]).cpu()
            counts_h, recv_h = both[:E], both[E:].view(R, E // R)
            send_splits = counts_h.view(R, E // R).sum(dim=1).tolist()
            recv_splits = recv_h.sum(dim=1).tolist()
            rows = exchange_rows(d.xperm, send_splits, recv_splits, self.group)
            offs = received_group_offsets(recv_counts)
        else:
            rows, offs = d.xperm, d.offsets
        mark("exchange")
        y_local = self._expert_ffn(rows, offs) if rows.shape[0] > 0 else rows
        mark("experts")
        if R > 1:
            y = exchange_rows(y_local, recv_splits, send_splits, self.group)
        else:
            y = y_local
        mark("exchange_back")
        out = ops.combine(y, d.perm_inv, r.gate2)
        mark("combine")
        return out.reshape(shape), None
