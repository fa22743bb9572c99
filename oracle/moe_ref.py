"""Restatement of the reference Top-2 MoE layer on CPU (fp32).  TEST ONLY.

Follows baseline/infer.py:
  TopKGate.forward  :298-309  logits = w_g(x); probs = softmax; topk(2)
  SMoE.forward      :323-353  per expert: (idx == e).nonzero() -> gather
                              rows -> Expert -> out[token_idx] += y * weight
  Expert.forward    :286-287  fc2(act(fc1(x)))
with the benchmark-configuration semantics as options:
  act="gelu"          exact-erf GELU instead of ReLU (:287),
  renorm=True         top-2 scores divided by their sum (:309 returns raw),
  tie_lower_id=True   stable descending sort, so exact ties go to the lower
                      expert id (torch.topk on CPU does not guarantee that).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F


@dataclass
class GateRef:
    idx: torch.Tensor  # [T, 2] int64
    score: torch.Tensor  # [T, 2] fp32
    probs: torch.Tensor  # [T, E] fp32


def gate_ref(x: torch.Tensor, wg: torch.Tensor, bg: torch.Tensor, renorm: bool = True,
             tie_lower_id: bool = True, force_idx: torch.Tensor | None = None) -> GateRef:
    """baseline/infer.py:298-309 (eval mode: no gating noise).  With
    `force_idx` [T, 2] the top-2 experts are taken from it instead of chosen
    (the scores are still this gate's probabilities of those experts): the
    end-to-end check runs the oracle on the routes the device chose."""
    logits = F.linear(x.float(), wg.float(), bg.float())
    probs = torch.softmax(logits, dim=-1)
    if force_idx is not None:
        order = force_idx.long()
        score = probs.gather(-1, order)
    elif tie_lower_id:
        order = torch.sort(probs, dim=-1, descending=True, stable=True).indices[..., :2]
        score = probs.gather(-1, order)
    else:
        score, order = torch.topk(probs, 2, dim=-1)
    if renorm:
        score = score / score.sum(dim=-1, keepdim=True)
    return GateRef(order, score, probs)


def expert_ref(x: torch.Tensor, w1, b1, w2, b2, act: str) -> torch.Tensor:
    """baseline/infer.py:286-287 with the activation as a parameter."""
    h = F.linear(x, w1, b1)
    h = F.gelu(h) if act == "gelu" else F.relu(h)
    return F.linear(h, w2, b2)


def smoe_ref(x: torch.Tensor, wg, bg, w1, b1, w2, b2, act: str = "gelu", renorm: bool = True,
             tie_lower_id: bool = True, force_idx: torch.Tensor | None = None):
    """baseline/infer.py:323-353.  x [T, D]; w1 [E, F, D]; w2 [E, D, F] (all cast
    to fp32).  Returns (out [T, D] fp32, GateRef).  `force_idx`: see gate_ref."""
    x = x.float()
    g = gate_ref(x, wg, bg, renorm, tie_lower_id, force_idx)
    out = torch.zeros_like(x)
    E = wg.shape[0]
    for e in range(E):
        mask = g.idx == e
        if not mask.any():
            continue
        token_idx, k_idx = mask.nonzero(as_tuple=True)
        y = expert_ref(x[token_idx], w1[e].float(), b1[e].float(), w2[e].float(), b2[e].float(), act)
        out[token_idx] += y * g.score[token_idx, k_idx].unsqueeze(-1)
    return out, g


def expert_segments(idx: torch.Tensor, num_experts: int):
    """Expected dispatch of baseline/infer.py:336-346: for each expert e, its
    routes in token order (k=0 before k=1 within a token).  Returns
    (offsets [E+1], sorted_token [2T], perm_inv [T, 2]) as int64."""
    T = idx.shape[0]
    flat = idx.reshape(-1)
    route = torch.arange(2 * T)
    counts = torch.bincount(flat, minlength=num_experts)
    offsets = torch.zeros(num_experts + 1, dtype=torch.int64)
    offsets[1:] = torch.cumsum(counts, 0)
    order = torch.sort(flat, stable=True).indices  # routes grouped by expert, token order kept
    sorted_token = route[order] // 2
    perm_inv = torch.empty(2 * T, dtype=torch.int64)
    perm_inv[order] = torch.arange(2 * T)
    return offsets, sorted_token, perm_inv.reshape(T, 2)


def logits_fp64(x: torch.Tensor, wg: torch.Tensor, bg: torch.Tensor) -> torch.Tensor:
    return x.double() @ wg.double().T + bg.double()


def near_tie_mask(x: torch.Tensor, wg: torch.Tensor, bg: torch.Tensor, band: float = 1e-5) -> torch.Tensor:
    """Tokens whose top-1/top-2 or top-2/top-3 logit gap (in fp64) is below
    `band`: fp32 sums in different orders may legitimately rank them
    differently, so index parity against a differently-ordered fp32 sum is
    only required outside this band."""
    l = logits_fp64(x, wg, bg)
    s = torch.sort(l, dim=-1, descending=True).values
    gap12 = s[:, 0] - s[:, 1]
    gap23 = s[:, 1] - s[:, 2] if s.shape[1] > 2 else torch.full_like(gap12, float("inf"))
    return torch.minimum(gap12, gap23) < band
