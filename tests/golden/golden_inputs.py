"""Seeded inputs of the golden fixtures (shared by make_golden.py and the tests).

Every generator uses its own CPU torch.Generator, and each fixture stores
the SHA-256 of the inputs it was made from, so a test first proves that it
regenerated exactly the same inputs before comparing outputs.
"""
from __future__ import annotations

import hashlib
import math

import numpy as np
import torch

# name -> (d_model, num_experts, dim_ff, tokens, act, renorm, zipf)
MOE_CASES = {
    "moe_refexact_d128_e8": (128, 8, 256, 128, "relu", False, None),
    "moe_config_d128_e8": (128, 8, 256, 128, "gelu", True, None),
    "moe_config_d256_e16_zipf": (256, 16, 1024, 64, "gelu", True, 1.2),
}


def tensor_digest(*ts: torch.Tensor) -> str:
    h = hashlib.sha256()
    for t in ts:
        h.update(t.detach().cpu().contiguous().numpy().tobytes())
    return h.hexdigest()


def moe_inputs(name: str, seed: int = 0):
    """x [T, D] and weights, all bf16-representable fp32 (expert weights and x
    are rounded to bf16; router weights stay fp32)."""
    D, E, F, T, act, renorm, zipf = MOE_CASES[name]
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, D, generator=g).bfloat16().float()
    wg = torch.randn(E, D, generator=g) * 0.02
    bg = torch.randn(E, generator=g) * 0.02
    if zipf is not None:
        ranks = torch.randperm(E, generator=g).double()
        p = (ranks + 1.0) ** (-zipf)
        bg = bg + torch.log(p / p.sum()).float()
    w1 = (torch.randn(E, F, D, generator=g) * 0.02).bfloat16().float()
    b1 = (torch.randn(E, F, generator=g) * 0.02).bfloat16().float()
    w2 = (torch.randn(E, D, F, generator=g) * 0.02).bfloat16().float()
    b2 = (torch.randn(E, D, generator=g) * 0.02).bfloat16().float()
    return dict(x=x, wg=wg, bg=bg, w1=w1, b1=b1, w2=w2, b2=b2, act=act, renorm=renorm)


def bag_inputs(per_feature: bool, seed: int = 0):
    """A small 28-slot batch in the reference's flat layout, with empty bags
    and out-of-range ids (negative and >= vocab, which the reference clamps)."""
    g = torch.Generator().manual_seed(seed + (100 if per_feature else 0))
    F, dim = 28, 64
    B = 8 if per_feature else 12
    if per_feature:
        vocab = (torch.randint(40, 400, (F,), generator=g)).long()
    else:
        vocab = torch.full((F,), 1000, dtype=torch.long)
    vals, offs, voff = [], [], []
    start = 0
    for f in range(F):
        lens = torch.randint(0, 7, (B,), generator=g)
        lens[f % B] = 0  # at least one empty bag per slot
        o = torch.zeros(B + 1, dtype=torch.long)
        o[1:] = torch.cumsum(lens, 0)
        n = int(o[-1])
        v = torch.randint(-3, int(vocab[f]) + 3, (n,), generator=g).long()
        vals.append(v)
        offs.append(o)
        voff.append(start)
        start += n
    if per_feature:
        base = torch.zeros(F, dtype=torch.long)
        base[1:] = torch.cumsum(vocab[:-1], 0)
        rows = int(base[-1] + vocab[-1])
    else:
        base = torch.zeros(F, dtype=torch.long)
        rows = int(vocab[0])
    table = (torch.randn(rows, dim, generator=g) * 0.02).half()
    return dict(values=torch.cat(vals), row_offsets=torch.cat(offs),
                val_offsets=torch.tensor(voff, dtype=torch.long), vocab=vocab,
                table_row_base=base, table=table, features=F, batch=B)
