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


# name -> (sequences, max_len, d_model, n_heads, layers, dim_ff, experts, vocab, weight_std)
# weight_std 0.02 is the configuration's init (logits near 0, where the 1e-3
# probability bound applies); the None case uses larger weights so that the
# logits spread over several units and every stage moves the result.
E2E_CASES = {
    "e2e_d128_l2": (6, 12, 128, 4, 2, 512, 8, 500, None),
    "e2e_d128_l2_init": (6, 12, 128, 4, 2, 512, 8, 500, 0.02),
}
E2E_SLOTS, E2E_EMB, E2E_HEAD = 28, 64, 128


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t.bfloat16().float()


def e2e_inputs(name: str, seed: int = 0):
    """A packed batch (flat pooling layout + user_offsets) and a state dict
    with the reference CTRModel's parameter names (baseline/infer.py:244-439,
    head replaced by the configuration's MLP).  Every weight except the
    routers is bf16-representable, so a bf16 model holds exactly these
    values; the routers stay fp32 like the product's."""
    N, Lmax, D, H, L, Fd, E, V, wstd = E2E_CASES[name]
    g = torch.Generator().manual_seed(seed + 500)
    lens = torch.randint(2, Lmax + 1, (N,), generator=g)
    uo = torch.zeros(N + 1, dtype=torch.long)
    uo[1:] = torch.cumsum(lens, 0)
    T = int(uo[-1])
    vals, offs, voff = [], [], []
    start = 0
    for f in range(E2E_SLOTS):
        bl = torch.randint(0, 5, (T,), generator=g)
        o = torch.zeros(T + 1, dtype=torch.long)
        o[1:] = torch.cumsum(bl, 0)
        v = torch.randint(-3, V + 3, (int(o[-1]),), generator=g).long()
        vals.append(v)
        offs.append(o)
        voff.append(start)
        start += int(o[-1])
    batch = {"_flat_values": torch.cat(vals), "_flat_row_offsets": torch.cat(offs),
             "_val_offsets": torch.tensor(voff, dtype=torch.long), "user_offsets": uo}

    def w(*shape, std=0.02):
        return _bf16(torch.randn(*shape, generator=g) * (std if wstd is None else wstd))

    def ln(n):
        return _bf16(1.0 + torch.randn(n, generator=g) * 0.1), _bf16(torch.randn(n, generator=g) * 0.1)

    sd = {}
    sd["rep_encoder.emb.weight"] = (torch.randn(V, E2E_EMB, generator=g) * 0.5).half().float()
    sd["rep_encoder.input_norm.weight"], sd["rep_encoder.input_norm.bias"] = ln(E2E_SLOTS * E2E_EMB)
    sd["rep_encoder.linear.weight"] = w(D, E2E_SLOTS * E2E_EMB, std=0.05)
    sd["rep_encoder.linear.bias"] = w(D)
    p = "seq_encoder."
    for i in range(L):
        sd[p + f"qkv_proj.{i}.weight"], sd[p + f"qkv_proj.{i}.bias"] = w(3 * D, D, std=0.1), w(3 * D)
        sd[p + f"out_proj.{i}.weight"], sd[p + f"out_proj.{i}.bias"] = w(D, D, std=0.1), w(D)
        sd[p + f"ffn1.{i}.weight"], sd[p + f"ffn1.{i}.bias"] = w(Fd, D), w(Fd)
        sd[p + f"ffn2.{i}.weight"], sd[p + f"ffn2.{i}.bias"] = w(D, Fd), w(D)
        sd[p + f"norm1.{i}.weight"], sd[p + f"norm1.{i}.bias"] = ln(D)
        sd[p + f"norm2.{i}.weight"], sd[p + f"norm2.{i}.bias"] = ln(D)
        m = p + f"moe.{i}."
        sd[m + "gate.w_g.weight"] = torch.randn(E, D, generator=g) * 0.1
        sd[m + "gate.w_g.bias"] = torch.randn(E, generator=g) * 0.1
        for e in range(E):
            sd[m + f"experts.{e}.fc1.weight"] = w(Fd, D, std=0.05)
            sd[m + f"experts.{e}.fc1.bias"] = w(Fd)
            sd[m + f"experts.{e}.fc2.weight"] = w(D, Fd, std=0.05)
            sd[m + f"experts.{e}.fc2.bias"] = w(D)
    sd["linear.0.weight"], sd["linear.0.bias"] = w(E2E_HEAD, D, std=0.1), w(E2E_HEAD)
    sd["linear.2.weight"], sd["linear.2.bias"] = w(1, E2E_HEAD, std=0.5), w(1)
    return batch, sd


def e2e_digest(batch: dict, sd: dict) -> str:
    ts = [batch[k] for k in ("_flat_values", "_flat_row_offsets", "_val_offsets", "user_offsets")]
    ts += [sd[k] for k in sorted(sd)]
    return tensor_digest(*ts)
