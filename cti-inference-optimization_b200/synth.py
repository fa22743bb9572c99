"""Seeded synthetic inputs for the benchmark configurations.

The reference measures on proprietary competition data (not available);
these generators produce inputs with the shapes and value distributions the
benchmark configurations name:

* cfg1  T=4096 tokens, d_model 128, 8 experts, d_ff 512;
* cfg2  512 samples, lengths U{16..256} packed with int32 cu_seqlens,
        d_model 256, 16 experts, d_ff 1024, Zipf(1.2) router bias;
* cfg3  batch 4096, 28 features, fp16 tables of dim 64 with vocabularies
        log-uniform in [1e4, 2e6], bag lengths Poisson(lambda_f) with
        lambda_f ~ U[1, 50], ids Zipf(1.1) over each vocabulary;
* cfg4  the full model at 2048 samples;
* cfg5  T=262144, d_model 1024, 64 experts, d_ff 4096.

All weights are N(0, 0.02).  The Zipf(1.2) expert profile: expert e gets
router bias log(p_e) with p proportional to (rank_e + 1)^-1.2 over a seeded
permutation of expert ranks.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch


@dataclass(frozen=True)
class MoEConfig:
    name: str
    d_model: int
    num_experts: int
    dim_ff: int
    samples: int = 0  # packed-sample configs: number of sequences
    min_len: int = 16
    max_len: int = 256
    tokens: int = 0  # fixed-T configs
    zipf_bias: float | None = 1.2


CFG1 = MoEConfig("cfg1", 128, 8, 512, tokens=4096, zipf_bias=None)
CFG2 = MoEConfig("cfg2", 256, 16, 1024, samples=512)
CFG5 = MoEConfig("cfg5", 1024, 64, 4096, tokens=262144)
MOE_CONFIGS = {c.name: c for c in (CFG1, CFG2, CFG5)}


def packed_lengths(samples: int, lo: int, hi: int, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.integers(lo, hi + 1, size=samples, dtype=np.int64)


def cu_seqlens(lengths: np.ndarray) -> torch.Tensor:
    cu = np.zeros(len(lengths) + 1, dtype=np.int32)
    np.cumsum(lengths, out=cu[1:])
    return torch.from_numpy(cu)


def zipf_router_bias(num_experts: int, s: float, seed: int = 0) -> torch.Tensor:
    rng = np.random.default_rng(seed + 7919)
    ranks = rng.permutation(num_experts)
    p = (ranks + 1.0) ** (-s)
    p = p / p.sum()
    return torch.from_numpy(np.log(p)).float()


@dataclass
class MoEWeights:
    wg: torch.Tensor  # [E, D] fp32
    bg: torch.Tensor  # [E] fp32
    w1: torch.Tensor  # [E, F, D] (nn.Linear layout of fc1)
    b1: torch.Tensor  # [E, F]
    w2: torch.Tensor  # [E, D, F]
    b2: torch.Tensor  # [E, D]


def moe_weights(d_model: int, num_experts: int, dim_ff: int, zipf_bias: float | None,
                seed: int = 0, device="cpu", expert_dtype=torch.bfloat16) -> MoEWeights:
    """N(0, 0.02) weights; expert weights rounded to `expert_dtype`."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    E, D, F = num_experts, d_model, dim_ff
    wg = torch.randn(E, D, generator=g) * 0.02
    bg = torch.randn(E, generator=g) * 0.02
    if zipf_bias is not None:
        bg = bg + zipf_router_bias(E, zipf_bias, seed)
    # Expert weights are drawn on the target device in slices (cfg5 holds
    # 1 GiB of fp32 draws per matrix).
    gd = torch.Generator(device=device).manual_seed(seed + 1)

    def draw(*shape):
        return (torch.randn(*shape, generator=gd, device=device) * 0.02).to(expert_dtype)

    w1 = draw(E, F, D)
    b1 = draw(E, F).float()
    w2 = draw(E, D, F)
    b2 = draw(E, D).float()
    return MoEWeights(wg.to(device), bg.to(device), w1, b1, w2, b2)


def moe_tokens(cfg: MoEConfig, seed: int = 0) -> tuple[int, torch.Tensor | None]:
    """Number of packed tokens and the int32 cu_seqlens (None for fixed-T configs)."""
    if cfg.samples:
        lens = packed_lengths(cfg.samples, cfg.min_len, cfg.max_len, seed)
        return int(lens.sum()), cu_seqlens(lens)
    return cfg.tokens, None


def moe_activations(T: int, d_model: int, seed: int = 0, device="cpu",
                    dtype=torch.bfloat16) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed + 2)
    return torch.randn(T, d_model, generator=g, device=device).to(dtype)


def load_moe_module(module, w: MoEWeights) -> None:
    """Copies generated weights into an SMoE-like module (reference key layout)."""
    with torch.no_grad():
        module.gate.w_g.weight.copy_(w.wg)
        module.gate.w_g.bias.copy_(w.bg)
        for e, ex in enumerate(module.experts):
            ex.fc1.weight.copy_(w.w1[e])
            ex.fc1.bias.copy_(w.b1[e])
            ex.fc2.weight.copy_(w.w2[e])
            ex.fc2.bias.copy_(w.b2[e])


# ---------------------------------------------------------------------------
# Embedding-bag batches (cfg3) in the reference's flat layout.
# ---------------------------------------------------------------------------
@dataclass
class BagBatch:
    values: torch.Tensor  # int64 [N]
    row_offsets: torch.Tensor  # int64 [F*(B+1)]
    val_offsets: torch.Tensor  # int64 [F]
    vocab: torch.Tensor  # int64 [F]
    table_row_base: torch.Tensor  # int64 [F]
    batch: int
    features: int

    @property
    def total_rows(self) -> int:
        return int(self.table_row_base[-1] + self.vocab[-1])


def log_uniform_vocab(features: int, lo: float, hi: float, rng) -> np.ndarray:
    return np.round(np.exp(rng.uniform(math.log(lo), math.log(hi), size=features))).astype(np.int64)


def zipf_ids(n: int, vocab: int, s: float, rng) -> np.ndarray:
    """n ids with P(rank k) proportional to (k+1)^-s over [0, vocab), by inverse
    CDF, mapped through a random permutation of the vocabulary."""
    w = np.arange(1, vocab + 1, dtype=np.float64) ** (-s)
    cdf = np.cumsum(w)
    cdf /= cdf[-1]
    # torch's searchsorted runs on all host threads and returns exactly what
    # np.searchsorted(side="right") does (the configuration-4 batch draws
    # about 200 M ids).
    ranks = torch.searchsorted(torch.from_numpy(cdf), torch.from_numpy(rng.random(n)),
                               right=True).numpy()
    ranks = np.minimum(ranks, vocab - 1)
    perm = rng.permutation(vocab)
    return perm[ranks]


def bag_batch(batch: int = 4096, features: int = 28, vocab_lo: float = 1e4, vocab_hi: float = 2e6,
              lam_lo: float = 1.0, lam_hi: float = 50.0, zipf_s: float = 1.1,
              seed: int = 0, vocab: np.ndarray | None = None) -> BagBatch:
    rng = np.random.default_rng(seed)
    if vocab is None:
        vocab = log_uniform_vocab(features, vocab_lo, vocab_hi, rng)
    lam = rng.uniform(lam_lo, lam_hi, size=features)
    vals, offs, voff = [], [], []
    start = 0
    for f in range(features):
        lens = rng.poisson(lam[f], size=batch).astype(np.int64)
        o = np.zeros(batch + 1, dtype=np.int64)
        np.cumsum(lens, out=o[1:])
        ids = zipf_ids(int(o[-1]), int(vocab[f]), zipf_s, rng)
        vals.append(ids)
        offs.append(o)
        voff.append(start)
        start += int(o[-1])
    base = np.zeros(features, dtype=np.int64)
    np.cumsum(vocab[:-1], out=base[1:])
    return BagBatch(
        values=torch.from_numpy(np.concatenate(vals)),
        row_offsets=torch.from_numpy(np.concatenate(offs)),
        val_offsets=torch.tensor(voff, dtype=torch.int64),
        vocab=torch.from_numpy(vocab.astype(np.int64)),
        table_row_base=torch.from_numpy(base),
        batch=batch,
        features=features,
    )


def embedding_table(total_rows: int, dim: int = 64, seed: int = 0, device="cpu") -> torch.Tensor:
    """fp16 [total_rows, dim] table ~ N(0, 0.02), drawn in slices."""
    g = torch.Generator(device=device).manual_seed(seed + 3)
    out = torch.empty(total_rows, dim, dtype=torch.float16, device=device)
    step = 1 << 22
    for s in range(0, total_rows, step):
        e = min(total_rows, s + step)
        out[s:e] = (torch.randn(e - s, dim, generator=g, device=device) * 0.02).half()
    return out


# ---------------------------------------------------------------------------
# The configuration-4 CTR model: batch and random init.
# ---------------------------------------------------------------------------
CFG4_SAMPLES = 2048


def cfg4_batch(seed: int = 0, samples: int = CFG4_SAMPLES):
    """Configuration 4: `samples` packed sequences with lengths U{16..256};
    every token carries the 28 configuration-3 bags.  Returns (BagBatch over
    the T tokens, int64 user_offsets [samples + 1], T)."""
    lens = packed_lengths(samples, 16, 256, seed)
    uo = torch.zeros(samples + 1, dtype=torch.int64)
    uo[1:] = torch.cumsum(torch.from_numpy(lens.astype(np.int64)), 0)
    T = int(uo[-1])
    return bag_batch(batch=T, seed=seed), uo, T


def init_ctr_model(model, seed: int = 0) -> None:
    """The configuration's random init of a CTR model (reference parameter
    names): weights ~N(0, 0.02), biases 0, LayerNorms (1, 0), and every
    router bias the Zipf(1.2) profile.  The embedding table is left alone
    (embedding_table() draws it)."""
    g = torch.Generator().manual_seed(seed + 11)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "rep_encoder.emb" in name:
                continue
            if "norm" in name:
                p.fill_(1.0 if name.endswith("weight") else 0.0)
            elif p.dim() > 1:
                p.copy_(torch.randn(p.shape, generator=g) * 0.02)
            else:
                p.zero_()
        for i, m in enumerate(model.seq_encoder.moe):
            m.gate.w_g.bias.copy_(zipf_router_bias(m.num_experts, 1.2, seed + i))


def sequence_subbatch(bb: BagBatch, user_offsets: torch.Tensor, seqs) -> dict:
    """The flat-layout batch of the sequences `seqs` (ascending indices into
    user_offsets) alone: their tokens in order, each feature's bags and ids
    copied out.  Sequences are independent in the CTR model, so the model's
    output on this batch equals its output on those sequences' tokens in the
    whole batch."""
    uo = user_offsets.long()
    F_ = bb.features
    T = int(uo[-1])
    offs = bb.row_offsets.view(F_, T + 1)
    ranges = [(int(uo[s]), int(uo[s + 1])) for s in seqs]
    lens = [b - a for a, b in ranges]
    new_uo = torch.zeros(len(seqs) + 1, dtype=torch.int64)
    new_uo[1:] = torch.cumsum(torch.tensor(lens, dtype=torch.int64), 0)
    vals, row_offs, voff = [], [], []
    start = 0
    for f in range(F_):
        v0 = int(bb.val_offsets[f])
        parts, counts = [], [torch.zeros(1, dtype=torch.int64)]
        for a, b in ranges:
            o = offs[f, a:b + 1]
            parts.append(bb.values[v0 + int(o[0]):v0 + int(o[-1])])
            counts.append(o[1:] - o[:-1])
        fv = torch.cat(parts)
        vals.append(fv)
        row_offs.append(torch.cumsum(torch.cat(counts), 0))
        voff.append(start)
        start += fv.numel()
    return {"_flat_values": torch.cat(vals), "_flat_row_offsets": torch.cat(row_offs),
            "_val_offsets": torch.tensor(voff, dtype=torch.int64), "user_offsets": new_uo}
