"""Drop-in ``RepEncoder`` whose 28-slot embedding-bag pooling runs on the
sm_100a kernel (``cti_embbag_sum``).

Follows ``RepEncoder`` of ``online_best/infer.py:945-1100`` /
``baseline/infer.py:244-266``: constructor ``(vocab_size, emb_dim,
padding_idx, slot_num, d_model)``, submodules ``emb``/``input_norm``/``linear``
(same state-dict keys), ``forward(batch)`` reading the flat layout
``_flat_values`` / ``_flat_row_offsets`` / ``_val_offsets`` and returning
``linear(input_norm(pooled))``.

Extension: ``vocab_sizes`` (one per slot) gives every slot its own table,
stored as consecutive row ranges of ``emb.weight``; each slot clamps its ids
to its own vocabulary.  Without it all slots share one table, as in the
reference.  Tables are fp16 (the benchmark configuration).
"""
from __future__ import annotations

from typing import Sequence

import torch
import torch.nn as nn

from . import ops


def flatten_slot_batch(batch: dict, slot_num: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Builds the flat layout from the per-slot ``batch[slot] = (values, offsets)``
    pairs of the baseline collate (online_best/infer.py:139-153)."""
    vals, offs, lens = [], [], [0]
    for s in range(1, slot_num + 1):
        v, o = batch[s]
        vals.append(v)
        offs.append(o)
        lens.append(lens[-1] + v.shape[0])
    return (torch.cat(vals).long(), torch.cat(offs).long(),
            torch.tensor(lens[:-1], dtype=torch.long))


class RepEncoder(nn.Module):
    def __init__(self, vocab_size: int, emb_dim: int, padding_idx: int = 0, slot_num: int = 28,
                 d_model: int = 256, vocab_sizes: Sequence[int] | None = None):
        super().__init__()
        if vocab_sizes is not None:
            if len(vocab_sizes) != slot_num:
                raise ValueError("vocab_sizes needs one entry per slot")
            sizes = [int(v) for v in vocab_sizes]
            base = [0]
            for v in sizes[:-1]:
                base.append(base[-1] + v)
            total = base[-1] + sizes[-1]
        else:
            sizes = [int(vocab_size)] * slot_num
            base = [0] * slot_num
            total = int(vocab_size)
        self.emb = nn.Embedding(total, emb_dim, padding_idx=padding_idx if vocab_sizes is None else None)
        self.emb_dim = emb_dim
        self.slot_num = slot_num
        self.input_norm = nn.LayerNorm(slot_num * emb_dim)
        self.linear = nn.Linear(slot_num * emb_dim, d_model)
        self.register_buffer("table_row_base", torch.tensor(base, dtype=torch.int64), persistent=False)
        self.register_buffer("vocab", torch.tensor(sizes, dtype=torch.int64), persistent=False)

    def pool(self, batch: dict, out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """The [B, slot_num*emb_dim] sum-pooled embeddings (slot-major columns)."""
        dev = self.emb.weight.device
        if "_flat_values" not in batch:
            v, o, vo = flatten_slot_batch(batch, self.slot_num)
        else:
            v, o, vo = batch["_flat_values"], batch["_flat_row_offsets"], batch["_val_offsets"]
        v = v.to(dev, torch.int64, non_blocking=True).contiguous()
        o = o.to(dev, torch.int64, non_blocking=True).contiguous()
        vo = vo.to(dev, torch.int64, non_blocking=True).contiguous()
        table = self.emb.weight
        if table.dtype != torch.float16:
            raise TypeError("the pooling kernel reads fp16 tables; call .half() on the embedding")
        return ops.embedding_bag_sum(v, o, vo, table.detach(), self.table_row_base, self.vocab,
                                     self.slot_num, out_dtype=out_dtype)

    def fused_supported(self) -> bool:
        """Whether forward_fused() can run (cti_rep_encoder_fused):
        64-wide fp16 tables, bf16 LayerNorm and Linear, d_model 128 or 256."""
        w = self.linear.weight
        return (self.emb_dim == 64 and w.is_cuda and w.dtype == torch.bfloat16
                and self.emb.weight.dtype == torch.float16 and w.shape[0] in (128, 256)
                and self.input_norm.weight.dtype == torch.bfloat16)

    @torch.no_grad()
    def fused_params(self):
        """(Wg bf16 [N, F*64] = W * gamma, r1 fp32 [N] = row sums of Wg,
        c fp32 [N] = W beta + b): the LayerNorm folded into the Linear,
        rebuilt when a parameter changes."""
        key = tuple((p.data_ptr(), p._version) for p in
                    (self.linear.weight, self.linear.bias, self.input_norm.weight,
                     self.input_norm.bias))
        cache = getattr(self, "_fused", None)
        if cache is None or cache[0] != key:
            W = self.linear.weight.float()
            wg = (W * self.input_norm.weight.float()[None, :]).to(torch.bfloat16).contiguous()
            r1 = wg.float().sum(1).contiguous()
            c = (W @ self.input_norm.bias.float() + self.linear.bias.float()).contiguous()
            cache = (key, wg, r1, c)
            self._fused = cache
        return cache[1], cache[2], cache[3]

    def forward(self, batch: dict) -> torch.Tensor:
        """linear(input_norm(pooled)) in bf16 (the model after
        prepare_for_inference): the pooling kernel writes the pooled rows
        (bf16), the LayerNorm kernel normalises them (it raises for widths it
        does not cover) and cuBLAS applies the Linear.  At the benchmark
        configuration this is faster than forward_fused: the pooling kernel
        walks the batch feature by feature over the whole GPU, so each
        table's hot rows stay in L2, while the fused kernel gathers all
        features of a token tile at once."""
        pooled = self.pool(batch, out_dtype=self.input_norm.weight.dtype)
        _, normed = ops.add_layernorm(pooled, None, self.input_norm.weight,
                                      self.input_norm.bias, self.input_norm.eps)
        return self.linear(normed)

    def forward_fused(self, batch: dict) -> torch.Tensor:
        """forward() as one sm_100a launch (cti_rep_encoder_fused): pooling,
        LayerNorm folded into the Linear, the pooled rows never written to
        HBM.  Needs fused_supported(); raises otherwise."""
        if not self.fused_supported():
            raise ValueError("forward_fused needs 64-wide fp16 tables, bf16 LayerNorm and "
                             "Linear, and d_model 128 or 256 on a CUDA device")
        dev = self.emb.weight.device
        if "_flat_values" not in batch:
            v, o, vo = flatten_slot_batch(batch, self.slot_num)
        else:
            v, o, vo = batch["_flat_values"], batch["_flat_row_offsets"], batch["_val_offsets"]
        v = v.to(dev, torch.int64, non_blocking=True).contiguous()
        o = o.to(dev, torch.int64, non_blocking=True).contiguous()
        vo = vo.to(dev, torch.int64, non_blocking=True).contiguous()
        wg, r1, c = self.fused_params()
        return ops.rep_encoder_fused(v, o, vo, self.emb.weight.detach(), self.table_row_base,
                                     self.vocab, self.slot_num, wg, r1, c, self.input_norm.eps)
