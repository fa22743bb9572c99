"""Restatement of the reference embedding-bag pooling on CPU (fp32).  TEST ONLY.

baseline/infer.py:253-263: for each slot i, values.clamp(0, V-1) ->
emb(values) -> torch.segment_reduce(sum, offsets, initial=0) -> cat over
slots (slot-major columns).  The flat layout (online_best/infer.py:139-182,
:1029-1033): feature f's values start at val_offsets[f]; its offsets are
row_offsets[f*(B+1):(f+1)*(B+1)].  Tables are upcast to fp32 before the sum,
which on CPU runs sequentially over each bag (checked against a Python loop
in the tests).
"""
from __future__ import annotations

import torch


def embbag_ref(values, row_offsets, val_offsets, table, table_row_base, vocab, num_features):
    F_ = num_features
    B = row_offsets.numel() // F_ - 1
    outs = []
    for f in range(F_):
        offs = row_offsets[f * (B + 1):(f + 1) * (B + 1)].long()
        v0 = int(val_offsets[f]) + int(offs[0])
        v1 = int(val_offsets[f]) + int(offs[-1])
        vals = values[v0:v1].long().clamp(0, int(vocab[f]) - 1)
        rows = table[int(table_row_base[f]) + vals].float()
        outs.append(torch.segment_reduce(rows, "sum", offsets=offs - offs[0], initial=0))
    return torch.cat(outs, dim=1)


def embbag_loop(values, row_offsets, val_offsets, table, table_row_base, vocab, num_features):
    """The same sum as an explicit sequential Python loop (small inputs only)."""
    F_ = num_features
    B = row_offsets.numel() // F_ - 1
    dim = table.shape[1]
    out = torch.zeros(B, F_ * dim, dtype=torch.float32)
    t32 = table.float()
    for f in range(F_):
        base = f * (B + 1)
        for b in range(B):
            acc = torch.zeros(dim, dtype=torch.float32)
            for i in range(int(row_offsets[base + b]), int(row_offsets[base + b + 1])):
                idv = int(values[int(val_offsets[f]) + i])
                idv = min(max(idv, 0), int(vocab[f]) - 1)
                acc = acc + t32[int(table_row_base[f]) + idv]
            out[b, f * dim:(f + 1) * dim] = acc
    return out
