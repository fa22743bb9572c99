"""Restatement of the reference CTR model forward on CPU (fp32).  TEST ONLY.

Follows baseline/infer.py with the configuration-4 semantics:
  RepEncoder.forward          :253-266  pooling (embbag_ref) -> LayerNorm -> Linear
  TransformerEncoder.forward  :384-411  per layer, pre-LN:
      qkv = qkv_proj(norm1(x)).view(T, H, 3*hd); q, k, v = split(hd)
      x = x + out_proj(softmax(q k^T / sqrt(hd) + causal mask) v)
      x = x + SMoE(norm2(x))               (smoe_ref: GELU, renormalised gates)
  CTRModel.forward            :429-439  head, then clamp(+-15); sigmoid at :686
The causal mask is the reference's get_sequence_causal_mask (:420-427): a
token attends to the tokens of its own sequence up to itself.  The head is
the configuration's MLP d -> 128 -> 1 with ReLU, under the state-dict name
``linear`` (nn.Sequential: linear.0, linear.2) instead of the reference's
single Linear.

The state dict uses the reference's parameter names; see
tests/golden/golden_inputs.py for how the fixtures build one.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from .embbag_ref import embbag_ref
from .moe_ref import gate_ref, logits_fp64, smoe_ref


def attention_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                  user_offsets: torch.Tensor) -> torch.Tensor:
    """q, k, v [T, H, hd] fp32 -> [T, H, hd]; causal within each sequence."""
    out = torch.empty_like(q)
    uo = user_offsets.long().tolist()
    hd = q.shape[-1]
    for a, b in zip(uo[:-1], uo[1:]):
        if b <= a:
            continue
        qs, ks, vs = (t[a:b].transpose(0, 1) for t in (q, k, v))  # [H, L, hd]
        s = qs @ ks.transpose(-1, -2) / math.sqrt(hd)
        L = b - a
        mask = torch.ones(L, L, dtype=torch.bool).tril()
        s = s.masked_fill(~mask, float("-inf"))
        out[a:b] = (torch.softmax(s, dim=-1) @ vs).transpose(0, 1)
    return out


def rep_encoder_ref(sd: dict, batch: dict, *, slot_num: int, table_row_base=None,
                    vocab=None) -> torch.Tensor:
    """RepEncoder.forward (baseline/infer.py:253-265): the sum pooling of
    every (sample, slot) bag, LayerNorm over the slot_num * emb_dim pooled
    columns, Linear to d_model; fp32 [B, d_model].  ``sd`` holds the
    ``rep_encoder.*`` parameters under the reference's names."""
    # The embedding table stays in its own dtype: the pooling upcasts only
    # the rows it gathers.
    g = {k: v.float() for k, v in sd.items()
         if k.startswith("rep_encoder.") and k != "rep_encoder.emb.weight"}
    table = sd["rep_encoder.emb.weight"]
    if table_row_base is None:  # one shared table, as in the reference
        table_row_base = torch.zeros(slot_num, dtype=torch.int64)
        vocab = torch.full((slot_num,), table.shape[0], dtype=torch.int64)
    pooled = embbag_ref(batch["_flat_values"], batch["_flat_row_offsets"], batch["_val_offsets"],
                        table, table_row_base, vocab, slot_num)
    x = F.layer_norm(pooled, (pooled.shape[1],), g["rep_encoder.input_norm.weight"],
                     g["rep_encoder.input_norm.bias"])
    return F.linear(x, g["rep_encoder.linear.weight"], g["rep_encoder.linear.bias"])


def ctr_forward_ref(sd: dict, batch: dict, *, slot_num: int, n_heads: int, num_layers: int,
                    num_experts: int, table_row_base=None, vocab=None, force_routes=None,
                    routing: list | None = None):
    """Returns (encoder output [T, D], clamped logits [T], probabilities [T]),
    all fp32.  ``sd`` maps reference parameter names to tensors.

    ``force_routes[i]`` ([T, 2]), when given, fixes layer i's top-2 experts
    (see moe_ref.gate_ref).  ``routing``, when a list, receives per layer
    (the gate's own top-2 [T, 2] on this run's activations, the fp64 gap
    [T] between its top-1/top-2 or top-2/top-3 logits, whichever is
    smaller)."""
    g = {k: v.float() for k, v in sd.items() if k != "rep_encoder.emb.weight"}
    x = rep_encoder_ref(sd, batch, slot_num=slot_num, table_row_base=table_row_base, vocab=vocab)
    T, D = x.shape
    hd = D // n_heads
    for i in range(num_layers):
        p = "seq_encoder."
        h = F.layer_norm(x, (D,), g[p + f"norm1.{i}.weight"], g[p + f"norm1.{i}.bias"])
        qkv = F.linear(h, g[p + f"qkv_proj.{i}.weight"], g[p + f"qkv_proj.{i}.bias"])
        q, k, v = torch.split(qkv.view(T, n_heads, 3 * hd), hd, dim=-1)
        a = attention_ref(q, k, v, batch["user_offsets"]).reshape(T, D)
        x = x + F.linear(a, g[p + f"out_proj.{i}.weight"], g[p + f"out_proj.{i}.bias"])
        h = F.layer_norm(x, (D,), g[p + f"norm2.{i}.weight"], g[p + f"norm2.{i}.bias"])
        m = p + f"moe.{i}."
        w1 = torch.stack([g[m + f"experts.{e}.fc1.weight"] for e in range(num_experts)])
        b1 = torch.stack([g[m + f"experts.{e}.fc1.bias"] for e in range(num_experts)])
        w2 = torch.stack([g[m + f"experts.{e}.fc2.weight"] for e in range(num_experts)])
        b2 = torch.stack([g[m + f"experts.{e}.fc2.bias"] for e in range(num_experts)])
        wg, bg = g[m + "gate.w_g.weight"], g[m + "gate.w_g.bias"]
        if routing is not None:
            own = gate_ref(h, wg, bg).idx
            s_ = logits_fp64(h, wg, bg).sort(dim=-1, descending=True).values
            gap = torch.minimum(s_[:, 0] - s_[:, 1], s_[:, 1] - s_[:, 2])
            routing.append((own, gap))
        y, _ = smoe_ref(h, wg, bg, w1, b1, w2, b2, act="gelu", renorm=True,
                        force_idx=None if force_routes is None else force_routes[i])
        x = x + y
    z = F.relu(F.linear(x, g["linear.0.weight"], g["linear.0.bias"]))
    logits = torch.clamp(F.linear(z, g["linear.2.weight"], g["linear.2.bias"]), -15.0, 15.0)
    logits = logits.reshape(-1)
    return x, logits, torch.sigmoid(logits)
