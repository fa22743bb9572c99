"""The CTR model around the hot path (the 8-layer forward of configuration 4).

Drop-ins for ``TransformerEncoder`` and ``CTRModel`` of ``baseline/infer.py``
(:360-439; the same graph runs in ``online_best/infer.py:2440-2620``), with
the reference's parameter names, so a reference state dict loads as is:

  * ``rep_encoder``: the ``RepEncoder`` drop-in (sm_100a pooling kernel,
    then LayerNorm over slot_num*emb_dim, then Linear - the reference order,
    ``baseline/infer.py:263-265``);
  * ``seq_encoder``: pre-LN layers, each
        x = x + out_proj(attention(qkv_proj(norm1(x))))
        x = x + moe(norm2(x))
    with the reference's interleaved per-head qkv layout (``qkv.view(T, H,
    3*head_dim)`` then split into q, k, v; ``baseline/infer.py:391-395``),
    causal attention inside each packed sequence, and the ``SMoE`` drop-in
    (sm_100a router, dispatch, fused expert FFN, combine).  ``ffn1`` /
    ``ffn2`` exist in the reference but are never called; they are kept so
    that state dicts match;
  * the head: the configuration's MLP d_model -> 128 -> 1 (ReLU between)
    under the reference's attribute name ``linear``, then clamp(+-15) as in
    ``baseline/infer.py:437``; ``predict`` applies the sigmoid
    (``baseline/infer.py:686``).

Attention over the packed sequences runs on this library's varlen causal
attention kernel (``cti_varlen_attention``, head_dim 32); the reference
builds a dense [T, T] mask instead (``get_sequence_causal_mask``,
``baseline/infer.py:420-427``), which does not fit at T = 278k.  There is
no other backend: shapes the kernels do not cover raise.  This module
is the model around the hot path; the hot path itself is the MoE layer and
the pooling.
"""
from __future__ import annotations

from typing import NamedTuple

import numpy as np
import torch
import torch.nn as nn

from . import ops
from .embedding import RepEncoder
from .moe import SMoE


def causal_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                     cu_seqlens: torch.Tensor, max_seqlen: int) -> torch.Tensor:
    """Causal attention inside each packed sequence on this library's kernel
    (cti_varlen_attention, head_dim 32).  q, k, v [T, H, hd] bf16 CUDA
    views; cu_seqlens int32 [N+1]."""
    return ops.varlen_attention(q, k, v, cu_seqlens, max_seqlen)


class SequenceGroups(NamedTuple):
    """A packed batch cut into groups of whole sequences (plan_sequence_groups)."""
    groups: list        # (first sequence, end sequence, first token, end token) per group
    lo: np.ndarray      # [G, F] start of each group's ids of feature f in _flat_values
    hi: np.ndarray      # [G, F] end of those ids
    lens: np.ndarray    # [G, F] hi - lo
    val_offsets: np.ndarray  # [G, F] the group's own _val_offsets (ids laid out f by f)
    cu: np.ndarray      # the groups' sequence offsets, rebased to 0, concatenated
    cu_start: np.ndarray  # [G] where each group's offsets start in cu


def plan_sequence_groups(user_offsets: torch.Tensor, row_offsets: torch.Tensor,
                         val_offsets: torch.Tensor, slot_num: int, chunks: int) -> SequenceGroups:
    """Cuts a batch in the reference's flat layout (``_flat_row_offsets``
    [slot_num*(T+1)] per-feature offsets, ``_val_offsets`` [slot_num],
    ``user_offsets`` [N+1] token offsets of the packed sequences) into up to
    ``chunks`` groups of whole sequences with about equal token counts.  Group
    g holds tokens [a, b); its ids of feature f are ``_flat_values[lo[g, f]:
    hi[g, f]]``; laid out feature by feature they form the group's own flat
    batch, whose row offsets are the slice [a, b] of each feature's offsets
    minus its first value and whose val_offsets are ``val_offsets[g]``."""
    F = int(slot_num)
    uo = user_offsets.numpy()
    T = row_offsets.numel() // F - 1
    ro = row_offsets.numpy().reshape(F, T + 1)
    vo = val_offsets.numpy()
    cuts = np.searchsorted(uo, np.linspace(0, T, max(1, int(chunks)) + 1)[1:-1])
    bounds = np.unique(np.concatenate([[0], cuts, [uo.size - 1]]))
    groups = []
    for s0, s1 in zip(bounds[:-1], bounds[1:]):
        a, b = int(uo[s0]), int(uo[s1])
        if b > a:
            groups.append((int(s0), int(s1), a, b))
    lo = vo[None, :] + ro[:, [g[2] for g in groups]].T
    hi = vo[None, :] + ro[:, [g[3] for g in groups]].T
    lens = hi - lo
    g_vo = np.zeros_like(lens)
    g_vo[:, 1:] = np.cumsum(lens, axis=1)[:, :-1]
    cu = np.concatenate([uo[s0:s1 + 1] - a for (s0, s1, a, _b) in groups]) if groups else \
        np.zeros(0, dtype=np.int64)
    starts = np.cumsum([0] + [s1 - s0 + 1 for (s0, s1, _a, _b) in groups])[:-1]
    return SequenceGroups(groups, lo, hi, lens, g_vo, cu.astype(np.int64),
                          np.asarray(starts, dtype=np.int64))


class TransformerEncoder(nn.Module):
    """``TransformerEncoder`` of ``baseline/infer.py:360-411`` with the MoE
    drop-in.  ``forward(x [T, D] or [1, T, D], extension)`` where
    ``extension`` holds ``cu_seqlens`` (int32 [N+1]) and ``max_seqlen``, and
    optionally ``mark(name)``, called after each layer's attention block
    ("attention") and MoE block ("moe") is enqueued (the benchmark records
    CUDA events there)."""

    def __init__(self, d_model: int, n_heads: int, num_layers: int, dim_ff: int,
                 num_experts: int = 8, activation: str = "gelu", renormalize: bool = True):
        super().__init__()
        if d_model % n_heads:
            raise ValueError("d_model must be a multiple of n_heads")
        self.d_model = d_model
        self.n_heads = n_heads
        self.head_dim = d_model // n_heads
        self.num_layers = num_layers
        self.qkv_proj = nn.ModuleList([nn.Linear(d_model, 3 * d_model) for _ in range(num_layers)])
        self.out_proj = nn.ModuleList([nn.Linear(d_model, d_model) for _ in range(num_layers)])
        self.ffn1 = nn.ModuleList([nn.Linear(d_model, dim_ff) for _ in range(num_layers)])
        self.ffn2 = nn.ModuleList([nn.Linear(dim_ff, d_model) for _ in range(num_layers)])
        self.norm1 = nn.ModuleList([nn.LayerNorm(d_model) for _ in range(num_layers)])
        self.norm2 = nn.ModuleList([nn.LayerNorm(d_model) for _ in range(num_layers)])
        self.moe = nn.ModuleList([
            SMoE(d_model, dim_ff, num_experts, k=2, activation=activation,
                 renormalize=renormalize)
            for _ in range(num_layers)
        ])

    @torch.no_grad()
    def prepare_for_inference(self) -> None:
        """Stores each qkv projection with its output rows reordered from the
        reference's per-head [q_h | k_h | v_h] interleave to [q | k | v], so
        that q, k and v are strided views of one GEMM output (no copies).
        The parameters themselves keep the reference layout."""
        D, H, hd = self.d_model, self.n_heads, self.head_dim
        w0 = self.qkv_proj[0].weight
        perm = torch.arange(3 * D, device=w0.device).view(H, 3, hd).transpose(0, 1).reshape(-1)
        self._qkv = [(l.weight[perm].contiguous(), l.bias[perm].contiguous()) for l in self.qkv_proj]
        self._prepared = (w0.device, w0.dtype)

    def _add_norm(self, x, r, norm):
        """(x + r, norm(x + r)) on the fused sm_100a kernel (bf16 rows; the
        kernel raises for widths it does not cover)."""
        return ops.add_layernorm(x, r, norm.weight, norm.bias, norm.eps)

    @torch.no_grad()
    def forward(self, x: torch.Tensor, extension: dict):
        squeeze = x.dim() == 3
        x = x.reshape(-1, self.d_model)
        w0 = self.qkv_proj[0].weight
        if getattr(self, "_prepared", None) != (w0.device, w0.dtype):
            self.prepare_for_inference()
        cu = extension["cu_seqlens"]
        max_len = int(extension["max_seqlen"])
        T = x.shape[0]
        H, hd = self.n_heads, self.head_dim
        mark = extension.get("mark") or (lambda name: None)
        pending = None  # the previous layer's MoE output, not yet added
        for i in range(self.num_layers):
            x, h = self._add_norm(x, pending, self.norm1[i])
            qkv = torch.nn.functional.linear(h, *self._qkv[i]).view(T, 3, H, hd)
            a = causal_attention(qkv[:, 0], qkv[:, 1], qkv[:, 2], cu, max_len).reshape(
                T, self.d_model)
            x, h = self._add_norm(x, self.out_proj[i](a), self.norm2[i])
            mark("attention")
            moe_out, _ = self.moe[i](h.unsqueeze(0))
            pending = moe_out[0]
            mark("moe")
        if pending is not None:
            x = x + pending
        return (x.unsqueeze(0) if squeeze else x), None


class CTRModel(nn.Module):
    """``CTRModel`` of ``baseline/infer.py:414-439`` with the configuration's
    MLP head.  ``forward(batch)`` reads the flat pooling layout plus
    ``user_offsets`` (int64 [N+1], token offsets of the packed sequences)
    and returns ``(logits [T, 1] clamped to +-15, None)``."""

    def __init__(self, rep_encoder: RepEncoder, seq_encoder: TransformerEncoder, d_model: int,
                 head_hidden: int = 128):
        super().__init__()
        self.rep_encoder = rep_encoder
        self.seq_encoder = seq_encoder
        self.d_model = d_model
        self.linear = nn.Sequential(nn.Linear(d_model, head_hidden), nn.ReLU(),
                                    nn.Linear(head_hidden, 1))

    @torch.no_grad()
    def prepare_for_inference(self, dtype: torch.dtype = torch.bfloat16) -> "CTRModel":
        """Casts the model to ``dtype`` for inference, except the routers,
        which stay fp32 (the fp32 router of the MoE layer).  The embedding
        tables are fp16, the pooling kernel's input type."""
        # Take the table and the routers out while the rest is cast, so that
        # their values never pass through `dtype`.
        emb = self.rep_encoder.emb
        self.rep_encoder.emb = None
        gates = [m.gate for m in self.seq_encoder.moe]
        for m in self.seq_encoder.moe:
            m.gate = None
        self.to(dtype)
        self.rep_encoder.emb = emb.half()
        for m, g in zip(self.seq_encoder.moe, gates):
            m.gate = g.float()
            m.prepare_for_inference()
        self.seq_encoder.prepare_for_inference()
        self._prepare_head()
        return self

    @torch.no_grad()
    def _prepare_head(self) -> None:
        """The head's weights as the fused head kernel takes them: W1 bf16,
        b1 / w2 / b2 fp32."""
        l1, l2 = self.linear[0], self.linear[2]
        self._head = (l1.weight.detach().to(torch.bfloat16).contiguous(),
                      l1.bias.detach().float().contiguous(),
                      l2.weight.detach().float().reshape(-1).contiguous(),
                      l2.bias.detach().float().reshape(1).contiguous(),
                      l1.weight.device)

    @staticmethod
    def sequence_info(batch: dict, device) -> tuple[torch.Tensor, int]:
        uo = batch["user_offsets"]
        cu = uo.to(device=device, dtype=torch.int32, non_blocking=True)
        if "max_seqlen" in batch:
            max_len = int(batch["max_seqlen"])
        else:
            max_len = int((uo[1:] - uo[:-1]).max())
        return cu, max_len

    @torch.no_grad()
    def forward(self, batch: dict):
        dev = self.linear[0].weight.device
        cu, max_len = self.sequence_info(batch, dev)
        x = self.rep_encoder(batch)
        h, _ = self.seq_encoder(x, {"cu_seqlens": cu, "max_seqlen": max_len})
        logits, _ = self.head(h, want_probs=False)
        return logits.reshape(-1, 1), None

    @torch.no_grad()
    def head(self, h: torch.Tensor, want_logits: bool = True, want_probs: bool = True):
        """The MLP head, clamped to +-15 (baseline/infer.py:437), and the
        sigmoid of predict (:686), in one launch (cti_ctr_head): returns
        (logits [T] fp32 or None, probabilities [T] fp32 or None)."""
        if getattr(self, "_head", None) is None or self._head[4] != self.linear[0].weight.device:
            self._prepare_head()
        w1, b1, w2, b2, _ = self._head
        return ops.ctr_head(h.reshape(-1, self.d_model), w1, b1, w2, b2, 15.0,
                            want_logits=want_logits, want_probs=want_probs)

    def _probs(self, batch: dict) -> torch.Tensor:
        dev = self.linear[0].weight.device
        cu, max_len = self.sequence_info(batch, dev)
        x = self.rep_encoder(batch)
        h, _ = self.seq_encoder(x, {"cu_seqlens": cu, "max_seqlen": max_len})
        return self.head(h, want_logits=False)[1]

    @torch.no_grad()
    def predict(self, batch: dict) -> torch.Tensor:
        """CTR probabilities [T] (fp32)."""
        return self._probs(batch)

    @torch.no_grad()
    def predict_host(self, batch: dict, chunks: int = 8,
                     out: torch.Tensor | None = None) -> torch.Tensor:
        """``predict`` for a batch in host memory (the reference's flat layout,
        ``online_best/infer.py:742-779`` moves it to the GPU before the
        forward): the packed sequences are cut into ``chunks`` groups of
        about equal token count; every group's ids and offsets are copied
        on a side stream first, and each group's forward starts as soon as
        its own copies have landed, overlapping the later groups' copies.  Every sequence is computed independently (pooling and
        MoE per token, attention inside the sequence), so the chunks give
        the whole batch's probabilities; only the library GEMMs' choice of
        kernel may change with the row count, within rounding.

        ``batch``: CPU int64 ``_flat_values``, ``_flat_row_offsets``
        [slot_num*(T+1)], ``_val_offsets`` [slot_num], ``user_offsets``
        [N+1] (page-locked for the copies to overlap).  Returns page-locked
        fp32 probabilities [T] (``out`` if given), valid once the current
        stream is synchronised."""
        dev = self.linear[0].weight.device
        F = self.rep_encoder.slot_num
        vals, ro, vo, uo = (batch[k] for k in ("_flat_values", "_flat_row_offsets",
                                               "_val_offsets", "user_offsets"))
        for name, t in (("_flat_values", vals), ("_flat_row_offsets", ro),
                        ("_val_offsets", vo), ("user_offsets", uo)):
            if t.is_cuda or t.dtype != torch.int64 or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous CPU int64 tensor")
        if ro.numel() % F:
            raise ValueError("_flat_row_offsets length must be a multiple of slot_num")
        T = ro.numel() // F - 1
        if int(uo[0]) != 0 or int(uo[-1]) != T:
            raise ValueError("user_offsets must run from 0 to the token count")
        if out is None:
            out = torch.empty(T, dtype=torch.float32, pin_memory=True)
        if T == 0:
            return out
        plan = plan_sequence_groups(uo, ro, vo, F, chunks)
        groups, lo, hi, lens = plan.groups, plan.lo, plan.hi, plan.lens
        # The groups' val_offsets and rebased sequence offsets, copied to the
        # GPU at once.
        small_h = torch.empty(len(groups) * F + plan.cu.size, dtype=torch.int64, pin_memory=True)
        sm = small_h.numpy()
        sm[:len(groups) * F] = plan.val_offsets.reshape(-1)
        sm[len(groups) * F:] = plan.cu
        cu_pos = [len(groups) * F + int(c) for c in plan.cu_start]
        uo_np = uo.numpy()

        total_vals = int(lens.sum())
        need = (total_vals, F * (T + len(groups)), small_h.numel())
        st = getattr(self, "_host_stage", None)
        if st is None or st[0].device != dev or any(x.numel() < n for x, n in zip(st, need)):
            st = tuple(torch.empty(n, dtype=torch.int64, device=dev) for n in need)
            self._host_stage = st
        vals_d, ro_d, small_d = st
        s_in = getattr(self, "_copy_stream", None)
        if s_in is None or s_in.device != dev:
            s_in = torch.cuda.Stream(dev)
            self._copy_stream = s_in
        s_comp = torch.cuda.current_stream(dev)
        s_in.wait_stream(s_comp)  # staging buffers are free once earlier work is done
        with torch.cuda.stream(s_in):
            small_d[:small_h.numel()].copy_(small_h, non_blocking=True)
        # Every group's copies first, so that the copy stream runs back to
        # back whatever the host's launch rate for the forwards below.
        vp = rp = 0
        staged = []
        for gi, (s0, s1, a, b) in enumerate(groups):
            n = b - a
            v0, r0 = vp, rp
            with torch.cuda.stream(s_in):
                for f in range(F):
                    ln = int(lens[gi, f])
                    if ln:
                        vals_d[vp:vp + ln].copy_(vals[int(lo[gi, f]):int(hi[gi, f])],
                                                 non_blocking=True)
                    vp += ln
                    base = f * (T + 1)
                    ro_d[rp:rp + n + 1].copy_(ro[base + a:base + b + 1], non_blocking=True)
                    rp += n + 1
                ready = torch.cuda.Event()
                ready.record(s_in)
            staged.append((v0, vp, r0, rp, ready))
        for gi, (s0, s1, a, b) in enumerate(groups):
            n = b - a
            v0, v1, r0, r1, ready = staged[gi]
            s_comp.wait_event(ready)
            ro_g = ro_d[r0:r1].view(F, n + 1)
            ro_g.sub_(ro_g[:, :1].clone())
            cu = small_d[cu_pos[gi]:cu_pos[gi] + s1 - s0 + 1]
            sub = {"_flat_values": vals_d[v0:v1], "_flat_row_offsets": ro_g.view(-1),
                   "_val_offsets": small_d[gi * F:(gi + 1) * F], "user_offsets": cu,
                   "max_seqlen": int((uo_np[s0 + 1:s1 + 1] - uo_np[s0:s1]).max())}
            out[a:b].copy_(self._probs(sub), non_blocking=True)
        return out


def build_ctr_model(vocab_sizes, emb_dim: int = 64, slot_num: int = 28, d_model: int = 256,
                    n_heads: int = 8, num_layers: int = 8, dim_ff: int = 1024,
                    num_experts: int = 16, head_hidden: int = 128) -> CTRModel:
    """The configuration-4 model: per-slot tables, 8 layers of 8 heads x 32,
    16 experts of d_ff 1024, MLP head 256 -> 128 -> 1."""
    rep = RepEncoder(vocab_size=int(sum(vocab_sizes)), emb_dim=emb_dim, padding_idx=0,
                     slot_num=slot_num, d_model=d_model, vocab_sizes=vocab_sizes)
    enc = TransformerEncoder(d_model, n_heads, num_layers, dim_ff, num_experts)
    return CTRModel(rep, enc, d_model, head_hidden)
