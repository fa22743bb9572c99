"""Tensor-level wrappers of the five hot-path stages.

Each function validates its tensors, passes raw device pointers and the
current CUDA stream to one ``libcti_b200.so`` entry point, and returns torch
tensors.  They are the building blocks of :class:`SMoE` and
:class:`RepEncoder`, and what the parity tests drive stage by stage.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from ._lib import check, lib, ptr, require_cuda, stream_handle, status_word


@dataclass
class RouterOut:
    idx2: torch.Tensor  # [T, 2] int32 expert ids (top-1, top-2)
    gate2: torch.Tensor  # [T, 2] fp32 gate weights
    route_rank: torch.Tensor  # [T, 2] int32 rank inside the 128-token router block
    block_hist: torch.Tensor  # [ceil(T/128), E] int32 per-block expert counts


@dataclass
class DispatchOut:
    offsets: torch.Tensor  # [E+1] int32 expert segment starts
    perm_inv: torch.Tensor  # [T, 2] int32 sorted position of each route
    sorted_token: torch.Tensor  # [2T] int32 token of each sorted row
    xperm: torch.Tensor | None  # [2T, D] bf16 rows in expert order


def router(x: torch.Tensor, wg: torch.Tensor, bg: torch.Tensor, renorm: bool = True) -> RouterOut:
    """Stage 1: fp32 Top-2 router (see cti_moe_router)."""
    require_cuda(x, "x", torch.bfloat16)
    require_cuda(wg, "wg", torch.float32)
    require_cuda(bg, "bg", torch.float32)
    T, D = x.shape
    E = wg.shape[0]
    dev = x.device
    nblk = (T + _lib.ROUTER_BLOCK_TOKENS - 1) // _lib.ROUTER_BLOCK_TOKENS
    idx2 = torch.empty((T, 2), dtype=torch.int32, device=dev)
    gate2 = torch.empty((T, 2), dtype=torch.float32, device=dev)
    rank = torch.empty((T, 2), dtype=torch.int32, device=dev)
    hist = torch.empty((max(nblk, 1), E), dtype=torch.int32, device=dev)
    check(
        lib.cti_moe_router(
            ptr(x), ptr(wg), ptr(bg), T, D, E, int(renorm), ptr(idx2), ptr(gate2), ptr(rank),
            ptr(hist), ptr(status_word(dev)), stream_handle(dev),
        ),
        "cti_moe_router",
    )
    return RouterOut(idx2, gate2, rank, hist)


def dispatch(x: torch.Tensor, r: RouterOut, num_experts: int, permute: bool = True) -> DispatchOut:
    """Stage 2: offsets + stable permutation of rows into expert order.

    Consumes ``r.block_hist`` (rewritten in place into per-block bases)."""
    require_cuda(x, "x", torch.bfloat16)
    T, D = x.shape
    dev = x.device
    offsets = torch.empty(num_experts + 1, dtype=torch.int32, device=dev)
    perm_inv = torch.empty((T, 2), dtype=torch.int32, device=dev)
    sorted_token = torch.empty(2 * T, dtype=torch.int32, device=dev)
    xperm = torch.empty((2 * T, D), dtype=torch.bfloat16, device=dev) if permute else None
    check(
        lib.cti_moe_dispatch(
            ptr(x), ptr(r.idx2), ptr(r.route_rank), ptr(r.block_hist), T, D, num_experts,
            ptr(offsets), ptr(perm_inv), ptr(sorted_token), ptr(xperm),
            ptr(status_word(dev)), stream_handle(dev),
        ),
        "cti_moe_dispatch",
    )
    return DispatchOut(offsets, perm_inv, sorted_token, xperm)


def grouped_gemm(
    a: torch.Tensor,
    w: torch.Tensor,
    bias: torch.Tensor | None,
    group_offsets: torch.Tensor,
    act: str = "none",
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Stage 3: C = act(A[group rows] @ W[g % Gw]^T + bias[g % Gw]).

    a [rows, K] bf16; w [Gw, N, K] bf16; bias [Gw, N] fp32 or None;
    group_offsets [G+1] int32 on the device."""
    require_cuda(a, "A", torch.bfloat16)
    require_cuda(w, "W", torch.bfloat16)
    require_cuda(group_offsets, "group_offsets", torch.int32)
    if bias is not None:
        require_cuda(bias, "bias", torch.float32)
    rows, K = a.shape
    Gw, N, K2 = w.shape
    if K2 != K:
        raise ValueError(f"K mismatch: A has {K}, W has {K2}")
    G = group_offsets.numel() - 1
    dev = a.device
    if out is None:
        out = torch.empty((rows, N), dtype=torch.bfloat16, device=dev)
    check(
        lib.cti_moe_grouped_gemm(
            ptr(a), ptr(w), ptr(bias), ptr(group_offsets), G, Gw, rows, N, K,
            _lib.ACTIVATIONS[act], ptr(out), ptr(status_word(dev)), stream_handle(dev),
        ),
        "cti_moe_grouped_gemm",
    )
    return out


def expert_ffn_fused(
    xp: torch.Tensor,
    w1: torch.Tensor,
    b1: torch.Tensor,
    w2: torch.Tensor,
    b2: torch.Tensor,
    group_offsets: torch.Tensor,
    act: str = "gelu",
    out: torch.Tensor | None = None,
    pair: bool = False,
) -> torch.Tensor:
    """Stage 3, fused: Y = act(Xp @ W1[e]^T + b1[e]) @ W2[e]^T + b2[e] per group.
    ``pair``: the CTA-pair kernel (cti_moe_expert_ffn_fused_pair, d_model 256)."""
    require_cuda(xp, "Xp", torch.bfloat16)
    require_cuda(w1, "W1", torch.bfloat16)
    require_cuda(w2, "W2", torch.bfloat16)
    require_cuda(b1, "b1", torch.float32)
    require_cuda(b2, "b2", torch.float32)
    rows, D = xp.shape
    Gw, F, _ = w1.shape
    G = group_offsets.numel() - 1
    dev = xp.device
    if out is None:
        out = torch.empty((rows, D), dtype=torch.bfloat16, device=dev)
    fn = lib.cti_moe_expert_ffn_fused_pair if pair else lib.cti_moe_expert_ffn_fused
    check(
        fn(
            ptr(xp), ptr(w1), ptr(b1), ptr(w2), ptr(b2), ptr(group_offsets), G, Gw, rows, D, F,
            _lib.ACTIVATIONS[act], ptr(out), ptr(status_word(dev)), stream_handle(dev),
        ),
        "cti_moe_expert_ffn_fused_pair" if pair else "cti_moe_expert_ffn_fused",
    )
    return out


def expert_ffn_fused_gather(
    x: torch.Tensor,
    sorted_token: torch.Tensor,
    w1: torch.Tensor,
    b1: torch.Tensor,
    w2: torch.Tensor,
    b2: torch.Tensor,
    group_offsets: torch.Tensor,
    act: str = "gelu",
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Stage 3, fused, rows gathered in the kernel: row r is x[sorted_token[r]]
    (no dispatched copy of the rows).  Equals expert_ffn_fused on the
    dispatched rows bit for bit."""
    require_cuda(x, "x", torch.bfloat16)
    require_cuda(sorted_token, "sorted_token", torch.int32)
    require_cuda(w1, "W1", torch.bfloat16)
    require_cuda(w2, "W2", torch.bfloat16)
    require_cuda(b1, "b1", torch.float32)
    require_cuda(b2, "b2", torch.float32)
    T, D = x.shape
    rows = sorted_token.numel()
    Gw, F, _ = w1.shape
    G = group_offsets.numel() - 1
    dev = x.device
    if out is None:
        out = torch.empty((rows, D), dtype=torch.bfloat16, device=dev)
    check(
        lib.cti_moe_expert_ffn_fused_gather(
            ptr(x), T, ptr(sorted_token), ptr(w1), ptr(b1), ptr(w2), ptr(b2), ptr(group_offsets),
            G, Gw, rows, D, F, _lib.ACTIVATIONS[act], ptr(out), ptr(status_word(dev)),
            stream_handle(dev),
        ),
        "cti_moe_expert_ffn_fused_gather",
    )
    return out


def combine(y: torch.Tensor, perm_inv: torch.Tensor, gate2: torch.Tensor,
            out: torch.Tensor | None = None) -> torch.Tensor:
    """Stage 4: out[t] = g0*Y[perm_inv[t,0]] + g1*Y[perm_inv[t,1]] (fp32 math, bf16 out)."""
    require_cuda(y, "Y", torch.bfloat16)
    require_cuda(perm_inv, "perm_inv", torch.int32)
    require_cuda(gate2, "gate2", torch.float32)
    T = perm_inv.shape[0]
    D = y.shape[1]
    dev = y.device
    if out is None:
        out = torch.empty((T, D), dtype=torch.bfloat16, device=dev)
    check(
        lib.cti_moe_combine(
            ptr(y), y.shape[0], ptr(perm_inv), ptr(gate2), T, D, ptr(out),
            ptr(status_word(dev)), stream_handle(dev),
        ),
        "cti_moe_combine",
    )
    return out


def embedding_bag_sum(
    values: torch.Tensor,
    row_offsets: torch.Tensor,
    val_offsets: torch.Tensor,
    table: torch.Tensor,
    table_row_base: torch.Tensor,
    vocab: torch.Tensor,
    num_features: int,
    out_dtype: torch.dtype = torch.float32,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Stage 5: pooled[b, f*dim:(f+1)*dim] = sum of clamped table rows of bag (b, f).

    The reference's flat layout: values int64 [N]; row_offsets int64
    [F*(B+1)] per-feature offsets; val_offsets int64 [F]."""
    for name, t in (("values", values), ("row_offsets", row_offsets),
                    ("val_offsets", val_offsets), ("table_row_base", table_row_base),
                    ("vocab", vocab)):
        require_cuda(t, name, torch.int64)
    require_cuda(table, "table", torch.float16)
    F = num_features
    if row_offsets.numel() % F != 0:
        raise ValueError("row_offsets length must be a multiple of the feature count")
    B = row_offsets.numel() // F - 1
    dim = table.shape[1]
    dev = table.device
    if out is None:
        out = torch.empty((B, F * dim), dtype=out_dtype, device=dev)
    check(
        lib.cti_embbag_sum(
            ptr(values), values.numel(), ptr(row_offsets), ptr(val_offsets),
            ptr(table_row_base), ptr(vocab), ptr(table), table.shape[0], B, F, dim, ptr(out),
            _lib.DTYPE_CODES[out.dtype], ptr(status_word(dev)), stream_handle(dev),
        ),
        "cti_embbag_sum",
    )
    return out


def rep_encoder_fused(values: torch.Tensor, row_offsets: torch.Tensor, val_offsets: torch.Tensor,
                      table: torch.Tensor, table_row_base: torch.Tensor, vocab: torch.Tensor,
                      num_features: int, wg: torch.Tensor, r1: torch.Tensor, c: torch.Tensor,
                      eps: float = 1e-5, out: torch.Tensor | None = None) -> torch.Tensor:
    """The RepEncoder in one launch (cti_rep_encoder_fused): the embedding-bag
    pooling of ``embedding_bag_sum`` (64-wide fp16 rows), LayerNorm over the
    pooled row and the Linear, with the LayerNorm folded into the weights:
    ``wg`` bf16 [N, F*64] = W * gamma, ``r1`` fp32 [N] = wg.float().sum(1),
    ``c`` fp32 [N] = W beta + b.  Returns bf16 [B, N]; N in {128, 256}."""
    for name, t in (("values", values), ("row_offsets", row_offsets),
                    ("val_offsets", val_offsets), ("table_row_base", table_row_base),
                    ("vocab", vocab)):
        require_cuda(t, name, torch.int64)
    require_cuda(table, "table", torch.float16)
    require_cuda(wg, "wg", torch.bfloat16)
    require_cuda(r1, "r1", torch.float32)
    require_cuda(c, "c", torch.float32)
    F = num_features
    if row_offsets.numel() % F != 0:
        raise ValueError("row_offsets length must be a multiple of the feature count")
    B = row_offsets.numel() // F - 1
    dim = table.shape[1]
    N = wg.shape[0]
    if wg.shape[1] != F * dim or r1.numel() != N or c.numel() != N:
        raise ValueError("wg must be [N, F*dim] with r1, c of length N")
    dev = table.device
    if out is None:
        out = torch.empty((B, N), dtype=torch.bfloat16, device=dev)
    check(
        lib.cti_rep_encoder_fused(
            ptr(values), values.numel(), ptr(row_offsets), ptr(val_offsets),
            ptr(table_row_base), ptr(vocab), ptr(table), table.shape[0], B, F, dim, ptr(wg),
            ptr(r1), ptr(c), N, float(eps), ptr(out), ptr(status_word(dev)), stream_handle(dev),
        ),
        "cti_rep_encoder_fused",
    )
    return out


def add_layernorm(x: torch.Tensor, residual: torch.Tensor | None, weight: torch.Tensor,
                  bias: torch.Tensor, eps: float = 1e-5, write_sum: bool = True):
    """The CTR model's residual add + LayerNorm: s = x + residual (bf16), out =
    LayerNorm(s).  Returns (s, out); s is x itself when residual is None.
    x, residual [rows, cols] bf16; weight, bias [cols] bf16."""
    require_cuda(x, "x", torch.bfloat16)
    if residual is not None:
        require_cuda(residual, "residual", torch.bfloat16)
        if residual.shape != x.shape:
            raise ValueError("x and residual must have the same shape")
    require_cuda(weight, "weight", torch.bfloat16)
    require_cuda(bias, "bias", torch.bfloat16)
    cols = x.shape[-1]
    rows = x.numel() // cols if cols else 0
    dev = x.device
    out = torch.empty_like(x)
    s = torch.empty_like(x) if (residual is not None and write_sum) else None
    check(
        lib.cti_add_layernorm(ptr(x), ptr(residual), ptr(weight), ptr(bias), rows, cols,
                              float(eps), ptr(s), ptr(out), stream_handle(dev)),
        "cti_add_layernorm",
    )
    return (x if residual is None else s), out


def varlen_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                     cu_seqlens: torch.Tensor, max_seqlen: int) -> torch.Tensor:
    """Causal attention inside packed sequences.  q, k, v [T, H, 32] bf16
    views whose last two dims are contiguous (any token stride, e.g. the
    thirds of one qkv projection); cu_seqlens int32 [N+1].  Returns a new
    contiguous [T, H, 32] bf16 tensor."""
    T, H, hd = q.shape
    for name, t in (("q", q), ("k", k), ("v", v)):
        if not t.is_cuda or t.dtype != torch.bfloat16:
            raise TypeError(f"{name} must be a bf16 CUDA tensor")
        if t.shape != q.shape or t.stride(2) != 1 or t.stride(1) != hd:
            raise ValueError(f"{name} must be [T, H, head_dim] with contiguous heads")
    require_cuda(cu_seqlens, "cu_seqlens", torch.int32)
    out = torch.empty((T, H, hd), dtype=torch.bfloat16, device=q.device)
    check(
        lib.cti_varlen_attention(ptr(q), ptr(k), ptr(v), q.stride(0), k.stride(0), v.stride(0),
                                 ptr(cu_seqlens), cu_seqlens.numel() - 1, int(max_seqlen), T, H,
                                 hd, ptr(out), ptr(status_word(q.device)),
                                 stream_handle(q.device)),
        "cti_varlen_attention",
    )
    return out


def ctr_head(h: torch.Tensor, w1: torch.Tensor, b1: torch.Tensor, w2: torch.Tensor,
             b2: torch.Tensor, limit: float = 15.0, want_logits: bool = True,
             want_probs: bool = True):
    """The CTR head in one launch (cti_ctr_head): logits = clamp(w2 .
    relu(W1 h + b1) + b2, +-limit) and probs = sigmoid(logits), fp32 [T].
    h [T, D] bf16; w1 [Hd, D] bf16; b1 [Hd], w2 [Hd], b2 [1] fp32.  Returns
    (logits or None, probs or None)."""
    require_cuda(h, "h", torch.bfloat16)
    require_cuda(w1, "W1", torch.bfloat16)
    for name, t in (("b1", b1), ("w2", w2), ("b2", b2)):
        require_cuda(t, name, torch.float32)
    T, D = h.shape
    Hd = w1.shape[0]
    dev = h.device
    logits = torch.empty(T, dtype=torch.float32, device=dev) if want_logits else None
    probs = torch.empty(T, dtype=torch.float32, device=dev) if want_probs else None
    check(
        lib.cti_ctr_head(ptr(h), ptr(w1), ptr(b1), ptr(w2), ptr(b2), T, D, Hd, float(limit),
                         ptr(logits), ptr(probs), ptr(status_word(dev)), stream_handle(dev)),
        "cti_ctr_head",
    )
    return logits, probs
