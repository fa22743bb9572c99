"""Torch references for the varlen causal attention kernel (test only).

The model always runs this library's kernel (cti_varlen_attention); these
two PyTorch formulations of the same attention are what the GPU tests
compare it with: PyTorch's variable-length flash attention, and
scaled_dot_product_attention over sequences padded to the longest one.
"""
import torch


def varlen_causal_attention(q, k, v, cu_seqlens, max_seqlen):
    """Causal attention inside each packed sequence.  q, k, v [T, H, hd]
    (bf16, CUDA); cu_seqlens int32 [N+1]."""
    from torch.nn.attention.varlen import varlen_attn

    return varlen_attn(q, k, v, cu_seqlens, cu_seqlens, max_seqlen, max_seqlen,
                       window_size=(-1, 0))


def padded_causal_attention(q, k, v, cu_seqlens, max_seqlen):
    """The same through scaled_dot_product_attention on sequences padded to
    max_seqlen.  Padding sits after each sequence's last token, so the
    causal mask alone keeps it out of every real query."""
    T, H, hd = q.shape
    N = cu_seqlens.numel() - 1
    starts = cu_seqlens[:-1].long()
    lens = (cu_seqlens[1:] - cu_seqlens[:-1]).long()
    seq = torch.repeat_interleave(torch.arange(N, device=q.device), lens)
    pos = torch.arange(T, device=q.device) - starts[seq]

    def pad(t):
        out = t.new_zeros(N, max_seqlen, H, hd)
        out[seq, pos] = t
        return out.transpose(1, 2)

    o = torch.nn.functional.scaled_dot_product_attention(pad(q), pad(k), pad(v), is_causal=True)
    return o.transpose(1, 2)[seq, pos]
