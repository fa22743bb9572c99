"""Varlen causal attention kernel (cti_varlen_attention) against a plain fp32
softmax per sequence.  Tolerance: max rel err 1e-2 (bf16 inputs and output,
fp32 scores and softmax)."""
import pytest
import torch

from helpers import max_rel_err

pytestmark = pytest.mark.gpu


def _reference(q, k, v, cu):
    out = torch.empty(q.shape, dtype=torch.float32)
    c = cu.tolist()
    for a, b in zip(c[:-1], c[1:]):
        if b <= a:
            continue
        qs, ks, vs = (t[a:b].float().transpose(0, 1) for t in (q, k, v))
        s = qs @ ks.transpose(-1, -2) / 32 ** 0.5
        m = torch.ones(b - a, b - a, dtype=torch.bool).tril()
        s = s.masked_fill(~m, float("-inf"))
        out[a:b] = (torch.softmax(s, -1) @ vs).transpose(0, 1)
    return out


@pytest.mark.parametrize("lens", [[1, 2, 63, 64, 65, 127, 128, 129, 256],
                                  [300, 5, 0, 17],
                                  [256] * 8])
@pytest.mark.parametrize("strided", [False, True])
def test_varlen_attention_matches_softmax(cuda_device, lens, strided):
    from cti_b200 import ops

    g = torch.Generator().manual_seed(sum(lens) + strided)
    cu = torch.zeros(len(lens) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(lens), 0)
    T, H = int(cu[-1]), 8
    qkv = (torch.randn(T, 3, H, 32, generator=g) * 2).bfloat16()
    if strided:  # q, k, v as thirds of one projection output
        q, k, v = (qkv[:, i] for i in range(3))
    else:
        q, k, v = (qkv[:, i].contiguous() for i in range(3))
    dev = cuda_device
    qd, kd, vd = (t.to(dev) for t in (q, k, v)) if not strided else \
        (lambda x: (x[:, 0], x[:, 1], x[:, 2]))(qkv.to(dev))
    out = ops.varlen_attention(qd, kd, vd, cu.to(dev), max(lens))
    ref = _reference(q, k, v, cu)
    assert out.shape == (T, H, 32)
    assert max_rel_err(out.float().cpu(), ref) < 1e-2


def test_varlen_attention_rejects_other_head_dims(cuda_device):
    from cti_b200 import _lib

    assert _lib.lib.cti_varlen_attention(None, None, None, 64, 64, 64, None, 1, 8, 1, 64, None,
                                         None) == _lib.CTI_ERR_UNSUPPORTED
