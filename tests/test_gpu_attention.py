"""Varlen causal attention kernel (cti_varlen_attention) against a plain fp32
softmax per sequence.  Tolerance: max rel err 1e-2 (bf16 inputs, bf16 P
into the PV product, bf16 output; fp32 scores, softmax and accumulation)."""
import ctypes

import pytest
import torch

from helpers import max_rel_err

pytestmark = pytest.mark.gpu


def _reference(q, k, v, cu):
    out = torch.zeros(q.shape, dtype=torch.float32)
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


def _cu(lens, first=0):
    cu = torch.zeros(len(lens) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(lens), 0)
    return cu + first


@pytest.mark.parametrize("lens", [[1, 2, 63, 64, 65, 127, 128, 129, 256],
                                  [300, 5, 0, 17],
                                  [256] * 8,
                                  [1000, 3, 0, 700, 129],
                                  [1] * 300,
                                  [0, 0, 130, 0]])
@pytest.mark.parametrize("strided", [False, True])
def test_varlen_attention_matches_softmax(cuda_device, lens, strided):
    from cti_b200 import ops

    g = torch.Generator().manual_seed(sum(lens) + strided)
    cu = _cu(lens)
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


@pytest.mark.parametrize("seed", [0, 1])
def test_varlen_attention_cfg4_lengths(cuda_device, seed):
    """Configuration-4 shape: packed sequences with lengths U{16..256}, 8
    heads, q/k/v thirds of one [T, 768] projection."""
    from cti_b200 import ops, synth

    lens = synth.packed_lengths(96, 16, 256, seed).tolist()
    cu = _cu(lens)
    T, H = int(cu[-1]), 8
    g = torch.Generator().manual_seed(seed)
    qkv = (torch.randn(T, 3, H, 32, generator=g) * 2).bfloat16()
    x = qkv.to(cuda_device)
    out = ops.varlen_attention(x[:, 0], x[:, 1], x[:, 2], cu.to(cuda_device), 256)
    ref = _reference(qkv[:, 0], qkv[:, 1], qkv[:, 2], cu)
    assert max_rel_err(out.float().cpu(), ref) < 1e-2


def test_varlen_attention_writes_only_sequence_tokens(cuda_device):
    """cu[0] > 0 and cu[-1] < tokens: rows outside [cu[0], cu[-1]) keep their
    contents; the rows inside match the reference."""
    from cti_b200 import _lib

    lens = [40, 200, 7]
    first, tail = 37, 50
    cu = _cu(lens, first)
    T, H = int(cu[-1]) + tail, 4
    g = torch.Generator().manual_seed(5)
    q, k, v = ((torch.randn(T, H, 32, generator=g) * 2).bfloat16() for _ in range(3))
    dev = cuda_device
    qd, kd, vd = (t.to(dev) for t in (q, k, v))
    out = torch.full((T, H, 32), 7.0, dtype=torch.bfloat16, device=dev)
    status = torch.zeros(2, dtype=torch.int32, device=dev)
    cud = cu.to(dev)
    rc = _lib.lib.cti_varlen_attention(
        qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), H * 32, H * 32, H * 32, cud.data_ptr(),
        len(lens), max(lens), T, H, 32, out.data_ptr(), status.data_ptr(),
        ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    assert rc == 0
    torch.cuda.synchronize(dev)
    assert status.tolist() == [0, 0]
    o = out.float().cpu()
    assert (o[:first] == 7.0).all() and (o[int(cu[-1]):] == 7.0).all()
    ref = _reference(q, k, v, cu)
    a, b = first, int(cu[-1])
    assert max_rel_err(o[a:b], ref[a:b]) < 1e-2


def test_varlen_attention_rejects_other_head_dims(cuda_device):
    from cti_b200 import _lib

    assert _lib.lib.cti_varlen_attention(None, None, None, 64, 64, 64, None, 1, 8, 8, 1, 64, None,
                                         None, None) == _lib.CTI_ERR_UNSUPPORTED
