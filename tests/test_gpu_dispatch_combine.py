"""Stages 2 and 4 on the B200: dispatch (offsets, permutation, row copies)
bit-exact vs the reference's nonzero() order; combine vs fp32 math."""
import pytest
import torch

from helpers import max_rel_err
from oracle import moe_ref as mr

pytestmark = pytest.mark.gpu


def _route(T, D, E, dev, bias=None, seed=0):
    from cti_b200 import ops

    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, D, generator=g).bfloat16()
    wg = torch.randn(E, D, generator=g) * 0.05
    bg = torch.zeros(E) if bias is None else bias
    xd = x.to(dev)
    r = ops.router(xd, wg.to(dev), bg.to(dev))
    return x, xd, r


@pytest.mark.parametrize("T,D,E", [(1, 128, 8), (129, 128, 8), (4096, 128, 8),
                                   (69632, 256, 16), (5000, 1024, 64), (3000, 256, 128)])
def test_dispatch_matches_reference_order(cuda_device, T, D, E):
    from cti_b200 import _lib, ops

    x, xd, r = _route(T, D, E, cuda_device, seed=T)
    d = ops.dispatch(xd, r, E)
    _lib.raise_on_status(cuda_device)
    offs, sorted_token, perm_inv = mr.expert_segments(r.idx2.cpu().long(), E)
    assert torch.equal(d.offsets.cpu().long(), offs)
    assert torch.equal(d.sorted_token.cpu().long(), sorted_token)
    assert torch.equal(d.perm_inv.cpu().long(), perm_inv)
    assert torch.equal(d.xperm.cpu(), x[sorted_token])


def test_dispatch_all_tokens_to_two_experts_and_empty_experts(cuda_device):
    from cti_b200 import _lib, ops

    E = 16
    bias = torch.full((E,), -30.0)
    bias[5] = 20.0
    bias[11] = 10.0  # logit noise here has std ~0.8, far below these gaps
    x, xd, r = _route(2000, 256, E, cuda_device, bias=bias)
    assert (r.idx2[:, 0] == 5).all() and (r.idx2[:, 1] == 11).all()
    d = ops.dispatch(xd, r, E)
    _lib.raise_on_status(cuda_device)
    off = d.offsets.cpu().tolist()
    assert off[:6] == [0] * 6 and off[6:12] == [2000] * 6 and off[12:] == [4000] * 5
    assert torch.equal(d.sorted_token.cpu()[:2000].long(), torch.arange(2000))


def test_combine_matches_fp32_math(cuda_device):
    from cti_b200 import _lib, ops

    T, D, E = 3000, 256, 16
    x, xd, r = _route(T, D, E, cuda_device, seed=9)
    d = ops.dispatch(xd, r, E)
    y = torch.randn(2 * T, D, device=cuda_device).bfloat16()
    out = ops.combine(y, d.perm_inv, r.gate2)
    _lib.raise_on_status(cuda_device)
    p = d.perm_inv.long()
    g = r.gate2
    ref = g[:, :1] * y[p[:, 0]].float() + g[:, 1:] * y[p[:, 1]].float()
    assert max_rel_err(out, ref) < 4e-3  # one bf16 rounding of the result


def test_combine_rejects_out_of_range_positions(cuda_device):
    from cti_b200 import _lib, ops

    T, D = 64, 128
    y = torch.randn(10, D, device=cuda_device).bfloat16()
    perm_inv = torch.zeros(T, 2, dtype=torch.int32, device=cuda_device)
    perm_inv[7, 1] = 10  # one past the end of Y
    gate2 = torch.full((T, 2), 0.5, device=cuda_device)
    ops.combine(y, perm_inv, gate2)
    code, detail = _lib.read_status(cuda_device)
    assert code == _lib.CTI_ERR_BOUNDS and detail == 7


def test_dispatch_marks_rejected_tokens_in_perm_inv(cuda_device):
    """A route whose expert id is out of range (planted on the host after
    routing) is reported as CTI_ERR_BOUNDS with its token, and that token's
    perm_inv entry is (-1, -1), so the combine skips it deterministically
    instead of reading stale positions."""
    from cti_b200 import _lib, ops

    T, D, E = 500, 128, 8
    x, xd, r = _route(T, D, E, cuda_device, seed=4)
    r.idx2[123, 1] = E  # one past the last expert
    d = ops.dispatch(xd, r, E)
    code, detail = _lib.read_status(cuda_device)
    assert code == _lib.CTI_ERR_BOUNDS and detail == 123
    assert d.perm_inv[123].tolist() == [-1, -1]
    ok = torch.ones(T, dtype=torch.bool)
    ok[123] = False
    assert (d.perm_inv.cpu()[ok] >= 0).all()
