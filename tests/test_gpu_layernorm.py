"""Residual add + LayerNorm kernel (cti_add_layernorm) against torch in
fp32: the bf16 sum bit-exact (x + r rounded once, as torch's bf16 add), the
normalised output within max rel err 1e-2 (one bf16 rounding of values of
order 1, after fp32 statistics)."""
import pytest
import torch
import torch.nn.functional as F

from helpers import max_rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,cols", [(1, 256), (7, 256), (4099, 256), (513, 1792), (64, 2048),
                                       (300, 512), (0, 256), (1000, 128), (77, 200), (33, 8),
                                       (129, 1800), (65, 264)])
@pytest.mark.parametrize("with_residual", [True, False])
def test_add_layernorm_matches_torch(cuda_device, rows, cols, with_residual):
    from cti_b200 import ops

    g = torch.Generator().manual_seed(rows * 7 + cols)
    x = (torch.randn(rows, cols, generator=g) * 3 + 1).bfloat16()
    r = torch.randn(rows, cols, generator=g).bfloat16() if with_residual else None
    w = (1 + 0.1 * torch.randn(cols, generator=g)).bfloat16()
    b = (0.1 * torch.randn(cols, generator=g)).bfloat16()
    dev = cuda_device
    s, out = ops.add_layernorm(x.to(dev), None if r is None else r.to(dev), w.to(dev), b.to(dev),
                               eps=1e-5)
    s_ref = x if r is None else (x.float() + r.float()).bfloat16()
    assert torch.equal(s.cpu(), s_ref)
    ref = F.layer_norm(s_ref.float(), (cols,), w.float(), b.float(), 1e-5)
    assert out.dtype == torch.bfloat16 and out.shape == (rows, cols)
    if rows:
        assert max_rel_err(out.float().cpu(), ref) < 1e-2


def test_add_layernorm_rejects_bad_shapes(cuda_device):
    from cti_b200 import _lib, ops

    # widths must be multiples of 8 (whole 16-byte vectors), at most 2048
    for cols in (100, 2056):
        x = torch.zeros(4, cols, dtype=torch.bfloat16, device=cuda_device)
        w = torch.ones(cols, dtype=torch.bfloat16, device=cuda_device)
        with pytest.raises(RuntimeError):
            ops.add_layernorm(x, None, w, w)
    assert _lib.lib.cti_add_layernorm(None, None, None, None, 4, 256, 1e-5, None, None,
                                      None) == _lib.CTI_ERR_INVALID_ARG
