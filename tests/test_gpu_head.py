"""The fused CTR head (cti_ctr_head: Linear -> ReLU -> dot -> clamp ->
sigmoid in one launch) against torch in fp32 on the same bf16 inputs.
The products of bf16 values are exact in fp32 and the hidden activation
stays fp32 on chip, so the logits agree to fp32 summation-order noise
(1e-4 absolute at magnitudes of order 1) and the probabilities to 1e-5."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(h, w1, b1, w2, b2, limit=15.0):
    z = torch.relu(h.float() @ w1.float().T + b1)
    lg = torch.clamp(z @ w2 + b2, -limit, limit)
    return lg, torch.sigmoid(lg)


@pytest.mark.parametrize("T,D,Hd,scale", [(1, 256, 128, 1.0), (127, 256, 128, 1.0),
                                          (129, 128, 32, 1.0), (5000, 256, 128, 1.0),
                                          (300001, 256, 128, 1.0), (4000, 192, 96, 1.0),
                                          (3000, 256, 128, 40.0)])
def test_ctr_head_matches_fp32(cuda_device, T, D, Hd, scale):
    from cti_b200 import _lib, ops

    g = torch.Generator().manual_seed(T + D + Hd)
    h = torch.randn(T, D, generator=g).bfloat16()
    w1 = (torch.randn(Hd, D, generator=g) * 0.05).bfloat16()
    b1 = torch.randn(Hd, generator=g) * 0.1
    w2 = torch.randn(Hd, generator=g) * 0.1 * scale   # scale 40 drives logits past +-15
    b2 = torch.randn(1, generator=g) * 0.1
    dev = cuda_device
    lg, pr = ops.ctr_head(h.to(dev), w1.to(dev), b1.to(dev), w2.to(dev), b2.to(dev))
    _lib.raise_on_status(dev)
    rl, rp = _ref(h, w1, b1, w2, b2)
    torch.testing.assert_close(lg.cpu(), rl, rtol=0, atol=1e-4 * scale)
    torch.testing.assert_close(pr.cpu(), rp, rtol=0, atol=1e-5)
    if scale > 1:
        assert (lg.abs() == 15.0).any()  # the clamp is exercised
    lg2, pr2 = ops.ctr_head(h.to(dev), w1.to(dev), b1.to(dev), w2.to(dev), b2.to(dev),
                            want_logits=False)
    assert lg2 is None and torch.equal(pr2, pr)


def test_ctr_head_rejects_unsupported_shapes(cuda_device):
    from cti_b200 import _lib

    for D, Hd in ((100, 128), (512, 128), (256, 256), (256, 48)):
        rc = _lib.lib.cti_ctr_head(None, None, None, None, None, 10, D, Hd, 15.0, None, None,
                                   None, None)
        assert rc == _lib.CTI_ERR_UNSUPPORTED, (D, Hd)
    assert _lib.lib.cti_ctr_head(None, None, None, None, None, 10, 256, 128, 15.0, None, None,
                                 None, None) == _lib.CTI_ERR_INVALID_ARG
