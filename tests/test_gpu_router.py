"""Stage 1 router on the B200 vs the order-matched C restatement (bit-exact
indices, fp32 gates) and vs the reference gate (indices outside the fp64
near-tie band)."""
import numpy as np
import pytest
import torch

from helpers import bf16_bits
from oracle import moe_ref as mr
from oracle.build import router_order

pytestmark = pytest.mark.gpu


def _run(x_cpu, wg, bg, renorm, dev):
    from cti_b200 import _lib, ops

    r = ops.router(x_cpu.to(dev), wg.to(dev), bg.to(dev), renorm=renorm)
    _lib.raise_on_status(dev)
    return r


@pytest.mark.parametrize("T,D,E", [(1, 128, 8), (255, 128, 8), (256, 128, 8), (257, 256, 16),
                                   (4096, 128, 8), (69632, 256, 16), (3000, 1024, 64),
                                   (500, 64, 2), (700, 96, 128), (513, 40, 33),
                                   (300, 2048, 16)])
@pytest.mark.parametrize("renorm", [True, False])
def test_router_bit_exact_vs_order_matched_oracle(cuda_device, T, D, E, renorm):
    g = torch.Generator().manual_seed(T + D + E)
    x = torch.randn(T, D, generator=g).bfloat16()
    wg = torch.randn(E, D, generator=g) * 0.02
    bg = torch.randn(E, generator=g) * 0.5
    r = _run(x, wg, bg, renorm, cuda_device)
    idx, gate, _ = router_order(bf16_bits(x), wg.numpy(), bg.numpy(), renorm)
    np.testing.assert_array_equal(r.idx2.cpu().numpy(), idx)
    # Gates: CUDA expf vs the host libm expf differ by a few ulps.
    np.testing.assert_allclose(r.gate2.cpu().numpy(), gate, rtol=2e-6, atol=1e-7)
    assert (r.idx2[:, 0] != r.idx2[:, 1]).all()


def test_router_matches_reference_gate_outside_near_ties(cuda_device):
    g = torch.Generator().manual_seed(11)
    T, D, E = 20000, 256, 16
    x = torch.randn(T, D, generator=g).bfloat16()
    wg = torch.randn(E, D, generator=g) * 0.02
    bg = torch.randn(E, generator=g) * 0.02
    r = _run(x, wg, bg, True, cuda_device)
    ref = mr.gate_ref(x.float(), wg, bg, renorm=True, tie_lower_id=True)
    tie = mr.near_tie_mask(x.float(), wg, bg).numpy()
    ok = ~tie
    np.testing.assert_array_equal(r.idx2.cpu().numpy()[ok], ref.idx.numpy()[ok])
    np.testing.assert_allclose(r.gate2.cpu().numpy()[ok], ref.score.numpy()[ok], rtol=1e-5,
                               atol=1e-6)
    print(f"near-tie band tokens: {int(tie.sum())} of {T}")


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_router_cfg2_matches_reference_gate_with_bounded_band(cuda_device, seed):
    """Configuration 2 (T = 72,214, D 256, E 16, Zipf(1.2) router bias) on
    every token against the reference gate (torch fp32 linear, softmax,
    stable top-2).  The fp64 near-tie band is bounded rather than only
    reported: at most 16 tokens (2.2e-4 of T) within a 1e-5 logit gap and at
    most 4 within 1e-6, and an index may differ from the reference only
    inside the 1e-6 band.  Measured with the order-matched C restatement
    (bit-exact to this kernel): 4 / 2 / 4 tokens in the 1e-5 band and
    0 / 0 / 1 in the 1e-6 band for seeds 0 / 1 / 2, and no index differs."""
    from cti_b200 import synth

    cfg = synth.CFG2
    T, _ = synth.moe_tokens(cfg)
    w = synth.moe_weights(cfg.d_model, cfg.num_experts, cfg.dim_ff, cfg.zipf_bias)
    x = synth.moe_activations(T, cfg.d_model, seed=seed)
    r = _run(x, w.wg, w.bg, True, cuda_device)
    ref = mr.gate_ref(x.float(), w.wg, w.bg, renorm=True, tie_lower_id=True)
    band5 = mr.near_tie_mask(x.float(), w.wg, w.bg, band=1e-5).numpy()
    band6 = mr.near_tie_mask(x.float(), w.wg, w.bg, band=1e-6).numpy()
    differs = (r.idx2.cpu().numpy() != ref.idx.numpy()).any(axis=1)
    print(f"seed {seed}: band 1e-5 {int(band5.sum())}, band 1e-6 {int(band6.sum())}, "
          f"differing {int(differs.sum())} of {T}")
    assert band5.sum() <= 16 and band6.sum() <= 4
    assert not (differs & ~band6).any()
    ok = ~band6
    np.testing.assert_allclose(r.gate2.cpu().numpy()[ok], ref.score.numpy()[ok], rtol=1e-5,
                               atol=1e-6)


def test_router_exact_ties_go_to_lower_expert_id(cuda_device):
    T, D, E = 300, 64, 16
    x = torch.randn(T, D).bfloat16()
    wg = torch.zeros(E, D)
    bg = torch.zeros(E)
    bg[[3, 7, 9, 12]] = 1.0
    r = _run(x, wg, bg, True, cuda_device)
    assert (r.idx2[:, 0] == 3).all() and (r.idx2[:, 1] == 7).all()
    torch.testing.assert_close(r.gate2.cpu(), torch.full((T, 2), 0.5))
    bg.zero_()
    r = _run(x, wg, bg, False, cuda_device)
    assert (r.idx2[:, 0] == 0).all() and (r.idx2[:, 1] == 1).all()
    torch.testing.assert_close(r.gate2.cpu(), torch.full((T, 2), 1.0 / E))


def test_router_block_metadata(cuda_device):
    from cti_b200 import _lib

    """block_hist counts every route of each 256-token block; route_rank is the
    route's position among the block's routes to the same expert."""
    g = torch.Generator().manual_seed(5)
    T, D, E = 1000, 128, 8
    x = torch.randn(T, D, generator=g).bfloat16()
    wg = torch.randn(E, D, generator=g) * 0.05
    bg = torch.zeros(E)
    r = _run(x, wg, bg, True, cuda_device)
    idx = r.idx2.cpu().long()
    rank = r.route_rank.cpu().long()
    hist = r.block_hist.cpu().long()
    B = _lib.ROUTER_BLOCK_TOKENS
    for b in range((T + B - 1) // B):
        blk = idx[b * B:(b + 1) * B].reshape(-1)
        assert torch.equal(hist[b], torch.bincount(blk, minlength=E))
        exp = torch.zeros_like(blk)
        seen = [0] * E
        for i, e in enumerate(blk.tolist()):
            exp[i] = seen[e]
            seen[e] += 1
        assert torch.equal(rank[b * B:(b + 1) * B].reshape(-1), exp)
