"""Stage 3 fused expert FFN (fc1 -> GELU -> fc2 with the hidden tile kept in
tensor memory) on the B200 vs a torch fp32 reference of the same op.
Tolerance: max rel err 1e-2 (bf16 hidden activations and bf16 output vs
fp32 throughout)."""
import pytest
import torch
import torch.nn.functional as F

from helpers import max_rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-2


def ref_ffn(x, w1, b1, w2, b2, offs, act, Gw):
    out = torch.zeros(x.shape[0], w2.shape[1])
    o = offs.tolist()
    for g in range(len(o) - 1):
        lo, hi = o[g], o[g + 1]
        if hi <= lo:
            continue
        e = g % Gw
        h = x[lo:hi].float() @ w1[e].float().T + b1[e]
        h = F.gelu(h) if act == "gelu" else F.relu(h) if act == "relu" else h
        out[lo:hi] = h @ w2[e].float().T + b2[e]
    return out


CASES = [
    # D, F, group sizes, Gw, act
    (256, 128, [128], 1, "gelu"),
    (256, 1024, [128], 1, "gelu"),
    (128, 512, [1, 0, 200, 55], 4, "gelu"),
    (256, 1024, [300, 0, 1000, 17, 128, 129, 5000, 2, 900, 0, 0, 33, 64, 65, 700, 1], 16, "gelu"),
    (256, 512, [640, 640, 384], 3, "relu"),
    (128, 256, [3000, 2000, 1000], 3, "none"),
    (256, 1024, [40000, 30000, 20000, 10000], 4, "gelu"),
]


@pytest.mark.parametrize("D,Fd,sizes,Gw,act", CASES)
def test_fused_ffn_matches_fp32(cuda_device, D, Fd, sizes, Gw, act):
    from cti_b200 import _lib, ops

    rows = sum(sizes)
    g = torch.Generator().manual_seed(rows + D + Fd)
    x = torch.randn(rows, D, generator=g).bfloat16()
    w1 = (torch.randn(Gw, Fd, D, generator=g) * 0.05).bfloat16()
    b1 = torch.randn(Gw, Fd, generator=g) * 0.1
    w2 = (torch.randn(Gw, D, Fd, generator=g) * 0.05).bfloat16()
    b2 = torch.randn(Gw, D, generator=g) * 0.1
    offs = torch.zeros(len(sizes) + 1, dtype=torch.int32)
    offs[1:] = torch.cumsum(torch.tensor(sizes), 0)
    dev = cuda_device
    y = ops.expert_ffn_fused(x.to(dev), w1.to(dev), b1.to(dev), w2.to(dev), b2.to(dev),
                             offs.to(dev), act=act)
    _lib.raise_on_status(dev)
    ref = ref_ffn(x, w1, b1, w2, b2, offs, act, Gw)
    err = max_rel_err(y, ref)
    assert err < TOL, f"max rel err {err}"


def test_fused_ffn_agrees_with_two_gemms(cuda_device):
    """The fused path and the two-GEMM path round the hidden activation to
    bf16 at the same point, so they agree to accumulation-order noise."""
    from cti_b200 import _lib, ops

    dev = cuda_device
    rows, D, Fd, E = 6000, 256, 1024, 16
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(rows, D, generator=g, device=dev).bfloat16()
    w1 = (torch.randn(E, Fd, D, generator=g, device=dev) * 0.05).bfloat16()
    b1 = torch.randn(E, Fd, generator=g, device=dev) * 0.1
    w2 = (torch.randn(E, D, Fd, generator=g, device=dev) * 0.05).bfloat16()
    b2 = torch.randn(E, D, generator=g, device=dev) * 0.1
    offs = torch.linspace(0, rows, E + 1, device=dev).round().int()
    y1 = ops.expert_ffn_fused(x, w1, b1, w2, b2, offs, act="gelu")
    h = ops.grouped_gemm(x, w1, b1, offs, act="gelu")
    y2 = ops.grouped_gemm(h, w2, b2, offs, act="none")
    _lib.raise_on_status(dev)
    assert max_rel_err(y1, y2) < 4e-3


def test_gelu_epilogue_accuracy(cuda_device):
    """GELU of the epilogue vs the exact erf GELU (fp64): a GEMM with an
    identity weight block returns gelu(x) rounded to bf16.  On [-4.5, 4.5]
    (the range of the polynomial fit) that must be within one bf16 ulp of
    the exact value (relative 2^-7); everywhere the absolute error must stay
    below 2e-6 (the fit's 7.2e-7 plus bf16 rounding of values under 1.3e-4),
    i.e. under one bf16 ulp of any output of magnitude 1.3e-4 or more."""
    from cti_b200 import _lib, ops

    dev = cuda_device
    xs = torch.linspace(-12.0, 12.0, 128 * 64 * 8).reshape(-1, 64)
    a = xs.bfloat16()
    w = torch.zeros(1, 128, 64)
    w[0, :64, :64] = torch.eye(64)
    w[0, 64:, :64] = torch.eye(64)
    offs = torch.tensor([0, a.shape[0]], dtype=torch.int32)
    out = ops.grouped_gemm(a.to(dev), w.bfloat16().to(dev), None, offs.to(dev), act="gelu")
    _lib.raise_on_status(dev)
    xa = a.double()
    exact = xa * 0.5 * torch.special.erfc(-xa / 2 ** 0.5)
    got = out[:, :64].double().cpu()
    err = (got - exact).abs()
    inner = xa.abs() <= 4.5
    assert (err[inner] <= exact[inner].abs() * 2.0 ** -7 + 1e-30).all(), err[inner].max()
    assert (err <= 2e-6 + exact.abs() * 2.0 ** -7).all(), err.max()
    assert torch.equal(out[:, :64].cpu(), out[:, 64:].cpu())


@pytest.mark.parametrize("D,Fd,T,E,act", [
    (256, 1024, 72214, 16, "gelu"),   # the cfg2 layer's shape
    (128, 512, 3001, 8, "gelu"),
    (256, 512, 5, 4, "relu"),         # partial tiles only
    (128, 256, 900, 3, "none"),
])
def test_fused_ffn_row_gather_equals_dispatched_rows(cuda_device, D, Fd, T, E, act):
    """cti_moe_expert_ffn_fused_gather (rows x[sorted_token[r]] copied by the
    kernel's gather warp into the swizzled tile) against the TMA path on the
    dispatched copy of the same rows: bit for bit."""
    from cti_b200 import _lib, ops

    g = torch.Generator().manual_seed(T)
    x = (torch.randn(T, D, generator=g)).bfloat16().to(cuda_device)
    wg = (torch.randn(E, D, generator=g) * 0.05).to(cuda_device)
    bg = torch.zeros(E).to(cuda_device)
    w1 = (torch.randn(E, Fd, D, generator=g) * 0.02).bfloat16().to(cuda_device)
    b1 = (torch.randn(E, Fd, generator=g) * 0.02).to(cuda_device)
    w2 = (torch.randn(E, D, Fd, generator=g) * 0.02).bfloat16().to(cuda_device)
    b2 = (torch.randn(E, D, generator=g) * 0.02).to(cuda_device)
    r = ops.router(x, wg, bg)
    d = ops.dispatch(x, r, E)
    y_tma = ops.expert_ffn_fused(d.xperm, w1, b1, w2, b2, d.offsets, act=act)
    y_gather = ops.expert_ffn_fused_gather(x, d.sorted_token, w1, b1, w2, b2, d.offsets, act=act)
    _lib.raise_on_status(cuda_device)
    assert torch.equal(y_gather, y_tma), (y_gather.float() - y_tma.float()).abs().max().item()


def test_layer_matches_staged_fused_and_support_query(cuda_device):
    """SMoE.forward (cti_moe_layer_forward) equals the staged path (dispatched
    copy, TMA fused FFN, combine) bit for bit at the cfg2 shape, and the
    fused-shape query answers for the layer's shapes."""
    from cti_b200 import _lib, synth
    from cti_b200._lib import lib
    import cti_b200

    assert lib.cti_moe_expert_ffn_fused_supported(256, 1024, 16, 144428) == 1
    assert lib.cti_moe_expert_ffn_fused_supported(1024, 4096, 64, 1000) == 0
    assert lib.cti_moe_expert_ffn_fused_supported(256, 1000, 16, 1000) == 0
    cfg = synth.CFG2
    T, _ = synth.moe_tokens(cfg, seed=0)
    w = synth.moe_weights(cfg.d_model, cfg.num_experts, cfg.dim_ff, cfg.zipf_bias, seed=7)
    m = cti_b200.SMoE(cfg.d_model, cfg.dim_ff, cfg.num_experts)
    synth.load_moe_module(m, w)
    m.to(cuda_device).prepare_for_inference()
    x = synth.moe_activations(T, cfg.d_model, seed=7).to(cuda_device)
    out = m(x.unsqueeze(0))[0][0]
    staged = m.forward_staged(x, fused=True)["out"]
    _lib.raise_on_status(cuda_device)
    assert torch.equal(out, staged)


# The CTA-pair kernel (d_model 256): 256-row tiles whose odd CTA may hold no
# rows (groups of <= 128 rows), single rows, empty groups, 120 groups.
PAIR_CASES = [
    (1024, [256], 1, "gelu"),
    (256, [1], 1, "gelu"),
    (1024, [300, 0, 1000, 17, 128, 129, 5000, 2, 900, 0, 0, 33, 64, 65, 700, 1], 16, "gelu"),
    (512, [640, 640, 384, 100, 129], 5, "relu"),
    (1024, [40000, 30000, 20000, 10000], 4, "gelu"),
    (256, [3, 250, 0, 257, 511, 1] * 20, 7, "none"),
]


@pytest.mark.parametrize("Fd,sizes,Gw,act", PAIR_CASES)
def test_fused_ffn_pair_matches_fp32_and_single_cta(cuda_device, Fd, sizes, Gw, act):
    """cti_moe_expert_ffn_fused_pair against the fp32 reference (max rel err
    1e-2) and against the one-CTA kernel on the same rows: every row is
    computed with the same K order and the same bf16 rounding of the hidden
    activation, so the two agree to fp32 accumulation noise (2e-3)."""
    from cti_b200 import _lib, ops

    D = 256
    rows = sum(sizes)
    g = torch.Generator().manual_seed(rows + Fd + len(sizes))
    x = torch.randn(rows, D, generator=g).bfloat16()
    w1 = (torch.randn(Gw, Fd, D, generator=g) * 0.05).bfloat16()
    b1 = torch.randn(Gw, Fd, generator=g) * 0.1
    w2 = (torch.randn(Gw, D, Fd, generator=g) * 0.05).bfloat16()
    b2 = torch.randn(Gw, D, generator=g) * 0.1
    offs = torch.zeros(len(sizes) + 1, dtype=torch.int32)
    offs[1:] = torch.cumsum(torch.tensor(sizes), 0)
    dev = cuda_device
    args = (x.to(dev), w1.to(dev), b1.to(dev), w2.to(dev), b2.to(dev), offs.to(dev))
    y_pair = ops.expert_ffn_fused(*args, act=act, pair=True)
    y_one = ops.expert_ffn_fused(*args, act=act)
    _lib.raise_on_status(dev)
    assert max_rel_err(y_pair, y_one.float()) < 2e-3
    ref = ref_ffn(x, w1, b1, w2, b2, offs, act, Gw)
    err = max_rel_err(y_pair, ref)
    assert err < TOL, f"max rel err {err}"


def test_fused_ffn_pair_leaves_rows_outside_groups_untouched(cuda_device):
    """Rows past the last group offset are neither read into results nor
    written; rows of a pair tile that belong to no group stay as they were."""
    from cti_b200 import _lib, ops

    dev = cuda_device
    rows, D, Fd = 700, 256, 512
    g = torch.Generator(device=dev).manual_seed(3)
    x = torch.randn(rows, D, generator=g, device=dev).bfloat16()
    w1 = (torch.randn(1, Fd, D, generator=g, device=dev) * 0.05).bfloat16()
    b1 = torch.zeros(1, Fd, device=dev)
    w2 = (torch.randn(1, D, Fd, generator=g, device=dev) * 0.05).bfloat16()
    b2 = torch.zeros(1, D, device=dev)
    offs = torch.tensor([0, 300], dtype=torch.int32, device=dev)
    y = torch.full((rows, D), 7.0, device=dev).bfloat16()
    ops.expert_ffn_fused(x, w1, b1, w2, b2, offs, out=y, pair=True)
    _lib.raise_on_status(dev)
    assert (y[300:] == 7.0).all()
    ref = ref_ffn(x[:300].cpu(), w1.cpu(), b1.cpu(), w2.cpu(), b2.cpu(),
                  torch.tensor([0, 300]), "gelu", 1)
    assert max_rel_err(y[:300], ref) < TOL
