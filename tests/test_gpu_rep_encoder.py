"""The fused RepEncoder (cti_rep_encoder_fused: pooling, LayerNorm folded
into the Linear, one launch) against the fp32 restatement of
baseline/infer.py:253-265 (oracle.e2e_ref.rep_encoder_ref) and against this
library's unfused path (pooling kernel, LayerNorm kernel, cuBLAS Linear).

Tolerances: max abs error / max |reference| below 2e-2 against the fp32
oracle (bf16 pooled rows, bf16 folded weights, bf16 output) and below 1e-2
against the unfused path (same bf16 pooled rows; the two round the
normalised row or the folded weight respectively)."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _encoder(dev, bb, d_model, seed):
    import cti_b200
    from cti_b200 import synth

    g = torch.Generator().manual_seed(seed)
    enc = cti_b200.RepEncoder(0, 64, 0, bb.features, d_model, vocab_sizes=bb.vocab.tolist())
    with torch.no_grad():
        enc.emb.weight = torch.nn.Parameter(synth.embedding_table(bb.total_rows, 64, seed=seed),
                                            requires_grad=False)
        K = bb.features * 64
        enc.input_norm.weight.copy_(1.0 + 0.2 * torch.randn(K, generator=g))
        enc.input_norm.bias.copy_(0.1 * torch.randn(K, generator=g))
        enc.linear.weight.copy_(0.02 * torch.randn(d_model, K, generator=g))
        enc.linear.bias.copy_(0.02 * torch.randn(d_model, generator=g))
    enc.input_norm.to(torch.bfloat16)
    enc.linear.to(torch.bfloat16)
    return enc.to(dev)


def _batch(bb):
    return {"_flat_values": bb.values, "_flat_row_offsets": bb.row_offsets,
            "_val_offsets": bb.val_offsets}


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return (a - b).abs().max().item() / max(b.abs().max().item(), 1e-30)


@pytest.mark.parametrize("B,d_model", [(1, 256), (129, 256), (3000, 256), (700, 128)])
def test_fused_rep_encoder_matches_oracle(cuda_device, B, d_model):
    from cti_b200 import _lib, synth
    from oracle.e2e_ref import rep_encoder_ref

    bb = synth.bag_batch(batch=B, seed=B, vocab_hi=2e5, lam_hi=50.0)
    enc = _encoder(cuda_device, bb, d_model, seed=B)
    assert enc.fused_supported()
    out = enc.forward_fused(_batch(bb))
    _lib.raise_on_status(cuda_device)
    assert out.shape == (B, d_model) and out.dtype == torch.bfloat16
    sd = {"rep_encoder." + k: v.detach().cpu() for k, v in enc.state_dict().items()}
    ref = rep_encoder_ref(sd, _batch(bb), slot_num=bb.features,
                          table_row_base=bb.table_row_base, vocab=bb.vocab)
    assert _rel(out, ref) < 2e-2


def test_fused_rep_encoder_matches_unfused_path(cuda_device):
    from cti_b200 import _lib, synth

    bb = synth.bag_batch(batch=2000, seed=7, vocab_hi=2e5, lam_hi=50.0)
    enc = _encoder(cuda_device, bb, 256, seed=7)
    batch = {k: v.to(cuda_device) for k, v in _batch(bb).items()}
    fused = enc.forward_fused(batch)
    unfused = enc(batch)
    _lib.raise_on_status(cuda_device)
    assert _rel(fused, unfused) < 1e-2


def test_fused_rep_encoder_bad_offsets_raise_status(cuda_device):
    from cti_b200 import _lib, ops, synth

    bb = synth.bag_batch(batch=300, seed=3, vocab_hi=2e5, lam_hi=20.0)
    enc = _encoder(cuda_device, bb, 256, seed=3)
    ro = bb.row_offsets.clone()
    ro[5] = ro[6] + 1  # feature 0, sample 5: start > end
    wg, r1, c = enc.fused_params()
    _lib.read_status(cuda_device, clear=True)
    ops.rep_encoder_fused(bb.values.to(cuda_device), ro.to(cuda_device),
                          bb.val_offsets.to(cuda_device), enc.emb.weight.detach(),
                          enc.table_row_base, enc.vocab, bb.features, wg, r1, c)
    code, _ = _lib.read_status(cuda_device, clear=True)
    assert code == _lib.CTI_ERR_BOUNDS


def test_fused_rep_encoder_rejects_unsupported(cuda_device):
    from cti_b200 import _lib

    lib = _lib.lib
    # dim 32 and N 192 are outside the kernel; B = 0 is a no-op.
    assert lib.cti_rep_encoder_fused(None, 0, None, None, None, None, None, 0, 4, 28, 32, None,
                                     None, None, 256, ctypes.c_float(1e-5), None, None,
                                     None) == _lib.CTI_ERR_UNSUPPORTED
    assert lib.cti_rep_encoder_fused(None, 0, None, None, None, None, None, 0, 4, 28, 64, None,
                                     None, None, 192, ctypes.c_float(1e-5), None, None,
                                     None) == _lib.CTI_ERR_UNSUPPORTED
    assert lib.cti_rep_encoder_fused(None, 0, None, None, None, None, None, 0, 0, 28, 64, None,
                                     None, None, 256, ctypes.c_float(1e-5), None, None,
                                     None) == 0
