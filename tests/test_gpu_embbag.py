"""Stage 5 embedding-bag pooling on the B200: bit-exact vs the reference's
pooling (golden fixtures and the CPU oracle, fp32 sequential sums)."""
import numpy as np
import pytest
import torch

import golden_inputs as gi
from helpers import load_golden
from oracle import embbag_ref as er

pytestmark = pytest.mark.gpu


def run_kernel(inp, dev, out_dtype=torch.float32):
    from cti_b200 import _lib, ops

    out = ops.embedding_bag_sum(
        inp["values"].to(dev), inp["row_offsets"].to(dev), inp["val_offsets"].to(dev),
        inp["table"].to(dev), inp["table_row_base"].to(dev), inp["vocab"].to(dev),
        inp["features"], out_dtype=out_dtype)
    _lib.raise_on_status(dev)
    return out


@pytest.mark.parametrize("per_feature", [False, True])
def test_embbag_bit_exact_vs_reference_fixture(cuda_device, per_feature):
    inp = gi.bag_inputs(per_feature)
    gold = load_golden("embbag_per_feature" if per_feature else "embbag_shared_table")
    out = run_kernel(inp, cuda_device)
    np.testing.assert_array_equal(out.cpu().numpy(), gold["pooled"])


def _synth_inputs(batch, seed, lam_hi=50.0, vocab_hi=2e5):
    from cti_b200 import synth

    bb = synth.bag_batch(batch=batch, seed=seed, vocab_hi=vocab_hi, lam_hi=lam_hi)
    table = synth.embedding_table(bb.total_rows, 64, seed=seed)
    return dict(values=bb.values, row_offsets=bb.row_offsets, val_offsets=bb.val_offsets,
                table=table, table_row_base=bb.table_row_base, vocab=bb.vocab,
                features=bb.features, batch=bb.batch)


@pytest.mark.parametrize("batch,seed", [(1, 0), (37, 1), (512, 2)])
def test_embbag_bit_exact_vs_oracle(cuda_device, batch, seed):
    inp = _synth_inputs(batch, seed)
    out = run_kernel(inp, cuda_device)
    ref = er.embbag_ref(inp["values"], inp["row_offsets"], inp["val_offsets"], inp["table"],
                        inp["table_row_base"], inp["vocab"], inp["features"])
    assert torch.equal(out.cpu(), ref)


def test_embbag_bf16_output_is_rounded_fp32_sum(cuda_device):
    inp = _synth_inputs(64, 4)
    out32 = run_kernel(inp, cuda_device)
    out16 = run_kernel(inp, cuda_device, torch.bfloat16)
    assert torch.equal(out16, out32.bfloat16())


def test_embbag_all_empty_bags_and_clamping(cuda_device):
    inp = gi.bag_inputs(False, seed=3)
    inp = dict(inp)
    F, B = inp["features"], inp["batch"]
    inp["row_offsets"] = torch.zeros(F * (B + 1), dtype=torch.long)
    out = run_kernel(inp, cuda_device)
    assert (out == 0).all()
    # Every id far out of range clamps to the first / last row.
    inp = gi.bag_inputs(False, seed=4)
    inp["values"] = torch.where(torch.arange(inp["values"].numel()) % 2 == 0,
                                torch.full_like(inp["values"], -10**12),
                                torch.full_like(inp["values"], 10**12))
    out = run_kernel(inp, cuda_device)
    ref = er.embbag_ref(inp["values"], inp["row_offsets"], inp["val_offsets"], inp["table"],
                        inp["table_row_base"], inp["vocab"], inp["features"])
    assert torch.equal(out.cpu(), ref)


def test_embbag_reports_offsets_past_values(cuda_device):
    from cti_b200 import _lib, ops

    inp = gi.bag_inputs(False, seed=6)
    dev = cuda_device
    vals = inp["values"][:5].to(dev)  # far fewer values than the offsets claim
    ops.embedding_bag_sum(vals, inp["row_offsets"].to(dev), inp["val_offsets"].to(dev),
                          inp["table"].to(dev), inp["table_row_base"].to(dev),
                          inp["vocab"].to(dev), inp["features"])
    code, _ = _lib.read_status(dev)
    assert code == _lib.CTI_ERR_BOUNDS


@pytest.mark.slow
def test_embbag_full_cfg3_sampled_bags(cuda_device):
    """Full configuration-3 batch (4096 x 28 bags, ~2.9M ids, vocabularies up
    to 2e6): every bag is checked against a CPU sum of the same rows for a
    seeded sample of 2000 bags, plus a global checksum (sum of all pooled
    values, fp64) against the oracle over the whole batch."""
    from cti_b200 import synth

    bb = synth.bag_batch(batch=4096, seed=0)
    dev = cuda_device
    table = synth.embedding_table(bb.total_rows, 64, seed=0, device=dev)
    inp = dict(values=bb.values, row_offsets=bb.row_offsets, val_offsets=bb.val_offsets,
               table=table, table_row_base=bb.table_row_base, vocab=bb.vocab,
               features=bb.features)
    out = run_kernel(inp, dev).cpu()
    rng = np.random.default_rng(0)
    B, F = bb.batch, bb.features
    for q in rng.choice(B * F, size=2000, replace=False):
        b, f = divmod(int(q), F)
        s = int(bb.row_offsets[f * (B + 1) + b])
        e = int(bb.row_offsets[f * (B + 1) + b + 1])
        v0 = int(bb.val_offsets[f])
        ids = bb.values[v0 + s:v0 + e].clamp(0, int(bb.vocab[f]) - 1) + int(bb.table_row_base[f])
        rows = table[ids.to(dev)].float().cpu()
        acc = torch.zeros(64)
        for i in range(rows.shape[0]):
            acc = acc + rows[i]
        assert torch.equal(out[b, f * 64:(f + 1) * 64], acc), (b, f)
