"""Host-side logic: module API parity with the reference, synthetic inputs.  No GPU."""
from pathlib import Path

import numpy as np
import pytest
import torch

import cti_b200
from cti_b200 import synth

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_state_dict_keys_match_reference():
    ref_keys = (GOLDEN / "reference_state_dict_keys.txt").read_text().split()
    moe_keys = list(cti_b200.SMoE(128, 256, 4).state_dict().keys())
    enc_keys = list(cti_b200.RepEncoder(100, 8, 0, 28, 16).state_dict().keys())
    assert moe_keys + enc_keys == ref_keys


def test_reference_state_dict_loads_into_drop_in():
    import golden_inputs as gi

    inp = gi.moe_inputs("moe_config_d128_e8")
    sd = {"gate.w_g.weight": inp["wg"], "gate.w_g.bias": inp["bg"]}
    for e in range(8):
        sd[f"experts.{e}.fc1.weight"] = inp["w1"][e]
        sd[f"experts.{e}.fc1.bias"] = inp["b1"][e]
        sd[f"experts.{e}.fc2.weight"] = inp["w2"][e]
        sd[f"experts.{e}.fc2.bias"] = inp["b2"][e]
    m = cti_b200.SMoE(128, 256, 8)
    m.load_state_dict(sd)
    assert torch.equal(m.experts[3].fc2.weight, inp["w2"][3])


def test_forward_refuses_cpu_inputs():
    m = cti_b200.SMoE(128, 256, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.zeros(1, 4, 128, dtype=torch.bfloat16))


def test_only_top2_supported():
    with pytest.raises(ValueError):
        cti_b200.SMoE(128, 256, 8, k=3)


def test_cfg2_token_set_is_deterministic():
    T, cu = synth.moe_tokens(synth.CFG2)
    T2, cu2 = synth.moe_tokens(synth.CFG2)
    assert T == T2 and torch.equal(cu, cu2)
    assert cu.dtype == torch.int32 and cu.numel() == 513 and int(cu[-1]) == T
    assert 512 * 16 <= T <= 512 * 256
    lens = (cu[1:] - cu[:-1]).numpy()
    assert lens.min() >= 16 and lens.max() <= 256


def test_zipf_router_bias_profile():
    b = synth.zipf_router_bias(16, 1.2)
    p = torch.exp(b.double())
    assert abs(p.sum().item() - 1.0) < 1e-6
    ps = torch.sort(p, descending=True).values
    ratio = (ps[0] / ps).numpy()
    np.testing.assert_allclose(ratio, np.arange(1, 17) ** 1.2, rtol=1e-5)


def test_bag_batch_layout_matches_reference_contract():
    bb = synth.bag_batch(batch=64, seed=1)
    F, B = bb.features, bb.batch
    assert bb.row_offsets.numel() == F * (B + 1)
    offs = bb.row_offsets.view(F, B + 1)
    assert (offs[:, 0] == 0).all()
    assert (offs[:, 1:] >= offs[:, :-1]).all()
    lens = offs[:, -1]
    assert torch.equal(bb.val_offsets[1:], torch.cumsum(lens, 0)[:-1])
    assert int(lens.sum()) == bb.values.numel()
    for f in range(F):
        v = bb.values[bb.val_offsets[f]:bb.val_offsets[f] + lens[f]]
        assert v.min() >= 0 and v.max() < bb.vocab[f]
    assert (bb.vocab >= 1e4 - 1).all() and (bb.vocab <= 2e6 + 1).all()


def test_zipf_ids_are_skewed():
    rng = np.random.default_rng(0)
    ids = synth.zipf_ids(200000, 10000, 1.1, rng)
    _, counts = np.unique(ids, return_counts=True)
    counts = np.sort(counts)[::-1]
    assert counts[0] > 20 * np.median(counts)


@pytest.mark.parametrize("chunks", [1, 3, 7, 25])
def test_sequence_groups_rebuild_the_batch(chunks):
    """CTRModel.predict_host's plan (model.plan_sequence_groups): each group's
    own flat batch (ids of each feature laid out f by f, row offsets sliced
    and rebased, the planned val_offsets), pooled by the oracle, gives that
    group's rows of the whole batch's pooling, bit for bit; the groups cover
    every token once, in order, and cut only at sequence starts."""
    from cti_b200.model import plan_sequence_groups
    from oracle import embbag_ref as er

    F = 28
    g = torch.Generator().manual_seed(11)
    lens = torch.randint(16, 257, (20,), generator=g)
    lens[4] = 1
    uo = torch.zeros(21, dtype=torch.long)
    uo[1:] = torch.cumsum(lens, 0)
    T = int(uo[-1])
    bb = synth.bag_batch(batch=T, seed=5, vocab_lo=1e3, vocab_hi=2e4)
    table = synth.embedding_table(bb.total_rows, 64, seed=5).float()
    full = er.embbag_ref(bb.values, bb.row_offsets, bb.val_offsets, table, bb.table_row_base,
                         bb.vocab, F)
    plan = plan_sequence_groups(uo, bb.row_offsets, bb.val_offsets, F, chunks)
    assert 1 <= len(plan.groups) <= chunks
    assert plan.groups[0][2] == 0 and plan.groups[-1][3] == T
    starts = set(uo.tolist())
    parts = []
    for gi, (s0, s1, a, b) in enumerate(plan.groups):
        assert a in starts and b in starts and a < b
        if gi:
            assert plan.groups[gi - 1][3] == a and plan.groups[gi - 1][1] == s0
        n = b - a
        vals = torch.cat([bb.values[int(plan.lo[gi, f]):int(plan.hi[gi, f])] for f in range(F)])
        ro = torch.cat([bb.row_offsets[f * (T + 1) + a:f * (T + 1) + b + 1] for f in range(F)])
        ro = (ro.view(F, n + 1) - ro.view(F, n + 1)[:, :1]).reshape(-1)
        vo = torch.from_numpy(plan.val_offsets[gi])
        parts.append(er.embbag_ref(vals, ro, vo, table, bb.table_row_base, bb.vocab, F))
        cu = plan.cu[plan.cu_start[gi]:plan.cu_start[gi] + s1 - s0 + 1]
        assert cu[0] == 0 and cu[-1] == n
        np.testing.assert_array_equal(cu, uo[s0:s1 + 1].numpy() - a)
    assert torch.equal(torch.cat(parts), full)


def test_sequence_subbatch_pools_like_the_whole_batch():
    """synth.sequence_subbatch (the oracle's sample of a configuration-4
    batch): pooling the sub-batch gives, bit for bit, the rows of the
    sampled sequences' tokens in the pooling of the whole batch; zero-length
    bags and a 1-token sequence included."""
    from cti_b200 import synth
    from oracle.embbag_ref import embbag_ref

    lens = torch.tensor([5, 1, 9, 3, 7, 2])
    uo = torch.zeros(lens.numel() + 1, dtype=torch.int64)
    uo[1:] = torch.cumsum(lens, 0)
    T = int(uo[-1])
    bb = synth.bag_batch(batch=T, seed=3, vocab_lo=50, vocab_hi=400, lam_lo=0.5, lam_hi=4)
    table = synth.embedding_table(bb.total_rows, 8, seed=3)
    full = embbag_ref(bb.values, bb.row_offsets, bb.val_offsets, table, bb.table_row_base,
                      bb.vocab, bb.features)
    seqs = [1, 2, 5]
    sub = synth.sequence_subbatch(bb, uo, seqs)
    assert sub["user_offsets"].tolist() == [0, 1, 10, 12]
    pooled = embbag_ref(sub["_flat_values"], sub["_flat_row_offsets"], sub["_val_offsets"],
                        table, bb.table_row_base, bb.vocab, bb.features)
    rows = torch.cat([torch.arange(int(uo[s]), int(uo[s + 1])) for s in seqs])
    assert torch.equal(pooled, full[rows])


def test_host_pipeline_workspace_halves_match_the_c_requirement():
    """forward_host with two compute streams needs the workspace of one chunk
    rounded up to 256 bytes plus that of a second chunk (the C entry point's
    check, include/cti_b200.h); SMoE._get_workspace(halves=2) sizes it so."""
    from cti_b200._lib import lib

    m = cti_b200.SMoE(256, 1024, 16)
    for chunk in (1, 1000, 4096, 9027):
        need = int(lib.cti_moe_layer_workspace_bytes(chunk, 256, 16, 1024))
        m._workspace = None
        one = m._get_workspace(chunk, torch.device("cpu"))
        m._workspace = None
        two = m._get_workspace(chunk, torch.device("cpu"), halves=2)
        assert one.numel() == need
        assert two.numel() == -(-need // 256) * 256 + need
