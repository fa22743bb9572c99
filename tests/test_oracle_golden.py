"""The CPU oracle against fixtures made by running the reference's own code
(tests/golden/make_golden.py).  No GPU."""
import numpy as np
import pytest
import torch

import golden_inputs as gi
from helpers import bf16_bits, load_golden
from oracle import embbag_ref as er
from oracle import moe_ref as mr
from oracle.build import router_order


@pytest.mark.parametrize("name", list(gi.MOE_CASES))
def test_moe_oracle_matches_reference_fixture(name):
    torch.set_num_threads(1)
    inp = gi.moe_inputs(name)
    gold = load_golden(name)
    digest = gi.tensor_digest(inp["x"], inp["wg"], inp["bg"], inp["w1"], inp["b1"], inp["w2"],
                              inp["b2"])
    assert digest == str(gold["input_sha256"]), "regenerated inputs differ from the fixture's"
    out, g = mr.smoe_ref(inp["x"], inp["wg"], inp["bg"], inp["w1"], inp["b1"], inp["w2"],
                         inp["b2"], act=inp["act"], renorm=inp["renorm"],
                         tie_lower_id=inp["renorm"])
    np.testing.assert_array_equal(g.idx.numpy(), gold["idx"])
    np.testing.assert_allclose(g.score.numpy(), gold["score"], rtol=1e-6, atol=0)
    np.testing.assert_allclose(out.numpy(), gold["out"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("per_feature", [False, True])
def test_embbag_oracle_matches_reference_fixture_bit_exact(per_feature):
    inp = gi.bag_inputs(per_feature)
    name = "embbag_per_feature" if per_feature else "embbag_shared_table"
    gold = load_golden(name)
    digest = gi.tensor_digest(inp["values"], inp["row_offsets"], inp["val_offsets"], inp["vocab"],
                              inp["table_row_base"], inp["table"])
    assert digest == str(gold["input_sha256"])
    out = er.embbag_ref(inp["values"], inp["row_offsets"], inp["val_offsets"], inp["table"],
                        inp["table_row_base"], inp["vocab"], inp["features"])
    np.testing.assert_array_equal(out.numpy(), gold["pooled"])


def test_embbag_oracle_sums_sequentially():
    """segment_reduce on CPU sums each bag in order: bitwise equal to a loop."""
    inp = gi.bag_inputs(True, seed=5)
    a = er.embbag_ref(inp["values"], inp["row_offsets"], inp["val_offsets"], inp["table"],
                      inp["table_row_base"], inp["vocab"], inp["features"])
    b = er.embbag_loop(inp["values"], inp["row_offsets"], inp["val_offsets"], inp["table"],
                       inp["table_row_base"], inp["vocab"], inp["features"])
    assert torch.equal(a, b)


@pytest.mark.parametrize("name", list(gi.MOE_CASES))
def test_order_matched_router_agrees_with_reference_gate(name):
    """The C router (kernel summation order) picks the reference's experts
    except inside the fp64 near-tie band, and its gates match to fp32 ulps."""
    inp = gi.moe_inputs(name)
    idx, gate, _ = router_order(bf16_bits(inp["x"]), inp["wg"].numpy(), inp["bg"].numpy(),
                                inp["renorm"])
    g = mr.gate_ref(inp["x"], inp["wg"], inp["bg"], renorm=inp["renorm"], tie_lower_id=True)
    tie = mr.near_tie_mask(inp["x"], inp["wg"], inp["bg"]).numpy()
    ok = ~tie
    np.testing.assert_array_equal(idx[ok], g.idx.numpy()[ok])
    np.testing.assert_allclose(gate[ok], g.score.numpy()[ok], rtol=2e-6, atol=1e-7)


def test_order_matched_router_ties_go_to_lower_id():
    x = torch.zeros(4, 64).bfloat16().float()
    wg = torch.zeros(8, 64)
    bg = torch.tensor([0.1, 0.3, 0.3, 0.3, 0.0, 0.3, 0.0, 0.0])
    idx, gate, _ = router_order(bf16_bits(x), wg.numpy(), bg.numpy(), True)
    assert (idx == np.array([1, 2])).all()
    np.testing.assert_allclose(gate, 0.5)
    g = mr.gate_ref(x, wg, bg, renorm=True, tie_lower_id=True)
    assert (g.idx.numpy() == np.array([1, 2])).all()


def test_expected_dispatch_is_reference_nonzero_order():
    """expert_segments reproduces `(idx == e).nonzero()` of baseline/infer.py:340."""
    g = torch.Generator().manual_seed(3)
    T, E = 300, 8
    idx = torch.stack([torch.randperm(E, generator=g)[:2] for _ in range(T)])
    offs, sorted_token, perm_inv = mr.expert_segments(idx, E)
    for e in range(E):
        tok, _ = (idx == e).nonzero(as_tuple=True)
        assert torch.equal(sorted_token[offs[e]:offs[e + 1]], tok)
    flat_pos = perm_inv.reshape(-1)
    assert torch.equal(torch.sort(flat_pos).values, torch.arange(2 * T))
