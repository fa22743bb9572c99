"""The CPU oracle of the configuration-4 model (oracle/e2e_ref.py) against the
golden fixture made by running the reference's own CTRModel
(tests/golden/make_golden.py).  No GPU."""
import numpy as np
import pytest
import torch

import golden_inputs as gi
from helpers import load_golden, max_rel_err
from oracle import e2e_ref


@pytest.mark.parametrize("name", list(gi.E2E_CASES))
def test_e2e_oracle_matches_reference_model(name):
    N, Lmax, D, H, L, Fd, E, V, wstd = gi.E2E_CASES[name]
    batch, sd = gi.e2e_inputs(name)
    gold = load_golden(name)
    assert str(gold["input_sha256"]) == gi.e2e_digest(batch, sd)
    torch.set_num_threads(1)
    hidden, logits, probs = e2e_ref.ctr_forward_ref(sd, batch, slot_num=gi.E2E_SLOTS, n_heads=H,
                                                    num_layers=L, num_experts=E)
    # The same fp32 arithmetic in a different association order (per
    # sequence attention instead of one masked [T, T] product).
    assert max_rel_err(hidden, torch.from_numpy(gold["hidden"])) < 1e-5
    np.testing.assert_allclose(probs.numpy(), gold["probs"], rtol=0, atol=1e-6)
    if wstd is None:  # the large-weight case is not degenerate
        assert gold["probs"].std() > 0.05 and np.abs(gold["logits"]).max() > 3


def test_e2e_fixture_covers_edge_inputs():
    batch, _ = gi.e2e_inputs("e2e_d128_l2")
    v = batch["_flat_values"]
    V = gi.E2E_CASES["e2e_d128_l2"][7]
    assert (v < 0).any() and (v >= V).any()  # ids the reference clamps
    T = int(batch["user_offsets"][-1])
    offs = batch["_flat_row_offsets"].view(gi.E2E_SLOTS, T + 1)
    assert ((offs[:, 1:] - offs[:, :-1]) == 0).any()  # empty bags
