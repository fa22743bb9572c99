"""The configuration-4 model on the B200 (bf16; sm_100a pooling and MoE
kernels, library attention) against the reference CTRModel fixture and the
CPU oracle.  Tolerances: CTR probabilities within 1e-3 absolute (the
north-star bound), encoder output within max rel err 2e-2 (bf16 vs fp32)."""
import numpy as np
import pytest
import torch

import golden_inputs as gi
from helpers import MOE_MAX_REL_ERR, load_golden, max_rel_err
from oracle import e2e_ref

pytestmark = pytest.mark.gpu
STRESS_MAX_REL_ERR = 5e-2


def _build(name, dev):
    import cti_b200
    from cti_b200.model import CTRModel, TransformerEncoder

    N, Lmax, D, H, L, Fd, E, V, _ = gi.E2E_CASES[name]
    rep = cti_b200.RepEncoder(vocab_size=V, emb_dim=gi.E2E_EMB, padding_idx=0,
                              slot_num=gi.E2E_SLOTS, d_model=D)
    enc = TransformerEncoder(D, H, L, Fd, num_experts=E)
    model = CTRModel(rep, enc, D, head_hidden=gi.E2E_HEAD)
    batch, sd = gi.e2e_inputs(name)
    model.load_state_dict(sd, strict=True)
    model.to(dev).prepare_for_inference()
    return model, batch, sd


@pytest.mark.parametrize("name", list(gi.E2E_CASES))
def test_ctr_model_matches_reference_fixture(cuda_device, name):
    """Configuration init (weight std 0.02): encoder output within max rel
    err 2e-2 and probabilities within 1e-3 absolute.
    Large-weight stress case (weights 2.5-5x the configuration's, logits of
    several units): two layers of bf16 activations against fp32 put the
    encoder output and the logits within max rel err 5e-2 (measured 2.9e-2),
    not 1e-3 in probability."""
    from cti_b200 import _lib

    model, batch, sd = _build(name, cuda_device)
    gold = load_golden(name)
    assert str(gold["input_sha256"]) == gi.e2e_digest(batch, sd)
    hidden = {}
    model.seq_encoder.register_forward_hook(lambda m, i, o: hidden.__setitem__("h", o[0]))
    logits, aux = model(batch)
    probs = model.predict(batch)
    _lib.raise_on_status(cuda_device)
    T = int(batch["user_offsets"][-1])
    assert aux is None and logits.shape == (T, 1)
    assert probs.shape == (T,) and probs.dtype == torch.float32
    assert model.seq_encoder.moe[0].gate.w_g.weight.dtype == torch.float32  # fp32 router
    init_scale = gi.E2E_CASES[name][-1] is not None
    tol = MOE_MAX_REL_ERR if init_scale else STRESS_MAX_REL_ERR
    assert max_rel_err(hidden["h"].float().cpu(), torch.from_numpy(gold["hidden"])) < tol
    if init_scale:
        np.testing.assert_allclose(probs.cpu().numpy(), gold["probs"], rtol=0, atol=1e-3)
    else:
        assert max_rel_err(logits.float().reshape(-1).cpu(), torch.from_numpy(gold["logits"])) < tol


def test_attention_kernel_agrees_with_torch_formulations(cuda_device):
    """The model's attention (this library's kernel) against PyTorch's
    varlen flash attention and padded SDPA (tests/attention_ref.py) on a
    larger packed batch, and one sequence against a plain fp32 softmax."""
    from attention_ref import padded_causal_attention, varlen_causal_attention
    from cti_b200.model import causal_attention

    g = torch.Generator().manual_seed(3)
    lens = torch.randint(1, 257, (64,), generator=g)
    cu = torch.zeros(65, dtype=torch.int32)
    cu[1:] = torch.cumsum(lens, 0)
    T = int(cu[-1])
    q, k, v = (torch.randn(T, 8, 32, generator=g).bfloat16().to(cuda_device) for _ in range(3))
    cu = cu.to(cuda_device)
    a = varlen_causal_attention(q, k, v, cu, 256).float()
    b = padded_causal_attention(q, k, v, cu, 256).float()
    c = causal_attention(q, k, v, cu, 256).float()
    assert max_rel_err(a, b) < 1e-2
    assert max_rel_err(c, b) < 1e-2
    # one sequence against a plain fp32 softmax
    s0, s1 = int(cu[5]), int(cu[6])
    qs, ks, vs = (t[s0:s1].float().transpose(0, 1) for t in (q, k, v))
    sc = (qs @ ks.transpose(-1, -2)) / 32 ** 0.5
    sc = sc.masked_fill(~torch.ones(s1 - s0, s1 - s0, dtype=torch.bool, device=cuda_device).tril(),
                        float("-inf"))
    ref = (torch.softmax(sc, -1) @ vs).transpose(0, 1)
    assert max_rel_err(a[s0:s1], ref) < 1e-2
    assert max_rel_err(c[s0:s1], ref) < 1e-2


def test_cfg4_shaped_model_matches_oracle(cuda_device):
    """The configuration-4 architecture and init (D 256, 8 heads x 32, 16
    experts of d_ff 1024 with the Zipf router bias, per-slot tables, weights
    ~N(0, 0.02)) at 2 layers and 24 sequences, against the oracle:
    probabilities within 1e-3 absolute."""
    from cti_b200 import _lib, synth
    from cti_b200.model import build_ctr_model

    nseq = 24
    lens = torch.randint(16, 257, (nseq,), generator=torch.Generator().manual_seed(1))
    uo = torch.zeros(nseq + 1, dtype=torch.long)
    uo[1:] = torch.cumsum(lens, 0)
    T = int(uo[-1])
    bb = synth.bag_batch(batch=T, seed=2, vocab_lo=1e3, vocab_hi=2e4)
    model = build_ctr_model(bb.vocab.tolist(), num_layers=2)
    synth.init_ctr_model(model)
    with torch.no_grad():
        model.rep_encoder.emb.weight.copy_(synth.embedding_table(bb.total_rows, 64, seed=2).float())
        for name, p in model.named_parameters():
            if "gate" not in name and "emb" not in name:
                p.copy_(p.bfloat16().float())
    sd = {k: v.clone() for k, v in model.state_dict().items()}
    batch = {"_flat_values": bb.values, "_flat_row_offsets": bb.row_offsets,
             "_val_offsets": bb.val_offsets, "user_offsets": uo}
    model.to(cuda_device).prepare_for_inference()
    logits, _ = model(batch)
    probs = model.predict(batch)
    _lib.raise_on_status(cuda_device)
    torch.set_num_threads(8)
    _, ref_logits, ref = e2e_ref.ctr_forward_ref(sd, batch, slot_num=28, n_heads=8, num_layers=2,
                                                 num_experts=16, table_row_base=bb.table_row_base,
                                                 vocab=bb.vocab)
    np.testing.assert_allclose(probs.cpu().numpy(), ref.numpy(), rtol=0, atol=1e-3)


def test_predict_host_chunks_match_predict(cuda_device):
    """CTRModel.predict_host (host batch, sequences cut into chunks whose
    host->device copies overlap the previous chunk's forward) against
    predict on the device batch and against the oracle: probabilities within
    1e-3 absolute, for 1, 3 and 7 chunks and a repeated call into the same
    output.  Zero-length bags and a 1-token sequence are included."""
    from cti_b200 import _lib, synth
    from cti_b200.model import build_ctr_model

    g = torch.Generator().manual_seed(11)
    lens = torch.randint(16, 257, (20,), generator=g)
    lens[4] = 1
    uo = torch.zeros(lens.numel() + 1, dtype=torch.long)
    uo[1:] = torch.cumsum(lens, 0)
    T = int(uo[-1])
    bb = synth.bag_batch(batch=T, seed=5, vocab_lo=1e3, vocab_hi=2e4)
    model = build_ctr_model(bb.vocab.tolist(), num_layers=2)
    synth.init_ctr_model(model, seed=5)
    with torch.no_grad():
        model.rep_encoder.emb.weight.copy_(synth.embedding_table(bb.total_rows, 64, seed=5).float())
        for name, p in model.named_parameters():
            if "gate" not in name and "emb" not in name:
                p.copy_(p.bfloat16().float())
    sd = {k: v.clone() for k, v in model.state_dict().items()}
    host = {"_flat_values": bb.values, "_flat_row_offsets": bb.row_offsets,
            "_val_offsets": bb.val_offsets, "user_offsets": uo}
    model.to(cuda_device).prepare_for_inference()
    dev_probs = model.predict({k: v.to(cuda_device) for k, v in host.items()}).cpu().numpy()
    pinned = {k: v.pin_memory() for k, v in host.items()}
    torch.set_num_threads(8)
    _, _, ref = e2e_ref.ctr_forward_ref(sd, host, slot_num=28, n_heads=8, num_layers=2,
                                        num_experts=16, table_row_base=bb.table_row_base,
                                        vocab=bb.vocab)
    out = None
    for chunks in (1, 3, 7, 7):
        probs = model.predict_host(pinned, chunks=chunks, out=out)
        torch.cuda.current_stream(cuda_device).synchronize()
        _lib.raise_on_status(cuda_device)
        assert probs.shape == (T,) and probs.dtype == torch.float32 and not probs.is_cuda
        if out is not None:
            assert probs.data_ptr() == out.data_ptr()
        np.testing.assert_allclose(probs.numpy(), dev_probs, rtol=0, atol=1e-3)
        np.testing.assert_allclose(probs.numpy(), ref.numpy(), rtol=0, atol=1e-3)
        out = probs


def test_full_cfg4_model_matches_oracle_on_sampled_sequences(cuda_device):
    """The whole configuration-4 forward: 2048 packed sequences (284,237
    tokens, 204 M ids), 8 layers, per-slot fp16 tables, run on the device
    as the benchmark runs it.  Sequences are independent, so the oracle runs
    on 24 seeded sampled sequences alone (their flat-layout sub-batch).

    The model's activations are bf16, so its router sees bf16 LayerNorm
    outputs, and a token whose top-2 logits are nearly tied (fp64 gap of a
    few 1e-3) can take a different second expert at some layer - the
    reference's own bf16 model (online_best casts everything but nothing
    else to bf16) does the same.  So the check is in two parts:
      * the oracle follows the device's routes at every layer (the experts
        the device chose; the oracle's own fp32 gate probabilities weight
        them): every probability within 1e-3 absolute, the north-star bound;
      * every route where the device differs from the oracle's own top-2
        lies in the fp64 near-tie band (gap below 1e-2, about 3 % of the
        logits' spread of 0.3; flips were measured at gaps up to 5.6e-3),
        and such routes are few (at most 3 % of token-layers; a CPU
        emulation of the bf16 rounding points gives about 1.3 %).
    Unforced, the largest difference is printed (about 1e-3, at a token
    whose layer-0 routing flips at a gap of 6e-4)."""
    from cti_b200 import _lib, synth
    from cti_b200.model import build_ctr_model

    bb, uo, T = synth.cfg4_batch(seed=0)
    model = build_ctr_model(bb.vocab.tolist())
    synth.init_ctr_model(model)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "gate" not in name and "emb" not in name:
                p.copy_(p.bfloat16().float())
    # Everything but the 1.4 GB table goes to the oracle in fp32.
    sd = {k: v.clone() for k, v in model.state_dict().items() if k != "rep_encoder.emb.weight"}
    model.rep_encoder.emb.weight = torch.nn.Parameter(torch.empty(0), requires_grad=False)
    table = synth.embedding_table(bb.total_rows, 64, seed=0)
    model.to(cuda_device)
    model.rep_encoder.emb.weight = torch.nn.Parameter(table.to(cuda_device), requires_grad=False)
    model.prepare_for_inference()
    batch = {"_flat_values": bb.values, "_flat_row_offsets": bb.row_offsets,
             "_val_offsets": bb.val_offsets, "user_offsets": uo}
    seqs = sorted(torch.randperm(synth.CFG4_SAMPLES,
                                 generator=torch.Generator().manual_seed(7))[:24].tolist())
    rows = torch.cat([torch.arange(int(uo[s]), int(uo[s + 1])) for s in seqs])
    # Each MoE layer's routes on the device (its gate on the layer's input).
    routes = []
    hooks = [m.register_forward_hook(
        lambda mod, inp, out: routes.append(mod.gate(inp[0])[0].reshape(-1, 2)[
            rows.to(cuda_device)].cpu())) for m in model.seq_encoder.moe]
    probs = model.predict({k: v.to(cuda_device) for k, v in batch.items()}).cpu()
    for h in hooks:
        h.remove()
    _lib.raise_on_status(cuda_device)
    assert probs.shape == (T,) and torch.isfinite(probs).all() and len(routes) == 8

    sub = synth.sequence_subbatch(bb, uo, seqs)
    sd["rep_encoder.emb.weight"] = table
    torch.set_num_threads(8)
    kw = dict(slot_num=28, n_heads=8, num_layers=8, num_experts=16,
              table_row_base=bb.table_row_base, vocab=bb.vocab)
    mine = probs[rows]
    _, _, free = e2e_ref.ctr_forward_ref(sd, sub, **kw)
    print(f"unforced: max |p - p_ref| {float((mine - free).abs().max()):.2e}")
    routing = []
    _, _, ref = e2e_ref.ctr_forward_ref(sd, sub, force_routes=routes, routing=routing, **kw)
    assert mine.numel() == ref.numel() == int(sub["user_offsets"][-1])
    np.testing.assert_allclose(mine.numpy(), ref.numpy(), rtol=0, atol=1e-3)
    flips = 0
    for layer, ((own, gap), dev_idx) in enumerate(zip(routing, routes)):
        differ = (own != dev_idx.long()).any(dim=1)
        assert (gap[differ] < 1e-2).all(), (layer, gap[differ].max())
        flips += int(differ.sum())
    print(f"routes differing from the oracle's own top-2: {flips} of {8 * mine.numel()}")
    assert flips <= 0.03 * 8 * mine.numel()
