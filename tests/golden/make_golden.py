"""Generates tests/golden/*.npz by running the REFERENCE's own code.

Run from the repository root, in a container where the reference checkout
exists (it is read, never modified):

    python tests/golden/make_golden.py /path/to/reference

What runs:
  * baseline/infer.py SMoE (Expert, TopKGate, SMoE; :280-358), in fp32 on
    CPU, in eval mode.  "refexact" fixtures run it unmodified (ReLU experts,
    raw top-2 softmax scores).  "config" fixtures run the same module with
    the benchmark semantics patched onto that instance only: Expert.forward
    -> fc2(gelu(fc1(x))), and TopKGate.forward -> stable descending sort
    (ties to the lower id) with the two scores renormalised to sum to 1.
    The per-expert gather / scatter-add loop of SMoE.forward is the
    reference's own.
  * baseline/infer.py RepEncoder pooling (:253-263) with input_norm and
    linear replaced by identities, so forward() returns the pooled
    [B, 28*64] tensor.  Per-feature tables run one single-slot RepEncoder
    per feature.
  * baseline/infer.py CTRModel (RepEncoder -> TransformerEncoder with its
    SMoE layers -> head, :244-439) in fp32 on CPU, eval mode, at a small
    size: the SMoE experts and gates patched as for the "config" fixtures,
    and CTRModel.linear replaced by the configuration's MLP head
    (d -> 128 -> 1, ReLU).  The attention is the reference's own
    scaled_dot_product with its dense causal sequence mask.
Each fixture stores the outputs plus the SHA-256 of the inputs
(tests/golden/golden_inputs.py regenerates the inputs from seeds).
"""
from __future__ import annotations

import importlib.util
import sys
import types
from pathlib import Path

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import golden_inputs as gi  # noqa: E402


def load_reference(ref_root: Path):
    spec = importlib.util.spec_from_file_location("ref_baseline_infer",
                                                  ref_root / "baseline" / "infer.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _gelu_expert_forward(self, x):
    return self.fc2(F.gelu(self.fc1(x)))


def _stable_renorm_gate_forward(self, x):
    logits = self.w_g(x)
    probs = torch.softmax(logits, dim=-1)
    order = torch.sort(probs, dim=-1, descending=True, stable=True).indices[..., : self.k]
    score = probs.gather(-1, order)
    score = score / score.sum(dim=-1, keepdim=True)
    return order, score, probs


def make_moe(ref, name: str):
    inp = gi.moe_inputs(name)
    D, E, Fd, T, act, renorm, _ = gi.MOE_CASES[name]
    m = ref.SMoE(D, Fd, E, k=2).eval()
    with torch.no_grad():
        m.gate.w_g.weight.copy_(inp["wg"])
        m.gate.w_g.bias.copy_(inp["bg"])
        for e, ex in enumerate(m.experts):
            ex.fc1.weight.copy_(inp["w1"][e])
            ex.fc1.bias.copy_(inp["b1"][e])
            ex.fc2.weight.copy_(inp["w2"][e])
            ex.fc2.bias.copy_(inp["b2"][e])
    if act == "gelu":
        for ex in m.experts:
            ex.forward = types.MethodType(_gelu_expert_forward, ex)
    if renorm:
        m.gate.forward = types.MethodType(_stable_renorm_gate_forward, m.gate)
    with torch.no_grad():
        x3 = inp["x"].unsqueeze(0)
        out, _ = m(x3)
        idx, score, probs = m.gate(x3)
    digest = gi.tensor_digest(inp["x"], inp["wg"], inp["bg"], inp["w1"], inp["b1"], inp["w2"],
                              inp["b2"])
    np.savez_compressed(HERE / f"{name}.npz", out=out[0].numpy(), idx=idx[0].numpy(),
                        score=score[0].numpy(), probs=probs[0].numpy(),
                        input_sha256=np.array(digest))


def make_bags(ref, per_feature: bool):
    inp = gi.bag_inputs(per_feature)
    F_, B = inp["features"], inp["batch"]
    dim = inp["table"].shape[1]
    outs = []
    if per_feature:
        for f in range(F_):
            enc = ref.RepEncoder(vocab_size=int(inp["vocab"][f]), emb_dim=dim, padding_idx=0,
                                 slot_num=1, d_model=4)
            enc.input_norm = nn.Identity()
            enc.linear = nn.Identity()
            lo = int(inp["table_row_base"][f])
            with torch.no_grad():
                enc.emb.weight.copy_(inp["table"][lo:lo + int(inp["vocab"][f])].float())
            offs = inp["row_offsets"][f * (B + 1):(f + 1) * (B + 1)]
            v0 = int(inp["val_offsets"][f])
            vals = inp["values"][v0:v0 + int(offs[-1])]
            with torch.no_grad():
                outs.append(enc({1: (vals, offs)}))
        pooled = torch.cat(outs, dim=1)
    else:
        enc = ref.RepEncoder(vocab_size=int(inp["vocab"][0]), emb_dim=dim, padding_idx=0,
                             slot_num=F_, d_model=4)
        enc.input_norm = nn.Identity()
        enc.linear = nn.Identity()
        with torch.no_grad():
            enc.emb.weight.copy_(inp["table"].float())
        batch = {}
        for f in range(F_):
            offs = inp["row_offsets"][f * (B + 1):(f + 1) * (B + 1)]
            v0 = int(inp["val_offsets"][f])
            batch[f + 1] = (inp["values"][v0:v0 + int(offs[-1])], offs)
        with torch.no_grad():
            pooled = enc(batch)
    digest = gi.tensor_digest(inp["values"], inp["row_offsets"], inp["val_offsets"],
                              inp["vocab"], inp["table_row_base"], inp["table"])
    name = "embbag_per_feature" if per_feature else "embbag_shared_table"
    np.savez_compressed(HERE / f"{name}.npz", pooled=pooled.numpy(),
                        input_sha256=np.array(digest))


def make_e2e(ref, name: str):
    batch, sd = gi.e2e_inputs(name)
    N, Lmax, D, H, L, Fd, E, V, _ = gi.E2E_CASES[name]
    rep = ref.RepEncoder(vocab_size=V, emb_dim=gi.E2E_EMB, padding_idx=0, slot_num=gi.E2E_SLOTS,
                         d_model=D)
    enc = ref.TransformerEncoder(D, H, L, Fd)
    model = ref.CTRModel(rep, enc, D)
    model.linear = nn.Sequential(nn.Linear(D, gi.E2E_HEAD), nn.ReLU(), nn.Linear(gi.E2E_HEAD, 1))
    model.load_state_dict(sd, strict=True)
    model.eval()
    for moe in enc.moe:
        assert moe.num_experts == E
        for ex in moe.experts:
            ex.forward = types.MethodType(_gelu_expert_forward, ex)
        moe.gate.forward = types.MethodType(_stable_renorm_gate_forward, moe.gate)
    T = int(batch["user_offsets"][-1])
    ref_batch = {"user_offsets": batch["user_offsets"]}
    for f in range(gi.E2E_SLOTS):
        offs = batch["_flat_row_offsets"][f * (T + 1):(f + 1) * (T + 1)]
        v0 = int(batch["_val_offsets"][f])
        ref_batch[f + 1] = (batch["_flat_values"][v0:v0 + int(offs[-1])], offs)
    hidden = {}
    enc.register_forward_hook(lambda mod, inp, out: hidden.__setitem__("h", out[0]))
    with torch.no_grad():
        logits, _ = model(ref_batch)
        probs = torch.sigmoid(logits)
    np.savez_compressed(HERE / f"{name}.npz", hidden=hidden["h"].reshape(T, D).numpy(),
                        logits=logits.reshape(-1).numpy(), probs=probs.reshape(-1).numpy(),
                        input_sha256=np.array(gi.e2e_digest(batch, sd)))


def main() -> None:
    ref_root = Path(sys.argv[1] if len(sys.argv) > 1 else "../reference")
    ref = load_reference(ref_root)
    torch.set_num_threads(1)
    for name in gi.MOE_CASES:
        make_moe(ref, name)
    make_bags(ref, per_feature=False)
    make_bags(ref, per_feature=True)
    for name in gi.E2E_CASES:
        make_e2e(ref, name)
    keys = list(ref.SMoE(128, 256, 4).state_dict().keys())
    keys += list(ref.RepEncoder(100, 8, 0, 28, 16).state_dict().keys())
    (HERE / "reference_state_dict_keys.txt").write_text("\n".join(keys) + "\n")
    with open(HERE / "MANIFEST.txt", "w") as fh:
        fh.write(f"generated by tests/golden/make_golden.py with torch {torch.__version__}\n")
        for p in sorted(HERE.glob("*.npz")):
            fh.write(f"{p.name} {p.stat().st_size}\n")


if __name__ == "__main__":
    main()
