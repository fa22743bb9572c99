"""Shared test helpers (tolerances are stated where they are used)."""
from __future__ import annotations

import numpy as np
import torch

GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"

# MoE outputs: bf16 kernels vs the fp32 reference.  "max rel err" is the
# largest absolute difference divided by the largest reference magnitude
# (||a - b||_inf / ||b||_inf), which stays meaningful where single outputs
# are near zero.
MOE_MAX_REL_ERR = 2e-2


def max_rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.float().cpu()
    b = b.float().cpu()
    denom = b.abs().max().item()
    return (a - b).abs().max().item() / max(denom, 1e-30)


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def bf16_bits(x: torch.Tensor) -> np.ndarray:
    return x.detach().cpu().contiguous().bfloat16().view(torch.int16).numpy().view(np.uint16)
