"""Compiles the C parts of the oracle (TEST ONLY) into oracle/_build/.

    gcc -O2 -fPIC -shared -ffp-contract=off router_order.c -lm

-ffp-contract=off keeps every multiply-add exactly as written (the explicit
fmaf calls stay fused, nothing else is contracted), so the reduction order
is the one the source states.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
BUILD = HERE / "_build"
LIB = BUILD / "liborder.so"


def build(force: bool = False) -> Path:
    src = HERE / "router_order.c"
    if not force and LIB.exists() and LIB.stat().st_mtime >= src.stat().st_mtime:
        return LIB
    BUILD.mkdir(exist_ok=True)
    subprocess.run(["gcc", "-O2", "-fPIC", "-shared", "-ffp-contract=off", "-o", str(LIB),
                    str(src), "-lm"], check=True)
    return LIB


def router_order(x_bf16_u16: np.ndarray, wg: np.ndarray, bg: np.ndarray, renorm: bool):
    """x as uint16 bf16 bits [T, D]; returns (idx2 [T,2] int32, gate2 [T,2] f32, logits [T,E])."""
    lib = ctypes.CDLL(str(build()))
    x = np.ascontiguousarray(x_bf16_u16, dtype=np.uint16)
    wg = np.ascontiguousarray(wg, dtype=np.float32)
    bg = np.ascontiguousarray(bg, dtype=np.float32)
    T, D = x.shape
    E = wg.shape[0]
    idx2 = np.empty((T, 2), np.int32)
    gate2 = np.empty((T, 2), np.float32)
    logits = np.empty((T, E), np.float32)
    P = ctypes.c_void_p
    lib.router_order_ref.argtypes = [P, P, P, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                     ctypes.c_int, P, P, P]
    lib.router_order_ref(x.ctypes.data, wg.ctypes.data, bg.ctypes.data, T, D, E, int(renorm),
                         idx2.ctypes.data, gate2.ctypes.data, logits.ctypes.data)
    return idx2, gate2, logits


if __name__ == "__main__":
    print(build(force=True))
