"""The C-ABI library: built, loadable, exporting exactly what the header
declares, and rejecting bad arguments before touching the device.  No GPU."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "cti_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(cti_\w+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    import cti_b200

    lib = ctypes.CDLL(str(cti_b200.LIB_PATH))
    syms = declared_symbols()
    assert len(syms) >= 12
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in cti_b200.h but not exported"


def test_ctypes_signatures_cover_the_header():
    from cti_b200 import _lib

    assert sorted(_lib.SIGNATURES) == declared_symbols()


def test_exports_match_nm():
    import cti_b200

    out = subprocess.run(["nm", "-D", "--defined-only", str(cti_b200.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = sorted(set(re.findall(r" T (cti_\w+)", out)))
    assert exported == declared_symbols()


def test_library_targets_sm100a_only():
    import cti_b200
    from cti_b200 import build

    assert "arch=compute_100a,code=sm_100a" in " ".join(build.ARCH_FLAGS)
    assert not build.is_stale(), "libcti_b200.so is older than its sources; run build()"


def test_argument_validation_needs_no_device():
    from cti_b200 import _lib

    lib = _lib.lib
    # E above the maximum, D not a multiple of 32, bad activation, bad shapes.
    assert lib.cti_moe_router(None, None, None, 16, 64, 200, 1, None, None, None, None, None,
                              None) == _lib.CTI_ERR_INVALID_ARG
    assert lib.cti_moe_router(None, None, None, 16, 36, 8, 1, None, None, None, None, None,
                              None) == _lib.CTI_ERR_UNSUPPORTED
    assert lib.cti_moe_grouped_gemm(None, None, None, None, 1, 1, 16, 128, 64, 7, None, None,
                                    None) == _lib.CTI_ERR_INVALID_ARG
    assert lib.cti_moe_grouped_gemm(None, None, None, None, 1, 1, 16, 100, 64, 0, None, None,
                                    None) == _lib.CTI_ERR_UNSUPPORTED
    assert lib.cti_moe_grouped_gemm(None, None, None, None, 2000, 1, 16, 128, 64, 0, None, None,
                                    None) == _lib.CTI_ERR_INVALID_ARG
    assert lib.cti_embbag_sum(None, 0, None, None, None, None, None, 0, 4, 28, 64, None, 0, None,
                              None) == _lib.CTI_ERR_INVALID_ARG
    assert lib.cti_moe_combine(None, 0, None, None, 4, 12, None, None, None) == \
        _lib.CTI_ERR_UNSUPPORTED
    # Empty inputs are a no-op, not an error.
    assert lib.cti_moe_router(None, None, None, 0, 64, 8, 1, None, None, None, None, None,
                              None) == _lib.CTI_OK
    assert lib.cti_embbag_sum(None, 0, None, None, None, None, None, 0, 0, 28, 64, None, 0, None,
                              None) == _lib.CTI_OK


def test_workspace_queries():
    from cti_b200 import _lib

    lib = _lib.lib
    assert lib.cti_moe_dispatch_workspace_bytes(69632, 16) == 544 * 16 * 4
    assert lib.cti_moe_dispatch_workspace_bytes(1, 8) == 8 * 4
    small = lib.cti_moe_layer_workspace_bytes(128, 256, 16, 1024)
    big = lib.cti_moe_layer_workspace_bytes(69632, 256, 16, 1024)
    assert 0 < small < big
    assert big % 256 == 0

