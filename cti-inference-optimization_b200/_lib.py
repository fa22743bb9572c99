"""ctypes binding of ``libcti_b200.so`` (declared in ``include/cti_b200.h``).

The library is the only compute path of this package: if it is missing or
fails to load, importing a module that needs it raises, and every wrapper
raises ``RuntimeError`` on a non-zero return code.  There is no eager-PyTorch
fallback.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libcti_b200.so"

CTI_OK = 0
CTI_ERR_INVALID_ARG = 1
CTI_ERR_UNSUPPORTED = 2
CTI_ERR_CUDA = 3
CTI_ERR_TIMEOUT = 4
CTI_ERR_BOUNDS = 5
ERROR_NAMES = {
    CTI_ERR_INVALID_ARG: "invalid argument",
    CTI_ERR_UNSUPPORTED: "unsupported shape",
    CTI_ERR_CUDA: "CUDA error",
    CTI_ERR_TIMEOUT: "device wait timed out",
    CTI_ERR_BOUNDS: "index out of bounds",
}

ACT_NONE, ACT_RELU, ACT_GELU = 0, 1, 2
ACTIVATIONS = {"none": ACT_NONE, "relu": ACT_RELU, "gelu": ACT_GELU}
DTYPE_CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
ROUTER_BLOCK_TOKENS = 128
MAX_EXPERTS = 128
NOALLOC_MAX_TOKENS = 131072
NOALLOC_MAX_EXPERTS = 128

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/cti_b200.h one to one.
SIGNATURES = {
    "cti_version": (ctypes.c_char_p, []),
    "cti_num_sms": (_I, [_I, _P]),
    "cti_status_read": (_I, [_P, _I, _P, _P, _P]),
    "cti_moe_router": (_I, [_P, _P, _P, _I64, _I, _I, _I, _P, _P, _P, _P, _P, _P]),
    "cti_moe_dispatch_workspace_bytes": (_SZ, [_I64, _I]),
    "cti_moe_dispatch": (_I, [_P, _P, _P, _P, _I64, _I, _I, _P, _P, _P, _P, _P, _P]),
    "cti_moe_route_dispatch_noalloc": (
        _I, [_P, _P, _P, _I64, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P]),
    "cti_moe_grouped_gemm": (_I, [_P, _P, _P, _P, _I, _I, _I64, _I, _I, _I, _P, _P, _P]),
    "cti_moe_expert_ffn_fused": (
        _I,
        [_P, _P, _P, _P, _P, _P, _I, _I, _I64, _I, _I, _I, _P, _P, _P],
    ),
    "cti_moe_expert_ffn_fused_gather": (
        _I,
        [_P, _I64, _P, _P, _P, _P, _P, _P, _I, _I, _I64, _I, _I, _I, _P, _P, _P],
    ),
    "cti_moe_expert_ffn_fused_pair": (
        _I,
        [_P, _P, _P, _P, _P, _P, _I, _I, _I64, _I, _I, _I, _P, _P, _P],
    ),
    "cti_moe_expert_ffn_fused_supported": (_I, [_I, _I, _I, _I64]),
    "cti_moe_combine": (_I, [_P, _I64, _P, _P, _I64, _I, _P, _P, _P]),
    "cti_moe_layer_workspace_bytes": (_SZ, [_I64, _I, _I, _I]),
    "cti_moe_layer_forward": (
        _I,
        [_P, _P, _P, _P, _P, _P, _P, _I64, _I, _I, _I, _I, _I, _P, _P, _SZ, _P, _P],
    ),
    "cti_moe_layer_forward_host": (
        _I,
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I, _I, _I, _I, _I, _I64, _P, _SZ, _P,
         _P, _P, _P, _P],
    ),
    "cti_embbag_sum": (
        _I,
        [_P, _I64, _P, _P, _P, _P, _P, _I64, _I64, _I, _I, _P, _I, _P, _P],
    ),
    "cti_selftest_wait_timeout": (_I, [_P, _I64, _P]),
    "cti_ctr_head": (_I, [_P, _P, _P, _P, _P, _I64, _I, _I, ctypes.c_float, _P, _P, _P, _P]),
    "cti_rep_encoder_fused": (
        _I, [_P, _I64, _P, _P, _P, _P, _P, _I64, _I64, _I, _I, _P, _P, _P, _I, ctypes.c_float, _P,
             _P, _P]),
    "cti_varlen_attention": (
        _I, [_P, _P, _P, _I64, _I64, _I64, _P, _I, _I, _I64, _I, _I, _P, _P, _P]),
    "cti_add_layernorm": (
        _I,
        [_P, _P, _P, _P, _I64, _I, ctypes.c_float, _P, _P, _P],
    ),
}


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH.name} is not built; run __graft_entry__.build() (nvcc, sm_100a) first"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def check(rc: int, what: str) -> None:
    if rc != CTI_OK:
        raise RuntimeError(f"{what} failed: {ERROR_NAMES.get(rc, 'error')} (code {rc})")


def ptr(t: torch.Tensor | None) -> int | None:
    """Device pointer of a tensor (None passes NULL)."""
    if t is None:
        return None
    return t.data_ptr()


def stream_handle(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_STATUS: dict[int, torch.Tensor] = {}


def status_word(device: torch.device) -> torch.Tensor:
    """The per-device int32[2] status word the kernels report into."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    st = _STATUS.get(idx)
    if st is None:
        st = torch.zeros(2, dtype=torch.int32, device=torch.device("cuda", idx))
        _STATUS[idx] = st
    return st


def read_status(device: torch.device, clear: bool = True) -> tuple[int, int]:
    """Synchronises the current stream and returns (code, detail)."""
    st = status_word(device)
    code = ctypes.c_int32(0)
    detail = ctypes.c_int32(0)
    check(
        lib.cti_status_read(
            ptr(st), int(clear), ctypes.byref(code), ctypes.byref(detail), stream_handle(device)
        ),
        "cti_status_read",
    )
    return code.value, detail.value


def raise_on_status(device: torch.device) -> None:
    code, detail = read_status(device, clear=True)
    if code != CTI_OK:
        raise RuntimeError(
            f"device reported {ERROR_NAMES.get(code, 'error')} (code {code}, detail {detail})"
        )


def require_cuda(t: torch.Tensor, name: str, dtype: torch.dtype | None = None) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (this library has no CPU path)")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
