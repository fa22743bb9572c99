"""Failure detection on the GPU without a fault: a bounded wait that runs out
(a barrier nothing arrives at) must leave CTI_ERR_TIMEOUT in the status
word, return, and leave the context usable for the next kernels."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives(cuda_device):
    from cti_b200 import _lib, ops, synth

    dev = cuda_device
    st = _lib.status_word(dev)
    _lib.read_status(dev, clear=True)
    t0 = time.perf_counter()
    assert _lib.lib.cti_selftest_wait_timeout(_lib.ptr(st), 20_000_000,
                                              _lib.stream_handle(dev)) == _lib.CTI_OK
    code, detail = _lib.read_status(dev, clear=True)
    elapsed = time.perf_counter() - t0
    assert code == _lib.CTI_ERR_TIMEOUT and detail == 0x7F0
    assert 0.015 < elapsed < 5.0
    # the context is intact: a normal layer runs and reports no error
    w = synth.moe_weights(128, 8, 256, None, device=dev)
    x = synth.moe_activations(512, 128, device=dev)
    r = ops.router(x, w.wg, w.bg)
    torch.cuda.synchronize(dev)
    assert _lib.read_status(dev) == (0, 0)
    assert r.idx2.shape == (512, 2)


def test_selftest_rejects_bad_limits(cuda_device):
    from cti_b200 import _lib

    st = _lib.status_word(cuda_device)
    for bad in (0, 999, 3_000_000_000):
        assert _lib.lib.cti_selftest_wait_timeout(_lib.ptr(st), bad, None) == _lib.CTI_ERR_INVALID_ARG
