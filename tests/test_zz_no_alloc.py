"""The allocation-free routing + dispatch entry point.

cti_moe_route_dispatch_noalloc serves callers that cannot hand the library a
device workspace: a host that binds only the C library and has no device
allocator of its own, or one that must run inside a fixed, pre-reserved
memory budget.  Its scratch lives in a device array inside the library.
This file checks, through the C ABI, that two calls in a row give exactly
the results of the normal router + dispatch entry points (routing and
dispatch are integer/index work plus fp32 gates, so the comparison is
bit-exact), and that sizes past the array's limit are refused.  It is named
to run last and also passes on its own in a fresh process.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(T, D, E, seed, dev):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(T, D, generator=g).bfloat16().to(dev)
    wg = (torch.randn(E, D, generator=g) * 0.05).to(dev)
    bg = torch.randn(E, generator=g).to(dev)
    return x, wg, bg


def _noalloc(x, wg, bg, E, dev):
    from cti_b200 import _lib

    T, D = x.shape
    idx2 = torch.full((T, 2), -7, dtype=torch.int32, device=dev)
    gate2 = torch.full((T, 2), -7.0, dtype=torch.float32, device=dev)
    offsets = torch.full((E + 1,), -7, dtype=torch.int32, device=dev)
    perm_inv = torch.full((T, 2), -7, dtype=torch.int32, device=dev)
    sorted_token = torch.full((2 * T,), -7, dtype=torch.int32, device=dev)
    xperm = torch.zeros((2 * T, D), dtype=torch.bfloat16, device=dev)
    st = _lib.status_word(dev)
    rc = _lib.lib.cti_moe_route_dispatch_noalloc(
        x.data_ptr(), wg.data_ptr(), bg.data_ptr(), T, D, E, 1, idx2.data_ptr(),
        gate2.data_ptr(), offsets.data_ptr(), perm_inv.data_ptr(), sorted_token.data_ptr(),
        xperm.data_ptr(), st.data_ptr(), _lib.stream_handle(dev))
    assert rc == _lib.CTI_OK
    _lib.raise_on_status(dev)
    return idx2, gate2, offsets, perm_inv, sorted_token, xperm


def _reference_path(x, wg, bg, E, dev):
    from cti_b200 import _lib, ops

    r = ops.router(x, wg, bg, renorm=True)
    d = ops.dispatch(x, r, E)
    _lib.raise_on_status(dev)
    return r.idx2, r.gate2, d.offsets, d.perm_inv, d.sorted_token, d.xperm


NAMES = ("idx2", "gate2", "offsets", "perm_inv", "sorted_token", "xperm")


def _check_pair(problems, dev):
    # Problems back to back: a call must not be affected by what the one
    # before it left in the shared device array.
    for T, D, E, seed in problems:
        x, wg, bg = _inputs(T, D, E, seed, dev)
        got = _noalloc(x, wg, bg, E, dev)
        want = _reference_path(x, wg, bg, E, dev)
        for name, a, b in zip(NAMES, got, want):
            assert torch.equal(a, b), (name, T, D, E)


def test_noalloc_matches_workspace_entry_points_twice_in_a_row():
    assert torch.cuda.is_available()
    _check_pair(((72214, 256, 16, 1), (5003, 128, 8, 2)), torch.device("cuda", 0))


@pytest.mark.parametrize("problems", [
    # the whole array: T at the limit with the most experts (every per-block
    # count slot used), then a small problem over the same array
    ((131072, 128, 128, 3), (300, 128, 8, 4)),
    # expert counts that do not divide the scan's chunking evenly
    ((9001, 256, 6, 5), (7777, 128, 100, 6)),
    # no tokens: only the offsets are written (all zero), between two calls
    ((1000, 128, 16, 7), (0, 128, 16, 8), (1000, 128, 16, 9)),
])
def test_noalloc_edges_match_workspace_entry_points(problems):
    _check_pair(problems, torch.device("cuda", 0))


def test_noalloc_refuses_sizes_past_its_array():
    from cti_b200 import _lib

    dev = torch.device("cuda", 0)
    T = _lib.NOALLOC_MAX_TOKENS + 1
    rc = _lib.lib.cti_moe_route_dispatch_noalloc(
        None, None, None, T, 256, 16, 1, None, None, None, None, None, None, None,
        _lib.stream_handle(dev))
    assert rc == _lib.CTI_ERR_UNSUPPORTED
    rc = _lib.lib.cti_moe_route_dispatch_noalloc(
        None, None, None, 100, 256, _lib.NOALLOC_MAX_EXPERTS + 1, 1, None, None, None, None,
        None, None, None, _lib.stream_handle(dev))
    assert rc == _lib.CTI_ERR_UNSUPPORTED
