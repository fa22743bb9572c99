"""The whole MoE layer on the B200 (SMoE.forward through cti_moe_layer_forward)
vs the reference: fixtures made by the reference's own code, and the CPU
oracle at the benchmark shapes.  Tolerance: max rel err 2e-2 (bf16 kernels
vs the fp32 reference; helpers.max_rel_err); expert indices bit-exact outside
the fp64 near-tie band."""
import numpy as np
import pytest
import torch

import golden_inputs as gi
from helpers import MOE_MAX_REL_ERR, load_golden, max_rel_err
from oracle import moe_ref as mr

pytestmark = pytest.mark.gpu


def build_module(inp, D, E, Fd, dev):
    import cti_b200

    m = cti_b200.SMoE(D, Fd, E, activation=inp["act"], renormalize=inp["renorm"])
    with torch.no_grad():
        m.gate.w_g.weight.copy_(inp["wg"])
        m.gate.w_g.bias.copy_(inp["bg"])
        for e, ex in enumerate(m.experts):
            ex.fc1.weight.copy_(inp["w1"][e])
            ex.fc1.bias.copy_(inp["b1"][e])
            ex.fc2.weight.copy_(inp["w2"][e])
            ex.fc2.bias.copy_(inp["b2"][e])
    m.to(dev)
    m.prepare_for_inference()
    return m


@pytest.mark.parametrize("name", list(gi.MOE_CASES))
def test_smoe_matches_reference_fixture(cuda_device, name):
    from cti_b200 import _lib

    D, E, Fd, T, act, renorm, _ = gi.MOE_CASES[name]
    inp = gi.moe_inputs(name)
    gold = load_golden(name)
    m = build_module(inp, D, E, Fd, cuda_device)
    x = inp["x"].bfloat16().to(cuda_device).unsqueeze(0)
    out, aux = m(x)
    _lib.raise_on_status(cuda_device)
    assert aux is None and out.shape == (1, T, D) and out.dtype == torch.bfloat16
    err = max_rel_err(out[0], torch.from_numpy(gold["out"]))
    assert err < MOE_MAX_REL_ERR, err
    idx, score = m.gate(x)
    np.testing.assert_array_equal(idx[0].cpu().numpy(), gold["idx"])
    np.testing.assert_allclose(score[0].cpu().numpy(), gold["score"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("cfg_name", ["cfg1", "cfg2"])
@pytest.mark.parametrize("fused", [False, None])
def test_smoe_matches_oracle_at_benchmark_shape(cuda_device, cfg_name, fused):
    from cti_b200 import _lib, synth

    cfg = synth.MOE_CONFIGS[cfg_name]
    T, _ = synth.moe_tokens(cfg)
    w = synth.moe_weights(cfg.d_model, cfg.num_experts, cfg.dim_ff, cfg.zipf_bias)
    x = synth.moe_activations(T, cfg.d_model)
    import cti_b200

    m = cti_b200.SMoE(cfg.d_model, cfg.dim_ff, cfg.num_experts)
    synth.load_moe_module(m, w)
    m.to(cuda_device).prepare_for_inference()
    xd = x.to(cuda_device)
    if fused is False:
        out = m.forward_staged(xd, fused=False)["out"]
    else:
        out = m(xd.unsqueeze(0))[0][0]
    _lib.raise_on_status(cuda_device)
    torch.set_num_threads(max(1, torch.get_num_threads()))
    ref, g = mr.smoe_ref(x.float(), w.wg, w.bg, w.w1.float(), w.b1, w.w2.float(), w.b2)
    err = max_rel_err(out, ref)
    assert err < MOE_MAX_REL_ERR, err
    tie = mr.near_tie_mask(x.float(), w.wg, w.bg)
    idx, _ = m.gate(xd.unsqueeze(0))
    ok = ~tie
    assert torch.equal(idx[0].cpu()[ok], g.idx[ok])


def test_smoe_matches_oracle_at_cfg5_shape(cuda_device):
    """Configuration 5's layer shape (d_model 1024, 64 experts, d_ff 4096,
    Zipf(1.2) router bias) on one GPU over 8,192 tokens - the unfused
    grouped-GEMM path the expert-parallel layer runs on every rank - against
    the oracle: max rel err 2e-2, indices exact outside the near-tie band."""
    from cti_b200 import _lib, synth
    import cti_b200

    cfg = synth.CFG5
    T = 8192
    w = synth.moe_weights(cfg.d_model, cfg.num_experts, cfg.dim_ff, cfg.zipf_bias, seed=4)
    x = synth.moe_activations(T, cfg.d_model, seed=4)
    m = cti_b200.SMoE(cfg.d_model, cfg.dim_ff, cfg.num_experts)
    synth.load_moe_module(m, w)
    m.to(cuda_device).prepare_for_inference()
    xd = x.to(cuda_device)
    out = m(xd.unsqueeze(0))[0][0]
    _lib.raise_on_status(cuda_device)
    ref, g = mr.smoe_ref(x.float(), w.wg, w.bg, w.w1.float(), w.b1, w.w2.float(), w.b2)
    err = max_rel_err(out, ref)
    assert err < MOE_MAX_REL_ERR, err
    idx, _ = m.gate(xd.unsqueeze(0))
    ok = ~mr.near_tie_mask(x.float(), w.wg, w.bg)
    assert torch.equal(idx[0].cpu()[ok], g.idx[ok])


def test_smoe_stages_agree_with_layer_call(cuda_device):
    from cti_b200 import _lib, synth
    import cti_b200

    cfg = synth.CFG2
    w = synth.moe_weights(cfg.d_model, cfg.num_experts, cfg.dim_ff, cfg.zipf_bias, seed=3)
    m = cti_b200.SMoE(cfg.d_model, cfg.dim_ff, cfg.num_experts)
    synth.load_moe_module(m, w)
    m.to(cuda_device).prepare_for_inference()
    x = synth.moe_activations(9000, cfg.d_model, seed=3).to(cuda_device)
    st = m.forward_staged(x, fused=False)
    out = m(x.unsqueeze(0))[0][0]
    _lib.raise_on_status(cuda_device)
    assert torch.equal(out, st["out"]) or max_rel_err(out, st["out"]) < 8e-3


@pytest.mark.parametrize("T", [1, 2, 255, 256, 257])
def test_smoe_small_token_counts(cuda_device, T):
    """The reference switches paths at T < 256 (online_best/infer.py:2077,
    :2196); here every T takes the same kernels."""
    from cti_b200 import _lib, synth
    import cti_b200

    w = synth.moe_weights(128, 8, 512, None, seed=T)
    m = cti_b200.SMoE(128, 512, 8)
    synth.load_moe_module(m, w)
    m.to(cuda_device).prepare_for_inference()
    x = synth.moe_activations(T, 128, seed=T)
    out = m(x.to(cuda_device).unsqueeze(0))[0][0]
    _lib.raise_on_status(cuda_device)
    ref, _ = mr.smoe_ref(x.float(), w.wg, w.bg, w.w1.float(), w.b1, w.w2.float(), w.b2)
    assert max_rel_err(out, ref) < MOE_MAX_REL_ERR


def test_smoe_empty_input(cuda_device):
    import cti_b200

    m = cti_b200.SMoE(128, 256, 8).to(cuda_device)
    out, _ = m(torch.zeros(1, 0, 128, dtype=torch.bfloat16, device=cuda_device))
    assert out.shape == (1, 0, 128)


def test_output_does_not_alias_input_and_residual_add_works(cuda_device):
    """The caller does torch.add(moe_out, residual, out=residual)
    (online_best/infer.py:2513)."""
    from cti_b200 import synth
    import cti_b200

    w = synth.moe_weights(256, 16, 1024, 1.2)
    m = cti_b200.SMoE(256, 1024, 16)
    synth.load_moe_module(m, w)
    m.to(cuda_device)
    x = synth.moe_activations(1000, 256).to(cuda_device).unsqueeze(0)
    residual = x.clone()
    out, _ = m(x)
    assert out.data_ptr() != x.data_ptr()
    expect = out.float() + residual.float()
    torch.add(out, residual, out=residual)
    assert max_rel_err(residual, expect) < 1e-2


def test_expert_forward_runs_on_the_grouped_gemm(cuda_device):
    from cti_b200 import _lib, synth
    import cti_b200

    w = synth.moe_weights(128, 8, 512, None)
    m = cti_b200.SMoE(128, 512, 8)
    synth.load_moe_module(m, w)
    m.to(cuda_device)
    x = synth.moe_activations(300, 128).to(cuda_device)
    y = m.experts[2](x)
    _lib.raise_on_status(cuda_device)
    ref = mr.expert_ref(x.float().cpu(), w.w1[2].float(), w.b1[2], w.w2[2].float(), w.b2[2], "gelu")
    assert max_rel_err(y, ref) < 1e-2


def _cfg2_module(dev, seed=0):
    from cti_b200 import synth
    import cti_b200

    cfg = synth.CFG2
    w = synth.moe_weights(cfg.d_model, cfg.num_experts, cfg.dim_ff, cfg.zipf_bias, seed=seed)
    m = cti_b200.SMoE(cfg.d_model, cfg.dim_ff, cfg.num_experts)
    synth.load_moe_module(m, w)
    m.to(dev).prepare_for_inference()
    return m


@pytest.mark.parametrize("T,chunk,pinned", [
    (None, None, True),     # the cfg2 batch, default chunking (8 chunks)
    (None, 5000, True),     # ragged last chunk
    (9000, 100000, True),   # one chunk larger than T
    (300, 7, True),         # many tiny chunks
    (1, None, True),
    (2000, 512, False),     # pageable host memory: copies serialise, same result
])
def test_forward_host_equals_device_forward(cuda_device, T, chunk, pinned):
    """SMoE.forward_host (cti_moe_layer_forward_host: chunked H2D / layer /
    D2H on three streams) gives the device forward's output bit for bit:
    every token's output depends only on its own row."""
    from cti_b200 import _lib, synth

    m = _cfg2_module(cuda_device)
    if T is None:
        T, _ = synth.moe_tokens(synth.CFG2, seed=0)
    x = synth.moe_activations(T, 256, seed=1)
    ref = m(x.to(cuda_device).unsqueeze(0))[0][0].cpu()
    x_h = x.pin_memory() if pinned else x.clone()
    out_h, aux = m.forward_host(x_h, chunk_tokens=chunk)
    torch.cuda.current_stream(cuda_device).synchronize()
    _lib.raise_on_status(cuda_device)
    assert aux is None and out_h.shape == x.shape and not out_h.is_cuda
    diff = (out_h.float() - ref.float()).abs().max().item()
    assert torch.equal(out_h, ref), diff


def test_forward_host_reuses_buffers_and_orders_after_prior_work(cuda_device):
    """Back-to-back calls into the same output buffer, then a device forward
    of another batch: each result is the one for its own input."""
    from cti_b200 import _lib, synth

    m = _cfg2_module(cuda_device, seed=2)
    xs = [synth.moe_activations(20000, 256, seed=s) for s in (5, 6)]
    refs = [m(x.to(cuda_device).unsqueeze(0))[0][0].cpu() for x in xs]
    out_h = torch.empty(20000, 256, dtype=torch.bfloat16).pin_memory()
    for x, ref in zip(xs, refs):
        m.forward_host(x.pin_memory(), out_h, chunk_tokens=3000)
        torch.cuda.current_stream(cuda_device).synchronize()
        assert torch.equal(out_h, ref)
    _lib.raise_on_status(cuda_device)


def test_forward_host_graph_replays_with_new_contents(cuda_device):
    """forward_host(graph=True): the first call runs and captures the
    pipeline, later calls replay it; new contents written into the same
    page-locked input buffer give their own outputs, bit for bit equal to the
    device forward."""
    from cti_b200 import _lib, synth

    m = _cfg2_module(cuda_device, seed=3)
    T = 30000
    x_h = torch.empty(T, 256, dtype=torch.bfloat16).pin_memory()
    out_h = torch.empty(T, 256, dtype=torch.bfloat16).pin_memory()
    for s in (7, 8, 9):
        x = synth.moe_activations(T, 256, seed=s)
        ref = m(x.to(cuda_device).unsqueeze(0))[0][0].cpu()
        x_h.copy_(x)
        out_h.zero_()
        m.forward_host(x_h, out_h, chunk_tokens=4096, graph=True)
        torch.cuda.current_stream(cuda_device).synchronize()
        assert torch.equal(out_h, ref), s
    _lib.raise_on_status(cuda_device)
    with pytest.raises(ValueError):
        m.forward_host(x_h.clone(), graph=True)  # pageable input


def test_layer_forward_host_c_abi_single_stream_and_errors(cuda_device):
    """The C entry point with the copy streams equal to the compute stream,
    and its argument checks."""
    from cti_b200 import _lib, synth
    from cti_b200._lib import lib, ptr, stream_handle, status_word

    m = _cfg2_module(cuda_device, seed=4)
    T, D = 4000, 256
    x = synth.moe_activations(T, D, seed=4)
    ref = m(x.to(cuda_device).unsqueeze(0))[0][0].cpu()
    x_h = x.pin_memory()
    out_h = torch.empty_like(x_h).pin_memory()
    xd = torch.empty(T, D, dtype=torch.bfloat16, device=cuda_device)
    od = torch.empty_like(xd)
    chunk = 1024
    ws = torch.empty(int(lib.cti_moe_layer_workspace_bytes(chunk, D, 16, 1024)), dtype=torch.uint8,
                     device=cuda_device)
    s = stream_handle(cuda_device)

    def call(xh=x_h, chunk_tokens=chunk, ws_bytes=None, s2=None, wsp=ws):
        return lib.cti_moe_layer_forward_host(
            ptr(xh) if xh is not None else None, ptr(out_h), ptr(xd), ptr(od), ptr(m._wg),
            ptr(m._bg), ptr(m._w1), ptr(m._b1), ptr(m._w2), ptr(m._b2), T, D, 16, 1024,
            _lib.ACTIVATIONS["gelu"], 1, chunk_tokens, ptr(wsp),
            wsp.numel() if ws_bytes is None else ws_bytes, ptr(status_word(cuda_device)), s, s, s,
            s2)

    assert call() == _lib.CTI_OK
    torch.cuda.current_stream(cuda_device).synchronize()
    _lib.raise_on_status(cuda_device)
    assert torch.equal(out_h, ref)
    assert call(chunk_tokens=0) == _lib.CTI_ERR_INVALID_ARG
    assert call(xh=None) == _lib.CTI_ERR_INVALID_ARG
    assert call(chunk_tokens=2048) == _lib.CTI_ERR_INVALID_ARG  # workspace sized for 1024
    assert call(ws_bytes=16) == _lib.CTI_ERR_INVALID_ARG
    # A second compute stream: odd chunks on it, on the workspace's second half.
    s2 = torch.cuda.Stream(cuda_device)
    assert call(s2=s2.cuda_stream) == _lib.CTI_ERR_INVALID_ARG  # one half only
    half = -(-ws.numel() // 256) * 256
    ws2 = torch.empty(half + ws.numel(), dtype=torch.uint8, device=cuda_device)
    out_h.zero_()
    assert call(s2=s2.cuda_stream, wsp=ws2) == _lib.CTI_OK
    torch.cuda.current_stream(cuda_device).synchronize()
    _lib.raise_on_status(cuda_device)
    assert torch.equal(out_h, ref)
