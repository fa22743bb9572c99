"""Drop-in Top-2 sparse MoE block (``SMoE``) running on the sm_100a kernels.

Module API, constructor arguments and state-dict keys follow the reference
(``online_best/infer.py:1781-1954``, ``baseline/infer.py:280-358``):

* ``Expert(d_model, dim_ff)`` with ``fc1``/``fc2`` ``nn.Linear`` submodules;
* ``TopKGate(d_model, num_experts, k=2)`` with ``w_g`` ``nn.Linear``;
* ``SMoE(d_model, dim_ff, num_experts, k=2)`` with ``experts`` and ``gate``,
  ``prepare_for_inference()`` and ``forward(x[B,S,D]) -> (out[B,S,D], None)``.

Differences from the reference, by design:

* ``prepare_for_inference`` stacks the expert weights but never prunes
  ``dim_ff`` (the reference prunes to 192 channels at
  ``online_best/infer.py:1886-1897``); it is also run automatically on the
  first forward if the caller did not.
* The expert activation and the gate normalisation are constructor options.
  ``activation="gelu", renormalize=True`` is the benchmark configuration;
  ``activation="relu", renormalize=False`` reproduces the reference model
  (``baseline/infer.py:287``, ``:305-309``).  Top-2 ties go to the lower
  expert id in both modes.
* The router runs in fp32 over bf16 activations whatever the module dtype.
* There is no CPU or eager fallback: ``forward`` takes bf16 CUDA tensors;
  ``forward_host`` takes bf16 host tensors and still computes on the GPU
  (the copies in and out overlap the layer, chunk by chunk).
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import _lib, ops
from ._lib import check, lib, ptr, stream_handle, status_word


def _prepare_x(x: torch.Tensor) -> torch.Tensor:
    if not x.is_cuda:
        raise RuntimeError("SMoE runs on the sm_100a kernels only; move the input to CUDA")
    if x.dtype != torch.bfloat16:
        raise TypeError(f"SMoE expects bf16 activations, got {x.dtype}")
    return x.contiguous()


class Expert(nn.Module):
    """One expert FFN: fc2(act(fc1(x))) (baseline/infer.py:280-287)."""

    def __init__(self, d_model: int, dim_ff: int, activation: str = "gelu"):
        super().__init__()
        self.fc1 = nn.Linear(d_model, dim_ff)
        self.fc2 = nn.Linear(dim_ff, d_model)
        self.activation = activation

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = _prepare_x(x).reshape(-1, shape[-1])
        offs = torch.tensor([0, x2.shape[0]], dtype=torch.int32, device=x2.device)
        w1 = self.fc1.weight.detach().to(torch.bfloat16).unsqueeze(0).contiguous()
        w2 = self.fc2.weight.detach().to(torch.bfloat16).unsqueeze(0).contiguous()
        b1 = self.fc1.bias.detach().float().unsqueeze(0).contiguous()
        b2 = self.fc2.bias.detach().float().unsqueeze(0).contiguous()
        h = ops.grouped_gemm(x2, w1, b1, offs, act=self.activation)
        y = ops.grouped_gemm(h, w2, b2, offs, act="none")
        return y.reshape(*shape[:-1], y.shape[-1])


class TopKGate(nn.Module):
    """Top-2 router (baseline/infer.py:289-309; online_best/infer.py:1790-1852).

    ``forward(x[B,S,D])`` returns ``(topk_idx[B,S,2] int64, topk_score[B,S,2] fp32)``
    like the online_best gate; logits are computed in fp32."""

    def __init__(self, d_model: int, num_experts: int, k: int = 2, noisy_gating: bool = True,
                 renormalize: bool = True):
        super().__init__()
        if k != 2:
            raise ValueError("only Top-2 routing is implemented")
        if num_experts > _lib.MAX_EXPERTS:
            raise ValueError(f"at most {_lib.MAX_EXPERTS} experts are supported")
        self.w_g = nn.Linear(d_model, num_experts)
        self.num_experts = num_experts
        self.k = k
        self.noisy_gating = noisy_gating
        self.renormalize = renormalize

    def router_weights(self) -> tuple[torch.Tensor, torch.Tensor]:
        return (self.w_g.weight.detach().float().contiguous(),
                self.w_g.bias.detach().float().contiguous())

    def route(self, x2: torch.Tensor) -> ops.RouterOut:
        wg, bg = self.router_weights()
        return ops.router(x2, wg, bg, renorm=self.renormalize)

    def forward(self, x: torch.Tensor):
        shape = x.shape
        r = self.route(_prepare_x(x).reshape(-1, shape[-1]))
        return (r.idx2.long().reshape(*shape[:-1], 2), r.gate2.reshape(*shape[:-1], 2))


class SMoE(nn.Module):
    """Top-2 sparse MoE layer: router -> dispatch -> grouped expert FFN -> combine."""

    # forward_host's default chunk: measured on one B200 at cfg2 (72,214
    # tokens, two compute streams), 4,096 tokens per chunk beat 2,048-9,027.
    HOST_CHUNK_TOKENS = 4096

    def __init__(self, d_model: int, dim_ff: int, num_experts: int, k: int = 2,
                 activation: str = "gelu", renormalize: bool = True):
        super().__init__()
        if activation not in ("gelu", "relu"):
            raise ValueError("activation must be 'gelu' or 'relu'")
        self.num_experts = num_experts
        self.k = k
        self.d_model = d_model
        self.dim_ff = dim_ff
        self.activation = activation
        self.experts = nn.ModuleList(
            [Expert(d_model, dim_ff, activation) for _ in range(num_experts)])
        self.gate = TopKGate(d_model, num_experts, k=k, renormalize=renormalize)
        self._fused_ready = False
        self._workspace: torch.Tensor | None = None

    # -- weights ---------------------------------------------------------
    @torch.no_grad()
    def prepare_for_inference(self) -> None:
        """Stacks the expert weights in the nn.Linear [out, in] layout (K-major
        operands of the tensor-core GEMMs).  No pruning."""
        dev = self.gate.w_g.weight.device
        self._w1 = torch.stack([e.fc1.weight for e in self.experts]).to(dev, torch.bfloat16).contiguous()
        self._b1 = torch.stack([e.fc1.bias for e in self.experts]).to(dev, torch.float32).contiguous()
        self._w2 = torch.stack([e.fc2.weight for e in self.experts]).to(dev, torch.bfloat16).contiguous()
        self._b2 = torch.stack([e.fc2.bias for e in self.experts]).to(dev, torch.float32).contiguous()
        self._wg, self._bg = self.gate.router_weights()
        self._fused_ready = True

    def _ensure_ready(self, device: torch.device) -> None:
        if not self._fused_ready or self._w1.device != device:
            self.prepare_for_inference()

    def _get_workspace(self, T: int, device: torch.device, halves: int = 1) -> torch.Tensor:
        need = int(lib.cti_moe_layer_workspace_bytes(T, self.d_model, self.num_experts, self.dim_ff))
        if halves == 2:  # two layers in flight: a 256-byte aligned first half, then the second
            need += -(-need // 256) * 256
        ws = self._workspace
        if ws is None or ws.device != device or ws.numel() < need:
            ws = torch.empty(need, dtype=torch.uint8, device=device)
            self._workspace = ws
        return ws

    # -- forward ---------------------------------------------------------
    @torch.no_grad()
    def forward(self, x: torch.Tensor):
        B, S, D = x.shape
        x2 = _prepare_x(x).reshape(-1, D)
        T = x2.shape[0]
        dev = x2.device
        self._ensure_ready(dev)
        out = torch.empty_like(x2)
        if T > 0:
            ws = self._get_workspace(T, dev)
            check(
                lib.cti_moe_layer_forward(
                    ptr(x2), ptr(self._wg), ptr(self._bg), ptr(self._w1), ptr(self._b1),
                    ptr(self._w2), ptr(self._b2), T, D, self.num_experts, self.dim_ff,
                    _lib.ACTIVATIONS[self.activation], int(self.gate.renormalize), ptr(out),
                    ptr(ws), ws.numel(), ptr(status_word(dev)), stream_handle(dev),
                ),
                "cti_moe_layer_forward",
            )
        return out.reshape(B, S, D), None

    @torch.no_grad()
    def forward_host(self, x_host: torch.Tensor, out_host: torch.Tensor | None = None,
                     chunk_tokens: int | None = None, device: torch.device | None = None,
                     graph: bool = False):
        """``forward`` for activations in host memory: copies x to the GPU,
        runs the layer and copies the output back, pipelined over chunks of
        tokens (``cti_moe_layer_forward_host``) so that the two copies and
        the layer overlap; neighbouring chunks' layers run on two compute
        streams, so that they overlap too.  x_host [..., D] bf16 on the CPU (page-locked
        for the overlap); returns ``(out_host, None)`` with out_host a
        page-locked CPU tensor of the same shape, valid once the current
        stream of ``device`` is synchronised.  The result equals
        ``forward`` on the same rows bit for bit.

        ``graph=True`` (page-locked x_host and out_host): the first call with
        a given pair of buffers runs the pipeline and captures it in a CUDA
        graph; later calls with the same buffers (whatever their contents)
        and shapes replay it, without the host launching each chunk's copies
        and kernels again."""
        if x_host.is_cuda or x_host.dtype != torch.bfloat16 or x_host.shape[-1] != self.d_model:
            raise ValueError("x_host must be a CPU bf16 tensor [..., d_model]")
        if not x_host.is_contiguous():
            raise ValueError("x_host must be contiguous")
        dev = device or self.gate.w_g.weight.device
        if dev.type != "cuda":
            raise RuntimeError("forward_host needs the module on a CUDA device")
        dev = torch.device("cuda", dev.index if dev.index is not None else torch.cuda.current_device())
        self._ensure_ready(dev)
        D = self.d_model
        T = x_host.numel() // D
        if out_host is None:
            out_host = torch.empty(x_host.shape, dtype=torch.bfloat16, pin_memory=True)
        elif (out_host.shape != x_host.shape or out_host.dtype != torch.bfloat16
              or out_host.is_cuda or not out_host.is_contiguous()):
            raise ValueError("out_host must be a contiguous CPU bf16 tensor shaped like x_host")
        if T == 0:
            return out_host, None
        if chunk_tokens is None:
            # Small chunks shorten the pipeline's fill and drain; with two
            # layers in flight their fixed cost (~50 us per layer) stays
            # below the copies' time.
            chunk_tokens = self.HOST_CHUNK_TOKENS
        chunk = min(int(chunk_tokens), T)
        stage = getattr(self, "_host_stage", None)
        if stage is None or stage[0].device != dev or stage[0].numel() < T * D:
            stage = (torch.empty(T * D, dtype=torch.bfloat16, device=dev),
                     torch.empty(T * D, dtype=torch.bfloat16, device=dev))
            self._host_stage = stage
        streams = getattr(self, "_copy_streams", None)
        if streams is None or streams[0].device != dev:
            streams = (torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev))
            self._copy_streams = streams
        two = T > chunk
        ws = self._get_workspace(chunk, dev, halves=2 if two else 1)
        status = status_word(dev)

        def launch():
            check(
                lib.cti_moe_layer_forward_host(
                    ptr(x_host), ptr(out_host), ptr(stage[0]), ptr(stage[1]), ptr(self._wg),
                    ptr(self._bg), ptr(self._w1), ptr(self._b1), ptr(self._w2), ptr(self._b2),
                    T, D, self.num_experts, self.dim_ff, _lib.ACTIVATIONS[self.activation],
                    int(self.gate.renormalize), chunk, ptr(ws), ws.numel(), ptr(status),
                    stream_handle(dev), streams[0].cuda_stream, streams[1].cuda_stream,
                    streams[2].cuda_stream if two else None,
                ),
                "cti_moe_layer_forward_host",
            )

        if not graph:
            launch()
            return out_host, None
        if not (x_host.is_pinned() and out_host.is_pinned()):
            raise ValueError("graph=True needs page-locked x_host and out_host")
        key = (dev.index, T, chunk, ptr(x_host), ptr(out_host), ptr(stage[0]), ptr(stage[1]),
               ptr(ws), ptr(status), ptr(self._wg), ptr(self._w1), ptr(self._w2))
        graphs = getattr(self, "_host_graphs", None)
        if graphs is None:
            graphs = self._host_graphs = {}
        g = graphs.get(key)
        if g is not None:
            g.replay()
            return out_host, None
        launch()  # this call's result; also sets up every kernel before the capture
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            launch()
        if len(graphs) >= 4:  # keep the few most recent buffer pairs
            graphs.pop(next(iter(graphs)))
        graphs[key] = g
        return out_host, None

    @torch.no_grad()
    def forward_staged(self, x2: torch.Tensor, fused: bool | None = None):
        """The same layer as separate stage calls; returns every intermediate
        (used by the stage-by-stage parity tests)."""
        x2 = _prepare_x(x2)
        self._ensure_ready(x2.device)
        r = ops.router(x2, self._wg, self._bg, renorm=self.gate.renormalize)
        hist_copy = r.block_hist.clone()
        d = ops.dispatch(x2, r, self.num_experts)
        if fused is None:
            fused = self.d_model in (128, 256)
        if fused:
            y = ops.expert_ffn_fused(d.xperm, self._w1, self._b1, self._w2, self._b2, d.offsets,
                                     act=self.activation)
            h = None
        else:
            h = ops.grouped_gemm(d.xperm, self._w1, self._b1, d.offsets, act=self.activation)
            y = ops.grouped_gemm(h, self._w2, self._b2, d.offsets, act="none")
        out = ops.combine(y, d.perm_inv, r.gate2)
        return {"router": r, "block_hist": hist_copy, "dispatch": d, "hidden": h, "y": y,
                "out": out}
