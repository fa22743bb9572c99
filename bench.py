"""Benchmark of the B200 MoE hot path (one JSON line on rank 0).

Default workload (every N): configuration 2 - one Top-2 MoE layer, d_model
256, 16 experts, d_ff 1024, 512 packed samples with lengths U{16..256}
(T = 72,214 tokens for seed 0), bf16 activations and experts, fp32 router,
Zipf(1.2) expert bias.  A step is one SMoE forward over the whole packed
batch.  With N GPUs every rank runs its own replica on its own batch (the
layer does not shard at this size), so scaling is weak.

value  tokens/s of the whole job, inputs resident in HBM, device time from
       CUDA events (max over ranks), L2 flushed between steps.
e2e    the same through the public API with host buffers
       (SMoE.forward_host -> cti_moe_layer_forward_host): pinned host x ->
       device, the layer, output -> pinned host, all inside the timed region;
       the copies of one token chunk overlap the layer on its neighbours.
roofline  the dominant kernel (the expert FFN GEMM) timed alone with CUDA
       events: algorithmic FLOPs / mean launch time vs the measured bf16 peak.
router_fp32  the router's exact fp32 logits against the nominal fp32 FMA
       rate (its roofline: the FMA pipe, not HBM).
cpu_baseline  the reference's PyTorch CPU expert loop (oracle port of
       baseline/infer.py:280-358, fp32) on a bounded token sample, rank 0,
       N=1 only; cpu_baseline_cfg1 the same loop at configuration 1.
ep     configuration 5 at this N (expert parallelism over the N ranks, T =
       262,144 tokens in total, strong scaling): "even" is the
       configuration's even sharding of the 64 experts, "replicas" (N >= 2)
       the placement that replicates the heaviest experts.
e2e_model  configuration 4 at N = 1: the 8-layer CTR model forward, ms per
       batch, with inputs on the device and with the host copies.

Other workloads (--config): cfg3 the 28-feature embedding-bag pooling
(GB/s); cfg4 the whole CTR model forward (ms per batch); cfg5 the
expert-parallel layer (d_model 1024, 64 experts, d_ff 4096, 262,144 tokens
split over the N ranks: strong scaling).  --profile STAGE runs one stage of
the cfg2 workload alone for an ncu capture.

--impl reference times that CPU implementation alone on the same workload
(rank 0 only; other ranks exit without work).
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_FLUSH_BYTES = 256 << 20
CPU_SAMPLE_TOKENS = 8192
CALIBRATION_TOKENS = 65536
EP_STEPS, EP_WARMUP = 10, 3      # the cfg5 and cfg4 measurements of the default line
E2E_MODEL_STEPS = 5


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


FP32_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12  # 74.4


def ncu_traffic(kernel_key: str):
    """DRAM bytes per launch of a kernel from its committed ncu capture
    (profiles/dram_traffic.json), or None."""
    p = ROOT / "profiles" / "dram_traffic.json"
    try:
        return json.loads(p.read_text())[kernel_key]["traffic_bytes"]
    except (OSError, KeyError, ValueError):
        return None


def stage_bandwidths(stages_ms: dict, T: int, D: int, E: int, hbm_gbs: float) -> dict:
    """Algorithmic HBM bytes of the layer's memory-bound stages (bf16 rows,
    int32 indices, fp32 gates, 128-token router blocks) over their stage
    times: GB/s and the fraction of the measured copy bandwidth.  Stages
    missing from `stages_ms` are left out."""
    R = 2 * T
    nblk = -(-T // 128)
    row = 2 * D
    nbytes = {
        # x read; idx2, gate2 and route ranks written; per-block histograms written
        "router": T * row + T * 2 * (4 + 4 + 4) + nblk * E * 4,
        # scan: histograms read and rewritten; scatter: routes and ranks read, x read
        # once and written to both sorted slots, perm_inv and sorted_token written
        "dispatch": 2 * nblk * E * 4 + T * 2 * (4 + 4) + T * row + R * row + T * 2 * 4 + R * 4,
        # both expert rows of every token read, the output row written; perm_inv, gates read
        "combine": R * row + T * row + T * 2 * (4 + 4),
    }
    out = {}
    for name, b in nbytes.items():
        ms = stages_ms.get(name)
        if not ms:
            continue
        gbs = b / (ms / 1e3) / 1e9
        out[name] = {"bytes": b, "gbs": gbs, "frac_of_hbm": gbs / hbm_gbs}
    return out


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    """Samples nvidia-smi every 200 ms while the timed region runs and keeps
    the rows of this process's GPU (matched by UUID)."""
    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device: torch.device):
        self.proc = None
        self.file = None
        try:
            self.uuid = str(torch.cuda.get_device_properties(device).uuid).replace("GPU-", "")
        except Exception:
            self.uuid = ""

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader", "-lms",
                 "200"], stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        rows = [r for r in csv.reader(io.StringIO(self.file.read())) if len(r) >= 9]
        os.unlink(self.file.name)
        mine = [r for r in rows if self.uuid and self.uuid in r[0]]
        rows = mine or rows
        sm, smax, reasons = [], [], set()
        for r in rows:
            try:
                sm.append(float(r[1].strip().split()[0]))
                smax.append(float(r[2].strip().split()[0]))
            except (ValueError, IndexError):
                continue
            for name, v in zip(self.REASONS, r[5:9]):
                if v.strip() == "Active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax),
                "reasons": sorted(reasons), "samples": len(sm), "matched_uuid": bool(mine)}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v: float, world: int, dev) -> float:
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(v: float, world: int, dev) -> float:
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t)
    return float(t.item())


# ---------------------------------------------------------------------------
# CPU baseline (the oracle port of the reference's expert loop)
# ---------------------------------------------------------------------------
def load_synth():
    """The package's synth.py loaded on its own.  Importing it through the
    package would load libcti_b200.so, which the reference arm must never
    map: that arm runs only the reference's CPU code path."""
    import importlib.util

    name = "_cti_b200_synth_standalone"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(
        name, ROOT / "cti-inference-optimization_b200" / "synth.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def cpu_baseline_moe(cfg, seconds: float, sample_tokens: int | None = CPU_SAMPLE_TOKENS):
    """The oracle port of the reference's fp32 expert loop
    (baseline/infer.py:280-358) on all host cores, repeated for about
    `seconds`, on the first `sample_tokens` tokens of the configuration
    (all of them when None)."""
    from oracle import moe_ref as mr

    synth = load_synth()
    torch.set_num_threads(os.cpu_count() or 1)
    T, _ = synth.moe_tokens(cfg)
    S = T if sample_tokens is None else min(sample_tokens, T)
    w = synth.moe_weights(cfg.d_model, cfg.num_experts, cfg.dim_ff, cfg.zipf_bias)
    x = synth.moe_activations(T, cfg.d_model)[:S].float()
    w1, w2 = w.w1.float(), w.w2.float()
    with torch.no_grad():
        mr.smoe_ref(x, w.wg, w.bg, w1, w.b1, w2, w.b2)  # warm-up
        n = 0
        t0 = time.perf_counter()
        while True:
            mr.smoe_ref(x, w.wg, w.bg, w1, w.b1, w2, w.b2)
            n += 1
            el = time.perf_counter() - t0
            if (el >= seconds and n >= 2) or n >= 10000:
                break
    return {"value": n * S / el, "unit": "tokens/s", "cores": torch.get_num_threads(),
            "kind": "port", "config": cfg.name,
            "sample": f"{S} of the {T} {cfg.name} tokens per call, {n} calls "
                      f"({el:.1f} s), fp32, oracle/moe_ref.py (baseline/infer.py:280-358)"}


def cpu_baseline_embbag(bb, table_dev, seconds: float, sample_bags: int = 1024) -> dict:
    """The oracle port of the reference pooling (baseline/infer.py:253-263:
    per slot, emb(values.clamp) then segment_reduce(sum), fp32) on all host
    cores over the first `sample_bags` samples of the batch (all 28
    features), repeated for about `seconds`; GB/s of the sample's algorithmic
    bytes, counted as for the GPU line."""
    from oracle import embbag_ref as er

    torch.set_num_threads(os.cpu_count() or 1)
    F_, B = bb.features, bb.batch
    S = min(sample_bags, B)
    ro = bb.row_offsets.view(F_, B + 1)
    sub_ro = ro[:, :S + 1].contiguous()
    n_ids = int((sub_ro[:, -1] - sub_ro[:, 0]).sum())
    table = table_dev.cpu()
    args = (bb.values, sub_ro.view(-1), bb.val_offsets, table, bb.table_row_base, bb.vocab, F_)
    byts = 8 * n_ids + 8 * F_ * (S + 1) + 128 * n_ids + 4 * S * F_ * 64
    er.embbag_ref(*args)  # warm-up
    n = 0
    t0 = time.perf_counter()
    while True:
        er.embbag_ref(*args)
        n += 1
        el = time.perf_counter() - t0
        if (el >= seconds and n >= 2) or n >= 10000:
            break
    return {"value": n * byts / el / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port", "config": "cfg3",
            "sample": f"the first {S} of {B} samples, all {F_} features ({n_ids} ids) per call, "
                      f"{n} calls ({el:.1f} s), fp32, oracle/embbag_ref.py "
                      f"(baseline/infer.py:253-263)"}


def run_reference(args, world, rank):
    """--impl reference: the reference's CPU expert loop (the oracle port of
    baseline/infer.py:280-358, fp32, all host cores) over the whole
    configuration-2 batch, on rank 0 only.  It never loads this repository's
    library: synth.py is loaded on its own and the oracle is plain torch."""
    if rank != 0:
        return
    from oracle import moe_ref as mr

    synth = load_synth()
    cfg = synth.CFG2
    torch.set_num_threads(os.cpu_count() or 1)
    T, _ = synth.moe_tokens(cfg)
    w = synth.moe_weights(cfg.d_model, cfg.num_experts, cfg.dim_ff, cfg.zipf_bias)
    x = synth.moe_activations(T, cfg.d_model).float()
    w1, w2 = w.w1.float(), w.w2.float()
    times = []
    with torch.no_grad():
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            mr.smoe_ref(x, w.wg, w.bg, w1, w.b1, w2, w.b2)
            if i >= args.warmup:
                times.append(time.perf_counter() - t0)
    step = statistics.mean(times)
    value = T / step
    line = {
        "impl": "reference", "metric": "moe_layer_tokens_per_s", "value": value,
        "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": step * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(cfg, T),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": f"all {T} tokens per step (oracle/moe_ref.py, the "
                                   f"reference's fp32 expert loop, baseline/infer.py:280-358)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(cfg, T):
    """The `config` object of the cfg2 line; both arms print the same one."""
    return {"workload": f"{cfg.name}: Top-2 MoE layer, d_model {cfg.d_model}, "
                        f"{cfg.num_experts} experts, d_ff {cfg.dim_ff}, {cfg.samples} packed "
                        f"samples U{{16..256}}",
            "tokens": T, "d_model": cfg.d_model, "experts": cfg.num_experts, "d_ff": cfg.dim_ff,
            "router_bias": "zipf(1.2)", "activation": "gelu", "gates": "renormalised",
            "l2": "flushed (256 MiB write) before every timed step",
            "per_gpu": "one replica"}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def device_wait(dev, ms: float = 1.0) -> None:
    """Parks the stream for about `ms` (a spin kernel) so the host enqueues
    the next step while the device waits; the step's events then time device
    execution only, not host launch latency."""
    torch.cuda._sleep(int(ms * 2.0e6))


def time_steps(fn, steps, flush, dev, hide_host=True):
    """Per-step device time (ms) of fn(), L2 flushed before each step outside
    the event pair."""
    times = []
    for _ in range(steps):
        flush.zero_()
        if hide_host:
            device_wait(dev)
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        times.append((s, e))
    torch.cuda.synchronize(dev)
    return [s.elapsed_time(e) for s, e in times]


def stage_times(m, x2, flush, dev, reps=10):
    """Median device time (ms) of each stage launched on its own: every stage
    runs once untimed first (module loading), and each timed launch sits
    behind an L2 flush and a device wait that hides the host enqueue."""
    from cti_b200 import ops

    fused = m.d_model in (128, 256)
    acc = {}

    def timed(name, fn, record=True):
        flush.zero_()
        device_wait(dev, 1.0)
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        out = fn()
        e.record()
        if record:
            acc.setdefault(name, []).append((s, e))
        return out

    for rep in range(reps + 1):
        rec = rep > 0
        r = timed("router", lambda: ops.router(x2, m._wg, m._bg, renorm=True), rec)
        d = timed("dispatch", lambda: ops.dispatch(x2, r, m.num_experts), rec)
        y = None
        if fused:
            y = timed("ffn_fused", lambda: ops.expert_ffn_fused(
                d.xperm, m._w1, m._b1, m._w2, m._b2, d.offsets, act="gelu"), rec)
        h = timed("ffn_fc1", lambda: ops.grouped_gemm(d.xperm, m._w1, m._b1, d.offsets,
                                                      act="gelu"), rec)
        y2 = timed("ffn_fc2", lambda: ops.grouped_gemm(h, m._w2, m._b2, d.offsets, act="none"),
                   rec)
        timed("combine", lambda: ops.combine(y if fused else y2, d.perm_inv, r.gate2), rec)
    torch.cuda.synchronize(dev)
    return {n: statistics.median(s.elapsed_time(e) for s, e in v) for n, v in acc.items()}


def run_ours(args, world, rank, local):
    import cti_b200
    from cti_b200 import _lib, synth

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = synth.CFG2
    T, cu = synth.moe_tokens(cfg, seed=0)
    w = synth.moe_weights(cfg.d_model, cfg.num_experts, cfg.dim_ff, cfg.zipf_bias, seed=0,
                          device=dev)
    m = cti_b200.SMoE(cfg.d_model, cfg.dim_ff, cfg.num_experts).to(dev)
    synth.load_moe_module(m, w)
    m.prepare_for_inference()
    x = synth.moe_activations(T, cfg.d_model, seed=rank, device=dev)
    x3 = x.unsqueeze(0)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    for _ in range(args.warmup):
        m(x3)
    torch.cuda.synchronize(dev)
    _lib.raise_on_status(dev)

    sampler = ClockSampler(dev) if rank == 0 else None
    barrier(world)
    torch.cuda.synchronize(dev)
    if sampler:
        sampler.start()
    times = time_steps(lambda: m(x3), args.steps, flush, dev)
    torch.cuda.synchronize(dev)
    barrier(world)
    clocks = sampler.stop() if sampler else None
    _lib.raise_on_status(dev)
    step_ms = max_over_ranks(statistics.mean(times), world, dev)
    tokens_all = sum_over_ranks(float(T), world, dev)
    value = tokens_all / (step_ms / 1e3)

    # End to end through the public API with host buffers: SMoE.forward_host
    # (cti_moe_layer_forward_host) copies x in, runs the layer and copies the
    # output back, chunk by chunk, with the copies overlapping the layer.
    x_h = x.cpu().pin_memory()
    out_h = torch.empty_like(x_h).pin_memory()

    def e2e_step():
        # The pipeline's copies and kernels, captured in a CUDA graph on the
        # first (warm-up) call and replayed on the same page-locked buffers.
        m.forward_host(x_h, out_h, graph=True)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    barrier(world)
    torch.cuda.synchronize(dev)
    e2e_times = time_steps(e2e_step, args.steps, flush, dev, hide_host=False)
    barrier(world)
    e2e_ms = max_over_ranks(statistics.mean(e2e_times), world, dev)
    e2e_value = tokens_all / (e2e_ms / 1e3)

    stages = stage_times(m, x, flush, dev)
    peaks, peak_src = load_peaks()
    R = 2 * T
    gemm_flops = 2.0 * R * cfg.d_model * cfg.dim_ff  # one of the two expert GEMMs
    if "ffn_fused" in stages:
        dom, dom_flops = "ffn_fused", 2 * gemm_flops
        launches_per_step = 5
    else:
        dom = "ffn_fc1" if stages["ffn_fc1"] >= stages["ffn_fc2"] else "ffn_fc2"
        dom_flops = gemm_flops
        launches_per_step = 6
    achieved = dom_flops / (stages[dom] / 1e3) / 1e12
    peak = float(peaks["bf16_tflops"])
    kernel_names = {"ffn_fused": "fused_ffn_kernel", "ffn_fc1": "grouped_gemm_kernel (fc1)",
                    "ffn_fc2": "grouped_gemm_kernel (fc2)"}

    # Configuration 5 at this N (expert parallelism, strong scaling): the
    # configuration's even sharding, and from N = 2 on the placement with
    # replicas of the heaviest experts beside it.
    ep = None
    if not args.no_ep:
        ep = {"config": cfg5_config(world),
              "even": measure_ep(args, world, rank, local, flush, "contiguous", EP_STEPS,
                                 EP_WARMUP)}
        if world > 1:
            ep["replicas"] = measure_ep(args, world, rank, local, flush, "balanced", EP_STEPS,
                                        EP_WARMUP)
    # Configuration 4 at N = 1: the 8-layer CTR model forward, ms per batch.
    e2e_model = None
    if world == 1 and not args.no_e2e_model:
        r4 = measure_e2e_model(args, world, rank, local, flush, E2E_MODEL_STEPS, EP_WARMUP)
        e2e_model = {"metric": "e2e_forward_ms_per_batch", "unit": "ms/batch",
                     "value": r4["ms_per_batch"], "config": cfg4_config(r4["tokens"], r4["ids"]),
                     "with_host_copies": {"value": r4["e2e_ms_per_batch"], "unit": "ms/batch",
                                          "h2d_bytes_per_step": r4["h2d_bytes_per_step"],
                                          "d2h_bytes_per_step": r4["d2h_bytes_per_step"],
                                          "chunks": r4["chunks"]},
                     "stages_ms": r4["stages_ms"], "tokens_per_s": r4["tokens_per_s"],
                     "expert_ffn_roofline": r4["roofline"], "pooling": r4["pooling"],
                     "rep_encoder": r4["rep_encoder"],
                     "attention_kernel": r4["attention_kernel"],
                     "steps": E2E_MODEL_STEPS, "warmup": EP_WARMUP}

    if rank != 0:
        return
    cpu = cpu1 = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_moe(cfg, args.cpu_seconds)
        # Configuration 1, the reference's CPU expert loop at its own shape
        # (T 4096, d_model 128, 8 experts, d_ff 512): the named CPU baseline.
        cpu1 = cpu_baseline_moe(synth.CFG1, min(args.cpu_seconds, 5.0), sample_tokens=None)
    line = {
        "metric": "moe_layer_tokens_per_s", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": workload_config(cfg, T),
        "timing": "value: device time per step (CUDA events), host enqueue hidden behind a "
                  "device-side wait before each step; e2e: host copies and enqueue included",
        "e2e": {"value": e2e_value, "unit": "tokens/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": x_h.numel() * x_h.element_size(),
                "d2h_bytes_per_step": out_h.numel() * out_h.element_size()},
        "roofline": {"bound": "tensor", "kernel": kernel_names[dom],
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_source": f"bf16_tflops of {peak_src}",
                     "flops_per_launch": dom_flops,
                     "traffic": ncu_traffic("fused_ffn_kernel<256> cfg2") if dom == "ffn_fused"
                     else None,
                     "traffic_source": "profiles/dram_traffic.json (one ncu capture of a "
                                       "launch of this workload)"},
        "layer_roofline_frac": (2 * gemm_flops * world / (step_ms / 1e3) / 1e12 / world) / peak,
        "stages_ms": stages,
        "stages_hbm": stage_bandwidths(stages, T, cfg.d_model, cfg.num_experts,
                                       float(peaks["hbm_gbs"])),
        # The router's exact fp32 logits run on the FMA pipe: T*E*D FMAs
        # against the nominal fp32 rate (148 SMs x 128 lanes x 2 FLOP at
        # 1.965 GHz), which alone needs 69 % of its HBM time at cfg2.
        "router_fp32": {"flops": 2.0 * T * cfg.num_experts * cfg.d_model,
                        "tflops": 2.0 * T * cfg.num_experts * cfg.d_model
                        / (stages["router"] / 1e3) / 1e12,
                        "peak_tflops": FP32_NOMINAL_TFLOPS,
                        "frac": 2.0 * T * cfg.num_experts * cfg.d_model
                        / (stages["router"] / 1e3) / 1e12 / FP32_NOMINAL_TFLOPS,
                        "peak_source": "nominal (148 SMs x 128 FP32 lanes x 2 FLOP x 1.965 GHz)"},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
        "cpu_baseline": cpu,
        "cpu_baseline_cfg1": cpu1,
        "ep": ep,
        "e2e_model": e2e_model,
    }
    print(json.dumps(line), flush=True)


def measure_ep(args, world, rank, local, flush, placement_kind: str, steps: int, warmup: int,
               sampler=None) -> dict:
    """Configuration 5 on the expert-parallel layer (d_model 1024, 64
    experts, d_ff 4096) over T = 262,144 tokens in total, split evenly across
    the N ranks (strong scaling).  placement_kind "contiguous": rank r owns
    experts [r*64/N, (r+1)*64/N), the configuration's even sharding;
    "balanced": slots placed by routing counts of a separate calibration
    batch, with replicas of the heaviest experts from N = 4 on.  Every rank
    calls this with the same arguments (collectives inside); the returned
    dict is complete on rank 0."""
    from cti_b200 import _lib, ops, synth
    from cti_b200.ep import ExpertParallelSMoE, balanced_placement

    dev = torch.device("cuda", local)
    cfg = synth.CFG5
    T = cfg.tokens
    D, E, F = cfg.d_model, cfg.num_experts, cfg.dim_ff
    w = synth.moe_weights(D, E, F, cfg.zipf_bias, seed=0, device=dev)
    placement = None
    if placement_kind == "balanced" and world > 1:
        # Calibrate on a separate batch (seed 1): its routing counts, summed
        # over the ranks, give each expert's expected load.
        xc = synth.moe_activations(CALIBRATION_TOKENS, D, seed=1, device=dev)
        rc = ops.router(xc, w.wg.float().contiguous(), w.bg.float().contiguous())
        load = torch.bincount(rc.idx2.reshape(-1).long(), minlength=E).to(torch.float64)
        import torch.distributed as dist

        dist.all_reduce(load)
        extra = args.ep_extra_slots
        if extra < 0:  # replicate only where one expert would bound a rank
            extra = 0 if world <= 2 else max(2, E // world // 2)
        placement = balanced_placement(load.tolist(), world, E // world + extra)
        del xc, rc
    m = ExpertParallelSMoE(D, F, E, placement=placement).to(dev)
    m.load_weights(w.wg, w.bg, w.w1, w.b1, w.w2, w.b2)
    m.prepare_for_inference()
    del w
    lo, hi = rank * T // world, (rank + 1) * T // world
    x = synth.moe_activations(T, D, seed=0, device=dev)[lo:hi].clone()
    torch.cuda.empty_cache()
    overlap = args.ep_exchange == "p2p"

    for _ in range(warmup):
        m(x, overlap=overlap)
    torch.cuda.synchronize(dev)
    _lib.raise_on_status(dev)
    barrier(world)
    torch.cuda.synchronize(dev)
    if sampler:
        sampler.start()
    times = time_steps(lambda: m(x, overlap=overlap), steps, flush, dev)
    torch.cuda.synchronize(dev)
    barrier(world)
    clocks = sampler.stop() if sampler else None
    _lib.raise_on_status(dev)
    step_ms = max_over_ranks(statistics.mean(times), world, dev)

    # End to end: this rank's tokens from pinned host memory, output back.
    x_h = x.cpu().pin_memory()
    out_h = torch.empty_like(x_h).pin_memory()
    x_d = torch.empty_like(x)

    def e2e_step():
        x_d.copy_(x_h, non_blocking=True)
        out, _ = m(x_d, overlap=overlap)
        out_h.copy_(out, non_blocking=True)

    for _ in range(max(1, warmup)):
        e2e_step()
    barrier(world)
    torch.cuda.synchronize(dev)
    e2e_times = time_steps(e2e_step, steps, flush, dev, hide_host=False)
    barrier(world)
    e2e_ms = max_over_ranks(statistics.mean(e2e_times), world, dev)

    # Stage split (CUDA events between the stages of one forward), median of
    # a few forwards, per rank; rows = rows this rank's experts computed.
    names = ["router", "dispatch", "exchange", "experts", "exchange_back", "combine"]
    per = {n: [] for n in names}
    for _ in range(5):
        flush.zero_()
        evs = [torch.cuda.Event(enable_timing=True)]
        evs[0].record()

        def mark(name, evs=evs):
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            evs.append(e)

        m(x, mark=mark, overlap=overlap)
        torch.cuda.synchronize(dev)
        for n, a, b in zip(names, evs[:-1], evs[1:]):
            per[n].append(a.elapsed_time(b))
    stages = {n: statistics.median(v) for n, v in per.items()}
    r = ops.router(x, m._wg, m._bg)
    cnt = torch.bincount(r.idx2.reshape(-1).long(), minlength=E).to(torch.float64)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(cnt)
    S = m.slots_per_rank
    nrep = torch.tensor([m.n_rep[e] for e in m.placement], dtype=torch.float64, device=dev)
    pos = torch.tensor([m.position[e] for e in m.placement], device=dev)  # router outputs
    share = cnt[pos] / nrep                                               # are dispatch positions
    rows_per_rank = share.view(world, S).sum(dim=1).tolist()
    rows_local = rows_per_rank[rank]
    exp_ms = torch.tensor([stages["experts"]], dtype=torch.float64, device=dev)
    if world > 1:
        import torch.distributed as dist

        gathered = [torch.empty_like(exp_ms) for _ in range(world)]
        dist.all_gather(gathered, exp_ms)
        experts_ms = [float(t.item()) for t in gathered]
    else:
        experts_ms = [stages["experts"]]
    flops_local = 4.0 * rows_local * D * F
    achieved = flops_local / (stages["experts"] / 1e3) / 1e12
    peaks, peak_src = load_peaks()
    peak = float(peaks["bf16_tflops"])
    total_flops = 4.0 * 2 * T * D * F
    exchange_ms = stages["exchange"] + stages["exchange_back"]
    del m, x, x_d
    torch.cuda.empty_cache()
    return {
        "tokens_per_s": T / (step_ms / 1e3), "ms_per_step": step_ms,
        "e2e_tokens_per_s": T / (e2e_ms / 1e3), "e2e_ms_per_step": e2e_ms,
        "h2d_bytes_per_step": x_h.numel() * x_h.element_size() * world,
        "d2h_bytes_per_step": out_h.numel() * out_h.element_size() * world,
        "placement": ("contiguous (even sharding, E/N experts per rank)" if placement is None else
                      f"balanced (LPT over the routing counts of a separate "
                      f"{CALIBRATION_TOKENS}-token calibration batch), "
                      f"{len(placement) // world} slots per rank, {len(placement) - E} replicas"),
        "exchange": ("none (one rank)" if world == 1 else
                     "counts: NCCL all_to_all_single; rows: NCCL point-to-point per peer, "
                     "overlapped with the experts over the rows a rank routes to itself; "
                     "results back the same way" if overlap else
                     "NCCL all_to_all_single (counts, then rows with uneven splits; the same "
                     "back)"),
        "stages_ms_rank0": stages,
        "exchange_share_rank0": exchange_ms / max(sum(stages.values()), 1e-9),
        "rows_per_rank": rows_per_rank,
        "experts_ms_per_rank": experts_ms,
        "experts_roofline_rank0": {"kernel": "grouped_gemm_kernel (fc1 + fc2)",
                                   "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                                   "frac": achieved / peak,
                                   "peak_source": f"bf16_tflops of {peak_src}",
                                   "flops": flops_local},
        "layer_roofline_frac": total_flops / (step_ms / 1e3) / 1e12 / world / peak,
        "clocks": clocks,
    }


def cfg5_config(world: int) -> dict:
    from cti_b200 import synth

    cfg = synth.CFG5
    return {"workload": f"cfg5: expert-parallel Top-2 MoE layer, d_model {cfg.d_model}, "
                        f"{cfg.num_experts} experts, d_ff {cfg.dim_ff}, {cfg.tokens} tokens in "
                        "total split evenly over the ranks",
            "tokens": cfg.tokens, "d_model": cfg.d_model, "experts": cfg.num_experts,
            "d_ff": cfg.dim_ff, "parallelism": f"ep{world}", "router_bias": "zipf(1.2)",
            "activation": "gelu", "gates": "renormalised",
            "l2": "flushed (256 MiB write) before every timed step"}


def run_ep(args, world, rank, local):
    """--config cfg5: the expert-parallel layer alone (strong scaling over N;
    N = 1 is the single-GPU baseline, no exchange)."""
    from cti_b200 import synth

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    sampler = ClockSampler(dev) if rank == 0 else None
    r = measure_ep(args, world, rank, local, flush, args.placement, args.steps, args.warmup,
                   sampler)
    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_moe(synth.CFG5, args.cpu_seconds, sample_tokens=1024)
    cfg = cfg5_config(world)
    cfg["placement"] = r["placement"]
    cfg["exchange"] = r["exchange"]
    line = {
        "metric": "moe_layer_tokens_per_s", "value": r["tokens_per_s"], "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": cfg,
        "e2e": {"value": r["e2e_tokens_per_s"], "unit": "tokens/s",
                "ms_per_step": r["e2e_ms_per_step"],
                "h2d_bytes_per_step": r["h2d_bytes_per_step"],
                "d2h_bytes_per_step": r["d2h_bytes_per_step"]},
        "roofline": dict(r["experts_roofline_rank0"], bound="tensor", traffic=None),
        "layer_roofline_frac": r["layer_roofline_frac"],
        "stages_ms_rank0": r["stages_ms_rank0"],
        "exchange_share_rank0": r["exchange_share_rank0"],
        "rows_per_rank": r["rows_per_rank"],
        "experts_ms_per_rank": r["experts_ms_per_rank"],
        "gpu_launches": 6 * args.steps,
        "clocks": r["clocks"],
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


E2E_CHUNKS = 8  # sequence groups of the cfg4 host pipeline


def measure_e2e_model(args, world, rank, local, flush, steps: int, warmup: int,
                      sampler=None, cpu_seconds: float = 0.0) -> dict:
    """Configuration 4: the full CTR model forward (pooling -> RepEncoder ->
    8 x (attention + MoE) -> MLP head) on one packed batch of 2048 sequences,
    ms per batch, with inputs resident on the device and end to end from
    pinned host buffers (CTRModel.predict_host).  Every rank runs its own
    replica (the model does not shard).  cpu_seconds > 0 also times the
    oracle on a sample (rank 0)."""
    from cti_b200 import _lib, ops, synth
    from cti_b200.model import build_ctr_model

    dev = torch.device("cuda", local)
    bb, uo, T = synth.cfg4_batch(seed=rank)
    model = build_ctr_model(bb.vocab.tolist())
    synth.init_ctr_model(model)
    model.rep_encoder.emb.weight = torch.nn.Parameter(torch.empty(0), requires_grad=False)
    model.to(dev)
    model.rep_encoder.emb.weight = torch.nn.Parameter(
        synth.embedding_table(bb.total_rows, 64, seed=rank, device=dev), requires_grad=False)
    model.prepare_for_inference()
    host = {"_flat_values": bb.values, "_flat_row_offsets": bb.row_offsets,
            "_val_offsets": bb.val_offsets, "user_offsets": uo}
    batch = {k: v.to(dev) for k, v in host.items()}
    batch["max_seqlen"] = 256

    for _ in range(warmup):
        model.predict(batch)
    torch.cuda.synchronize(dev)
    _lib.raise_on_status(dev)
    barrier(world)
    torch.cuda.synchronize(dev)
    if sampler:
        sampler.start()
    times = time_steps(lambda: model.predict(batch), steps, flush, dev)
    torch.cuda.synchronize(dev)
    barrier(world)
    clocks = sampler.stop() if sampler else None
    _lib.raise_on_status(dev)
    step_ms = max_over_ranks(statistics.median(times), world, dev)

    # End to end: pinned host ids/offsets -> device, forward, probabilities ->
    # host, through CTRModel.predict_host: the sequences go in E2E_CHUNKS
    # groups, each group's copy overlapping the previous group's forward.
    pinned = {k: v.pin_memory() for k, v in host.items()}
    probs_h = torch.empty(T, dtype=torch.float32).pin_memory()

    def e2e_step():
        model.predict_host(pinned, chunks=E2E_CHUNKS, out=probs_h)

    for _ in range(max(1, warmup)):
        e2e_step()
    barrier(world)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(statistics.median(time_steps(e2e_step, steps, flush, dev,
                                                         hide_host=False)), world, dev)

    # Stage split of one forward (CUDA events), median of 3.
    enc = model.seq_encoder
    stage = {"rep_encoder": [], "attention": [], "moe": [], "head": []}
    for _ in range(3):
        flush.zero_()
        evs = []

        def mark(name):
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            evs.append((name, e))

        mark("start")
        x = model.rep_encoder(batch)
        mark("rep_encoder")
        cu = batch["user_offsets"].to(torch.int32)
        h, _ = enc(x, {"cu_seqlens": cu, "max_seqlen": 256, "mark": mark})
        model.head(h)
        mark("head")
        torch.cuda.synchronize(dev)
        acc = {k: 0.0 for k in stage}
        for (_, a), (name, b) in zip(evs[:-1], evs[1:]):
            acc[name] += a.elapsed_time(b)
        for k in stage:
            stage[k].append(acc[k])
    stages = {k: statistics.median(v) for k, v in stage.items()}

    # Roofline of the largest kernel, the fused expert FFN (one launch per
    # layer): timed alone on the first layer's routed rows of this batch.
    moe0 = enc.moe[0]
    x0 = model.rep_encoder(batch)
    r0 = ops.router(x0, moe0._wg, moe0._bg)
    d0 = ops.dispatch(x0, r0, moe0.num_experts)
    y0 = torch.empty_like(d0.xperm)
    ffn = lambda: ops.expert_ffn_fused(d0.xperm, moe0._w1, moe0._b1, moe0._w2, moe0._b2,
                                       d0.offsets, out=y0)
    ffn()
    ffn_ms = statistics.median(time_steps(ffn, 5, flush, dev))
    ffn_flops = 4.0 * (2 * T) * enc.d_model * moe0.dim_ff
    peaks, peak_src = load_peaks()
    ffn_tflops = ffn_flops / (ffn_ms / 1e3) / 1e12
    # The RepEncoder: the model's path (the stage above: pooling kernel
    # writing [T, 1792] bf16, LayerNorm kernel, cuBLAS Linear) against the
    # fused kernel timed alone; and the pooling kernel against HBM
    # (algorithmic bytes; Zipf ids re-hit rows in L2).
    rep = model.rep_encoder
    pool = lambda: rep.pool(batch, out_dtype=torch.bfloat16)
    pool()
    pool_ms = statistics.median(time_steps(pool, 3, flush, dev))

    fused = lambda: rep.forward_fused(batch)
    fused()
    fused_ms = statistics.median(time_steps(fused, 3, flush, dev))
    N = bb.values.numel()
    pool_bytes = 8 * N + 8 * 28 * (T + 1) + 128 * N + 2 * T * 28 * 64
    pool_gbs = pool_bytes / (pool_ms / 1e3) / 1e9
    # The attention kernel alone on layer 0's q, k, v of this batch, times the
    # layer count (the "attention" stage also holds the qkv and output
    # projections and the two add + LayerNorm launches).
    layer0 = enc.norm1[0]
    _, h0 = ops.add_layernorm(x0, None, layer0.weight, layer0.bias, layer0.eps)
    qkv0 = torch.nn.functional.linear(h0, *enc._qkv[0]).view(T, 3, enc.n_heads, enc.head_dim)
    cu0 = batch["user_offsets"].to(torch.int32)
    att = lambda: ops.varlen_attention(qkv0[:, 0], qkv0[:, 1], qkv0[:, 2], cu0, 256)
    att()
    att_ms = statistics.median(time_steps(att, 5, flush, dev))
    cpu = None
    if rank == 0 and cpu_seconds > 0:
        cpu = cpu_baseline_e2e(model, bb, uo, cpu_seconds)
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    out = {
        "ms_per_batch": step_ms, "tokens": T, "ids": N,
        "e2e_ms_per_batch": e2e_ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": T * 4,
        "chunks": E2E_CHUNKS,
        "roofline": {"bound": "tensor", "kernel": "fused expert FFN (one layer, timed alone)",
                     "achieved": ffn_tflops, "peak": float(peaks["bf16_tflops"]),
                     "unit": "TFLOP/s", "frac": ffn_tflops / float(peaks["bf16_tflops"]),
                     "peak_source": f"bf16_tflops of {peak_src}", "flops_per_launch": ffn_flops,
                     "ms_per_launch": ffn_ms, "traffic": None},
        "pooling": {"kernel": "embbag_kernel<64, bf16>", "ms": pool_ms,
                    "algorithmic_gbs": pool_gbs, "bytes_per_launch": pool_bytes,
                    "note": "algorithmic bytes (128 B per id) over time; Zipf ids re-hit rows "
                            "in L2, so this exceeds the HBM copy bandwidth"},
        "rep_encoder": {"stage_ms": stages["rep_encoder"],
                        "path": "pooling kernel -> [T, 1792] bf16 -> LayerNorm kernel -> "
                                "cuBLAS Linear",
                        "fused_ms": fused_ms,
                        "fused": "cti_rep_encoder_fused, timed alone (pooling, LayerNorm "
                                 "folded into the Linear, no [T, 1792] in HBM)"},
        "attention_kernel": {"ms_per_layer": att_ms, "ms_per_batch": att_ms * enc.num_layers,
                             "kernel": "varlen_attention_kernel (tcgen05)"},
        "stages_ms": stages, "tokens_per_s": T / (step_ms / 1e3),
        # Ours per batch: pooling and LayerNorm, per layer 2 add + LayerNorm,
        # the attention and the MoE chain of 5, and the head.
        "launches_per_batch": 3 + 8 * enc.num_layers, "clocks": clocks, "cpu_baseline": cpu,
    }
    del model, batch, pinned
    torch.cuda.empty_cache()
    return out


def cfg4_config(T: int, N: int) -> dict:
    from cti_b200 import synth

    return {"workload": f"cfg4: CTR model forward, {synth.CFG4_SAMPLES} packed sequences "
                        f"U{{16..256}} ({T} tokens), 28 bags per token, RepEncoder "
                        "LN(1792)+Linear(1792->256), 8 x (varlen causal attention 8x32 + "
                        "Top-2 MoE 16 experts d_ff 1024), MLP head 256->128->1",
            "tokens": T, "ids": N, "layers": 8,
            "attention": "cti_varlen_attention (this library)",
            "l2": "flushed (256 MiB write) before every timed step", "per_gpu": "one replica"}


def run_e2e(args, world, rank, local):
    """--config cfg4: the full CTR model forward alone; metric = ms per batch."""
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    sampler = ClockSampler(dev) if rank == 0 else None
    r = measure_e2e_model(args, world, rank, local, flush, args.steps, args.warmup, sampler,
                          cpu_seconds=0.0 if (world > 1 or args.no_cpu_baseline)
                          else args.cpu_seconds)
    if rank != 0:
        return
    line = {
        "metric": "e2e_forward_ms_per_batch", "value": r["ms_per_batch"], "unit": "ms/batch",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": r["ms_per_batch"], "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": cfg4_config(r["tokens"], r["ids"]),
        "e2e": {"value": r["e2e_ms_per_batch"], "unit": "ms/batch",
                "h2d_bytes_per_step": r["h2d_bytes_per_step"],
                "d2h_bytes_per_step": r["d2h_bytes_per_step"], "chunks": r["chunks"]},
        "roofline": r["roofline"], "pooling": r["pooling"], "stages_ms": r["stages_ms"],
        "rep_encoder": r["rep_encoder"], "attention_kernel": r["attention_kernel"],
        "tokens_per_s": r["tokens_per_s"],
        "gpu_launches": r["launches_per_batch"] * args.steps,
        "clocks": r["clocks"], "cpu_baseline": r["cpu_baseline"],
    }
    print(json.dumps(line), flush=True)


def cpu_baseline_e2e(model, bb, uo, seconds: float, sample_seqs: int = 2):
    """The oracle (fp32 CPU restatement of the reference model) on the first
    `sample_seqs` sequences of the batch, scaled to the whole batch by
    tokens."""
    from cti_b200 import synth
    from oracle import e2e_ref

    torch.set_num_threads(os.cpu_count() or 1)
    T = int(uo[-1])
    t_s = int(uo[sample_seqs])
    F_ = 28
    offs = bb.row_offsets.view(F_, T + 1)[:, :t_s + 1]
    vals, voff = [], []
    start = 0
    for f in range(F_):
        v0 = int(bb.val_offsets[f])
        n = int(offs[f, -1])
        vals.append(bb.values[v0:v0 + n])
        voff.append(start)
        start += n
    batch = {"_flat_values": torch.cat(vals), "_flat_row_offsets": offs.reshape(-1).clone(),
             "_val_offsets": torch.tensor(voff, dtype=torch.int64),
             "user_offsets": uo[:sample_seqs + 1].clone()}
    sd = {k: v.detach().float().cpu() for k, v in model.state_dict().items()}
    kw = dict(slot_num=28, n_heads=8, num_layers=8, num_experts=16,
              table_row_base=bb.table_row_base, vocab=bb.vocab)
    e2e_ref.ctr_forward_ref(sd, batch, **kw)  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        e2e_ref.ctr_forward_ref(sd, batch, **kw)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds or n >= 1000:
            break
    per_call = el / n
    return {"value": per_call * (T / t_s) * 1e3, "unit": "ms/batch",
            "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{sample_seqs} of {synth.CFG4_SAMPLES} sequences ({t_s} of {T} tokens), "
                      f"{n} calls ({el:.1f} s), scaled to the batch by tokens; fp32, "
                      "oracle/e2e_ref.py (baseline/infer.py:244-439)"}


def run_profile_workload(args):
    """--profile STAGE: the configuration-2 workload with one stage launched
    warmup + steps times and nothing else timed; the small, self-contained
    command the ncu captures under profiles/ are taken on."""
    import cti_b200
    from cti_b200 import _lib, ops, synth

    dev = torch.device("cuda", 0)
    if args.profile == "embbag":
        bb = synth.bag_batch(batch=4096, seed=0)
        table = synth.embedding_table(bb.total_rows, 64, seed=0, device=dev)
        a = [bb.values.to(dev), bb.row_offsets.to(dev), bb.val_offsets.to(dev), table,
             bb.table_row_base.to(dev), bb.vocab.to(dev), bb.features]
        for _ in range(args.warmup + args.steps):
            ops.embedding_bag_sum(*a)
        torch.cuda.synchronize(dev)
        _lib.raise_on_status(dev)
        print(f"profile workload embbag: {bb.values.numel()} ids")
        return
    if args.profile == "attention":
        # Configuration 4's attention: 2048 packed sequences U{16..256}, 8
        # heads of 32, q/k/v the thirds of one [T, 768] projection output.
        lens = synth.packed_lengths(synth.CFG4_SAMPLES, 16, 256, 0)
        cu = synth.cu_seqlens(lens).to(dev)
        T = int(lens.sum())
        g = torch.Generator(device=dev).manual_seed(0)
        qkv = torch.randn(T, 768, generator=g, device=dev).bfloat16().view(T, 3, 8, 32)
        for _ in range(args.warmup + args.steps):
            ops.varlen_attention(qkv[:, 0], qkv[:, 1], qkv[:, 2], cu, 256)
        torch.cuda.synchronize(dev)
        _lib.raise_on_status(dev)
        print(f"profile workload attention: T={T}, {args.warmup + args.steps} launches")
        return
    cfg = synth.CFG2
    T, _ = synth.moe_tokens(cfg)
    w = synth.moe_weights(cfg.d_model, cfg.num_experts, cfg.dim_ff, cfg.zipf_bias, device=dev)
    m = cti_b200.SMoE(cfg.d_model, cfg.dim_ff, cfg.num_experts).to(dev)
    synth.load_moe_module(m, w)
    m.prepare_for_inference()
    x = synth.moe_activations(T, cfg.d_model, device=dev)
    r = ops.router(x, m._wg, m._bg)
    d = ops.dispatch(x, ops.router(x, m._wg, m._bg), m.num_experts)
    y = ops.expert_ffn_fused(d.xperm, m._w1, m._b1, m._w2, m._b2, d.offsets)
    stage = {
        "router": lambda: ops.router(x, m._wg, m._bg),
        "dispatch": lambda: ops.dispatch(x, ops.router(x, m._wg, m._bg), m.num_experts),
        "ffn_fused": lambda: ops.expert_ffn_fused(d.xperm, m._w1, m._b1, m._w2, m._b2,
                                                  d.offsets, out=y),
        "ffn_gather": lambda: ops.expert_ffn_fused_gather(x, d.sorted_token, m._w1, m._b1, m._w2,
                                                          m._b2, d.offsets, out=y),
        "ffn_fc1": lambda: ops.grouped_gemm(d.xperm, m._w1, m._b1, d.offsets, act="gelu"),
        "combine": lambda: ops.combine(y, d.perm_inv, r.gate2),
        "layer": lambda: m(x.unsqueeze(0)),
    }[args.profile]
    for _ in range(args.warmup + args.steps):
        stage()
    torch.cuda.synchronize(dev)
    _lib.raise_on_status(dev)
    print(f"profile workload {args.profile}: T={T}, {args.warmup + args.steps} launches")


def run_embbag(args, world, rank, local):
    """--config cfg3: the 28-feature embedding-bag pooling (fp32 output),
    metric = algorithmic GB/s; every rank pools its own batch."""
    from cti_b200 import _lib, ops, synth

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    bb = synth.bag_batch(batch=4096, seed=rank)
    table = synth.embedding_table(bb.total_rows, 64, seed=rank, device=dev)
    a = [bb.values.to(dev), bb.row_offsets.to(dev), bb.val_offsets.to(dev), table,
         bb.table_row_base.to(dev), bb.vocab.to(dev), bb.features]
    out = torch.empty(bb.batch, bb.features * 64, dtype=torch.float32, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    N = bb.values.numel()
    byts = 8 * N + 8 * bb.features * (bb.batch + 1) + 128 * N + 4 * bb.batch * bb.features * 64
    for _ in range(args.warmup):
        ops.embedding_bag_sum(*a, out=out)
    torch.cuda.synchronize(dev)
    _lib.raise_on_status(dev)
    sampler = ClockSampler(dev) if rank == 0 else None
    barrier(world)
    torch.cuda.synchronize(dev)
    if sampler:
        sampler.start()
    times = time_steps(lambda: ops.embedding_bag_sum(*a, out=out), args.steps, flush, dev)
    torch.cuda.synchronize(dev)
    barrier(world)
    clocks = sampler.stop() if sampler else None
    step_ms = max_over_ranks(statistics.median(times), world, dev)
    value = sum_over_ranks(float(byts), world, dev) / (step_ms / 1e3) / 1e9
    # end to end: pinned host ids/offsets -> device, pooling, pooled rows -> pinned host
    host = [t.pin_memory() for t in (bb.values, bb.row_offsets, bb.val_offsets)]
    dev_in = [torch.empty_like(t, device=dev) for t in host]
    out_h = torch.empty(out.shape, dtype=out.dtype).pin_memory()

    def e2e():
        for d_, h_ in zip(dev_in, host):
            d_.copy_(h_, non_blocking=True)
        ops.embedding_bag_sum(dev_in[0], dev_in[1], dev_in[2], table, a[4], a[5], bb.features,
                              out=out)
        out_h.copy_(out, non_blocking=True)

    for _ in range(args.warmup):
        e2e()
    e2e_ms = max_over_ranks(statistics.median(time_steps(e2e, args.steps, flush, dev,
                                                         hide_host=False)), world, dev)
    h2d = sum(t.numel() * t.element_size() for t in host)
    peaks, src = load_peaks()
    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_embbag(bb, table, min(args.cpu_seconds, 15.0))
    line = {
        "metric": "embedding_bag_GBps", "value": value, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16->f32",
        "data": "synthetic",
        "config": {"workload": "cfg3: 28-feature embedding-bag sum pooling, batch 4096, dim 64",
                   "ids": N, "table_rows": bb.total_rows, "algorithmic_bytes": byts,
                   "l2": "flushed (256 MiB write) before every timed step"},
        "e2e": {"value": sum_over_ranks(float(byts), world, dev) / (e2e_ms / 1e3) / 1e9
                if world == 1 else None, "unit": "GB/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": out_h.numel() * 4},
        "roofline": {"bound": "hbm", "kernel": "embbag_kernel<64, float>",
                     "achieved": value / world, "peak": float(peaks["hbm_gbs"]), "unit": "GB/s",
                     "frac": value / world / float(peaks["hbm_gbs"]),
                     "peak_source": f"hbm_gbs of {src}",
                     "traffic": ncu_traffic("embbag_kernel<64, float> cfg3"),
                     "traffic_source": "profiles/dram_traffic.json (one ncu capture of a "
                                       "launch of this workload)",
                     "note": "achieved counts algorithmic bytes (128 B per id); Zipf ids re-hit "
                             "rows in L2, so the DRAM traffic is about a quarter of them and the "
                             "kernel is bound by its dependent gathers, not by HBM"},
        "gpu_launches": args.steps,
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ep", action="store_true",
                    help="leave the cfg5 expert-parallel measurement out of the cfg2 line")
    ap.add_argument("--no-e2e-model", action="store_true",
                    help="leave the cfg4 model forward out of the cfg2 line")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--config", default="cfg2", choices=["cfg2", "cfg3", "cfg4", "cfg5"],
                    help="cfg2: MoE layer (default, the headline); cfg3: embedding bag; "
                         "cfg4: full CTR model forward (ms per batch); "
                         "cfg5: expert-parallel MoE layer (strong scaling over N)")
    ap.add_argument("--placement", default="balanced", choices=["balanced", "contiguous"],
                    help="cfg5 expert placement over the ranks")
    ap.add_argument("--ep-extra-slots", type=int, default=-1,
                    help="cfg5 replica slots per rank beyond E/N (-1: 0 up to 2 ranks, "
                         "max(2, E/N/2) above)")
    ap.add_argument("--ep-exchange", default="p2p", choices=["p2p", "all_to_all"],
                    help="cfg5 rows exchange: overlapped point-to-point or plain all_to_all")
    ap.add_argument("--profile", default=None,
                    choices=["router", "dispatch", "ffn_fused", "ffn_gather", "ffn_fc1", "combine",
                             "layer", "embbag", "attention"],
                    help="run one stage of the configuration-2 workload (attention: of configuration 4) for an ncu capture")
    args = ap.parse_args()
    if args.profile:
        run_profile_workload(args)
        return
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.impl == "reference":
        run_reference(args, int(os.environ.get("WORLD_SIZE", "1")),
                      int(os.environ.get("RANK", "0")))
        return
    world, rank, local = dist_setup()
    try:
        if args.config == "cfg3":
            run_embbag(args, world, rank, local)
        elif args.config == "cfg5":
            run_ep(args, world, rank, local)
        elif args.config == "cfg4":
            run_e2e(args, world, rank, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
