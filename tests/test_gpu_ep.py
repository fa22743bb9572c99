"""Expert parallelism on GPUs (NCCL): the sharded layer equals the
single-GPU layer on the same tokens.  Runs one process per visible GPU (at
most 2; a single GPU runs the degenerate one-rank group).  Per-row results
do not depend on how rows are grouped into GEMM tiles, so the sharded output
must match the unsharded one to within bf16 rounding noise, and every case,
configuration 5's shape included, against the CPU oracle (max rel err
2e-2)."""
import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, D, E, F, T, balanced, overlap, extra=0):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=dev)
    try:
        import cti_b200
        from cti_b200 import _lib, synth
        from cti_b200.ep import ExpertParallelSMoE
        from helpers import max_rel_err
        from oracle import moe_ref as mr

        w = synth.moe_weights(D, E, F, 1.2, seed=5)
        full = cti_b200.SMoE(D, F, E)
        synth.load_moe_module(full, w)
        x = synth.moe_activations(T, D, seed=5)
        lo, hi = rank * T // world, (rank + 1) * T // world
        placement = None
        if balanced:
            from cti_b200.ep import balanced_placement
            placement = balanced_placement(torch.softmax(w.bg, 0).tolist(), world,
                                           E // world + extra)
            if world > 1 or extra:
                assert placement != list(range(E))
        ep = ExpertParallelSMoE(D, F, E, placement=placement).to(dev)
        ep.load_global_state_dict(full.state_dict())
        out, _ = ep(x[lo:hi].to(dev), overlap=overlap)
        _lib.raise_on_status(dev)
        full.to(dev).prepare_for_inference()
        ref_gpu, _ = full(x[lo:hi].to(dev).unsqueeze(0))
        assert max_rel_err(out, ref_gpu[0]) < 2e-3
        ref, _ = mr.smoe_ref(x[lo:hi].float(), w.wg, w.bg, w.w1.float(), w.b1,
                             w.w2.float(), w.b2)
        assert max_rel_err(out, ref) < 2e-2
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("D,E,F,T,balanced,overlap,extra", [
    (1024, 64, 4096, 8192, False, False, 0),
    (1024, 64, 4096, 8192, True, True, 0),
    (1024, 64, 4096, 8192, True, True, 3),   # replicated experts
    (256, 16, 1024, 6000, True, True, 0),
    (256, 16, 1024, 6000, True, True, 2),
    (256, 16, 1024, 6000, False, True, 0)])
def test_expert_parallel_layer_matches_single_gpu(D, E, F, T, balanced, overlap, extra):
    world = min(2, torch.cuda.device_count())
    assert world >= 1
    mp.spawn(_worker, args=(world, _free_port(), D, E, F, T, balanced, overlap, extra),
             nprocs=world, join=True)
