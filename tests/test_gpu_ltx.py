"""LTX-like DiT step: one GPU, and tensor-parallel over 2 GPUs against the one-GPU step.

The tensor-parallel form keeps each rank's heads / output columns of the same seeded weights, gathers attention
heads with peer stores (``heads_to_rows``) and projection / MLP columns inside the GEMM.  Every linear therefore sees
the same activation codes and computes the same int32 sums and epilogue as on one GPU, and attention runs per head,
so the two steps agree to rel-L2 <= 1e-3 (the bound written below; in practice they are bit-identical).
The 2-GPU case runs as two child processes (NCCL, a 60 s process-group timeout) and is skipped on a 1-GPU machine.
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _small_cfg():
    from comfy_quant_bench_b200 import ltx
    return ltx.LTXConfig(blocks=2, hidden=512, heads=8, ffn=1024, frames=2, height=8, width=16, ctx_tokens=32)


def test_ltx_one_gpu_step_is_finite_and_deterministic():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from comfy_quant_bench_b200 import ltx, _lib
    model = ltx.LTXDiT(_small_cfg(), device="cuda", seed=3)
    x, ctx = model.inputs(seed=4)
    a = model.step(x, ctx)
    b = model.step(x, ctx)
    torch.cuda.synchronize()
    assert torch.isfinite(a.float()).all()
    assert torch.equal(a, b)
    assert _lib.take_device_status() == (0, 0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_worker(rank: int, world: int, port: int, q) -> None:
    import datetime
    import torch.distributed as dist
    from comfy_quant_bench_b200 import ltx, mmdit, _lib
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        cfg = _small_cfg()
        model = ltx.LTXDiT(cfg, device=f"cuda:{rank}", seed=3, rank=rank, world=world)
        x, ctx = model.inputs(seed=4)
        out = model.step(x, ctx)
        torch.cuda.synchronize()
        if rank == 0:
            single = ltx.LTXDiT(cfg, device="cuda:0", seed=3)
            ref = single.step(x, ctx)
            torch.cuda.synchronize()
            q.put((mmdit.rel_l2(out, ref), bool(torch.equal(out, ref)), _lib.take_device_status()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_ltx_tensor_parallel_matches_one_gpu():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 CUDA devices")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    rel, same, status = q.get(timeout=10)
    assert status == (0, 0)
    assert rel <= 1e-3, (rel, same)
