"""LTX-like DiT step: one GPU, and tensor-parallel over 2 GPUs against the one-GPU step.

Two tensor-parallel forms, each against the one-GPU step of the same seeded weights:

* gather (``row_parallel=False``): each rank keeps its heads / output columns, gathers attention heads with peer
  stores (``heads_to_rows``) and projection / MLP columns inside the GEMM.  Every linear sees the same activation
  codes and computes the same int32 sums as on one GPU; the one-GPU step applies GELU and the gated residuals in
  the GEMM epilogue instead of torch ops, so the steps agree to rel-L2 <= 1e-3.
* row-parallel (the default): the output projections and MLP-down split their input columns over the ranks and
  all-reduce bf16 partial products.  The codes are the one-GPU codes (the scale comes from the combined maximum),
  but the partial sums are rounded to bf16 before they are added, so the bound is rel-L2 <= 1e-2 over 2 blocks.

The 2-GPU cases run as two child processes (NCCL, a 60 s process-group timeout) and are skipped on a 1-GPU
machine.  The row-parallel pieces are also checked on one GPU, with the K split emulated by column slices.
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


def _tp_worker(rank: int, world: int, port: int, q, row_parallel: bool) -> None:
    import datetime
    import torch.distributed as dist
    from comfy_quant_bench_b200 import ltx, mmdit, _lib
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        cfg = _small_cfg()
        model = ltx.LTXDiT(cfg, device=f"cuda:{rank}", seed=3, rank=rank, world=world, row_parallel=row_parallel)
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


@pytest.mark.parametrize("row_parallel,bound", [(True, 1e-2), (False, 1e-3)])
def test_ltx_tensor_parallel_matches_one_gpu(row_parallel, bound):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 CUDA devices")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, q, row_parallel)) for r in range(2)]
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
    assert rel <= bound, (rel, same)


# ----------------------------------------------------------------------------------------------
# row-parallel linear pieces, emulated on one GPU (the K split over "ranks" as column slices)
# ----------------------------------------------------------------------------------------------

@pytest.mark.parametrize("m,k,parts", [(300, 4096, 2), (77, 2048, 8), (16, 512, 2)])
def test_split_activation_quant_equals_the_whole_row(m, k, parts):
    """Per-rank maxima combined by a maximum, then each slice quantized with the combined scale: the codes, scales
    and group sums are exactly those of the unsplit row, slice by slice (a NaN row and an inf row included)."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from comfy_quant_bench_b200 import ops, _lib
    g = torch.Generator(device="cuda").manual_seed(m + k)
    x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    x[3, 5] = float("nan")
    x[7, k - 1] = float("inf")
    mp = (m + 15) // 16 * 16
    q, s, gs = ops.rotquant(x, 256, _lib.CQ_ACT_INT8_ROW, m_pad=mp, group_sums=True, kperm=True)
    kl = k // parts
    slices = [x[:, r * kl:(r + 1) * kl].contiguous() for r in range(parts)]
    amax = torch.stack([ops.rotquant_absmax(xs, 256, m_pad=mp) for xs in slices]).amax(dim=0)
    for r, xs in enumerate(slices):
        qr, sr, gr = ops.rotquant_scaled(xs, 256, amax.contiguous(), m_pad=mp, group_sums=True, kperm=True)
        assert torch.equal(qr, q[:, r * kl:(r + 1) * kl])
        assert torch.equal(sr, s)
        g0 = r * kl // 128
        nl = kl // 128
        assert torch.equal(gr[:, :nl], gs[:, g0:g0 + nl])                 # hi parts
        ng = k // 128
        assert torch.equal(gr[:, nl:2 * nl], gs[:, ng + g0:ng + g0 + nl])   # lo parts
    torch.cuda.synchronize()
    assert _lib.take_device_status() == (0, 0)


def test_row_parallel_partials_sum_to_the_linear():
    """The row-parallel linear's partial GEMMs (K slices, bias on the first) add up to the one-GPU linear within the
    bf16 rounding of the partials (world 1 emulation of the sum the all-reduce forms)."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from comfy_quant_bench_b200 import ops, dist as cqdist
    m, n, k, parts = 512, 1024, 4096, 4
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    w = torch.randn(n, k, device="cuda", generator=g) * 0.02
    bias = (0.01 * torch.randn(n, device="cuda", generator=g)).to(torch.bfloat16)
    qw, sc, z = ops.quantize_affine_w4_weight(w, 128, 256)
    full = ops.w4a8_affine_linear(x, qw, sc, z, bias, 128, 256)
    mp = (m + 15) // 16 * 16
    kl = k // parts
    amax = torch.stack([ops.rotquant_absmax(x[:, r * kl:(r + 1) * kl].contiguous(), 256, m_pad=mp)
                        for r in range(parts)]).amax(dim=0).contiguous()
    acc = torch.zeros(m, n, device="cuda")
    for r in range(parts):
        qr, sr, zr = cqdist.shard_affine_k(qw, sc, z, r, parts)
        a, sa, gsr = ops.rotquant_scaled(x[:, r * kl:(r + 1) * kl].contiguous(), 256, amax, m_pad=mp, group_sums=True,
                                         kperm=True)
        acc += ops.gemm_affine(a[:m], sa[:m], gsr, qr, sr, zr, bias if r == 0 else None, a_kperm=True).float()
    rel = float((acc - full.float()).norm() / full.float().norm())
    # each of the 4 partials is rounded to bf16 (relative 2^-9) before the sum, and partials can be larger than
    # the total they add up to
    assert rel <= 5e-3, rel
