"""Multi-GPU execution of the quantized linear: one process per GPU, torch.distributed for the plumbing.

Two schemes, both new relative to comfy-quant-bench (which runs on one GPU):

* ``ColumnParallelLinear``: rank r holds output rows ``[r*N/P, (r+1)*N/P)`` of the packed weight (and the
  matching scale / zero columns and bias), runs the local W4A8 / W4A4 kernels on the full activation and
  all-gathers the bf16 output columns over NCCL (NVLink / NVSwitch).  This is the path for large-token layers
  whose weight or output does not fit one GPU's budget.
* ``split_batch`` / data-parallel replicas: sampler batches (cond / uncond, several seeds) are split across
  ranks with no collective in the step.

``FusedColumnParallelW4A8`` removes the separate gather: its GEMM stores each output tile into every rank's
(symmetric-memory) output buffer over NVLink as the tile finishes.  Nothing in the library's kernels waits on a
peer; the ranks synchronize with torch's symmetric-memory barrier around the launch.

``RowParallelW4A8`` splits the weight by input columns instead: each rank quantizes its columns of the activation
with the scale of the whole row (a small all-reduce MAX of per-token maxima), runs its K slice, and one all-reduce
SUM of the bf16 partial products gives the output.  Paired with a column-parallel layer before it (an MLP-up, or a
head-parallel attention), the activation between the two never leaves its rank.
"""
from __future__ import annotations

from typing import Callable

import torch


def shard_bounds(n: int, rank: int, world: int) -> tuple[int, int]:
    if n % world:
        raise ValueError(f"out_features {n} is not divisible by the {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


def shard_affine(qweight, scale, zeros, bias, rank: int, world: int):
    """Column shard of an awq-layout weight: qweight rows, scale/zeros columns ([K/G, N] layout), bias."""
    a, b = shard_bounds(qweight.shape[0], rank, world)
    return (qweight[a:b].contiguous(), scale[:, a:b].contiguous(), zeros[:, a:b].contiguous(),
            None if bias is None else bias[a:b].contiguous())


def shard_rowscaled(qweight, wscale, bias, rank: int, world: int):
    """Column shard of a per-row-scaled weight (ConvRot W4A4 or int8): qweight rows, scale rows, bias."""
    a, b = shard_bounds(qweight.shape[0], rank, world)
    return (qweight[a:b].contiguous(), wscale.reshape(-1)[a:b].contiguous(),
            None if bias is None else bias[a:b].contiguous())


def gather_columns(local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """[M, N/P] per rank -> [M, N] on every rank (rank-major column blocks), one all_gather_into_tensor."""
    import torch.distributed as dist
    m, nl = local.shape
    buf = torch.empty(world * m, nl, dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(buf, local.contiguous(), group=group)
    return buf.view(world, m, nl).permute(1, 0, 2).reshape(m, world * nl)


class ColumnParallelLinear:
    """y = x @ W^T + b with W split over ranks by output rows and the output all-gathered.

    ``local_linear(x2d) -> [M, N/P]`` runs this rank's shard; the factories below bind it to the CUDA ops.
    """

    def __init__(self, local_linear: Callable[[torch.Tensor], torch.Tensor], out_features: int, rank: int,
                 world: int, group=None):
        self.local_linear = local_linear
        self.out_features = out_features
        self.rank = rank
        self.world = world
        self.group = group

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        x2 = x.reshape(-1, x.shape[-1])
        y = self.local_linear(x2)
        if self.world > 1:
            y = gather_columns(y, self.world, self.group)
        return y.reshape(*x.shape[:-1], self.out_features)

    @classmethod
    def w4a8_affine(cls, qweight, scale, zeros, bias, rank, world, group_size=128, convrot_groupsize=0, group=None):
        from . import ops
        q, s, z, b = shard_affine(qweight, scale, zeros, bias, rank, world)
        return cls(lambda x2: ops.w4a8_affine_linear(x2, q, s, z, b, group_size=group_size,
                                                     convrot_groupsize=convrot_groupsize),
                   qweight.shape[0], rank, world, group)

    @classmethod
    def convrot_w4a4(cls, qweight, wscales, bias, rank, world, convrot_groupsize=256, linear_dtype="int4",
                     group=None):
        from . import ops
        q, s, b = shard_rowscaled(qweight, wscales, bias, rank, world)
        return cls(lambda x2: ops.convrot_w4a4_linear(x2, q, s, b, convrot_groupsize=convrot_groupsize,
                                                      linear_dtype=linear_dtype),
                   qweight.shape[0], rank, world, group)


class FusedColumnParallelW4A8:
    """Column-parallel W4A8 affine linear whose GEMM writes its output columns straight into every rank's output.

    Each rank holds output rows ``[r*N/P, (r+1)*N/P)`` of the packed weight.  The [max_tokens, N] bf16 output is
    one symmetric-memory allocation per rank (torch.distributed symmetric memory: every rank maps every other
    rank's buffer).  The GEMM epilogue stores each finished output tile, by TMA over NVLink, into all P buffers at
    this rank's columns.  The gather therefore overlaps the GEMM and needs no separate collective or re-layout
    copy.  A device-side barrier before the launch keeps any rank from overwriting an output that a peer is still
    reading; one after it makes every rank's columns visible.
    """

    def __init__(self, qweight, scale, zeros, bias, rank: int, world: int, max_tokens: int, group=None,
                 group_size: int = 128, convrot_groupsize: int = 0):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        from . import ops
        if world > 8:
            raise ValueError("the fused column-parallel GEMM writes at most 8 output buffers")
        q, s, z, b = shard_affine(qweight, scale, zeros, bias, rank, world)
        self.q, self.s, self.b = q, s, b
        self.zt = ops.prepare_affine_zeros(z, group_size)
        self.n = qweight.shape[0]
        self.col0 = rank * q.shape[0]
        self.group_size, self.convrot_groupsize = group_size, convrot_groupsize
        self.out = symm_mem.empty(max_tokens, self.n, dtype=torch.bfloat16, device=q.device)
        self.hdl = symm_mem.rendezvous(self.out, group if group is not None else dist.group.WORLD)
        self.ptrs = [int(p) for p in self.hdl.buffer_ptrs]

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        """The gathered [..., N] output.

        The result is a view of the layer's persistent symmetric-memory buffer, valid until the next call of this
        layer on ANY rank: that call's peer stores overwrite it on every rank.  A caller that keeps the output past
        the next call (a residual, a cached activation) must ``clone()`` it.
        """
        from . import ops
        x2 = x.reshape(-1, x.shape[-1])
        m = x2.shape[0]
        if m > self.out.shape[0]:
            raise ValueError(f"{m} tokens exceed the layer's max_tokens {self.out.shape[0]}")
        self.hdl.barrier(channel=0)
        ops.w4a8_affine_linear_into(x2, self.q, self.s, self.zt, self.b, self.ptrs, self.col0, self.n,
                                    group_size=self.group_size, convrot_groupsize=self.convrot_groupsize)
        self.hdl.barrier(channel=0)
        return self.out[:m].reshape(*x.shape[:-1], self.n)


def shard_affine_k(qweight, scale, zeros, rank: int, world: int, group_size: int = 128):
    """Row-parallel (input-column) shard of an awq-layout weight: this rank's K/P input columns of the packed
    weight (two codes per byte) and the matching groups (rows of the [K/G, N] scale / zeros)."""
    k = qweight.shape[1] * 2
    a, b = shard_bounds(k, rank, world)
    if a % group_size or b % group_size:
        raise ValueError(f"the {world} K slices must hold whole {group_size}-column groups")
    return (qweight[:, a // 2:b // 2].contiguous(), scale[a // group_size:b // group_size].contiguous(),
            zeros[a // group_size:b // group_size].contiguous())


class RowParallelW4A8:
    """y = x @ W^T + b with W split over ranks by INPUT columns and the partial outputs summed.

    Rank r holds input columns ``[r*K/P, (r+1)*K/P)`` of the weight and receives the same columns of x (a
    head-parallel attention's output, or a column-parallel MLP-up's activation, stays where it was computed).
    The per-token int8 scale needs the whole row: each rank writes its columns' maximum and NaN flag
    (``rotquant_absmax``), one all-reduce MAX of [2, M] floats combines them, and ``rotquant_scaled`` quantizes
    with the combined values, so every rank's codes equal those of the unsplit row.  Each rank's GEMM over its K
    slice gives a partial product (the bias on rank 0 only), and one all-reduce SUM of the bf16 partials over NCCL
    yields the output on every rank.  The sum is taken in a different order than the one-GPU GEMM's fp32
    accumulation over all groups, so the result agrees with the one-GPU linear to the bf16 rounding of the
    partials, not bit for bit.
    """

    def __init__(self, qweight, scale, zeros, bias, rank: int, world: int, group=None, group_size: int = 128,
                 convrot_groupsize: int = 0):
        from . import ops
        q, s, z = shard_affine_k(qweight, scale, zeros, rank, world, group_size)
        if convrot_groupsize and (q.shape[1] * 2) % convrot_groupsize:
            raise ValueError("the rotation groups must lie inside one rank's columns")
        self.q, self.s = q, s
        self.zt = ops.prepare_affine_zeros(z, group_size)
        self.b = bias if rank == 0 else None
        self.n = qweight.shape[0]
        self.rank, self.world, self.group = rank, world, group
        self.convrot_groupsize = convrot_groupsize

    def __call__(self, x_local: torch.Tensor) -> torch.Tensor:
        """x_local [..., K/P] (this rank's columns) -> the full [..., N] output on every rank."""
        import torch.distributed as dist
        from . import ops
        x2 = x_local.reshape(-1, x_local.shape[-1])
        m = x2.shape[0]
        mp = (m + 15) // 16 * 16
        rot = self.convrot_groupsize
        if self.world > 1:
            amax = ops.rotquant_absmax(x2, rot, m_pad=mp)
            dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=self.group)
            q, sx, gs = ops.rotquant_scaled(x2, rot, amax, m_pad=mp, group_sums=True, kperm=True)
        else:
            q, sx, gs = ops.rotquant(x2, rot, 0, m_pad=mp, group_sums=True, kperm=True)
        y = ops.gemm_affine(q[:m], sx[:m], gs, self.q, self.s, None, self.b, a_kperm=True, zeros_prepared=self.zt)
        if self.world > 1:
            dist.all_reduce(y, op=dist.ReduceOp.SUM, group=self.group)
        return y.reshape(*x_local.shape[:-1], self.n)


def split_batch(x: torch.Tensor, rank: int, world: int, dim: int = 0) -> torch.Tensor:
    """This rank's slice of a sampler batch (data-parallel replicas, no collective in the step)."""
    n = x.shape[dim]
    per = (n + world - 1) // world
    return x.narrow(dim, min(rank * per, n), max(0, min(per, n - rank * per)))
