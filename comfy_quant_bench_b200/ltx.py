"""LTX-like 22B-class video DiT denoise step on W4A8 affine linears, on one GPU or tensor-parallel over P GPUs.

A stack of single-stream video DiT blocks (random init), every linear on the W4A8 affine path (ConvRot g256 +
per-token int8 activations, awq-layout weights with group 128):

    y = LayerNorm(x) * (1 + scale_sa) + shift_sa                       (inside the QKV activation kernel)
    q, k, v = Wqkv y;  q, k = rope(RMSNorm_head(q)), rope(RMSNorm_head(k))   (one glue kernel)
    x = x + gate_sa * Wo attention(q, k, v)                            (32 heads x 128)
    x = x + Wco attention(RMSNorm_head(Wcq LayerNorm(x)), RMSNorm_head(Wck c), Wcv c)   (text context c)
    x = x + gate_ff * W2 gelu_tanh(W1 (LayerNorm(x) * (1 + scale_ff) + shift_ff))

Tensor parallelism over P ranks (one process per GPU, torch.distributed + torch symmetric memory):

* attention is head-parallel: the QKV and cross-attention Q / KV linears keep the rows of this rank's H/P heads,
  so q, k, v and the attention itself stay rank-local; ``heads_to_rows`` then writes every rank's head outputs
  into every rank's [tokens, hidden] buffer (plain peer stores over NVLink);
* the output projections and both MLP linears are column-parallel: each rank computes N/P output columns and the
  GEMM's epilogue stores every finished tile into every rank's output buffer (``gemm_affine_into`` with the peer
  pointers), so the all-gather over N runs inside the GEMM;
* norms, modulation, GELU and residual updates run on every rank on the full activations (replicated);
* torch's symmetric-memory barrier orders the ranks around each exchange: before a rank's peer stores into a
  shared buffer (its previous readers on every rank are done) and after them (every rank's columns have landed).

Every rank builds the same full weights from the same seed and keeps its rows, so the P-rank step computes every
linear exactly as the one-GPU step does (the same codes, the same int32 sums and epilogue).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import ops
from . import _lib
from .dist import RowParallelW4A8
from .mmdit import rel_l2  # noqa: F401


@dataclass(frozen=True)
class LTXConfig:
    blocks: int = 48
    hidden: int = 4096
    heads: int = 32
    ffn: int = 16384
    frames: int = 8             # latent grid 8 x 64 x 64 = 32,768 tokens
    height: int = 64
    width: int = 64
    ctx_tokens: int = 128
    group_size: int = 128
    convrot_groupsize: int = 256

    @property
    def tokens(self) -> int:
        return self.frames * self.height * self.width

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


class AffineLinear:
    """W4A8 affine linear holding selected output rows of a full seeded weight."""

    def __init__(self, in_f: int, out_f: int, rows, gen: torch.Generator, device, cfg: LTXConfig):
        w = torch.randn(out_f, in_f, generator=gen, device=device, dtype=torch.float32).mul_(0.02)
        bias = (torch.randn(out_f, generator=gen, device=device) * 0.01).to(torch.bfloat16)
        q, s, z = ops.quantize_affine_w4_weight(w, cfg.group_size, cfg.convrot_groupsize)
        del w
        idx = torch.as_tensor(rows, device=device, dtype=torch.long) if rows is not None else None
        if idx is not None:
            q, s, z, bias = q[idx].contiguous(), s[:, idx].contiguous(), z[:, idx].contiguous(), bias[idx].contiguous()
        self.qweight, self.scale, self.zeros, self.bias = q, s, z, bias
        self.zt = ops.prepare_affine_zeros(z, cfg.group_size)
        self.cfg = cfg
        self.in_f, self.out_f = in_f, q.shape[0]

    def __call__(self, x):
        return ops.w4a8_affine_linear(x, self.qweight, self.scale, self.zeros, self.bias, self.cfg.group_size,
                                      self.cfg.convrot_groupsize, zeros_prepared=self.zt)

    def lnmod(self, x, shift, scale1p):
        return ops.w4a8_affine_linear_lnmod(x, shift, scale1p, self.qweight, self.scale, self.zt, self.bias,
                                            self.cfg.group_size, self.cfg.convrot_groupsize)

    def op(self, x, out_op, *, residual=None, gate=None, shift=None, scale=None):
        """This linear with GELU (``"gelu"``) or the gated residual (``"gated"``) in the GEMM epilogue, and with
        shift / the modulation scale the modulated layer norm (by the bf16 1 + scale) in the activation kernel
        (``ops.w4a8_affine_linear_op``)."""
        return ops.w4a8_affine_linear_op(x, self.qweight, self.scale, self.zt, self.bias, out_op=out_op,
                                         residual=residual, gate=gate, shift=shift, scale=scale,
                                         group_size=self.cfg.group_size, convrot_groupsize=self.cfg.convrot_groupsize)

    def quantize(self, x, shift=None, scale1p=None):
        """The activation stage alone (codes, scales, split group sums), optionally of the modulated layer norm."""
        mp = (x.shape[0] + 15) // 16 * 16
        if shift is not None:
            return ops.rotquant_lnmod(x, self.cfg.convrot_groupsize, shift, scale1p, m_pad=mp, group_sums=True,
                                      kperm=True)
        return ops.rotquant(x, self.cfg.convrot_groupsize, _lib.CQ_ACT_INT8_ROW, m_pad=mp, group_sums=True, kperm=True)

    def into(self, act, m: int, outs, col0: int, ldo: int):
        q, sx, gs = act
        ops.gemm_affine_into(q, sx, gs, self.qweight, self.scale, self.zt, self.bias, outs, col0, ldo, m=m)

    def weight_bytes(self) -> int:
        return self.qweight.numel() + 2 * self.scale.numel() * 2 + self.zt.numel() * 2


def _head_rows(part_rows: int, parts: int, h0: int, h1: int, d: int):
    """Rows of a fused [parts * part_rows, K] weight belonging to heads [h0, h1): each part's head block, in order."""
    return [p * part_rows + r for p in range(parts) for r in range(h0 * d, h1 * d)]


def _rope3d(cfg: LTXConfig, device) -> torch.Tensor:
    d = cfg.head_dim
    half = d // 2
    parts = (half - 2 * (half // 3), half // 3, half // 3)
    grids = torch.meshgrid(torch.arange(cfg.frames, device=device), torch.arange(cfg.height, device=device),
                           torch.arange(cfg.width, device=device), indexing="ij")
    angs = []
    for pos, n in zip(grids, parts):
        inv = 1.0 / (10000.0 ** (torch.arange(n, device=device, dtype=torch.float32) / n))
        angs.append(pos.reshape(-1, 1).float() * inv[None, :])
    ang = torch.cat(angs, dim=1)
    return torch.complex(torch.cos(ang), torch.sin(ang))


class _Block:
    def __init__(self, gen, device, cfg: LTXConfig, rank: int, world: int, row_parallel: bool, group=None):
        h, f, d = cfg.hidden, cfg.ffn, cfg.head_dim
        hp = cfg.heads // world
        h0, h1 = rank * hp, (rank + 1) * hp
        cols = lambda n: list(range(rank * n // world, (rank + 1) * n // world)) if world > 1 else None  # noqa: E731
        heads = lambda parts, n: _head_rows(n, parts, h0, h1, d) if world > 1 else None  # noqa: E731
        rp = row_parallel and world > 1

        def row_par(lin: AffineLinear):
            # the full weight, split by input columns (the same seeded draws as every other form)
            return RowParallelW4A8(lin.qweight, lin.scale, lin.zeros, lin.bias, rank, world, group, cfg.group_size,
                                   cfg.convrot_groupsize)

        self.qkv = AffineLinear(h, 3 * h, heads(3, h), gen, device, cfg)
        self.out = AffineLinear(h, h, None if rp else cols(h), gen, device, cfg)
        self.cq = AffineLinear(h, h, heads(1, h), gen, device, cfg)
        self.ckv = AffineLinear(h, 2 * h, heads(2, h), gen, device, cfg)
        self.co = AffineLinear(h, h, None if rp else cols(h), gen, device, cfg)
        self.ff1 = AffineLinear(h, f, cols(f), gen, device, cfg)
        self.ff2 = AffineLinear(f, h, None if rp else cols(h), gen, device, cfg)
        if rp:
            self.out, self.co, self.ff2 = row_par(self.out), row_par(self.co), row_par(self.ff2)
        self.mod = (torch.randn(6, h, generator=gen, device=device) * 0.1).to(torch.bfloat16)
        self.scale1p = (1.0 + self.mod[[1, 4]]).contiguous()
        self.norms = (1 + 0.1 * torch.randn(4, d, generator=gen, device=device)).to(torch.bfloat16)
        self.zero_shift = torch.zeros(h, dtype=torch.bfloat16, device=device)
        self.one = torch.ones(h, dtype=torch.bfloat16, device=device)

    def linears(self):
        return [self.qkv, self.out, self.cq, self.ckv, self.co, self.ff1, self.ff2]

    def weight_bytes(self) -> int:
        tot = 0
        for l in self.linears():
            if isinstance(l, RowParallelW4A8):
                tot += l.q.numel() + 2 * l.s.numel() * 2 + l.zt.numel() * 2
            else:
                tot += l.weight_bytes()
        return tot


class LTXDiT:
    """The LTX-like step on this rank: ``world`` > 1 runs the tensor-parallel form (call from every rank)."""

    def __init__(self, cfg: LTXConfig = LTXConfig(), device="cuda", seed: int = 0, rank: int = 0, world: int = 1,
                 group=None, row_parallel: bool = True):
        if cfg.heads % world or cfg.hidden % world or cfg.ffn % world:
            raise ValueError(f"heads, hidden and ffn must divide by the {world} ranks")
        self.cfg, self.rank, self.world = cfg, rank, world
        self.row_parallel = row_parallel and world > 1
        self.group = group
        self.device = torch.device(device)
        gen = torch.Generator(device=self.device)
        gen.manual_seed(seed)
        self.blocks = [_Block(gen, self.device, cfg, rank, world, row_parallel, group) for _ in range(cfg.blocks)]
        self.rope = _rope3d(cfg, self.device)
        s, h, f = cfg.tokens, cfg.hidden, cfg.ffn
        if world > 1 and not self.row_parallel:
            import torch.distributed as dist
            import torch.distributed._symmetric_memory as symm_mem
            grp = group if group is not None else dist.group.WORLD
            self._bufs = {}
            for name, n in (("attn", h), ("hid", h), ("ffn", f)):
                t = symm_mem.empty(s, n, dtype=torch.bfloat16, device=self.device)
                hdl = symm_mem.rendezvous(t, grp)
                self._bufs[name] = (t, [int(p) for p in hdl.buffer_ptrs], hdl)
            self._hdl = self._bufs["attn"][2]
        else:
            self._bufs = {name: (torch.empty(s, n, dtype=torch.bfloat16, device=self.device), None, None)
                          for name, n in (("attn", h), ("hid", h), ("ffn", f))}
            self._hdl = None

    # ---- exchanges ----
    def _barrier(self):
        if self._hdl is not None:
            self._hdl.barrier(channel=0)

    def _outs(self, name):
        t, ptrs, _ = self._bufs[name]
        return ptrs if ptrs is not None else [t]

    def _heads_gather(self, o: torch.Tensor) -> torch.Tensor:
        """o [1, H/P, S, D] -> full [S, hidden] on every rank."""
        c = self.cfg
        self._barrier()                                   # every rank is done reading the previous contents
        ops.heads_to_rows(o, self._outs("attn"), self.rank * (c.heads // self.world) * c.head_dim, c.hidden)
        self._barrier()                                   # every rank's heads have landed
        return self._bufs["attn"][0]

    def _col_linear(self, lin: AffineLinear, x: torch.Tensor, name: str, shift=None, scale1p=None) -> torch.Tensor:
        """Column-parallel linear: the full [S, N] output in buffer ``name`` on every rank (the gather inside the
        GEMM).  Every earlier reader of the buffer, on every rank, must be ordered before this call by a barrier
        (step arranges it); the barrier after the GEMM makes all ranks' columns visible."""
        if self.world == 1:
            return lin.lnmod(x, shift, scale1p) if shift is not None else lin(x)
        act = lin.quantize(x, shift, scale1p)
        n_full = lin.out_f * self.world
        lin.into(act, x.shape[0], self._outs(name), self.rank * lin.out_f, n_full)
        self._barrier()
        return self._bufs[name][0][: x.shape[0]]

    def _heads_local(self, o: torch.Tensor) -> torch.Tensor:
        """o [1, H/P, S, D] -> this rank's heads as [S, H/P * D] rows (the row-parallel projections' input): a view
        when o is token-major in memory (attention over token-major q), else a copy."""
        _, hp, s, d = o.shape
        if o.transpose(1, 2).is_contiguous():
            return o.transpose(1, 2).reshape(s, hp * d)
        a = torch.empty(s, hp * d, dtype=torch.bfloat16, device=o.device)
        ops.heads_to_rows(o, [a], 0, hp * d)
        return a

    # ---- the step ----
    def step(self, x: torch.Tensor, ctx: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return self._step_one_gpu(x, ctx)
        if self.row_parallel:
            return self._step_row_parallel(x, ctx)
        return self._step_gather(x, ctx)

    def _attn_inputs(self, s: int, device):
        """q, k, v of this rank's heads as [1, H/P, S, D] views of token-major [1, S, H/P, D] memory, so that the
        attention's output is token-major too and reaches the output projection as rows without a copy."""
        c = self.cfg
        hp = c.heads // self.world
        return tuple(torch.empty(1, s, hp, c.head_dim, dtype=torch.bfloat16, device=device).transpose(1, 2)
                     for _ in range(3))

    def _cross_attention(self, b, x, ctx, s: int):
        c = self.cfg
        d, hp = c.head_dim, c.heads // self.world
        cq = F.rms_norm(b.cq.lnmod(x, b.zero_shift, b.one).view(s, hp, d), (d,), b.norms[2], eps=1e-6)
        kv = b.ckv(ctx).view(-1, 2, hp, d)
        ck = F.rms_norm(kv[:, 0], (d,), b.norms[3], eps=1e-6)
        return F.scaled_dot_product_attention(cq.transpose(0, 1)[None], ck.transpose(0, 1)[None],
                                              kv[:, 1].transpose(0, 1)[None])

    def _step_one_gpu(self, x: torch.Tensor, ctx: torch.Tensor) -> torch.Tensor:
        """One GPU: the gated residuals and GELU in the GEMM epilogues, the norms in the activation kernels."""
        s = x.shape[0]
        q, k, v = self._attn_inputs(s, x.device)
        for b in self.blocks:
            m = b.mod
            y = b.qkv.lnmod(x, m[0], b.scale1p[0])
            ops.qkv_rmsnorm_rope(y, b.norms[0], b.norms[1], self.rope, q, k, v, 0, eps=1e-6)
            x = b.out.op(self._heads_local(F.scaled_dot_product_attention(q, k, v)), "gated", residual=x, gate=m[2])
            x = b.co.op(self._heads_local(self._cross_attention(b, x, ctx, s)), "gated", residual=x, gate=b.one)
            g = b.ff1.op(x, "gelu", shift=m[3], scale=m[4])
            x = b.ff2.op(g, "gated", residual=x, gate=m[5])
        return x

    def _step_row_parallel(self, x: torch.Tensor, ctx: torch.Tensor) -> torch.Tensor:
        """P ranks, Megatron-style: attention heads and the MLP's hidden columns stay on their rank; the output
        projections and MLP-down are row-parallel (an all-reduce of the partial products, NCCL), so the only
        full-size exchanges per block are three all-reduces of [S, hidden] bf16."""
        s = x.shape[0]
        q, k, v = self._attn_inputs(s, x.device)
        for b in self.blocks:
            m = b.mod
            y = b.qkv.lnmod(x, m[0], b.scale1p[0])
            ops.qkv_rmsnorm_rope(y, b.norms[0], b.norms[1], self.rope, q, k, v, 0, eps=1e-6)
            x = torch.addcmul(x, m[2], b.out(self._heads_local(F.scaled_dot_product_attention(q, k, v))))
            x = x + b.co(self._heads_local(self._cross_attention(b, x, ctx, s)))
            g = b.ff1.op(x, "gelu", shift=m[3], scale=m[4])      # this rank's ffn/P hidden columns
            x = torch.addcmul(x, m[5], b.ff2(g))
        return x

    def _step_gather(self, x: torch.Tensor, ctx: torch.Tensor) -> torch.Tensor:
        """P ranks, every linear column-parallel with the all-gather inside the GEMM (peer stores)."""
        c = self.cfg
        h, d = c.hidden, c.head_dim
        hp = c.heads // self.world
        s = x.shape[0]
        q = torch.empty(1, hp, s, d, dtype=torch.bfloat16, device=x.device)
        k = torch.empty_like(q)
        v = torch.empty_like(q)
        for b in self.blocks:
            m = b.mod
            # self-attention, head-parallel
            y = b.qkv.lnmod(x, m[0], b.scale1p[0])
            ops.qkv_rmsnorm_rope(y, b.norms[0], b.norms[1], self.rope, q, k, v, 0, eps=1e-6)
            a = self._heads_gather(F.scaled_dot_product_attention(q, k, v))
            x = torch.addcmul(x, m[2], self._col_linear(b.out, a, "hid"))
            # cross-attention to the text context, head-parallel
            cq = F.rms_norm(b.cq.lnmod(x, b.zero_shift, b.one).view(s, hp, d), (d,), b.norms[2], eps=1e-6)
            kv = b.ckv(ctx).view(-1, 2, hp, d)
            ck = F.rms_norm(kv[:, 0], (d,), b.norms[3], eps=1e-6)
            o = F.scaled_dot_product_attention(cq.transpose(0, 1)[None], ck.transpose(0, 1)[None],
                                               kv[:, 1].transpose(0, 1)[None])
            a = self._heads_gather(o)
            x = x + self._col_linear(b.co, a, "hid")
            # MLP, column-parallel (the up projection's activation stage also forms the modulated layer norm).  The
            # last readers of "ffn" (the previous block's GELU) and of "hid" (the residual updates above) ran before
            # barriers every rank has passed, so both buffers are free to be written here.
            u = self._col_linear(b.ff1, x, "ffn", m[3], b.scale1p[1])
            g = F.gelu(u, approximate="tanh")
            x = torch.addcmul(x, m[5], self._col_linear(b.ff2, g, "hid"))
        return x

    def linears(self):
        return [l for b in self.blocks for l in b.linears()]

    def weight_bytes(self) -> int:
        return sum(b.weight_bytes() for b in self.blocks)

    def linear_int_ops(self) -> float:
        """2 * M * N * K of the whole model's linears for one step (all ranks together)."""
        c = self.cfg
        h, f, s, t = c.hidden, c.ffn, c.tokens, c.ctx_tokens
        per_block = 2.0 * s * (3 * h * h + h * h + h * h + h * h + 2 * h * f) + 2.0 * t * (2 * h * h)
        return per_block * c.blocks

    def attention_flops(self) -> float:
        c = self.cfg
        return c.blocks * 4.0 * c.tokens * (c.tokens + c.ctx_tokens) * c.hidden

    def inputs(self, seed: int = 1):
        c = self.cfg
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        x = torch.randn(c.tokens, c.hidden, generator=g, device=self.device).to(torch.bfloat16)
        ctx = torch.randn(c.ctx_tokens, c.hidden, generator=g, device=self.device).to(torch.bfloat16)
        return x, ctx
