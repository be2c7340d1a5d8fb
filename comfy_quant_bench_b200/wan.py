"""Wan-2.2-5B-like video DiT denoise step on the mixed W4A4 / W8A8 plan (random init).

The model-level workload of the ConvRot W4A4 and int8 W8A8 linears: a stack of single-stream video DiT blocks
(self-attention with 3-D rotary embedding, cross-attention to a text context, GELU feed-forward, adaLN-style
modulation) where a seeded 35 % of the linears run ``ops.convrot_w4a4_linear`` (rotated per-row int4 weights,
Hadamard group 64, per-token int4 activations) and the rest ``ops.int8_linear`` (int8_tensorwise weights, per-token
int8 activations).  The block follows the public Wan 2.x layout:

    y = LayerNorm(x) * (1 + scale_sa) + shift_sa
    q = RMSNorm(Wq y), k = RMSNorm(Wk y), v = Wv y         (RMSNorm over the whole hidden dim, with weight)
    x = x + gate_sa * Wo attention(rope(q), rope(k), v)     (24 heads x 128)
    y = LayerNorm_affine(x);  c = text context [512, hidden]
    x = x + Wo' attention(RMSNorm(Wq' y), RMSNorm(Wk' c), Wv' c)
    x = x + gate_ff * W2 gelu_tanh(W1 (LayerNorm(x) * (1 + scale_ff) + shift_ff))

The per-block modulation vectors (shift/scale/gate) are drawn at random, standing in for the model's time
embedding.  On the kernel path (``fused_glue``) the q/k RMSNorm and the rotary embedding run as one library
kernel per tensor (``ops.rmsnorm_rope_rows``), the modulated layer norms inside the activation kernels of the QKV
and MLP-up linears, and GELU and the residual updates in the GEMM epilogues (``ops.convrot_w4a4_linear_op`` /
``ops.int8_linear_op``); the affine layer norm before the cross-attention and the attention itself stay torch ops.  ``step(..., reference=True)`` replaces
every linear by a torch fp32 product of its dequantized weight and the dequantized activation codes the library's
own activation kernel produced.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import ops
from . import _lib
from .mmdit import rel_l2


@dataclass(frozen=True)
class WanConfig:
    blocks: int = 30
    hidden: int = 3072
    heads: int = 24
    ffn: int = 14336
    frames: int = 31            # latent grid 31 x 22 x 40 = 27,280 tokens
    height: int = 22
    width: int = 40
    ctx_tokens: int = 512
    w4a4_fraction: float = 0.35
    w4a4_rot: int = 64          # Hadamard group of the W4A4 linears
    w8a8_rot: int = 0           # int8_tensorwise without rotation
    fused_glue: bool = True     # kernel path: q/k RMSNorm (+ rotary) as one library kernel per tensor, the
                                # modulated layer norms in the activation kernels of the QKV and MLP-up linears, GELU
                                # and the (gated) residual updates in the GEMM epilogues

    @property
    def tokens(self) -> int:
        return self.frames * self.height * self.width

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


def _unpack_int4_signed(q: torch.Tensor, n: int, k: int) -> torch.Tensor:
    """Packed signed nibbles (low nibble = even column) -> int values [N, K] as fp32."""
    u = q.view(torch.uint8)
    v = torch.stack((u & 15, u >> 4), dim=-1).reshape(n, k).to(torch.int16)
    return torch.where(v >= 8, v - 16, v).float()


class W4A4Linear:
    """ConvRot W4A4: rotated per-row int4 weight (Hadamard group ``rot``), per-token int4 activations."""

    kind = "w4a4"

    def __init__(self, in_f: int, out_f: int, gen: torch.Generator, device, rot: int):
        w = torch.randn(out_f, in_f, generator=gen, device=device, dtype=torch.float32).mul_(0.02)
        self.qweight, self.wscale = ops.quantize_convrot_w4a4_weight(w, rot)
        del w
        self.bias = (torch.randn(out_f, generator=gen, device=device) * 0.01).to(torch.bfloat16)
        self.rot, self.in_f, self.out_f = rot, in_f, out_f

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return ops.convrot_w4a4_linear(x, self.qweight, self.wscale, self.bias, convrot_groupsize=self.rot)

    def op(self, x: torch.Tensor, out_op: str, **kw) -> torch.Tensor:
        """This linear with the step after it in the GEMM's epilogue (``ops.convrot_w4a4_linear_op``)."""
        return ops.convrot_w4a4_linear_op(x, self.qweight, self.wscale, self.bias, out_op=out_op,
                                          convrot_groupsize=self.rot, **kw)

    def reference(self, x: torch.Tensor) -> torch.Tensor:
        x2 = x.reshape(-1, x.shape[-1]).to(torch.bfloat16).contiguous()
        q, sx, _ = ops.rotquant(x2, self.rot, _lib.CQ_ACT_INT4_ROW, int4_as_int8=True)
        w = _unpack_int4_signed(self.qweight, self.out_f, self.in_f) * self.wscale.float()[:, None]
        y = (q.float() * sx[:, None]) @ w.t() + self.bias.float()
        return y.to(torch.bfloat16).reshape(*x.shape[:-1], self.out_f)

    def weight_bytes(self) -> int:
        return self.qweight.numel() + self.wscale.numel() * 4


class W8A8Linear:
    """int8_tensorwise W8A8 (optional ConvRot), per-token int8 activations."""

    kind = "w8a8"

    def __init__(self, in_f: int, out_f: int, gen: torch.Generator, device, rot: int):
        w = torch.randn(out_f, in_f, generator=gen, device=device, dtype=torch.float32).mul_(0.02)
        self.qweight, self.wscale = ops.quantize_int8_convrot_weight(w, rot)
        del w
        self.bias = (torch.randn(out_f, generator=gen, device=device) * 0.01).to(torch.bfloat16)
        self.rot, self.in_f, self.out_f = rot, in_f, out_f

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return ops.int8_linear(x, self.qweight, self.wscale, self.bias, convrot=self.rot > 0,
                               convrot_groupsize=max(self.rot, 16))

    def op(self, x: torch.Tensor, out_op: str, **kw) -> torch.Tensor:
        """This linear with the step after it in the GEMM's epilogue (``ops.int8_linear_op``)."""
        return ops.int8_linear_op(x, self.qweight, self.wscale, self.bias, out_op=out_op, convrot=self.rot > 0,
                                  convrot_groupsize=max(self.rot, 16), **kw)

    def reference(self, x: torch.Tensor) -> torch.Tensor:
        x2 = x.reshape(-1, x.shape[-1]).to(torch.bfloat16).contiguous()
        q, sx, _ = ops.rotquant(x2, self.rot, _lib.CQ_ACT_INT8_ROW)
        w = self.qweight.float() * self.wscale.float().reshape(-1, 1)
        y = (q.float() * sx[:, None]) @ w.t() + self.bias.float()
        return y.to(torch.bfloat16).reshape(*x.shape[:-1], self.out_f)

    def weight_bytes(self) -> int:
        return self.qweight.numel() + self.wscale.numel() * 4


class _Block:
    NAMES = ("q", "k", "v", "o", "cq", "ck", "cv", "co", "ff1", "ff2")

    def __init__(self, gen, device, cfg: WanConfig, kinds: list[str]):
        h, f = cfg.hidden, cfg.ffn
        shapes = {"q": (h, h), "k": (h, h), "v": (h, h), "o": (h, h), "cq": (h, h), "ck": (h, h), "cv": (h, h),
                  "co": (h, h), "ff1": (h, f), "ff2": (f, h)}
        self.lin = {}
        for name, kind in zip(self.NAMES, kinds):
            i, o = shapes[name]
            self.lin[name] = (W4A4Linear(i, o, gen, device, cfg.w4a4_rot) if kind == "w4a4"
                              else W8A8Linear(i, o, gen, device, cfg.w8a8_rot))
        self.mod = (torch.randn(6, h, generator=gen, device=device) * 0.1).to(torch.bfloat16)
        self.norm_q = (1 + 0.1 * torch.randn(h, generator=gen, device=device)).to(torch.bfloat16)
        self.norm_k = (1 + 0.1 * torch.randn(h, generator=gen, device=device)).to(torch.bfloat16)
        self.norm_cq = (1 + 0.1 * torch.randn(h, generator=gen, device=device)).to(torch.bfloat16)
        self.norm_ck = (1 + 0.1 * torch.randn(h, generator=gen, device=device)).to(torch.bfloat16)
        self.norm3_w = (1 + 0.1 * torch.randn(h, generator=gen, device=device)).to(torch.bfloat16)
        self.norm3_b = (0.1 * torch.randn(h, generator=gen, device=device)).to(torch.bfloat16)


def _rope3d(cfg: WanConfig, device) -> torch.Tensor:
    """3-D rotary factors [tokens, D/2] complex64: the head dim split into temporal / height / width parts."""
    d = cfg.head_dim
    half = d // 2
    parts = (half - 2 * (half // 3), half // 3, half // 3)
    grids = torch.meshgrid(torch.arange(cfg.frames, device=device), torch.arange(cfg.height, device=device),
                           torch.arange(cfg.width, device=device), indexing="ij")
    angs = []
    for pos, n in zip(grids, parts):
        inv = 1.0 / (10000.0 ** (torch.arange(n, device=device, dtype=torch.float32) * 2.0 / (2 * n)))
        angs.append(pos.reshape(-1, 1).float() * inv[None, :])
    ang = torch.cat(angs, dim=1)
    return torch.complex(torch.cos(ang), torch.sin(ang))


def _rope(x: torch.Tensor, rot: torch.Tensor) -> torch.Tensor:
    """x [S, H, D] bf16 rotated on interleaved pairs by rot [S, D/2] -> bf16."""
    xc = torch.view_as_complex(x.float().reshape(*x.shape[:-1], -1, 2))
    return torch.view_as_real(xc * rot[:, None, :]).reshape(x.shape).to(torch.bfloat16)


class WanDiT:
    def __init__(self, cfg: WanConfig = WanConfig(), device="cuda", seed: int = 0):
        self.cfg = cfg
        self.device = torch.device(device)
        gen = torch.Generator(device=self.device)
        gen.manual_seed(seed)
        n_lin = cfg.blocks * len(_Block.NAMES)
        pick = torch.randperm(n_lin, generator=torch.Generator().manual_seed(seed + 17))
        w4 = set(pick[: round(cfg.w4a4_fraction * n_lin)].tolist())
        kinds = ["w4a4" if i in w4 else "w8a8" for i in range(n_lin)]
        nb = len(_Block.NAMES)
        self.blocks = [_Block(gen, self.device, cfg, kinds[b * nb:(b + 1) * nb]) for b in range(cfg.blocks)]
        self.rope = _rope3d(cfg, self.device)
        self.one = torch.ones(cfg.hidden, dtype=torch.bfloat16, device=self.device)

    def linears(self):
        return [l for b in self.blocks for l in b.lin.values()]

    def weight_bytes(self) -> int:
        return sum(l.weight_bytes() for l in self.linears())

    def plan(self) -> dict:
        ls = self.linears()
        return {"w4a4": sum(l.kind == "w4a4" for l in ls), "w8a8": sum(l.kind == "w8a8" for l in ls)}

    def launches_per_step(self) -> int:
        """The library's kernel launches in one kernel-path step: an activation kernel and a GEMM per linear, and
        with the fused glue the q/k norm kernel for q, k and the cross-attention's q, k."""
        return 2 * len(self.linears()) + (4 * self.cfg.blocks if self.cfg.fused_glue else 0)

    def linear_int_ops(self) -> float:
        c = self.cfg
        tot = 0.0
        for b in self.blocks:
            for name, l in b.lin.items():
                m = c.ctx_tokens if name in ("ck", "cv") else c.tokens
                tot += 2.0 * m * l.out_f * l.in_f
        return tot

    def attention_flops(self) -> float:
        c = self.cfg
        return c.blocks * 4.0 * c.tokens * (c.tokens + c.ctx_tokens) * c.hidden

    def step(self, x: torch.Tensor, ctx: torch.Tensor, reference: bool = False) -> torch.Tensor:
        """One denoise step: x [tokens, hidden], ctx [ctx_tokens, hidden] (bf16) -> x."""
        for b in self.blocks:
            x = self._block(b, x, ctx, reference)
        return x

    def block_errors(self, x: torch.Tensor, ctx: torch.Tensor) -> list[float]:
        """Teacher-forced check: each block run by the kernel path and by the fp32-linear reference on the kernel
        path's own input to that block; the rel-L2 of the two outputs per block."""
        errs = []
        for b in self.blocks:
            ref = self._block(b, x, ctx, True)
            x = self._block(b, x, ctx, False)
            errs.append(rel_l2(x, ref))
        return errs

    def _block(self, b: "_Block", x: torch.Tensor, ctx: torch.Tensor, reference: bool) -> torch.Tensor:
        c = self.cfg
        h, nh, d = c.hidden, c.heads, c.head_dim
        s = x.shape[0]

        def lin(l, t):
            return l.reference(t) if reference else l(t)

        fused = c.fused_glue and not reference

        def norm(t, w, rope):
            """RMSNorm over the hidden dim (then the rotary embedding): one library kernel, in place, on the kernel
            path; torch rms_norm and the complex multiply on the reference path."""
            if fused:
                return ops.rmsnorm_rope_rows(t, w, rope, d, eps=1e-6, out=t).view(-1, nh, d)
            t = F.rms_norm(t, (h,), w, eps=1e-6).view(-1, nh, d)
            return _rope(t, rope) if rope is not None else t

        m = b.mod
        if fused:
            return self._block_fused(b, x, ctx, norm)
        y = torch.addcmul(m[0], F.layer_norm(x, (h,), eps=1e-6), 1.0 + m[1])
        q = norm(lin(b.lin["q"], y), b.norm_q, self.rope)
        k = norm(lin(b.lin["k"], y), b.norm_k, self.rope)
        v = lin(b.lin["v"], y).view(s, nh, d)
        a = F.scaled_dot_product_attention(q.transpose(0, 1)[None], k.transpose(0, 1)[None],
                                           v.transpose(0, 1)[None])[0].transpose(0, 1).reshape(s, h)
        x = torch.addcmul(x, m[2], lin(b.lin["o"], a))
        y = F.layer_norm(x, (h,), b.norm3_w, b.norm3_b, eps=1e-6)
        cq = norm(lin(b.lin["cq"], y), b.norm_cq, None)
        ck = norm(lin(b.lin["ck"], ctx), b.norm_ck, None)
        cv = lin(b.lin["cv"], ctx).view(-1, nh, d)
        a = F.scaled_dot_product_attention(cq.transpose(0, 1)[None], ck.transpose(0, 1)[None],
                                           cv.transpose(0, 1)[None])[0].transpose(0, 1).reshape(s, h)
        x = x + lin(b.lin["co"], a)
        y = torch.addcmul(m[3], F.layer_norm(x, (h,), eps=1e-6), 1.0 + m[4])
        x = torch.addcmul(x, m[5], lin(b.lin["ff2"], F.gelu(lin(b.lin["ff1"], y), approximate="tanh")))
        return x

    def _block_fused(self, b: "_Block", x: torch.Tensor, ctx: torch.Tensor, norm) -> torch.Tensor:
        """The kernel path's block: the modulated layer norms inside the QKV and MLP-up activation kernels, the q/k
        norm + rotary kernel, GELU and the residual updates in the GEMM epilogues (the cross-attention residual as a
        gated residual with gate 1: bf16(x + y), torch's bf16 add)."""
        c = self.cfg
        h, nh, d = c.hidden, c.heads, c.head_dim
        s = x.shape[0]
        m = b.mod
        L = b.lin
        q = norm(L["q"].op(x, "plain", shift=m[0], scale=m[1]), b.norm_q, self.rope)
        k = norm(L["k"].op(x, "plain", shift=m[0], scale=m[1]), b.norm_k, self.rope)
        v = L["v"].op(x, "plain", shift=m[0], scale=m[1]).view(s, nh, d)
        a = F.scaled_dot_product_attention(q.transpose(0, 1)[None], k.transpose(0, 1)[None],
                                           v.transpose(0, 1)[None])[0].transpose(0, 1).reshape(s, h)
        x = L["o"].op(a, "gated", residual=x, gate=m[2])
        y = F.layer_norm(x, (h,), b.norm3_w, b.norm3_b, eps=1e-6)
        cq = norm(L["cq"](y), b.norm_cq, None)
        ck = norm(L["ck"](ctx), b.norm_ck, None)
        cv = L["cv"](ctx).view(-1, nh, d)
        a = F.scaled_dot_product_attention(cq.transpose(0, 1)[None], ck.transpose(0, 1)[None],
                                           cv.transpose(0, 1)[None])[0].transpose(0, 1).reshape(s, h)
        x = L["co"].op(a, "gated", residual=x, gate=self.one)
        g = L["ff1"].op(x, "gelu", shift=m[3], scale=m[4])
        return L["ff2"].op(g, "gated", residual=x, gate=m[5])

    def inputs(self, seed: int = 1):
        c = self.cfg
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        x = torch.randn(c.tokens, c.hidden, generator=g, device=self.device).to(torch.bfloat16)
        ctx = torch.randn(c.ctx_tokens, c.hidden, generator=g, device=self.device).to(torch.bfloat16)
        return x, ctx
