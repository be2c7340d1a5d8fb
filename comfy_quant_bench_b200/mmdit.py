"""Qwen-Image-like dual-stream MMDiT denoise step with every linear on the W4A8 affine path (random init).

This is the model-level workload of the quantized-linear path: a stack of dual-stream (image + text) MMDiT
blocks whose linears - per-stream adaLN modulation, QKV, attention output, MLP up and down - all run
``ops.w4a8_affine_linear`` (ConvRot-256 rotation + per-token int8 activations, packed uint4 weights with bf16
per-128-group scale/zero, tcgen05 GEMM).  The block follows the usual MMDiT layout (SD3 / Flux / Qwen-Image):

    mod   = Linear(silu(temb))                    -> shift1, scale1, gate1, shift2, scale2, gate2 per stream
    x_n   = LayerNorm(x) * (1 + scale1) + shift1  (no affine)
    q,k,v = Linear_qkv(x_n) per stream, RMSNorm(q), RMSNorm(k) per head, rotary embedding on q, k
    joint attention over [text; image] tokens (torch scaled_dot_product_attention)
    x     = x + gate1 * Linear_out(attn)
    x     = x + gate2 * Linear_fc2(gelu_tanh(Linear_fc1(LayerNorm(x) * (1 + scale2) + shift2)))

Attention is a torch op (scaled_dot_product_attention).  On the kernel path the rest of the glue runs inside the
library's kernels: the layer norm + modulation before the QKV and MLP-up linears in the activation kernel
(``ops.w4a8_affine_linear_lnmod`` / ``ops.w4a8_affine_linear_op``), the GELU after MLP-up and the two gated residuals
in the GEMM epilogues (``ops.w4a8_affine_linear_op``), the q/k RMSNorm + rotary embedding + joint attention layout as
one kernel (``ops.qkv_rmsnorm_rope``), writing q, k, v token-major so that the attention's output is already the
[tokens, hidden] rows of the output projection (``ops.heads_to_rows`` copies it when the attention returns head-major
memory); ``fused_glue=False`` runs them as torch ops instead.  The text stream's linears (256 tokens: few output
tiles, latency-bound) run on a second CUDA stream that joins the main one only at the joint attention, so they
overlap the image stream's GEMMs (``text_side_stream``).  Weights are drawn N(0, 0.02) per linear from a
seeded generator, quantized on the device with the library's weight kernel, and only the packed form is kept.

``MMDiT.step(..., reference=True)`` runs the same step with every linear replaced by a torch fp32 product of the
dequantized weights (W = (q - 8) * scale + zeros, in the rotated basis) and the dequantized activation codes that
the library's own activation kernel produced: it checks the GEMM and its epilogue inside the whole model.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import ops
from . import _lib


@dataclass(frozen=True)
class MMDiTConfig:
    blocks: int = 60
    hidden: int = 3072
    heads: int = 24
    mlp: int = 12288
    img_tokens: int = 4096        # 1024^2 latent with 2x2 patches
    txt_tokens: int = 256
    group_size: int = 128
    convrot_groupsize: int = 256
    quantize_modulation: bool = True   # every linear W4A8; the reference's profiles leave modulation unquantized
    fused_glue: bool = True            # kernel path: layer norm + modulation inside the activation kernel of the
                                       # QKV and MLP-up linears, q/k RMSNorm + rotary + attention layout in one kernel
    epilogue_gated: bool = True        # with fused_glue: the gated residuals in the GEMM epilogues of the
                                       # attention-output and MLP-down linears (False: torch addcmul)
    epilogue_gelu: bool = True         # with fused_glue: GELU in the MLP-up GEMM's epilogue (False: torch gelu)
    batched_modulation: bool = True    # with fused_glue and quantize_modulation: the adaLN modulation linears of every
                                       # block and stream, which all read the same timestep embedding, as one
                                       # few-token product over their joined weights at the start of the step
    token_major_qkv: bool = True       # with fused_glue: q, k, v in [tokens, heads, D] memory, passed to the attention
                                       # as strided views, whose output then is the [tokens, hidden] rows of the output
                                       # projection (False: head-major q, k, v and the head-to-rows copy)
    text_side_stream: bool = True      # with fused_glue and token_major_qkv: the text stream's linears on a second CUDA
                                       # stream, joined only at the attention, so its few-tile 256-token GEMMs can run
                                       # beside the image stream's GEMMs instead of after them
    text_split_k: bool | None = None   # whether the text stream's few-tile GEMMs split K over more CTAs; None: split on
                                       # one stream (where their idle SMs are idle), not beside the image stream

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


class QLinear:
    """One W4A8 affine linear (packed uint4 weight, bf16 scale/zero [K/128, N], prepared zero operand)."""

    def __init__(self, in_f: int, out_f: int, gen: torch.Generator, device, cfg: MMDiTConfig, bias: bool = True):
        w = torch.randn(out_f, in_f, generator=gen, device=device, dtype=torch.float32).mul_(0.02)
        self.qweight, self.scale, self.zeros = ops.quantize_affine_w4_weight(w, cfg.group_size, cfg.convrot_groupsize)
        del w
        self.zt = ops.prepare_affine_zeros(self.zeros, cfg.group_size)
        self.bias = (torch.randn(out_f, generator=gen, device=device, dtype=torch.float32) * 0.01).to(torch.bfloat16) if bias else None
        self.cfg = cfg
        self.in_f, self.out_f = in_f, out_f

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return ops.w4a8_affine_linear(x, self.qweight, self.scale, self.zeros, self.bias, self.cfg.group_size,
                                      self.cfg.convrot_groupsize, zeros_prepared=self.zt)

    def lnmod(self, x: torch.Tensor, shift: torch.Tensor, scale1p: torch.Tensor) -> torch.Tensor:
        """This linear of bf16(shift + bf16(layer_norm(x)) * scale1p), the norm and modulation fused into the
        activation kernel."""
        return ops.w4a8_affine_linear_lnmod(x, shift, scale1p, self.qweight, self.scale, self.zt, self.bias,
                                            self.cfg.group_size, self.cfg.convrot_groupsize, eps=1e-6)

    def op(self, x: torch.Tensor, out_op: str, *, residual=None, gate=None, shift=None, scale=None,
           split_k: bool = True) -> torch.Tensor:
        """This linear with the step after it in the GEMM's epilogue: ``plain``, ``gelu`` (tanh) or ``gated``
        (residual + gate * y); with shift / the modulation scale, the layer norm + modulation (by the bf16 1 + scale)
        before it in the activation kernel."""
        return ops.w4a8_affine_linear_op(x, self.qweight, self.scale, self.zt, self.bias, out_op=out_op,
                                         residual=residual, gate=gate, shift=shift, scale=scale,
                                         group_size=self.cfg.group_size, convrot_groupsize=self.cfg.convrot_groupsize,
                                         eps=1e-6, split_k=split_k)

    @classmethod
    def joined(cls, parts: list["QLinear"]) -> "QLinear":
        """One linear with the parts' output features in order (the same input; every output row is the same
        product as in its part).  The parts' packed weights, zero operands and biases become views of the joined
        tensors, so the packed weights are held once."""
        lin = cls.__new__(cls)
        lin.cfg, lin.in_f = parts[0].cfg, parts[0].in_f
        lin.out_f = sum(p.out_f for p in parts)
        lin.qweight = torch.cat([p.qweight for p in parts])
        lin.scale = torch.cat([p.scale for p in parts], dim=1)
        lin.zeros = torch.cat([p.zeros for p in parts], dim=1)
        lin.zt = torch.cat([p.zt for p in parts])
        lin.bias = torch.cat([p.bias for p in parts]) if parts[0].bias is not None else None
        off = 0
        for p in parts:
            p.qweight, p.zt = lin.qweight[off:off + p.out_f], lin.zt[off:off + p.out_f]
            if lin.bias is not None:
                p.bias = lin.bias[off:off + p.out_f]
            off += p.out_f
        return lin

    def dequantized_weight(self) -> torch.Tensor:
        """W in the rotated basis, fp32 [N, K]: (q - 8) * scale + zeros per 128-wide group."""
        q8 = self.qweight.view(torch.uint8)
        q = torch.stack((q8 & 15, q8 >> 4), dim=-1).reshape(self.out_f, self.in_f).float()
        g = self.cfg.group_size
        s = self.scale.float().t().repeat_interleave(g, dim=1)
        z = self.zeros.float().t().repeat_interleave(g, dim=1)
        return (q - 8.0) * s + z

    def reference(self, x: torch.Tensor) -> torch.Tensor:
        """The same linear in torch fp32 on the library's own activation codes (dequantized) and the dequantized
        weight; bf16 out."""
        x2 = x.reshape(-1, x.shape[-1]).to(torch.bfloat16).contiguous()
        q, sx, _ = ops.rotquant(x2, self.cfg.convrot_groupsize, _lib.CQ_ACT_INT8_ROW)
        m = x2.shape[0]
        xa = q[:m].float() * sx[:m, None]
        y = xa @ self.dequantized_weight().t()
        if self.bias is not None:
            y = y + self.bias.float()
        return y.to(torch.bfloat16).reshape(*x.shape[:-1], self.out_f)


class _Stream:
    """The per-stream (image or text) linears and norm weights of one block."""

    def __init__(self, gen, device, cfg: MMDiTConfig):
        h = cfg.hidden
        self.mod = QLinear(h, 6 * h, gen, device, cfg) if cfg.quantize_modulation else None
        self.mod_bf16 = None
        if not cfg.quantize_modulation:
            self.mod_bf16 = (torch.randn(6 * h, h, generator=gen, device=device) * 0.02).to(torch.bfloat16)
        self.qkv = QLinear(h, 3 * h, gen, device, cfg)
        self.out = QLinear(h, h, gen, device, cfg)
        self.fc1 = QLinear(h, cfg.mlp, gen, device, cfg)
        self.fc2 = QLinear(cfg.mlp, h, gen, device, cfg)
        self.q_norm = torch.ones(cfg.head_dim, device=device, dtype=torch.bfloat16)
        self.k_norm = torch.ones(cfg.head_dim, device=device, dtype=torch.bfloat16)


def _rope_table(n: int, dim: int, device, offset: int = 0) -> torch.Tensor:
    """Rotary factors exp(i * pos * 10000^(-2j/dim)) for positions offset..offset+n-1, complex64 [n, dim/2]."""
    inv = 1.0 / (10000.0 ** (torch.arange(0, dim, 2, device=device, dtype=torch.float32) / dim))
    pos = torch.arange(offset, offset + n, device=device, dtype=torch.float32)
    ang = torch.outer(pos, inv)
    return torch.complex(torch.cos(ang), torch.sin(ang))


def _apply_rope(x: torch.Tensor, rot: torch.Tensor) -> torch.Tensor:
    """Rotate interleaved pairs of the head dim: x [S, H, D] bf16 by rot [S, D/2] complex64 -> bf16."""
    xc = torch.view_as_complex(x.float().reshape(*x.shape[:-1], -1, 2))
    return torch.view_as_real(xc * rot[:, None, :]).reshape(x.shape).to(torch.bfloat16)


class MMDiT:
    def __init__(self, cfg: MMDiTConfig = MMDiTConfig(), device="cuda", seed: int = 0):
        self.cfg = cfg
        self.device = torch.device(device)
        gen = torch.Generator(device=self.device)
        gen.manual_seed(seed)
        self.blocks = [(_Stream(gen, self.device, cfg), _Stream(gen, self.device, cfg)) for _ in range(cfg.blocks)]
        # every block's image- and text-stream modulation linear, joined (block order, image stream first)
        self.mod_all = QLinear.joined([st.mod for blk in self.blocks for st in blk]) if cfg.quantize_modulation else None
        d = cfg.head_dim
        self.rope_txt = _rope_table(cfg.txt_tokens, d, self.device)
        self.rope_img = _rope_table(cfg.img_tokens, d, self.device, offset=cfg.txt_tokens)
        self._side = None     # the text stream's CUDA stream (text_side_stream)
        self._qkv_bufs = None # two token-major q, k, v sets, alternating by block (text_side_stream)

    # ---- per-linear dispatch (kernel path or torch reference) ----
    @staticmethod
    def _lin(layer: QLinear, x: torch.Tensor, reference: bool) -> torch.Tensor:
        return layer.reference(x) if reference else layer(x)

    def _mod(self, st: _Stream, temb_act: torch.Tensor, reference: bool) -> torch.Tensor:
        if st.mod is not None:
            return self._lin(st.mod, temb_act, reference)
        return F.linear(temb_act, st.mod_bf16)

    def linears(self):
        """Every QLinear of the model, in block order."""
        out = []
        for img, txt in self.blocks:
            for st in (img, txt):
                out += [l for l in (st.mod, st.qkv, st.out, st.fc1, st.fc2) if l is not None]
        return out

    def launches_per_step(self) -> int:
        """The library's kernel launches in one kernel-path step (attention and the timestep embedding's torch ops
        not counted)."""
        c = self.cfg
        n = 0
        for m in (c.img_tokens, c.txt_tokens):
            # the text stream's linears on the side stream never split K: activation kernel + GEMM
            unsplit = m == c.txt_tokens and not self._text_split_k(self._two_streams(False))
            n += sum(2 if unsplit else ops.affine_linear_launches(m, nn, kk) for nn, kk in
                     ((3 * c.hidden, c.hidden), (c.hidden, c.hidden), (c.mlp, c.hidden), (c.hidden, c.mlp)))
            n += 1 if c.fused_glue else 0                                        # q/k norm + rotary + layout
        n *= c.blocks
        if c.fused_glue and not c.token_major_qkv:
            n += c.blocks                                                        # head-major output to rows
        if self.mod_all is not None:
            n += 2 if (c.batched_modulation and c.fused_glue) else 2 * 2 * c.blocks
        return n

    def weight_bytes(self) -> int:
        return sum(l.qweight.numel() + 2 * l.scale.numel() * 2 + l.zt.numel() * 2 for l in self.linears())

    def linear_int_ops(self) -> float:
        """2 * M * N * K summed over the quantized linears of one step."""
        c = self.cfg
        tot = 0.0
        for img, txt in self.blocks:
            for st, m in ((img, c.img_tokens), (txt, c.txt_tokens)):
                if st.mod is not None:
                    tot += 2.0 * 1 * st.mod.out_f * st.mod.in_f
                for l in (st.qkv, st.out, st.fc1, st.fc2):
                    tot += 2.0 * m * l.out_f * l.in_f
        return tot

    def attention_flops(self) -> float:
        c = self.cfg
        s = c.img_tokens + c.txt_tokens
        return 4.0 * s * s * c.hidden * c.blocks

    def step(self, img: torch.Tensor, txt: torch.Tensor, temb: torch.Tensor, reference: bool = False):
        """One denoise step: img [S_img, hidden], txt [S_txt, hidden], temb [1, hidden] (bf16).  Returns img, txt.

        The glue around the linears stays in bf16 (fp32 inside the norms and the rotary rotation): layer norm,
        modulation as one fused multiply-add, q/k/v written straight into the joint [heads, tokens, dim]
        attention layout, GELU on bf16, gated residual as one fused multiply-add.  With ``fused_glue`` (kernel path
        only) the layer norm + modulation run inside the activation kernel of the QKV and MLP-up linears and the
        q/k RMSNorm + rotary + layout copies are one kernel; the reference path always runs the torch ops."""
        temb_act = F.silu(temb.float()).to(torch.bfloat16)
        c = self.cfg
        mods = None
        if c.batched_modulation and c.fused_glue and self.mod_all is not None and not reference:
            # [1, 2 * blocks * 6 * hidden]: one activation kernel and one weight stream for all modulation linears
            mods = self.mod_all(temb_act).split(6 * c.hidden, dim=-1)
        if self._two_streams(reference):
            return self._step_two_streams(img, txt, temb_act, mods)
        for i, blk in enumerate(self.blocks):
            img, txt = self._block(blk, img, txt, temb_act, reference, None if mods is None else mods[2 * i:2 * i + 2])
        return img, txt

    def _text_split_k(self, two_streams: bool) -> bool:
        c = self.cfg
        return (not two_streams) if c.text_split_k is None else c.text_split_k

    def _two_streams(self, reference: bool) -> bool:
        c = self.cfg
        return c.text_side_stream and c.fused_glue and c.token_major_qkv and c.epilogue_gated and c.epilogue_gelu \
            and not reference

    def _step_two_streams(self, img: torch.Tensor, txt: torch.Tensor, temb_act: torch.Tensor, mods):
        """The fused step with the text stream's work on a second stream.  Per block the text stream waits for the
        main stream once (the joint attention's output) and the main stream waits for the text stream once (the
        text q, k, v before the attention).  q, k, v live in two persistent buffer sets used by alternate blocks:
        block i + 2 rewrites block i's set only after the attention of block i, which both streams are ordered
        after.  The attention output is marked as used by the text stream, so the allocator does not hand its
        memory out again before the text stream has read it.  The step ends with the main stream waiting for the
        text stream.  By default the text linears do not split K: beside the image stream's GEMMs the SMs that their
        few output tiles leave free are in use (60 blocks: 62.1-62.7 ms per step against 63.6-65.0 ms with split K)."""
        c = self.cfg
        h, nh, d = c.hidden, c.heads, c.head_dim
        main = torch.cuda.current_stream(self.device)
        if self._side is None:
            self._side = torch.cuda.Stream(self.device)
        side = self._side
        st_txt, st_img = txt.shape[0], img.shape[0]
        s_all = st_txt + st_img
        if self._qkv_bufs is None or self._qkv_bufs[0][0].shape[2] != s_all:
            self._qkv_bufs = [tuple(torch.empty(1, s_all, nh, d, dtype=torch.bfloat16, device=self.device).transpose(1, 2)
                                    for _ in range(3)) for _ in range(2)]
        if mods is None:
            mods = []
            for si, st in self.blocks:
                mods += [self._mod(si, temb_act, False), self._mod(st, temb_act, False)]
        tsk = self._text_split_k(True)
        side.wait_stream(main)              # the step's inputs and the modulation outputs
        for i, (si, st) in enumerate(self.blocks):
            q, k, v = self._qkv_bufs[i % 2]
            mi, mt = mods[2 * i].chunk(6, dim=-1), mods[2 * i + 1].chunk(6, dim=-1)
            with torch.cuda.stream(side):
                y = st.qkv.op(txt, "plain", shift=mt[0], scale=mt[1], split_k=tsk)
                ops.qkv_rmsnorm_rope(y, st.q_norm, st.k_norm, self.rope_txt, q, k, v, 0, eps=1e-6)
            y = si.qkv.op(img, "plain", shift=mi[0], scale=mi[1])
            ops.qkv_rmsnorm_rope(y, si.q_norm, si.k_norm, self.rope_img, q, k, v, st_txt, eps=1e-6)
            main.wait_stream(side)
            o = F.scaled_dot_product_attention(q, k, v)
            if o.transpose(1, 2).is_contiguous():
                a = o.transpose(1, 2).reshape(s_all, h)
            else:
                a = torch.empty(s_all, h, dtype=torch.bfloat16, device=self.device)
                ops.heads_to_rows(o, [a], 0, h)
            a.record_stream(side)
            side.wait_stream(main)
            with torch.cuda.stream(side):
                x = st.out.op(a[:st_txt], "gated", residual=txt, gate=mt[2], split_k=tsk)
                f = st.fc1.op(x, "gelu", shift=mt[3], scale=mt[4], split_k=tsk)
                txt = st.fc2.op(f, "gated", residual=x, gate=mt[5], split_k=tsk)
            x = si.out.op(a[st_txt:], "gated", residual=img, gate=mi[2])
            f = si.fc1.op(x, "gelu", shift=mi[3], scale=mi[4])
            img = si.fc2.op(f, "gated", residual=x, gate=mi[5])
        main.wait_stream(side)
        txt.record_stream(main)
        return img, txt

    def block_errors(self, img: torch.Tensor, txt: torch.Tensor, temb: torch.Tensor) -> list[float]:
        """Teacher-forced check: every block run by the kernel path and by the fp32-linear reference on the kernel
        path's own input to that block; the rel-L2 of the two image-stream outputs (the larger stream) per block."""
        temb_act = F.silu(temb.float()).to(torch.bfloat16)
        errs = []
        for blk in self.blocks:
            ref_img, _ = self._block(blk, img, txt, temb_act, True)
            img, txt = self._block(blk, img, txt, temb_act, False)
            errs.append(rel_l2(img, ref_img))
        return errs

    def _block(self, blk, img: torch.Tensor, txt: torch.Tensor, temb_act: torch.Tensor, reference: bool, mods=None):
        """One dual-stream block on (img, txt); returns the new (img, txt).  ``mods``: the block's (image, text)
        modulation outputs when computed ahead for the whole step."""
        c = self.cfg
        h, nh, d = c.hidden, c.heads, c.head_dim
        fused = c.fused_glue and not reference
        st_txt, st_img = txt.shape[0], img.shape[0]
        s_all = st_txt + st_img
        if fused and c.token_major_qkv:
            q, k, v = (torch.empty(1, s_all, nh, d, dtype=torch.bfloat16, device=img.device).transpose(1, 2)
                       for _ in range(3))
        else:
            q = torch.empty(1, nh, s_all, d, dtype=torch.bfloat16, device=img.device)
            k = torch.empty_like(q)
            v = torch.empty_like(q)
        si, st = blk
        mi = (mods[0] if mods is not None else self._mod(si, temb_act, reference)).chunk(6, dim=-1)
        mt = (mods[1] if mods is not None else self._mod(st, temb_act, reference)).chunk(6, dim=-1)
        tsk = self._text_split_k(False)
        for x, s, m, rot, lo, hi, sk in ((txt, st, mt, self.rope_txt, 0, st_txt, tsk),
                                         (img, si, mi, self.rope_img, st_txt, s_all, True)):
            if fused:
                y = s.qkv.op(x, "plain", shift=m[0], scale=m[1], split_k=sk)
                ops.qkv_rmsnorm_rope(y, s.q_norm, s.k_norm, rot, q, k, v, lo, eps=1e-6)
                continue
            xn = torch.addcmul(m[0], F.layer_norm(x, (h,), eps=1e-6), 1.0 + m[1])
            y = self._lin(s.qkv, xn, reference).view(x.shape[0], 3, nh, d)
            q[0, :, lo:hi] = _apply_rope(F.rms_norm(y[:, 0], (d,), s.q_norm, eps=1e-6), rot).transpose(0, 1)
            k[0, :, lo:hi] = _apply_rope(F.rms_norm(y[:, 1], (d,), s.k_norm, eps=1e-6), rot).transpose(0, 1)
            v[0, :, lo:hi] = y[:, 2].transpose(0, 1)
        if fused:
            o = F.scaled_dot_product_attention(q, k, v)
            if o.transpose(1, 2).is_contiguous():
                a = o.transpose(1, 2).reshape(s_all, h)   # token-major output: already the [tokens, hidden] rows
            else:
                a = torch.empty(s_all, h, dtype=torch.bfloat16, device=img.device)
                ops.heads_to_rows(o, [a], 0, h)
        else:
            a = F.scaled_dot_product_attention(q, k, v)[0].transpose(0, 1).reshape(s_all, h)
        new = []
        for x, s, m, att, sk in ((txt, st, mt, a[:st_txt], tsk), (img, si, mi, a[st_txt:], True)):
            if fused:
                # layer norm + modulation in the activation kernels; GELU and the gated residuals in the GEMM
                # epilogues, or as torch ops on the linears' outputs
                if c.epilogue_gated:
                    x = s.out.op(att, "gated", residual=x, gate=m[2], split_k=sk)
                else:
                    x = torch.addcmul(x, m[2], s.out(att))
                if c.epilogue_gelu:
                    f = s.fc1.op(x, "gelu", shift=m[3], scale=m[4], split_k=sk)
                else:
                    f = F.gelu(s.fc1.lnmod(x, m[3], 1.0 + m[4]), approximate="tanh")
                new.append(s.fc2.op(f, "gated", residual=x, gate=m[5], split_k=sk) if c.epilogue_gated
                           else torch.addcmul(x, m[5], s.fc2(f)))
                continue
            x = torch.addcmul(x, m[2], self._lin(s.out, att, reference))
            xn = torch.addcmul(m[3], F.layer_norm(x, (h,), eps=1e-6), 1.0 + m[4])
            f = F.gelu(self._lin(s.fc1, xn, reference), approximate="tanh")
            new.append(torch.addcmul(x, m[5], self._lin(s.fc2, f, reference)))
        txt, img = new
        return img, txt

    def inputs(self, seed: int = 1):
        c = self.cfg
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        img = torch.randn(c.img_tokens, c.hidden, generator=g, device=self.device).to(torch.bfloat16)
        txt = torch.randn(c.txt_tokens, c.hidden, generator=g, device=self.device).to(torch.bfloat16)
        temb = torch.randn(1, c.hidden, generator=g, device=self.device).to(torch.bfloat16)
        return img, txt, temb


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a64, b64 = a.double(), b.double()
    return float((a64 - b64).norm() / b64.norm().clamp_min(1e-30))
