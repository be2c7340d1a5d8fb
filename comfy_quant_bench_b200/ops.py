"""Torch-level operators of the quantized-linear hot path, mirroring comfy-kitchen's CUDA backend API.

Names, argument meaning and error behaviour follow the call sites in comfy-quant-bench:

* ``quantize_int4_rowwise_convrot64(x, convrot_groupsize)`` (``g64_quant_test.py:105-112``,
  ``node/__init__.py:148``) and ``swiglu_quantize_int4_rowwise_convrot64(h)`` (``tools/ck_swiglu/swiglu_quant.cu:111-137``);
* ``quant(x, group, swiglu, pad)``: the reference's own per-group activation quantizer
  (``experiments/qwen21-kernel/kernels/g64_quant.cu:113-130``);
* ``quantize_convrot_w4a4_weight`` / ``quantize_int8_convrot_weight`` (``tools/_formats.py:72-76, 149-156``) and
  ``quantize_affine_w4_weight`` (the awq_w4a16 layout, ``tools/_formats.py:191-212``) - the converter kernels;
* ``int4_linear`` (``g64_bench6.py:109``), ``convrot_w4a4_linear`` (``patches/comfy_kitchen_swiglu_w4a4_fused.patch:41-95``),
  ``int8_linear`` (``tools/_native_probe.py:234-255``) and ``w4a8_affine_linear`` (W4A8 on awq-layout weights).

Every op runs the CUDA kernels of libcq_b200.so on the input's device and the current torch stream.  Inputs
on the CPU or on a non-sm_100 device are rejected: there is no eager fallback.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

ROT_GROUPS = (0, 16, 64, 256)
INT4_GROUP_SIZE = 64          # comfy-kitchen's loader constant (tools/_formats.py:57-59)


def _stream(dev: torch.device):
    return torch.cuda.current_stream(dev).cuda_stream


def _ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def _require_cuda(*ts: torch.Tensor | None) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("comfy_quant_bench_b200 ops run on CUDA tensors only (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def _check_rot(g: int) -> int:
    g = int(g)
    if g not in ROT_GROUPS:
        raise ValueError(f"convrot_groupsize must be one of {ROT_GROUPS[1:]} (or 0 for none), got {g}")
    return g


def _as2d(x: torch.Tensor) -> torch.Tensor:
    x2 = x.reshape(-1, x.shape[-1])
    if x2.dtype != torch.bfloat16:
        x2 = x2.to(torch.bfloat16)
    return x2.contiguous()


def _bias_bf16(bias: torch.Tensor | None) -> torch.Tensor | None:
    if bias is None:
        return None
    return bias.to(torch.bfloat16).contiguous()


# --------------------------------------------------------------------------------------------------
# activation quantizers
# --------------------------------------------------------------------------------------------------

def rotquant(x: torch.Tensor, rot_group: int, mode: int, *, swiglu: bool = False, act_group: int = 0,
             m_pad: int | None = None, int4_as_int8: bool = False, group_sums: bool = False, kperm: bool = False):
    """Raw activation stage: returns (q, scale, gsplit or None).  See cq_rotquant in include/cq_b200.h.

    ``group_sums`` also returns the per-token code sums over 128-wide K groups, split into bf16 hi/lo parts
    ([M_pad, cq_group_sum_cols(K)]; the zero-point operand of ``gemm_affine``).

    ``kperm`` writes int8 codes with each 8-column block of K in the order 0,2,4,6,1,3,5,7 (the order the
    int4-weight GEMMs unpack into; pass ``a_kperm=True`` to them)."""
    dev = _require_cuda(x)
    x2 = _as2d(x)
    m = x2.shape[0]
    k = x2.shape[1] // 2 if swiglu else x2.shape[1]
    mp = m if m_pad is None else int(m_pad)
    if mode == _lib.CQ_ACT_INT8_ROW or int4_as_int8:
        q = torch.empty(mp, k, dtype=torch.int8, device=dev)
    else:
        q = torch.empty(mp, k // 2, dtype=torch.int8, device=dev)
    if mode == _lib.CQ_ACT_INT4_GROUP:
        scale = torch.empty(k // act_group, mp, dtype=torch.float32, device=dev)
    else:
        scale = torch.empty(mp, dtype=torch.float32, device=dev)
    gs = torch.empty(mp, int(_lib.load().cq_group_sum_cols(k)), dtype=torch.bfloat16, device=dev) if group_sums else None
    flags = (_lib.CQ_Q_INT8_CODES if int4_as_int8 else 0) | (_lib.CQ_Q_KPERM if kperm else 0)
    _lib.call("cq_rotquant", _ptr(x2), m, k, _check_rot(rot_group), int(bool(swiglu)), int(mode), int(act_group), mp,
              flags, _ptr(q), _ptr(scale), _ptr(gs), _stream(dev))
    return q, scale, gs


def rotquant_absmax(x: torch.Tensor, rot_group: int, *, m_pad: int | None = None) -> torch.Tensor:
    """First phase of per-token int8 activations whose K columns are split over ranks: f32 [2, M_pad] holding each
    token's NaN-ignoring max |rotated x| over these columns and a NaN flag.  Combine the ranks' arrays with an
    all-reduce MAX, then call ``rotquant_scaled`` (cq_rotquant_absmax)."""
    dev = _require_cuda(x)
    x2 = _as2d(x)
    m, k = x2.shape
    mp = m if m_pad is None else int(m_pad)
    amax = torch.empty(2, mp, dtype=torch.float32, device=dev)
    _lib.call("cq_rotquant_absmax", _ptr(x2), m, k, _check_rot(rot_group), mp, _ptr(amax), _stream(dev))
    return amax


def rotquant_scaled(x: torch.Tensor, rot_group: int, amax: torch.Tensor, *, m_pad: int | None = None,
                    group_sums: bool = False, kperm: bool = False):
    """Second phase: per-token int8 codes of these columns with the scale of the whole row, from the combined
    ``amax`` [2, M_pad].  Returns (q, scale, gsplit or None) as ``rotquant`` (cq_rotquant_scaled)."""
    dev = _require_cuda(x, amax)
    x2 = _as2d(x)
    m, k = x2.shape
    mp = m if m_pad is None else int(m_pad)
    if amax.dtype != torch.float32 or tuple(amax.shape) != (2, mp) or not amax.is_contiguous():
        raise ValueError(f"amax must be contiguous f32 [2, {mp}]")
    q = torch.empty(mp, k, dtype=torch.int8, device=dev)
    scale = torch.empty(mp, dtype=torch.float32, device=dev)
    gs = torch.empty(mp, int(_lib.load().cq_group_sum_cols(k)), dtype=torch.bfloat16, device=dev) if group_sums else None
    _lib.call("cq_rotquant_scaled", _ptr(x2), m, k, _check_rot(rot_group), _ptr(amax), mp,
              _lib.CQ_Q_KPERM if kperm else 0, _ptr(q), _ptr(scale), _ptr(gs), _stream(dev))
    return q, scale, gs


def quantize_int4_rowwise_convrot64(x: torch.Tensor, convrot_groupsize: int = 256):
    """Rotate (block Hadamard) + per-token int4: (q [M, K/2] int8 packed, scale [M] f32)."""
    q, s, _ = rotquant(x, convrot_groupsize, _lib.CQ_ACT_INT4_ROW)
    return q, s


def swiglu_quantize_int4_rowwise_convrot64(h: torch.Tensor):
    """silu(gate)*up (fp32, rounded once to bf16) + ConvRot-256 + per-token int4 from h = [gate | up]."""
    if h.shape[-1] % 2:
        raise ValueError("h must hold gate | up halves")
    k = h.shape[-1] // 2
    if k % 256 or k > 16384:
        raise ValueError("K must be a multiple of 256 and <= 16384")
    q, s, _ = rotquant(h, 256, _lib.CQ_ACT_INT4_ROW, swiglu=True)
    return q, s


def quantize_int8_rowwise_convrot(x: torch.Tensor, convrot_groupsize: int = 256, *, swiglu: bool = False):
    """Rotate + per-token int8: (q [M, K] int8, scale [M] f32)."""
    q, s, _ = rotquant(x, convrot_groupsize, _lib.CQ_ACT_INT8_ROW, swiglu=swiglu)
    return q, s


def quant(x: torch.Tensor, group: int, swiglu: bool = False, pad: int = 128):
    """The reference's per-group quantizer: ConvRot-256, int4 per (token, group) with bf16-up scales.

    Returns q [M_pad, K/2] packed and s [K/group, M_pad] f32; rows M..M_pad-1 are zero.
    """
    if group not in (64, 128):
        raise ValueError("group 64 or 128")
    m = x.reshape(-1, x.shape[-1]).shape[0]
    mp = (m + pad - 1) // pad * pad
    q, s, _ = rotquant(x, 256, _lib.CQ_ACT_INT4_GROUP, swiglu=swiglu, act_group=group, m_pad=mp)
    return q, s


# --------------------------------------------------------------------------------------------------
# weight quantizers (the converter's rotate-and-quantize step)
# --------------------------------------------------------------------------------------------------

def _weight_in(weight: torch.Tensor):
    _require_cuda(weight)
    if weight.dim() != 2:
        raise ValueError("weight must be 2-D [N, K]")
    if weight.dtype == torch.bfloat16:
        return weight.contiguous(), 1
    return weight.to(torch.float32).contiguous(), 0


def quantize_convrot_w4a4_weight(weight: torch.Tensor, convrot_groupsize: int = 256,
                                 quant_group_size: int = INT4_GROUP_SIZE, stochastic_rounding: int = 0):
    """ConvRot W4A4 weight: (qdata [N, K/2] int8 packed signed int4, scale [N] f32)."""
    if quant_group_size != INT4_GROUP_SIZE:
        raise ValueError(f"int4 MMA kernel requires quant_group_size {INT4_GROUP_SIZE}")
    if stochastic_rounding:
        raise ValueError("stochastic_rounding is not supported (the converters always pass 0)")
    w, is_bf16 = _weight_in(weight)
    n, k = w.shape
    q = torch.empty(n, k // 2, dtype=torch.int8, device=w.device)
    s = torch.empty(n, dtype=torch.float32, device=w.device)
    _lib.call("cq_weight_rotquant", _ptr(w), is_bf16, n, k, _check_rot(convrot_groupsize), _lib.CQ_W_INT4_ROW, 0,
              _ptr(q), _ptr(s), None, _stream(w.device))
    return q, s


def quantize_int8_convrot_weight(weight: torch.Tensor, group_size: int = 256):
    """int8_tensorwise (ConvRot when group_size > 0): (qdata [N, K] int8, scale [N, 1] f32)."""
    w, is_bf16 = _weight_in(weight)
    n, k = w.shape
    q = torch.empty(n, k, dtype=torch.int8, device=w.device)
    s = torch.empty(n, 1, dtype=torch.float32, device=w.device)
    _lib.call("cq_weight_rotquant", _ptr(w), is_bf16, n, k, _check_rot(group_size), _lib.CQ_W_INT8_ROW, 0,
              _ptr(q), _ptr(s), None, _stream(w.device))
    return q, s


def quantize_affine_w4_weight(weight: torch.Tensor, group_size: int = 128, convrot_groupsize: int = 0):
    """Asymmetric per-group int4 in the awq_w4a16 layout: W ~ (q - 8) * scale + zeros.

    Returns (qweight [N, K/2] int8 packed uint4, scale bf16 [K/G, N], zeros bf16 [K/G, N]).
    """
    w, is_bf16 = _weight_in(weight)
    n, k = w.shape
    q = torch.empty(n, k // 2, dtype=torch.int8, device=w.device)
    s = torch.empty(k // group_size, n, dtype=torch.bfloat16, device=w.device)
    z = torch.empty(k // group_size, n, dtype=torch.bfloat16, device=w.device)
    _lib.call("cq_weight_rotquant", _ptr(w), is_bf16, n, k, _check_rot(convrot_groupsize),
              _lib.CQ_W_AFFINE_INT4_GROUP, int(group_size), _ptr(q), _ptr(s), _ptr(z), _stream(w.device))
    return q, s, z


def quantize_int4_groupwise_weight(weight: torch.Tensor, group_size: int = 128, convrot_groupsize: int = 256):
    """Per-group symmetric int4 with bf16-up scales (the reference's pol 1/3/4 weights): (q packed, s [K/G, N])."""
    w, is_bf16 = _weight_in(weight)
    n, k = w.shape
    q = torch.empty(n, k // 2, dtype=torch.int8, device=w.device)
    s = torch.empty(k // group_size, n, dtype=torch.float32, device=w.device)
    _lib.call("cq_weight_rotquant", _ptr(w), is_bf16, n, k, _check_rot(convrot_groupsize),
              _lib.CQ_W_INT4_GROUP_BF16UP, int(group_size), _ptr(q), _ptr(s), None, _stream(w.device))
    return q, s


# --------------------------------------------------------------------------------------------------
# GEMMs and fused linears
# --------------------------------------------------------------------------------------------------

def gemm_rowcol(a: torch.Tensor, sa: torch.Tensor, b: torch.Tensor, sb: torch.Tensor, bias=None, *,
                b_int8: bool = False, a_kperm: bool = False) -> torch.Tensor:
    """out = (a @ b^T) * sa[:, None] * sb[None, :] + bias -> bf16.  a int8 codes [M, K]; b packed int4 or int8."""
    dev = _require_cuda(a, sa, b, sb, bias)
    m, k = a.shape
    n = b.shape[0]
    if (b.shape[1] if b_int8 else 2 * b.shape[1]) != k:
        raise ValueError(f"Input K={k} does not match weight K={b.shape[1] * (1 if b_int8 else 2)}")
    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    bias = _bias_bf16(bias)
    _lib.call("cq_gemm_rowcol", _ptr(a), int(bool(a_kperm)), _ptr(sa.float().contiguous()), _ptr(b),
              _lib.CQ_B_INT8 if b_int8 else _lib.CQ_B_INT4_SIGNED, _ptr(sb.float().contiguous()), _ptr(bias),
              _ptr(out), m, n, k, _stream(dev))
    return out


def int4_linear(qact: torch.Tensor, qweight: torch.Tensor, x_scale: torch.Tensor, wscales: torch.Tensor,
                bias: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """Packed int4 activations x packed int4 weights, row x column scales (comfy-kitchen int4_linear)."""
    dev = _require_cuda(qact, qweight, x_scale, wscales, bias)
    m, kh = qact.shape
    a8 = torch.empty(m, 2 * kh, dtype=torch.int8, device=dev)
    _lib.call("cq_unpack_int4", _ptr(qact.contiguous()), m, 2 * kh, _ptr(a8), _stream(dev))
    out = gemm_rowcol(a8, x_scale.reshape(-1), qweight.contiguous(), wscales.reshape(-1), bias)
    return out if out_dtype == torch.bfloat16 else out.to(out_dtype)


def gemm_groupwise(a: torch.Tensor, sa_g: torch.Tensor, b: torch.Tensor, sb_g: torch.Tensor, bias=None, *,
                   m: int | None = None, a_kperm: bool = False) -> torch.Tensor:
    """Per-group scales on both sides (the reference GEMM's policy 4, ``g64_gemm6.cu:5-7, 228-229``):
    out = sum_g round(P_g * sb_g[g, n]) * sa_g[g, m] + bias -> bf16 [m, N], accumulated over the 128-wide groups
    in order.  a int4 values as int8 codes [M_pad, K]; sa_g f32 [K/128, M_pad]; b packed int4 [N, K/2];
    sb_g f32 [K/128, N]."""
    dev = _require_cuda(a, sa_g, b, sb_g, bias)
    mp, k = a.shape
    m = mp if m is None else int(m)
    n = b.shape[0]
    if 2 * b.shape[1] != k:
        raise ValueError(f"Input K={k} does not match weight K={2 * b.shape[1]}")
    if sa_g.shape[0] != k // 128 or sb_g.shape != (k // 128, n):
        raise ValueError("sa_g must be [K/128, M_pad] and sb_g [K/128, N]")
    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    sa_g = sa_g.float().contiguous()
    _lib.call("cq_gemm_groupwise", _ptr(a), int(bool(a_kperm)), _ptr(sa_g), sa_g.shape[1], _ptr(b),
              _ptr(sb_g.float().contiguous()), _ptr(_bias_bf16(bias)), _ptr(out), m, n, k, 128, _stream(dev))
    return out


def gemm(a: torch.Tensor, b: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, ca=None, cw=None, bias=None,
         pol: int = 0, cfg=None) -> torch.Tensor:
    """The reference GEMM's interface, ``g64_gemm6.gemm(a, b, sa, sb, ca, cw, bias, pol, cfg)``
    (``experiments/qwen21-kernel/kernels/g64_gemm6.cu:383-411``), for the policies built here:

    * pol 0: row x column, sa [M] f32, sb [N] f32;
    * pol 4: g128 x g128, sa [K/128, M_pad] f32 (the per-group quantizer's layout), sb [K/128, N] f32;
    * pol 5 / 7: integer weight ratios cw int32 [K/64, N] / [K/128, N] summed in int32, sa [M], sb [N] f32;
    * pol 15 / 17: the same with cw uint8.

    a packed int4 [M_pad, K/2]; b packed int4 [N, K/2]; bias bf16 [N] or empty; returns bf16 [M_pad, N].  ``ca``
    and ``cfg`` (the reference's tile configuration) are accepted and not used."""
    dev = _require_cuda(a, b, sa, sb)
    if bias is not None and bias.numel() == 0:
        bias = None
    mp, kh = a.shape
    a8 = torch.empty(mp, 2 * kh, dtype=torch.int8, device=dev)
    _lib.call("cq_unpack_int4", _ptr(a.contiguous()), mp, 2 * kh, _ptr(a8), _stream(dev))
    if pol == 0:
        return gemm_rowcol(a8, sa.reshape(-1), b.contiguous(), sb.reshape(-1), bias)
    if pol == 4:
        return gemm_groupwise(a8, sa, b.contiguous(), sb, bias)
    if pol in (5, 7, 15, 17):
        return gemm_intratio(a8, sa.reshape(-1), b.contiguous(), sb.reshape(-1), cw, 64 if pol % 10 == 5 else 128, bias)
    raise ValueError(f"policy {pol} is not built (0, 4, 5, 7, 15, 17 are)")


def gemm_intratio(a: torch.Tensor, sa: torch.Tensor, b: torch.Tensor, sb: torch.Tensor, cw: torch.Tensor, group: int,
                  bias=None, *, a_kperm: bool = False) -> torch.Tensor:
    """Integer weight ratios per group (the reference's policies 5/7/15/17, ``cq_gemm_intratio``): a int8-held int4
    codes [M, K], b packed int4 [N, K/2], sa [M], sb [N] f32, cw int32 or uint8 [K/group, N]."""
    dev = _require_cuda(a, sa, b, sb, cw, bias)
    m, k = a.shape
    n = b.shape[0]
    if cw.dtype not in (torch.int32, torch.uint8) or tuple(cw.shape) != (k // group, n) or not cw.is_contiguous():
        raise ValueError(f"cw (K/G, N): int32 (pol 5/7) or uint8 (15/17), [{k // group}, {n}]")
    if sa.numel() != m or sb.numel() != n:
        raise ValueError("per-row scales sa (M,), sb (N,)")
    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    _lib.call("cq_gemm_intratio", _ptr(a), int(bool(a_kperm)), _ptr(sa.float().contiguous()), _ptr(b),
              _ptr(sb.float().contiguous()), _ptr(cw), int(cw.dtype == torch.uint8), int(group), _ptr(_bias_bf16(bias)),
              _ptr(out), m, n, k, _stream(dev))
    return out


def w4a4_groupwise_linear(x: torch.Tensor, qweight: torch.Tensor, sb_g: torch.Tensor, bias=None,
                          swiglu: bool = False) -> torch.Tensor:
    """The reference node's forward with policy 4 (``experiments/qwen21-kernel/node/__init__.py:152-187``): the
    per-group quantizer (ConvRot-256, int4 per token and 128-wide group, bf16-up scales) on x (or on silu(gate) * up
    of x = [gate | up] with ``swiglu``), then the g128 x g128 GEMM.  The activation codes go to the GEMM as int8 in
    the K order the int4 weights unpack into, so nothing is packed and unpacked in between.  x [..., K] (or 2K)."""
    dev = _require_cuda(x, qweight, sb_g, bias)
    x2 = _as2d(x)
    m = x2.shape[0]
    k = 2 * qweight.shape[1]
    mp = (m + 127) // 128 * 128
    q, sa_g, _ = rotquant(x2, 256, _lib.CQ_ACT_INT4_GROUP, swiglu=swiglu, act_group=128, m_pad=mp,
                          int4_as_int8=True, kperm=True)
    if q.shape[1] != k:
        raise ValueError(f"Input K={q.shape[1]} does not match weight K={k}")
    y = gemm_groupwise(q, sa_g, qweight, sb_g, bias, m=m, a_kperm=True)
    return y.reshape(*x.shape[:-1], y.shape[-1])


def _workspace(m: int, k: int, dev, n: int | None = None) -> torch.Tensor:
    """Scratch for a fused linear; with ``n`` (W4A8 affine linears) also room for the K-split partial sums the GEMM
    takes when its tiles leave most SMs idle."""
    lib = _lib.load()
    nbytes = int(lib.cq_linear_workspace_bytes_n(m, k, n) if n is not None else lib.cq_linear_workspace_bytes(m, k))
    return torch.empty(nbytes + 256, dtype=torch.uint8, device=dev)


def _ws_ptr(ws: torch.Tensor) -> tuple[int, int]:
    p = ws.data_ptr()
    aligned = (p + 255) // 256 * 256
    return aligned, ws.numel() - (aligned - p)


def convrot_w4a4_linear(x: torch.Tensor, qweight: torch.Tensor, wscales: torch.Tensor, bias: torch.Tensor | None = None,
                        convrot_groupsize: int = 256, quant_group_size: int = INT4_GROUP_SIZE,
                        linear_dtype: str = "int4", input_act: str | None = None) -> torch.Tensor:
    """act(x) @ W^T + bias with ConvRot W4A4 weights (rotated per-row int4) and int4 or int8 activations."""
    if linear_dtype not in {"int4", "int8"}:
        raise ValueError(f"ConvRot W4A4 linear_dtype must be 'int4' or 'int8', got {linear_dtype!r}")
    if quant_group_size != INT4_GROUP_SIZE:
        raise ValueError(f"int4 MMA kernel requires quant_group_size {INT4_GROUP_SIZE}")
    if input_act not in (None, "swiglu"):
        raise ValueError(f"input_act {input_act!r} is not fused; apply it before the call")
    swiglu = input_act == "swiglu"
    k = x.shape[-1] // 2 if swiglu else x.shape[-1]
    if k != qweight.shape[-1] * 2:
        raise ValueError(f"Input K={k} does not match qweight K={qweight.shape[-1] * 2}")
    if k % max(int(convrot_groupsize), 1) != 0:
        raise ValueError(f"Input K={k} is not divisible by convrot_groupsize={convrot_groupsize}")
    dev = _require_cuda(x, qweight, wscales, bias)
    x2 = _as2d(x)
    m, n = x2.shape[0], qweight.shape[0]
    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    ws = _workspace(m, k, dev)
    wp, wn = _ws_ptr(ws)
    bias = _bias_bf16(bias)
    _lib.call("cq_linear_convrot_w4a4", _ptr(x2), m, k, n, _check_rot(convrot_groupsize), int(swiglu),
              4 if linear_dtype == "int4" else 8, _ptr(qweight.contiguous()),
              _ptr(wscales.float().reshape(-1).contiguous()), _ptr(bias), _ptr(out), wp, wn, _stream(dev))
    out = out.reshape(*x.shape[:-1], n)
    return out if x.dtype == torch.bfloat16 else out.to(x.dtype)


def int8_linear(x: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor, bias: torch.Tensor | None = None,
                out_dtype: torch.dtype | None = None, convrot: bool = False, convrot_groupsize: int = 256,
                input_act: str | None = None) -> torch.Tensor:
    """W8A8 (int8_tensorwise) linear with optional ConvRot rotation and per-token int8 activations."""
    if input_act not in (None, "swiglu"):
        raise ValueError(f"input_act {input_act!r} is not fused; apply it before the call")
    swiglu = input_act == "swiglu"
    k = x.shape[-1] // 2 if swiglu else x.shape[-1]
    if weight.dtype != torch.int8 or weight.shape[-1] != k:
        raise ValueError(f"weight must be int8 [N, {k}]")
    dev = _require_cuda(x, weight, weight_scale, bias)
    x2 = _as2d(x)
    m, n = x2.shape[0], weight.shape[0]
    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    ws = _workspace(m, k, dev)
    wp, wn = _ws_ptr(ws)
    bias = _bias_bf16(bias)
    _lib.call("cq_linear_w8a8", _ptr(x2), m, k, n, _check_rot(convrot_groupsize if convrot else 0), int(swiglu),
              _ptr(weight.contiguous()), _ptr(weight_scale.float().reshape(-1).contiguous()), _ptr(bias), _ptr(out),
              wp, wn, _stream(dev))
    out = out.reshape(*x.shape[:-1], n)
    dt = out_dtype or x.dtype
    return out if dt == torch.bfloat16 else out.to(dt)


def affine_linear_launches(m: int, n: int, k: int) -> int:
    """Kernels one fused W4A8 affine linear of [m, k] x [k, n] launches: the activation kernel and the product, plus
    the split-K finalize kernel when the GEMM splits K (the workspace then holds fp32 partial sums)."""
    lib = _lib.load()
    return 3 if m > 8 and lib.cq_linear_workspace_bytes_n(m, k, n) > lib.cq_linear_workspace_bytes(m, k) else 2


def prepare_affine_zeros(zeros: torch.Tensor, group_size: int = 128) -> torch.Tensor:
    """The zero-point operand of the W4A8 GEMM, built once per weight from the awq-layout zeros [K/G, N]:
    zt [N, cq_group_sum_cols(K)] bf16 with zt[n, j] = zeros[j mod G, n] for j < 2G, else 0."""
    dev = _require_cuda(zeros)
    g, n = zeros.shape
    k = g * group_size
    z = zeros.to(torch.bfloat16).contiguous()
    zt = torch.empty(n, int(_lib.load().cq_group_sum_cols(k)), dtype=torch.bfloat16, device=dev)
    _lib.call("cq_prepare_affine_zeros", _ptr(z), n, k, int(group_size), _ptr(zt), _stream(dev))
    return zt


def w4a8_affine_linear(x: torch.Tensor, qweight: torch.Tensor, scale: torch.Tensor, zeros: torch.Tensor,
                       bias: torch.Tensor | None = None, group_size: int = 128, convrot_groupsize: int = 0,
                       input_act: str | None = None, out_dtype: torch.dtype | None = None,
                       zeros_prepared: torch.Tensor | None = None) -> torch.Tensor:
    """W4A8 linear with awq-layout weights (W = (q - 8) * scale + zeros, scale/zeros [K/G, N] bf16).

    Activations are (optionally rotated and) quantized per token to int8; the GEMM accumulates int8 x int4
    products per 128-group in int32 and applies scale, zero-point, activation scale and bias in fp32.
    ``zeros_prepared`` (from ``prepare_affine_zeros``) skips rebuilding the zero-point operand on every call.
    """
    if group_size != 128:
        raise ValueError("the W4A8 affine kernel supports group_size 128")
    if input_act not in (None, "swiglu"):
        raise ValueError(f"input_act {input_act!r} is not fused; apply it before the call")
    swiglu = input_act == "swiglu"
    k = x.shape[-1] // 2 if swiglu else x.shape[-1]
    if k != qweight.shape[-1] * 2:
        raise ValueError(f"Input K={k} does not match qweight K={qweight.shape[-1] * 2}")
    n = qweight.shape[0]
    if tuple(scale.shape) != (k // group_size, n) or tuple(zeros.shape) != (k // group_size, n):
        raise ValueError(f"scale/zeros must be [{k // group_size}, {n}]")
    dev = _require_cuda(x, qweight, scale, zeros, bias)
    x2 = _as2d(x)
    m = x2.shape[0]
    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    ws = _workspace(m, k, dev, n)
    wp, wn = _ws_ptr(ws)
    bias = _bias_bf16(bias)
    zt = zeros_prepared if zeros_prepared is not None else prepare_affine_zeros(zeros, group_size)
    _lib.call("cq_linear_w4a8_affine", _ptr(x2), m, k, n, _check_rot(convrot_groupsize), int(swiglu),
              _ptr(qweight.contiguous()), _ptr(scale.to(torch.bfloat16).contiguous()), _ptr(zt), int(group_size),
              _ptr(bias), _ptr(out), wp, wn, _stream(dev))
    out = out.reshape(*x.shape[:-1], n)
    dt = out_dtype or x.dtype
    return out if dt == torch.bfloat16 else out.to(dt)


def w4a8_affine_linear_into(x: torch.Tensor, qweight: torch.Tensor, scale: torch.Tensor, zeros_prepared: torch.Tensor,
                            bias: torch.Tensor | None, outs, col0: int, ldo: int, group_size: int = 128,
                            convrot_groupsize: int = 0) -> None:
    """Column-parallel W4A8 linear: this shard's N = qweight.shape[0] output columns are written into every buffer
    of ``outs`` (bf16 [M, ldo] tensors, or raw device pointers of such buffers, e.g. the peer buffers of a symmetric
    memory allocation) at columns [col0, col0 + N).  The zeros must be prepared (``prepare_affine_zeros``)."""
    if group_size != 128:
        raise ValueError("the W4A8 affine kernel supports group_size 128")
    k = x.shape[-1]
    if k != qweight.shape[-1] * 2:
        raise ValueError(f"Input K={k} does not match qweight K={qweight.shape[-1] * 2}")
    n = qweight.shape[0]
    dev = _require_cuda(x, qweight, scale, zeros_prepared, bias)
    x2 = _as2d(x)
    m = x2.shape[0]
    ptrs = []
    for o in outs:
        if isinstance(o, torch.Tensor):
            if o.dtype != torch.bfloat16 or o.dim() != 2 or o.shape[1] != ldo or o.shape[0] < m or not o.is_contiguous():
                raise ValueError(f"output buffers must be contiguous bf16 [>= {m}, {ldo}]")
            ptrs.append(o.data_ptr())
        else:
            ptrs.append(int(o))
    arr = (ctypes.c_void_p * len(ptrs))(*ptrs)
    ws = _workspace(m, k, dev)
    wp, wb = _ws_ptr(ws)
    _lib.call("cq_linear_w4a8_affine_peers", _ptr(x2), m, k, n, _check_rot(convrot_groupsize), 0, _ptr(qweight),
              _ptr(scale), _ptr(zeros_prepared), int(group_size), _ptr(_bias_bf16(bias)), arr, len(ptrs), int(col0),
              int(ldo), wp, wb, _stream(dev))


def gemm_affine(a: torch.Tensor, sa: torch.Tensor, gsplit: torch.Tensor, qweight: torch.Tensor, scale: torch.Tensor,
                zeros: torch.Tensor, bias=None, *, a_kperm: bool = False,
                zeros_prepared: torch.Tensor | None = None) -> torch.Tensor:
    """The affine GEMM alone on pre-quantized activations (a int8 [M, K], sa [M], gsplit from ``rotquant``)."""
    dev = _require_cuda(a, sa, gsplit, qweight, scale, zeros, bias)
    zt = zeros_prepared if zeros_prepared is not None else prepare_affine_zeros(zeros, 128)
    m, k = a.shape
    n = qweight.shape[0]
    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    bias = _bias_bf16(bias)
    _lib.call("cq_gemm_affine", _ptr(a), int(bool(a_kperm)), _ptr(sa), _ptr(gsplit), _ptr(qweight),
              _ptr(scale.contiguous()), _ptr(zt), _ptr(bias), _ptr(out), m, n, k, 128, _stream(dev))
    return out


# ----------------------------------------------------------------------------------------------
# DiT-step glue: the modulated layer norm fused into the activation kernel, and q/k RMSNorm + rotary
# embedding + the joint attention layout in one kernel (see cq_rotquant_lnmod / cq_qkv_rmsnorm_rope)
# ----------------------------------------------------------------------------------------------

def _vec_bf16(v: torch.Tensor, k: int, name: str) -> torch.Tensor:
    v = v.reshape(-1)
    if v.numel() != k:
        raise ValueError(f"{name} must hold {k} values, got {v.numel()}")
    v = v.to(torch.bfloat16).contiguous()
    if v.data_ptr() % 16:
        v = v.clone()
    return v


def rotquant_lnmod(x: torch.Tensor, rot_group: int, shift: torch.Tensor, scale1p: torch.Tensor, *, eps: float = 1e-6,
                   m_pad: int | None = None, group_sums: bool = False, kperm: bool = False):
    """Per-token int8 quantization (``rotquant`` mode CQ_ACT_INT8_ROW) of the modulated layer norm
    bf16(shift + bf16(layer_norm(x)) * scale1p), computed inside the activation kernel.  Returns (q, scale, gsplit)."""
    dev = _require_cuda(x, shift, scale1p)
    x2 = _as2d(x)
    m, k = x2.shape
    mp = m if m_pad is None else int(m_pad)
    sh, sc = _vec_bf16(shift, k, "shift"), _vec_bf16(scale1p, k, "scale1p")
    q = torch.empty(mp, k, dtype=torch.int8, device=dev)
    scale = torch.empty(mp, dtype=torch.float32, device=dev)
    gs = torch.empty(mp, int(_lib.load().cq_group_sum_cols(k)), dtype=torch.bfloat16, device=dev) if group_sums else None
    _lib.call("cq_rotquant_lnmod", _ptr(x2), m, k, _check_rot(rot_group), _ptr(sh), _ptr(sc), float(eps), mp,
              _lib.CQ_Q_KPERM if kperm else 0, _ptr(q), _ptr(scale), _ptr(gs), _stream(dev))
    return q, scale, gs


def w4a8_affine_linear_lnmod(x: torch.Tensor, shift: torch.Tensor, scale1p: torch.Tensor, qweight: torch.Tensor,
                             scale: torch.Tensor, zeros_prepared: torch.Tensor, bias: torch.Tensor | None = None,
                             group_size: int = 128, convrot_groupsize: int = 0, eps: float = 1e-6) -> torch.Tensor:
    """``w4a8_affine_linear(bf16(shift + bf16(layer_norm(x, eps)) * scale1p), ...)`` with the layer norm and the
    modulation done inside the activation kernel (no normalized copy of x in HBM).  ``scale1p`` is 1 + scale,
    rounded to bf16 (as the torch expression ``1 + scale`` on a bf16 tensor gives)."""
    if group_size != 128:
        raise ValueError("the W4A8 affine kernel supports group_size 128")
    k = x.shape[-1]
    if k != qweight.shape[-1] * 2:
        raise ValueError(f"Input K={k} does not match qweight K={qweight.shape[-1] * 2}")
    n = qweight.shape[0]
    dev = _require_cuda(x, shift, scale1p, qweight, scale, zeros_prepared, bias)
    x2 = _as2d(x)
    m = x2.shape[0]
    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    ws = _workspace(m, k, dev, n)
    wp, wn = _ws_ptr(ws)
    sh, sc = _vec_bf16(shift, k, "shift"), _vec_bf16(scale1p, k, "scale1p")
    _lib.call("cq_linear_w4a8_affine_lnmod", _ptr(x2), m, k, n, _check_rot(convrot_groupsize), _ptr(sh), _ptr(sc),
              float(eps), _ptr(qweight.contiguous()), _ptr(scale.to(torch.bfloat16).contiguous()), _ptr(zeros_prepared),
              int(group_size), _ptr(_bias_bf16(bias)), _ptr(out), wp, wn, _stream(dev))
    return out.reshape(*x.shape[:-1], n)


def w4a8_affine_linear_op(x: torch.Tensor, qweight: torch.Tensor, wscale: torch.Tensor, zeros_prepared: torch.Tensor,
                          bias: torch.Tensor | None = None, *, out_op: str = "plain",
                          residual: torch.Tensor | None = None, gate: torch.Tensor | None = None,
                          shift: torch.Tensor | None = None, scale: torch.Tensor | None = None,
                          group_size: int = 128, convrot_groupsize: int = 0, eps: float = 1e-6,
                          out: torch.Tensor | None = None, split_k: bool = True) -> torch.Tensor:
    """A DiT-block linear with the elementwise step after it done in the GEMM's epilogue.

    With y the bf16 output of ``w4a8_affine_linear`` (or, when ``shift`` and the modulation ``scale`` are given, of
    ``w4a8_affine_linear_lnmod(x, shift, 1 + scale, ...)`` with the bf16 ``1 + scale`` formed in the activation
    kernel), returns
      ``out_op="plain"``:  y
      ``out_op="gelu"``:   ``F.gelu(y, approximate="tanh")``            (the MLP-up activation)
      ``out_op="gated"``:  ``torch.addcmul(residual, gate, y)``         (the gated residual after the attention
                           output and MLP-down linears; ``gate`` [N] or [1, N], ``residual`` [..., N] bf16)
    ``out`` (bf16, contiguous, the output's shape) receives the result if given; it may be ``residual`` itself
    (an in-place residual update).  ``split_k=False`` gives the call only the base workspace, so a GEMM with few
    output tiles keeps one CTA per tile instead of splitting K over more CTAs (for a linear that runs beside other
    work on another stream, where the idle SMs are not idle)."""
    if group_size != 128:
        raise ValueError("the W4A8 affine kernel supports group_size 128")
    k = x.shape[-1]
    if k != qweight.shape[-1] * 2:
        raise ValueError(f"Input K={k} does not match qweight K={qweight.shape[-1] * 2}")
    n = qweight.shape[0]
    dev = _require_cuda(x, qweight, wscale, zeros_prepared, bias, shift, scale, residual, gate, out)
    x2 = _as2d(x)
    m = x2.shape[0]
    op, keep, out, sh, sc = _op_args(out_op, residual, gate, shift, scale, out, m, n, k, dev)
    ws = _workspace(m, k, dev, n if split_k else None)
    wp, wn = _ws_ptr(ws)
    _lib.call("cq_linear_w4a8_op", _ptr(x2), m, k, n, _check_rot(convrot_groupsize), _ptr(sh), _ptr(sc), float(eps),
              _ptr(qweight.contiguous()), _ptr(wscale.to(torch.bfloat16).contiguous()), _ptr(zeros_prepared),
              int(group_size), _ptr(_bias_bf16(bias)), ctypes.byref(op), _ptr(out), wp, wn, _stream(dev))
    return out.reshape(*x.shape[:-1], n)


def _op_args(out_op, residual, gate, shift, scale, out, m: int, n: int, k: int, dev):
    """The output operation struct of the op linears (and the tensors its pointers refer to, kept alive by the
    caller), the output buffer, and the modulation vectors as bf16 [K]."""
    kinds = {"plain": _lib.CQ_OUT_PLAIN, "gelu": _lib.CQ_OUT_GELU_TANH, "gated": _lib.CQ_OUT_GATED_RESIDUAL}
    if out_op not in kinds:
        raise ValueError(f"out_op must be one of {sorted(kinds)}")
    if (shift is None) != (scale is None):
        raise ValueError("shift and scale go together")
    op = _lib.CQOutOp(kinds[out_op], None, 0, None)
    keep = []
    if out_op == "gated":
        if residual is None or gate is None:
            raise ValueError("the gated residual needs residual and gate")
        if residual.dtype != torch.bfloat16 or residual.shape[-1] != n or residual.numel() != m * n:
            raise ValueError(f"residual must be bf16 with {m} rows of {n}")
        r2 = residual.reshape(m, n)
        if r2.stride(1) != 1:
            raise ValueError("residual rows must be contiguous")
        g = _vec_bf16(gate, n, "gate")
        keep += [r2, g]
        op.residual, op.residual_ld, op.gate = _ptr(r2), r2.stride(0), _ptr(g)
    if out is None:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    elif out.dtype != torch.bfloat16 or out.numel() != m * n or not out.is_contiguous():
        raise ValueError(f"out must be contiguous bf16 with {m} x {n} elements")
    sh = _vec_bf16(shift, k, "shift") if shift is not None else None
    sc = _vec_bf16(scale, k, "scale") if scale is not None else None
    return op, keep, out, sh, sc


def convrot_w4a4_linear_op(x: torch.Tensor, qweight: torch.Tensor, wscales: torch.Tensor,
                           bias: torch.Tensor | None = None, *, out_op: str = "plain",
                           residual: torch.Tensor | None = None, gate: torch.Tensor | None = None,
                           shift: torch.Tensor | None = None, scale: torch.Tensor | None = None,
                           convrot_groupsize: int = 256, linear_dtype: str = "int4", eps: float = 1e-6,
                           out: torch.Tensor | None = None) -> torch.Tensor:
    """``convrot_w4a4_linear`` with the elementwise step after it in the GEMM's epilogue and, with ``shift`` and
    the modulation ``scale``, the modulated layer norm bf16(shift + bf16(layer_norm(x)) * bf16(1 + scale)) formed in
    the activation kernel; ``out_op``, ``residual``, ``gate`` and ``out`` as in ``w4a8_affine_linear_op``."""
    if linear_dtype not in {"int4", "int8"}:
        raise ValueError(f"ConvRot W4A4 linear_dtype must be 'int4' or 'int8', got {linear_dtype!r}")
    k = x.shape[-1]
    if k != qweight.shape[-1] * 2:
        raise ValueError(f"Input K={k} does not match qweight K={qweight.shape[-1] * 2}")
    n = qweight.shape[0]
    dev = _require_cuda(x, qweight, wscales, bias, shift, scale, residual, gate, out)
    x2 = _as2d(x)
    m = x2.shape[0]
    op, keep, out, sh, sc = _op_args(out_op, residual, gate, shift, scale, out, m, n, k, dev)
    ws = _workspace(m, k, dev)
    wp, wn = _ws_ptr(ws)
    _lib.call("cq_linear_convrot_w4a4_op", _ptr(x2), m, k, n, _check_rot(convrot_groupsize),
              4 if linear_dtype == "int4" else 8, _ptr(sh), _ptr(sc), float(eps), _ptr(qweight.contiguous()),
              _ptr(wscales.float().reshape(-1).contiguous()), _ptr(_bias_bf16(bias)), ctypes.byref(op), _ptr(out),
              wp, wn, _stream(dev))
    return out.reshape(*x.shape[:-1], n)


def int8_linear_op(x: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor, bias: torch.Tensor | None = None,
                   *, out_op: str = "plain", residual: torch.Tensor | None = None, gate: torch.Tensor | None = None,
                   shift: torch.Tensor | None = None, scale: torch.Tensor | None = None, convrot: bool = False,
                   convrot_groupsize: int = 256, eps: float = 1e-6, out: torch.Tensor | None = None) -> torch.Tensor:
    """``int8_linear`` with the elementwise step after it in the GEMM's epilogue and the optional modulated layer
    norm in the activation kernel (as ``convrot_w4a4_linear_op``)."""
    k = x.shape[-1]
    if weight.dtype != torch.int8 or weight.shape[-1] != k:
        raise ValueError(f"weight must be int8 [N, {k}]")
    n = weight.shape[0]
    dev = _require_cuda(x, weight, weight_scale, bias, shift, scale, residual, gate, out)
    x2 = _as2d(x)
    m = x2.shape[0]
    op, keep, out, sh, sc = _op_args(out_op, residual, gate, shift, scale, out, m, n, k, dev)
    ws = _workspace(m, k, dev)
    wp, wn = _ws_ptr(ws)
    _lib.call("cq_linear_w8a8_op", _ptr(x2), m, k, n, _check_rot(convrot_groupsize if convrot else 0), _ptr(sh),
              _ptr(sc), float(eps), _ptr(weight.contiguous()), _ptr(weight_scale.float().reshape(-1).contiguous()),
              _ptr(_bias_bf16(bias)), ctypes.byref(op), _ptr(out), wp, wn, _stream(dev))
    return out.reshape(*x.shape[:-1], n)


def qkv_rmsnorm_rope(y: torch.Tensor, q_norm: torch.Tensor, k_norm: torch.Tensor, rope: torch.Tensor,
                     q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, s0: int, eps: float = 1e-6) -> None:
    """One stream's QKV output y [S, 3*H*D] (bf16) into the joint attention layout q, k, v [1, H, S_all, D] at
    tokens [s0, s0 + S): q and k RMS-normalized per head (weights q_norm / k_norm [D]) and rotated by ``rope``
    ([S, D/2] complex64, or its real view [S, D/2, 2] of (cos, sin)); v copied.

    q, k, v are either contiguous (head-major memory) or all three ``transpose(1, 2)`` views of contiguous
    [1, S_all, H, D] tensors (token-major memory: the [tokens, hidden] rows, which an attention kernel reads as
    strided views and mirrors in its output)."""
    dev = _require_cuda(y, q_norm, k_norm, rope, q, k, v)
    if q.dim() != 4 or q.shape[0] != 1:
        raise ValueError("q, k, v must be [1, H, S_all, D]")
    _, h, s_all, d = q.shape
    if k.shape != q.shape or v.shape != q.shape or q.dtype != torch.bfloat16 or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q, k, v must be bf16 of one shape")
    if all(t.is_contiguous() for t in (q, k, v)):
        token_major = 0
    elif all(t.transpose(1, 2).is_contiguous() for t in (q, k, v)):
        token_major = 1
    else:
        raise ValueError("q, k, v must all be contiguous [1, H, S_all, D] or all transposed views of contiguous "
                         "[1, S_all, H, D]")
    y2 = _as2d(y)
    s = y2.shape[0]
    if y2.shape[1] != 3 * h * d:
        raise ValueError(f"y must be [S, {3 * h * d}]")
    if rope.is_complex():
        rope = torch.view_as_real(rope)
    rope = rope.to(torch.float32).contiguous()
    if tuple(rope.shape) != (s, d // 2, 2):
        raise ValueError(f"rope must be [{s}, {d // 2}] complex (or [{s}, {d // 2}, 2] real)")
    qn, kn = q_norm.to(torch.bfloat16).contiguous(), k_norm.to(torch.bfloat16).contiguous()
    _lib.call("cq_qkv_rmsnorm_rope_layout", _ptr(y2), s, h, d, _ptr(qn), _ptr(kn), float(eps), _ptr(rope), _ptr(q),
              _ptr(k), _ptr(v), s_all, int(s0), token_major, _stream(dev))


def rmsnorm_rope_rows(x: torch.Tensor, weight: torch.Tensor, rope: torch.Tensor | None = None, head_dim: int = 128,
                      eps: float = 1e-6, out: torch.Tensor | None = None) -> torch.Tensor:
    """RMSNorm over whole rows of x [S, C] (bf16; a Wan-style q/k norm over the hidden dim), weight [C], one bf16
    rounding, then with ``rope`` ([S, D/2] complex64 or its real view [S, D/2, 2]) each head_dim-wide head's
    interleaved pairs rotated, as torch's rms_norm followed by the complex-multiply rotary embedding.  ``out`` may
    be x."""
    dev = _require_cuda(x, weight, rope, out)
    x2 = _as2d(x)
    if x2.dtype != torch.bfloat16 or not x2.is_contiguous():
        raise ValueError("x must be contiguous bf16")
    s, c = x2.shape
    w = weight.to(torch.bfloat16).contiguous()
    if w.numel() != c:
        raise ValueError(f"weight must have {c} elements")
    rp = None
    if rope is not None:
        if rope.is_complex():
            rope = torch.view_as_real(rope)
        rp = rope.to(torch.float32).contiguous()
        if tuple(rp.shape) != (s, head_dim // 2, 2):
            raise ValueError(f"rope must be [{s}, {head_dim // 2}] complex (or [{s}, {head_dim // 2}, 2] real)")
    if out is None:
        out = torch.empty_like(x2)
    elif out.shape != x2.shape or out.dtype != torch.bfloat16 or not out.is_contiguous():
        raise ValueError("out must be contiguous bf16 of x's shape")
    _lib.call("cq_rmsnorm_rope_rows", _ptr(x2), s, c, _ptr(w), float(eps), _ptr(rp), int(head_dim), _ptr(out),
              _stream(dev))
    return out.reshape(x.shape)


def _out_ptrs(outs, rows: int, ldo: int):
    ptrs = []
    for o in outs:
        if isinstance(o, torch.Tensor):
            if o.dtype != torch.bfloat16 or o.dim() != 2 or o.shape[1] != ldo or o.shape[0] < rows or not o.is_contiguous():
                raise ValueError(f"output buffers must be contiguous bf16 [>= {rows}, {ldo}]")
            ptrs.append(o.data_ptr())
        else:
            ptrs.append(int(o))
    return (ctypes.c_void_p * len(ptrs))(*ptrs), len(ptrs)


def heads_to_rows(o: torch.Tensor, outs, col0: int, ldo: int) -> None:
    """Attention output o [1, Hp, S, D] (bf16) into rows [S, ldo] at columns col0 + h*D of every buffer in ``outs``
    (tensors or raw device pointers, e.g. the peer buffers of a symmetric allocation)."""
    dev = _require_cuda(o)
    if o.dim() != 4 or o.shape[0] != 1 or o.dtype != torch.bfloat16:
        raise ValueError("o must be bf16 [1, Hp, S, D]")
    o = o.contiguous()
    _, hp, s, d = o.shape
    arr, n = _out_ptrs(outs, s, ldo)
    _lib.call("cq_heads_to_rows", _ptr(o), s, hp, d, arr, n, int(col0), int(ldo), _stream(dev))


def gemm_affine_into(a: torch.Tensor, sa: torch.Tensor, gsplit: torch.Tensor, qweight: torch.Tensor,
                     scale: torch.Tensor, zeros_prepared: torch.Tensor, bias, outs, col0: int, ldo: int, *,
                     m: int | None = None, a_kperm: bool = True) -> None:
    """The affine GEMM on pre-quantized activations (``rotquant`` / ``rotquant_lnmod`` outputs; the first ``m`` rows)
    writing its N = qweight.shape[0] columns into every buffer of ``outs`` at [col0, col0 + N)."""
    dev = _require_cuda(a, sa, gsplit, qweight, scale, zeros_prepared, bias)
    m = a.shape[0] if m is None else int(m)
    k = a.shape[1]
    n = qweight.shape[0]
    arr, cnt = _out_ptrs(outs, m, ldo)
    _lib.call("cq_gemm_affine_peers", _ptr(a), int(bool(a_kperm)), _ptr(sa), _ptr(gsplit), _ptr(qweight),
              _ptr(scale), _ptr(zeros_prepared), _ptr(_bias_bf16(bias)), arr, cnt, int(col0), int(ldo), m, n, k, 128,
              _stream(dev))


# ----------------------------------------------------------------------------------------------
# ConvRot W4A4 linear with the SwiGLU output silu(y[:, :N/2]) * y[:, N/2:] fused into the GEMM epilogue
# ----------------------------------------------------------------------------------------------

def swiglu_output_rows(n: int, device=None) -> torch.Tensor:
    """Row order of a SwiGLU-output weight: each group of 32 rows holds 16 gate rows (of y[:, :n/2]) then the
    matching 16 up rows (of y[:, n/2:]), so one TMEM lane quadrant of the GEMM holds both halves of 16 outputs;
    entry p is the original row."""
    if n % 128:
        raise ValueError(f"the SwiGLU output needs N % 128 == 0, got {n}")
    p = torch.arange(n, device=device)
    t, r = p // 32, p % 32
    return torch.where(r < 16, 16 * t + r, n // 2 + 16 * t + (r - 16))


def prepare_swiglu_output_weight(qweight: torch.Tensor, wscales: torch.Tensor, bias: torch.Tensor | None = None):
    """ConvRot W4A4 weight (packed [N, K/2], scales [N], bias [N]) in the tile-interleaved row order of
    ``convrot_w4a4_linear_swiglu``, built once per weight."""
    n = qweight.shape[0]
    idx = swiglu_output_rows(n, qweight.device)
    qw = qweight.index_select(0, idx).contiguous()
    ws = wscales.float().reshape(-1).index_select(0, idx.to(wscales.device)).contiguous()
    b = None if bias is None else _bias_bf16(bias).index_select(0, idx.to(bias.device)).contiguous()
    return qw, ws, b


def convrot_w4a4_linear_swiglu(x: torch.Tensor, qweight_glu: torch.Tensor, wscales_glu: torch.Tensor,
                               bias_glu: torch.Tensor | None = None, convrot_groupsize: int = 256,
                               linear_dtype: str = "int4") -> torch.Tensor:
    """silu(y[..., :N/2]) * y[..., N/2:] of the ConvRot W4A4 linear y = convrot_w4a4_linear(x, W, ...), with the
    SwiGLU computed in the GEMM's epilogue (weights from ``prepare_swiglu_output_weight``): [..., N/2] bf16."""
    if linear_dtype not in {"int4", "int8"}:
        raise ValueError(f"ConvRot W4A4 linear_dtype must be 'int4' or 'int8', got {linear_dtype!r}")
    k = x.shape[-1]
    if k != qweight_glu.shape[-1] * 2:
        raise ValueError(f"Input K={k} does not match qweight K={qweight_glu.shape[-1] * 2}")
    dev = _require_cuda(x, qweight_glu, wscales_glu, bias_glu)
    x2 = _as2d(x)
    m, n = x2.shape[0], qweight_glu.shape[0]
    out = torch.empty(m, n // 2, dtype=torch.bfloat16, device=dev)
    ws = _workspace(m, k, dev)
    wp, wn = _ws_ptr(ws)
    _lib.call("cq_linear_convrot_w4a4_swiglu", _ptr(x2), m, k, n, _check_rot(convrot_groupsize),
              4 if linear_dtype == "int4" else 8, _ptr(qweight_glu), _ptr(wscales_glu.float().contiguous()),
              _ptr(_bias_bf16(bias_glu)), _ptr(out), wp, wn, _stream(dev))
    return out.reshape(*x.shape[:-1], n // 2)
