"""CPU oracle for the quantized-linear hot path (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.  The library in
``comfy_quant_bench_b200`` never routes through it and has no CPU fallback.

It restates, in numpy float32/int64 arithmetic, the algorithm comfy-quant-bench runs on this path:

* Hadamard rotation: the "regular" Hadamard of order 4, ``H4r x: y_i = (x0+x1+x2+x3)/2 - x_{3-i}``, applied
  as radix-4 stages (``experiments/qwen21-kernel/kernels/g64_quant.cu:2-7, 68-87``); a rotation group of
  ``4**p`` elements is ``kron^p(H4r) / 2**p`` (256 -> p=4 is the one the reference pins; 64 and 16 are the
  same construction with fewer stages).
* Per-token activation quantization (ConvRot W4A4 ``quantize_int4_rowwise_convrot64``):
  ``scale = max(absmax * (1/7), 1e-10)``, ``q = clamp(rint(v * (1/scale)), -7, 7)``, two codes per byte,
  low nibble = even column (``tools/ck_swiglu/swiglu_quant.cu:84-96``, ``g64_bench6.py:44-47``).
  The int8 variant uses 127 (``tools/activation_balance.py:65-71`` with ``limit=127``).
* Per-group activation quantization with the scale rounded UP to bf16
  (``g64_quant.cu:18-25, 88-106``; layout ``s [K/G, M_pad]``).
* SwiGLU prologue ``silu(gate) * up`` in fp32, rounded once to bf16 before the rotation
  (``swiglu_quant.cu:58-67``; ``[gate | up]`` halves, ``patches/comfyui_swiglu_triton_env.patch:19``).
* Weight quantizers: ConvRot per-row int4 (``experiments/qwen21-kernel/node/__init__.py:89-97``, pol 0),
  per-group bf16_up int4 (same file :98-112, pol 1/3/4) and the affine per-group layout of ``awq_w4a16``
  ``W = (q - 8) * scale + zeros`` with scale/zeros bf16 ``[K/G, N]``
  (``patches/comfyui_awq_w4a16_format.patch:79-80``).
* Integer GEMM (int64 accumulation) and the fp epilogues of ``g64_bench6.py:50-68`` (row x row scales,
  per-group scales) plus the affine zero-point term.
* Dequantize-and-matmul (``patches/tests/test_comfyui_fase4_dispatch.py:98``): the reference path that the
  quantized linears' bf16 outputs are checked against.

Float32 evaluation order is spelled out (every ``np.float32`` op rounds once, numpy never fuses a multiply
and an add), so the CUDA kernels, which use explicitly rounded intrinsics in the same order, match this
module bit for bit on codes and scales.

Parity pinning: ``tests/golden/make_golden.py`` runs the reference's own Python functions
(``g64_quant_test.bf16_up/unpack/ref``, ``g64_bench6.pack/ref``, ``activation_balance.quantize_rowwise``,
``node._pack/_quant_weight``, ``test_comfy_kitchen_awq.old_cuda_torch_chain``, ``_formats`` shapes) on seeded
inputs and commits their outputs under ``tests/golden``; ``tests/test_oracle_golden.py`` checks this module
against them with the reference's own acceptance rules.  What stays unpinned: comfy-kitchen's
``_build_hadamard`` for groups 64 and 16, its ``finite_absmax_for_int4_scale`` (taken as the identity on
finite input) and its W4A8 codebook / ALS quantizer (comfy-kitchen is not vendored in the reference).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
INT4_MAX = 7
INT8_MAX = 127
ROT_GROUPS = (0, 16, 64, 256)


# ----------------------------------------------------------------------------------------------
# bf16 helpers
# ----------------------------------------------------------------------------------------------

def bf16_round(x) -> np.ndarray:
    """float32 -> nearest bf16 (ties to even), returned as float32. NaN is not expected on this path."""
    u = np.ascontiguousarray(x, dtype=F32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return r.astype(np.uint32).view(F32)


def bf16_up(x) -> np.ndarray:
    """Smallest bf16 value >= x for x > 0 (``g64_quant_test.py:41-45``, ``g64_quant.cu:18-25``)."""
    u = np.ascontiguousarray(x, dtype=F32).view(np.uint32).astype(np.uint64)
    low = u & 0xFFFF
    u = (u & 0xFFFF0000) + (low != 0).astype(np.uint64) * 0x10000
    return u.astype(np.uint32).view(F32)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(F32)


def f32_to_bf16_bits(x) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


# ----------------------------------------------------------------------------------------------
# Hadamard rotation
# ----------------------------------------------------------------------------------------------

def h4r() -> np.ndarray:
    """The regular order-4 Hadamard matrix, normalised: (H4r x)_i = (x0+x1+x2+x3)/2 - x_{3-i}."""
    return 0.5 * np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=np.float64)


def build_hadamard(n: int) -> np.ndarray:
    """kron^p(H4r)/2^p for n = 4^p, as float64: symmetric, orthonormal and its own inverse."""
    if n not in (4, 16, 64, 256, 1024):
        raise ValueError(f"rotation group {n} is not a power of 4 in [4, 1024]")
    h = np.ones((1, 1))
    while h.shape[0] < n:
        h = np.kron(h, h4r())
    return h


def fwht_stages(x: np.ndarray, group: int) -> np.ndarray:
    """Rotate every ``group``-wide block of the last axis by kron^p(H4r)/2^p, in float32.

    Radix-4 stages with strides 1, 4, 16, 64 (the order of ``g64_quant.cu:68-85``); each butterfly is
    ``hs = 0.5 * (((x0 + x1) + x2) + x3); y_i = hs - x_{3-i}`` with one rounding per operation.
    """
    x = np.ascontiguousarray(x, dtype=F32)
    if group == 0:
        return x.copy()
    lead, k = x.shape[:-1], x.shape[-1]
    if k % group:
        raise ValueError(f"K={k} is not a multiple of the rotation group {group}")
    v = x.reshape(-1, k // group, group)
    st = 1
    while st < group:
        w = v.reshape(v.shape[0], v.shape[1], group // (4 * st), 4, st)
        x0, x1, x2, x3 = w[..., 0, :], w[..., 1, :], w[..., 2, :], w[..., 3, :]
        hs = F32(0.5) * (((x0 + x1) + x2) + x3)
        v = np.stack([hs - x3, hs - x2, hs - x1, hs - x0], axis=-2).reshape(v.shape)
        st *= 4
    return v.reshape(*lead, k)


def rotate_matmul(x: np.ndarray, group: int) -> np.ndarray:
    """The reference's matrix form ``x.reshape(M, K/g, g) @ H`` (``g64_quant_test.py:64``), float32 result."""
    x = np.asarray(x, dtype=np.float64)
    if group == 0:
        return x.astype(F32)
    m, k = x.shape
    return (x.reshape(m, k // group, group) @ build_hadamard(group)).reshape(m, k).astype(F32)


# ----------------------------------------------------------------------------------------------
# int4 packing
# ----------------------------------------------------------------------------------------------

def pack_int4(codes: np.ndarray) -> np.ndarray:
    """(R, K) ints -> (R, K/2) int8, low nibble = even column (``g64_bench6.py:44-47``)."""
    c = np.asarray(codes).astype(np.int16)
    lo = c[:, 0::2] & 0xF
    hi = c[:, 1::2] & 0xF
    return (lo | (hi << 4)).astype(np.uint8).view(np.int8)


def unpack_int4_signed(packed: np.ndarray, k: int | None = None) -> np.ndarray:
    """(R, K/2) int8 -> (R, K) int16 in [-8, 7] (``g64_quant_test.py:48-52``)."""
    u = np.asarray(packed).view(np.uint8).astype(np.int16)
    v = np.stack([u & 0xF, (u >> 4) & 0xF], axis=-1).reshape(u.shape[0], -1)
    return np.where(v >= 8, v - 16, v)


def unpack_uint4(packed: np.ndarray) -> np.ndarray:
    """(R, K/2) bytes -> (R, K) int16 in [0, 15] (the awq_w4a16 / lowbit code layout)."""
    u = np.asarray(packed).view(np.uint8).astype(np.int16)
    return np.stack([u & 0xF, (u >> 4) & 0xF], axis=-1).reshape(u.shape[0], -1)


# ----------------------------------------------------------------------------------------------
# activation quantization
# ----------------------------------------------------------------------------------------------

def swiglu_product(h_bf16_bits: np.ndarray, round_bf16: bool = True) -> np.ndarray:
    """[gate | up] bf16 bits (M, 2K) -> silu(gate) * up computed in fp32 (float32 result).

    ``round_bf16``: round the product once to bf16 (comfy-kitchen's fused quantizer,
    ``swiglu_quant.cu:58-67``); the reference's per-group quantizer keeps it in fp32 (``g64_quant.cu:40-50``).
    """
    h = bf16_bits_to_f32(h_bf16_bits)
    k = h.shape[1] // 2
    g, u = h[:, :k], h[:, k:]
    with np.errstate(over="ignore"):
        v = (g / (F32(1.0) + np.exp(-g)) * u).astype(F32)
    return bf16_round(v) if round_bf16 else v


def quant_rowwise(v: np.ndarray, qmax: int):
    """Per-token symmetric quantization of float32 rows: (codes int16, scale f32 [M]).

    ``scale = max(absmax * (1/qmax), 1e-10)``; ``q = clamp(rint(v * (1/scale)), -qmax, qmax)``.
    """
    v = np.asarray(v, dtype=F32)
    am = np.abs(v).max(axis=1) if v.shape[1] else np.zeros(v.shape[0], F32)
    scale = np.maximum(am * (F32(1.0) / F32(qmax)), F32(1e-10)).astype(F32)
    inv = (F32(1.0) / scale).astype(F32)
    q = np.clip(np.rint(v * inv[:, None]), -qmax, qmax).astype(np.int16)
    return q, scale


def quant_groupwise_bf16up(v: np.ndarray, group: int, qmax: int = INT4_MAX):
    """Per-(token, group) symmetric quantization with the scale rounded up to bf16 (``g64_quant.cu:88-106``).

    Returns codes (M, K) int16 and scales (K/G, M) float32 (group-major, the reference's layout).
    """
    v = np.asarray(v, dtype=F32)
    m, k = v.shape
    g = v.reshape(m, k // group, group)
    am = np.abs(g).max(axis=2)
    sc = np.where(am > 0, bf16_up(am / F32(qmax)), F32(0)).astype(F32)
    inv = np.where(sc > 0, F32(1.0) / np.where(sc > 0, sc, F32(1)), F32(0)).astype(F32)
    q = np.clip(np.rint(g * inv[..., None]), -qmax, qmax).astype(np.int16).reshape(m, k)
    return q, np.ascontiguousarray(sc.T)


def group_sums(q: np.ndarray, group: int = 128) -> np.ndarray:
    """R[m, g] = sum of the activation codes of token m over K-group g (int32), for the affine zero term."""
    q = np.asarray(q).astype(np.int64)
    m, k = q.shape
    return q.reshape(m, k // group, group).sum(axis=2).astype(np.int32)


def group_sum_cols(k: int) -> int:
    """Columns of the split group-sum array: 64 * ceil((K / 128) / 32)."""
    return 64 * ((k // 128 + 31) // 32)


def group_sums_split(q: np.ndarray, group: int = 128) -> np.ndarray:
    """The zero-point operand of the affine GEMM: R = group_sums(q) split exactly into bf16 parts,
    hi = 128 * floor(R / 128) in column g and lo = R - hi in column G + g, zero-padded to group_sum_cols(K).
    Returned as float32 values (every entry is exactly representable in bf16)."""
    r = group_sums(q, group).astype(np.int64)
    m, g = r.shape
    hi = np.floor_divide(r, 128) * 128
    out = np.zeros((m, group_sum_cols(g * group)), np.float32)
    out[:, :g] = hi
    out[:, g:2 * g] = r - hi
    return out


def rotquant(x_bits: np.ndarray, rot_group: int, mode: str, swiglu: bool = False, act_group: int = 0):  # noqa: F811
    """The activation stage: (optional SwiGLU) -> rotation -> quantization.

    ``x_bits``: bf16 bits (M, K) or (M, 2K) with ``swiglu``.  ``mode``: "int8" (per token, 127),
    "int4" (per token, 7) or "int4_group" (per ``act_group`` group, bf16_up scale).  The per-token modes
    round the SwiGLU product to bf16 once (comfy-kitchen's contract); "int4_group" keeps it in fp32 like the
    reference's per-group quantizer.  Returns (codes int16 (M, K), scales).
    """
    if swiglu:
        v = swiglu_product(x_bits, round_bf16=(mode != "int4_group"))
    else:
        v = bf16_bits_to_f32(x_bits)
    r = fwht_stages(v, rot_group)
    if mode == "int8":
        return quant_rowwise(r, INT8_MAX)
    if mode == "int4":
        return quant_rowwise(r, INT4_MAX)
    if mode == "int4_group":
        return quant_groupwise_bf16up(r, act_group, INT4_MAX)
    raise ValueError(mode)


# ----------------------------------------------------------------------------------------------
# weight quantization (the converter's rotate-and-quantize step)
# ----------------------------------------------------------------------------------------------

def weight_quant_convrot_rowwise(w: np.ndarray, rot_group: int):
    """ConvRot W4A4 weight: rotate, then per-row int4 (``node/__init__.py:93-97``).

    ``s = max(amax_row / 7, 1e-12)``; ``q = clamp(rint(wr / s), -7, 7)``.  Returns (codes (N, K) int16,
    scale (N,) f32).
    """
    wr = fwht_stages(np.asarray(w, dtype=F32), rot_group)
    am = np.abs(wr).max(axis=1)
    s = np.maximum(am / F32(7.0), F32(1e-12)).astype(F32)
    q = np.clip(np.rint(wr / s[:, None]), -7, 7).astype(np.int16)
    return q, s


def weight_quant_groupwise_bf16up(w: np.ndarray, rot_group: int, group: int = 128):
    """Per-group int4 weight with the scale rounded up to bf16 (``node/__init__.py:98-112``, pol 1/3/4).

    Returns (codes (N, K) int16 in [-7, 7], scale f32 (K/G, N)).
    """
    wr = fwht_stages(np.asarray(w, dtype=F32), rot_group)
    n, k = wr.shape
    g = wr.reshape(n, k // group, group)
    am = np.abs(g).max(axis=2)
    s = bf16_up(np.maximum(am / F32(7.0), F32(1e-30)))
    q = np.clip(np.rint(g / s[..., None]), -7, 7).astype(np.int16).reshape(n, k)
    return q, np.ascontiguousarray(s.T)


def weight_quant_int8_rowwise(w: np.ndarray, rot_group: int):
    """int8_tensorwise weight (optionally ConvRot): per-row absmax/127, scale (N, 1) f32."""
    wr = fwht_stages(np.asarray(w, dtype=F32), rot_group)
    am = np.abs(wr).max(axis=1)
    s = np.maximum(am / F32(127.0), F32(1e-12)).astype(F32)
    q = np.clip(np.rint(wr / s[:, None]), -127, 127).astype(np.int16)
    return q, s.reshape(-1, 1)


def weight_quant_affine(w: np.ndarray, rot_group: int, group: int = 128):
    """Asymmetric per-group int4 in the awq_w4a16 layout ``W = (q - 8) * scale + zeros``.

    Per (row, K-group) of the rotated weight: ``s = bf16(max((max - min) / 15, 1e-8))``,
    ``z = bf16(min + 8 * s)``, ``q = clamp(rint((w - z) / s) + 8, 0, 15)`` (codes from the STORED s and z).
    Returns (codes (N, K) uint4 in int16, scale bf16-valued f32 (K/G, N), zeros bf16-valued f32 (K/G, N)).
    """
    wr = fwht_stages(np.asarray(w, dtype=F32), rot_group)
    n, k = wr.shape
    g = wr.reshape(n, k // group, group)
    lo = g.min(axis=2)
    hi = g.max(axis=2)
    s = bf16_round(np.maximum((hi - lo) / F32(15.0), F32(1e-8)))
    z = bf16_round(lo + F32(8.0) * s)
    q = np.clip(np.rint((g - z[..., None]) / s[..., None]) + F32(8.0), 0, 15).astype(np.int16).reshape(n, k)
    return q, np.ascontiguousarray(s.T), np.ascontiguousarray(z.T)


def dequant_affine(codes: np.ndarray, scale: np.ndarray, zeros: np.ndarray) -> np.ndarray:
    """(q - 8) * scale + zeros in float64 (exact for bf16 scale/zero), the awq_w4a16 formula."""
    q = np.asarray(codes, dtype=np.float64)
    n, k = q.shape
    g = k // scale.shape[0]
    s = np.asarray(scale, np.float64).T[:, :, None]
    z = np.asarray(zeros, np.float64).T[:, :, None]
    return ((q.reshape(n, k // g, g) - 8.0) * s + z).reshape(n, k)


# ----------------------------------------------------------------------------------------------
# GEMM + epilogues
# ----------------------------------------------------------------------------------------------

def int_gemm(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Exact sum_k a[m,k] * b[n,k] as float64 (exact: every partial sum of int8 x int8 products stays far
    below 2**53; float64 BLAS is used because numpy has no fast integer matmul)."""
    return np.asarray(a, np.float64) @ np.asarray(b, np.float64).T


def linear_rowcol(qa, sa, qw, sw, bias=None) -> np.ndarray:
    """(sum qa*qw) * sa[m] * sw[n] + bias[n], float64 (the int4_linear / int8_linear epilogue)."""
    acc = int_gemm(qa, qw)
    out = acc * np.asarray(sa, np.float64).reshape(-1, 1) * np.asarray(sw, np.float64).reshape(1, -1)
    if bias is not None:
        out = out + np.asarray(bias, np.float64).reshape(1, -1)
    return out


def linear_affine(qx, sx, qw_u4, scale, zeros, bias=None, group: int = 128) -> np.ndarray:
    """y = sx[m] * sum_g (s[g,n] * sum_{k in g} qx*(q-8) + z[g,n] * sum_{k in g} qx) + bias, float64."""
    qx = np.asarray(qx, np.float64)
    w = np.asarray(qw_u4, np.float64) - 8.0
    m, k = qx.shape
    ng = k // group
    out = np.zeros((m, w.shape[0]), np.float64)
    s = np.asarray(scale, np.float64)
    z = np.asarray(zeros, np.float64)
    for g in range(ng):
        sl = slice(g * group, (g + 1) * group)
        p = qx[:, sl] @ w[:, sl].T          # exact integers in float64
        r = qx[:, sl].sum(axis=1)
        out += p * s[g][None, :] + r[:, None] * z[g][None, :]
    out *= np.asarray(sx, np.float64).reshape(-1, 1)
    if bias is not None:
        out = out + np.asarray(bias, np.float64).reshape(1, -1)
    return out


def linear_groupwise(qa, sa_g, qw, sw_g, bias=None, group: int = 128) -> np.ndarray:
    """Per-group scales on both sides (``g64_bench6.py:56-60``, policy 4): sa_g (K/G, M), sw_g (K/G, N)."""
    qa = np.asarray(qa, np.float64)
    qw = np.asarray(qw, np.float64)
    m, k = qa.shape
    out = np.zeros((m, qw.shape[0]), np.float64)
    for g in range(k // group):
        sl = slice(g * group, (g + 1) * group)
        out += (qa[:, sl] @ qw[:, sl].T) * np.asarray(sa_g[g], np.float64)[:, None] * \
            np.asarray(sw_g[g], np.float64)[None, :]
    if bias is not None:
        out = out + np.asarray(bias, np.float64).reshape(1, -1)
    return out


def intratio_acc(qa, qw, cw, group: int) -> np.ndarray:
    """Integer weight ratios per group (policies 5/7/15/17, ``g64_gemm6.cu:8-11``; ``g64_bench6.py:62-67``):
    acc[m, n] = sum_g cw[g, n] * sum_{k in g} qa[m, k] * qw[n, k], exact (int64)."""
    qa = np.asarray(qa, np.int64)
    qw = np.asarray(qw, np.int64)
    cw = np.asarray(cw, np.int64)
    m, k = qa.shape
    acc = np.zeros((m, qw.shape[0]), np.int64)
    for g in range(k // group):
        sl = slice(g * group, (g + 1) * group)
        acc += (qa[:, sl] @ qw[:, sl].T) * cw[g][None, :]
    return acc


def linear_intratio(qa, sa, qw, sb, cw, group: int, bias=None) -> np.ndarray:
    """The policies' output in the reference kernel's fp32 order (``g64_gemm6.cu:306-330``): t = fp32(fp32(acc) * sa[m]),
    then t * sb[n] + bias[n] with one rounding (a fused multiply-add), as float32 values."""
    acc = intratio_acc(qa, qw, cw, group)
    t = (acc.astype(np.float32) * np.asarray(sa, np.float32).reshape(-1, 1)).astype(np.float32)
    b = np.zeros(acc.shape[1], np.float64) if bias is None else np.asarray(bias, np.float64)
    return (t.astype(np.float64) * np.asarray(sb, np.float32).astype(np.float64).reshape(1, -1) + b.reshape(1, -1)
            ).astype(np.float32)


def dequant_matmul(x_deq: np.ndarray, w_deq: np.ndarray, bias=None) -> np.ndarray:
    """F.linear in float64 of already-dequantized operands (the reference's dequantize-and-matmul path)."""
    out = np.asarray(x_deq, np.float64) @ np.asarray(w_deq, np.float64).T
    if bias is not None:
        out = out + np.asarray(bias, np.float64).reshape(1, -1)
    return out


def rel_l2(ref: np.ndarray, got: np.ndarray) -> float:
    ref = np.asarray(ref, np.float64)
    got = np.asarray(got, np.float64)
    den = np.linalg.norm(ref)
    return float(np.linalg.norm(got - ref) / (den if den > 0 else 1.0))


# ----------------------------------------------------------------------------------------------
# seeded synthetic inputs (the benchmark shapes' value distributions)
# ----------------------------------------------------------------------------------------------

def synth_activations(m: int, k: int, seed: int = 0, outlier_frac: float = 0.01, outlier_gain: float = 20.0):
    """X ~ N(0,1) with ``outlier_frac`` of the channels multiplied by ``outlier_gain``; bf16 bits (M, K)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k), dtype=np.float32)
    n_out = max(1, int(round(outlier_frac * k))) if outlier_frac > 0 else 0
    if n_out:
        cols = rng.permutation(k)[:n_out]
        x[:, cols] *= F32(outlier_gain)
    return f32_to_bf16_bits(x)


def synth_weight(n: int, k: int, seed: int = 1, std: float = 0.02) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((n, k), dtype=np.float32) * F32(std)).astype(F32)


def synth_bias(n: int, seed: int = 2, std: float = 0.01) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return f32_to_bf16_bits(rng.standard_normal(n, dtype=np.float32) * F32(std))
