"""The reference's CPU path for the W4A8 linear, timed as the CPU baseline (TEST INFRASTRUCTURE ONLY).

comfy-kitchen's eager backend - the path comfy-quant-bench takes without a native kernel - quantizes the
activations with torch ops, dequantizes the packed weight on every call and runs a plain ``F.linear``
(``patches/tests/test_comfy_kitchen_awq.py:30-37, 51-55``: unpack, ``(q - 8) * scale + zeros``, matmul;
``tools/weight_balance.py:161-173``: dequantize + un-rotate).  This module restates one such call with torch CPU
ops on all host threads:

    x --(rotation x.reshape(M, K/g, g) @ H, per-token int8)--> xq*sx --F.linear--> dequant(W)  (+ bias)

The rotation is the reference's matrix form (``experiments/qwen21-kernel/kernels/g64_quant_test.py:64``), so its
fp32 rounding differs from the radix-4 stages of ``ref.fwht_stages``; codes agree with ``ref.rotquant`` up to
+-1 at rounding ties (``tests/test_oracle_properties.py``).

Only ``bench.py`` (its ``cpu_baseline`` leg and ``--impl reference``) and the tests use it.
"""
from __future__ import annotations

import time

import numpy as np
import torch

from . import ref

_HADAMARD: dict[int, torch.Tensor] = {}


def hadamard_f32(group: int) -> torch.Tensor:
    """kron^p(H4r)/2^p as a float32 torch matrix (cached)."""
    if group not in _HADAMARD:
        _HADAMARD[group] = torch.from_numpy(ref.build_hadamard(group).astype(np.float32))
    return _HADAMARD[group]


def dequant_affine_torch(qweight: torch.Tensor, scale: torch.Tensor, zeros: torch.Tensor, group: int) -> torch.Tensor:
    """(q - 8) * scale + zeros in fp32 from packed uint4 [N, K/2] and [K/G, N] scale/zeros (the awq formula).

    One float pass over the weight, updated in place: (q - 8) is exact, then one rounding for the multiply and
    one for the add, as in the reference's chain.
    """
    n, kh = qweight.shape
    k = 2 * kh
    u = qweight.view(torch.uint8)
    codes = torch.stack([u & 0xF, u >> 4], dim=-1).view(n, k // group, group).to(torch.float32)
    s = scale.to(torch.float32).t().unsqueeze(-1)
    z = zeros.to(torch.float32).t().unsqueeze(-1)
    return codes.sub_(8.0).mul_(s).add_(z).view(n, k)


def rotquant_int8_torch(x: torch.Tensor, rot: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token int8 activation quantization of bf16 x [M, K] after the block rotation, in torch (all threads).

    ``scale = max(absmax * (1/127), 1e-10)``, ``q = clamp(round(v * (1/scale)), -127, 127)`` with round half to
    even (``tools/activation_balance.py:65-71`` with ``limit=127``).  Returns (codes float32 [M, K], scale [M]).
    """
    m, k = x.shape
    v = x.to(torch.float32)
    if rot:
        v = torch.matmul(v.view(m, k // rot, rot), hadamard_f32(rot)).view(m, k)
    am = v.abs().amax(dim=1) if k else torch.zeros(m)
    scale = torch.clamp(am * np.float32(1.0 / 127.0), min=1e-10)
    inv = torch.reciprocal(scale)
    q = torch.clamp(torch.round(v.mul_(inv[:, None])), -127, 127)
    return q, scale


def w4a8_affine_call(x: torch.Tensor, rot: int, qweight: torch.Tensor, scale: torch.Tensor, zeros: torch.Tensor,
                     bias: torch.Tensor | None, group: int = 128, timings: list | None = None) -> torch.Tensor:
    """One linear call on the CPU: activation quantization, weight dequantization, fp32 F.linear (+ bias).

    ``timings``: if given, the call appends (activation quant s, weight dequant s, F.linear s).
    """
    t0 = time.perf_counter()
    q, sx = rotquant_int8_torch(x, rot)
    xd = q.mul_(sx[:, None])
    t1 = time.perf_counter()
    w = dequant_affine_torch(qweight, scale, zeros, group)
    t2 = time.perf_counter()
    y = torch.nn.functional.linear(xd, w, None if bias is None else bias.to(torch.float32))
    t3 = time.perf_counter()
    if timings is not None:
        timings.append((t1 - t0, t2 - t1, t3 - t2))
    return y
