"""The reference's CPU path for the W4A8 / W4A4 linear, timed as the CPU baseline (TEST INFRASTRUCTURE ONLY).

comfy-kitchen's eager backend - the path comfy-quant-bench takes without a native kernel - dequantizes the
packed weight and runs a plain ``F.linear`` (``patches/tests/test_comfy_kitchen_awq.py:30-37, 51-55``: unpack,
``(q - 8) * scale + zeros``, matmul; ``tools/weight_balance.py:161-173``: dequantize + un-rotate).  This module
restates that path with torch CPU ops (all host threads) on the oracle's quantized activations:

    x --(oracle rotation + per-token int8)--> xq*sx --F.linear--> dequant(W)  (+ bias)

Only ``bench.py`` (its ``cpu_baseline`` leg and ``--impl reference``) and the tests use it.
"""
from __future__ import annotations

import numpy as np
import torch

from . import ref


def dequant_affine_torch(qweight: torch.Tensor, scale: torch.Tensor, zeros: torch.Tensor, group: int) -> torch.Tensor:
    """(q - 8) * scale + zeros in fp32 from packed uint4 [N, K/2] and [K/G, N] scale/zeros (the awq formula)."""
    n, kh = qweight.shape
    k = 2 * kh
    u = qweight.view(torch.uint8).to(torch.int32)
    codes = torch.stack([u & 0xF, (u >> 4) & 0xF], dim=-1).reshape(n, k).to(torch.float32)
    s = scale.to(torch.float32).t().unsqueeze(-1)
    z = zeros.to(torch.float32).t().unsqueeze(-1)
    return ((codes.view(n, k // group, group) - 8.0) * s + z).view(n, k)


def w4a8_affine_step(x_bits: np.ndarray, rot: int, qweight: torch.Tensor, scale: torch.Tensor, zeros: torch.Tensor,
                     bias: torch.Tensor | None, group: int = 128) -> torch.Tensor:
    """One linear call on the CPU: activation quantization (oracle), weight dequantization, F.linear (fp32)."""
    qx, sx = ref.rotquant(x_bits, rot, "int8")
    xd = torch.from_numpy(qx.astype(np.float32) * sx[:, None])
    w = dequant_affine_torch(qweight, scale, zeros, group)
    return torch.nn.functional.linear(xd, w, None if bias is None else bias.to(torch.float32))
