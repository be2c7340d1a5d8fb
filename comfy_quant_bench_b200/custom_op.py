"""Opaque ``torch.library`` custom ops for the quantized linears (torch.compile boundary).

Same contract as comfy-quant-bench's ``compile_support.py:75-117``: the linear is registered as a
``torch.library.custom_op`` with a fake (meta) implementation returning ``x.new_empty(*x.shape[:-1], N)``, so
Dynamo treats the CUDA kernels as one opaque node instead of tracing into a data pointer.  The ops are
registered once, on import.
"""
from __future__ import annotations

import torch

from . import ops

NAMESPACE = "comfy_quant_b200"


@torch.library.custom_op(f"{NAMESPACE}::convrot_w4a4_linear", mutates_args=())
def convrot_w4a4_linear(x: torch.Tensor, qweight: torch.Tensor, wscales: torch.Tensor, bias: torch.Tensor | None,
                        convrot_groupsize: int, quant_group_size: int, linear_dtype: str) -> torch.Tensor:
    return ops.convrot_w4a4_linear(x, qweight, wscales, bias, convrot_groupsize=convrot_groupsize,
                                   quant_group_size=quant_group_size, linear_dtype=linear_dtype)


@convrot_w4a4_linear.register_fake
def _(x, qweight, wscales, bias, convrot_groupsize, quant_group_size, linear_dtype):
    # qweight is [out_features, in_features // 2]: int8 storage holding two signed int4 each
    return x.new_empty((*x.shape[:-1], qweight.shape[0]))


@torch.library.custom_op(f"{NAMESPACE}::w4a8_affine_linear", mutates_args=())
def w4a8_affine_linear(x: torch.Tensor, qweight: torch.Tensor, scale: torch.Tensor, zeros: torch.Tensor,
                       bias: torch.Tensor | None, group_size: int, convrot_groupsize: int) -> torch.Tensor:
    return ops.w4a8_affine_linear(x, qweight, scale, zeros, bias, group_size=group_size,
                                  convrot_groupsize=convrot_groupsize)


@w4a8_affine_linear.register_fake
def _(x, qweight, scale, zeros, bias, group_size, convrot_groupsize):
    return x.new_empty((*x.shape[:-1], qweight.shape[0]))


@torch.library.custom_op(f"{NAMESPACE}::int8_linear", mutates_args=())
def int8_linear(x: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor, bias: torch.Tensor | None,
                convrot: bool, convrot_groupsize: int) -> torch.Tensor:
    return ops.int8_linear(x, weight, weight_scale, bias, convrot=convrot, convrot_groupsize=convrot_groupsize)


@int8_linear.register_fake
def _(x, weight, weight_scale, bias, convrot, convrot_groupsize):
    return x.new_empty((*x.shape[:-1], weight.shape[0]))


def dispatching_convrot_w4a4_linear(x, qweight, wscales, bias=None, convrot_groupsize=256, quant_group_size=64,
                                    linear_dtype="int4"):
    """Drop-in for comfy-kitchen's ``convrot_w4a4_linear`` that goes through the opaque op."""
    return torch.ops.comfy_quant_b200.convrot_w4a4_linear(x, qweight, wscales, bias, int(convrot_groupsize),
                                                          int(quant_group_size), str(linear_dtype))
