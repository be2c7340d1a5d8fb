"""ComfyUI quant-format plugin boundary: layout classes, their ``QUANT_ALGOS`` entries and registration.

Mirrors the plugin API comfy-quant-bench extends (``patches/comfyui_awq_w4a16_format.patch:25-100``) and the
shape of its own third-party layout plugin (``custom_nodes/comfy-lowbit-loader/layout.py:27-91``):

* a layout class with a frozen ``Params`` dataclass and the classmethods ``quantize(tensor, **kw)``,
  ``dequantize(qdata, params)``, ``get_plain_tensors(qtensor)`` and ``state_dict_tensors(qdata, params)``;
* ``QUANT_ALGOS[format] = {"storage_t", "parameters", "comfy_tensor_layout", "quantize_input",
  "params_from_state_dict"}`` with the reader signature ``(layer_name, module, weight, pop_scale, layer_conf)``;
* ``register_layout_class(name, cls)``.

``register()`` installs the layouts into a live ComfyUI (``comfy.quant_ops``) when one is importable and into
this module's own registry otherwise, so ``comfy_ops.Linear`` and the tests run without ComfyUI.  The linear
itself always goes through ``ops`` (the CUDA kernels); ``dequantize`` is the layout API's reconstruction for
callers that need the float weight (LoRA patching, inspection) and is not a fallback of the linear.
"""
from __future__ import annotations

import logging
from dataclasses import dataclass, field

import torch

from . import formats as F


@dataclass(frozen=True)
class BaseLayoutParams:
    scale: torch.Tensor
    orig_dtype: torch.dtype = torch.bfloat16
    orig_shape: tuple = ()

    def _tensor_fields(self):
        return ["scale"]


class QuantizedLayout:
    """Base of the layouts: quantize / dequantize / plain tensors / state-dict tensors."""
    MIN_SM_VERSION = (10, 0)
    QUANTIZES_INPUT = True
    Params = BaseLayoutParams

    @classmethod
    def quantize(cls, tensor: torch.Tensor, **kwargs):
        raise NotImplementedError

    @classmethod
    def dequantize(cls, qdata: torch.Tensor, params) -> torch.Tensor:
        raise NotImplementedError

    @classmethod
    def get_plain_tensors(cls, qtensor):
        return qtensor.qdata, qtensor.params.scale

    @classmethod
    def state_dict_tensors(cls, qdata, params) -> dict:
        return {"": qdata, "_scale": params.scale}

    @classmethod
    def linear(cls, x, qdata, params, bias=None, input_act=None):
        raise NotImplementedError


# ---------------------------------------------------------------------------------------------------
# helpers shared by the dequantize methods (float reconstruction of the stored weight)
# ---------------------------------------------------------------------------------------------------

def _unpack_nibbles(qdata: torch.Tensor, signed: bool) -> torch.Tensor:
    u = qdata.view(torch.uint8).to(torch.int16)
    v = torch.stack([u & 0xF, (u >> 4) & 0xF], dim=-1).reshape(qdata.shape[0], -1)
    return torch.where(v >= 8, v - 16, v) if signed else v


def _hadamard(n: int, device, dtype=torch.float32) -> torch.Tensor:
    h4 = 0.5 * torch.tensor([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=torch.float64)
    h = torch.ones(1, 1, dtype=torch.float64)
    while h.shape[0] < n:
        h = torch.kron(h, h4)
    return h.to(device=device, dtype=dtype)


def _unrotate(w: torch.Tensor, group: int) -> torch.Tensor:
    """Undo the block rotation of a weight (the Hadamard blocks are symmetric involutions)."""
    if not group:
        return w
    n, k = w.shape
    return (w.reshape(n, k // group, group) @ _hadamard(group, w.device)).reshape(n, k)


# ---------------------------------------------------------------------------------------------------
# layouts
# ---------------------------------------------------------------------------------------------------

class B200ConvRotW4A4Layout(QuantizedLayout):
    """ConvRot W4A4: rotated per-row symmetric int4 weight [N, K/2] + f32 scale [N]."""

    @dataclass(frozen=True)
    class Params(BaseLayoutParams):
        convrot_groupsize: int = 256
        quant_group_size: int = 64
        linear_dtype: str = "int4"

    @classmethod
    def quantize(cls, tensor, convrot_groupsize=256, quant_group_size=64, linear_dtype="int4", **kw):
        from .ops import quantize_convrot_w4a4_weight
        q, s = quantize_convrot_w4a4_weight(tensor, convrot_groupsize, quant_group_size, 0)
        return q, cls.Params(scale=s, orig_dtype=tensor.dtype, orig_shape=tuple(tensor.shape),
                             convrot_groupsize=convrot_groupsize, quant_group_size=quant_group_size,
                             linear_dtype=linear_dtype)

    @classmethod
    def dequantize(cls, qdata, params):
        w = _unpack_nibbles(qdata, True).float() * params.scale.float().reshape(-1, 1)
        return _unrotate(w, params.convrot_groupsize).to(params.orig_dtype)

    @classmethod
    def linear(cls, x, qdata, params, bias=None, input_act=None):
        from .ops import convrot_w4a4_linear
        return convrot_w4a4_linear(x, qdata, params.scale, bias, convrot_groupsize=params.convrot_groupsize,
                                   quant_group_size=params.quant_group_size, linear_dtype=params.linear_dtype,
                                   input_act=input_act)


class B200AffineW4A8Layout(QuantizedLayout):
    """awq-layout affine int4 weight (uint4 [N, K/2], bf16 scale/zeros [K/G, N]) with int8 activations."""

    @dataclass(frozen=True)
    class Params(BaseLayoutParams):
        zeros: torch.Tensor = None
        group_size: int = 128
        convrot_groupsize: int = 0

        def _tensor_fields(self):
            return ["scale", "zeros"]

    @classmethod
    def quantize(cls, tensor, group_size=128, convrot_groupsize=0, **kw):
        from .ops import quantize_affine_w4_weight
        q, s, z = quantize_affine_w4_weight(tensor, group_size, convrot_groupsize)
        return q, cls.Params(scale=s, zeros=z, orig_dtype=tensor.dtype, orig_shape=tuple(tensor.shape),
                             group_size=group_size, convrot_groupsize=convrot_groupsize)

    @classmethod
    def dequantize(cls, qdata, params):
        n = qdata.shape[0]
        k = qdata.shape[1] * 2
        g = params.group_size
        codes = _unpack_nibbles(qdata, False).float().view(n, k // g, g)
        w = ((codes - 8.0) * params.scale.float().t().unsqueeze(-1) + params.zeros.float().t().unsqueeze(-1)).view(n, k)
        return _unrotate(w, params.convrot_groupsize).to(params.orig_dtype)

    @classmethod
    def get_plain_tensors(cls, qtensor):
        return qtensor.qdata, qtensor.params.scale, qtensor.params.zeros

    @classmethod
    def state_dict_tensors(cls, qdata, params):
        return {"": qdata, "_scale": params.scale, "_zeros": params.zeros}

    @classmethod
    def prepared_zeros(cls, params):
        """The GEMM's zero-point operand for these params, built on first use and kept on the params object
        (rebuilt if the zeros tensor is modified in place)."""
        from .ops import prepare_affine_zeros
        cached = params.__dict__.get("_zt")
        if cached is None or cached[0] != params.zeros._version or cached[1].device != params.zeros.device:
            cached = (params.zeros._version, prepare_affine_zeros(params.zeros, params.group_size))
            object.__setattr__(params, "_zt", cached)   # frozen dataclass: a cache, not a field
        return cached[1]

    @classmethod
    def linear(cls, x, qdata, params, bias=None, input_act=None):
        from .ops import w4a8_affine_linear
        return w4a8_affine_linear(x, qdata, params.scale, params.zeros, bias, group_size=params.group_size,
                                  convrot_groupsize=params.convrot_groupsize, input_act=input_act,
                                  zeros_prepared=cls.prepared_zeros(params))


class B200TensorWiseINT8Layout(QuantizedLayout):
    """int8_tensorwise: int8 weight [N, K] (optionally ConvRot) + f32 scale [N, 1]."""

    @dataclass(frozen=True)
    class Params(BaseLayoutParams):
        convrot: bool = False
        convrot_groupsize: int = 256

    @classmethod
    def quantize(cls, tensor, convrot=True, convrot_groupsize=256, **kw):
        from .ops import quantize_int8_convrot_weight
        q, s = quantize_int8_convrot_weight(tensor, convrot_groupsize if convrot else 0)
        return q, cls.Params(scale=s, orig_dtype=tensor.dtype, orig_shape=tuple(tensor.shape), convrot=convrot,
                             convrot_groupsize=convrot_groupsize)

    @classmethod
    def dequantize(cls, qdata, params):
        w = qdata.float() * params.scale.float().reshape(-1, 1)
        return _unrotate(w, params.convrot_groupsize if params.convrot else 0).to(params.orig_dtype)

    @classmethod
    def linear(cls, x, qdata, params, bias=None, input_act=None):
        from .ops import int8_linear
        return int8_linear(x, qdata, params.scale, bias, convrot=params.convrot,
                           convrot_groupsize=params.convrot_groupsize, input_act=input_act)


@dataclass
class QuantizedWeight:
    """A quantized weight: packed data + layout name + layout params (the role of comfy's QuantizedTensor)."""
    qdata: torch.Tensor
    layout: str
    params: object
    extra: dict = field(default_factory=dict)

    @property
    def layout_cls(self):
        return get_layout_class(self.layout)

    @property
    def shape(self):
        return self.params.orig_shape

    def dequantize(self) -> torch.Tensor:
        return self.layout_cls.dequantize(self.qdata, self.params)

    def linear(self, x, bias=None, input_act=None):
        return self.layout_cls.linear(x, self.qdata, self.params, bias, input_act)

    def to(self, device):
        def mv(v):
            return v.to(device) if isinstance(v, torch.Tensor) else v
        p = self.params
        kw = {f: mv(getattr(p, f)) for f in p.__dataclass_fields__}
        return QuantizedWeight(self.qdata.to(device), self.layout, type(p)(**kw), dict(self.extra))


# ---------------------------------------------------------------------------------------------------
# registry + QUANT_ALGOS
# ---------------------------------------------------------------------------------------------------

_LAYOUTS: dict[str, type] = {}
QUANT_ALGOS: dict[str, dict] = {}


def register_layout_class(name: str, cls: type) -> None:
    _LAYOUTS[name] = cls


def get_layout_class(name: str) -> type:
    try:
        return _LAYOUTS[name]
    except KeyError:
        raise KeyError(f"layout {name!r} is not registered") from None


def _convrot_params(layer_name, module, weight, pop_scale, layer_conf):
    scale = pop_scale("weight_scale")
    if scale is None:
        raise ValueError(f"Missing ConvRot W4A4 weight_scale for layer {layer_name}")
    return {"scale": scale, "convrot_groupsize": int(layer_conf.get("convrot_groupsize", 256)),
            "quant_group_size": int(layer_conf.get("quant_group_size", 64)),
            "linear_dtype": str(layer_conf.get("linear_dtype", "int4"))}


def _affine_params(layer_name, module, weight, pop_scale, layer_conf):
    # uint4 weight (packed int8 [N, K/2]), per-group scale and zero [K/G, N]: W = (q - 8) * scale + zeros.
    scale = pop_scale("weight_scale")
    zeros = pop_scale("weight_zeros")
    if scale is None or zeros is None:
        raise ValueError(f"Missing affine W4A8 scale/zeros for layer {layer_name}")
    params_conf = layer_conf.get("params", {})
    if not isinstance(params_conf, dict):
        params_conf = {}
    return {"scale": scale, "zeros": zeros,
            "group_size": int(layer_conf.get("group_size", params_conf.get("group_size", 128))),
            "convrot_groupsize": int(layer_conf.get("convrot_groupsize", params_conf.get("convrot_groupsize", 0)))}


def _int8_params(layer_name, module, weight, pop_scale, layer_conf):
    scale = pop_scale("weight_scale")
    if scale is None:
        raise ValueError(f"Missing int8 weight_scale for layer {layer_name}")
    return {"scale": scale, "convrot": bool(layer_conf.get("convrot", False)),
            "convrot_groupsize": int(layer_conf.get("convrot_groupsize", 256))}


LAYOUTS = {
    "B200ConvRotW4A4Layout": B200ConvRotW4A4Layout,
    "B200AffineW4A8Layout": B200AffineW4A8Layout,
    "B200TensorWiseINT8Layout": B200TensorWiseINT8Layout,
}

ALGOS = {
    F.ConvrotW4A4.name: {"storage_t": torch.int8, "parameters": {"weight_scale"},
                         "comfy_tensor_layout": "B200ConvRotW4A4Layout", "quantize_input": True,
                         "params_from_state_dict": _convrot_params},
    F.AffineW4A8.name: {"storage_t": torch.int8, "parameters": {"weight_scale", "weight_zeros"},
                        "comfy_tensor_layout": "B200AffineW4A8Layout", "quantize_input": True,
                        "params_from_state_dict": _affine_params},
    F.Int8Tensorwise.name: {"storage_t": torch.int8, "parameters": {"weight_scale"},
                            "comfy_tensor_layout": "B200TensorWiseINT8Layout", "quantize_input": True,
                            "params_from_state_dict": _int8_params},
}


def register(target=None) -> str:
    """Register the layouts and formats.  ``target``: a ``comfy.quant_ops``-like module; by default the live
    ComfyUI one if importable, else this module's registry.  Returns where they went."""
    if target is None:
        try:
            import comfy.quant_ops as target  # type: ignore[no-redef]
        except Exception:  # noqa: BLE001 - no ComfyUI in this process
            target = None
    for name, cls in LAYOUTS.items():
        register_layout_class(name, cls)
        if target is not None:
            target.register_layout_class(name, cls)
    for fmt, algo in ALGOS.items():
        QUANT_ALGOS[fmt] = dict(algo)
        if target is not None:
            target.QUANT_ALGOS[fmt] = dict(algo)
    where = getattr(target, "__name__", "comfy_quant_bench_b200.layout") if target is not None else \
        "comfy_quant_bench_b200.layout"
    logging.info("comfy_quant_bench_b200 layouts registered in %s", where)
    return where


register_local = register  # alias kept for callers that want the local registry explicitly
