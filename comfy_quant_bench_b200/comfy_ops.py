"""The ComfyUI ``ops`` surface of the quantized linear: ``Linear`` and ``linear_input_act``.

Keeps the signatures comfy-quant-bench patches in ComfyUI's ``comfy/ops.py``:

* ``Linear(in_features, out_features, bias=True, device=None, dtype=None)`` whose ``forward(x)`` runs the
  layer's quantized layout (the ``mixed_precision_ops().Linear`` role) and whose ``load_state_dict`` reads a
  layer's scales through ``QUANT_ALGOS[format]["params_from_state_dict"]``
  (``patches/comfyui_awq_w4a16_format.patch:14-24``; the ``comfy_quant`` per-layer JSON or
  ``_quantization_metadata`` gives the format);
* ``linear_input_act(linear, x, input_act, act_weight=None, act_eps=0.0, residual=None, residual_scale=None)``
  (``patches/comfyui_swiglu_triton_env.patch:62-104``): ``linear(act(x))`` with ``act`` folded into the
  activation quantizer when the layout supports it (SwiGLU: ``x = [gate | up]``), then the optional residual
  ``residual + residual_scale * out``.

Unlike the reference there is no eager fallback for the quantized linear itself: unsupported activations are
applied eagerly *before* the quantized call (as ComfyUI's own path does), the linear always runs the kernels.
"""
from __future__ import annotations

import json

import torch

from . import layout as L


def _swiglu_eager(x: torch.Tensor) -> torch.Tensor:
    gate, up = x.chunk(2, dim=-1)
    return torch.nn.functional.silu(gate).mul_(up)


INPUT_ACT_EAGER = {
    "gelu_tanh": lambda x: torch.nn.functional.gelu(x, approximate="tanh"),
    "swiglu": _swiglu_eager,
}

# activations the quantizer kernels fold in, per layout
_FUSED_ACTS = {"B200ConvRotW4A4Layout": {"swiglu"}, "B200AffineW4A8Layout": {"swiglu"},
               "B200TensorWiseINT8Layout": {"swiglu"}}


class Linear(torch.nn.Module):
    """A quantized Linear: ``weight`` is a ``layout.QuantizedWeight`` once a quantized state dict is loaded."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None, dtype=None):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.weight = None
        self.quant_format = None
        self.layout_type = None
        self._orig_shape = (out_features, in_features)
        self.compute_dtype = dtype or torch.bfloat16
        self.bias = torch.nn.Parameter(torch.zeros(out_features, device=device, dtype=dtype or torch.bfloat16),
                                       requires_grad=False) if bias else None
        self.weight_function = []
        self.bias_function = []

    # -- loading ------------------------------------------------------------------------------------
    @classmethod
    def from_quantized(cls, qweight: "L.QuantizedWeight", bias: torch.Tensor | None = None, fmt: str | None = None):
        n, k = qweight.params.orig_shape
        lin = cls(k, n, bias=bias is not None, device=qweight.qdata.device, dtype=qweight.params.orig_dtype)
        lin.weight = qweight
        lin.layout_type = qweight.layout
        lin.quant_format = fmt
        if bias is not None:
            lin.bias = torch.nn.Parameter(bias.to(qweight.qdata.device), requires_grad=False)
        return lin

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                              error_msgs):
        key = prefix + "weight"
        conf_key = prefix + "comfy_quant"
        layer_conf = None
        if conf_key in state_dict:
            layer_conf = json.loads(bytes(state_dict.pop(conf_key).to(torch.uint8).tolist()).decode("utf-8"))
        elif isinstance(local_metadata, dict) and "comfy_quant" in local_metadata:
            layer_conf = local_metadata["comfy_quant"]
        if layer_conf is None or key not in state_dict:
            return super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys,
                                                 unexpected_keys, error_msgs)
        fmt = layer_conf.get("format")
        if fmt not in L.QUANT_ALGOS:
            L.register()
        if fmt not in L.QUANT_ALGOS:
            error_msgs.append(f"{prefix}: unknown quantization format {fmt!r}")
            return
        algo = L.QUANT_ALGOS[fmt]
        qdata = state_dict.pop(key)

        def pop_scale(name, dtype=None):
            t = state_dict.pop(prefix + name, None)
            return t if t is None or dtype is None else t.view(dtype)

        kw = algo["params_from_state_dict"](prefix.rstrip("."), self, qdata, pop_scale, layer_conf)
        cls = L.get_layout_class(algo["comfy_tensor_layout"])
        params = cls.Params(orig_dtype=self.compute_dtype, orig_shape=self._orig_shape, **kw)
        self.weight = L.QuantizedWeight(qdata, algo["comfy_tensor_layout"], params)
        self.layout_type = algo["comfy_tensor_layout"]
        self.quant_format = fmt
        bkey = prefix + "bias"
        if bkey in state_dict:
            b = state_dict.pop(bkey)
            if self.bias is None:
                self.bias = torch.nn.Parameter(b, requires_grad=False)
            else:
                self.bias = torch.nn.Parameter(b.to(self.bias.dtype), requires_grad=False)
        elif self.bias is not None and strict:
            missing_keys.append(bkey)

    def quantized_state_dict(self, prefix: str = "") -> dict:
        """The layer's tensors as written to disk, plus the per-layer ``comfy_quant`` config."""
        w = self.weight
        out = {prefix + "weight" + suffix: t for suffix, t in w.layout_cls.state_dict_tensors(w.qdata, w.params).items()}
        if self.bias is not None:
            out[prefix + "bias"] = self.bias.data
        conf = {"format": self.quant_format}
        p = w.params
        for f in ("convrot_groupsize", "group_size", "convrot", "linear_dtype"):
            if hasattr(p, f):
                conf[f] = getattr(p, f)
        out[prefix + "comfy_quant"] = torch.tensor(list(json.dumps(conf).encode("utf-8")), dtype=torch.uint8)
        return out

    # -- compute ------------------------------------------------------------------------------------
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.weight is None:
            raise RuntimeError("Linear has no quantized weight loaded")
        if self.weight_function or self.bias_function:
            # a LoRA / weight patch needs the float weight: the layout reconstructs it, torch does the matmul
            w = self.weight.dequantize()
            for f in self.weight_function:
                w = f(w)
            b = self.bias
            for f in self.bias_function:
                b = f(b)
            return torch.nn.functional.linear(x, w.to(x.dtype), None if b is None else b.to(x.dtype))
        return self.weight.linear(x, self.bias)


def _fused_input_act(linear, x, input_act):
    """The quantized layer folds ``input_act`` into its activation quantizer, or None when it cannot."""
    w = getattr(linear, "weight", None)
    if (not isinstance(w, L.QuantizedWeight) or input_act not in _FUSED_ACTS.get(w.layout, ())
            or x.requires_grad or len(getattr(linear, "weight_function", ())) or len(getattr(linear, "bias_function", ()))):
        return None
    return w.linear(x, linear.bias, input_act=input_act)


def linear_input_act(linear, x, input_act, act_weight=None, act_eps=0.0, residual=None, residual_scale=None):
    """``linear(act(x))`` with ``act`` folded into the activation quantizer when possible, then the residual."""

    def _residual_out(out):
        if residual is None:
            return out
        if residual_scale is None:
            return residual + out
        return torch.addcmul(residual, out, residual_scale)

    if act_weight is not None:
        # the reference folds an RMS-norm weight into the INT8 quantizer; here it is applied eagerly first
        x = x * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + act_eps).to(x.dtype) * act_weight
    out = _fused_input_act(linear, x, input_act)
    if out is not None:
        return _residual_out(out)
    act = INPUT_ACT_EAGER.get(input_act)
    if act is None:
        raise ValueError(f"unknown input_act {input_act!r}")
    return _residual_out(linear(act(x)))


def mixed_precision_ops(quant_config: dict | None = None):
    """``comfy.ops.mixed_precision_ops(...)``-style namespace exposing ``Linear``."""
    class _Ops:
        pass
    _Ops.Linear = Linear
    return _Ops
