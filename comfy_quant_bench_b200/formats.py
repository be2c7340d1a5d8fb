"""Packed-tensor formats of the quantized-linear path: what a layer becomes on disk and in HBM.

Mirrors the format model of comfy-quant-bench's ``tools/_formats.py:53-293`` so checkpoints keep the same
tensor names, dtypes, shapes and ``_quantization_metadata`` JSON.  Each format answers:

    accepts(shape)         does the layer fit the format (divisibility of K)?
    tensors(name, shape)   output tensors, with dtype and shape, in write order
    layer_config()         the layer's entry in ``_quantization_metadata["layers"]``
    quantize(weight)       the B200 weight kernel, returning tensors in the order of ``tensors()``

``AffineW4A8`` is new here: the awq_w4a16 tensor layout (``W = (q - 8) * scale + zeros``, scale/zeros bf16
[K/G, N]) executed with per-token int8 activations by the W4A8 affine kernel.
"""
from __future__ import annotations

import json
from dataclasses import dataclass

import torch

FORMAT_VERSION = "1.0"


def _base(name: str) -> str:
    return name.removesuffix(".weight")


@dataclass(frozen=True)
class ConvrotW4A4:
    """ConvRot W4A4: int4 packed in I8 [N, K/2] + F32 per-row scale [N] (tools/_formats.py:53-76)."""
    convrot_groupsize: int = 256
    quant_group_size: int = 64
    name = "convrot_w4a4"

    def accepts(self, shape: list[int]) -> bool:
        return len(shape) == 2 and shape[1] % self.convrot_groupsize == 0

    def tensors(self, name: str, shape: list[int]) -> list[tuple[str, str, list[int]]]:
        rows, cols = shape
        return [(name, "I8", [rows, cols // 2]), (f"{_base(name)}.weight_scale", "F32", [rows])]

    def layer_config(self) -> dict:
        return {"format": self.name, "convrot_groupsize": self.convrot_groupsize}

    def quantize(self, weight: torch.Tensor) -> tuple[list[torch.Tensor], dict]:
        from .ops import quantize_convrot_w4a4_weight
        q, s = quantize_convrot_w4a4_weight(weight, convrot_groupsize=self.convrot_groupsize,
                                            quant_group_size=self.quant_group_size, stochastic_rounding=0)
        return [q, s], {}


@dataclass(frozen=True)
class AsymW4A8:
    """asym_w4a8_int8 (symmetric in practice): I8 [N, K/2], fp8 s_rel (U8) [N, K/gs], F32 s_channel [N] and,
    with the Lloyd-Max codebook, F32 codebook [16] (tools/_formats.py:79-125).

    The tensor layout is kept for drop-in loading; its quantizer (codebook fit + ALS scale refinement) lives in
    comfy-kitchen, whose source the reference does not vendor, so no kernel here claims to reproduce it.
    """
    group_size: int = 16
    convrot_groupsize: int = 256
    codebook: bool = True
    name = "asym_w4a8_int8"

    def accepts(self, shape: list[int]) -> bool:
        if len(shape) != 2:
            return False
        k = shape[1]
        if k % 16 or k % self.group_size or k % self.convrot_groupsize:
            return False
        if self.group_size < 4 or (16 % self.group_size and self.group_size % 16):
            return False
        return True

    def tensors(self, name: str, shape: list[int]) -> list[tuple[str, str, list[int]]]:
        rows, cols = shape
        base = _base(name)
        out = [(name, "I8", [rows, cols // 2]),
               (f"{base}.weight_s_rel", "U8", [rows, cols // self.group_size]),
               (f"{base}.weight_s_channel", "F32", [rows])]
        if self.codebook:
            out.append((f"{base}.weight_codebook", "F32", [16]))
        return out

    def layer_config(self) -> dict:
        return {"format": self.name, "group_size": self.group_size, "convrot_groupsize": self.convrot_groupsize}

    def quantize(self, weight: torch.Tensor):
        raise NotImplementedError("asym_w4a8_int8 weights come from comfy-kitchen's codebook/ALS quantizer, which is "
                                  "not part of this library; use AffineW4A8 for the W4A8 kernel")


@dataclass(frozen=True)
class Int8Tensorwise:
    """int8_tensorwise per row, with or without ConvRot: I8 [N, K] + F32 [N, 1] (tools/_formats.py:128-167)."""
    convrot: bool = True
    convrot_groupsize: int = 256
    name = "int8_tensorwise"

    def accepts(self, shape: list[int]) -> bool:
        return len(shape) == 2 and (not self.convrot or shape[1] % self.convrot_groupsize == 0)

    def tensors(self, name: str, shape: list[int]) -> list[tuple[str, str, list[int]]]:
        rows, cols = shape
        return [(name, "I8", [rows, cols]), (f"{name}_scale", "F32", [rows, 1])]

    def layer_config(self) -> dict:
        conf = {"format": self.name}
        if self.convrot:
            conf.update({"convrot": True, "convrot_groupsize": self.convrot_groupsize})
        return conf

    def quantize(self, weight: torch.Tensor) -> tuple[list[torch.Tensor], dict]:
        from .ops import quantize_int8_convrot_weight
        q, s = quantize_int8_convrot_weight(weight, group_size=self.convrot_groupsize if self.convrot else 0)
        return [q, s.float()], {}


@dataclass(frozen=True)
class AwqW4A16:
    """awq_w4a16: I8 [N, K/2] + BF16 scale and zeros [K/G, N] (tools/_formats.py:191-212)."""
    group_size: int = 32
    name = "awq_w4a16"

    def accepts(self, shape: list[int]) -> bool:
        return len(shape) == 2 and shape[1] % self.group_size == 0

    def tensors(self, name: str, shape: list[int]) -> list[tuple[str, str, list[int]]]:
        rows, cols = shape
        base = _base(name)
        return [(name, "I8", [rows, cols // 2]),
                (f"{base}.weight_scale", "BF16", [cols // self.group_size, rows]),
                (f"{base}.weight_zeros", "BF16", [cols // self.group_size, rows])]

    def layer_config(self) -> dict:
        return {"format": self.name, "group_size": self.group_size}

    def quantize(self, weight: torch.Tensor) -> tuple[list[torch.Tensor], dict]:
        from .ops import quantize_affine_w4_weight
        if self.group_size not in (64, 128):
            raise ValueError("the affine weight kernel supports group_size 64 and 128")
        q, s, z = quantize_affine_w4_weight(weight, group_size=self.group_size, convrot_groupsize=0)
        return [q, s, z], {}


@dataclass(frozen=True)
class AffineW4A8:
    """The W4A8 format: awq_w4a16 tensors (group 128), optional ConvRot, int8 per-token activations."""
    group_size: int = 128
    convrot_groupsize: int = 0
    name = "affine_w4a8"

    def accepts(self, shape: list[int]) -> bool:
        if len(shape) != 2:
            return False
        k = shape[1]
        return k % self.group_size == 0 and k % 256 == 0 and (self.convrot_groupsize == 0 or k % self.convrot_groupsize == 0)

    def tensors(self, name: str, shape: list[int]) -> list[tuple[str, str, list[int]]]:
        return AwqW4A16(self.group_size).tensors(name, shape)

    def layer_config(self) -> dict:
        conf = {"format": self.name, "group_size": self.group_size}
        if self.convrot_groupsize:
            conf["convrot_groupsize"] = self.convrot_groupsize
        return conf

    def quantize(self, weight: torch.Tensor) -> tuple[list[torch.Tensor], dict]:
        from .ops import quantize_affine_w4_weight
        q, s, z = quantize_affine_w4_weight(weight, group_size=self.group_size,
                                            convrot_groupsize=self.convrot_groupsize)
        return [q, s, z], {}


QuantFormat = ConvrotW4A4 | AsymW4A8 | Int8Tensorwise | AwqW4A16 | AffineW4A8
FORMAT_NAMES = (ConvrotW4A4.name, AsymW4A8.name, Int8Tensorwise.name, AwqW4A16.name, AffineW4A8.name)


def format_from_config(conf: dict) -> QuantFormat:
    """Inverse of ``layer_config()``: the format instance a layer's metadata entry describes."""
    fmt = conf.get("format")
    params = conf.get("params", {}) if isinstance(conf.get("params", {}), dict) else {}
    get = lambda k, d: conf.get(k, params.get(k, d))  # noqa: E731
    if fmt == ConvrotW4A4.name:
        return ConvrotW4A4(convrot_groupsize=int(get("convrot_groupsize", 256)))
    if fmt == AsymW4A8.name:
        return AsymW4A8(group_size=int(get("group_size", 16)), convrot_groupsize=int(get("convrot_groupsize", 256)))
    if fmt == Int8Tensorwise.name:
        conv = bool(get("convrot", False))
        return Int8Tensorwise(convrot=conv, convrot_groupsize=int(get("convrot_groupsize", 256)))
    if fmt == AwqW4A16.name:
        return AwqW4A16(group_size=int(get("group_size", 64)))
    if fmt == AffineW4A8.name:
        return AffineW4A8(group_size=int(get("group_size", 128)), convrot_groupsize=int(get("convrot_groupsize", 0)))
    raise ValueError(f"unknown quantization format {fmt!r}")


def layer_configs(formats: dict) -> dict:
    """{weight name: format} -> ``_quantization_metadata["layers"]`` ({layer: config})."""
    return {_base(name): fmt.layer_config() for name, fmt in formats.items()}


def quant_metadata(metadata: dict, layers: dict, quantization: str, extra: dict | None = None) -> dict:
    """The output ``__metadata__``: the source's keys, then ``_quantization_metadata``, ``quantization``, extras."""
    out = dict(metadata)
    out["_quantization_metadata"] = json.dumps({"format_version": FORMAT_VERSION, "layers": layers},
                                               separators=(",", ":"))
    out["quantization"] = quantization
    if extra:
        out.update(extra)
    return out
