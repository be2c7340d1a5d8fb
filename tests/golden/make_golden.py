"""Generate the golden fixtures that pin ``oracle/ref.py`` to comfy-quant-bench's own code.

Run once in a container where the reference checkout is mounted (it is never read at test time):

    python tests/golden/make_golden.py /path/to/comfy-quant-bench

Every fixture is produced by calling the reference's OWN Python functions on seeded inputs:

* ``experiments/qwen21-kernel/kernels/g64_quant_test.py``: ``bf16_up``, ``unpack`` and ``ref`` (rotation by
  the Hadamard matrix, per-group absmax, scale rounded up to bf16, int4 codes), for G = 64 and 128,
  with and without the SwiGLU prologue.  ``ref`` imports ``_build_hadamard`` from comfy-kitchen, which the
  reference does not vendor; it is served here by a stub module returning kron^4 of the regular H4 divided
  by 16, the construction ``g64_quant.cu:2-7`` states equals ``_build_hadamard(256)``.
* ``tools/activation_balance.py``: ``quantize_rowwise`` (per-row int4 / int8, the shipped per-token scale).
* ``experiments/qwen21-kernel/kernels/g64_bench6.py``: ``pack`` and ``ref`` (GEMM reference, scale
  policies 0 = row x row and 4 = g128 x g128).
* ``experiments/qwen21-kernel/node/__init__.py``: ``_pack`` and ``_quant_weight`` (ConvRot weight
  quantization, pol 0 = per row, pol 4 = per group 128 with bf16-up scales); ``comfy.ops`` / ``comfy.sd``
  are stubbed (the module only patches them when G64_POL is set).
* ``patches/tests/test_comfy_kitchen_awq.py``: ``awq_inputs`` and ``old_cuda_torch_chain`` (the affine
  ``(q - 8) * scale + zeros`` dequantization), with comfy-kitchen stubbed out.
* ``tools/_formats.py``: the tensor names, dtypes and shapes each format writes, its layer config and the
  quantization metadata.

Outputs: ``tests/golden/ref_golden.npz`` and ``tests/golden/formats_golden.json``.
"""
from __future__ import annotations

import importlib.util
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _h4r_kron(n: int, dtype=torch.float32, device="cpu") -> torch.Tensor:
    h4 = 0.5 * torch.tensor([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=torch.float64)
    h = torch.ones(1, 1, dtype=torch.float64)
    while h.shape[0] < n:
        h = torch.kron(h, h4)
    return h.to(device=device, dtype=dtype)


def _install_stubs() -> None:
    """Minimal stand-ins for the third-party modules the reference files import at top level."""
    ck = types.ModuleType("comfy_kitchen")
    backends = types.ModuleType("comfy_kitchen.backends")
    eager = types.ModuleType("comfy_kitchen.backends.eager")
    convrot = types.ModuleType("comfy_kitchen.backends.eager.convrot_w4a4")
    convrot._build_hadamard = lambda n, device="cpu", dtype=torch.float32: _h4r_kron(n, dtype, device)
    awq = types.ModuleType("comfy_kitchen.backends.eager.awq")
    registry = types.ModuleType("comfy_kitchen.registry")
    registry.registry = object()
    eager.convrot_w4a4 = convrot
    eager.awq = awq
    backends.eager = eager
    ck.backends = backends
    ck.registry = registry
    comfy = types.ModuleType("comfy")
    comfy.ops = types.ModuleType("comfy.ops")
    comfy.sd = types.ModuleType("comfy.sd")
    for name, mod in {"comfy_kitchen": ck, "comfy_kitchen.backends": backends,
                      "comfy_kitchen.backends.eager": eager,
                      "comfy_kitchen.backends.eager.convrot_w4a4": convrot,
                      "comfy_kitchen.backends.eager.awq": awq, "comfy_kitchen.registry": registry,
                      "comfy": comfy, "comfy.ops": comfy.ops, "comfy.sd": comfy.sd}.items():
        sys.modules.setdefault(name, mod)


def _load(name: str, path: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16).copy()


def main(root: str) -> None:
    sys.dont_write_bytecode = True
    os.environ.pop("G64_POL", None)
    _install_stubs()
    sys.path.insert(0, os.path.join(root, "tools"))
    kern = os.path.join(root, "experiments", "qwen21-kernel", "kernels")
    qt = _load("g64_quant_test", os.path.join(kern, "g64_quant_test.py"))
    gb = _load("g64_bench6", os.path.join(kern, "g64_bench6.py"))
    ab = _load("activation_balance", os.path.join(root, "tools", "activation_balance.py"))
    node = _load("g64_node", os.path.join(root, "experiments", "qwen21-kernel", "node", "__init__.py"))
    awqt = _load("test_comfy_kitchen_awq", os.path.join(root, "patches", "tests", "test_comfy_kitchen_awq.py"))
    _load("_conversion", os.path.join(root, "tools", "_conversion.py"))
    fm = _load("_formats", os.path.join(root, "tools", "_formats.py"))

    out: dict[str, np.ndarray] = {}

    # bf16_up on a spread of magnitudes, exact bf16 values included
    gen = torch.Generator().manual_seed(0)
    v = torch.cat([torch.rand(4000, generator=gen) * 10 ** torch.randint(-8, 6, (4000,), generator=gen),
                   torch.tensor([1.0, 0.5, 3.0, 1.0078125, 2 ** -20])]).float()
    out["bf16_up_in"] = v.numpy()
    out["bf16_up_out"] = qt.bf16_up(v).numpy()

    # unpack of every byte value
    q = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(torch.int8).reshape(2, 128)
    out["unpack_in"] = q.numpy()
    out["unpack_out"] = qt.unpack(q, 256).numpy()

    # activation quantizer reference (rotation + per-group bf16-up int4), g64_quant_test.py:54-70
    for (m, k, swiglu, seed) in ((37, 1024, False, 1), (19, 512, True, 2)):
        gen = torch.Generator().manual_seed(seed)
        cols = 2 * k if swiglu else k
        x = (torch.randn(m, cols, generator=gen) * (1 + 8 * (torch.rand(1, cols, generator=gen) > 0.99))).to(torch.bfloat16)
        tag = f"act_m{m}_k{k}_{'swiglu' if swiglu else 'plain'}"
        out[f"{tag}_x"] = _bf16_bits(x)
        for g in (64, 128):
            qr, sr, tr = qt.ref(x, g, swiglu)
            out[f"{tag}_g{g}_q"] = qr.numpy().astype(np.int16)
            out[f"{tag}_g{g}_s"] = sr.numpy()
            out[f"{tag}_g{g}_t"] = tr.numpy()

    # per-row symmetric quantization of a rotated activation (tools/activation_balance.py:65-71)
    gen = torch.Generator().manual_seed(3)
    xr = torch.randn(64, 768, generator=gen) * (1 + 19 * (torch.rand(1, 768, generator=gen) > 0.99))
    out["rowwise_in"] = xr.numpy()
    for lim in (7, 127):
        codes, _ = ab.quantize_rowwise(xr, lim, None)
        out[f"rowwise_q{lim}"] = codes.numpy().astype(np.int16)
        out[f"rowwise_s{lim}"] = (xr.abs().amax(dim=-1) / lim).clamp(min=1e-10).numpy()

    # GEMM reference with scale policies 0 and 4 (g64_bench6.py:50-68)
    gen = torch.Generator().manual_seed(4)
    M, N, K = 64, 48, 512
    a = torch.randint(-7, 8, (M, K), generator=gen, dtype=torch.int32)
    b = torch.randint(-7, 8, (N, K), generator=gen, dtype=torch.int32)
    bias = (torch.randn(N, generator=gen) * 0.1).to(torch.bfloat16)
    out["gemm_a"] = a.numpy().astype(np.int8)
    out["gemm_b"] = b.numpy().astype(np.int8)
    out["gemm_bias"] = _bf16_bits(bias)
    out["gemm_a_packed"] = gb.pack(a).numpy()
    e0 = {"sa": torch.rand(M, generator=gen) * 0.01 + 0.005, "sb": torch.rand(N, generator=gen) * 0.01 + 0.005}
    out["gemm_p0_sa"], out["gemm_p0_sb"] = e0["sa"].numpy(), e0["sb"].numpy()
    out["gemm_p0_out"] = gb.ref(a, b, e0, bias, 0, slice(0, M)).numpy()
    e4 = {"sa": torch.rand(K // 128, M, generator=gen) * 0.01 + 0.005,
          "sb": torch.rand(K // 128, N, generator=gen) * 0.01 + 0.005}
    out["gemm_p4_sa"], out["gemm_p4_sb"] = e4["sa"].numpy(), e4["sb"].numpy()
    out["gemm_p4_out"] = gb.ref(a, b, e4, bias, 4, slice(0, M)).numpy()

    # ConvRot weight quantization (node/__init__.py:89-126), pol 0 (per row) and pol 4 (g128 bf16-up)
    gen = torch.Generator().manual_seed(5)
    w = torch.randn(40, 768, generator=gen) * 0.02
    out["wq_in"] = w.numpy()
    h = _h4r_kron(256)
    for pol in (0, 4):
        res = node._quant_weight(w, pol, h)
        out[f"wq_p{pol}_packed"] = res["g64_q"].numpy()
        out[f"wq_p{pol}_scale"] = res["g64_sb"].numpy()

    # affine dequantization (patches/tests/test_comfy_kitchen_awq.py:21-37)
    codes, qweight, wscales, wzeros = awqt.awq_inputs(n=48, k=256, group_size=64, dtype=torch.float32, seed=0)
    out["awq_codes"] = codes.numpy().astype(np.int16)
    out["awq_qweight"] = qweight.numpy()
    out["awq_scale"] = wscales.numpy()
    out["awq_zeros"] = wzeros.numpy()
    out["awq_deq_f32"] = awqt.old_cuda_torch_chain(qweight, wscales, wzeros, 64).numpy()
    _, qb, sb, zb = awqt.awq_inputs(n=48, k=256, group_size=64, dtype=torch.bfloat16, seed=0)
    out["awq_scale_bf16"] = _bf16_bits(sb)
    out["awq_zeros_bf16"] = _bf16_bits(zb)
    out["awq_deq_bf16"] = _bf16_bits(awqt.old_cuda_torch_chain(qb, sb, zb, 64))

    np.savez_compressed(os.path.join(HERE, "ref_golden.npz"), **out)

    formats = {}
    for fmt in (fm.ConvrotW4A4(), fm.ConvrotW4A4(convrot_groupsize=64), fm.AsymW4A8(),
                fm.AsymW4A8(codebook=False), fm.Int8Tensorwise(), fm.Int8Tensorwise(convrot=False),
                fm.AwqW4A16(), fm.AwqW4A16(group_size=128)):
        key = repr(fmt)
        formats[key] = {
            "layer_config": fmt.layer_config(),
            "accepts": {str(s): fmt.accepts(s) for s in ([3072, 3072], [12288, 3072], [64, 200], [64, 96])},
            "tensors": fmt.tensors("blocks.0.mlp.fc1.weight", [12288, 3072]),
        }
    formats["__metadata__"] = fm.quant_metadata({"a": "b"}, {"blocks.0.mlp.fc1": fm.ConvrotW4A4().layer_config()},
                                                "convrot_w4a4", {"x": "y"})
    with open(os.path.join(HERE, "formats_golden.json"), "w", encoding="utf-8") as f:
        json.dump(formats, f, indent=1, sort_keys=True)
    print("wrote", sorted(out)[:5], "...", len(out), "arrays")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("CQB_REFERENCE_ROOT", ""))
