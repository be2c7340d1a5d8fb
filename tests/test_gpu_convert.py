"""Checkpoint conversion with the weight kernel on the GPU, then loading it through the ComfyUI ops surface.

The converted tensors must equal the weight kernel's output for the same source weight (bit-exact), unselected
tensors must be copied byte for byte, and a ``comfy_ops.Linear`` loaded from the converted state dict with the
layer's ``_quantization_metadata`` entry must compute exactly what the library linear computes on the same weight.
"""
import json

import pytest
import torch
from safetensors import safe_open
from safetensors.torch import save_file

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fmt_name,extra", [("affine_w4a8", ["--convrot-groupsize", "256"]), ("convrot_w4a4", []),
                                            ("int8_tensorwise", ["--convrot-groupsize", "256"])])
def test_convert_and_load(tmp_path, fmt_name, extra):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from comfy_quant_bench_b200 import convert as C, formats as F, comfy_ops, _lib
    g = torch.Generator().manual_seed(5)
    w = (torch.randn(384, 1024, generator=g) * 0.02).to(torch.bfloat16)
    bias = (torch.randn(384, generator=g) * 0.01).to(torch.bfloat16)
    src = tmp_path / "m.safetensors"
    save_file({"layer.weight": w, "layer.bias": bias, "other": torch.arange(10, dtype=torch.float32)}, str(src))
    out = tmp_path / "q.safetensors"
    assert C.main(["--input", str(src), "--output", str(out), "--format", fmt_name, *extra]) == 0

    with safe_open(str(out), "pt") as f:
        layers = json.loads(f.metadata()["_quantization_metadata"])["layers"]
        sd = {k: f.get_tensor(k) for k in f.keys()}
    fmt = F.format_from_config(layers["layer"])
    want = fmt.quantize(w.cuda().float())[0]
    for (key, _, _), t in zip(fmt.tensors("layer.weight", [384, 1024]), want):
        assert torch.equal(sd[key], t.cpu()), key
    assert torch.equal(sd["other"], torch.arange(10, dtype=torch.float32))
    assert torch.equal(sd["layer.bias"], bias)

    lin = comfy_ops.Linear(1024, 384, bias=True, device="cuda", dtype=torch.bfloat16)
    state = {k.removeprefix("layer."): v.cuda() for k, v in sd.items() if k.startswith("layer.")}
    lin._load_from_state_dict(state, "", {"comfy_quant": layers["layer"]}, True, [], [], [])
    x = torch.randn(70, 1024, device="cuda").to(torch.bfloat16)
    y = lin(x)
    from comfy_quant_bench_b200 import ops
    q = [t.cuda() for t in want]
    b = bias.cuda()
    if fmt_name == "affine_w4a8":
        ref = ops.w4a8_affine_linear(x, q[0], q[1], q[2], b, 128, 256)
    elif fmt_name == "convrot_w4a4":
        ref = ops.convrot_w4a4_linear(x, q[0], q[1], b, convrot_groupsize=256)
    else:
        ref = ops.int8_linear(x, q[0], q[1], b, convrot=True, convrot_groupsize=256)
    torch.cuda.synchronize()
    assert torch.equal(y, ref)
    assert json.loads((tmp_path / "q.quant.json").read_text())["quantized_tensors"] == 1
    assert _lib.take_device_status() == (0, 0)
