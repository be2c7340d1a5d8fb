"""Host-side tests of the ComfyUI boundary (no GPU): layout registration, QUANT_ALGOS readers, state-dict
loading, linear_input_act routing and the opaque custom ops' fake implementations.

Modelled on the reference's dispatch tests (``patches/tests/test_comfyui_fase4_dispatch.py:60-86``: a Mock
spy on the kernel entry point) and its format-reader test (``patches/comfyui_awq_w4a16_format.patch``,
``test_format_reader_from_quant_algos_builds_params``).
"""
import json
import types
import unittest.mock

import numpy as np
import pytest
import torch

from comfy_quant_bench_b200 import comfy_ops, layout as L
from oracle import ref


@pytest.fixture(autouse=True)
def registered():
    L.register(target=None)
    yield


def _affine_state_dict(n=16, k=256, group=128, seed=0):
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 16, size=(n, k))
    qweight = torch.from_numpy(ref.pack_int4(codes))
    scale = (torch.rand(k // group, n, generator=torch.Generator().manual_seed(seed)) * 0.01 + 0.001).to(torch.bfloat16)
    zeros = (torch.randn(k // group, n, generator=torch.Generator().manual_seed(seed + 1)) * 0.01).to(torch.bfloat16)
    bias = torch.randn(n, dtype=torch.bfloat16)
    conf = {"format": "affine_w4a8", "group_size": group}
    sd = {"layer.weight": qweight, "layer.bias": bias, "layer.weight_scale": scale, "layer.weight_zeros": zeros,
          "layer.comfy_quant": torch.tensor(list(json.dumps(conf).encode()), dtype=torch.uint8)}
    return sd, codes, scale, zeros, bias


def test_register_into_a_comfyui_like_module():
    fake = types.SimpleNamespace(QUANT_ALGOS={}, layouts={})
    fake.register_layout_class = lambda name, cls: fake.layouts.__setitem__(name, cls)
    fake.__name__ = "comfy.quant_ops"
    assert L.register(target=fake) == "comfy.quant_ops"
    assert set(fake.QUANT_ALGOS) == {"convrot_w4a4", "affine_w4a8", "int8_tensorwise"}
    for algo in fake.QUANT_ALGOS.values():
        assert set(algo) == {"storage_t", "parameters", "comfy_tensor_layout", "quantize_input",
                             "params_from_state_dict"}
        assert algo["comfy_tensor_layout"] in fake.layouts


def test_state_dict_loads_through_params_reader_and_dequantizes():
    sd, codes, scale, zeros, bias = _affine_state_dict()
    model = torch.nn.Module()
    model.layer = comfy_ops.mixed_precision_ops({}).Linear(256, 16, device="cpu", dtype=torch.bfloat16)
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert missing == [] and unexpected == []
    w = model.layer.weight
    assert isinstance(w, L.QuantizedWeight) and w.layout == "B200AffineW4A8Layout"
    assert w.params.group_size == 128
    want = ref.dequant_affine(codes, scale.float().numpy(), zeros.float().numpy())
    got = w.dequantize().float().numpy()
    assert np.allclose(got, ref.bf16_round(want.astype(np.float32)), rtol=0, atol=0)
    saved = model.layer.quantized_state_dict("layer.")
    assert json.loads(bytes(saved["layer.comfy_quant"].tolist()))["format"] == "affine_w4a8"
    assert torch.equal(saved["layer.weight_zeros"], zeros)


def test_reader_hook_is_called_once_per_layer():
    sd, *_ = _affine_state_dict()
    calls = []
    orig = L.QUANT_ALGOS["affine_w4a8"]["params_from_state_dict"]

    def reader(layer_name, module, qdata, pop_scale, layer_conf):
        calls.append((layer_name, tuple(qdata.shape), layer_conf["format"]))
        return orig(layer_name, module, qdata, pop_scale, layer_conf)

    with unittest.mock.patch.dict(L.QUANT_ALGOS["affine_w4a8"], {"params_from_state_dict": reader}):
        model = torch.nn.Module()
        model.layer = comfy_ops.Linear(256, 16, dtype=torch.bfloat16)
        model.load_state_dict(sd, strict=False)
    assert calls == [("layer", (16, 128), "affine_w4a8")]


def test_missing_zeros_raise_like_the_reference_reader():
    sd, *_ = _affine_state_dict()
    del sd["layer.weight_zeros"]
    model = torch.nn.Module()
    model.layer = comfy_ops.Linear(256, 16, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="Missing affine W4A8 scale/zeros"):
        model.load_state_dict(sd, strict=False)


def _loaded_layer():
    sd, *_ = _affine_state_dict(n=16, k=256)
    lin = comfy_ops.Linear(256, 16, dtype=torch.bfloat16)
    m = torch.nn.Module()
    m.layer = lin
    m.load_state_dict(sd, strict=False)
    return lin


def test_linear_input_act_folds_swiglu_into_the_quantized_call():
    lin = _loaded_layer()
    x = torch.randn(4, 512, dtype=torch.bfloat16)
    spy = unittest.mock.Mock(return_value=torch.zeros(4, 16, dtype=torch.bfloat16))
    with unittest.mock.patch.object(L.B200AffineW4A8Layout, "linear", spy):
        out = comfy_ops.linear_input_act(lin, x, "swiglu")
    assert spy.call_args.args[0] is x                       # the [gate | up] pair, not the activation
    assert spy.call_args.args[4] == "swiglu"
    assert out.shape == (4, 16)


def test_linear_input_act_applies_other_acts_eagerly_then_residual():
    lin = _loaded_layer()
    x = torch.randn(4, 256, dtype=torch.bfloat16)
    seen = {}

    def fake_linear(xx, qdata, params, bias=None, input_act=None):
        seen["x"], seen["act"] = xx, input_act
        return torch.ones(4, 16, dtype=torch.bfloat16)

    res = torch.full((4, 16), 2.0, dtype=torch.bfloat16)
    with unittest.mock.patch.object(L.B200AffineW4A8Layout, "linear", side_effect=fake_linear):
        out = comfy_ops.linear_input_act(lin, x, "gelu_tanh", residual=res, residual_scale=torch.tensor(0.5))
    assert seen["act"] is None
    assert torch.equal(seen["x"], torch.nn.functional.gelu(x, approximate="tanh"))
    assert torch.allclose(out.float(), torch.full((4, 16), 2.5))


def test_lora_patch_takes_the_dequantized_weight():
    lin = _loaded_layer()
    lin.weight_function.append(lambda w: w * 0)
    x = torch.randn(3, 256, dtype=torch.bfloat16)
    out = lin(x)
    assert torch.allclose(out.float(), lin.bias.float().expand(3, 16))
    assert comfy_ops._fused_input_act(lin, torch.randn(3, 512), "swiglu") is None


def test_custom_op_fake_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode
    from comfy_quant_bench_b200 import custom_op  # noqa: F401
    with FakeTensorMode():
        x = torch.empty(2, 7, 256, dtype=torch.bfloat16)
        q = torch.empty(48, 128, dtype=torch.int8)
        y = torch.ops.comfy_quant_b200.convrot_w4a4_linear(x, q, torch.empty(48), None, 256, 64, "int4")
        assert y.shape == (2, 7, 48)
        s = torch.empty(2, 48, dtype=torch.bfloat16)
        y2 = torch.ops.comfy_quant_b200.w4a8_affine_linear(x, q, s, s, None, 128, 0)
        assert y2.shape == (2, 7, 48)
        y3 = torch.ops.comfy_quant_b200.int8_linear(x, torch.empty(48, 256, dtype=torch.int8), torch.empty(48, 1),
                                                     None, True, 256)
        assert y3.shape == (2, 7, 48)
