"""MMDiT denoise step on the W4A8 affine path: the kernel path against the torch fp32 reference of the same step.

The reference replaces every linear by an fp32 product of its dequantized weight (W = (q - 8) * scale + zeros,
rotated basis) and the dequantized activation codes, and runs the rest of the block (norms, rotary embedding,
attention, GELU, modulation) as torch ops; the kernel path runs the fused glue kernels (``fused_glue``) or the
same torch ops.  Each linear's bf16 output agrees to within bf16 rounding, so after a few
blocks the step outputs agree to a relative L2 error well under 1e-2 (the bound written below).
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mmdit():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from comfy_quant_bench_b200 import mmdit as mm
    return mm


@pytest.mark.parametrize("quantize_modulation,fused_glue", [(True, True), (False, True), (True, False)])
def test_mmdit_step_matches_reference(mmdit, quantize_modulation, fused_glue):
    cfg = mmdit.MMDiTConfig(blocks=2, hidden=512, heads=4, mlp=1024, img_tokens=300, txt_tokens=40,
                            quantize_modulation=quantize_modulation, fused_glue=fused_glue)
    model = mmdit.MMDiT(cfg, device="cuda", seed=3)
    img, txt, temb = model.inputs(seed=4)
    out_img, out_txt = model.step(img, txt, temb)
    ref_img, ref_txt = model.step(img, txt, temb, reference=True)
    torch.cuda.synchronize()
    assert torch.isfinite(out_img.float()).all() and torch.isfinite(out_txt.float()).all()
    assert mmdit.rel_l2(out_img, ref_img) <= 1e-2
    assert mmdit.rel_l2(out_txt, ref_txt) <= 1e-2
    from comfy_quant_bench_b200 import _lib
    assert _lib.take_device_status() == (0, 0)


def test_mmdit_step_is_deterministic_and_graph_capturable(mmdit):
    cfg = mmdit.MMDiTConfig(blocks=1, hidden=512, heads=4, mlp=1024, img_tokens=256, txt_tokens=32)
    model = mmdit.MMDiT(cfg, device="cuda", seed=5)
    img, txt, temb = model.inputs(seed=6)
    eager = model.step(img, txt, temb)[0].clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        model.step(img, txt, temb)   # warm the allocator on the capture stream
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        graphed = model.step(img, txt, temb)[0]
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(graphed, eager)
    assert torch.equal(model.step(img, txt, temb)[0], eager)


def test_mmdit_layout_and_modulation_forms_are_bit_identical(mmdit):
    """The joined modulation product (one activation kernel and one weight stream for every block's modulation
    linears), the token-major attention layout and the text stream's work on a second CUDA stream change only how
    the work is launched: with the text linears' K split fixed, the step output equals the per-stream, head-major,
    one-stream form bit for bit."""
    from dataclasses import replace
    for text_split_k in (False, True):
        _check_launch_forms(mmdit, replace, text_split_k)


def _check_launch_forms(mmdit, replace, text_split_k):
    cfg = mmdit.MMDiTConfig(blocks=3, hidden=512, heads=4, mlp=1024, img_tokens=300, txt_tokens=40,
                            text_split_k=text_split_k)
    model = mmdit.MMDiT(cfg, device="cuda", seed=9)
    img, txt, temb = model.inputs(seed=10)
    base = model.step(img, txt, temb)
    outs = []
    assert cfg.text_side_stream
    for batched, token_major, side in ((False, True, True), (True, True, False), (True, False, False),
                                       (False, False, False)):
        model.cfg = replace(cfg, batched_modulation=batched, token_major_qkv=token_major, text_side_stream=side)
        outs.append(model.step(img, txt, temb))
    model.cfg = cfg
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o[0], base[0]) and torch.equal(o[1], base[1])
    from comfy_quant_bench_b200 import _lib
    assert _lib.take_device_status() == (0, 0)


def test_wan_step_matches_reference():
    """Wan-like block stack on the mixed plan (W4A4 ConvRot g64 and W8A8 linears) against the fp32-linear
    reference of the same step (the same rel-L2 bound as the MMDiT step)."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from comfy_quant_bench_b200 import wan, _lib
    cfg = wan.WanConfig(blocks=2, hidden=512, heads=4, ffn=1536, frames=3, height=5, width=20, ctx_tokens=64)
    model = wan.WanDiT(cfg, device="cuda", seed=7)
    assert model.plan()["w4a4"] == round(0.35 * 20) and model.plan()["w8a8"] == 20 - round(0.35 * 20)
    x, ctx = model.inputs(seed=8)
    out = model.step(x, ctx)
    ref = model.step(x, ctx, reference=True)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    assert wan.rel_l2(out, ref) <= 1e-2
    assert max(model.block_errors(x, ctx)) <= 1e-2
    assert _lib.take_device_status() == (0, 0)
