"""Full-depth model steps at the BASELINE configurations against the fp32-linear reference.

The reference runs the same step with every linear as a torch fp32 product of the dequantized weight and the
dequantized activation codes; the glue is the same torch code.  Two checks per model:

* teacher-forced, per block: each block run by the kernel path and by the reference on the kernel path's own input
  to that block.  This isolates one block's linears (the kernels under test) from the drift of earlier blocks.
* step-level: the whole step against the whole reference step.  A step is a long chain of blocks that requantize
  their activations (int8 for W4A8; int4 for the Wan plan's W4A4 linears), so a one-rounding difference in a block's
  input can move a quantization code and grow through later blocks.  The bound is therefore calibrated in the same
  run: the step-level difference must stay within twice the difference the kernel path itself shows when 1 % of its
  input elements move by one bf16 ulp - a perturbation of the size of one rounding.  A kernel error beyond bf16
  rounding would show up as a step difference far above that drift.

Measured on a B200 (60-block MMDiT: per block <= 0.012, step 0.027, one-ulp drift 0.027; 30-block Wan: per block
<= 0.022, step 0.147, one-ulp drift 0.149, and the same drift on the reference path itself).
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ulp_perturb(x: torch.Tensor, frac: float = 0.01, seed: int = 123) -> torch.Tensor:
    """x with one bf16 ulp added to a seeded random `frac` of its elements."""
    g = torch.Generator(device=x.device).manual_seed(seed)
    mask = torch.rand(x.shape, generator=g, device=x.device) < frac
    bits = x.view(torch.int16)
    return torch.where(mask, bits + 1, bits).view(torch.bfloat16)


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda")


def test_mmdit_60_blocks_at_the_baseline_config(cuda):
    from comfy_quant_bench_b200 import mmdit as mm, _lib
    model = mm.MMDiT(mm.MMDiTConfig(), device="cuda", seed=0)   # 60 blocks, hidden 3072, 4096 + 256 tokens
    img, txt, temb = model.inputs(seed=1)
    out_img, out_txt = model.step(img, txt, temb)
    ref_img, ref_txt = model.step(img, txt, temb, reference=True)
    drift = mm.rel_l2(model.step(_ulp_perturb(img), txt, temb)[0], out_img)
    errs = model.block_errors(img, txt, temb)
    torch.cuda.synchronize()
    assert torch.isfinite(out_img.float()).all() and torch.isfinite(out_txt.float()).all()
    assert len(errs) == 60 and max(errs) <= 2e-2, errs
    step_img, step_txt = mm.rel_l2(out_img, ref_img), mm.rel_l2(out_txt, ref_txt)
    assert step_img <= 2 * drift and step_txt <= 2 * drift, (step_img, step_txt, drift)
    assert step_img <= 5e-2 and step_txt <= 5e-2
    assert _lib.take_device_status() == (0, 0)
    del model
    torch.cuda.empty_cache()


def test_wan_30_blocks_at_the_baseline_config(cuda):
    from comfy_quant_bench_b200 import wan, _lib
    model = wan.WanDiT(wan.WanConfig(), device="cuda", seed=0)   # 30 blocks, 27,280 tokens, 35 % W4A4 / 65 % W8A8
    x, ctx = model.inputs(seed=1)
    out = model.step(x, ctx)
    ref = model.step(x, ctx, reference=True)
    drift = wan.rel_l2(model.step(_ulp_perturb(x), ctx), out)
    drift_ref = wan.rel_l2(model.step(_ulp_perturb(x), ctx, reference=True), ref)
    errs = model.block_errors(x, ctx)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    # the blocks whose linears requantize to int4 (Hadamard g64) move most; one rounding there is 1/7 of a token's range
    assert len(errs) == 30 and max(errs) <= 3e-2, errs
    step = wan.rel_l2(out, ref)
    # the drift is a property of the model, not of the kernels: the reference path drifts by the same amount
    assert 0.5 * drift_ref <= drift <= 2 * drift_ref, (drift, drift_ref)
    assert step <= 2 * drift, (step, drift)
    assert _lib.take_device_status() == (0, 0)
    del model
    torch.cuda.empty_cache()
