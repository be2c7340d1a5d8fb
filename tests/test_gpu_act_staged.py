"""GPU: the two kernel forms of the per-token activation kernels give the same bits.

The staged form (persistent CTAs, each token pair's rows brought into shared memory by bulk copies while the CTA
works on its previous pair) runs the same per-pair arithmetic as the one-pair-per-CTA form, so codes, scales and
group sums must agree bit for bit, in every per-token mode, for any number of pairs per CTA, with padding rows,
non-finite tokens, the layer-norm prologue and the two-phase (split-column) scales.  The oracle parity of the
default (staged) form is covered by tests/test_gpu_parity.py.
"""
import numpy as np
import pytest
import torch

from oracle import ref

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from comfy_quant_bench_b200 import _lib, ops
    _lib.load()
    yield _lib, ops
    _lib.set_act_variant(_lib.CQ_ACT_AUTO)


def bf16_dev(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def both_forms(lib, fn):
    """fn() under the one-pair-per-CTA form, then under the staged form; each result as a tuple of host arrays."""
    out = []
    for form in (lib.CQ_ACT_WAVES, lib.CQ_ACT_STAGED):
        lib.set_act_variant(form)
        res = fn()
        torch.cuda.synchronize()
        out.append(tuple(None if t is None else t.detach().cpu().contiguous().view(torch.uint8).numpy().copy()
                         for t in res))
    lib.set_act_variant(lib.CQ_ACT_AUTO)
    assert lib.take_device_status() == (0, 0)
    return out


def assert_same(a, b):
    assert len(a) == len(b)
    for i, (x, y) in enumerate(zip(a, b)):
        if x is None:
            assert y is None
        else:
            assert np.array_equal(x, y), f"output {i} differs between the kernel forms"


@pytest.mark.parametrize("m,k", [(1, 256), (37, 768), (1001, 3072), (4096, 3072), (20000, 3072), (3, 12288),
                                 (515, 12288)])
@pytest.mark.parametrize("rot", [0, 16, 64, 256])
def test_int8_codes_scales_group_sums(env, m, k, rot):
    lib, ops = env
    x = bf16_dev(ref.synth_activations(m, k, seed=m + k + rot))
    w, s = both_forms(lib, lambda: ops.rotquant(x, rot, lib.CQ_ACT_INT8_ROW, group_sums=True, kperm=True))
    assert_same(w, s)


@pytest.mark.parametrize("m,m_pad", [(5, 16), (6, 7), (1, 2), (2999, 3001)])
def test_padding_rows(env, m, m_pad):
    lib, ops = env
    x = bf16_dev(ref.synth_activations(m, 3072, seed=3 + m))
    w, s = both_forms(lib, lambda: ops.rotquant(x, 256, lib.CQ_ACT_INT8_ROW, m_pad=m_pad, group_sums=True, kperm=True))
    assert_same(w, s)


@pytest.mark.parametrize("int4_as_int8", [False, True])
@pytest.mark.parametrize("m,k,rot", [(19, 1024, 256), (4096, 3072, 256), (77, 3072, 64), (8, 12288, 16)])
def test_int4_rowwise(env, int4_as_int8, m, k, rot):
    lib, ops = env
    x = bf16_dev(ref.synth_activations(m, k, seed=7 + k + m))
    w, s = both_forms(lib, lambda: ops.rotquant(x, rot, lib.CQ_ACT_INT4_ROW, int4_as_int8=int4_as_int8))
    assert_same(w, s)


def test_nonfinite_tokens(env):
    lib, ops = env
    x = ref.synth_activations(9, 3072, seed=5)
    x[1, 600] = np.uint16(0x7FC0)   # NaN
    x[2, 77] = np.uint16(0x7F80)    # +inf
    x[7, 3000] = np.uint16(0xFF80)  # -inf
    xd = bf16_dev(x)
    w, s = both_forms(lib, lambda: ops.rotquant(xd, 256, lib.CQ_ACT_INT8_ROW, group_sums=True))
    assert_same(w, s)


def test_layer_norm_prologue(env):
    lib, ops = env
    m, k = 333, 3072
    x = bf16_dev(ref.synth_activations(m, k, seed=21))
    g = torch.Generator(device="cpu").manual_seed(4)
    shift = (torch.randn(k, generator=g) * 0.1).to(torch.bfloat16).cuda()
    scale = (torch.randn(k, generator=g) * 0.1).to(torch.bfloat16).cuda()
    w, s = both_forms(lib, lambda: ops.rotquant_lnmod(x, 256, shift, scale, group_sums=True, kperm=True))
    assert_same(w, s)


def test_split_column_scales(env):
    lib, ops = env
    m, k = 257, 1536
    x = bf16_dev(ref.synth_activations(m, k, seed=13))
    w, s = both_forms(lib, lambda: (ops.rotquant_absmax(x, 256),))
    assert_same(w, s)
    amax = ops.rotquant_absmax(x, 256)
    w, s = both_forms(lib, lambda: ops.rotquant_scaled(x, 256, amax, group_sums=True, kperm=True))
    assert_same(w, s)


def test_unaligned_rows_are_refused_before_any_launch(env):
    """Rows that do not start on a 16-byte boundary are refused by the C ABI (CQ_ERR_ALIGN) under either form, so
    neither the 16-byte vector loads nor the bulk copies ever see them."""
    lib, ops = env
    from comfy_quant_bench_b200._lib import CQShapeError
    m, k = 64, 3072
    base = bf16_dev(ref.synth_activations(1, m * k + 4, seed=2))[0]
    x = base[4:].view(m, k)            # 8 bytes past an aligned allocation
    assert x.data_ptr() % 16 == 8
    for form in (lib.CQ_ACT_WAVES, lib.CQ_ACT_STAGED):
        lib.set_act_variant(form)
        with pytest.raises(CQShapeError):
            ops.rotquant(x, 256, lib.CQ_ACT_INT8_ROW)
    lib.set_act_variant(lib.CQ_ACT_AUTO)


def test_variant_switch_rejects_unknown_values(env):
    lib, _ = env
    from comfy_quant_bench_b200._lib import CQShapeError
    with pytest.raises(CQShapeError):
        lib.set_act_variant(7)
