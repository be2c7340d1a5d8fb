"""Properties of the CPU oracle that the GPU parity tests lean on, checked on CPU at small sizes.

* The affine linear in integer form (group partial sums scaled per group, plus the zero-point term) equals the
  reference's dequantize-and-matmul path (``patches/tests/test_comfyui_fase4_dispatch.py:98``) on the same codes.
* The split group sums (the affine GEMM's zero-point operand) are exact in bf16 and add back to the group sums.
* The rotation is the block-diagonal Hadamard product ``x.reshape(M, K/g, g) @ H`` (``g64_quant_test.py:64``) and
  preserves each token's norm.
* The row/column linear equals the product of dequantized operands.
"""
import numpy as np
import pytest

from oracle import ref


@pytest.mark.parametrize("m,n,k,rot", [(5, 24, 256, 256), (17, 40, 512, 64), (3, 16, 384, 0)])
def test_affine_integer_form_equals_dequantize_and_matmul(m, n, k, rot):
    x = ref.synth_activations(m, k, seed=m)
    w = ref.synth_weight(n, k, seed=n)
    bias = ref.bf16_bits_to_f32(ref.synth_bias(n, seed=3))
    qx, sx = ref.rotquant(x, rot, "int8")
    q, s, z = ref.weight_quant_affine(w, rot, 128)
    got = ref.linear_affine(qx, sx, q, s, z, bias, 128)
    want = ref.dequant_matmul(qx * np.asarray(sx, np.float64)[:, None], ref.dequant_affine(q, s, z), bias)
    assert ref.rel_l2(want, got) < 1e-12


@pytest.mark.parametrize("k", [128, 384, 4096, 4224])
def test_split_group_sums_are_exact_in_bf16(k):
    rng = np.random.default_rng(k)
    q = rng.integers(-127, 128, size=(9, k)).astype(np.int8)
    r = ref.group_sums(q, 128).astype(np.int64)
    sp = ref.group_sums_split(q, 128)
    g = k // 128
    hi, lo = sp[:, :g].astype(np.int64), sp[:, g:2 * g].astype(np.int64)
    assert np.array_equal(hi + lo, r)
    assert (hi % 128 == 0).all() and (lo >= 0).all() and (lo < 128).all()
    assert (sp[:, 2 * g:] == 0).all()
    # every entry survives a round trip through bf16
    assert np.array_equal(ref.bf16_round(sp.astype(np.float32)), sp.astype(np.float32))


@pytest.mark.parametrize("g", [16, 64, 256])
def test_rotation_is_the_block_hadamard_product(g):
    rng = np.random.default_rng(g)
    x = rng.standard_normal((4, 1024)).astype(np.float64)
    h = ref.build_hadamard(g).astype(np.float64)
    want = (x.reshape(4, 1024 // g, g) @ h).reshape(4, 1024)
    got = ref.fwht_stages(x.astype(np.float32), g).astype(np.float64)
    assert np.abs(got - want).max() < 1e-5 * np.abs(want).max()
    assert np.allclose(np.linalg.norm(got, axis=1), np.linalg.norm(x, axis=1), rtol=1e-5)


def test_rowcol_linear_equals_dequantized_product():
    rng = np.random.default_rng(7)
    qa = rng.integers(-7, 8, size=(6, 256))
    qw = rng.integers(-7, 8, size=(10, 256))
    sa = rng.uniform(0.01, 0.1, 6)
    sw = rng.uniform(0.01, 0.1, 10)
    got = ref.linear_rowcol(qa, sa, qw, sw)
    want = ref.dequant_matmul(qa * sa[:, None], qw * sw[:, None])
    assert ref.rel_l2(want, got) < 1e-12


@pytest.mark.parametrize("rot", [256, 64, 0])
def test_cpu_baseline_activation_quant_matches_the_oracle(rot):
    """The CPU baseline's torch activation quantizer (rotation in the reference's matrix form x @ H) gives the
    oracle's codes up to +-1 at rounding ties on at most 0.1 % of them, and scales within a few fp32 ulp."""
    import torch
    from oracle import cpu_path
    m, k = 64, 1024
    x = ref.synth_activations(m, k, seed=9)
    q, s = cpu_path.rotquant_int8_torch(torch.from_numpy(x.view(np.int16)).view(torch.bfloat16), rot)
    qo, so = ref.rotquant(x, rot, "int8")
    d = np.abs(q.numpy().astype(np.int32) - qo)
    assert d.max() <= 1 and (d > 0).mean() <= 1e-3
    np.testing.assert_allclose(s.numpy(), so, rtol=1e-6)


@pytest.mark.parametrize("rot", [256, 0])
def test_cpu_baseline_call_computes_the_affine_linear(rot):
    """The timed CPU baseline call (torch CPU: activation quantization, weight dequantization, fp32 F.linear)
    computes the same linear as the oracle's integer form on the codes it quantized, to fp32 rounding."""
    import torch
    from oracle import cpu_path
    m, n, k = 7, 48, 512
    x = ref.synth_activations(m, k, seed=5)
    w = ref.synth_weight(n, k, seed=6)
    bias = ref.bf16_bits_to_f32(ref.synth_bias(n, seed=7))
    q, s, z = ref.weight_quant_affine(w, rot, 128)
    packed = torch.from_numpy(ref.pack_int4(q))
    xt = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16)
    timings = []
    got = cpu_path.w4a8_affine_call(xt, rot, packed, torch.from_numpy(s), torch.from_numpy(z),
                                    torch.from_numpy(bias), timings=timings).numpy()
    qx, sx = cpu_path.rotquant_int8_torch(xt, rot)
    want = ref.linear_affine(qx.numpy().astype(np.int64), sx.numpy(), q, s, z, bias, 128)
    assert ref.rel_l2(want, got) < 1e-5
    assert len(timings) == 1 and all(t >= 0 for t in timings[0])


def test_intratio_oracle_is_the_per_element_sum():
    """Policies 5/7 (g64_gemm6.cu:8-11): acc[m, n] = sum_g cw[g, n] * sum_{k in g} a[m, k] * b[n, k], summed
    element by element for a tiny case; the fp32 output order of the reference kernel on top of it."""
    import numpy as np
    from oracle import ref
    rng = np.random.default_rng(0)
    m, n, k, g = 3, 4, 256, 64
    a = rng.integers(-7, 8, size=(m, k))
    b = rng.integers(-7, 8, size=(n, k))
    cw = rng.integers(1, 256, size=(k // g, n))
    acc = ref.intratio_acc(a, b, cw, g)
    for i in range(m):
        for j in range(n):
            want = sum(int(cw[kk // g, j]) * int(a[i, kk]) * int(b[j, kk]) for kk in range(k))
            assert acc[i, j] == want
    sa = np.full(m, 0.01, np.float32)
    sb = np.full(n, 0.02 / 255, np.float32)
    out = ref.linear_intratio(a, sa, b, sb, cw, g)
    assert out.dtype == np.float32
    assert np.allclose(out, acc * 0.01 * (0.02 / 255), rtol=1e-6)
