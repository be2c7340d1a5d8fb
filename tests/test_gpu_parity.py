"""GPU parity: the CUDA path (through the C ABI, via comfy_quant_bench_b200.ops) against the CPU oracle.

Bars: integer and byte outputs bit-exact (codes, packed nibbles, group sums, int32 accumulators); scales
bit-exact; bf16 outputs within rel-L2 <= 1e-3 of the oracle's float64 result rounded to bf16, with at most 1e-3 of
the elements off by more than one bf16 rounding.  The SwiGLU prologue computes silu with the device's hardware
exponential (and, per token, its fast division, as comfy-kitchen's fast-math build does), so its codes may differ
by 1 at rounding ties (<= 0.1 % of codes), the reference's own rule (g64_quant_test.py:72-103).
"""
import numpy as np
import pytest
import torch

from oracle import ref

pytestmark = pytest.mark.gpu

REL_L2 = 1e-3


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from comfy_quant_bench_b200 import ops as _ops, _lib
    _lib.load()
    return _ops


def bf16_dev(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def bits_of(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)


def f32_of(t: torch.Tensor) -> np.ndarray:
    return ref.bf16_bits_to_f32(bits_of(t))


def assert_bf16_close(got: torch.Tensor, want: np.ndarray, rel=REL_L2):
    g = f32_of(got).astype(np.float64)
    w = ref.bf16_round(np.asarray(want, np.float32)).astype(np.float64)
    r = ref.rel_l2(w, g)          # bf16 against the oracle rounded once to bf16
    assert r <= rel, f"rel-L2 {r:.3e}"
    # one bf16 rounding step of slack per element
    ulp = np.abs(w) * 2.0 ** -7 + 1e-30
    off = np.abs(g - w) > ulp
    assert off.mean() <= 1e-3, f"{off.mean():.2e} of elements beyond one bf16 ulp"


def codes_within_ties(got, want, frac=1e-3):
    d = np.abs(np.asarray(got, np.int32) - np.asarray(want, np.int32))
    assert d.max() <= 1
    assert (d > 0).mean() <= frac


@pytest.fixture(params=["one_sm", "pair"])
def gemm_variant(request, ops):
    """Runs a test once per kernel form of the int4-weight GEMM (one CTA per tile, or a CTA pair per tile)."""
    from comfy_quant_bench_b200 import _lib
    _lib.set_gemm_variant(_lib.CQ_GEMM_ONE_SM if request.param == "one_sm" else _lib.CQ_GEMM_PAIR)
    yield request.param
    _lib.set_gemm_variant(_lib.CQ_GEMM_AUTO)


def _check_status():
    from comfy_quant_bench_b200 import _lib
    torch.cuda.synchronize()
    assert _lib.take_device_status() == (0, 0)


# ----------------------------------------------------------------------------------------------
# activation rotation + quantization
# ----------------------------------------------------------------------------------------------

@pytest.mark.parametrize("m,k", [(1, 256), (37, 768), (64, 3072), (256, 3072), (5, 16384), (3, 20480), (2, 32768)])
@pytest.mark.parametrize("rot", [0, 16, 64, 256])
def test_rotquant_int8_rowwise_bit_exact(ops, m, k, rot):
    x = ref.synth_activations(m, k, seed=m + k + rot)
    q, s, gs = ops.rotquant(bf16_dev(x), rot, 0, group_sums=True)
    qr, sr = ref.rotquant(x, rot, "int8")
    assert np.array_equal(q.cpu().numpy(), qr.astype(np.int8))
    assert np.array_equal(s.cpu().numpy().view(np.uint32), sr.view(np.uint32))
    assert np.array_equal(f32_of(gs), ref.group_sums_split(qr, 128))
    # K-permuted int8 codes: each 8-column block in the order 0,2,4,6,1,3,5,7
    qp, _, _ = ops.rotquant(bf16_dev(x), rot, 0, kperm=True)
    perm = np.concatenate([np.arange(0, 8, 2), np.arange(1, 8, 2)])
    want = qr.reshape(m, k // 8, 8)[:, :, perm].reshape(m, k).astype(np.int8)
    assert np.array_equal(qp.cpu().numpy(), want)
    _check_status()


@pytest.mark.parametrize("m,m_pad", [(5, 16), (6, 7), (0, 3)])
def test_rotquant_int8_padding_rows_are_zero(ops, m, m_pad):
    k = 3072
    x = ref.synth_activations(max(m, 1), k, seed=11 + m)[:m]
    q, s, gs = ops.rotquant(bf16_dev(x), 256, 0, m_pad=m_pad, group_sums=True, kperm=True)
    qr, sr = ref.rotquant(x, 256, "int8") if m else (np.zeros((0, k), np.int16), np.zeros(0, np.float32))
    perm = np.concatenate([np.arange(0, 8, 2), np.arange(1, 8, 2)])
    q_np, s_np, g_np = q.cpu().numpy(), s.cpu().numpy(), f32_of(gs)
    assert np.array_equal(q_np[:m], qr.reshape(m, k // 8, 8)[:, :, perm].reshape(m, k).astype(np.int8))
    assert np.array_equal(s_np[:m].view(np.uint32), sr.view(np.uint32))
    assert np.array_equal(g_np[:m], ref.group_sums_split(qr, 128))
    assert not q_np[m:].any() and not s_np[m:].any() and not g_np[m:].any()
    _check_status()


@pytest.mark.parametrize("k", [1024, 32768])
def test_rotquant_int8_nonfinite_tokens(ops, k):
    """A NaN is ignored by the token's maximum and its rotation block quantizes to 0; an infinity gives the token
    scale inf and all codes 0.  The other token of a two-token CTA is unaffected."""
    x = ref.synth_activations(4, k, seed=5)
    nan_bits = np.uint16(0x7FC0)
    inf_bits = np.uint16(0x7F80)
    x[1, 600] = nan_bits
    x[2, 77] = inf_bits
    q, s, gs = ops.rotquant(bf16_dev(x), 256, 0, group_sums=True)
    q_np, s_np = q.cpu().numpy(), s.cpu().numpy()
    clean = x.copy()
    clean[1, 512:768] = 0           # the NaN's rotation block
    qr, sr = ref.rotquant(clean, 256, "int8")
    for r in (0, 1, 3):
        assert np.array_equal(q_np[r], qr[r].astype(np.int8)), r
        assert s_np[r].view(np.uint32) == sr[r].view(np.uint32), r
    assert not q_np[2].any() and np.isposinf(s_np[2])
    want_codes = qr.copy()
    want_codes[2] = 0
    assert np.array_equal(f32_of(gs), ref.group_sums_split(want_codes, 128))
    _check_status()


@pytest.mark.parametrize("m,k,rot", [(19, 1024, 256), (64, 3072, 64), (7, 512, 16), (3, 768, 0)])
def test_rotquant_int4_rowwise_packed_bit_exact(ops, m, k, rot):
    x = ref.synth_activations(m, k, seed=7 + k)
    q, s = ops.quantize_int4_rowwise_convrot64(bf16_dev(x), rot)
    qr, sr = ref.rotquant(x, rot, "int4")
    assert np.array_equal(q.cpu().numpy(), ref.pack_int4(qr))
    assert np.array_equal(s.cpu().numpy().view(np.uint32), sr.view(np.uint32))
    q8, s8, _ = ops.rotquant(bf16_dev(x), rot, 1, int4_as_int8=True)
    assert np.array_equal(q8.cpu().numpy(), qr.astype(np.int8))


@pytest.mark.parametrize("group", [64, 128])
@pytest.mark.parametrize("m,k", [(300, 4096), (77, 1024)])
def test_groupwise_quant_matches_oracle_and_pads(ops, group, m, k):
    x = ref.synth_activations(m, k, seed=group + m)
    q, s = ops.quant(bf16_dev(x), group, False, 128)
    mp = (m + 127) // 128 * 128
    assert q.shape == (mp, k // 2) and s.shape == (k // group, mp)
    qr, sr = ref.rotquant(x, 256, "int4_group", act_group=group)
    assert np.array_equal(q[:m].cpu().numpy(), ref.pack_int4(qr))
    assert np.array_equal(s[:, :m].cpu().numpy().view(np.uint32), sr.view(np.uint32))
    assert (q[m:] == 0).all() and (s[:, m:] == 0).all()


@pytest.mark.parametrize("group", [64, 128])
def test_groupwise_swiglu_quant_at_the_reference_test_shape(ops, group):
    """g64_quant_test.py's SwiGLU case (M=517, K=12288, h = [gate | up] of 2K columns): codes within rounding ties
    of the oracle, scales equal except at rare bf16 boundaries (the reference's rule), padding rows zero."""
    m, k = 517, 12288
    h = ref.synth_activations(m, 2 * k, seed=group)
    q, s = ops.quant(bf16_dev(h), group, True, 128)
    mp = (m + 127) // 128 * 128
    assert q.shape == (mp, k // 2) and s.shape == (k // group, mp)
    qr, sr = ref.rotquant(h, 256, "int4_group", swiglu=True, act_group=group)
    codes_within_ties(ref.unpack_int4_signed(q[:m].cpu().numpy()), qr)
    assert (s[:, :m].cpu().numpy() != sr).mean() <= 1e-3
    assert (q[m:] == 0).all() and (s[:, m:] == 0).all()


def test_groupwise_quant_matches_reference_golden(ops):
    """The reference's own quantizer reference (g64_quant_test.ref), with its acceptance rule."""
    import os
    g = dict(np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_golden.npz")))
    for tag, swiglu in (("act_m37_k1024_plain", False), ("act_m19_k512_swiglu", True)):
        for grp in (64, 128):
            q, s = ops.quant(bf16_dev(g[f"{tag}_x"]), grp, swiglu, 128)
            m = g[f"{tag}_x"].shape[0]
            codes_within_ties(ref.unpack_int4_signed(q[:m].cpu().numpy()), g[f"{tag}_g{grp}_q"])
            ss = s[:, :m].cpu().numpy()
            diff = ss != g[f"{tag}_g{grp}_s"]
            assert diff.mean() <= 1e-3


@pytest.mark.parametrize("mode,name", [(1, "int4"), (0, "int8")])
def test_swiglu_rotquant_within_ties(ops, mode, name):
    m, k = 48, 3072
    h = ref.synth_activations(m, 2 * k, seed=11)
    q, s, _ = ops.rotquant(bf16_dev(h), 256, mode, swiglu=True, int4_as_int8=True)
    qr, sr = ref.rotquant(h, 256, name, swiglu=True)
    codes_within_ties(q.cpu().numpy(), qr)
    assert np.allclose(s.cpu().numpy(), sr, rtol=1e-5)


def test_swiglu_fused_equals_quantizer_of_rounded_product_exactly(ops):
    """test_comfyui_fase4_dispatch.py:100-110, the reference's own assertion: on 64 x 2048 standard-normal bf16
    inputs the fused SwiGLU quantizer (hardware exponential, fast division, as comfy-kitchen's fast-math build)
    gives codes and scales identical to the plain quantizer fed torch's silu(gate) * up rounded once to bf16.  The
    two silu forms round a bf16 intermediate differently in about 1 of 1e8 elements; none of these 65k does."""
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(64, 2048, generator=g, device="cuda").to(torch.bfloat16)
    k = x.shape[-1] // 2
    qf, sf = ops.swiglu_quantize_int4_rowwise_convrot64(x)
    qc, sc = ops.quantize_int4_rowwise_convrot64(
        (torch.nn.functional.silu(x[:, :k].float()) * x[:, k:].float()).to(x.dtype), 256)
    assert torch.equal(qf, qc) and torch.equal(sf.reshape(-1), sc.reshape(-1))


def test_swiglu_fused_equals_quantizer_of_rounded_product(ops):
    """test_comfyui_fase4_dispatch.py:108-110 on the synthetic activations (outlier channels): the fused SwiGLU
    quantizer equals the plain quantizer fed torch's silu(gate)*up rounded once to bf16, within rounding ties
    (the fused silu takes the hardware exponential and fast division)."""
    m, k = 64, 1024
    h = bf16_dev(ref.synth_activations(m, 2 * k, seed=5))
    qf, sf = ops.swiglu_quantize_int4_rowwise_convrot64(h)
    prod = (torch.nn.functional.silu(h[:, :k].float()) * h[:, k:].float()).to(torch.bfloat16)
    qc, sc = ops.quantize_int4_rowwise_convrot64(prod, 256)
    codes_within_ties(ref.unpack_int4_signed(qf.cpu().numpy()), ref.unpack_int4_signed(qc.cpu().numpy()), 2e-3)
    assert torch.allclose(sf, sc, rtol=1e-5)


# ----------------------------------------------------------------------------------------------
# weight rotate-and-quantize
# ----------------------------------------------------------------------------------------------

@pytest.mark.parametrize("rot", [0, 64, 256])
@pytest.mark.parametrize("bf16_in", [False, True])
def test_weight_quantizers_bit_exact(ops, rot, bf16_in):
    n, k = 96, 1536
    w = ref.synth_weight(n, k, seed=rot + 3)
    if bf16_in:
        w = ref.bf16_round(w)
    wt = torch.from_numpy(w).cuda()
    wt = wt.to(torch.bfloat16) if bf16_in else wt
    q, s = ops.quantize_convrot_w4a4_weight(wt, convrot_groupsize=rot) if rot else (None, None)
    if rot:
        qr, sr = ref.weight_quant_convrot_rowwise(w, rot)
        assert np.array_equal(q.cpu().numpy(), ref.pack_int4(qr))
        assert np.array_equal(s.cpu().numpy().view(np.uint32), sr.view(np.uint32))
    q8, s8 = ops.quantize_int8_convrot_weight(wt, group_size=rot)
    qr8, sr8 = ref.weight_quant_int8_rowwise(w, rot)
    assert np.array_equal(q8.cpu().numpy(), qr8.astype(np.int8))
    assert np.array_equal(s8.cpu().numpy().view(np.uint32), sr8.view(np.uint32))
    qa, sa, za = ops.quantize_affine_w4_weight(wt, group_size=128, convrot_groupsize=rot)
    qra, sra, zra = ref.weight_quant_affine(w, rot, 128)
    assert np.array_equal(ref.unpack_uint4(qa.cpu().numpy()), qra)
    assert np.array_equal(f32_of(sa), sra) and np.array_equal(f32_of(za), zra)
    qg, sg = ops.quantize_int4_groupwise_weight(wt, group_size=128, convrot_groupsize=rot)
    qrg, srg = ref.weight_quant_groupwise_bf16up(w, rot, 128)
    assert np.array_equal(ref.unpack_int4_signed(qg.cpu().numpy()), qrg)
    assert np.array_equal(sg.cpu().numpy(), srg)


def test_weight_quant_matches_reference_golden(ops):
    import os
    g = dict(np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_golden.npz")))
    w = torch.from_numpy(g["wq_in"]).cuda()
    q, s = ops.quantize_convrot_w4a4_weight(w, 256)
    codes_within_ties(ref.unpack_int4_signed(q.cpu().numpy()), ref.unpack_int4_signed(g["wq_p0_packed"]))
    assert np.allclose(s.cpu().numpy(), g["wq_p0_scale"], rtol=1e-6)


# ----------------------------------------------------------------------------------------------
# GEMMs
# ----------------------------------------------------------------------------------------------

def _sparse_codes(rng, shape, density, lo, hi):
    c = rng.integers(lo, hi + 1, size=shape)
    return np.where(rng.random(shape) < density, c, 0)


@pytest.mark.parametrize("m,n,k", [(256, 128, 128), (300, 200, 3072), (1000, 640, 1024)])
def test_int32_accumulators_bit_exact_rowcol(ops, gemm_variant, m, n, k):
    """Unit scales and sparse +-1 codes keep |acc| <= 256, exactly representable in bf16: out == acc."""
    rng = np.random.default_rng(m + n)
    a = _sparse_codes(rng, (m, k), 0.05, -1, 1).astype(np.int8)
    b = _sparse_codes(rng, (n, k), 0.05, -1, 1).astype(np.int8)
    acc = ref.int_gemm(a, b)
    assert np.abs(acc).max() <= 256
    ones_m = torch.ones(m, device="cuda")
    ones_n = torch.ones(n, device="cuda")
    out4 = ops.gemm_rowcol(torch.from_numpy(a).cuda(), ones_m, torch.from_numpy(ref.pack_int4(b)).cuda(), ones_n)
    assert np.array_equal(f32_of(out4), acc.astype(np.float32))
    out8 = ops.gemm_rowcol(torch.from_numpy(a).cuda(), ones_m, torch.from_numpy(b).cuda(), ones_n, b_int8=True)
    assert np.array_equal(f32_of(out8), acc.astype(np.float32))
    _check_status()


@pytest.mark.parametrize("m,n,k", [(256, 128, 128), (300, 200, 3072)])
def test_int32_accumulators_bit_exact_affine(ops, gemm_variant, m, n, k):
    """scale 1, zero 0: out == sum over groups of the exact int32 partials."""
    rng = np.random.default_rng(m * 3 + n)
    a = _sparse_codes(rng, (m, k), 0.05, -1, 1).astype(np.int8)
    q = (8 + _sparse_codes(rng, (n, k), 0.05, -1, 1)).astype(np.int16)
    acc = ref.int_gemm(a, q - 8)
    s = torch.ones(k // 128, n, dtype=torch.bfloat16, device="cuda")
    z = torch.zeros_like(s)
    gs = torch.from_numpy(ref.group_sums_split(a, 128)).to(torch.bfloat16).cuda()
    out = ops.gemm_affine(torch.from_numpy(a).cuda(), torch.ones(m, device="cuda"), gs,
                          torch.from_numpy(ref.pack_int4(q)).cuda(), s, z)
    assert np.array_equal(f32_of(out), acc.astype(np.float32))


@pytest.mark.parametrize("m,n,k", [(256, 128, 128), (300, 200, 3072), (64, 128, 4224)])
def test_affine_zero_point_term_exact(ops, gemm_variant, m, n, k):
    """scale 0, zero 1: out == sum_g R[g, m] (the tensor-core zero-point pass on the split group sums)."""
    rng = np.random.default_rng(m + k)
    a = _sparse_codes(rng, (m, k), 0.02, -1, 1).astype(np.int8)
    q = np.full((n, k), 8, np.int16)
    want = ref.group_sums(a, 128).sum(axis=1).astype(np.float32)
    assert np.abs(want).max() <= 256
    s = torch.zeros(k // 128, n, dtype=torch.bfloat16, device="cuda")
    z = torch.ones_like(s)
    gs = torch.from_numpy(ref.group_sums_split(a, 128)).to(torch.bfloat16).cuda()
    out = ops.gemm_affine(torch.from_numpy(a).cuda(), torch.ones(m, device="cuda"), gs,
                          torch.from_numpy(ref.pack_int4(q)).cuda(), s, z)
    assert np.array_equal(f32_of(out), np.repeat(want[:, None], n, axis=1))


@pytest.mark.parametrize("m,n,k,bias", [(300, 200, 768, True), (512, 1024, 3072, True), (64, 384, 2048, False)])
@pytest.mark.parametrize("kperm", [False, True])
def test_gemm_rowcol_random_scales(ops, gemm_variant, m, n, k, bias, kperm):
    rng = np.random.default_rng(k + m)
    a = rng.integers(-127, 128, size=(m, k)).astype(np.int8)
    b = rng.integers(-7, 8, size=(n, k)).astype(np.int8)
    sa = (rng.random(m) * 0.01 + 0.005).astype(np.float32)
    sb = (rng.random(n) * 0.01 + 0.005).astype(np.float32)
    bb = ref.synth_bias(n, seed=k) if bias else None
    want = ref.linear_rowcol(a, sa, b, sb, None if bb is None else ref.bf16_bits_to_f32(bb))
    ad = a
    if kperm:
        perm = np.concatenate([np.arange(0, 8, 2), np.arange(1, 8, 2)])
        ad = a.reshape(m, k // 8, 8)[:, :, perm].reshape(m, k)
    out = ops.gemm_rowcol(torch.from_numpy(np.ascontiguousarray(ad)).cuda(), torch.from_numpy(sa).cuda(),
                          torch.from_numpy(ref.pack_int4(b)).cuda(), torch.from_numpy(sb).cuda(),
                          None if bb is None else bf16_dev(bb), a_kperm=kperm)
    assert_bf16_close(out, want)


@pytest.mark.parametrize("m,n,k", [(4096, 4096, 4096), (4096, 24576, 4096), (16384, 4096, 12288)])
def test_gemm_rowcol_at_reference_bench_shapes(ops, m, n, k):
    """g64_bench6.py's GEMM check (:50-79, 110-128, 154) at its shapes: random int4 codes in [-7, 7] on both sides,
    scales U(0.005, 0.015); on the first and last 256 rows rel-L2 < 3e-3 and max |diff| < 4 % of the reference's
    standard deviation; two runs bit-identical."""
    rng = np.random.default_rng(n + k + m)
    a = rng.integers(-7, 8, size=(m, k), dtype=np.int8)
    b = rng.integers(-7, 8, size=(n, k), dtype=np.int8)
    sa = rng.uniform(0.005, 0.015, m).astype(np.float32)
    sb = rng.uniform(0.005, 0.015, n).astype(np.float32)
    args = (torch.from_numpy(a).cuda(), torch.from_numpy(sa).cuda(), torch.from_numpy(ref.pack_int4(b)).cuda(),
            torch.from_numpy(sb).cuda(), None)
    y1 = ops.gemm_rowcol(*args)
    assert torch.equal(y1, ops.gemm_rowcol(*args)), "two runs differ"
    _check_status()
    bf = b.astype(np.float64)
    for rows in (slice(0, 256), slice(m - 256, m)):
        want = (a[rows].astype(np.float64) @ bf.T) * sa[rows, None].astype(np.float64) * sb[None, :].astype(np.float64)
        d = f32_of(y1[rows]).astype(np.float64) - want
        assert np.linalg.norm(d) / np.linalg.norm(want) < 3e-3
        assert np.abs(d).max() / want.std() < 0.04


def test_int4_linear_matches_reference_policy0_golden(ops):
    import os
    g = dict(np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_golden.npz")))
    # int4_linear(qact, qweight, x_scale, wscales, bias): the order of g64_bench6.py:109
    out = ops.int4_linear(torch.from_numpy(g["gemm_a_packed"]).cuda(), torch.from_numpy(ref.pack_int4(g["gemm_b"])).cuda(),
                          torch.from_numpy(g["gemm_p0_sa"]).cuda(), torch.from_numpy(g["gemm_p0_sb"]).cuda(),
                          bf16_dev(g["gemm_bias"]))
    assert_bf16_close(out, g["gemm_p0_out"].astype(np.float64))


# ----------------------------------------------------------------------------------------------
# fused linears (activation stage + GEMM) against the oracle pipeline
# ----------------------------------------------------------------------------------------------

@pytest.mark.parametrize("m,n,k,rot", [(300, 384, 1024, 256), (256, 3072, 3072, 0), (129, 256, 3072, 64)])
def test_w4a8_affine_linear_vs_oracle(ops, gemm_variant, m, n, k, rot):
    x = ref.synth_activations(m, k, seed=m)
    w = ref.synth_weight(n, k, seed=n)
    bb = ref.synth_bias(n, seed=3)
    qw, sw, zw = ops.quantize_affine_w4_weight(torch.from_numpy(w).cuda(), 128, rot)
    out = ops.w4a8_affine_linear(bf16_dev(x), qw, sw, zw, bf16_dev(bb), group_size=128, convrot_groupsize=rot)
    qx, sx = ref.rotquant(x, rot, "int8")
    qr, sr, zr = ref.weight_quant_affine(w, rot, 128)
    want = ref.linear_affine(qx, sx, qr, sr, zr, ref.bf16_bits_to_f32(bb), 128)
    assert_bf16_close(out, want)
    # the dequantize-and-matmul path (patches/tests/test_comfyui_fase4_dispatch.py:98) gives the same numbers
    deq = ref.dequant_matmul(qx * sx[:, None].astype(np.float64), ref.dequant_affine(qr, sr, zr),
                             ref.bf16_bits_to_f32(bb))
    assert ref.rel_l2(deq, want) < 1e-6
    # and the quantized linear tracks the full-precision one (liveness, cf. tools/verify_w4a4.py:32-38)
    full = ref.bf16_bits_to_f32(x).astype(np.float64) @ w.astype(np.float64).T + ref.bf16_bits_to_f32(bb)
    assert ref.rel_l2(full, f32_of(out)) < 0.15
    _check_status()


@pytest.mark.parametrize("m,n,k,rot,dtype", [(300, 384, 1024, 256, "int4"), (64, 512, 3072, 64, "int8"),
                                             (200, 256, 768, 16, "int4")])
def test_convrot_w4a4_linear_vs_oracle(ops, gemm_variant, m, n, k, rot, dtype):
    x = ref.synth_activations(m, k, seed=k)
    w = ref.synth_weight(n, k, seed=m)
    bb = ref.synth_bias(n, seed=5)
    qw, sw = ops.quantize_convrot_w4a4_weight(torch.from_numpy(w).cuda(), rot)
    out = ops.convrot_w4a4_linear(bf16_dev(x), qw, sw, bf16_dev(bb), convrot_groupsize=rot, linear_dtype=dtype)
    qx, sx = ref.rotquant(x, rot, dtype)
    qr, sr = ref.weight_quant_convrot_rowwise(w, rot)
    want = ref.linear_rowcol(qx, sx, qr, sr, ref.bf16_bits_to_f32(bb))
    assert_bf16_close(out, want)


def test_convrot_w4a4_swiglu_linear(ops):
    m, n, k = 128, 256, 1024
    h = ref.synth_activations(m, 2 * k, seed=21)
    w = ref.synth_weight(n, k, seed=22)
    qw, sw = ops.quantize_convrot_w4a4_weight(torch.from_numpy(w).cuda(), 256)
    out = ops.convrot_w4a4_linear(bf16_dev(h), qw, sw, None, input_act="swiglu")
    qx, sx = ref.rotquant(h, 256, "int4", swiglu=True)
    qr, sr = ref.weight_quant_convrot_rowwise(w, 256)
    want = ref.linear_rowcol(qx, sx, qr, sr)
    # a code flipped at a tie moves a row by one quantization step: compare at the linear's level
    assert ref.rel_l2(ref.bf16_round(want.astype(np.float32)), f32_of(out)) < 5e-3


def test_int8_linear_vs_oracle(ops):
    m, n, k = 200, 320, 2048
    x = ref.synth_activations(m, k, seed=31)
    w = ref.synth_weight(n, k, seed=32)
    qw, sw = ops.quantize_int8_convrot_weight(torch.from_numpy(w).cuda(), 256)
    out = ops.int8_linear(bf16_dev(x), qw, sw, None, convrot=True, convrot_groupsize=256)
    qx, sx = ref.rotquant(x, 256, "int8")
    qr, sr = ref.weight_quant_int8_rowwise(w, 256)
    assert_bf16_close(out, ref.linear_rowcol(qx, sx, qr, sr.reshape(-1)))


# ----------------------------------------------------------------------------------------------
# full benchmark size (M=4096, K=3072, N=12288): size-independent properties + a row slice against the oracle
# ----------------------------------------------------------------------------------------------

def _full_size_affine_check(ops, m, n, k, rot, y, x, w, bias_bits):
    """Row slices spread over all of M (eight slices of 64 rows, both ends included) against the oracle, with the
    bias, plus the reference bench's own acceptance check per slice (g64_bench6.py:71-79, 154): rel-L2 < 3e-3 and
    max |diff| < 4 % of the reference's standard deviation."""
    starts = np.linspace(0, m - 64, 8).astype(int)
    rows = np.concatenate([np.arange(s0, s0 + 64) for s0 in starts])
    qx, sx = ref.rotquant(x[rows], rot, "int8")
    qr, sr, zr = ref.weight_quant_affine(w, rot, 128)
    want = ref.linear_affine(qx, sx, qr, sr, zr, ref.bf16_bits_to_f32(bias_bits), 128)
    got = y[torch.from_numpy(rows).cuda()]
    assert_bf16_close(got, want)
    g = f32_of(got).astype(np.float64)
    for i in range(len(starts)):
        sl = slice(64 * i, 64 * i + 64)
        d = g[sl] - want[sl]
        assert np.linalg.norm(d) / np.linalg.norm(want[sl]) < 3e-3
        assert np.abs(d).max() / want[sl].std() < 0.04
    return qr


def test_full_size_w4a8_properties(ops, gemm_variant):
    m, n, k = 4096, 12288, 3072
    x = ref.synth_activations(m, k, seed=0)
    w = ref.synth_weight(n, k, seed=1)
    b = ref.synth_bias(n, seed=2)
    xt, bt = bf16_dev(x), bf16_dev(b)
    qw, sw, zw = ops.quantize_affine_w4_weight(torch.from_numpy(w).cuda(), 128, 256)
    y1 = ops.w4a8_affine_linear(xt, qw, sw, zw, bt, convrot_groupsize=256)
    y2 = ops.w4a8_affine_linear(xt, qw, sw, zw, bt, convrot_groupsize=256)
    assert torch.equal(y1, y2), "two runs differ (shared-memory or TMEM race)"
    y0 = ops.w4a8_affine_linear(xt, qw, sw, zw, None, convrot_groupsize=256)
    y3 = ops.w4a8_affine_linear(xt * 2, qw, sw, zw, None, convrot_groupsize=256)
    assert torch.equal(y3, y0 * 2), "output must scale exactly with a power-of-two input scale"
    qr = _full_size_affine_check(ops, m, n, k, 256, y1, x, w, b)
    assert np.array_equal(ref.unpack_uint4(qw.cpu().numpy()), qr)
    _check_status()


def test_c1_at_its_own_shape_with_bias(ops, gemm_variant):
    """BASELINE config 1 at its shape: W4A8 M=4096, N=K=3072, affine int4 g128, no rotation, bias."""
    m, n, k = 4096, 3072, 3072
    x = ref.synth_activations(m, k, seed=10)
    w = ref.synth_weight(n, k, seed=11)
    b = ref.synth_bias(n, seed=12)
    qw, sw, zw = ops.quantize_affine_w4_weight(torch.from_numpy(w).cuda(), 128, 0)
    y = ops.w4a8_affine_linear(bf16_dev(x), qw, sw, zw, bf16_dev(b), convrot_groupsize=0)
    _full_size_affine_check(ops, m, n, k, 0, y, x, w, b)
    _check_status()


def test_full_size_w4a4_properties(ops, gemm_variant):
    m, n, k = 4096, 12288, 3072
    x = ref.synth_activations(m, k, seed=0)
    w = ref.synth_weight(n, k, seed=1)
    xt = bf16_dev(x)
    qw, sw = ops.quantize_convrot_w4a4_weight(torch.from_numpy(w).cuda(), 256)
    y1 = ops.convrot_w4a4_linear(xt, qw, sw)
    assert torch.equal(y1, ops.convrot_w4a4_linear(xt, qw, sw))
    rows = np.r_[0:256, m - 256:m]
    qx, sx = ref.rotquant(x[rows], 256, "int4")
    qr, sr = ref.weight_quant_convrot_rowwise(w, 256)
    assert_bf16_close(y1[torch.from_numpy(rows).cuda()], ref.linear_rowcol(qx, sx, qr, sr))


# ----------------------------------------------------------------------------------------------
# error behaviour (host-side checks, nothing launched)
# ----------------------------------------------------------------------------------------------

def test_errors_raise(ops):
    from comfy_quant_bench_b200._lib import CQShapeError
    x = torch.zeros(4, 300, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(CQShapeError):
        ops.quantize_int4_rowwise_convrot64(x, 256)
    with pytest.raises(ValueError):
        ops.convrot_w4a4_linear(torch.zeros(4, 256, device="cuda"), torch.zeros(8, 64, dtype=torch.int8, device="cuda"),
                                torch.ones(8, device="cuda"))
    with pytest.raises(ValueError):
        ops.quantize_int4_rowwise_convrot64(torch.zeros(4, 256, dtype=torch.bfloat16), 256)
    with pytest.raises(ValueError):
        ops.convrot_w4a4_linear(torch.zeros(4, 256, device="cuda"), torch.zeros(8, 128, dtype=torch.int8, device="cuda"),
                                torch.ones(8, device="cuda"), linear_dtype="fp8")


@pytest.mark.parametrize("m", [1, 2, 3, 5, 8, 9])
@pytest.mark.parametrize("n,k", [(320, 1280), (392, 3072)])
def test_w4a8_affine_linear_few_tokens_vs_oracle(ops, m, n, k):
    """M <= 8 runs the one-warp-per-row product (K/32 chunks not a multiple of 32 at K=1280; N not a multiple of
    the 8 rows per CTA at 392); M = 9 the tensor-core GEMM.  Both against the oracle, deterministic, and exact under
    a power-of-two input scale without bias."""
    x = ref.synth_activations(m, k, seed=40 + m)
    w = ref.synth_weight(n, k, seed=41)
    bb = ref.synth_bias(n, seed=42)
    qw, sw, zw = ops.quantize_affine_w4_weight(torch.from_numpy(w).cuda(), 128, 256)
    xt = bf16_dev(x)
    out = ops.w4a8_affine_linear(xt, qw, sw, zw, bf16_dev(bb), group_size=128, convrot_groupsize=256)
    _check_status()
    qx, sx = ref.rotquant(x, 256, "int8")
    qr, sr, zr = ref.weight_quant_affine(w, 256, 128)
    assert_bf16_close(out, ref.linear_affine(qx, sx, qr, sr, zr, ref.bf16_bits_to_f32(bb), 128))
    y1 = ops.w4a8_affine_linear(xt, qw, sw, zw, None, group_size=128, convrot_groupsize=256)
    assert torch.equal(y1, ops.w4a8_affine_linear(xt, qw, sw, zw, None, group_size=128, convrot_groupsize=256))
    assert torch.equal(ops.w4a8_affine_linear(xt * 2, qw, sw, zw, None, group_size=128, convrot_groupsize=256),
                       y1 * 2)


# n % 64 == 0: 64-column boxes shared by two epilogue warps; n = 96: 32-column boxes (one warp each)
@pytest.mark.parametrize("m,n,k,col0,ldo", [(300, 256, 1024, 256, 768), (1000, 640, 3072, 0, 1280),
                                            (130, 96, 1024, 32, 256), (77, 128, 512, 40, 256)])
def test_affine_linear_into_several_buffers_at_an_offset(ops, gemm_variant, m, n, k, col0, ldo):
    """The column-parallel form writes this shard's columns into every output buffer at col0; the rest stays."""
    from comfy_quant_bench_b200 import _lib
    x = bf16_dev(ref.synth_activations(m, k, seed=11))
    w = torch.from_numpy(ref.synth_weight(n, k, seed=12)).cuda()
    qw, s, z = ops.quantize_affine_w4_weight(w, 128, 256)
    zt = ops.prepare_affine_zeros(z, 128)
    bias = bf16_dev(ref.synth_bias(n, seed=13))
    # the same codes through the unsplit GEMM (the fused linear may split K for this few-tile shape, which changes
    # the fp32 summation order; the column-parallel form never splits)
    q, sx, gs = ops.rotquant(x, 256, _lib.CQ_ACT_INT8_ROW, m_pad=(m + 15) // 16 * 16, group_sums=True, kperm=True)
    want = ops.gemm_affine(q[:m], sx[:m], gs, qw, s, z, bias, a_kperm=True, zeros_prepared=zt)
    outs = [torch.full((m, ldo), 7.0, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    ops.w4a8_affine_linear_into(x, qw, s, zt, bias, outs, col0, ldo, convrot_groupsize=256)
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o[:, col0:col0 + n], want)
        assert (o[:, :col0] == 7.0).all() and (o[:, col0 + n:] == 7.0).all()


def test_affine_linear_into_rejects_bad_layouts(ops):
    from comfy_quant_bench_b200 import _lib
    m, n, k = 64, 256, 256
    x = bf16_dev(ref.synth_activations(m, k, seed=1))
    w = torch.from_numpy(ref.synth_weight(n, k, seed=2)).cuda()
    qw, s, z = ops.quantize_affine_w4_weight(w, 128, 0)
    zt = ops.prepare_affine_zeros(z, 128)
    out = torch.zeros(m, 512, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.CQShapeError):      # columns past the row
        ops.w4a8_affine_linear_into(x, qw, s, zt, None, [out], 384, 512)
    with pytest.raises(_lib.CQShapeError):      # offset not a multiple of 8
        ops.w4a8_affine_linear_into(x, qw, s, zt, None, [out], 4, 512)
    with pytest.raises(_lib.CQError):           # more than 8 buffers
        ops.w4a8_affine_linear_into(x, qw, s, zt, None, [out] * 9, 0, 512)


@pytest.mark.parametrize("m,n,k,rot,dtype", [(300, 384, 1024, 256, "int4"), (4096, 12288, 3072, 64, "int4"),
                                             (77, 256, 512, 16, "int8")])
def test_convrot_w4a4_swiglu_output_matches_torch_composite(ops, gemm_variant, m, n, k, rot, dtype):
    """The SwiGLU output fused into the W4A4 GEMM's epilogue equals torch's silu(y[:, :N/2]) * y[:, N/2:] on the
    bf16 output of the plain linear (same codes, same int32 sums, the same two bf16 roundings)."""
    import torch.nn.functional as F
    x = bf16_dev(ref.synth_activations(m, k, seed=m + n))
    w = torch.from_numpy(ref.synth_weight(n, k, seed=n)).cuda()
    qw, sw = ops.quantize_convrot_w4a4_weight(w, rot)
    bias = bf16_dev(ref.synth_bias(n, seed=3))
    y = ops.convrot_w4a4_linear(x, qw, sw, bias, convrot_groupsize=rot, linear_dtype=dtype)
    want = F.silu(y[:, : n // 2]) * y[:, n // 2:]
    qg, sg, bg = ops.prepare_swiglu_output_weight(qw, sw, bias)
    got = ops.convrot_w4a4_linear_swiglu(x, qg, sg, bg, convrot_groupsize=rot, linear_dtype=dtype)
    _check_status()
    assert got.shape == (m, n // 2)
    g, w_ = got.float(), want.float()
    assert float((g - w_).abs().max()) <= float(w_.abs().max()) * 2.0 ** -7
    assert float((got != want).float().mean()) <= 1e-3


def test_swiglu_output_rows_interleave_tiles(ops):
    idx = ops.swiglu_output_rows(256)
    assert idx[:16].tolist() == list(range(16)) and idx[16:32].tolist() == list(range(128, 144))
    assert idx[32:48].tolist() == list(range(16, 32)) and idx[240:].tolist() == list(range(240, 256))
    assert sorted(idx.tolist()) == list(range(256))


# ----------------------------------------------------------------------------------------------
# per-group scales on both sides (the reference GEMM's policy 4)
# ----------------------------------------------------------------------------------------------

def test_groupwise_gemm_matches_reference_policy4_golden(ops):
    """The reference's own policy-4 outputs (g64_bench6.ref on its seeded inputs, committed by make_golden.py)."""
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_golden.npz"))
    a, b = g["gemm_a"], g["gemm_b"]
    out = ops.gemm(torch.from_numpy(g["gemm_a_packed"]).cuda(), torch.from_numpy(ref.pack_int4(b)).cuda(),
                   torch.from_numpy(g["gemm_p4_sa"]).cuda(), torch.from_numpy(g["gemm_p4_sb"]).cuda(),
                   bias=bf16_dev(g["gemm_bias"]), pol=4)
    assert out.shape == (a.shape[0], b.shape[0])
    assert_bf16_close(out, g["gemm_p4_out"])
    _check_status()


@pytest.mark.parametrize("m,n,k", [(4096, 4096, 4096), (384, 512, 1024), (1000, 768, 3072)])
def test_groupwise_gemm_vs_oracle_with_reference_acceptance(ops, m, n, k):
    """Random int4 codes and per-group scales: the oracle's float64 policy-4 product, with the reference bench's
    rule on the first and last 256 rows (g64_bench6.py:71-79: rel-L2 < 3e-3, max |diff| < 4 % of the std) and two
    runs bit-identical."""
    rng = np.random.default_rng(m + n + k)
    a = rng.integers(-7, 8, size=(m, k)).astype(np.int8)
    b = rng.integers(-8, 8, size=(n, k)).astype(np.int8)
    sa = rng.uniform(0.005, 0.015, size=(k // 128, m)).astype(np.float32)
    sb = ref.bf16_round(rng.uniform(0.005, 0.015, size=(k // 128, n)).astype(np.float32))
    bias = ref.synth_bias(n, seed=5)
    args = (torch.from_numpy(a).cuda(), torch.from_numpy(sa).cuda(), torch.from_numpy(ref.pack_int4(b)).cuda(),
            torch.from_numpy(sb).cuda(), bf16_dev(bias))
    y1 = ops.gemm_groupwise(*args)
    y2 = ops.gemm_groupwise(*args)
    assert torch.equal(y1, y2)
    rows = np.r_[0:min(256, m), max(0, m - 256):m]
    want = ref.linear_groupwise(a[rows], sa[:, rows], b, sb, ref.bf16_bits_to_f32(bias), 128)
    got = y1[torch.from_numpy(rows).cuda()]
    assert_bf16_close(got, want)
    gv = f32_of(got).astype(np.float64)
    half = len(rows) // 2
    for sl in (slice(0, half), slice(half, len(rows))):
        d = gv[sl] - want[sl]
        assert np.linalg.norm(d) / np.linalg.norm(want[sl]) < 3e-3
        assert np.abs(d).max() / want[sl].std() < 0.04
    _check_status()


# ----------------------------------------------------------------------------------------------
# integer weight ratios per group (the reference GEMM's policies 5 / 7 / 15 / 17)
# ----------------------------------------------------------------------------------------------

def _intratio_case(m, n, k, group, seed):
    rng = np.random.default_rng(seed)
    a = rng.integers(-7, 8, size=(m, k)).astype(np.int8)
    b = rng.integers(-7, 8, size=(n, k)).astype(np.int8)
    sa = rng.uniform(0.005, 0.015, size=m).astype(np.float32)
    sb = (rng.uniform(0.005, 0.015, size=n) / 255).astype(np.float32)
    cw = rng.integers(1, 256, size=(k // group, n)).astype(np.int32)
    bias = ref.synth_bias(n, seed=seed + 1)
    return a, b, sa, sb, cw, bias


@pytest.mark.parametrize("pol,m,n,k", [(7, 4096, 4096, 4096), (5, 4096, 4096, 4096), (7, 512, 768, 12288),
                                       (5, 300, 512, 12288), (7, 77, 256, 1024)])
def test_intratio_gemm_vs_oracle_with_reference_acceptance(ops, pol, m, n, k):
    """Policies 5 (g64) and 7 (g128), through the reference's interface ops.gemm (packed activations): the int32 sum
    of P_g * cw[g, n] is exact, and the output follows the reference kernel's fp32 order, so it equals the oracle's
    fp32 emulation of that order up to a rounding tie (<= 1e-4 of the outputs one bf16 step away); the reference
    bench's acceptance rule on the first and last 256 rows; the uint8-ratio policies (15 / 17) bit-identical to
    5 / 7; two runs bit-identical.  K = 12288 takes the path that shifts each group's sum before the ratio."""
    group = 64 if pol == 5 else 128
    a, b, sa, sb, cw, bias = _intratio_case(m, n, k, group, seed=m + n + k + pol)
    ap = torch.from_numpy(ref.pack_int4(a)).cuda()
    bp = torch.from_numpy(ref.pack_int4(b)).cuda()
    sa_t, sb_t, cw_t = torch.from_numpy(sa).cuda(), torch.from_numpy(sb).cuda(), torch.from_numpy(cw).cuda()
    y1 = ops.gemm(ap, bp, sa_t, sb_t, None, cw_t, bf16_dev(bias), pol=pol)
    y2 = ops.gemm(ap, bp, sa_t, sb_t, None, cw_t, bf16_dev(bias), pol=pol)
    y8 = ops.gemm(ap, bp, sa_t, sb_t, None, cw_t.to(torch.uint8), bf16_dev(bias), pol=pol + 10)
    assert torch.equal(y1, y2) and torch.equal(y1, y8)
    rows = np.r_[0:min(256, m), max(0, m - 256):m]
    want32 = ref.linear_intratio(a[rows], sa[rows], b, sb, cw, group, ref.bf16_bits_to_f32(bias))
    got = y1[torch.from_numpy(rows).cuda()]
    gb = bits_of(got)
    wb = ref.f32_to_bf16_bits(want32)
    d = np.abs(gb.astype(np.int32) - wb.astype(np.int32))
    assert d.max() <= 1 and (d > 0).mean() <= 1e-4, ((d > 0).mean(), d.max())
    want = ref.intratio_acc(a[rows], b, cw, group).astype(np.float64) * sa[rows, None] * sb[None, :] + \
        ref.bf16_bits_to_f32(bias)[None, :]
    gv = f32_of(got).astype(np.float64)
    half = len(rows) // 2
    for sl in (slice(0, half), slice(half, len(rows))):
        dd = gv[sl] - want[sl]
        assert np.linalg.norm(dd) / np.linalg.norm(want[sl]) < 3e-3
        assert np.abs(dd).max() / want[sl].std() < 0.04
    _check_status()


def test_intratio_gemm_rejects_bad_arguments(ops):
    from comfy_quant_bench_b200 import _lib
    a = torch.zeros(256, 512, dtype=torch.int8, device="cuda")
    b = torch.zeros(256, 256, dtype=torch.int8, device="cuda")
    s = torch.ones(256, device="cuda")
    with pytest.raises(ValueError):      # ratios of the wrong shape
        ops.gemm_intratio(a, s, b, s, torch.ones(3, 256, dtype=torch.int32, device="cuda"), 128)
    with pytest.raises(ValueError):      # ratios of the wrong type
        ops.gemm_intratio(a, s, b, s, torch.ones(4, 256, dtype=torch.int16, device="cuda"), 128)
    with pytest.raises(_lib.CQShapeError):
        ops.gemm_intratio(a, s, b, s, torch.ones(16, 256, dtype=torch.int32, device="cuda"), 32)   # group 32
    _check_status()


@pytest.mark.parametrize("swiglu", [False, True])
def test_groupwise_linear_matches_the_node_path(ops, swiglu):
    """The node's policy-4 forward: per-group quantizer (ConvRot-256, g128, bf16-up scales), then the GEMM, against
    the oracle's quantizers and policy-4 product on the same inputs."""
    m, n, k = 300, 384, 1024
    x = ref.synth_activations(m, 2 * k if swiglu else k, seed=21)
    w = ref.synth_weight(n, k, seed=22)
    bias = ref.synth_bias(n, seed=23)
    qw, sw = ops.quantize_int4_groupwise_weight(torch.from_numpy(w).cuda(), 128, 256)
    y = ops.w4a4_groupwise_linear(bf16_dev(x), qw, sw, bf16_dev(bias), swiglu=swiglu)
    qa, sa = ref.rotquant(x, 256, "int4_group", swiglu=swiglu, act_group=128)
    qr, sr = ref.weight_quant_groupwise_bf16up(w, 256, 128)
    want = ref.linear_groupwise(qa, sa, qr, sr, ref.bf16_bits_to_f32(bias), 128)
    assert_bf16_close(y, want, rel=2e-3 if swiglu else REL_L2)
    _check_status()
