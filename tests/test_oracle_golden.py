"""Pin the CPU oracle (oracle/ref.py) to the reference's own functions (fixtures from tests/golden/make_golden.py).

Acceptance rules are the reference's own (``g64_quant_test.py:1-11``): codes equal except rounding ties
(<= 0.1 % of codes, |diff| == 1); scales equal, or exactly one bf16 ulp where the reference's value sits
within 1e-5 (relative) of a bf16 boundary.
"""
import json
import os

import numpy as np
import pytest

from oracle import ref

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def g():
    return dict(np.load(os.path.join(GOLD, "ref_golden.npz")))


def _codes_match(got, want, frac=1e-3):
    d = np.abs(np.asarray(got, np.int32) - np.asarray(want, np.int32))
    assert d.max() <= 1, f"code differs by {d.max()}"
    assert (d > 0).mean() <= frac, f"{(d > 0).mean():.2e} of codes differ"


def test_bf16_up_matches_reference(g):
    assert np.array_equal(ref.bf16_up(g["bf16_up_in"]).view(np.uint32), g["bf16_up_out"].view(np.uint32))


def test_unpack_matches_reference(g):
    assert np.array_equal(ref.unpack_int4_signed(g["unpack_in"]), g["unpack_out"])


def test_pack_roundtrip_matches_reference(g):
    a = g["gemm_a"]
    assert np.array_equal(ref.pack_int4(a), g["gemm_a_packed"])
    assert np.array_equal(ref.unpack_int4_signed(ref.pack_int4(a)), a)


def test_hadamard_is_orthonormal_involution():
    for n in (16, 64, 256):
        h = ref.build_hadamard(n)
        assert np.allclose(h @ h, np.eye(n), atol=1e-12)
        assert np.allclose(h, h.T)
        x = np.random.default_rng(n).standard_normal((5, 4 * n)).astype(np.float32)
        assert np.abs(ref.fwht_stages(x, n) - ref.rotate_matmul(x, n)).max() < 1e-5


@pytest.mark.parametrize("tag", ["act_m37_k1024_plain", "act_m19_k512_swiglu"])
@pytest.mark.parametrize("grp", [64, 128])
def test_groupwise_activation_quant_matches_reference(g, tag, grp):
    x = g[f"{tag}_x"]
    q, s = ref.rotquant(x, 256, "int4_group", swiglu="swiglu" in tag, act_group=grp)
    want_q, want_s, want_t = g[f"{tag}_g{grp}_q"], g[f"{tag}_g{grp}_s"], g[f"{tag}_g{grp}_t"]
    _codes_match(q, want_q)
    diff = s != want_s
    if diff.any():
        steps = np.abs(s.view(np.int32).astype(np.int64) - want_s.view(np.int32).astype(np.int64))[diff]
        assert (steps == 0x10000).all()
        t = want_t[diff]
        lower = (t.view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)
        dist = np.minimum(t - lower, ref.bf16_up(t) - t) / t
        assert dist.max() <= 1e-5
        assert diff.mean() <= 1e-3


@pytest.mark.parametrize("lim", [7, 127])
def test_rowwise_quant_matches_reference(g, lim):
    q, s = ref.quant_rowwise(g["rowwise_in"], lim)
    _codes_match(q, g[f"rowwise_q{lim}"])
    # the reference divides by the limit, the production kernel multiplies by its reciprocal
    assert np.allclose(s, g[f"rowwise_s{lim}"], rtol=2e-7, atol=0)


def test_gemm_policies_match_reference(g):
    a, b = g["gemm_a"], g["gemm_b"]
    bias = ref.bf16_bits_to_f32(g["gemm_bias"])
    out0 = ref.linear_rowcol(a, g["gemm_p0_sa"], b, g["gemm_p0_sb"], bias)
    assert ref.rel_l2(g["gemm_p0_out"], out0) < 1e-6
    out4 = ref.linear_groupwise(a, g["gemm_p4_sa"], b, g["gemm_p4_sb"], bias, 128)
    assert ref.rel_l2(g["gemm_p4_out"], out4) < 1e-6


def test_weight_quant_matches_reference(g):
    w = g["wq_in"]
    q0, s0 = ref.weight_quant_convrot_rowwise(w, 256)
    _codes_match(q0, ref.unpack_int4_signed(g["wq_p0_packed"]))
    assert np.allclose(s0, g["wq_p0_scale"], rtol=1e-6)
    q4, s4 = ref.weight_quant_groupwise_bf16up(w, 256, 128)
    _codes_match(q4, ref.unpack_int4_signed(g["wq_p4_packed"]))
    assert (s4 != g["wq_p4_scale"]).mean() <= 1e-2


def test_affine_dequant_matches_reference(g):
    codes = g["awq_codes"]
    assert np.array_equal(ref.unpack_uint4(g["awq_qweight"]), codes)
    deq = ref.dequant_affine(codes, g["awq_scale"], g["awq_zeros"])
    assert np.allclose(deq, g["awq_deq_f32"], rtol=0, atol=1e-7)
    s = ref.bf16_bits_to_f32(g["awq_scale_bf16"])
    z = ref.bf16_bits_to_f32(g["awq_zeros_bf16"])
    # the reference chain evaluates in bf16: (q - 8) * s rounds once, + z rounds again
    n, k = codes.shape
    prod = ref.bf16_round(((codes.reshape(n, k // 64, 64) - 8).astype(np.float32) * s.T[:, :, None]))
    chain = ref.bf16_round(prod + z.T[:, :, None]).reshape(n, k)
    assert np.array_equal(ref.f32_to_bf16_bits(chain), g["awq_deq_bf16"])
    # and the exact formula is within the chain's two bf16 roundings of it
    exact = ref.dequant_affine(codes, s, z)
    mag = (np.abs(codes.reshape(n, k // 64, 64) - 8) * s.T[:, :, None] + np.abs(z.T[:, :, None])).reshape(n, k)
    assert (np.abs(exact - ref.bf16_bits_to_f32(g["awq_deq_bf16"])) <= 2 ** -7 * mag + 1e-12).all()


def test_formats_match_reference():
    from comfy_quant_bench_b200 import formats as F
    gold = json.load(open(os.path.join(GOLD, "formats_golden.json"), encoding="utf-8"))
    mine = {
        "ConvrotW4A4(convrot_groupsize=256, quant_group_size=64)": F.ConvrotW4A4(),
        "ConvrotW4A4(convrot_groupsize=64, quant_group_size=64)": F.ConvrotW4A4(convrot_groupsize=64),
        "AsymW4A8(group_size=16, convrot_groupsize=256, codebook=True)": F.AsymW4A8(),
        "AsymW4A8(group_size=16, convrot_groupsize=256, codebook=False)": F.AsymW4A8(codebook=False),
        "Int8Tensorwise(convrot=True, convrot_groupsize=256)": F.Int8Tensorwise(),
        "Int8Tensorwise(convrot=False, convrot_groupsize=256)": F.Int8Tensorwise(convrot=False),
        "AwqW4A16(group_size=32)": F.AwqW4A16(),
        "AwqW4A16(group_size=128)": F.AwqW4A16(group_size=128),
    }
    for key, fmt in mine.items():
        want = gold[key]
        assert fmt.layer_config() == want["layer_config"]
        for shape, ok in want["accepts"].items():
            assert fmt.accepts(json.loads(shape)) == ok, (key, shape)
        got = [[n, d, list(s)] for n, d, s in fmt.tensors("blocks.0.mlp.fc1.weight", [12288, 3072])]
        assert got == want["tensors"], key
    md = F.quant_metadata({"a": "b"}, {"blocks.0.mlp.fc1": F.ConvrotW4A4().layer_config()}, "convrot_w4a4",
                          {"x": "y"})
    assert md == gold["__metadata__"]
