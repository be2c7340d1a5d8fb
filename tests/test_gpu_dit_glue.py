"""DiT-step glue kernels against the torch ops they replace (bf16 tensors on the GPU).

* ``qkv_rmsnorm_rope``: per-head RMSNorm of q and k (fp32, one bf16 rounding), rotary rotation of interleaved pairs
  (fp32, one bf16 rounding), and the joint [1, H, S_all, D] attention layout.  v is a pure copy (bit-exact); q and k
  may differ from the torch composite by one bf16 rounding where fp32 summation order differs.
* ``rotquant_lnmod`` / ``w4a8_affine_linear_lnmod``: the modulated layer norm bf16(shift + bf16(LN(x)) * scale1p)
  formed inside the activation kernel.  Its mean and variance are summed in a different order than torch's Welford
  kernel, so a normalized value can land one bf16 rounding away; the codes then differ by at most 1 at a few
  positions and the linear's output agrees to rel-L2 <= 1e-3 (the bounds written below).
"""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from comfy_quant_bench_b200 import ops as _ops, _lib
    _lib.load()
    return _ops


def _status_clear():
    from comfy_quant_bench_b200 import _lib
    torch.cuda.synchronize()
    assert _lib.take_device_status() == (0, 0)


def _rope_table(n, d, offset, device):
    inv = 1.0 / (10000.0 ** (torch.arange(0, d, 2, device=device, dtype=torch.float32) / d))
    ang = torch.outer(torch.arange(offset, offset + n, device=device, dtype=torch.float32), inv)
    return torch.complex(torch.cos(ang), torch.sin(ang))


def _torch_rope(x, rot):
    xc = torch.view_as_complex(x.float().reshape(*x.shape[:-1], -1, 2))
    return torch.view_as_real(xc * rot[:, None, :]).reshape(x.shape).to(torch.bfloat16)


def _within_one_rounding(got, want):
    g, w = got.float(), want.float()
    tol = w.abs() * 2.0 ** -7 + 1e-6
    assert bool(((g - w).abs() <= tol).all()), float(((g - w).abs() - tol).max())
    assert float((g != w).float().mean()) <= 0.02


def _qkv_buffers(h, s_all, d, token_major):
    if token_major:   # [1, S_all, H, D] memory seen as [1, H, S_all, D]
        return tuple(torch.full((1, s_all, h, d), 3.0, dtype=torch.bfloat16, device="cuda").transpose(1, 2)
                     for _ in range(3))
    return tuple(torch.full((1, h, s_all, d), 3.0, dtype=torch.bfloat16, device="cuda") for _ in range(3))


@pytest.mark.parametrize("token_major", [False, True])
@pytest.mark.parametrize("s,h,d,s0,s_all", [(300, 24, 128, 40, 345), (17, 4, 64, 0, 17)])
def test_qkv_rmsnorm_rope_matches_torch(ops, s, h, d, s0, s_all, token_major):
    g = torch.Generator(device="cuda").manual_seed(s + h)
    y = torch.randn(s, 3 * h * d, generator=g, device="cuda").to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(d, generator=g, device="cuda")).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(d, generator=g, device="cuda")).to(torch.bfloat16)
    rot = _rope_table(s, d, s0, "cuda")
    q, k, v = _qkv_buffers(h, s_all, d, token_major)
    ops.qkv_rmsnorm_rope(y, qn, kn, rot, q, k, v, s0, eps=1e-6)
    yv = y.view(s, 3, h, d)
    want_q = _torch_rope(F.rms_norm(yv[:, 0], (d,), qn, eps=1e-6), rot).transpose(0, 1)
    want_k = _torch_rope(F.rms_norm(yv[:, 1], (d,), kn, eps=1e-6), rot).transpose(0, 1)
    _status_clear()
    assert torch.equal(v[0, :, s0:s0 + s], yv[:, 2].transpose(0, 1))
    _within_one_rounding(q[0, :, s0:s0 + s], want_q)
    _within_one_rounding(k[0, :, s0:s0 + s], want_k)
    for t in (q, k, v):   # tokens of the other stream are untouched
        assert bool((t[0, :, :s0] == 3.0).all()) and bool((t[0, :, s0 + s:] == 3.0).all())


def test_qkv_token_major_equals_head_major_and_attention_output_is_rows(ops):
    """The token-major layout holds the same values as the head-major one, and the attention over strided
    token-major views returns [tokens, hidden] rows equal to the head-major attention's output transposed."""
    s, h, d = 272, 8, 128
    g = torch.Generator(device="cuda").manual_seed(7)
    y = torch.randn(s, 3 * h * d, generator=g, device="cuda").to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(d, generator=g, device="cuda")).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(d, generator=g, device="cuda")).to(torch.bfloat16)
    rot = _rope_table(s, d, 0, "cuda")
    hm = _qkv_buffers(h, s, d, False)
    tm = _qkv_buffers(h, s, d, True)
    ops.qkv_rmsnorm_rope(y, qn, kn, rot, *hm, 0, eps=1e-6)
    ops.qkv_rmsnorm_rope(y, qn, kn, rot, *tm, 0, eps=1e-6)
    _status_clear()
    for a, b in zip(hm, tm):
        assert torch.equal(a, b)
    o_hm = F.scaled_dot_product_attention(*hm)
    o_tm = F.scaled_dot_product_attention(*tm)
    rows = torch.empty(s, h * d, dtype=torch.bfloat16, device="cuda")
    ops.heads_to_rows(o_hm, [rows], 0, h * d)
    _status_clear()
    got = o_tm.transpose(1, 2).reshape(s, h * d)
    assert (got - rows).abs().max().item() <= 2.0 ** -6 * rows.abs().max().item()


@pytest.mark.parametrize("s,c,d,with_rope,in_place", [(300, 3072, 128, True, False), (300, 3072, 128, False, True),
                                                        (37, 5120, 128, True, True), (9, 512, 64, True, False),
                                                        (5, 16384, 128, False, False)])
def test_rmsnorm_rope_rows_matches_torch(ops, s, c, d, with_rope, in_place):
    """RMSNorm over whole rows (Wan's q/k norm over the hidden dim) then the rotary embedding, against torch's
    rms_norm and the complex multiply: within one bf16 rounding."""
    g = torch.Generator(device="cuda").manual_seed(s + c)
    x = (torch.randn(s, c, generator=g, device="cuda") * 3.0).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(c, generator=g, device="cuda")).to(torch.bfloat16)
    rot = _rope_table(s, d, 5, "cuda") if with_rope else None
    want = F.rms_norm(x, (c,), w, eps=1e-6)
    if with_rope:
        want = _torch_rope(want.view(s, c // d, d), rot).view(s, c)
    src = x.clone()
    got = ops.rmsnorm_rope_rows(src, w, rot, d, eps=1e-6, out=src if in_place else None)
    _status_clear()
    if in_place:
        assert got.data_ptr() == src.data_ptr()
    _within_one_rounding(got, want)


def test_rmsnorm_rope_rows_rejects_bad_arguments(ops):
    from comfy_quant_bench_b200 import _lib
    w = torch.ones(1004, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.CQShapeError):          # C not a multiple of 8
        ops.rmsnorm_rope_rows(torch.zeros(4, 1004, dtype=torch.bfloat16, device="cuda"), w)
    w = torch.ones(3072, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):                  # rope table of the wrong length
        ops.rmsnorm_rope_rows(torch.zeros(4, 3072, dtype=torch.bfloat16, device="cuda"), w,
                              torch.zeros(5, 64, 2, device="cuda"), 128)
    with pytest.raises(ValueError):                  # weight length
        ops.rmsnorm_rope_rows(torch.zeros(4, 3072, dtype=torch.bfloat16, device="cuda"), w[:100])


def test_qkv_rejects_mixed_layouts(ops):
    s, h, d = 16, 2, 64
    y = torch.zeros(s, 3 * h * d, dtype=torch.bfloat16, device="cuda")
    w = torch.ones(d, dtype=torch.bfloat16, device="cuda")
    rot = _rope_table(s, d, 0, "cuda")
    (q, _, _), (_, k, v) = _qkv_buffers(h, s, d, False), _qkv_buffers(h, s, d, True)
    with pytest.raises(ValueError):
        ops.qkv_rmsnorm_rope(y, w, w, rot, q, k, v, 0)


def _lnmod_inputs(m, k, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(m, k, generator=g, device="cuda")
    x[:, torch.randperm(k, generator=g, device="cuda")[: k // 100]] *= 20.0   # outlier channels
    x = (x + 0.5).to(torch.bfloat16)
    shift = (0.3 * torch.randn(k, generator=g, device="cuda")).to(torch.bfloat16)
    scale1p = (1.0 + 0.3 * torch.randn(k, generator=g, device="cuda")).to(torch.bfloat16)
    return x, shift, scale1p


def _torch_lnmod(x, shift, scale1p):
    return torch.addcmul(shift, F.layer_norm(x, (x.shape[-1],), eps=1e-6), scale1p)


@pytest.mark.parametrize("m,k,rot,m_pad", [(300, 3072, 256, 304), (37, 1024, 64, 37), (8, 12288, 256, 16),
                                           (5, 768, 0, 8)])
def test_rotquant_lnmod_matches_torch_composite(ops, m, k, rot, m_pad):
    from comfy_quant_bench_b200 import _lib
    x, shift, scale1p = _lnmod_inputs(m, k, seed=m + k)
    q, s, gs = ops.rotquant_lnmod(x, rot, shift, scale1p, m_pad=m_pad, group_sums=True, kperm=True)
    qr, sr, gr = ops.rotquant(_torch_lnmod(x, shift, scale1p), rot, _lib.CQ_ACT_INT8_ROW, m_pad=m_pad,
                              group_sums=True, kperm=True)
    _status_clear()
    d = (q[:m].int() - qr[:m].int()).abs()
    assert int(d.max()) <= 1 and float((d > 0).float().mean()) <= 1e-3
    assert float(((s[:m] - sr[:m]).abs() / sr[:m]).max()) <= 1e-3
    assert float((gs[:m].float() - gr[:m].float()).abs().max()) <= 128.0   # split sums of codes within +-1
    assert not q[m:].any() and not s[m:].any() and not gs[m:].float().any()


def test_w4a8_affine_linear_lnmod_matches_composite(ops):
    m, k, n = 257, 3072, 1024
    x, shift, scale1p = _lnmod_inputs(m, k, seed=3)
    w = torch.randn(n, k, device="cuda", generator=torch.Generator(device="cuda").manual_seed(4)) * 0.02
    qw, sc, z = ops.quantize_affine_w4_weight(w, 128, 256)
    zt = ops.prepare_affine_zeros(z, 128)
    bias = (0.01 * torch.randn(n, device="cuda")).to(torch.bfloat16)
    got = ops.w4a8_affine_linear_lnmod(x, shift, scale1p, qw, sc, zt, bias, 128, 256)
    want = ops.w4a8_affine_linear(_torch_lnmod(x, shift, scale1p), qw, sc, z, bias, 128, 256, zeros_prepared=zt)
    _status_clear()
    rel = float((got.float() - want.float()).norm() / want.float().norm())
    assert rel <= 1e-3, rel


def test_dit_glue_rejects_bad_arguments(ops):
    from comfy_quant_bench_b200 import _lib
    x = torch.zeros(4, 1000, dtype=torch.bfloat16, device="cuda")       # K not a multiple of 256
    v = torch.zeros(1000, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.CQShapeError):
        ops.rotquant_lnmod(x, 256, v, v)
    with pytest.raises(ValueError):
        ops.rotquant_lnmod(torch.zeros(4, 1024, dtype=torch.bfloat16, device="cuda"), 256, v, v)   # wrong length
    y = torch.zeros(8, 3 * 2 * 96, dtype=torch.bfloat16, device="cuda")   # head dim 96: not supported
    q = torch.zeros(1, 2, 8, 96, dtype=torch.bfloat16, device="cuda")
    w = torch.ones(96, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.CQShapeError):
        ops.qkv_rmsnorm_rope(y, w, w, torch.zeros(8, 48, 2, device="cuda"), q, q.clone(), q.clone(), 0)


# ----------------------------------------------------------------------------------------------
# output operations in the W4A8 affine GEMM's epilogue (GELU-tanh, gated residual)
# ----------------------------------------------------------------------------------------------

def _affine_layer(n, k, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randn(n, k, device="cuda", generator=g) * 0.02
    from comfy_quant_bench_b200 import ops as _ops
    qw, sc, z = _ops.quantize_affine_w4_weight(w, 128, 256)
    bias = (0.01 * torch.randn(n, device="cuda", generator=g)).to(torch.bfloat16)
    return qw, sc, z, _ops.prepare_affine_zeros(z, 128), bias


def _plain_via_gemm(ops, x, qw, sc, z, zt, bias):
    """The plain linear's bf16 output through the tensor-core GEMM: inputs of eight tokens or fewer take the
    few-token product, whose fp32 summation order differs, so they are padded to 16 rows and sliced."""
    m = x.shape[0]
    xp = torch.cat([x, torch.zeros(16 - m, x.shape[1], dtype=x.dtype, device=x.device)]) if m < 16 else x
    return ops.w4a8_affine_linear(xp, qw, sc, z, bias, 128, 256, zeros_prepared=zt)[:m]


@pytest.fixture(params=["one_sm", "pair"])
def gemm_variant(request, ops):
    """Runs a test once per kernel form of the int4-weight GEMM (one CTA per tile, or a CTA pair per tile)."""
    from comfy_quant_bench_b200 import _lib
    _lib.set_gemm_variant(_lib.CQ_GEMM_ONE_SM if request.param == "one_sm" else _lib.CQ_GEMM_PAIR)
    yield request.param
    _lib.set_gemm_variant(_lib.CQ_GEMM_AUTO)


# (M, N, K): the MMDiT image-stream MLP-up shape, a text-stream shape, ragged M with N a multiple of 64 / of 32 only,
# a few tokens (the GEMM, not the few-token product, applies the operation), N a multiple of 8 only
_OP_SHAPES = [(4096, 12288, 3072), (256, 3072, 3072), (300, 384, 1024), (77, 416, 1024), (5, 256, 1024), (33, 264, 512)]


@pytest.mark.parametrize("m,n,k", _OP_SHAPES)
def test_gelu_output_matches_torch_gelu_of_the_linear(ops, gemm_variant, m, n, k):
    """out = bf16(gelu_tanh(y)) on y, the plain linear's bf16 output: torch's F.gelu(y, approximate="tanh") up to
    a few fp32 ulp before the bf16 rounding (the logistic form of tanh), so at most one bf16 rounding apart."""
    g = torch.Generator(device="cuda").manual_seed(m + n)
    x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    qw, sc, z, zt, bias = _affine_layer(n, k, seed=n)
    y = _plain_via_gemm(ops, x, qw, sc, z, zt, bias)
    got = ops.w4a8_affine_linear_op(x, qw, sc, zt, bias, out_op="gelu", convrot_groupsize=256)
    _status_clear()
    _within_one_rounding(got, F.gelu(y, approximate="tanh"))
    assert float((got != F.gelu(y, approximate="tanh")).float().mean()) <= 2e-3


@pytest.mark.parametrize("m,n,k", _OP_SHAPES)
def test_gated_residual_output_matches_addcmul(ops, gemm_variant, m, n, k):
    """out = bf16(residual + gate * y): torch.addcmul(residual, gate, y) on the plain linear's bf16 output.  The
    epilogue rounds the exact value once (packed bf16 fused multiply-add) where torch rounds an fp32 result to bf16,
    so the two differ only where that fp32 value lands on a bf16 rounding tie (about 2^-16 of the outputs, by one
    step); also in place (out is the residual) and with a residual whose rows are strided (a column slice of a wider
    tensor), both bit-identical to the plain call."""
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n)
    x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    qw, sc, z, zt, bias = _affine_layer(n, k, seed=n + 1)
    res = torch.randn(m, n, device="cuda", generator=g).to(torch.bfloat16)
    gate = torch.randn(1, n, device="cuda", generator=g).to(torch.bfloat16)
    y = _plain_via_gemm(ops, x, qw, sc, z, zt, bias)
    want = torch.addcmul(res, gate, y)
    got = ops.w4a8_affine_linear_op(x, qw, sc, zt, bias, out_op="gated", residual=res, gate=gate, convrot_groupsize=256)
    wide = torch.randn(m, n + 64, device="cuda", generator=g).to(torch.bfloat16)
    wide[:, 16:16 + n] = res
    got_strided = ops.w4a8_affine_linear_op(x, qw, sc, zt, bias, out_op="gated", residual=wide[:, 16:16 + n],
                                            gate=gate, convrot_groupsize=256)
    inplace = res.clone()
    ops.w4a8_affine_linear_op(x, qw, sc, zt, bias, out_op="gated", residual=inplace, gate=gate, out=inplace,
                              convrot_groupsize=256)
    _status_clear()
    g, w = got.float(), want.float()
    assert bool(((g - w).abs() <= w.abs() * 2.0 ** -7 + 1e-30).all())
    assert float((got != want).float().mean()) <= 1e-4
    assert torch.equal(got_strided, got)
    assert torch.equal(inplace, got)


def test_lnmod_gelu_output_matches_composite(ops, gemm_variant):
    """The MLP-up linear of a DiT block in one call: layer norm + modulation (with the bf16 1 + scale formed in the
    activation kernel) and GELU in the GEMM epilogue, against F.gelu of w4a8_affine_linear_lnmod with torch's
    1 + scale."""
    m, k, n = 1024, 3072, 12288
    x, shift, _ = _lnmod_inputs(m, k, seed=9)
    scale = (0.3 * torch.randn(k, device="cuda", generator=torch.Generator(device="cuda").manual_seed(8))).to(torch.bfloat16)
    qw, sc, z, zt, bias = _affine_layer(n, k, seed=10)
    want = F.gelu(ops.w4a8_affine_linear_lnmod(x, shift, 1.0 + scale, qw, sc, zt, bias, 128, 256), approximate="tanh")
    got = ops.w4a8_affine_linear_op(x, qw, sc, zt, bias, out_op="gelu", shift=shift, scale=scale,
                                    convrot_groupsize=256)
    plain = ops.w4a8_affine_linear_op(x, qw, sc, zt, bias, shift=shift, scale=scale, convrot_groupsize=256)
    assert torch.equal(plain, ops.w4a8_affine_linear_lnmod(x, shift, 1.0 + scale, qw, sc, zt, bias, 128, 256))
    _status_clear()
    _within_one_rounding(got, want)
    assert float((got != want).float().mean()) <= 2e-3


def test_output_op_rejects_bad_arguments(ops):
    from comfy_quant_bench_b200 import _lib
    m, n, k = 64, 256, 512
    x = torch.zeros(m, k, dtype=torch.bfloat16, device="cuda")
    qw, sc, z, zt, bias = _affine_layer(n, k, seed=11)
    res = torch.zeros(m, n, dtype=torch.bfloat16, device="cuda")
    gate = torch.zeros(n, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):            # gated without a residual
        ops.w4a8_affine_linear_op(x, qw, sc, zt, bias, out_op="gated", gate=gate)
    with pytest.raises(ValueError):            # unknown operation
        ops.w4a8_affine_linear_op(x, qw, sc, zt, bias, out_op="relu")
    out = torch.zeros(m + 1, n, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.CQShapeError):     # residual overlaps the output without being it
        ops.w4a8_affine_linear_op(x, qw, sc, zt, bias, out_op="gated", residual=out[1:], gate=gate, out=out[:m])
    x196 = torch.zeros(m, k, dtype=torch.bfloat16, device="cuda")
    qw2, sc2, z2, zt2, b2 = _affine_layer(196, k, seed=12)
    with pytest.raises(_lib.CQShapeError):     # N not a multiple of 8: the operations need the staged stores
        ops.w4a8_affine_linear_op(x196, qw2, sc2, zt2, b2, out_op="gelu")
    op = _lib.CQOutOp(7, None, 0, None)         # kind out of range, through the C ABI
    ws = torch.empty(_lib.load().cq_linear_workspace_bytes(m, k), dtype=torch.uint8, device="cuda")
    st = _lib.load().cq_linear_w4a8_op(x.data_ptr(), m, k, n, 256, None, None, 1e-6, qw.data_ptr(), sc.data_ptr(),
                                        zt.data_ptr(), 128, bias.data_ptr(), _lib.ctypes.byref(op), res.data_ptr(),
                                        ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert st == _lib.CQ_ERR_ARG
    _status_clear()


# ----------------------------------------------------------------------------------------------
# few-token-tile affine GEMMs split over K (a DiT's text stream: one 256-token tile)
# ----------------------------------------------------------------------------------------------

@pytest.mark.parametrize("m,n,k,out_op", [(256, 3072, 12288, "gated"), (256, 3072, 3072, "plain"), (300, 3072, 3072, "gelu"),
                                          (256, 9216, 3072, "plain")])
def test_split_k_linear_matches_the_unsplit_gemm(ops, m, n, k, out_op):
    """With room for the partial sums (the workspace the ops allocate), the linear splits K over more CTAs and adds the
    partial tiles in a fixed order: deterministic, equal to the unsplit GEMM (the standalone cq_gemm_affine on the
    same codes) up to fp32 summation order (within one bf16 step, a small fraction off), and to the oracle-free
    composite for the output operations."""
    from comfy_quant_bench_b200 import _lib
    lib = _lib.load()
    assert lib.cq_linear_workspace_bytes_n(m, k, n) > lib.cq_linear_workspace_bytes(m, k)   # this shape splits
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    qw, sc, z, zt, bias = _affine_layer(n, k, seed=n + k)
    res = torch.randn(m, n, device="cuda", generator=g).to(torch.bfloat16)
    gate = torch.randn(n, device="cuda", generator=g).to(torch.bfloat16)
    kw = {"residual": res, "gate": gate} if out_op == "gated" else {}
    y1 = ops.w4a8_affine_linear_op(x, qw, sc, zt, bias, out_op=out_op, convrot_groupsize=256, **kw)
    y2 = ops.w4a8_affine_linear_op(x, qw, sc, zt, bias, out_op=out_op, convrot_groupsize=256, **kw)
    q, s, gs = ops.rotquant(x, 256, _lib.CQ_ACT_INT8_ROW, m_pad=(m + 15) // 16 * 16, group_sums=True, kperm=True)
    unsplit = ops.gemm_affine(q[:m], s[:m], gs, qw, sc, z, bias, a_kperm=True, zeros_prepared=zt)
    if out_op == "gelu":
        want = F.gelu(unsplit, approximate="tanh")
    elif out_op == "gated":
        want = torch.addcmul(res, gate, unsplit)
    else:
        want = unsplit
    _status_clear()
    assert torch.equal(y1, y2)
    a, b = y1.float(), want.float()
    assert bool(((a - b).abs() <= b.abs() * 2.0 ** -7 + 1e-6).all()), float(((a - b).abs() - b.abs() * 2.0 ** -7).max())
    assert float((y1 != want).float().mean()) <= 0.02


# ----------------------------------------------------------------------------------------------
# output operations and the modulated layer norm on the row/col linears (ConvRot W4A4, W8A8)
# ----------------------------------------------------------------------------------------------

def _rowcol_layer(ops, kind, n, k, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randn(n, k, device="cuda", generator=g) * 0.02
    bias = (0.01 * torch.randn(n, device="cuda", generator=g)).to(torch.bfloat16)
    if kind == "w8a8":
        qw, ws = ops.quantize_int8_convrot_weight(w, 0)
        return (lambda x: ops.int8_linear(x, qw, ws, bias),
                lambda x, out_op, **kw: ops.int8_linear_op(x, qw, ws, bias, out_op=out_op, **kw))
    qw, ws = ops.quantize_convrot_w4a4_weight(w, 64)
    dt = "int4" if kind == "w4a4" else "int8"
    return (lambda x: ops.convrot_w4a4_linear(x, qw, ws, bias, convrot_groupsize=64, linear_dtype=dt),
            lambda x, out_op, **kw: ops.convrot_w4a4_linear_op(x, qw, ws, bias, out_op=out_op, convrot_groupsize=64,
                                                               linear_dtype=dt, **kw))


_ROWCOL_SHAPES = [(4096, 3072, 3072), (300, 384, 1024), (77, 416, 1024), (33, 264, 512)]


@pytest.mark.parametrize("kind", ["w4a4", "w4a4_int8act", "w8a8"])
@pytest.mark.parametrize("m,n,k", _ROWCOL_SHAPES)
def test_rowcol_output_ops_match_torch(ops, gemm_variant, kind, m, n, k):
    """The row/col linears' epilogue operations on y, the plain linear's bf16 output: plain is y bit for bit, GELU
    is F.gelu(y, approximate="tanh") within one bf16 rounding, the gated residual is torch.addcmul(residual, gate, y)
    but at bf16 rounding ties (also in place, bit-identical)."""
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    plain, op = _rowcol_layer(ops, kind, n, k, seed=n + 3)
    y = plain(x)
    assert torch.equal(op(x, "plain"), y)
    got = op(x, "gelu")
    res = torch.randn(m, n, device="cuda", generator=g).to(torch.bfloat16)
    gate = torch.randn(n, device="cuda", generator=g).to(torch.bfloat16)
    gated = op(x, "gated", residual=res, gate=gate)
    inplace = res.clone()
    op(x, "gated", residual=inplace, gate=gate, out=inplace)
    _status_clear()
    want_gelu = F.gelu(y, approximate="tanh")
    _within_one_rounding(got, want_gelu)
    assert float((got != want_gelu).float().mean()) <= 2e-3
    want = torch.addcmul(res, gate, y)
    gf, wf = gated.float(), want.float()
    assert bool(((gf - wf).abs() <= wf.abs() * 2.0 ** -7 + 1e-30).all())
    assert float((gated != want).float().mean()) <= 1e-4
    assert torch.equal(inplace, gated)


@pytest.mark.parametrize("kind", ["w4a4", "w8a8"])
def test_rowcol_lnmod_prologue_matches_composite(ops, gemm_variant, kind):
    """The modulated layer norm formed in the activation kernel of a row/col linear, against the plain linear of
    torch's composite bf16(shift + bf16(layer_norm(x)) * bf16(1 + scale)): the activation codes may differ by one
    where the composite's two bf16 roundings land differently, so the outputs agree to rel-L2 1e-3."""
    m, k, n = 1024, 3072, 3072
    x, shift, _ = _lnmod_inputs(m, k, seed=21)
    scale = (0.3 * torch.randn(k, device="cuda", generator=torch.Generator(device="cuda").manual_seed(22))).to(torch.bfloat16)
    plain, op = _rowcol_layer(ops, kind, n, k, seed=23)
    want = plain(_torch_lnmod(x, shift, 1.0 + scale))
    got = op(x, "plain", shift=shift, scale=scale)
    got_gelu = op(x, "gelu", shift=shift, scale=scale)
    _status_clear()
    from comfy_quant_bench_b200.mmdit import rel_l2
    assert rel_l2(got, want) <= 1e-3
    _within_one_rounding(got_gelu, F.gelu(got, approximate="tanh"))


def test_rowcol_op_rejects_bad_arguments(ops):
    plain, op = _rowcol_layer(ops, "w8a8", 264, 512, seed=1)
    x = torch.zeros(8, 512, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        op(x, "gated")                                   # no residual / gate
    with pytest.raises(ValueError):
        op(x, "relu")
    with pytest.raises(ValueError):
        op(x, "plain", shift=torch.zeros(512, dtype=torch.bfloat16, device="cuda"))   # shift without scale
