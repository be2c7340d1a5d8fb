"""CPU-side checks of the C ABI: the library loads without a GPU, exports every symbol include/cq_b200.h
declares, and rejects bad arguments on the host before touching a device."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "cq_b200.h"), encoding="utf-8").read()
    return sorted(set(re.findall(r"CQ_API\s+[\w\s\*]+?\b(cq_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from comfy_quant_bench_b200 import _lib
    return _lib.load()


def test_header_and_binding_agree():
    from comfy_quant_bench_b200 import _lib
    assert _declared() == sorted(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    for name in _declared():
        assert hasattr(lib, name), name


def test_version_and_status_strings(lib):
    assert b"sm_100a" in lib.cq_version()
    assert lib.cq_status_string(0) == b"ok"
    assert lib.cq_status_string(2) == b"unsupported shape"


def test_host_side_argument_checks_need_no_device(lib):
    from comfy_quant_bench_b200 import _lib
    vp = ctypes.c_void_p(16)
    # K not a multiple of 256
    assert lib.cq_rotquant(vp, 4, 300, 256, 0, 0, 0, 4, 0, vp, vp, None, None) == _lib.CQ_ERR_SHAPE
    # bad rotation group
    assert lib.cq_rotquant(vp, 4, 512, 32, 0, 0, 0, 4, 0, vp, vp, None, None) == _lib.CQ_ERR_ARG
    # M_pad < M
    assert lib.cq_rotquant(vp, 8, 512, 256, 0, 0, 0, 4, 0, vp, vp, None, None) == _lib.CQ_ERR_SHAPE
    # per-group mode needs act_group 64/128
    assert lib.cq_rotquant(vp, 4, 512, 256, 0, 2, 32, 4, 0, vp, vp, None, None) == _lib.CQ_ERR_ARG
    # GEMM: K must be a multiple of 128; bad weight format
    assert lib.cq_gemm_rowcol(vp, 0, vp, vp, 0, vp, None, vp, 4, 8, 100, None) == _lib.CQ_ERR_SHAPE
    assert lib.cq_gemm_rowcol(vp, 0, vp, vp, 7, vp, None, vp, 4, 8, 128, None) == _lib.CQ_ERR_ARG
    # K-permuted activations only make sense with int4 weights
    assert lib.cq_gemm_rowcol(vp, 1, vp, vp, 1, vp, None, vp, 4, 8, 128, None) == _lib.CQ_ERR_ARG
    # affine: only group 128; the split group sums must be 16-byte aligned
    assert lib.cq_gemm_affine(vp, 0, vp, vp, vp, vp, vp, None, vp, 4, 8, 128, 64, None) == _lib.CQ_ERR_ARG
    assert lib.cq_gemm_affine(vp, 0, vp, ctypes.c_void_p(18), vp, vp, vp, None, vp, 4, 8, 128, 128, None) == \
        _lib.CQ_ERR_ALIGN
    assert lib.cq_group_sum_cols(3072) == 64 and lib.cq_group_sum_cols(4096) == 64
    assert lib.cq_group_sum_cols(4224) == 128 and lib.cq_group_sum_cols(12288) == 192
    # misaligned pointer
    assert lib.cq_gemm_rowcol(ctypes.c_void_p(17), 0, vp, vp, 0, vp, None, vp, 4, 8, 128, None) == _lib.CQ_ERR_ALIGN
    # empty problems are no-ops
    assert lib.cq_gemm_rowcol(None, 0, None, None, 0, None, None, None, 0, 8, 128, None) == _lib.CQ_OK
    # rotquant: K-permuted packed int4 output is not a layout
    assert lib.cq_rotquant(vp, 4, 512, 256, 0, 1, 0, 4, 2, vp, vp, None, None) == _lib.CQ_ERR_ARG
    # workspace sizing is pure arithmetic
    assert lib.cq_linear_workspace_bytes(4096, 3072) >= 4096 * 3072 + 4096 * 4
    assert lib.cq_linear_workspace_bytes(-1, 3072) == -1


def test_swiglu_output_argument_checks_need_no_device(lib):
    from comfy_quant_bench_b200 import _lib
    vp = ctypes.c_void_p(16)
    # whole 128-row weight tiles (N % 128); K a multiple of 128; activation bits 4 or 8
    assert lib.cq_gemm_rowcol_swiglu(vp, vp, vp, vp, None, vp, 4, 192, 256, None) == _lib.CQ_ERR_SHAPE
    assert lib.cq_gemm_rowcol_swiglu(vp, vp, vp, vp, None, vp, 4, 256, 100, None) == _lib.CQ_ERR_SHAPE
    assert lib.cq_gemm_rowcol_swiglu(vp, None, vp, vp, None, vp, 4, 256, 256, None) == _lib.CQ_ERR_ARG
    assert lib.cq_gemm_rowcol_swiglu(None, None, None, None, None, None, 0, 256, 256, None) == _lib.CQ_OK
    assert lib.cq_linear_convrot_w4a4_swiglu(vp, 4, 256, 256, 256, 5, vp, vp, None, vp, vp, 1 << 20, None) == \
        _lib.CQ_ERR_ARG
    # the N check comes before any work on the activations
    assert lib.cq_linear_convrot_w4a4_swiglu(vp, 4, 256, 192, 256, 4, vp, vp, None, vp, vp, 1 << 20, None) == \
        _lib.CQ_ERR_SHAPE
    # too small a workspace
    assert lib.cq_linear_convrot_w4a4_swiglu(vp, 4096, 256, 256, 256, 4, vp, vp, None, vp, vp, 64, None) != _lib.CQ_OK


def test_swiglu_output_rows_are_a_permutation_of_whole_groups():
    from comfy_quant_bench_b200 import ops
    idx = ops.swiglu_output_rows(384).tolist()
    assert sorted(idx) == list(range(384))
    for p, r in enumerate(idx):
        grp, i = divmod(p, 32)
        assert r == (16 * grp + i if i < 16 else 192 + 16 * grp + i - 16)
    with pytest.raises(ValueError):
        ops.swiglu_output_rows(192)


def test_prepare_swiglu_output_weight_permutes_rows_scales_and_bias_together():
    import torch
    from comfy_quant_bench_b200 import ops
    n, kh = 256, 64
    qw = torch.arange(n, dtype=torch.int8).reshape(n, 1).repeat(1, kh)   # row r holds r (mod 256) everywhere
    ws = torch.arange(n, dtype=torch.float32)
    bias = torch.arange(n, dtype=torch.float32).to(torch.bfloat16)
    q2, s2, b2 = ops.prepare_swiglu_output_weight(qw, ws, bias)
    idx = ops.swiglu_output_rows(n)
    assert torch.equal(q2, qw[idx]) and torch.equal(s2, ws[idx]) and torch.equal(b2, bias[idx])
    assert q2.is_contiguous() and s2.dtype == torch.float32 and b2.dtype == torch.bfloat16
    assert ops.prepare_swiglu_output_weight(qw, ws, None)[2] is None


def test_dit_glue_argument_checks_need_no_device(lib):
    from comfy_quant_bench_b200 import _lib
    vp = ctypes.c_void_p(16)
    f = ctypes.c_float(1e-6)
    # layer-norm prologue: K multiple of 256 and at most 24576; only CQ_Q_KPERM; negative eps; misaligned shift
    assert lib.cq_rotquant_lnmod(vp, 4, 300, 256, vp, vp, f, 4, 0, vp, vp, None, None) == _lib.CQ_ERR_SHAPE
    assert lib.cq_rotquant_lnmod(vp, 4, 32768, 256, vp, vp, f, 4, 0, vp, vp, None, None) == _lib.CQ_ERR_SHAPE
    assert lib.cq_rotquant_lnmod(vp, 4, 512, 256, vp, vp, f, 4, 1, vp, vp, None, None) == _lib.CQ_ERR_ARG
    assert lib.cq_rotquant_lnmod(vp, 4, 512, 256, vp, vp, ctypes.c_float(-1.0), 4, 0, vp, vp, None, None) == \
        _lib.CQ_ERR_ARG
    assert lib.cq_rotquant_lnmod(vp, 4, 512, 256, ctypes.c_void_p(18), vp, f, 4, 0, vp, vp, None, None) == \
        _lib.CQ_ERR_ALIGN
    assert lib.cq_rotquant_lnmod(vp, 4, 512, 256, None, vp, f, 4, 0, vp, vp, None, None) == _lib.CQ_ERR_ARG
    # q/k RMSNorm + rotary: head dim 64 or 128; the stream's tokens inside the joint sequence
    assert lib.cq_qkv_rmsnorm_rope(vp, 8, 4, 96, vp, vp, f, vp, vp, vp, vp, 8, 0, None) == _lib.CQ_ERR_SHAPE
    assert lib.cq_qkv_rmsnorm_rope(vp, 8, 4, 128, vp, vp, f, vp, vp, vp, vp, 10, 4, None) == _lib.CQ_ERR_SHAPE
    assert lib.cq_qkv_rmsnorm_rope(vp, 0, 4, 128, None, None, f, None, None, None, None, 10, 4, None) == _lib.CQ_OK
    assert lib.cq_qkv_rmsnorm_rope_layout(vp, 8, 4, 128, vp, vp, f, vp, vp, vp, vp, 8, 0, 2, None) == _lib.CQ_ERR_ARG
    assert lib.cq_qkv_rmsnorm_rope_layout(vp, 8, 4, 96, vp, vp, f, vp, vp, vp, vp, 8, 0, 1, None) == _lib.CQ_ERR_SHAPE
    # row RMSNorm + rotary: C a multiple of 8 up to 16384; with a rope table, head dim 64 or 128 dividing C
    assert lib.cq_rmsnorm_rope_rows(vp, 4, 1004, vp, f, None, 128, vp, None) == _lib.CQ_ERR_SHAPE
    assert lib.cq_rmsnorm_rope_rows(vp, 4, 32768, vp, f, None, 128, vp, None) == _lib.CQ_ERR_SHAPE
    assert lib.cq_rmsnorm_rope_rows(vp, 4, 3072, vp, f, ctypes.cast(vp, ctypes.POINTER(ctypes.c_float)), 96, vp,
                                    None) == _lib.CQ_ERR_SHAPE
    assert lib.cq_rmsnorm_rope_rows(vp, 4, 3072, vp, ctypes.c_float(-1.0), None, 128, vp, None) == _lib.CQ_ERR_ARG
    assert lib.cq_rmsnorm_rope_rows(ctypes.c_void_p(24), 4, 3072, vp, f, None, 128, vp, None) == _lib.CQ_ERR_ALIGN
    assert lib.cq_rmsnorm_rope_rows(None, 0, 3072, None, f, None, 128, None, None) == _lib.CQ_OK
    # head gather: 1..8 buffers, 16-byte aligned, columns inside the rows
    outs = (ctypes.c_void_p * 2)(16, 32)
    assert lib.cq_heads_to_rows(vp, 8, 4, 128, outs, 0, 0, 512, None) == _lib.CQ_ERR_ARG
    assert lib.cq_heads_to_rows(vp, 8, 4, 128, outs, 9, 0, 512, None) == _lib.CQ_ERR_ARG
    assert lib.cq_heads_to_rows(vp, 8, 4, 128, outs, 2, 8, 512, None) == _lib.CQ_ERR_SHAPE
    assert lib.cq_heads_to_rows(vp, 8, 4, 128, outs, 2, 4, 1024, None) == _lib.CQ_ERR_SHAPE
    bad = (ctypes.c_void_p * 2)(16, 40)
    assert lib.cq_heads_to_rows(vp, 8, 4, 128, bad, 2, 0, 512, None) == _lib.CQ_ERR_ALIGN


def test_dit_glue_ops_reject_bad_layouts_on_the_host():
    import torch
    from comfy_quant_bench_b200 import ops
    with pytest.raises(ValueError):
        ops.heads_to_rows(torch.zeros(2, 4, 8, 128, dtype=torch.bfloat16), [], 0, 512)   # CPU tensor
    with pytest.raises(ValueError):
        ops.qkv_rmsnorm_rope(torch.zeros(8, 1536, dtype=torch.bfloat16), torch.ones(128), torch.ones(128),
                             torch.zeros(8, 64, 2), torch.zeros(1, 4, 8, 128), torch.zeros(1, 4, 8, 128),
                             torch.zeros(1, 4, 8, 128), 0)


def test_python_errors_map_to_exceptions():
    from comfy_quant_bench_b200 import _lib
    with pytest.raises(_lib.CQShapeError):
        _lib.check("cq_rotquant", _lib.CQ_ERR_SHAPE)
    with pytest.raises(_lib.CQError):
        _lib.check("cq_gemm_rowcol", _lib.CQ_ERR_TIMEOUT)
    _lib.check("x", _lib.CQ_OK)


def test_ops_reject_cpu_tensors():
    import torch
    from comfy_quant_bench_b200 import ops
    with pytest.raises(ValueError, match="no CPU fallback"):
        ops.quantize_int4_rowwise_convrot64(torch.zeros(2, 256, dtype=torch.bfloat16))
