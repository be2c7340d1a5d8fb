"""The W4A8 linear entry point that allocates nothing (cq_linear_w4a8_affine_noalloc).

It exists for callers that cannot allocate device memory where they run the linear - a frozen or defragmenting
memory pool, allocator hooks that must not re-enter the allocator, plugins handed only input and output
buffers - and keeps its scratch in a fixed 32 MiB device array inside the library.  This test calls it through
the C ABI and checks it against cq_linear_w4a8_affine (caller workspace) on calls in a row with different shapes
and inputs (a tensor-core tile case, a few-token case, a SwiGLU-prologue case), so a later call cannot pass on
stale scratch from an earlier one.  Both entries launch the same kernels on the same inputs, so their outputs must
be bit-identical.  The file name sorts last so that a run stopping at the first failure has already run every
other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import ref

pytestmark = pytest.mark.gpu


def _bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from comfy_quant_bench_b200 import _lib
    return _lib.load()


def _problem(m, n, k, rot, seed, swiglu=0):
    from comfy_quant_bench_b200 import ops
    x = _bf16(ref.synth_activations(m, 2 * k if swiglu else k, seed=seed))
    w = torch.from_numpy(ref.synth_weight(n, k, seed=seed + 1)).cuda()
    qw, s, z = ops.quantize_affine_w4_weight(w, 128, rot)
    zt = ops.prepare_affine_zeros(z, 128)
    bias = _bf16(ref.synth_bias(n, seed=seed + 2))
    return x, qw, s, zt, bias


def _with_workspace(lib, x, qw, s, zt, bias, m, n, k, rot, swiglu=0):
    ws_bytes = int(lib.cq_linear_workspace_bytes(m, k))
    ws = torch.empty(ws_bytes + 256, dtype=torch.uint8, device="cuda")
    wp = (ws.data_ptr() + 255) // 256 * 256
    out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.cq_linear_w4a8_affine(x.data_ptr(), m, k, n, rot, swiglu, qw.data_ptr(), s.data_ptr(), zt.data_ptr(), 128,
                                   bias.data_ptr(), out.data_ptr(), wp, ws_bytes, st)
    assert rc == 0, rc
    return out


def _noalloc(lib, x, qw, s, zt, bias, m, n, k, rot, swiglu=0):
    out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.cq_linear_w4a8_affine_noalloc(x.data_ptr(), m, k, n, rot, swiglu, qw.data_ptr(), s.data_ptr(),
                                           zt.data_ptr(), 128, bias.data_ptr(), out.data_ptr(), st)
    assert rc == 0, rc
    return out


def test_noalloc_matches_workspace_entry_on_calls_in_a_row(lib):
    from comfy_quant_bench_b200 import _lib
    # (M, N, K, rotation group, seed, swiglu): tensor-core tiles with a partial last tile, the few-token (M <= 8)
    # product, the SwiGLU prologue, and the first shape again with new inputs
    cases = [(1000, 768, 3072, 256, 3, 0), (5, 384, 1024, 64, 7, 0), (300, 512, 2048, 256, 11, 1),
             (1000, 768, 3072, 256, 13, 0)]
    for m, n, k, rot, seed, swiglu in cases:
        x, qw, s, zt, bias = _problem(m, n, k, rot, seed, swiglu)
        got = _noalloc(lib, x, qw, s, zt, bias, m, n, k, rot, swiglu)
        want = _with_workspace(lib, x, qw, s, zt, bias, m, n, k, rot, swiglu)
        torch.cuda.synchronize()
        assert torch.isfinite(want.float()).all()
        assert torch.equal(got, want), (m, n, k, rot, swiglu)
    torch.cuda.synchronize()
    assert _lib.take_device_status() == (0, 0)


def test_noalloc_rejects_problems_larger_than_its_scratch(lib):
    from comfy_quant_bench_b200 import _lib
    vp = ctypes.c_void_p(256)
    # M = 16384 at K = 3072 needs more than the 32 MiB scratch array: refused before any launch
    rc = lib.cq_linear_w4a8_affine_noalloc(vp, 16384, 3072, 256, 256, 0, vp, vp, vp, 128, None, vp, None)
    assert rc == _lib.CQ_ERR_CAPACITY
