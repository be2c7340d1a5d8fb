"""The failure path on the GPU, without a fault: a wait that nothing satisfies gives up after the library's wait
limit, the device status word reports it (CQ_ERR_TIMEOUT and the waiting site), and the context stays usable."""
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_a_stuck_wait_surfaces_as_a_status_and_the_context_stays_usable():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from comfy_quant_bench_b200 import _lib, ops
    from oracle import ref
    torch.cuda.synchronize()
    assert _lib.take_device_status() == (0, 0)
    t0 = time.monotonic()
    _lib.call("cq_selftest_bounded_wait", None)
    torch.cuda.synchronize()
    elapsed = time.monotonic() - t0
    code, site = _lib.take_device_status()
    assert code == _lib.CQ_ERR_TIMEOUT and site in (90, 91)
    assert 1.5 < elapsed < 60.0
    assert _lib.take_device_status() == (0, 0), "reading the status clears it"
    # the next call works and is exact
    x = ref.synth_activations(64, 1024, seed=3)
    q, s, _ = ops.rotquant(torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda(), 256, _lib.CQ_ACT_INT8_ROW)
    qr, sr = ref.rotquant(x, 256, "int8")
    assert np.array_equal(q[:64].cpu().numpy(), qr.astype(np.int8))
    assert _lib.take_device_status() == (0, 0)
