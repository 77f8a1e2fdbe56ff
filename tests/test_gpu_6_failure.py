"""Failure detection on the GPU without a fault: a bounded wait that runs out records a status code, the kernel
returns, and the context stays usable. The test shortens every bounded wait (debug knob 1) and makes the wide GEMV's
producer withhold its copies (knob 2), so the consumers' stages never fill -- a flag that nothing sets."""
import numpy as np
import pytest
import torch

from oracle import codec, gemv as ogemv

pytestmark = pytest.mark.gpu
AIB_DEV_TIMEOUT_FULL, AIB_DEV_TIMEOUT_EMPTY = 101, 102


@pytest.fixture(scope="module")
def lib(cuda_dev):
    from ai_b200 import build, _lib
    build.build()
    return _lib.lib()


def test_gemv_wait_runs_out_reports_status_and_recovers(lib):
    from ai_b200 import wcomp, _lib
    g = np.random.default_rng(3)
    wb = codec.f32_to_bf16_bits((g.standard_normal((1024, 4096)) * 0.02).astype(np.float32))
    c = wcomp.compress(torch.from_numpy(wb.view(np.int16)).view(torch.bfloat16).cuda())
    x = torch.from_numpy(g.standard_normal(4096).astype(np.float32)).cuda()
    y = torch.zeros(1024, device="cuda")
    _lib.status(clear=True)
    _lib.call("aib_debug_knob", 1, 4096)
    _lib.call("aib_debug_knob", 2, 1)
    try:
        wcomp.gemvc1(x, c, y, 0)
        torch.cuda.synchronize()
        st = _lib.status(clear=True)
    finally:
        _lib.call("aib_debug_knob", 2, 0)
        _lib.call("aib_debug_knob", 1, 0)
    # whichever side gives up first records its code: the consumers (stage never filled) or the producer (slot
    # never released by consumers still waiting)
    assert st in (AIB_DEV_TIMEOUT_FULL, AIB_DEV_TIMEOUT_EMPTY)
    # the context is intact: the same call now returns the right product and no status
    wcomp.gemvc1(x, c, y, 0)
    torch.cuda.synchronize()
    W = codec.bf16_bits_to_f32(wb).astype(np.float64)
    xn = x.cpu().numpy().astype(np.float64)
    d = np.abs(y.cpu().numpy() - W @ xn)
    assert (d <= 2e-5 * (np.abs(W) @ np.abs(xn)) + 1e-6).all()
    assert _lib.status() == 0
