"""The allocation-free attention entry point, through the C ABI.

Callers that may not allocate device memory while running (an application embedding the library that
budgets all device memory itself, or a decode loop that must not enter cudaMalloc because it can stall the
device) use aib_rope_attn_decode_noalloc, whose scratch lives in a fixed array inside the library. This
checks it against aib_rope_attn_decode (caller-provided workspace) on two calls in a row, within the
tolerance of the other attention tests. The file is named so that pytest collects it last.
"""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _p(t):
    return C.c_void_p(t.data_ptr())


def test_noalloc_attention_matches_workspace_entry_point(cuda_dev):
    from ai_b200 import build, _lib
    build.build()
    L = _lib.lib()
    H, KV, HD, maxt, eps = 32, 8, 128, 640, 1e-6
    scale = HD ** -0.5
    g = torch.Generator(device="cuda").manual_seed(42)
    kc0 = torch.randn(KV, maxt, HD, generator=g, device="cuda").bfloat16()
    vc0 = torch.randn(KV, maxt, HD, generator=g, device="cuda").bfloat16()
    qn = (1 + 0.1 * torch.randn(HD, generator=g, device="cuda")).bfloat16()
    kn = (1 + 0.1 * torch.randn(HD, generator=g, device="cuda")).bfloat16()
    inv = (1.0 / (1e6 ** (torch.arange(0, HD, 2, dtype=torch.float32) / HD))).cuda()
    ws = torch.zeros(L.aib_attn_workspace(H, KV, HD, maxt, 1), dtype=torch.uint8, device="cuda")
    kc_a, vc_a = kc0.clone(), vc0.clone()  # workspace entry point
    kc_b, vc_b = kc0.clone(), vc0.clone()  # allocation-free entry point
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for step, p in enumerate((517, 518)):  # two calls in a row, the second sees the first one's K/V row
        qkv = torch.randn((H + 2 * KV) * HD, generator=g, device="cuda") * 2
        pos = torch.tensor([p], dtype=torch.int64, device="cuda")
        out_a = torch.zeros(H * HD, device="cuda")
        out_b = torch.full((H * HD,), float("nan"), device="cuda")
        rc = L.aib_rope_attn_decode(_p(qkv), _p(qn.view(torch.int16)), _p(kn.view(torch.int16)), _p(inv), _p(pos),
                                    _p(kc_a.view(torch.int16)), _p(vc_a.view(torch.int16)), _p(out_a), H, KV, HD,
                                    maxt, eps, scale, _p(ws), ws.numel(), stream)
        assert rc == 0, L.aib_last_error()
        rc = L.aib_rope_attn_decode_noalloc(_p(qkv), _p(qn.view(torch.int16)), _p(kn.view(torch.int16)), _p(inv),
                                            _p(pos), _p(kc_b.view(torch.int16)), _p(vc_b.view(torch.int16)),
                                            _p(out_b), H, KV, HD, maxt, eps, scale, stream)
        assert rc == 0, L.aib_last_error()
        torch.cuda.synchronize()
        np.testing.assert_allclose(out_b.cpu().numpy(), out_a.cpu().numpy(), rtol=2e-4, atol=2e-5,
                                   err_msg=f"call {step}")
        assert torch.equal(kc_b.view(torch.int16), kc_a.view(torch.int16))
        assert torch.equal(vc_b.view(torch.int16), vc_a.view(torch.int16))
    assert _lib.status() == 0


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda_dev):
    from ai_b200 import _lib
    L = _lib.lib()
    d = torch.zeros(16, device="cuda")
    # 2048 KV groups need more ticket counters and partials than the fixed scratch holds
    rc = L.aib_rope_attn_decode_noalloc(_p(d), _p(d), _p(d), _p(d), _p(d), _p(d), _p(d), _p(d), 2048, 2048, 128, 64,
                                        1e-6, 0.1, None)
    assert rc == _lib.AIB_EINVAL
    assert b"scratch" in L.aib_last_error()
