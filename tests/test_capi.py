"""C-ABI checks that need no GPU: the library loads, exports every symbol the header declares, the host
encoder is bit-exact with the reference codec, and argument errors are reported without touching a device."""
import ctypes as C
import os
import re

import numpy as np
import pytest
import torch

from conftest import ROOT, golden, cases, cdict
from oracle import codec

HEADER = os.path.join(ROOT, "include", "ai_b200.h")


@pytest.fixture(scope="module")
def L():
    from ai_b200 import build, _lib
    build.build()
    return _lib.lib()


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(aib_[a-z0-9_]+)\s*\(", src)))


def test_header_symbols_exported(L):
    from ai_b200._lib import SIGNATURES
    names = declared()
    assert len(names) >= 18
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(SIGNATURES), set(names) ^ set(SIGNATURES)


def test_abi_version(L):
    assert L.aib_abi_version() == 1


@pytest.mark.parametrize("name", cases(golden("codec")))
def test_host_encoder_bit_exact(L, name):
    from ai_b200 import wcomp
    z = golden("codec")
    w = torch.from_numpy(z[f"{name}/w"].view(np.int16)).view(torch.bfloat16)
    c = wcomp.compress(w)  # CPU tensor -> host encoder of the library
    ref = cdict(z, f"{name}/")
    assert c["base"] == ref["base"]
    for k in ("m8", "e4", "rp", "er", "ec"):
        np.testing.assert_array_equal(c[k].numpy(), ref[k], err_msg=k)
    np.testing.assert_array_equal(c["ev"].numpy().view(np.uint32), ref["ev"].view(np.uint32))


def test_host_encoder_matches_oracle_random(L):
    from ai_b200 import wcomp
    g = torch.Generator().manual_seed(3)
    for N, K, s in ((33, 768, 0.02), (7, 256, 30.0), (128, 2048, 1e-3)):
        w = (torch.randn(N, K, generator=g) * s).bfloat16()
        c = wcomp.compress(w)
        o = codec.compress(w.view(torch.int16).numpy().view(np.uint16))
        assert c["base"] == o["base"]
        for k in ("m8", "e4", "rp", "er", "ec"):
            np.testing.assert_array_equal(c[k].numpy(), o[k])


def test_host_encoder_capacity_protocol(L):
    from ai_b200._lib import AIB_ESPACE
    w = np.zeros((2, 256), np.uint16)
    w[0, 3] = 0x7F80  # +inf: an exception
    m8 = np.zeros((2, 256), np.uint8)
    e4 = np.zeros((2, 128), np.uint8)
    rp = np.zeros(3, np.int32)
    base, n = C.c_int32(0), C.c_int64(0)
    p = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
    rc = L.aib_c12_encode_host(p(w), 2, 256, p(m8), p(e4), p(rp), C.byref(base), C.byref(n), None, None, None, 0)
    assert rc == AIB_ESPACE and n.value == 1 and rp[-1] == 1


def test_argument_errors_are_reported(L):
    from ai_b200._lib import C12Desc, AIB_EINVAL
    d = C12Desc()
    d.N, d.K, d.CH = 4, 300, 256  # K not a multiple of 256
    rc = L.aib_gemv_c12(C.byref(d), None, None, 1, 0, 0, 0, None, 1e-6, None, 0, None)
    assert rc == AIB_EINVAL
    assert b"null" in L.aib_last_error() or b"multiple" in L.aib_last_error()
    assert L.aib_rmsnorm(None, None, None, 1, 8, 1e-6, None) == AIB_EINVAL
    assert L.aib_sample(None, 1, 10, 10, None, None, 0, None, None, None, None, 0, None) == AIB_EINVAL


def test_wrappers_raise_value_error_like_reference(L):
    from ai_b200 import wcomp
    with pytest.raises(ValueError):
        wcomp.compress(torch.zeros(4, 100).bfloat16())
    with pytest.raises(ValueError):
        wcomp.compress(torch.zeros(4, 256))
