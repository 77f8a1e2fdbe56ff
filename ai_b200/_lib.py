"""ctypes binding of `libai_b200.so` (the C ABI declared in include/ai_b200.h).

There is no fallback: if the library is missing or fails to load, every call raises. Non-zero status codes
become exceptions (ValueError for bad arguments, like the reference launchers, RuntimeError otherwise).
"""
import ctypes as C
import os

from . import build as _build

LIB_PATH = _build.LIB

AIB_OK, AIB_EINVAL, AIB_ECUDA, AIB_EWORKSPACE, AIB_ENOTSUP, AIB_ESPACE = 0, -1, -2, -3, -4, -5

P = C.c_void_p
I32, I64, F32, SZ = C.c_int32, C.c_int64, C.c_float, C.c_size_t


class C12Desc(C.Structure):
    """Mirror of `aib_c12`."""
    _fields_ = [("m8", P), ("e4", P), ("rp", P), ("er", P), ("ec", P), ("ev", P), ("base", I32), ("N", I32),
                ("K", I32), ("CH", I32), ("n_exc", I64)]


class SampleParams(C.Structure):
    """Mirror of `aib_sample_params`."""
    _fields_ = [("temperature", F32), ("top_k", I32), ("top_p", F32), ("repetition_penalty", F32),
                ("presence_penalty", F32), ("frequency_penalty", F32)]


# name -> (restype, argtypes); every function declared in include/ai_b200.h
SIGNATURES = {
    "aib_abi_version": (I32, []),
    "aib_last_error": (C.c_char_p, []),
    "aib_set_pdl": (None, [I32]),
    "aib_status_read": (I32, [C.POINTER(I32), I32]),
    "aib_debug_knob": (I32, [I32, I32]),
    "aib_c12_encode_host": (I32, [P, I32, I32, P, P, P, P, P, P, P, P, I64]),
    "aib_c12_encode_workspace": (SZ, [I32]),
    "aib_c12_encode_planes": (I32, [P, I32, I32, P, P, P, P, P, SZ, P]),
    "aib_c12_encode_exceptions": (I32, [P, I32, I32, I32, P, P, P, P, P]),
    "aib_c12_decode": (I32, [C.POINTER(C12Desc), I32, I32, P, I32, P]),
    "aib_gemv_c12_workspace": (SZ, [C.POINTER(C12Desc), I32]),
    "aib_head8_tables": (I32, [P, I32, I32, P, P, P, P, P, P]),
    "aib_head8_workspace": (SZ, [I32, I32, I32]),
    "aib_head8_bounds": (I32, [P, I32, I32, P, P, P, P, P, I32, I32, P, I32, P, P, SZ, P]),
    "aib_head8_greedy": (I32, [P, I32, I32, C.POINTER(C12Desc), P, I32, P, P, P, SZ, P]),
    "aib_head8_bounds_topk": (I32, [P, I32, I32, P, P, P, P, P, I32, I32, P, I32, P, I32, P, SZ, P]),
    "aib_head8_candidate_logits": (I32, [P, I32, I32, C.POINTER(C12Desc), P, I32, P, P, I32, P, SZ, P]),
    "aib_head_exact_logits": (I32, [P, I32, I32, C.POINTER(C12Desc), P, I32, P]),
    "aib_gemv_c12": (I32, [C.POINTER(C12Desc), P, P, I32, I32, I32, I32, P, F32, P, SZ, P]),
    "aib_gemm_c12_workspace": (SZ, [I32, I32, I32]),
    "aib_gemm_c12": (I32, [C.POINTER(C12Desc), P, I32, I32, I32, P, F32, P, I32, I32, I32, P, SZ, P]),
    "aib_rmsnorm": (I32, [P, P, P, I32, I32, F32, P]),
    "aib_embed": (I32, [P, P, I32, I32, I32, P, P]),
    "aib_step_advance": (I32, [P, P, P, I32, P, I32, P]),
    "aib_batch_advance": (I32, [P, P, P, I32, P]),
    "aib_allreduce_oneshot": (I32, [P, I32, I32, P, P, I32, I32, P, P]),
    "aib_attn_workspace": (SZ, [I32, I32, I32, I32, I32]),
    "aib_rope_attn_decode": (I32, [P, P, P, P, P, P, P, P, I32, I32, I32, I32, F32, F32, P, SZ, P]),
    "aib_rope_attn_decode_noalloc": (I32, [P, P, P, P, P, P, P, P, I32, I32, I32, I32, F32, F32, P]),
    "aib_attn_batch_workspace": (SZ, [I32, I32, I32, I32, I32]),
    "aib_rope_attn_decode_batch": (I32, [P, I32, P, P, P, P, P, P, I64, P, I32, I32, I32, I32, I32, I32, F32, F32, P,
                                         SZ, P]),
    "aib_qk_rope_cache": (I32, [P, P, P, P, P, P, P, P, I32, I32, I32, I32, I32, F32, P]),
    "aib_attn_cached": (I32, [P, P, P, P, P, I32, I32, I32, I32, I32, F32, P, SZ, P]),
    "aib_attn_prefill": (I32, [P, P, P, P, I32, I32, I32, I32, I32, I32, F32, P]),
    "aib_sample_workspace": (SZ, [I32, I32]),
    "aib_sample": (I32, [P, I32, I32, I32, C.POINTER(SampleParams), P, I32, P, P, P, P, SZ, P]),
}

_lib = None


def lib():
    """Load (once) and return the CDLL with typed signatures. Raises if the library is unavailable."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m ai_b200.build` (no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        if L.aib_abi_version() != 1:
            raise RuntimeError("libai_b200.so ABI version mismatch")
        _lib = L
    return _lib


def check(rc, what=""):
    if rc == AIB_OK:
        return
    msg = lib().aib_last_error().decode(errors="replace")
    if rc == AIB_EINVAL:
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what} failed ({rc}): {msg}")


def call(name, *args):
    rc = getattr(lib(), name)(*args)
    check(rc, name)
    return rc


def status(clear=True):
    """Device status word (0 = no device-side failure)."""
    v = I32(0)
    call("aib_status_read", C.byref(v), 1 if clear else 0)
    return v.value


def ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def stream_ptr(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)
