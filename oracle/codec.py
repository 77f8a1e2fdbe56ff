"""12-bit lossless bf16 codec, numpy restatement (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py).

Follows `ramvi/engine/ramvi_engine/kernels/wcomp.py`:
  compress   :13-32   decompress :35-45   _dec :48-54
and the row-block decoder `kernels/prefill.py:23-42` (`weight_rows`) / `prefill_kernels.py:59-110`.
"""
import numpy as np


def compress(w_bits, CH=256):
    """w_bits: uint16 [N, K] (bf16 bit patterns) -> dict like the reference `compress` (wcomp.py:13-32)."""
    w_bits = np.ascontiguousarray(w_bits, dtype=np.uint16)
    N, K = w_bits.shape
    assert K % CH == 0
    b = w_bits.astype(np.int32)
    e = (b >> 7) & 0xFF                                        # wcomp.py:18
    cnt = np.bincount(e.ravel(), minlength=256).astype(np.int64)
    cs = np.concatenate([[0], np.cumsum(cnt)])                 # wcomp.py:20
    base = int(np.argmax(cs[15:] - cs[:-15]))                  # wcomp.py:21 (first window wins ties)
    code = e - base
    exc = (code < 0) | (code > 14)                             # wcomp.py:23
    code = np.where(exc, 15, code)
    m8 = (((b >> 15) << 7) | (b & 0x7F)).astype(np.uint8)      # wcomp.py:25
    c = code.reshape(N, K // CH, 2, CH // 2)
    e4 = (c[:, :, 0] | (c[:, :, 1] << 4)).astype(np.uint8).reshape(N, K // 2)  # wcomp.py:26-27
    r, col = np.nonzero(exc)                                   # row-major order (wcomp.py:28)
    rp = np.zeros(N + 1, np.int32)
    rp[1:] = np.cumsum(np.bincount(r, minlength=N))
    ev = bf16_bits_to_f32(w_bits[r, col])
    return {"m8": m8, "e4": e4, "base": base, "rp": rp, "er": r.astype(np.int32), "ec": col.astype(np.int32),
            "ev": ev, "N": N, "K": K, "CH": CH}


def bf16_bits_to_f32(u):
    return (np.asarray(u, np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x):
    """Round-to-nearest-even fp32 -> bf16 (what torch `.to(bfloat16)` and Triton `.to(tl.bfloat16)` do)."""
    x = np.ascontiguousarray(x, np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r = np.where(nan, np.uint16(0x7FC0), r)
    return r


def f32_to_bf16_bits_rtz(x):
    """Truncating fp32 -> bf16 (what the Triton 3.6 *interpreter* does for `.to(tl.bfloat16)`; compiled
    Triton on a GPU rounds to nearest-even). Used only to pin the oracle against interpreter goldens."""
    return (np.ascontiguousarray(x, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def to_bf16_bits(x, rounding="rne"):
    return f32_to_bf16_bits(x) if rounding == "rne" else f32_to_bf16_bits_rtz(x)


def round_bf16(x, rounding="rne"):
    return bf16_bits_to_f32(to_bf16_bits(x, rounding))


def decode_bits(m8, e4, base, CH=256):
    """fp32 bit patterns of the planes, code 15 -> 0 (wcomp.py:35-42, _dec :48-54)."""
    N, K = m8.shape
    e = e4.astype(np.int32).reshape(N, K // CH, CH // 2)
    code = np.stack([e & 15, e >> 4], 2).reshape(N, K)
    m = m8.astype(np.int32)
    bits = ((m >> 7) << 31) | ((code + base) << 23) | ((m & 0x7F) << 16)
    bits = np.where(code == 15, 0, bits)
    return bits.astype(np.uint32)


def decompress(c):
    """dict -> uint16 bf16 bits [N, K] (wcomp.py:35-45)."""
    W = decode_bits(c["m8"], c["e4"], c["base"], c["CH"]).view(np.float32).copy()
    W[c["er"].astype(np.int64), c["ec"].astype(np.int64)] = c["ev"]
    return f32_to_bf16_bits(W)


def weight_rows(c, first, last):
    """fp32 rows [first, last) with exceptions (prefill.py:23-42 / prefill_kernels.py:221-231)."""
    W = decode_bits(c["m8"][first:last], c["e4"][first:last], c["base"], c["CH"]).view(np.float32).copy()
    a, b = int(c["rp"][first]), int(c["rp"][last])
    W[c["er"][a:b].astype(np.int64) - first, c["ec"][a:b].astype(np.int64)] = c["ev"][a:b]
    return W


def dense_f32(c):
    return weight_rows(c, 0, c["N"])
