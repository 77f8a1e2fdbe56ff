"""Whole-prompt prefill on the GPU: the tcgen05 codec GEMM and the causal prefill attention against the reference
goldens (`tests/golden/prefill.npz`: mm_k and att_k run by the reference) and the oracle.

Tolerances: precision 3 (three bf16 parts of the activations, exact products, fp32 accumulation) is held to the
fp32-accumulation bound |y - ref| <= 2e-5 * sum|w||x| + 1e-6, as the GEMV tests; precision 1 (bf16 activations)
to 8e-3 * sum|w||x| (the activation rounding, 2^-9 relative per product, plus accumulation).
"""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import codec, gemv as ogemv

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib(cuda_dev):
    from ai_b200 import build, _lib
    build.build()
    return _lib.lib()


def from_bits(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).cuda()


def status_clear():
    from ai_b200 import _lib
    return _lib.status(clear=True)


def check(got, want, mag, precision):
    rtol = 2e-5 if precision == 3 else 8e-3
    d = np.abs(np.asarray(got, np.float64) - np.asarray(want, np.float64))
    bad = d > rtol * mag + 1e-6
    assert not bad.any(), f"{bad.sum()} of {bad.size} off, max |d| {d.max():.3e}"


@pytest.mark.parametrize("precision", [3, 1])
def test_gemm_matches_reference_mm_golden(lib, precision):
    """Y = X W^T of the reference's fp32 mm_k on its golden inputs: W [40, 512] with a 1e-30 and a 1e20
    exception, X [37, 512]; both M and N are ragged (partial tiles)."""
    from ai_b200 import wcomp, prefill
    z = golden("prefill")
    w, x, want = z["rows/w"], z["mm/x"], z["mm/y"]
    c = wcomp.compress(from_bits(w))
    assert int(c["ev"].numel()) >= 2
    X = torch.from_numpy(x).cuda()
    Y = torch.full((x.shape[0], w.shape[0]), float("nan"), device="cuda")
    prefill.matrix(X, c, Y, precision=precision)
    torch.cuda.synchronize()
    W = codec.bf16_bits_to_f32(w).astype(np.float64)
    mag = np.abs(x.astype(np.float64)) @ np.abs(W).T
    check(Y.cpu().numpy(), want, mag, precision)
    assert status_clear() == 0


CASES = [  # (M, N, K, xmode, ymode, rms)
    (128, 256, 512, 0, 0, False), (37, 300, 1024, 0, 1, False), (300, 384, 256, 0, 0, True),
    (200, 256, 1024, 2, 1, False), (64, 512, 768, 0, 3, True), (17, 128, 4096, 0, 0, True),
    (513, 640, 2048, 0, 1, False),
    # M <= 16: split-K over up to 8 CTAs per weight tile (partials added in split order by the last split)
    (1, 256, 4096, 0, 1, True), (8, 4096, 4096, 0, 3, True), (16, 1024, 12288, 2, 1, False), (5, 640, 2048, 0, 0, False),
]


def test_gemm_split_k_deterministic(lib):
    """Few tokens split K over several CTAs per weight tile: repeated launches give identical bits, and the
    result equals the same product with one row at a time (each row is its own token tile either way)."""
    from ai_b200 import wcomp, prefill
    gen = torch.Generator(device="cuda").manual_seed(5)
    N, K, M = 4096, 12288, 8
    c = wcomp.compress((torch.randn(N, K, generator=gen, device="cuda") * 0.02).bfloat16())
    X = torch.randn(M, K, generator=gen, device="cuda")
    outs = []
    for _ in range(3):
        Y = torch.zeros(M, N, device="cuda")
        prefill.matrix(X, c, Y, precision=3)
        outs.append(Y)
    torch.cuda.synchronize()
    assert all(torch.equal(outs[0], o) for o in outs[1:])
    assert status_clear() == 0


@pytest.mark.parametrize("precision", [3, 1])
@pytest.mark.parametrize("M,N,K,xmode,ymode,rms", CASES)
def test_gemm_vs_oracle(lib, M, N, K, xmode, ymode, rms, precision):
    """Ragged M and N tiles, several K blocks, the SiLU-gated input (xmode 2), accumulate (ymode 1), gated output
    (ymode 3), the RMSNorm prologue, and exceptions on a few rows -- against the float64 oracle."""
    from ai_b200 import wcomp, prefill
    g = np.random.default_rng(M * 7 + N + K + ymode + precision)
    wf = (g.standard_normal((N, K)) * 0.02).astype(np.float32)
    wf[5, ::131] = 1e-30
    wf[N - 1, 7] = 5.0
    wb = codec.f32_to_bf16_bits(wf)
    xin_cols = 2 * K if xmode == 2 else K
    x = g.standard_normal((M, xin_cols)).astype(np.float32)
    lnw = codec.f32_to_bf16_bits((1 + 0.1 * g.standard_normal(K)).astype(np.float32)) if rms else None
    y0 = g.standard_normal((M, N // 2 if ymode == 3 else N)).astype(np.float32)
    c = wcomp.compress(from_bits(wb))
    assert int(c["ev"].numel()) > 0
    X = torch.from_numpy(x).cuda()
    Y = torch.from_numpy(y0.copy()).cuda()
    prefill.matrix(X, c, Y, add=ymode == 1, precision=precision, lnw=from_bits(lnw) if rms else None,
                   silu_input=xmode == 2, gated=ymode == 3)
    torch.cuda.synchronize()
    xe = ogemv.xin(x, K, xmode, lnw, 1e-6).astype(np.float64)
    W = codec.bf16_bits_to_f32(wb).astype(np.float64)
    acc = xe @ W.T
    mag = np.abs(xe) @ np.abs(W).T
    if ymode == 3:
        g_, u_ = acc[:, 0::2].astype(np.float32), acc[:, 1::2].astype(np.float32)
        want = ogemv.silu_mul(g_, u_)
        check(Y.cpu().numpy(), want, 1.2 * (np.abs(u_) * mag[:, 0::2] + np.abs(g_) * mag[:, 1::2]), precision)
    else:
        want = acc + (y0 if ymode == 1 else 0)
        check(Y.cpu().numpy(), want, mag, precision)
    assert status_clear() == 0


def test_gemm_deterministic_and_large(lib):
    """A Qwen3-8B-shaped gate/up matrix (24576 x 4096) over 512 prompt rows: repeated launches give identical
    bits, and sampled rows match the oracle."""
    from ai_b200 import wcomp, prefill
    gen = torch.Generator(device="cuda").manual_seed(3)
    N, K, M = 24576, 4096, 512
    Wt = (torch.randn(N, K, generator=gen, device="cuda") * 0.02).bfloat16()
    c = wcomp.compress(Wt)
    X = torch.randn(M, K, generator=gen, device="cuda")
    Y1 = torch.empty(M, N, device="cuda")
    Y2 = torch.empty(M, N, device="cuda")
    ws = prefill.workspace(M, K, 3)
    prefill.matrix(X, c, Y1, ws=ws)
    prefill.matrix(X, c, Y2, ws=ws)
    torch.cuda.synchronize()
    assert torch.equal(Y1, Y2)
    rows = torch.tensor([0, 1, 255, 511], device="cuda")
    cols = torch.arange(0, N, 97, device="cuda")
    W64 = Wt[cols].double()
    want = (X[rows].double() @ W64.T).cpu().numpy()
    mag = (X[rows].double().abs() @ W64.abs().T).cpu().numpy()
    check(Y1[rows][:, cols].cpu().numpy(), want, mag, 3)
    assert status_clear() == 0


# --------------------------------------------------------------------------------- prefill attention
def bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def test_prefill_attention_matches_reference_golden(lib):
    """att_k's own output on its golden inputs (H 4, KV 2, HD 64, 37 prompt rows after 20 cached positions)."""
    from ai_b200 import prefill
    z = golden("prefill")
    H, KV, HD, maxt, n, start = (int(v) for v in z["att/cfg"])
    q = torch.from_numpy(z["att/q"]).cuda()
    out = torch.full((n, H * HD), float("nan"), device="cuda")
    prefill.attention(q, from_bits(z["att/kc"]), from_bits(z["att/vc"]), out, start, H, KV, HD)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), z["att/out"], rtol=2e-4, atol=2e-5)
    assert status_clear() == 0


@pytest.mark.parametrize("H,KV,HD,n,start", [(32, 8, 128, 300, 0), (16, 8, 128, 129, 17), (8, 1, 128, 70, 5),
                                             (4, 4, 64, 33, 2), (64, 8, 128, 517, 1000)])
def test_prefill_attention_vs_oracle(lib, H, KV, HD, n, start):
    """Causal attention of n prompt rows after `start` cached positions, GQA ratios 1..8, ragged query tiles,
    against the oracle's exact softmax."""
    from ai_b200 import prefill
    from oracle import attn as oattn
    g = np.random.default_rng(n + H + start)
    maxt = start + n + 3
    q = g.standard_normal((n, H * HD)).astype(np.float32)
    kc = codec.f32_to_bf16_bits(g.standard_normal((KV, maxt, HD)).astype(np.float32))
    vc = codec.f32_to_bf16_bits(g.standard_normal((KV, maxt, HD)).astype(np.float32))
    out = torch.full((n, H * HD), float("nan"), device="cuda")
    prefill.attention(torch.from_numpy(q).cuda(), from_bits(kc), from_bits(vc), out, start, H, KV, HD)
    torch.cuda.synchronize()
    rows = np.unique(np.r_[0, 1, n // 2, n - 1, g.integers(0, n, 12)])
    ref = np.stack([oattn.prefill_attention(q[r:r + 1], kc, vc, start + int(r), H, KV, HD)[0] for r in rows])
    np.testing.assert_allclose(out.cpu().numpy()[rows], ref, rtol=2e-4, atol=2e-5)
    assert status_clear() == 0


# ------------------------------------------------------------------------------------ engine prefill
@pytest.mark.parametrize("name", ["small", "small-1k"])
def test_engine_prefill_matches_chunked_path(lib, name, monkeypatch):
    """A 53-token prompt through the whole-prompt prefill gives the same next token as the 16-token chunk path
    (the reference's legacy path), a KV cache within bf16 rounding of it, and the same greedy continuation."""
    from ai_b200.engine import Engine
    from ai_b200.model import CONFIGS, RandomWeights
    cfg = CONFIGS[name]
    rw = RandomWeights(cfg, seed=11, norm_noise=0.1, std=0.05)
    prompt = [int(t) for t in np.random.default_rng(9).integers(0, cfg.V, 53)]
    a = Engine(cfg, maxt=128, weights=rw, log=None)
    b = Engine(cfg, maxt=128, weights=rw, log=None)
    ta = list(a.generate(prompt, max_new=12))
    monkeypatch.setenv("AIB_PREFILL", "legacy")
    tb = list(b.generate(prompt, max_new=12))
    assert ta == tb
    ka, kb = a.kv[:, :, :, :53].float().cpu().numpy(), b.kv[:, :, :, :53].float().cpu().numpy()
    # a bf16 rounding step apart (fp32 sums in another order can round the other way), with an absolute floor at
    # 1e-3 of the cache's scale for entries near zero, where the two paths' fp32 rounding differences dominate
    d = np.abs(ka - kb)
    bad = d > 2.0 ** -7 * np.maximum(np.abs(ka), np.abs(kb)) + 1e-3 * np.abs(kb).max()
    assert not bad.any(), f"{bad.sum()} of {bad.size} cache entries differ; max |d| {d.max():.3e}"
    assert status_clear() == 0
