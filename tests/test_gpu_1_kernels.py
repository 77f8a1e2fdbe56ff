"""Parity of every CUDA kernel of the decode path against the CPU oracle and the reference goldens.

Tolerances: integer/byte work (codec encode/decode, K/V bf16 rounding, sampler ids) is bit-exact.
Floating-point outputs are compared with the fp32-accumulation bound |y - ref| <= RTOL * (|W| |x|) + ATOL,
RTOL = 2e-5 (far inside the rel-err 1e-2 that the path's spec allows for bf16 weights with fp32 accumulate).
"""
import numpy as np
import pytest
import torch

from conftest import golden, cases, cdict
from oracle import codec, gemv as ogemv, attn as oattn, sampler as osamp

pytestmark = pytest.mark.gpu
RTOL, ATOL = 2e-5, 1e-6


@pytest.fixture(scope="module")
def lib(cuda_dev):
    from ai_b200 import build, _lib
    build.build()
    return _lib.lib()


def bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def from_bits(a, dev="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(dev)


def close(y, ref, mag, rtol=RTOL, atol=ATOL):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    bad = np.abs(y - ref) > rtol * np.asarray(mag, np.float64) + atol
    assert not bad.any(), f"{bad.sum()} mismatches, max |d| {np.abs(y - ref).max():.3e}"


def standin_mag(oc, x):
    """|x| weighted by the stand-in bound 2^(base+16-127) at every exception: the wide GEMV kernels decode an
    exception as a finite stand-in G (|G| < 2^(base+16-127)) and add (v - G) x afterwards, so their rounding
    error scales with sum max(|w|, |G|) |x| rather than sum |w| |x| (which only matters for rows made of tiny
    exceptions)."""
    N = int(oc["N"])
    rp, ec = np.asarray(oc["rp"]), np.asarray(oc["ec"])
    g = 2.0 ** (int(oc["base"]) + 16 - 127)
    ax = np.abs(np.asarray(x, np.float64))
    out = np.zeros(N)
    for r in range(N):
        out[r] = g * ax[ec[rp[r]:rp[r + 1]]].sum()
    return out


def status_clear():
    from ai_b200 import _lib
    return _lib.status(clear=True)


# ------------------------------------------------------------------------------------------- codec
@pytest.mark.parametrize("name", cases(golden("codec")))
def test_device_encoder_bit_exact(lib, name):
    from ai_b200 import wcomp
    z = golden("codec")
    c = wcomp.compress(from_bits(z[f"{name}/w"]))
    ref = cdict(z, f"{name}/")
    assert c["base"] == ref["base"]
    for k in ("m8", "e4", "rp", "er", "ec"):
        np.testing.assert_array_equal(c[k].cpu().numpy(), ref[k], err_msg=k)
    np.testing.assert_array_equal(c["ev"].cpu().numpy().view(np.uint32), ref["ev"].view(np.uint32))


def test_device_encoder_large_matrix_matches_oracle(lib):
    from ai_b200 import wcomp
    g = torch.Generator(device="cuda").manual_seed(1)
    w = (torch.randn(6144, 4096, generator=g, device="cuda") * 0.02).bfloat16()
    w[17, 100] = 3e4
    c = wcomp.compress(w)
    o = codec.compress(bits(w))
    assert c["base"] == o["base"] and c["ev"].numel() == len(o["ev"])
    for k in ("m8", "e4", "rp", "er", "ec"):
        assert np.array_equal(c[k].cpu().numpy(), o[k]), k
    # decode round trip, bf16 and fp32 rows
    assert torch.equal(wcomp.decompress(c).view(torch.int16), w.view(torch.int16))
    assert torch.equal(wcomp.weight_rows(c, 10, 30), w[10:30].float())


@pytest.mark.parametrize("name", cases(golden("codec")))
def test_decode_roundtrip_golden(lib, name):
    from ai_b200 import wcomp
    z = golden("codec")
    w = from_bits(z[f"{name}/w"])
    c = wcomp.compress(w)
    d = bits(wcomp.decompress(c))
    f = codec.bf16_bits_to_f32(z[f"{name}/w"])
    nan = np.isnan(f)
    np.testing.assert_array_equal(d[~nan], z[f"{name}/w"][~nan])


def test_weight_rows_matches_reference_decode_rows(lib):
    from ai_b200 import wcomp
    z = golden("prefill")
    c = wcomp.compress(from_bits(z["rows/w"]))
    out = wcomp.weight_rows(c, int(z["rows/first"]), int(z["rows/last"])).cpu().numpy()
    np.testing.assert_array_equal(out.view(np.uint32), z["rows/out"].view(np.uint32))


# -------------------------------------------------------------------------------------------- gemv
@pytest.mark.parametrize("name", cases(golden("gemv")))
def test_gemvc1_matches_reference_golden(lib, variant, name):
    from ai_b200 import wcomp
    z = golden("gemv")
    c = wcomp.compress(from_bits(z[f"{name}/w"]))
    x = torch.from_numpy(z[f"{name}/x"]).cuda()
    y = torch.from_numpy(z[f"{name}/y0"]).cuda()
    lnw = from_bits(z[f"{name}/lnw"]) if f"{name}/lnw" in z.files else None
    mode = int(z[f"{name}/mode"])
    wcomp.gemvc1(x, c, y, mode, lnw=lnw, eps=1e-6)
    W = np.abs(codec.bf16_bits_to_f32(z[f"{name}/w"])).astype(np.float64)
    xe = np.abs(ogemv.xin(z[f"{name}/x"], c["K"], mode, z.get(f"{name}/lnw") if lnw is not None else None))
    close(y.cpu().numpy(), z[f"{name}/y"], W @ xe + np.abs(z[f"{name}/y0"]) * (mode > 0), rtol=4e-5)
    assert status_clear() == 0


GEMV_SHAPES = [(64, 1024, 0, False), (6144, 4096, 0, True), (4096, 4096, 1, False), (24576, 4096, 0, True), (4096, 12288, 2, False),
               (1024, 2048, 1, False), (4096, 1024, 0, True), (517, 768, 2, False), (40, 256, 0, True),
               (100, 3072, 1, True), (33, 2048, 0, False), (1000, 5120, 2, False),
               (64, 16384, 1, False), (200, 8192, 0, True)]  # many CTAs per row tile under stream-K


@pytest.fixture(params=[1, 3, 4], ids=["cudacore", "widetc", "widetc1"])
def variant(request, lib):
    """T = 1 GEMV kernel (test knob 4): the CUDA-core 12 KB-stage kernel, the tensor-core wide-stage kernel
    (default: two CTAs per SM where the shape fits) and its one-CTA-per-SM geometry."""
    assert lib.aib_debug_knob(4, request.param) == 0
    yield request.param
    assert lib.aib_debug_knob(4, 3) == 0  # library default


@pytest.mark.parametrize("streamk", [False, True], ids=["tiles", "streamk"])
@pytest.mark.parametrize("N,K,mode,rms", GEMV_SHAPES)
def test_gemvc1_shapes_vs_oracle(lib, variant, N, K, mode, rms, streamk):
    from ai_b200 import wcomp
    g = torch.Generator(device="cuda").manual_seed(N + K + mode)
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).bfloat16()
    idx = torch.randint(0, N * K, (37,), generator=g, device="cuda")
    w.view(-1)[idx] = (torch.randn(37, generator=g, device="cuda") * 1e4).bfloat16()  # exceptions
    c = wcomp.compress(w)
    assert c["ev"].numel() >= 30
    xin = 2 * K if mode == 2 else K
    x = torch.randn(xin, generator=g, device="cuda") * (2.0 if rms else 1.0)
    y0 = torch.randn(N, generator=g, device="cuda")
    lnw = (1 + 0.1 * torch.randn(K, generator=g, device="cuda")).bfloat16() if rms else None
    y = y0.clone()
    ws = wcomp.gemv_workspace([c], "cuda") if streamk else None
    wcomp.gemvc1(x, c, y, mode, lnw=lnw, eps=1e-6, ws=ws)
    if ws is not None:  # the call left its flags / tickets at zero: a second call gives the same bits
        y2 = y0.clone()
        wcomp.gemvc1(x, c, y2, mode, lnw=lnw, eps=1e-6, ws=ws)
        assert torch.equal(y, y2)
    oc = codec.compress(bits(w))
    ref = ogemv.gemvc1(x.cpu().numpy(), oc, y0.cpu().numpy(), mode, bits(lnw) if rms else None, 1e-6)
    xe = ogemv.xin(x.cpu().numpy(), K, mode, bits(lnw) if rms else None, 1e-6)
    mag = np.abs(codec.dense_f32(oc)).astype(np.float64) @ np.abs(xe) + np.abs(y0.cpu().numpy()) * (mode > 0)
    close(y.cpu().numpy(), ref, mag)
    assert status_clear() == 0


@pytest.mark.parametrize("T", [1, 2, 5, 16])
@pytest.mark.parametrize("N,K", [(4096, 1024), (3000, 4096), (1000, 1536)])
def test_gemv_gated_output(lib, T, N, K):
    """Mode 3: rows (gate_i, up_i) interleaved, y[i] = silu(g_i) * u_i -- same values as mode 0 + the SiLU gate
    of mode 2 on the reference's [gate; up] layout (T == 1 needs K % 1024 == 0: wide kernels)."""
    from ai_b200 import wcomp
    if T == 1 and K % 1024:
        pytest.skip("T = 1 gated output needs K % 1024 == 0")
    g = torch.Generator(device="cuda").manual_seed(N + K + T)
    gu = (torch.randn(N, K, generator=g, device="cuda") * 0.02).bfloat16()
    gu.view(-1)[torch.randint(0, N * K, (20,), generator=g, device="cuda")] = 3e3  # exceptions
    il = wcomp.interleave_gate_up(gu)
    c_il, c_ref = wcomp.compress(il), wcomp.compress(gu)
    X = torch.randn(16, K, generator=g, device="cuda")
    Y = torch.full((16, N // 2), 7.0, device="cuda")
    R = torch.zeros(16, N, device="cuda")
    wcomp.gemvc_tc(X, c_il, Y, 3, T)
    wcomp.gemvc_tc(X, c_ref, R, 0, T)
    gate, up = R[:T, : N // 2], R[:T, N // 2:]
    ref = gate / (1.0 + torch.exp(-gate)) * up
    torch.testing.assert_close(Y[:T], ref, rtol=1e-5, atol=1e-6)
    assert torch.equal(Y[T:], torch.full_like(Y[T:], 7.0))
    assert status_clear() == 0


@pytest.mark.parametrize("T", [2, 3, 8, 16])
@pytest.mark.parametrize("mode", [0, 1, 2])
def test_gemvc_tc_vs_oracle(lib, T, mode):
    from ai_b200 import wcomp
    N, K = 1000, 1536
    g = torch.Generator(device="cuda").manual_seed(T * 10 + mode)
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).bfloat16()
    w[5, 7] = 1e5
    w[999, 1535] = -3e-20
    c = wcomp.compress(w)
    xs = 2 * K if mode == 2 else K
    X = torch.randn(16, xs, generator=g, device="cuda")
    Y0 = torch.randn(16, N, generator=g, device="cuda")
    Y = Y0.clone()
    wcomp.gemvc_tc(X, c, Y, mode, T)
    oc = codec.compress(bits(w))
    ref = ogemv.gemvc_tc(X.cpu().numpy(), oc, Y0.cpu().numpy(), mode, T)
    xe = np.abs(ogemv.xin(X.cpu().numpy()[:T], K, mode))
    mag = np.zeros((16, N))
    mag[:T] = xe @ np.abs(codec.dense_f32(oc)).T.astype(np.float64) + np.abs(Y0.cpu().numpy()[:T]) * (mode > 0)
    close(Y.cpu().numpy(), ref, mag)
    assert torch.equal(Y[T:], Y0[T:])  # rows >= T untouched


def test_gemv_dense_exceptions(lib, variant):
    """Rows full of exceptions (every code 15 in a chunk / a whole row) through both kernels."""
    from ai_b200 import wcomp
    g = torch.Generator(device="cuda").manual_seed(77)
    N, K = 48, 1024
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).bfloat16()
    w[5] = (torch.randn(K, generator=g, device="cuda") * 1e5).bfloat16()
    w[20, 256:512] = (torch.randn(256, generator=g, device="cuda") * 1e-9).bfloat16()
    w[47, ::3] = 7e3
    c = wcomp.compress(w)
    x = torch.randn(K, generator=g, device="cuda")
    y = torch.zeros(N, device="cuda")
    wcomp.gemvc1(x, c, y, 0)
    W = codec.bf16_bits_to_f32(bits(w)).astype(np.float64)
    xn = x.cpu().numpy().astype(np.float64)
    close(y.cpu().numpy(), W @ xn, np.abs(W) @ np.abs(xn) + standin_mag(codec.compress(bits(w)), xn))


def test_gemv_exceptions_beyond_staged_capacity(lib, variant):
    """One CTA holding more exceptions than the wide kernel stages in shared memory (read from global)."""
    from ai_b200 import wcomp
    g = torch.Generator(device="cuda").manual_seed(78)
    N, K = 16, 4096
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).bfloat16()
    w[3] = (torch.randn(K, generator=g, device="cuda") * 1e5).bfloat16()
    w[9] = (torch.randn(K, generator=g, device="cuda") * 1e-12).bfloat16()
    c = wcomp.compress(w)
    assert c["ev"].numel() > 8000
    x = torch.randn(K, generator=g, device="cuda")
    y0 = torch.randn(N, generator=g, device="cuda")
    y = y0.clone()
    wcomp.gemvc1(x, c, y, 1)
    W = codec.bf16_bits_to_f32(bits(w)).astype(np.float64)
    xn = x.cpu().numpy().astype(np.float64)
    mag = np.abs(W) @ np.abs(xn) + np.abs(y0.cpu().numpy()) + standin_mag(codec.compress(bits(w)), xn)
    close(y.cpu().numpy(), W @ xn + y0.cpu().numpy(), mag)
    assert status_clear() == 0


@pytest.mark.parametrize("K", [4096, 12288])
def test_gemv_deterministic(lib, K):
    """Repeated calls give identical bits, with and without the stream-K workspace (split tiles are added in
    a fixed order whichever CTA finishes last)."""
    from ai_b200 import wcomp
    g = torch.Generator(device="cuda").manual_seed(9)
    c = wcomp.compress((torch.randn(4096, K, generator=g, device="cuda") * 0.02).bfloat16())
    x = torch.randn(K, generator=g, device="cuda")
    ws = wcomp.gemv_workspace([c], "cuda")
    for w in (None, ws):
        outs = []
        for _ in range(4):
            y = torch.zeros(4096, device="cuda")
            wcomp.gemvc1(x, c, y, 0, ws=w)
            outs.append(y)
        assert all(torch.equal(outs[0], o) for o in outs[1:])


# ----------------------------------------------------------------------------------- norm / embed
def test_rmsnorm_vs_golden(lib):
    from ai_b200 import tkernels
    z = golden("attn")
    x = torch.from_numpy(z["rms/x"]).cuda()
    out = torch.zeros_like(x)
    tkernels.rmsg(x, from_bits(z["rms/w"]), out, 1e-6)
    np.testing.assert_allclose(out.cpu().numpy(), z["rms/out"], rtol=2e-6, atol=2e-6)


def test_embed(lib):
    from ai_b200 import tkernels
    emb = torch.randn(300, 96, device="cuda").bfloat16()
    ids = torch.tensor([0, 299, 17], device="cuda")
    out = torch.zeros(3, 96, device="cuda")
    tkernels.embed(emb, ids, out)
    assert torch.equal(out, emb[ids].float())
    bad = torch.tensor([300], device="cuda")
    tkernels.embed(emb, bad, out[:1])
    from ai_b200._lib import status
    assert status(clear=True) == 103  # AIB_DEV_BAD_TOKEN, no fault


# -------------------------------------------------------------------------------------- attention
def _attn_case(H, KV, HD, maxt, pos, seed):
    g = np.random.default_rng(seed)
    qkv = (g.standard_normal((H + 2 * KV) * HD) * 2).astype(np.float32)
    qn = codec.f32_to_bf16_bits((1 + 0.1 * g.standard_normal(HD)).astype(np.float32))
    kn = codec.f32_to_bf16_bits((1 + 0.1 * g.standard_normal(HD)).astype(np.float32))
    kc = codec.f32_to_bf16_bits(g.standard_normal((KV, maxt, HD)).astype(np.float32))
    vc = codec.f32_to_bf16_bits(g.standard_normal((KV, maxt, HD)).astype(np.float32))
    return qkv, qn, kn, kc, vc


@pytest.fixture(params=[0, 2], ids=["ticket", "cluster"])
def cluster_sizes(request, lib):
    """Attention merge: the default ticket merge, and the cluster merge (clusters of 16 where the device places
    one per group, else of 8 CTAs; split partials through distributed shared memory)."""
    assert lib.aib_debug_knob(3, request.param) == 0
    yield request.param
    assert lib.aib_debug_knob(3, 0) == 0


@pytest.mark.parametrize("H,KV,HD,pos", [(8, 2, 64, 0), (8, 2, 64, 77), (32, 8, 128, 1), (32, 8, 128, 4100),
                                         (16, 8, 128, 300), (64, 8, 128, 2047)])
def test_rope_attn_vs_oracle(lib, cluster_sizes, H, KV, HD, pos):
    from ai_b200 import tkernels
    maxt = max(128, pos + 1)
    qkv, qn, kn, kc, vc = _attn_case(H, KV, HD, maxt, pos, pos + H)
    inv = oattn.rope_inv(HD, 1e6)
    kc_ref, vc_ref = kc.copy(), vc.copy()
    ref = oattn.rope_attn(qkv, qn, kn, inv, pos, kc_ref, vc_ref, H, KV, HD, 1e-6)
    KC, VC = from_bits(kc), from_bits(vc)
    out = torch.zeros(H * HD, device="cuda")
    P = torch.tensor([pos], dtype=torch.int64, device="cuda")
    tkernels.rope_attn(torch.from_numpy(qkv).cuda(), from_bits(qn), from_bits(kn), torch.from_numpy(inv).cuda(), P,
                       KC, VC, out, maxt, 1e-6, HD ** -0.5, H, KV, HD)
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=2e-4, atol=2e-5)
    # cache rows: written row at pos matches RNE rounding (<= 1 bf16 ulp where fp32 sums differ), rest untouched
    dk = np.abs(bits(KC).astype(np.int32) - kc_ref.astype(np.int32))
    assert dk.max() <= 1 and (dk > 0).sum() <= 4
    np.testing.assert_array_equal(bits(VC), vc_ref)
    assert status_clear() == 0


def test_rope_attn_matches_reference_golden_semantics(lib):
    """Golden cases of rope_attn_k: same inputs; the GPU rounds K/V to nearest-even where the interpreter
    truncated, so the check is against the oracle pinned to those goldens, in RNE mode."""
    from ai_b200 import tkernels
    z = golden("attn")
    H, KV, HD, maxt = (int(v) for v in z["cfg"])
    for name in cases(z):
        pos = int(z[f"{name}/pos"])
        kc_ref, vc_ref = z[f"{name}/kc0"].copy(), z[f"{name}/vc0"].copy()
        ref = oattn.rope_attn(z[f"{name}/qkv"], z[f"{name}/qn"], z[f"{name}/kn"], z["inv"], pos, kc_ref, vc_ref, H, KV,
                              HD, 1e-6)
        KC, VC = from_bits(z[f"{name}/kc0"]), from_bits(z[f"{name}/vc0"])
        out = torch.zeros(H * HD, device="cuda")
        tkernels.rope_attn(torch.from_numpy(z[f"{name}/qkv"]).cuda(), from_bits(z[f"{name}/qn"]),
                           from_bits(z[f"{name}/kn"]), torch.from_numpy(z["inv"]).cuda(),
                           torch.tensor([pos], device="cuda"), KC, VC, out, maxt, 1e-6, HD ** -0.5, H, KV, HD)
        np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=2e-4, atol=2e-5)
        # and within bf16-rounding distance of the reference's own output
        np.testing.assert_allclose(out.cpu().numpy(), z[f"{name}/out"], rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("T,pos", [(2, 0), (5, 40), (16, 1000)])
def test_batched_attention_vs_oracle(lib, T, pos):
    from ai_b200 import tkernels
    H, KV, HD = 32, 8, 128
    maxt = pos + T + 8
    g = np.random.default_rng(T)
    qkv = (g.standard_normal((T, (H + 2 * KV) * HD))).astype(np.float32)
    _, qn, kn, kc, vc = _attn_case(H, KV, HD, maxt, pos, T + 5)
    inv = oattn.rope_inv(HD, 1e6)
    kc_ref, vc_ref = kc.copy(), vc.copy()
    Qr = oattn.qk_rope_cache(qkv, qn, kn, inv, pos, kc_ref, vc_ref, H, KV, HD, 1e-6)
    KC, VC = from_bits(kc), from_bits(vc)
    q = torch.zeros(T, H * HD, device="cuda")
    P = torch.tensor([pos], dtype=torch.int64, device="cuda")
    tkernels.qk_rope_cache(torch.from_numpy(qkv).cuda(), from_bits(qn), from_bits(kn), torch.from_numpy(inv).cuda(),
                           P, q, KC, VC, maxt, 1e-6, H, KV, HD, T)
    np.testing.assert_allclose(q.cpu().numpy(), Qr, rtol=1e-5, atol=1e-5)
    dk = np.abs(bits(KC).astype(np.int32) - kc_ref.astype(np.int32))
    assert dk.max() <= 1
    np.testing.assert_array_equal(bits(VC), vc_ref)
    out = torch.zeros(T, H * HD, device="cuda")
    tkernels.attn(q, KC, VC, P, out, maxt, HD ** -0.5, H, KV, HD, T)
    ref = oattn.attn(q.cpu().numpy(), bits(KC), bits(VC), pos, H, KV, HD)
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=2e-4, atol=2e-5)
    assert status_clear() == 0


# ---------------------------------------------------------------------------------------- sampler
@pytest.mark.parametrize("two_phase", [True, False], ids=["slices", "onecta"])
@pytest.mark.parametrize("name", cases(golden("sampler")))
def test_sampler_matches_reference_pick(lib, name, two_phase):
    from ai_b200 import sampler
    z = golden("sampler")
    lg = torch.from_numpy(z[f"{name}/logits"]).cuda()
    mask = torch.from_numpy(z[f"{name}/mask"]).cuda() if f"{name}/mask" in z.files else None
    ids = sampler.sample(lg, float(z[f"{name}/temp"]), float(z[f"{name}/top_p"]), 0, z[f"{name}/u"], mask=mask,
                         two_phase=two_phase)
    np.testing.assert_array_equal(ids, z[f"{name}/ids"])


@pytest.mark.parametrize("name", cases(golden("sampler"), "head_names"))
def test_sampler_matches_reference_head_pick(lib, name):
    from ai_b200 import sampler
    from oracle import head as ohead
    z = golden("sampler")
    ex = ohead.exact_logits(z[f"{name}/w"], z[f"{name}/h"])
    ids = sampler.sample(torch.from_numpy(ex).cuda(), float(z[f"{name}/temp"]), float(z[f"{name}/top_p"]), 0,
                         [float(z[f"{name}/u"])])
    assert ids[0] == int(z[f"{name}/ids"][0])


SAMPLER_CASES = [  # (V, T, top_k, top_p, rep, pres, freq, masked)
    (151936, 0.7, 20, 0.8, 1.05, 0.0, 0.0, False),  # BASELINE config 1 sampler settings
    (151936, 0.7, 50, 0.95, 1.1, 0.5, 0.3, True),   # config 4 sweep settings
    (151936, 0.7, 1, 0.8, 1.1, 0.5, 0.3, False),
    (151936, 0.6, 20, 0.8, 1.0, 0.0, 0.0, False),   # config 3 decode settings
    (151936, 0.0, 0, 1.0, 1.3, 0.2, 0.1, True),
    (151936, 0.7, 0, 0.8, 1.0, 0.0, 0.0, False),    # top-p over the whole vocabulary
    (5000, 1.5, 0, 1.0, 1.0, 0.0, 0.0, False),
    (5000, 0.9, 0, 0.9, 2.0, 1.0, 1.0, True),
    (151936, 0.8, 100, 0.9, 1.0, 0.0, 0.0, False),  # top_k above the per-slice candidates: merge falls back
    (300, 0.5, 0, 0.99, 1.0, 0.0, 0.0, True),       # fewer tokens than slices x candidates
]


@pytest.mark.parametrize("two_phase", [True, False], ids=["slices", "onecta"])
@pytest.mark.parametrize("case", SAMPLER_CASES)
def test_sampler_extended_vs_oracle(lib, case, two_phase):
    from ai_b200 import sampler
    V, T, k, p, rep, pres, freq, masked = case
    B = 4
    rng = np.random.default_rng(V + k)
    scale = 2.0 if V > 10000 else 3.0
    lg = (rng.standard_normal((B, V)) * scale).astype(np.float32)
    prior = rng.integers(0, V, (B, 1024)).astype(np.int32)
    prior[:, :64] = prior[:, 64:128]  # repeated ids -> counts > 1
    prior[0, 5] = -1
    words = (V + 31) // 32
    mask = None
    if masked:
        mask = (rng.random((B, words * 32)) < 0.1).reshape(B, words, 32)
        mask = (mask * (1 << np.arange(32, dtype=np.uint64))).sum(-1).astype(np.uint32).view(np.int32)
        mask[:, 0] |= 1  # token 0 always allowed
    us = [np.random.default_rng(b).random() for b in range(B)]
    ids = sampler.sample(torch.from_numpy(lg).cuda(), T, p, k, us, prior=torch.from_numpy(prior).cuda(),
                         mask=torch.from_numpy(mask).cuda() if mask is not None else None, repetition_penalty=rep,
                         presence_penalty=pres, frequency_penalty=freq, two_phase=two_phase)
    ref = [osamp.sample_row(lg[b], T, k, p, rep, pres, freq, prior[b], mask[b] if mask is not None else None, us[b])
           for b in range(B)]
    assert ids == ref
    assert status_clear() == 0


@pytest.mark.parametrize("two_phase", [True, False], ids=["slices", "onecta"])
def test_sampler_many_rows_and_greedy_ties(lib, two_phase):
    from ai_b200 import sampler
    lg = torch.zeros(64, 1000, device="cuda")
    lg[:, 17] = 1.0
    lg[:, 400] = 1.0
    assert sampler.sample(lg, two_phase=two_phase) == [17] * 64


def test_sampler_ties_across_slices(lib):
    """Equal maxima in different vocabulary slices: the first index wins; sampling ties keep index order."""
    from ai_b200 import sampler
    lg = torch.full((2, 151936), -5.0, device="cuda")
    lg[:, 150000] = 3.0
    lg[:, 70000] = 3.0
    lg[:, 5] = 2.0
    assert sampler.sample(lg) == [70000, 70000]
    ids = sampler.sample(lg, 1.0, 1.0, 2, [0.25, 0.75])  # top-2 = the tied pair, index order, p = 1/2 each
    assert ids == [70000, 150000]
    ids = sampler.sample(lg, 1.0, 0.5, 2, [0.25, 0.75])  # exclusive cumsum 0.5 is not < 0.5: one token kept
    assert ids == [70000, 70000]


# ------------------------------------------------------------------------------------ int8 vocab head
from oracle import head as ohead  # noqa: E402


def _head_tables(w_bits):
    from ai_b200 import _lib
    V, D = w_bits.shape
    w = from_bits(w_bits)
    Q = torch.empty(V, D, dtype=torch.int8, device="cuda")
    S, C1, C2, AM = (torch.empty(V, device="cuda") for _ in range(4))
    from ai_b200._lib import ptr, stream_ptr
    _lib.call("aib_head8_tables", ptr(w.view(torch.int16)), V, D, ptr(Q), ptr(S), ptr(C1), ptr(C2), ptr(AM),
              stream_ptr())
    torch.cuda.synchronize()
    return Q, S, C1, C2, AM


def _check_tables(got, ref):
    Q, S, C1, C2, AM = (t.cpu().numpy() for t in got)
    rq, rs, rc1, rc2, ram = ref
    np.testing.assert_array_equal(Q, rq)
    np.testing.assert_array_equal(S, rs)
    np.testing.assert_array_equal(C1, rc1)
    np.testing.assert_array_equal(AM, ram)
    # C2 sums squares in float64 in another order: equal after rounding to fp32 up to one fp32 ulp
    np.testing.assert_array_max_ulp(C2, rc2, maxulp=1)


def test_head8_tables_golden(lib):
    """Head.__init__ tables of the reference's own fixture (generation/head.py:29-50), bit for bit."""
    z = golden("head")
    _check_tables(_head_tables(z["w"]), (z["q"], z["s"], z["c1"], z["c2"], z["am"]))


def test_head8_tables_vs_oracle(lib):
    """Random head with the edge rows the quantiser meets: all zeros, one tiny row, exact .5 quotients, a row
    whose max is negative."""
    g = np.random.default_rng(5)
    w = (g.standard_normal((2000, 1024)) * 0.02).astype(np.float32)
    w[3] = 0.0
    w[4] *= 1e-30
    w[5, :8] = [127.0, 63.5, -63.5, 0.5, 1.5, -2.5, 31.75, 0.25]
    w[5, 8:] = 0.0
    w[6] = -np.abs(w[6]) * 3
    wb = codec.f32_to_bf16_bits(w)
    _check_tables(_head_tables(wb), ohead.tables(wb))


def _head_case(seed, V, D, T, ties=False, exceptions=False):
    from ai_b200 import wcomp
    g = np.random.default_rng(seed)
    w = (g.standard_normal((V, D)) * 0.02).astype(np.float32)
    if ties:  # rows 17 and 9 identical and strongest: the smaller id must win
        w[17] = w[9] = np.abs(w[9]) * 4
    if exceptions:  # strongest row holds values far outside the exponent window (codec exceptions)
        w[33] = np.abs(w[33]) * 4
        w[33, ::97] = 1e-30
        w[33, 5] = 3.0
    wb = codec.f32_to_bf16_bits(w)
    h = g.standard_normal((T, D)).astype(np.float32)
    if ties or exceptions:
        h = np.abs(h)
    c = wcomp.compress(from_bits(wb))
    return wb, h, c


@pytest.mark.parametrize("T", [1, 3, 10])
def test_head8_bounds_vs_oracle(lib, T):
    """HI / LO of vocab_a_k against the float64 oracle, and the property the greedy pick relies on: every exact
    logit lies at or below its HI, and the best exact logit at or above LO."""
    from ai_b200.head import Head
    wb, h, c = _head_case(100 + T, 4096, 512, T)
    hd = Head(from_bits(wb), c)
    H = torch.from_numpy(h).cuda()
    HI, LO = hd.bounds(H, T)
    torch.cuda.synchronize()
    rhi, rlo = ohead.bounds(h, *ohead.tables(wb))
    scale = (np.abs(ohead.tables(wb)[0]).astype(np.float64) @ np.abs(h).T.astype(np.float64)).T * \
        ohead.tables(wb)[1][None].astype(np.float64)
    np.testing.assert_allclose(HI.cpu().numpy(), rhi, rtol=0, atol=float(4e-6 * scale.max() + 1e-6))
    np.testing.assert_allclose(LO.cpu().numpy(), rlo, rtol=0, atol=float(4e-6 * scale.max() + 1e-6))
    ex = ohead.exact_logits(wb, h)
    assert (ex <= HI.cpu().numpy()).all()
    assert (ex.max(1) >= LO.cpu().numpy()).all()
    assert status_clear() == 0


def test_head8_bounds_golden(lib):
    """HI / LO of the reference's fixture (3 rows of h, a 300 x 64 head), within fp32 accumulation order."""
    from ai_b200._lib import ptr, stream_ptr
    from ai_b200 import _lib
    z = golden("head")
    V, D = z["w"].shape
    T = z["h"].shape[0]
    Q, S, C1, C2, AM = _head_tables(z["w"])
    h = torch.from_numpy(z["h"]).cuda()
    HI = torch.empty(T, V, device="cuda")
    LO = torch.empty(T, device="cuda")
    ws = torch.zeros(lib.aib_head8_workspace(V, D, T), dtype=torch.uint8, device="cuda")
    _lib.call("aib_head8_bounds", ptr(h), T, D, ptr(Q), ptr(S), ptr(C1), ptr(C2), ptr(AM), V, D, ptr(HI), V,
              ptr(LO), ptr(ws), ws.numel(), stream_ptr())
    torch.cuda.synchronize()
    np.testing.assert_allclose(HI.cpu().numpy(), z["hi"], rtol=2e-6, atol=2e-5)
    np.testing.assert_allclose(LO.cpu().numpy(), z["lo"], rtol=2e-6, atol=2e-5)


@pytest.mark.parametrize("T,ties,exc", [(1, False, False), (3, False, False), (10, False, False), (2, True, False),
                                        (1, False, True)])
def test_head8_greedy_vs_oracle(lib, T, ties, exc):
    """Greedy pick = argmax of the exact fp32 logits (head.py:19-26, sequential sum), smallest id on ties, with
    the candidate rows decoded from the 12-bit codec (exceptions included); repeated calls agree."""
    from ai_b200.head import Head
    wb, h, c = _head_case(200 + T + 7 * ties + 11 * exc, 3000, 512, T, ties=ties, exceptions=exc)
    hd = Head(from_bits(wb), c)
    H = torch.from_numpy(h).cuda()
    ex = ohead.exact_logits(wb, h)
    want = [int(np.flatnonzero(ex[t] == ex[t].max()).min()) for t in range(T)]
    for _ in range(2):
        got = hd.pick(H, T).cpu().numpy().tolist()
        assert got == want
    if ties:
        assert want[0] == 9 and want[1] == 9
    if exc:
        assert int(c["rp"][34] - c["rp"][33]) > 0 and want[0] == 33
    assert status_clear() == 0


@pytest.mark.parametrize("T,k,ties,exc", [(1, 1, False, False), (1, 20, False, True), (3, 32, True, False),
                                         (2, 5, True, True)])
def test_head8_topk_logits_vs_oracle(lib, T, k, ties, exc):
    """Top-k candidate logits: every row of the exact top k (ties at the k-th value included) is kept with its
    exact fp32 logit (bit-identical to exact_rows, head.py:19-26), every other row is either kept exactly or set
    to -inf, and the rows set to -inf are all below the k-th largest exact logit."""
    from ai_b200.head import Head
    wb, h, c = _head_case(400 + T + 3 * k + 7 * ties + 11 * exc, 3000, 512, T, ties=ties, exceptions=exc)
    hd = Head(from_bits(wb), c)
    H = torch.from_numpy(h).cuda()
    ex = ohead.exact_logits(wb, h)
    out = torch.full((T, 3000), float("nan"), device="cuda")
    for _ in range(2):
        got = hd.topk_logits(H, T, k, out).cpu().numpy()
        for t in range(T):
            kth = np.sort(ex[t])[::-1][k - 1]
            kept = np.isfinite(got[t])
            assert not np.isnan(got[t]).any()
            np.testing.assert_array_equal(got[t][kept], ex[t][kept])
            assert kept[ex[t] >= kth].all()
            assert (ex[t][~kept] < kth).all()
            if not (exc or ties):  # plain random rows: the bounds prune most of the vocabulary
                assert kept.sum() < 3000
    assert status_clear() == 0


# ------------------------------------------------------------------------------ exact vocabulary logits
def _exact(c, h, T):
    from ai_b200.head import exact_logits
    H = torch.from_numpy(np.ascontiguousarray(h, np.float32)).cuda()
    out = torch.full((T, int(c["N"])), float("nan"), device="cuda")
    exact_logits(H, c, T, out)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_exact_logits_reference_golden(lib):
    """Full-vocabulary exact logits are bit-identical to the reference's exact_rows (head.py:19-26) output in
    the golden file. D = 64 there, so rows and h are zero-padded to the codec's 256-column chunk: the padding
    adds exact zeros after the 64 real terms and cannot change a nonzero sequential sum."""
    from ai_b200 import wcomp
    z = golden("head")
    w, h, want = z["w"], z["h"], z["exact"]
    V, D = w.shape
    T = h.shape[0]
    wp = np.zeros((V, 256), np.uint16)
    wp[:, :D] = w
    hp = np.zeros((T, 256), np.float32)
    hp[:, :D] = h
    c = wcomp.compress(from_bits(wp))
    got = _exact(c, hp, T)
    nz = want != 0  # the all-zero row 7 sums to +0 either way
    assert np.array_equal(got[nz].view(np.uint32), want[nz].view(np.uint32))
    assert (got[~nz] == 0).all()
    assert status_clear() == 0


@pytest.mark.parametrize("V,D,T,exc", [(3000, 512, 1, True), (3001, 768, 3, True), (1000, 256, 8, False),
                                       (777, 1024, 11, True), (151936, 1024, 1, False)])
def test_exact_logits_vs_oracle(lib, V, D, T, exc):
    """Bit-exact against the oracle's exact_rows restatement (fp32 products, sequential fp32 sum), with codec
    exceptions (tiny and huge values outside the exponent window) on some rows, ragged V and T > 8 (two
    token passes); the full Qwen3 vocabulary at D = 1024."""
    wb, h, c = _head_case(300 + V + T, V, D, T, exceptions=exc)
    if exc:
        assert int(c["rp"][34] - c["rp"][33]) > 0
    got = _exact(c, h, T)
    want = ohead.exact_logits(wb, h)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"{(got != want).sum()} of {got.size} logits differ"
    assert status_clear() == 0
