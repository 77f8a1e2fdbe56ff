"""BASELINE.json configurations at their stated shapes, on the GPU through the library.

one Qwen3-0.6B-shaped MLP block (gate/up [3072, 1024], down [1024, 3072], N(0, 0.02) bf16, seed 0,
12-bit encoded; x bf16 [1, 1024] N(0, 1); RMSNorm eps 1e-6 with weight 1; SiLU(gate) * up; down_proj) and the
sampler on fp32 logits [1, 151936] N(0, 2) with temperature 0.7, top-k 20, top-p 0.8, repetition penalty 1.05
over 64 prior ids uniform in [0, 151936) and the fixed draw u = 0.37. Inputs come from
np.random.default_rng(0) in that order: gate, up, down, x, logits, prior ids.

Qwen3-0.6B random-init (28 layers, hidden 1024, 16/8 heads, head_dim 128, FF 3072, vocab 151936,
tied), a 128-token prompt of uniform random ids, greedy tokens against the oracle decode that uses the
reference's exact head arithmetic. The test runs 32 tokens (bench.py --parity runs the full 256); at a
divergence it reports the oracle's top-2 logit gap there.
"""
import numpy as np
import pytest
import torch

from oracle import codec, gemv as ogemv, sampler as osamp

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib(cuda_dev):
    from ai_b200 import build, _lib
    build.build()
    return _lib.lib()


def bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def from_bits(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).cuda()


def config0_inputs():
    rng = np.random.default_rng(0)
    gate = codec.f32_to_bf16_bits((rng.standard_normal((3072, 1024)) * 0.02).astype(np.float32))
    up = codec.f32_to_bf16_bits((rng.standard_normal((3072, 1024)) * 0.02).astype(np.float32))
    down = codec.f32_to_bf16_bits((rng.standard_normal((1024, 3072)) * 0.02).astype(np.float32))
    x = codec.bf16_bits_to_f32(codec.f32_to_bf16_bits(rng.standard_normal(1024).astype(np.float32)))
    logits = (rng.standard_normal(151936) * 2.0).astype(np.float32)
    prior = rng.integers(0, 151936, 64).astype(np.int32)
    return gate, up, down, x, logits, prior


def test_config0_mlp_block(lib):
    """The MLP block through the codec GEMVs, in the reference layout (gu = [gate; up] encoded as one matrix, down
    with the SiLU-gated input, mode 2), in the engine's layout (gate/up rows interleaved, gated output, mode 3)
    and with gate and up encoded separately (each its own exponent base): all within the fp32-accumulation bound
    of the float64 oracle."""
    from ai_b200 import wcomp
    gate, up, down, x, _, _ = config0_inputs()
    ones = np.full(1024, 0x3F80, np.uint16)
    xin = ogemv.xin(x, 1024, 0, ones, 1e-6)
    g = (codec.bf16_bits_to_f32(gate).astype(np.float64) @ xin.astype(np.float64)).astype(np.float32)
    u = (codec.bf16_bits_to_f32(up).astype(np.float64) @ xin.astype(np.float64)).astype(np.float32)
    mid = ogemv.silu_mul(g, u)
    Wd = codec.bf16_bits_to_f32(down).astype(np.float64)
    want = (Wd @ mid.astype(np.float64)).astype(np.float32)
    mag = np.abs(Wd) @ np.abs(mid.astype(np.float64))
    X = torch.from_numpy(x).cuda()
    lnw = from_bits(ones)
    cd = wcomp.compress(from_bits(down))
    # reference layout
    gu = torch.zeros(6144, device="cuda")
    wcomp.gemvc1(X, wcomp.compress(from_bits(np.concatenate([gate, up]))), gu, 0, lnw=lnw, eps=1e-6)
    y = torch.zeros(1024, device="cuda")
    wcomp.gemvc1(gu, cd, y, 2)
    # engine layout
    gi = wcomp.interleave_gate_up(from_bits(np.concatenate([gate, up])))
    m = torch.zeros(3072, device="cuda")
    wcomp.gemvc1(X, wcomp.compress(gi), m, 3, lnw=lnw, eps=1e-6)
    y3 = torch.zeros(1024, device="cuda")
    wcomp.gemvc1(m, cd, y3, 1)
    # separately encoded gate and up
    gs, us = torch.zeros(3072, device="cuda"), torch.zeros(3072, device="cuda")
    wcomp.gemvc1(X, wcomp.compress(from_bits(gate)), gs, 0, lnw=lnw, eps=1e-6)
    wcomp.gemvc1(X, wcomp.compress(from_bits(up)), us, 0, lnw=lnw, eps=1e-6)
    ys = torch.zeros(1024, device="cuda")
    wcomp.gemvc1(torch.cat([gs, us]), cd, ys, 2)
    torch.cuda.synchronize()
    for got in (y, y3, ys):
        d = np.abs(got.cpu().numpy().astype(np.float64) - want)
        assert (d <= 1e-4 * mag + 1e-6).all(), d.max()
    from ai_b200._lib import status
    assert status() == 0


@pytest.mark.parametrize("two_phase", [False, True])
def test_config0_sampler(lib, two_phase):
    """The configs[0] sampler case: the id equals the oracle's (penalty, temperature, top-k, top-p, u = 0.37)."""
    from ai_b200 import sampler
    *_, logits, prior = config0_inputs()
    L = torch.from_numpy(logits).cuda()[None]
    P = torch.from_numpy(prior).cuda()[None]
    got = sampler.sample(L, temperature=0.7, top_p=0.8, top_k=20, us=[0.37], prior=P, repetition_penalty=1.05,
                         two_phase=two_phase)
    want = osamp.sample_row(logits, 0.7, 20, 0.8, rep=1.05, prior_ids=prior, u=0.37)
    assert got == [want]


def test_qwen3_0p6b_greedy_matches_oracle(lib):
    from ai_b200.engine import Engine
    from ai_b200.model import CONFIGS, RandomWeights
    from oracle.model import DecodeOracle
    cfg = CONFIGS["qwen3-0.6b"]
    rw = RandomWeights(cfg, seed=0)
    prompt = [int(t) for t in np.random.default_rng(0).integers(0, cfg.V, 128)]
    n = 32
    eng = Engine(cfg, maxt=256, weights=rw, log=None)
    toks = list(eng.generate(prompt, max_new=n))
    del eng
    torch.cuda.empty_cache()
    layers = [{k: bits(v) for k, v in rw.layer(i).items()} for i in range(cfg.L)]
    o = DecodeOracle(cfg, layers, bits(rw.embedding()), bits(rw.head()), bits(rw.final_norm()), 256,
                     exact_head=True, codec_roundtrip=False)
    ref, lgs = o.greedy(prompt, n)
    ref = ref[:len(toks)]
    if toks != ref:
        i = next(j for j, (a, b) in enumerate(zip(toks, ref)) if a != b)
        top2 = np.sort(lgs[i])[-2:]
        pytest.fail(f"token {i}: engine {toks[i]} oracle {ref[i]}; oracle top-2 gap {top2[1] - top2[0]:.3e}")
    from ai_b200._lib import status
    assert status() == 0
