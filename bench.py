"""Benchmark: Qwen3-8B 12-bit decode tokens/s at batch 1 (BASELINE.json `metric`, `configs[2]`).

Workload (one "step" = one decode pass of one token): random-init Qwen3-8B (N(0,0.02) bf16 matrices encoded in
the 12-bit codec), bf16 KV cache pre-filled to 4096 positions from N(0,1), sampling top-k 20 / top-p 0.8 /
temperature 0.6, on one B200 per rank. The 10.4 GB of weights streamed per step exceed the 126 MB L2, so no
explicit flush is needed between steps.

  value  = tokens/s with inputs resident: K CUDA-graph replays timed with CUDA events (ids / position chained
           on the device), max over ranks. N > 1 runs one sequence tensor-parallel over the N ranks (BASELINE
           configs[2], "scaling": "strong"); --replicas runs N independent sequences instead ("weak").
  e2e    = tokens/s through the public API, Engine.generate (host u draw in, host token id out every step).
  roofline = the dominant kernel, the codec GEMV: algorithmic bytes (12-bit planes + CSR) per launch over its
           CUDA-event duration, for the 5 matrices of a layer + the head, against MEASURED_PEAKS.json.
  cpu_baseline = the reference's CPU decode path (its Numba CpuLayer kernels + exact_rows head, restated
           bit-identically in oracle/cpu_ref.py) on the host cores, a bounded sample scaled to one token.

`--impl reference` times that CPU path alone (the reference package itself does not travel to the GPU box; its
Numba kernels, restated, stand in) and prints its own JSON line.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CTX = 4096
SAMPLING = dict(temperature=0.6, top_k=20, top_p=0.8)
METRIC = "decode tok/s Qwen3-8B bs1 12-bit weights"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampler run during a timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "100"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm = [float(r[1]) for r in self.rows if len(r) > 2 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) > 2 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows if len(r) >= 9 for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": float(sorted(sm)[len(sm) // 2]) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(sm)}


# ---------------------------------------------------------------------------------- CPU baseline
def cpu_baseline(layer_reps=36, head_frac=4):
    """The reference's CPU decode path on the host cores: its Numba CpuLayer kernels and exact_rows head
    (`ramvi_engine/cpu/cpu_layer.py`, `generation/head.py:19-26`, restated bit-identically in oracle/cpu_ref.py --
    oracle/check_cpu_ref.py compares both in the build container), all host threads. Bounded sample: one Qwen3-8B
    layer (bf16 weights, fp32 KV cache at ctx 4096) run `layer_reps` times and 1/head_frac of the vocabulary's
    exact logits, scaled to one token (36 layers + the whole head). Also times BASELINE configs[0], the
    Qwen3-0.6B MLP block (RMSNorm, gate/up, SiLU*up, down)."""
    import numba
    import numpy as np
    from ai_b200.model import CONFIGS
    from oracle import codec, cpu_ref, attn
    numba.set_num_threads(numba.config.NUMBA_NUM_THREADS)
    cfg = CONFIGS["qwen3-8b"]
    rng = np.random.default_rng(0)
    P = cfg.layer_params()
    W = {n: codec.f32_to_bf16_bits((rng.standard_normal(P[n], dtype=np.float32) * 0.02)) for n in P}
    one_d, one_h = np.ones(cfg.D, np.float32), np.ones(cfg.HD, np.float32)
    lay = cpu_ref.CpuLayer(W["qkv"], W["o"], W["gu"], W["down"], one_d, one_d, one_h, one_h, cfg, CTX + 8)
    lay.K[:, :CTX] = rng.standard_normal((cfg.KV, CTX, cfg.HD), dtype=np.float32)
    lay.V[:, :CTX] = rng.standard_normal((cfg.KV, CTX, cfg.HD), dtype=np.float32)
    inv = attn.rope_inv(cfg.HD, cfg.theta)
    x = rng.standard_normal((1, cfg.D), dtype=np.float32)
    rows = cfg.V // head_frac
    hw = codec.f32_to_bf16_bits(rng.standard_normal((rows, cfg.D), dtype=np.float32) * 0.02)
    toks, trow, lg = np.arange(rows), np.zeros(rows, np.int64), np.empty(rows, np.float32)
    h = rng.standard_normal((1, cfg.D), dtype=np.float32)
    lay(x.copy(), CTX, inv)  # JIT compile outside the timed region
    cpu_ref.exact_rows(hw, toks, trow, h, lg)
    t0 = time.perf_counter()
    for _ in range(layer_reps):
        lay(x, CTX, inv)
    t1 = time.perf_counter()
    cpu_ref.exact_rows(hw, toks, trow, h, lg)
    t2 = time.perf_counter()
    sec = (t1 - t0) / layer_reps * cfg.L + (t2 - t1) * head_frac
    # Qwen3-0.6B MLP block (gu fused [6144, 1024], down [1024, 3072]), x bf16 N(0, 1)
    c6 = CONFIGS["qwen3-0.6b"]
    g0 = np.random.default_rng(0)
    gate = codec.f32_to_bf16_bits((g0.standard_normal((c6.FF, c6.D)) * 0.02).astype(np.float32))
    up = codec.f32_to_bf16_bits((g0.standard_normal((c6.FF, c6.D)) * 0.02).astype(np.float32))
    down = codec.f32_to_bf16_bits((g0.standard_normal((c6.D, c6.FF)) * 0.02).astype(np.float32))
    gu = np.concatenate([gate, up])
    xb = codec.bf16_bits_to_f32(codec.f32_to_bf16_bits(g0.standard_normal((1, c6.D)).astype(np.float32)))

    def block():
        hh = np.empty_like(xb)
        cpu_ref.rms_rows(xb, np.ones(c6.D, np.float32), hh, np.float32(1e-6))
        g2 = np.empty((1, 2 * c6.FF), np.float32)
        cpu_ref.matmat16(gu, hh, g2, False)
        m = np.empty((1, c6.FF), np.float32)
        cpu_ref.silu_mul(g2, m, c6.FF)
        y = np.zeros((1, c6.D), np.float32)
        cpu_ref.matmat16(down, m, y, False)
    block()
    bt = min(_timed(block) for _ in range(20))
    return {"value": 1.0 / sec, "unit": "tok/s", "cores": numba.get_num_threads(), "kind": "port",
            "sample": f"{layer_reps} runs of one Qwen3-8B layer (bf16 weights, fp32 KV at ctx {CTX}) and 1/{head_frac} "
                      f"of the exact-logit head, scaled to one token; the reference's Numba CpuLayer/exact_rows "
                      f"kernels restated bit-identically in oracle/cpu_ref.py; measured {t2 - t0:.2f} s",
            "config0_mlp_block_us": round(bt * 1e6, 1),
            "config0_mlp_block_gbs": round((gu.size + down.size) * 2 / bt / 1e9, 1)}


def _timed(fn):
    t = time.perf_counter()
    fn()
    return time.perf_counter() - t


# ------------------------------------------------------------------------------------ GPU arm
def gemv_roofline(eng, peak, reps=20):
    """The dominant kernel of the decode step, the codec GEMV, timed alone (CUDA events on the launching stream)
    as the engine runs it: one layer's four matrices in the engine's modes (qkv with the RMS prologue, o +=,
    gate/up gated, down +=), back to back. achieved = their algorithmic bytes (12-bit planes + CSR) / time. The
    vocabulary head -- the exact-logit kernel the sampling step runs -- is reported beside it."""
    import torch
    from ai_b200 import wcomp
    from ai_b200.head import exact_logits
    W, s = eng.W[0], eng.small[0]
    gu_mode, down_mode = (3, 1) if eng.gated else (0, 2)  # the engine's own modes
    gws = eng.gws if eng.gated else None  # gate/up with the engine's stream-K workspace
    launches = [(W["qkv"], eng.xb[0], eng.qkvb[0], 0, s["ln1"], None), (W["o"], eng.attb[0], eng.xb[1], 1, None, None),
                (W["gu"], eng.xb[0], eng.gub[0], gu_mode, s["ln2"], gws),
                (W["down"], eng.gub[0], eng.xb[1], down_mode, None, None)]
    eng.xb[:2].normal_()
    eng.attb[0].normal_()
    eng.gub[0].normal_()
    total_bytes = sum(c.nbytes for c, *_ in launches)
    st = torch.cuda.current_stream()

    def run_layer():
        for c, x, y, m, lnw, ws in launches:
            wcomp.gemvc1(x, c, y, m, lnw=lnw, eps=eng.eps, ws=ws)

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(reps):
            fn()
        e1.record(st)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 1e3 / reps

    sec = timed(run_layer)
    achieved = total_bytes / sec / 1e9
    hsec = timed(lambda: exact_logits(eng.hb[:1], eng.head, 1, eng.logits[:1]))
    # DRAM traffic per launch: the ncu capture of one gate/up-shaped launch (profiles/gemv_tc_gu.md: read + write
    # bytes over the launch's algorithmic bytes), scaled to this average launch by its algorithmic bytes
    per_launch = total_bytes // len(launches)
    traffic, ratio = None, None
    tp = os.path.join(ROOT, "profiles", "gemv_tc_gu.md")
    if os.path.exists(tp):
        for line in open(tp):
            if line.startswith("| traffic / algorithmic bytes |"):
                ratio = float(line.rsplit("=", 1)[1].strip(" |\n"))
        if ratio:
            traffic = int(per_launch * ratio)
    return {"bound": "hbm", "kernel": "aib gemv_tc_kernel (codec GEMV, T=1): one layer's qkv, o, gate/up, down",
            "achieved": round(achieved, 1), "peak": peak[0], "peak_kind": peak[1], "unit": "GB/s",
            "frac": round(achieved / peak[0], 4), "traffic": traffic,
            "traffic_source": "ncu 24576x4096 launch, scaled by algorithmic bytes" if traffic else None,
            "algorithmic_bytes_per_launch": per_launch, "avg_launch_us": round(sec / len(launches) * 1e6, 2),
            "head": {"kernel": "aib exact_logits_kernel (full-vocabulary exact logits)", "bytes": eng.head.nbytes,
                     "us": round(hsec * 1e6, 1), "GBps": round(eng.head.nbytes / hsec / 1e9, 1),
                     "frac": round(eng.head.nbytes / hsec / 1e9 / peak[0], 4)}}


def bench_prefill(eng, n=2048, reps=3):
    """Whole-prompt prefill of an n-token random prompt (BASELINE configs[4] runs 2048 tokens): tokens/s, and the
    tensor-pipe fraction of the linear layers' algorithmic FLOPs (2 * n * params, counted once -- the default
    precision-3 GEMMs execute three bf16 MMAs per product) against the measured bf16 peak."""
    import numpy as np
    import torch
    from ai_b200 import sampler
    toks = [int(t) for t in np.random.default_rng(5).integers(0, eng.V, n)]
    prm = sampler.params()
    eng._prefill(toks, 0, prm, None, False)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        eng._prefill(toks, 0, prm, None, False)
    e1.record()
    torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / reps
    params = sum(int(c["N"]) * int(c["K"]) for c in eng.W[0].values()) * eng.L
    lin = 2.0 * n * params
    att = 2.0 * 2 * eng.L * eng.H * eng.HD * n * (n + 1) / 2
    tf = bf16_peak()
    return {"tokens": n, "ms": round(sec * 1e3, 2), "tok_s": round(n / sec, 1), "precision": eng.prefill_precision,
            "linear_tflops": round(lin / sec / 1e12, 1), "attention_tflops": round(att / sec / 1e12, 2),
            "tensor_frac_algorithmic": round(lin / sec / 1e12 / tf[0], 4),
            "tensor_frac_executed": round(eng.prefill_precision * lin / sec / 1e12 / tf[0], 4),
            "peak_tflops": tf[0], "peak_kind": tf[1]}


def bench_batch(eng, B=8, steps=16, warmup=3):
    """BASELINE configs[2] at batch 8: B sequences, each with its own KV cache pre-filled N(0, 1) to 4096
    positions, decoded together (one weight read per step), top-k 20 / top-p 0.8 / T 0.6."""
    import torch
    from ai_b200 import sampler
    bt = eng._batch(B)
    g = torch.Generator(device=eng.device).manual_seed(77)
    bt.kv[:, :, :, :, :CTX].normal_(generator=g)
    bt.ids.random_(0, eng.V, generator=g)
    bt.u.uniform_(generator=g)
    prm = sampler.params(**SAMPLING)
    bt.pos.fill_(CTX)
    for _ in range(warmup):
        bt.run(prm)
    bt.pos.fill_(CTX)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        bt.run(prm)
    e1.record()
    torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / steps
    nb = bt.bytes_per_step(CTX + steps // 2)
    hbm = peaks()
    out = {"batch": B, "ms_per_step": round(sec * 1e3, 3), "tok_s": round(B / sec, 1), "bytes_per_step": nb,
           "achieved_gbs": round(nb / sec / 1e9, 1), "frac": round(nb / sec / 1e9 / hbm[0], 4)}
    del eng._bt
    return out


def bf16_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def gpu_arm(args, rank, world):
    import torch
    import torch.distributed as dist
    from ai_b200 import build
    from ai_b200.engine import Engine
    build.build()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    maxt = CTX + 2 * (args.steps + args.warmup) + 64
    tp = 1 if args.replicas else world
    # replicas: one sequence per GPU (own weights seed); tensor parallel: one sequence over all ranks
    seq = 0 if tp > 1 else rank
    eng = Engine("qwen3-8b", maxt=maxt, seed=seq, log=None, tp=tp)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    eng.kv[:, :, :, :CTX].normal_(generator=g)
    torch.cuda.synchronize()
    from ai_b200 import sampler
    import numpy as np
    samp = dict(temperature=0.0, top_k=0, top_p=1.0) if args.greedy else SAMPLING
    prm = sampler.params(**samp)
    rng = np.random.default_rng(seq)
    eng.u.copy_(torch.from_numpy(rng.random(16)))
    eng.ids[0] = 1
    eng.pos.fill_(CTX)
    for _ in range(max(args.warmup, 1)):
        eng._run(1, prm, 1, False)
    torch.cuda.synchronize()
    eng.pos.fill_(CTX)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(dev.index) as ck:
        e0.record(st)
        for _ in range(args.steps):
            eng._run(1, prm, 1, False)
        e1.record(st)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    nseq = 1 if tp > 1 else world  # sequences decoded by the whole job
    value = nseq * args.steps / (ms_max / 1e3)
    # e2e through the public API: Engine.generate, host buffers every step
    eng.ctx = [1] * CTX
    prompt = eng.ctx + [1]
    stats = {}
    with Clocks(dev.index) as ck2:
        n = 0
        for _ in eng.generate(prompt, max_new=args.steps + 1, seed=seq, stats=stats, **samp):
            n += 1
    e2e_local = stats["decode_n"] / (stats["gen_ms"] / 1e3)
    te = torch.tensor([stats["gen_ms"]], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e = nseq * stats["decode_n"] / (float(te.item()) / 1e3)
    peak = peaks()
    roof = gemv_roofline(eng, peak) if rank == 0 else None
    step_bytes = eng.bytes_per_token(CTX + args.steps // 2)
    from ai_b200._lib import status
    dev_status = status()
    extra = {}
    if rank == 0 and tp == 1 and not args.no_extra:
        extra["prefill"] = bench_prefill(eng)
        extra["batch"] = bench_batch(eng)
    if tp > 1:
        eng.close()  # its graphs hold NCCL calls: release them before the process group goes
    if rank != 0:
        return None
    # embed, 5 per layer (qkv GEMV, attention, o, gate/up, down), final norm, then sampling: exact logits +
    # sampler (2 phases), or greedy: bounds, candidates, exact pick; advance
    launches_per_step = 1 + 5 * eng.L + 1 + 3 + 1
    out = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
        "scaling": "strong" if tp > 1 else "weak", "vs_baseline": None, "dtype": "fp32 activations x exact bf16 weights (12-bit codec), "
        "bf16 KV", "data": "synthetic (random-init N(0,0.02) weights, KV pre-filled N(0,1) to 4096)",
        "config": {"workload": "Qwen3-8B decode bs1, 12-bit weights, ctx 4096->, " +
                   ("greedy (int8 head + exact candidates)" if args.greedy else "top-k 20 / top-p 0.8 / T 0.6"),
                   "model": "qwen3-8b", "global_batch": nseq, "seq_len": CTX,
                   "parallelism": f"tp{tp}" if tp > 1 else ("replicas" if world > 1 else "single"),
                   "l2": "weights (10.4 GB) > L2 every step"},
        "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8,
                "per_rank": round(e2e_local, 2)},
        "roofline": roof,
        "step_roofline": {"bytes_per_token": step_bytes, "per": "rank",
                          "achieved_gbs": round(step_bytes * value / nseq / 1e9, 1),
                          "frac": round(step_bytes * value / nseq / 1e9 / peak[0], 4)},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": ck.summary(), "clocks_e2e": ck2.summary(), "device_status": dev_status,
        **extra,
    }
    if not args.no_cpu:
        out["cpu_baseline"] = cpu_baseline()
    return out


def micro_attn(args):
    """Fused T=1 attention of a Qwen3-8B layer at position 4096 (bf16 KV, 8 groups x 4 heads). Successive
    calls walk the 36 layers' caches (680 MB), as the decode step does, so the K/V rows come from HBM."""
    import torch
    from ai_b200 import tkernels
    H, KV, HD, maxt, pos, L = 32, 8, 128, 4608, CTX, 36
    g = torch.Generator(device="cuda").manual_seed(0)
    kv = torch.randn(L, 2, KV, maxt, HD, generator=g, device="cuda").bfloat16()
    qkv = torch.randn((H + 2 * KV) * HD, generator=g, device="cuda")
    qn = torch.ones(HD, dtype=torch.bfloat16, device="cuda")
    inv = (1.0 / (1e6 ** (torch.arange(0, HD, 2, dtype=torch.float32) / HD))).cuda()
    P = torch.tensor([pos], device="cuda")
    out = torch.zeros(H * HD, device="cuda")
    nbytes = 2 * KV * (pos + 1) * HD * 2
    calls = [0]

    def run():
        layer = calls[0] % L
        calls[0] += 1
        tkernels.rope_attn(qkv, qn, qn, inv, P, kv[layer, 0], kv[layer, 1], out, maxt, 1e-6, HD ** -0.5, H, KV, HD)
    return run, nbytes


def micro_head8(args):
    """Greedy pick through the int8 head at the Qwen3-8B vocabulary size (151936 x 4096): int8 bounds over the
    622 MB copy, then exact logits of the candidate rows from the 12-bit head. Returns (bounds-only, full pick)
    callables and the int8 bytes of one bounds pass."""
    import torch
    from ai_b200 import wcomp
    from ai_b200.head import Head
    g = torch.Generator(device="cuda").manual_seed(0)
    V, D = 151936, 4096
    w = (torch.randn(V, D, generator=g, device="cuda") * 0.02).bfloat16()
    hd = Head(w, wcomp.compress(w), TM=1)
    del w
    h = torch.randn(1, D, generator=g, device="cuda")
    return (lambda: hd.bounds(h, 1)), (lambda: hd.pick(h, 1)), V * D + 16 * V


def micro_sample(args):
    """Sampler on one [1, 151936] fp32 logits row, top-k 20 / top-p 0.8 / T 0.6."""
    import torch
    from ai_b200 import sampler
    g = torch.Generator(device="cuda").manual_seed(0)
    lg = torch.randn(1, 151936, generator=g, device="cuda") * 2
    out = torch.zeros(1, dtype=torch.int64, device="cuda")
    u = torch.full((1,), 0.37, dtype=torch.float64, device="cuda")
    prm = sampler.params(**SAMPLING)
    ws = sampler.workspace(1, lg.shape[-1], lg.device)  # the engine's two-phase path
    return (lambda: sampler.sample_into(lg, out, prm, u, ws=ws)), lg.numel() * 4


def micro(args):
    """One kernel alone on a small case (for ncu captures and quick A/B timing), timed as `--steps` calls
    captured in one CUDA graph and replayed (device time, no host launch overhead). gemv: the codec GEMV on a
    Qwen3-8B gu-shaped matrix [24576, 4096] (151 MB of planes, > L2), T = 1 with the RMS prologue;
    gemv_down: [4096, 12288] with the SiLU-gated input; gemv_qkv / gemv_o: the [6144, 4096] / [4096, 4096]
    matrices; attn: a layer's decode attention at ctx 4096 (K/V from HBM);
    sample: the sampler on one vocabulary row."""
    import torch
    from ai_b200 import build, wcomp, _lib
    build.build()
    torch.cuda.set_device(0)
    if args.gemv_variant is not None:
        _lib.call("aib_debug_knob", 4, args.gemv_variant)
    def timed(run, reps):
        """Device time per call: `reps` calls captured in one CUDA graph (no host launch overhead), replayed."""
        for _ in range(3):
            run()
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                for _ in range(reps):
                    run()
        torch.cuda.current_stream().wait_stream(s)
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / reps

    if args.micro == "head8":
        bnd, pick, nbytes = micro_head8(args)
        ub = timed(bnd, max(args.steps, 1))
        up = timed(pick, max(args.steps, 1))
        print(json.dumps({"micro": "head8", "bytes": nbytes, "bounds_us": round(ub, 2),
                          "bounds_GBps": round(nbytes / ub / 1e3, 1), "pick_us": round(up, 2),
                          "device_status": _lib.status()}))
        return
    if args.micro in ("gemm", "gemm1"):  # prefill GEMM, gate/up-shaped [24576, 4096] over 2048 prompt rows
        from ai_b200 import prefill
        g = torch.Generator(device="cuda").manual_seed(0)
        c = wcomp.compress((torch.randn(24576, 4096, generator=g, device="cuda") * 0.02).bfloat16())
        M, prec = 2048, (3 if args.micro == "gemm" else 1)
        X = torch.randn(M, 4096, generator=g, device="cuda")
        Y = torch.empty(M, 24576, device="cuda")
        ws = prefill.workspace(M, 4096, prec)
        us = timed(lambda: prefill.matrix(X, c, Y, precision=prec, ws=ws), max(args.steps, 1))
        fl = 2.0 * M * 24576 * 4096
        print(json.dumps({"micro": args.micro, "M": M, "N": 24576, "K": 4096, "precision": prec,
                          "us_per_launch": round(us, 1), "tflops_algorithmic": round(fl / us / 1e6, 1),
                          "tflops_executed": round(prec * fl / us / 1e6, 1), "device_status": _lib.status()}))
        return
    if args.micro == "exact":  # exact logits of the whole Qwen3-8B vocabulary for one row
        from ai_b200.head import exact_logits
        g = torch.Generator(device="cuda").manual_seed(0)
        c = wcomp.compress((torch.randn(151936, 4096, generator=g, device="cuda") * 0.02).bfloat16())
        h = torch.randn(1, 4096, generator=g, device="cuda")
        out = torch.empty(1, 151936, device="cuda")
        us = timed(lambda: exact_logits(h, c, 1, out), max(args.steps, 1))
        print(json.dumps({"micro": "exact", "bytes": c.nbytes, "us_per_launch": round(us, 1),
                          "GBps": round(c.nbytes / us / 1e3, 1), "device_status": _lib.status()}))
        return
    if args.micro == "sampler_sweep":
        import numpy as np
        from ai_b200 import sampler
        V, res = 151936, []
        for B in (1, 16, 64, 256):
            g = torch.Generator(device="cuda").manual_seed(B)
            lg = torch.randn(B, V, generator=g, device="cuda") * 3.0
            prior = torch.randint(0, V, (B, 1024), generator=g, device="cuda", dtype=torch.int32)
            bits = np.random.default_rng(B).random((B, (V + 31) // 32 * 32)) < 0.1  # 10 % of tokens allowed
            packed = np.packbits(bits, axis=1, bitorder="little").view(np.int32).copy()  # bit j of word w: 32w + j
            packed[:, 0] |= 1
            mask = torch.from_numpy(packed).cuda()
            u = torch.from_numpy(np.array([np.random.default_rng(r).random() for r in range(B)])).cuda()
            out = torch.zeros(B, dtype=torch.int64, device="cuda")
            ws = sampler.workspace(B, V, lg.device)
            for k in (1, 20, 50):
                for p in (0.8, 0.95):
                    prm = sampler.params(0.7, k, p, 1.1, 0.5, 0.3)
                    us = timed(lambda: sampler.sample_into(lg, out, prm, u, prior, mask, ws=ws), max(args.steps, 1))
                    nb = B * V * 4 + mask.numel() * 4 + prior.numel() * 4
                    res.append({"B": B, "top_k": k, "top_p": p, "us": round(us, 2), "GBps": round(nb / us / 1e3, 1)})
        print(json.dumps({"micro": "sampler_sweep", "rows": res, "device_status": _lib.status()}))
        return
    if args.micro in ("attn", "sample"):
        run, nbytes = (micro_attn if args.micro == "attn" else micro_sample)(args)
        us = timed(run, max(args.steps, 1))
        print(json.dumps({"micro": args.micro, "bytes": nbytes, "us_per_launch": round(us, 2),
                          "GBps": round(nbytes / us / 1e3, 1)}))
        return
    g = torch.Generator(device="cuda").manual_seed(0)
    # Qwen3-8B layer shapes: (N, K, mode, RMS prologue)
    N, K, mode, rms = {"gemv": (24576, 4096, 0, True), "gemv_down": (4096, 12288, 2, False),
                       "gemv_qkv": (6144, 4096, 0, True), "gemv_o": (4096, 4096, 1, False)}[args.micro]
    c = wcomp.compress((torch.randn(N, K, generator=g, device="cuda") * 0.02).bfloat16())
    x = torch.randn(K * 2, generator=g, device="cuda")
    y = torch.zeros(N, device="cuda")
    lnw = torch.ones(K, dtype=torch.bfloat16, device="cuda")
    ws = wcomp.gemv_workspace([c], x.device) if args.streamk else None
    run = lambda: wcomp.gemvc1(x, c, y, mode, lnw=lnw if rms else None, ws=ws)  # noqa: E731
    us = timed(run, max(args.steps, 1))
    torch.cuda.synchronize()
    st = _lib.status()
    print(json.dumps({"micro": args.micro, "variant": args.gemv_variant, "streamk": bool(args.streamk),
                      "device_status": st, "N": N, "K": K, "bytes": c.nbytes, "us_per_launch": round(us, 2),
                      "GBps": round(c.nbytes / us / 1e3, 1)}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--micro", choices=["gemv", "gemv_down", "gemv_qkv", "gemv_o", "attn", "sample", "head8", "gemm",
                                        "gemm1", "exact", "sampler_sweep"],
                    default=None,
                    help="time one kernel alone on a small case (for ncu) instead of the decode benchmark")
    ap.add_argument("--gemv-variant", type=int, default=None, choices=[1, 3, 4],
                    help="codec GEMV kernel for --micro (test knob 4): 1 CUDA-core 12 KB stages, 3 tensor-core wide stages with two CTAs per SM where they fit (default), 4 tensor-core 48 KB stages, one CTA per SM")
    ap.add_argument("--streamk", action="store_true", help="--micro gemv*: pass the stream-K workspace")
    ap.add_argument("--greedy", action="store_true",
                    help="greedy decoding (the int8 head's exact-candidate pick) instead of the default sampling")
    ap.add_argument("--tp", action="store_true", help="tensor parallel over the N ranks (the default for N > 1)")
    ap.add_argument("--replicas", action="store_true",
                    help="with --gpus N under torchrun: N independent sequences, one per GPU, instead of one sequence "
                         "tensor-parallel over the N ranks")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the prefill (2048-token prompt) and batch-8 decode measurements of the default run")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.micro:
        return micro(args)
    if args.impl == "reference":
        if rank != 0:
            return
        cb = cpu_baseline(layer_reps=max(36, min(args.steps, 72)))
        v = cb["value"]
        print(json.dumps({"impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus,
                          "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                          "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
                          "config": {"workload": "Qwen3-8B decode bs1, ctx 4096 (the reference's Numba CPU path, "
                                                 "bf16 weights)",
                                     "model": "qwen3-8b", "global_batch": 1, "seq_len": CTX},
                          "cpu_baseline": cb, "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0,
                                                      "d2h_bytes_per_step": 0}}))
        return
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    try:
        out = gpu_arm(args, rank, world)
        if out is not None:
            print(json.dumps(out))
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
