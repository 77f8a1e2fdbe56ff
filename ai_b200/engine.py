"""Qwen3 decode engine on the 12-bit codec -- the reference `Engine` surface (core/engine.py:195-803) on sm_100a.

Load (`Engine.__init__`, core/engine.py:196-263): the reference encodes each fused matrix (qkv = [q;k;v],
gu = [gate;up], formats/model.py:92-102) with `compress` on the GPU; here the device encoder of
libai_b200.so does it. All layers stay resident (a B200 holds any dense model up to ~100B params in the
12-bit codec), so the reference's gpu/stream/cpu placement, pinned arena and loader thread have no
counterpart.

Step (`_gpu_layer` :329-341 for T = 1, `_batch_layer` :344-356 for T <= 16), captured once per shape in a
CUDA graph (`_capture` :415-444) and replayed with the position and the input ids in device memory:
    embed(ids) -> per layer: gemv(qkv, RMS ln1) -> rope_attn -> gemv(o, +=) -> gemv(gu, RMS ln2) -> gemv(down,
    silu*up, +=)  -> final RMSNorm -> head -> advance(ids, pos)
T > 1 uses rmsnorm + batched gemv + qk_rope_cache + cached attention. The head is the reference's `Head.pick`
(generation/head.py:59-88) on the device: greedy steps take the int8 bounds + exact candidate logits, sampling
steps the exact logits of the whole vocabulary (the reference computes those on the CPU after a D2H copy), then
the device sampler: one 8-byte read per generated token.

`process(tokens, pos0, ...)` and `generate(prompt, ...)` keep the reference arguments and errors
(core/engine.py:489-694), with top_k / penalties added. Prompts longer than 16 tokens that need only the last
pick run through the whole-prompt prefill (`ai_b200.prefill`: tcgen05 codec GEMMs + causal flash attention,
the reference's blocked path, core/engine.py:446-487); others run in 16-token batched chunks (the reference's
legacy path, core/engine.py:471-480).
"""
import gc
import os
import time

import numpy as np
import torch

from .head import Head as Head8, exact_logits
from . import _lib, wcomp, tkernels, sampler, codecfile, prefill
from ._lib import ptr, stream_ptr
from .model import CONFIGS, Ckpt, RandomWeights, Qwen3Config, check_tp, shard_layer


def _collect_before_capture():
    """Collect unreachable Python objects before a CUDA-graph capture. torch no longer does this by default, and a
    collection that runs during the capture and frees an object holding CUDA resources (a dropped engine's graphs,
    for instance) makes a call that invalidates the capture."""
    gc.collect()

MATS = ("qkv", "o", "gu", "down")
MAXB = 16


class Engine:
    def __init__(self, name, maxt=2048, device="cuda", seed=0, log=print, norm_noise=0.0, weights=None,
                 graphs=True, head8=True, tp=1, codec_cache=None, prefill_precision=3):
        """name: an HF Qwen3 folder, or a key of ai_b200.model.CONFIGS / a Qwen3Config for random-init
        weights (N(0, 0.02) matrices, seed `seed`). weights: an explicit weight source (RandomWeights/Ckpt).
        head8: greedy steps without penalties pick through the int8 head (the reference's Head: bounds over an
        int8 copy, exact fp32 logits of the candidates) instead of the full 12-bit head GEMV + sampler.
        tp: tensor-parallel ranks (> 1 needs an initialised torch.distributed group of that size, one rank per
        GPU, every rank making the same calls): each rank holds its KV groups' share of every layer
        (`model.shard_layer`), and one all-reduce after o_proj and after down_proj sums the ranks' partial
        residual updates. Embedding, final norm, head and sampler are replicated: every rank picks the same
        token from the same all-reduced state.
        codec_cache: path of a `codecfile` with this model's encoded matrices (per tensor-parallel rank: the
        path gets a `.tp{N}r{rank}` suffix). Loaded when present and made for this model and layout,
        written after encoding otherwise.
        prefill_precision: activations of the whole-prompt prefill GEMMs as three bf16 parts (3, fp32-accurate
        products, the reference's fp32 mm_k) or one (1, bf16, three times the tensor throughput)."""
        if not isinstance(maxt, int) or isinstance(maxt, bool) or maxt < 1:
            raise ValueError("maxt must be a positive integer")
        t0 = time.time()
        dev = torch.device(device)
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        torch.cuda.set_device(dev)
        if weights is not None:
            src = weights
            cfg = weights.cfg if hasattr(weights, "cfg") else weights.config
        elif isinstance(name, Qwen3Config):
            cfg, src = name, RandomWeights(name, seed=seed, norm_noise=norm_noise, device="cuda")
        elif isinstance(name, str) and name in CONFIGS:
            cfg = CONFIGS[name]
            src = RandomWeights(cfg, seed=seed, norm_noise=norm_noise, device="cuda")
        else:
            src = Ckpt(name)
            cfg = src.config
        self.cfg = cfg
        if prefill_precision not in (1, 3):
            raise ValueError("prefill_precision must be 1 or 3")
        self.prefill_precision = prefill_precision
        self.tp, self.tp_rank = int(tp), 0
        if self.tp > 1:
            import torch.distributed as dist
            if not dist.is_initialized() or dist.get_world_size() != self.tp:
                raise ValueError("tp > 1 needs an initialised torch.distributed group of that size")
            check_tp(cfg, self.tp)
            self.tp_rank = dist.get_rank()
        # per-rank shapes (the whole model when tp == 1); Vs: the rank's share of the vocabulary head
        self.L, self.D, self.HD, self.V = cfg.L, cfg.D, cfg.HD, cfg.V
        if self.tp > 1 and cfg.V % self.tp:
            raise ValueError(f"vocabulary {cfg.V} does not split over {self.tp} ranks")
        self.Vs = cfg.V // self.tp
        self.H, self.KV, self.FF = cfg.H // self.tp, cfg.KV // self.tp, cfg.FF // self.tp
        self.eps, self.maxt, self.log = cfg.eps, maxt, log
        self.eos = set(cfg.eos)
        dev = self.device
        self.inv = (1.0 / (cfg.theta ** (torch.arange(0, self.HD, 2, dtype=torch.float32) / self.HD))).to(dev)
        # ---- weights. When the hidden size allows the wide GEMV kernels (a multiple of 1024), gate and up rows
        # are interleaved so the gate/up GEMV writes silu(gate) * up directly (mode 3) and down reads it as a
        # plain input; otherwise [gate; up] and the SiLU-gated input of down (mode 2), as the reference.
        self.gated = cfg.D % 1024 == 0
        self.W, self.small = [], []
        cache = None
        if codec_cache:
            cache = codec_cache if self.tp == 1 else f"{codec_cache}.tp{self.tp}r{self.tp_rank}"
        cmeta = {"model": cfg.name, "L": cfg.L, "D": cfg.D, "H": cfg.H, "KV": cfg.KV, "HD": cfg.HD, "FF": cfg.FF,
                 "V": cfg.V, "tied": cfg.tied, "gu_layout": "interleaved" if self.gated else "fused",
                 "tp": f"{self.tp}:{self.tp_rank}",
                 "source": f"random:{src.seed}:{src.std}" if isinstance(src, RandomWeights) else
                 os.path.abspath(getattr(src, "dir", ""))}
        mats = codecfile.load(cache, dev, expect=cmeta) if cache and os.path.exists(cache) else None
        self.emb = src.embedding().to(dev).contiguous()
        if mats is not None:  # encoded planes from disk: only the norm weights come from the source
            for i in range(self.L):
                self.W.append({n: mats[f"layers.{i}.{n}"] for n in MATS})
                lw = src.layer_small(i)
                self.small.append({k: lw[k].to(dev).contiguous() for k in ("ln1", "ln2", "qn", "kn")})
            self.head = mats["head"]
            hw = wcomp.decompress(self.head) if head8 and self.tp == 1 else None  # lossless: the bf16 head
        else:
            for i in range(self.L):
                lw = src.layer(i)
                if self.tp > 1:
                    lw = shard_layer(lw, cfg, self.tp_rank, self.tp)
                if self.gated:
                    lw["gu"] = wcomp.interleave_gate_up(lw["gu"])
                self.W.append({n: wcomp.compress(lw[n].to(dev)) for n in MATS})
                self.small.append({k: lw[k].to(dev).contiguous() for k in ("ln1", "ln2", "qn", "kn")})
                del lw
            hw = self.emb if cfg.tied else src.head().to(dev)
            if self.tp > 1:  # vocabulary-sharded head: this rank's rows only
                hw = hw[self.tp_rank * self.Vs:(self.tp_rank + 1) * self.Vs].contiguous()
            self.head = wcomp.compress(hw)
            if cache:
                torch.cuda.synchronize()
                out = {f"layers.{i}.{n}": self.W[i][n] for i in range(self.L) for n in MATS}
                out["head"] = self.head
                codecfile.save(cache, out, cmeta)
        # the int8 greedy head needs the whole vocabulary on one GPU; tensor-parallel ranks pick from gathered logits
        self.head8 = Head8(hw, self.head, TM=MAXB) if head8 and self.tp == 1 else None
        del hw
        self.norm = src.final_norm().to(dev).contiguous()
        torch.cuda.synchronize()
        # ---- KV cache (bf16) and work buffers
        self.kv = torch.zeros(self.L, 2, self.KV, maxt, self.HD, dtype=torch.bfloat16, device=dev)
        f = lambda n: torch.zeros(MAXB, n, device=dev)  # noqa: E731
        H, KV, HD = self.H, self.KV, self.HD
        self.xb, self.hb = f(self.D), f(self.D)
        self.qkvb, self.qb, self.attb, self.gub = f((H + 2 * KV) * HD), f(H * HD), f(H * HD), f(2 * self.FF)
        self.logits = torch.zeros(MAXB, self.V, device=dev)
        if self.tp > 1:  # this rank's logit columns, and every rank's gathered ([tp, rows, Vs] per call)
            self.logits_part = torch.zeros(MAXB, self.Vs, device=dev)
            self.logits_all = torch.zeros(self.tp * MAXB * self.Vs, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int64, device=dev)
        self.ids = torch.zeros(MAXB, dtype=torch.int64, device=dev)
        self.out_ids = torch.zeros(MAXB, dtype=torch.int64, device=dev)
        self.u = torch.zeros(MAXB, dtype=torch.float64, device=dev)
        self.prior = torch.full((1, sampler.PMAX), -1, dtype=torch.int32, device=dev)
        self.sample_ws = sampler.workspace(MAXB, self.cfg.V, dev)
        self.tws = prefill.workspace(MAXB, max(int(c["K"]) for c in self.W[0].values()), 3, dev)  # T <= 16 passes
        wsz = max(_lib.lib().aib_attn_workspace(H, KV, HD, maxt, t) for t in range(1, MAXB + 1))
        self.ws = torch.zeros(wsz, dtype=torch.uint8, device=dev)
        # stream-K workspace of the gate/up GEMV (the one matrix whose whole-tile split leaves a long tail: 1536
        # row tiles over 296 CTAs); the other matrices run whole row tiles (measured faster for them)
        self.gws = wcomp.gemv_workspace([w["gu"] for w in self.W], dev)
        self.use_graphs = graphs
        self.graphs = {}
        self._setup_allreduce()
        self.ctx = []
        self.scale = HD ** -0.5
        self.weight_bytes = sum(c.nbytes for w in self.W for c in w.values())
        self.head_bytes = self.head.nbytes
        self.load_s = time.time() - t0
        if log:
            log(f"loaded {cfg.name}: {self.weight_bytes / 2**30:.2f} GiB layers + {self.head_bytes / 2**30:.2f} GiB "
                f"head (12-bit), KV {self.kv.numel() * 2 / 2**30:.2f} GiB, {self.load_s:.1f} s")

    def close(self):
        self.graphs.clear()

    # ------------------------------------------------------------------------------------ step body
    @property
    def _add(self):
        """GEMV mode of the residual updates: add into x (1) on rank 0 (and without tensor parallelism); the
        other ranks write their partial (0) and the all-reduce sums x + every rank's partial."""
        return 1 if self.tp_rank == 0 else 0

    def _reduce(self, x):
        """Sum x over the tensor-parallel ranks: the one-shot peer-memory all-reduce for decode-sized blocks,
        NCCL for larger ones (whole-prompt prefill) or when symmetric memory is unavailable."""
        if self.tp > 1:
            a = self.ar
            if a is not None and x.numel() <= a["nmax"]:
                _lib.call("aib_allreduce_oneshot", ptr(x), x.numel(), a["nmax"], a["bufs"], a["flags"], self.tp_rank,
                          self.tp, ptr(a["epoch"]), stream_ptr())
                return
            import torch.distributed as dist
            dist.all_reduce(x)

    def _setup_allreduce(self):
        """Symmetric buffers (two slots of MAXB * D floats) and flag words mapped on every rank, for the one-shot
        all-reduce (AIB_ALLREDUCE=nccl keeps NCCL for every exchange)."""
        self.ar = None
        if self.tp == 1 or os.environ.get("AIB_ALLREDUCE", "oneshot") != "oneshot":
            return
        import ctypes as C
        import torch.distributed as dist
        try:
            import torch.distributed._symmetric_memory as symm_mem
            nmax = MAXB * self.D
            buf = symm_mem.empty(2 * nmax, dtype=torch.float32, device=self.device)
            hb = symm_mem.rendezvous(buf, dist.group.WORLD)
            flg = symm_mem.empty(self.tp, dtype=torch.int32, device=self.device)
            flg.zero_()
            hf = symm_mem.rendezvous(flg, dist.group.WORLD)
            bufs = (C.c_int64 * self.tp)(*[int(v) for v in hb.buffer_ptrs])
            flags = (C.c_int64 * self.tp)(*[int(v) for v in hf.buffer_ptrs])
        except Exception as exc:  # no symmetric memory on this system: NCCL for every exchange
            if self.log:
                self.log(f"one-shot all-reduce unavailable ({exc}); using NCCL")
            return
        torch.cuda.synchronize()
        dist.barrier()
        self.ar = {"buf": buf, "flg": flg, "hb": hb, "hf": hf, "nmax": nmax, "bufs": bufs, "flags": flags,
                   "epoch": torch.zeros(1, dtype=torch.int32, device=self.device)}

    def _layers(self, T):
        H, KV, HD = self.H, self.KV, self.HD
        for l in range(self.L):
            W, s = self.W[l], self.small[l]
            kc, vc = self.kv[l, 0], self.kv[l, 1]
            if T == 1:
                x = self.xb[0]
                wcomp.gemvc1(x, W["qkv"], self.qkvb[0], 0, lnw=s["ln1"], eps=self.eps)
                tkernels.rope_attn(self.qkvb[0], s["qn"], s["kn"], self.inv, self.pos, kc, vc, self.attb[0], self.maxt,
                                   self.eps, self.scale, H, KV, HD, ws=self.ws)
                wcomp.gemvc1(self.attb[0], W["o"], x, self._add)
                self._reduce(self.xb[:1])
                if self.gated:
                    wcomp.gemvc1(x, W["gu"], self.gub[0], 3, lnw=s["ln2"], eps=self.eps, ws=self.gws)
                    wcomp.gemvc1(self.gub[0], W["down"], x, self._add)
                else:
                    wcomp.gemvc1(x, W["gu"], self.gub[0], 0, lnw=s["ln2"], eps=self.eps)
                    if not self._add:
                        x.zero_()
                    wcomp.gemvc1(self.gub[0], W["down"], x, 2)
                self._reduce(self.xb[:1])
            else:
                # T <= 16 rows: the tcgen05 codec GEMM (RMSNorm and SiLU gate fused, three bf16 parts of the
                # activations so the products are fp32-exact): each weight matrix is read once for all rows
                x, pr, ws, add = self.xb[:T], 3, self.tws, self._add == 1
                prefill.matrix(x, W["qkv"], self.qkvb[:T], precision=pr, lnw=s["ln1"], eps=self.eps, ws=ws)
                tkernels.qk_rope_cache(self.qkvb[:T], s["qn"], s["kn"], self.inv, self.pos, self.qb[:T], kc, vc,
                                       self.maxt, self.eps, H, KV, HD, T)
                tkernels.attn(self.qb[:T], kc, vc, self.pos, self.attb[:T], self.maxt, self.scale, H, KV, HD, T,
                              ws=self.ws)
                prefill.matrix(self.attb[:T], W["o"], x, add=add, precision=pr, ws=ws)
                self._reduce(x)
                if self.gated:
                    prefill.matrix(x, W["gu"], self.gub[:T], precision=pr, lnw=s["ln2"], eps=self.eps, gated=True,
                                   ws=ws)
                    prefill.matrix(self.gub[:T], W["down"], x, add=add, precision=pr, ws=ws)
                else:
                    prefill.matrix(x, W["gu"], self.gub[:T], precision=pr, lnw=s["ln2"], eps=self.eps, ws=ws)
                    prefill.matrix(self.gub[:T], W["down"], x, add=add, precision=pr, silu_input=True, ws=ws)
                self._reduce(x)

    def _step(self, T, prm, rows, penal):
        """Everything that runs on the device for one pass of T tokens (graph body)."""
        tkernels.embed(self.emb, self.ids[:T], self.xb[:T])
        self._layers(T)
        self._pick(T, prm, rows, penal)

    def _pick(self, T, prm, rows, penal):
        """Final norm of the last `rows` rows of xb[:T], the head's pick into out_ids, then advance(ids, pos)."""
        r0 = T - rows
        tkernels.rmsg(self.xb[r0:T], self.norm, self.hb[r0:T], self.eps)
        if self.head8 is not None and prm.temperature <= 0 and not penal:
            # greedy: int8 bounds, exact logits of the candidate rows (Head.pick, head.py:59-88)
            self.head8.pick(self.hb[r0:T], rows, out=self.out_ids[r0:T])
        else:
            # sampling (or penalties): exact logits of the whole vocabulary, as Head.pick computes them for
            # sampling (head.py:62-71), then the device sampler. (Head.topk_logits would restrict top-k sampling
            # to the int8 bounds' candidates; on the random-init benchmark head the bounds keep nearly every row
            # and that path measured 4.64 vs 3.36 ms per step, so it is not the engine's default.)
            self._exact(r0, T, rows)
            sampler.sample_into(self.logits[r0:T], self.out_ids[r0:T], prm,
                                self.u[:rows] if prm.temperature > 0 else None, self.prior if penal else None, None,
                                B=rows, ws=self.sample_ws)
        _lib.call("aib_step_advance", ptr(self.pos), ptr(self.ids), ptr(self.out_ids), T,
                  ptr(self.prior) if penal else None, sampler.PMAX if penal else 0, stream_ptr())

    def _exact(self, r0, T, rows):
        """Exact logits of rows hb[r0:T] into logits[r0:T]. Tensor parallel: each rank computes its vocabulary slice
        and one all-gather gives every rank the whole row, so all ranks sample the same token."""
        if self.tp == 1:
            exact_logits(self.hb[r0:T], self.head, rows, self.logits[r0:T])
            return
        import torch.distributed as dist
        exact_logits(self.hb[r0:T], self.head, rows, self.logits_part[:rows])
        n = self.tp * rows * self.Vs
        dist.all_gather_into_tensor(self.logits_all[:n], self.logits_part[:rows].reshape(-1))
        self.logits[r0:T].view(rows, self.tp, self.Vs).copy_(
            self.logits_all[:n].view(self.tp, rows, self.Vs).transpose(0, 1))

    def _prefill(self, tokens, pos0, prm, us, penal):
        """Whole-prompt prefill (the reference's blocked path, core/engine.py:446-487 with kernels/prefill.py):
        every layer runs over all n prompt rows at once -- tcgen05 GEMMs that read each weight matrix once per
        token tile, causal flash attention -- then the head picks after the last row. Returns [token]."""
        n = len(tokens)
        ids = torch.tensor(tokens, dtype=torch.int64).to(self.device)
        x = torch.empty(n, self.D, device=self.device)
        tkernels.embed(self.emb, ids, x)
        bufs = prefill.Buffers(self, n)
        for l in range(self.L):
            prefill.layer(self, l, x, pos0, bufs)
        self.xb[0].copy_(x[n - 1])
        self.pos.fill_(pos0 + n - 1)  # the head step advances it to pos0 + n
        if prm.temperature > 0:
            self.u[0] = us[0]
        self._pick(1, prm, 1, penal)
        return self.out_ids[:1].tolist()

    def _run(self, T, prm, rows, penal):
        key = (T, rows, penal, prm.temperature, prm.top_k, prm.top_p, prm.repetition_penalty, prm.presence_penalty,
               prm.frequency_penalty)
        if not self.use_graphs:
            self._step(T, prm, rows, penal)
            return
        g = self.graphs.get(key)
        if g is None:
            # First use of this shape: run the step eagerly (it is the real step; one-time library setup such
            # as shared-memory attributes happens outside capture), then capture it for later replays.
            self._step(T, prm, rows, penal)
            _collect_before_capture()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, capture_error_mode="thread_local"):
                self._step(T, prm, rows, penal)
            self.graphs[key] = g
            return
        g.replay()

    # ----------------------------------------------------------------------------------------- API
    def _validate_process(self, tokens, pos0):
        if not isinstance(pos0, int) or isinstance(pos0, bool) or not 0 <= pos0 <= len(self.ctx):
            raise ValueError("position does not extend a valid prefix")
        if not tokens:
            raise ValueError("an empty pass is not supported")
        for t in tokens:
            try:
                i = t.__index__()
            except (AttributeError, TypeError) as exc:
                raise ValueError("token ids must be integers") from exc
            if isinstance(t, bool) or i < 0 or i >= self.V:
                raise ValueError("token id outside the vocabulary")

    def _pass(self, tokens, pos0, prm, us, last_only, penal=False):
        """Run tokens from pos0: whole-prompt prefill for long prompts that need only the last pick, else chunks of
        <= 16; returns the sampled ids (last chunk only if last_only)."""
        out = []
        n = len(tokens)
        if last_only and prefill.enabled(n):
            return self._prefill(tokens, pos0, prm, us, penal)
        c = 0
        while c < n:
            T = min(MAXB, n - c)
            final = c + T >= n
            rows = (1 if last_only else T) if final else 0
            self.ids[:T].copy_(torch.tensor(tokens[c:c + T], dtype=torch.int64))
            self.pos.fill_(pos0 + c)
            if rows:
                if prm.temperature > 0:
                    self.u[:rows].copy_(torch.tensor(us[:rows], dtype=torch.float64))
                self._run(T, prm, rows, penal)
                out = self.out_ids[T - rows:T].tolist()
            else:
                self._run(T, sampler.params(), 1, False)  # intermediate chunk: fills the KV cache
            c += T
        return out

    def process(self, tokens, pos0, temperature=0.0, top_p=1.0, rng=None, last_only=False, top_k=0):
        """Run `tokens` from position pos0 (KV before pos0 already cached). Returns the next-token pick after
        each token (only after the last one for last_only or prompts longer than 16 tokens), like the
        reference `Engine.process` (core/engine.py:505-526)."""
        self._validate_process(tokens, pos0)
        if pos0 + len(tokens) > self.maxt:
            raise ValueError(f"text longer than {self.maxt} tokens")
        previous = self.ctx[:pos0]
        last_only = last_only or len(tokens) > MAXB
        rows = 1 if last_only else len(tokens)
        us = None
        if temperature > 0:
            rng = rng or np.random.default_rng()
            us = [rng.random() for _ in range(rows)]
        prm = sampler.params(temperature, top_k, top_p)
        try:
            result = self._pass(list(tokens), pos0, prm, us, last_only)
        except Exception:
            self.ctx = []
            raise
        self.ctx = previous + list(tokens)
        return result

    def draft(self, seq, k):
        """This engine as the drafter (reference Engine.draft, core/engine.py:787-803): up to k greedy tokens
        after seq, reusing the cached prefix it shares with seq."""
        if k <= 0:
            return []
        c = min(self.common(seq), len(seq) - 1)
        out = [self.process(list(seq[c:]), c, last_only=True)[-1]]
        for i in range(k - 1):
            out.append(self.process([out[-1]], len(seq) + i)[0])
        return out

    def common(self, seq):
        n = 0
        for a, b in zip(self.ctx, seq):
            if a != b:
                break
            n += 1
        return n

    def generate(self, prompt, max_new=256, temperature=0.0, top_p=1.0, seed=None, top_k=0, repetition_penalty=1.0,
                 presence_penalty=0.0, frequency_penalty=0.0, stats=None, draft=None, k=None, force=None, cons=None):
        """Yield up to max_new tokens (reference generate, core/engine.py:538-694). Penalties count the prompt and
        the generated tokens (the most recent 4096 ids).
        draft: another Engine that proposes up to k (default 15) greedy tokens per pass; this engine verifies
        the last token plus the proposal in one batched pass (the weights are read once for all of them) and
        keeps the proposal's longest prefix that matches its own picks, plus its own next token (the
        reference's speculative loop, engine.py:589-694, without its cost-model gating). Greedy only, as in
        the reference; stats gain drafted / accepted counts."""
        if cons is not None:
            raise NotImplementedError("grammar constraints are not part of this engine")
        if draft is not None and (temperature > 0 or repetition_penalty != 1.0 or presence_penalty != 0.0 or
                                  frequency_penalty != 0.0):
            raise NotImplementedError("the draft path verifies greedy decoding without penalties, as the reference")
        if not isinstance(max_new, int) or isinstance(max_new, bool) or max_new < 0:
            raise ValueError("max_new must be a non-negative integer")
        if max_new == 0:
            if stats is not None:
                stats.update(prompt_n=0, prompt_ms=0.0, gen_n=0, decode_n=0, gen_ms=0.0)
            return
        if not prompt:
            raise ValueError("an empty prompt is not supported; pass BOS or text")
        P = len(prompt)
        if P > self.maxt:
            raise ValueError(f"prompt longer than the context {self.maxt}")
        rng = np.random.default_rng(seed)
        max_new = min(max_new, self.maxt - P + 1)
        c = min(self.common(prompt), P - 1)
        prm = sampler.params(temperature, top_k, top_p, repetition_penalty, presence_penalty, frequency_penalty)
        penal = repetition_penalty != 1.0 or presence_penalty != 0.0 or frequency_penalty != 0.0
        if penal:
            ring = np.full(sampler.PMAX, -1, np.int32)
            for i, t in enumerate(prompt):
                ring[i % sampler.PMAX] = t
            self.prior.copy_(torch.from_numpy(ring)[None])
        self._validate_process(list(prompt[c:]), c)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        us = [rng.random()] if temperature > 0 else None
        try:
            tok = self._pass(list(prompt[c:]), c, prm, us, True, penal)[-1]
        except Exception:
            self.ctx = []
            raise
        self.ctx = list(prompt)
        t1 = time.perf_counter()
        st = stats if stats is not None else {}
        st.update(prompt_n=P - c, prompt_ms=(t1 - t0) * 1000, first_token_ms=(t1 - t0) * 1000, gen_n=1, decode_n=0,
                  gen_ms=0.0, passes=0)
        gen = [tok]
        yield tok
        if draft is not None:
            st.update(drafted=0, accepted=0)
            while len(gen) < max_new and gen[-1] not in self.eos:
                ts = time.perf_counter()
                seq = list(prompt) + gen
                kmax = min(k or 15, MAXB - 1, max_new - len(gen) - 1, self.maxt - len(seq),
                           max(0, draft.maxt - len(seq)))
                d = draft.draft(seq, kmax) if kmax > 0 else []
                res = self.process([gen[-1]] + d, len(seq) - 1)  # the KV holds seq[:-1]
                n = 0
                while n < len(d) and d[n] == res[n]:
                    n += 1
                st["drafted"] += len(d)
                st["accepted"] += n
                st["gen_ms"] += (time.perf_counter() - ts) * 1000
                st["passes"] += 1
                for t in d[:n] + [res[n]]:
                    if len(gen) >= max_new or gen[-1] in self.eos:
                        break
                    gen.append(t)
                    st["gen_n"] = len(gen)
                    st["decode_n"] = len(gen) - 1
                    yield t
            return
        # decode loop: the graph chains ids and pos on the device; the host supplies u and reads one id
        while len(gen) < max_new and gen[-1] not in self.eos:
            ts = time.perf_counter()
            if temperature > 0:
                self.u[0] = rng.random()
            self._run(1, prm, 1, penal)
            t = int(self.out_ids[0].item())
            self.ctx.append(gen[-1])
            st["gen_ms"] += (time.perf_counter() - ts) * 1000
            st["passes"] += 1
            gen.append(t)
            st["gen_n"] = len(gen)
            st["decode_n"] = len(gen) - 1
            yield t

    # ------------------------------------------------------------------------------ bench helpers
    def bytes_per_token(self, ctx):
        """Algorithmic HBM bytes of one T=1 decode step at context length ctx: 12-bit layer weights +
        12-bit head + the bf16 K/V rows attended (ctx positions) + the current K/V written."""
        kv = self.L * 2 * self.KV * (ctx + 1) * self.HD * 2
        return self.weight_bytes + self.head_bytes + kv

    # ------------------------------------------------------------------------------ batched decode
    def generate_batch(self, prompts, max_new=256, temperature=0.0, top_p=1.0, top_k=0, seed=None):
        """Decode B <= 16 independent sequences together (no reference counterpart: the reference engine decodes
        one sequence). Each prompt is prefilled into its own KV cache; then every step reads each weight matrix
        once for all B tokens. Returns B token lists of max_new tokens each (no early stop at EOS, so the batch
        stays aligned). Uniform draws come from np.random.default_rng(seed), B per step in sequence order."""
        B = len(prompts)
        if not 1 <= B <= MAXB:
            raise ValueError(f"generate_batch takes 1..{MAXB} prompts")
        for p in prompts:
            if not p:
                raise ValueError("an empty prompt is not supported; pass BOS or text")
            self._validate_process(list(p), 0)
            if len(p) + max_new > self.maxt:
                raise ValueError(f"prompt + max_new longer than the context {self.maxt}")
        bt = self._batch(B)
        prm = sampler.params(temperature, top_k, top_p)
        rng = np.random.default_rng(seed)
        out = [[] for _ in range(B)]
        for b, p in enumerate(prompts):
            us = [rng.random()] if temperature > 0 else None
            out[b].append(bt.prefill(b, list(p), prm, us))
        for _ in range(max_new - 1):
            if temperature > 0:
                bt.u.copy_(torch.from_numpy(rng.random(B)))
            bt.run(prm)
            for b, t in enumerate(bt.out_ids.tolist()):
                out[b].append(t)
        return out

    def _batch(self, B):
        bt = getattr(self, "_bt", None)
        if bt is None or bt.B != B:
            self._bt = bt = Batch(self, B)
        return bt


class Batch:
    """Device state of B sequences decoded together by one engine: per-sequence KV caches [B, L, 2, KV, maxt, HD]
    (bf16), positions and input ids, and [B, n] work rows. A step is one CUDA graph: the batched codec GEMVs (rows =
    sequences, each weight read once), the batched fused attention (each sequence at its own position over its own
    cache), the head's pick for B rows and a per-sequence advance."""

    def __init__(self, eng, B):
        self.eng, self.B = eng, B
        dev, H, KV, HD = eng.device, eng.H, eng.KV, eng.HD
        self.kv = torch.zeros(B, eng.L, 2, KV, eng.maxt, HD, dtype=torch.bfloat16, device=dev)
        self.pos = torch.zeros(B, dtype=torch.int64, device=dev)
        self.ids = torch.zeros(B, dtype=torch.int64, device=dev)
        self.out_ids = torch.zeros(B, dtype=torch.int64, device=dev)
        self.u = torch.zeros(B, dtype=torch.float64, device=dev)
        f = lambda n: torch.zeros(B, n, device=dev)  # noqa: E731
        self.xb, self.hb = f(eng.D), f(eng.D)
        self.qkvb, self.attb, self.gub = f((H + 2 * KV) * HD), f(H * HD), f(2 * eng.FF)
        self.logits = torch.zeros(B, eng.V, device=dev)
        self.ws = torch.zeros(_lib.lib().aib_attn_batch_workspace(H, KV, HD, eng.maxt, B), dtype=torch.uint8,
                              device=dev)
        self.sample_ws = sampler.workspace(B, eng.V, dev)
        self.seq_stride = eng.L * 2 * KV * eng.maxt * HD  # elements between two sequences' caches
        self.graphs = {}

    def prefill(self, b, tokens, prm, us):
        """Prompt of sequence b into its cache (whole-prompt prefill); returns its first token."""
        eng = self.eng
        own = eng.kv
        eng.kv = self.kv[b]
        try:
            tok = eng._prefill(tokens, 0, prm, us, False)[0]
        finally:
            eng.kv = own
        self.pos[b] = len(tokens)
        self.ids[b] = tok
        return tok

    def _attn(self, l):
        eng, s = self.eng, self.eng.small[l]
        H, KV, HD = eng.H, eng.KV, eng.HD
        _lib.call("aib_rope_attn_decode_batch", ptr(self.qkvb), self.qkvb.stride(0), ptr(s["qn"].view(torch.int16)),
                  ptr(s["kn"].view(torch.int16)), ptr(eng.inv), ptr(self.pos), ptr(self.kv[0, l, 0].view(torch.int16)),
                  ptr(self.kv[0, l, 1].view(torch.int16)), self.seq_stride, ptr(self.attb), self.attb.stride(0), self.B,
                  H, KV, HD, eng.maxt, float(eng.eps), float(eng.scale), ptr(self.ws), self.ws.numel(), stream_ptr())

    def _step(self, prm):
        eng, B = self.eng, self.B
        x, h = self.xb, self.hb
        tkernels.embed(eng.emb, self.ids, x)
        ws, add = eng.tws, eng._add == 1
        for l in range(eng.L):
            W, s = eng.W[l], eng.small[l]
            prefill.matrix(x, W["qkv"], self.qkvb, precision=3, lnw=s["ln1"], eps=eng.eps, ws=ws)
            self._attn(l)
            prefill.matrix(self.attb, W["o"], x, add=add, precision=3, ws=ws)
            eng._reduce(x)
            if eng.gated:
                prefill.matrix(x, W["gu"], self.gub, precision=3, lnw=s["ln2"], eps=eng.eps, gated=True, ws=ws)
                prefill.matrix(self.gub, W["down"], x, add=add, precision=3, ws=ws)
            else:
                prefill.matrix(x, W["gu"], self.gub, precision=3, lnw=s["ln2"], eps=eng.eps, ws=ws)
                prefill.matrix(self.gub, W["down"], x, add=add, precision=3, silu_input=True, ws=ws)
            eng._reduce(x)
        tkernels.rmsg(x, eng.norm, h, eng.eps)
        if eng.head8 is not None and prm.temperature <= 0:
            eng.head8.pick(h, B, out=self.out_ids)
        else:
            if eng.tp > 1:
                raise NotImplementedError("batched decode runs on one GPU (or as replicas)")
            exact_logits(h, eng.head, B, self.logits)
            sampler.sample_into(self.logits, self.out_ids, prm, self.u if prm.temperature > 0 else None, None, None,
                                B=B, ws=self.sample_ws)
        _lib.call("aib_batch_advance", ptr(self.pos), ptr(self.ids), ptr(self.out_ids), B, stream_ptr())

    def run(self, prm):
        key = (prm.temperature, prm.top_k, prm.top_p)
        if not self.eng.use_graphs:
            self._step(prm)
            return
        g = self.graphs.get(key)
        if g is None:
            self._step(prm)
            _collect_before_capture()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, capture_error_mode="thread_local"):
                self._step(prm)
            self.graphs[key] = g
            return
        g.replay()

    def bytes_per_step(self, ctx):
        """Algorithmic HBM bytes of one batched step at context ctx: weights once, each sequence's K/V."""
        eng = self.eng
        kv = self.B * eng.L * 2 * eng.KV * (ctx + 1) * eng.HD * 2
        return eng.weight_bytes + eng.head_bytes + kv
