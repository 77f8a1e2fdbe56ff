"""Qwen3 dense checkpoint description: configs, random-init weights and a safetensors reader.

Mirrors the reference checkpoint reader `ramvi/engine/ramvi_engine/formats/model.py` (class `Ckpt`,
:37-106): the same config fields (L, D, H, KV, HD, FF, eps, theta, tied, eos) and, crucially, the same
matrix fusion before encoding -- `qkv = cat(q, k, v)` and `gu = cat(gate, up)` (`Ckpt.layer`, :92-102) --
so the 12-bit codec picks its exponent window per *fused* matrix exactly as the reference does.

No checkpoint can be downloaded here, so benchmarks and tests use `random_weights`, which draws every
matrix from N(0, 0.02) in fp32 and rounds to bf16 (the HF random-init recipe named by the benchmark
configs). Norm weights are ones unless `norm_noise` is set (tests use noisy norms to exercise them).
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass, field, asdict

import numpy as np
import torch


@dataclass(frozen=True)
class Qwen3Config:
    L: int            # decoder layers
    D: int            # hidden size
    H: int            # query heads
    KV: int           # key/value heads
    HD: int           # head dim
    FF: int           # MLP intermediate size
    V: int            # vocab size
    eps: float = 1e-6
    theta: float = 1e6
    tied: bool = False
    eos: tuple = field(default_factory=tuple)
    name: str = "qwen3"

    def layer_params(self):
        """(N, K) of the four encoded matrices; same as `Ckpt.layer_params` (formats/model.py:104-106)."""
        D, H, KV, HD, FF = self.D, self.H, self.KV, self.HD, self.FF
        return {"qkv": ((H + 2 * KV) * HD, D), "o": (D, H * HD), "gu": (2 * FF, D), "down": (D, FF)}

    def n_layer_params(self):
        return self.L * sum(n * k for n, k in self.layer_params().values())

    def to_json(self):
        d = asdict(self)
        d["eos"] = list(self.eos)
        return d


CONFIGS = {
    "qwen3-0.6b": Qwen3Config(L=28, D=1024, H=16, KV=8, HD=128, FF=3072, V=151936, tied=True,
                              eos=(151643, 151645), name="qwen3-0.6b"),
    "qwen3-8b": Qwen3Config(L=36, D=4096, H=32, KV=8, HD=128, FF=12288, V=151936, tied=False,
                            eos=(151643, 151645), name="qwen3-8b"),
    "qwen3-32b": Qwen3Config(L=64, D=5120, H=64, KV=8, HD=128, FF=25600, V=151936, tied=False,
                             eos=(151643, 151645), name="qwen3-32b"),
    # test-sized models (same family, small shapes)
    "tiny": Qwen3Config(L=2, D=256, H=4, KV=2, HD=64, FF=512, V=1000, tied=False, name="tiny"),
    "tiny-tied": Qwen3Config(L=2, D=256, H=4, KV=2, HD=64, FF=512, V=1000, tied=True, name="tiny-tied"),
    "small": Qwen3Config(L=4, D=512, H=8, KV=4, HD=128, FF=1536, V=4096, tied=False, name="small"),
    # hidden size 1024: the engine takes the wide T = 1 GEMV kernels and the gated gate/up GEMV (mode 3)
    "small-1k": Qwen3Config(L=2, D=1024, H=8, KV=4, HD=128, FF=2048, V=2048, tied=False, name="small-1k"),
}


def layer_tensor_names(i):
    p = f"model.layers.{i}."
    a, m = p + "self_attn.", p + "mlp."
    return {"q": a + "q_proj.weight", "k": a + "k_proj.weight", "v": a + "v_proj.weight",
            "o": a + "o_proj.weight", "gate": m + "gate_proj.weight", "up": m + "up_proj.weight",
            "down": m + "down_proj.weight", "ln1": p + "input_layernorm.weight",
            "ln2": p + "post_attention_layernorm.weight", "qn": a + "q_norm.weight", "kn": a + "k_norm.weight"}


class RandomWeights:
    """Deterministic random-init Qwen3 weights, produced lazily per tensor.

    Every tensor gets its own generator seeded from (seed, tensor index), so a layer can be produced on
    any device without materialising the whole model, and the CPU stream is identical on every machine.
    `device="cuda"` uses CUDA generators (fast, for the 8B/32B benchmark models); tests use "cpu".
    """

    def __init__(self, cfg: Qwen3Config, seed: int = 0, std: float = 0.02, norm_noise: float = 0.0,
                 device: str = "cpu"):
        self.cfg, self.seed, self.std, self.norm_noise, self.device = cfg, seed, std, norm_noise, device

    def _gen(self, idx):
        g = torch.Generator(device=self.device)
        g.manual_seed((self.seed * 1000003 + idx * 7919) & 0x7FFFFFFFFFFF)
        return g

    def _mat(self, idx, n, k):
        g = self._gen(idx)
        return (torch.randn(n, k, generator=g, device=self.device, dtype=torch.float32) * self.std).bfloat16()

    def _norm(self, idx, n):
        if self.norm_noise == 0.0:
            return torch.ones(n, dtype=torch.bfloat16, device=self.device)
        g = self._gen(idx)
        return (1.0 + self.norm_noise * torch.randn(n, generator=g, device=self.device)).bfloat16()

    def layer(self, i):
        """Fused layer dict like `Ckpt.layer` (formats/model.py:92-102): qkv, o, gu, down, ln1, ln2, qn, kn."""
        c = self.cfg
        b = 100 + 16 * i
        q = self._mat(b + 0, c.H * c.HD, c.D)
        k = self._mat(b + 1, c.KV * c.HD, c.D)
        v = self._mat(b + 2, c.KV * c.HD, c.D)
        gate = self._mat(b + 4, c.FF, c.D)
        up = self._mat(b + 5, c.FF, c.D)
        return {"qkv": torch.cat([q, k, v]), "o": self._mat(b + 3, c.D, c.H * c.HD),
                "gu": torch.cat([gate, up]), "down": self._mat(b + 6, c.D, c.FF),
                "ln1": self._norm(b + 7, c.D), "ln2": self._norm(b + 8, c.D),
                "qn": self._norm(b + 9, c.HD), "kn": self._norm(b + 10, c.HD)}

    def layer_small(self, i):
        """The layer's norm weights only (ln1, ln2, qn, kn), without producing its matrices."""
        c = self.cfg
        b = 100 + 16 * i
        return {"ln1": self._norm(b + 7, c.D), "ln2": self._norm(b + 8, c.D), "qn": self._norm(b + 9, c.HD),
                "kn": self._norm(b + 10, c.HD)}

    def embedding(self):
        return self._mat(1, self.cfg.V, self.cfg.D)

    def head(self):
        return self.embedding() if self.cfg.tied else self._mat(2, self.cfg.V, self.cfg.D)

    def final_norm(self):
        return self._norm(3, self.cfg.D)


# ----------------------------------------------------------------------------------------------
# safetensors checkpoints (HF folder with config.json), read tensor by tensor without torch.load
# ----------------------------------------------------------------------------------------------
_ST_DTYPES = {"BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32}


def _st_index(path):
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        meta = json.loads(f.read(n))
    meta.pop("__metadata__", None)
    return 8 + n, meta


class Ckpt:
    """HF Qwen3 folder reader with the reference's surface (`Ckpt` in formats/model.py:37-106).

    `t(name)` returns a CPU tensor, `mm(name)` a uint16 numpy memmap of a BF16 tensor, `layer(i)` the
    fused dict, `head_name()` picks `lm_head.weight` unless the embeddings are tied.
    """

    def __init__(self, path):
        if not os.path.isdir(path):
            raise FileNotFoundError(f"model folder {path} not found")
        self.dir = path
        self.cfg = json.load(open(os.path.join(path, "config.json")))
        if self.cfg.get("model_type") != "qwen3":
            raise NotImplementedError(f"architecture {self.cfg.get('model_type')} is not supported (qwen3 only)")
        self.files = {}
        for fn in sorted(os.listdir(path)):
            if fn.endswith(".safetensors"):
                fp = os.path.join(path, fn)
                off, meta = _st_index(fp)
                for k, m in meta.items():
                    self.files[k] = (fp, off, m)
        c = self.cfg
        eos = c.get("eos_token_id", [])
        self.config = Qwen3Config(L=c["num_hidden_layers"], D=c["hidden_size"], H=c["num_attention_heads"],
                                  KV=c["num_key_value_heads"], HD=c.get("head_dim", c["hidden_size"] // c["num_attention_heads"]),
                                  FF=c["intermediate_size"], V=c["vocab_size"], eps=c["rms_norm_eps"],
                                  theta=c.get("rope_theta", 10000.0), tied=c.get("tie_word_embeddings", False),
                                  eos=tuple(eos if isinstance(eos, list) else [eos]), name=os.path.basename(path))

    def mm(self, k):
        fp, off, m = self.files[k]
        if m["dtype"] != "BF16":
            raise ValueError(f"the HF path needs BF16 tensors, got {m['dtype']} for {k}")
        a, _ = m["data_offsets"]
        return np.memmap(fp, dtype=np.uint16, mode="r", offset=off + a, shape=tuple(m["shape"]))

    def t(self, k):
        fp, off, m = self.files[k]
        a, b = m["data_offsets"]
        with open(fp, "rb") as f:
            f.seek(off + a)
            raw = bytearray(f.read(b - a))
        return torch.frombuffer(raw, dtype=_ST_DTYPES[m["dtype"]]).reshape(m["shape"]).clone()

    def head_name(self):
        if self.config.tied or "lm_head.weight" not in self.files:
            return "model.embed_tokens.weight"
        return "lm_head.weight"

    def layer(self, i):
        n = layer_tensor_names(i)
        t = self.t
        return {"qkv": torch.cat([t(n["q"]), t(n["k"]), t(n["v"])]), "o": t(n["o"]),
                "gu": torch.cat([t(n["gate"]), t(n["up"])]), "down": t(n["down"]),
                "ln1": t(n["ln1"]), "ln2": t(n["ln2"]), "qn": t(n["qn"]), "kn": t(n["kn"])}

    def layer_small(self, i):
        """The layer's norm weights only (ln1, ln2, qn, kn), without reading its matrices."""
        n = layer_tensor_names(i)
        return {k: self.t(n[k]) for k in ("ln1", "ln2", "qn", "kn")}

    def embedding(self):
        return self.t("model.embed_tokens.weight")

    def head(self):
        return self.t(self.head_name())

    def final_norm(self):
        return self.t("model.norm.weight")


def check_tp(cfg: Qwen3Config, n):
    """Raise ValueError unless the layer matrices split into n tensor-parallel shards: whole KV groups (and
    their query heads) per rank and an MLP slice that the codec can encode (a multiple of 256 columns)."""
    if n < 1 or cfg.KV % n or cfg.H % n or cfg.FF % n or (cfg.FF // n) % 256:
        raise ValueError(f"{cfg.name}: cannot split H={cfg.H}, KV={cfg.KV}, FF={cfg.FF} over {n} ranks")


def shard_layer(lw, cfg: Qwen3Config, rank, n):
    """Rank `rank` of n tensor-parallel shards of one layer's fused matrices (the split of the Megatron-style
    decode layer: qkv by KV group, o by the matching input columns, gate/up by MLP rows, down by the matching
    input columns). qkv keeps the [q; k; v] order with the rank's heads only; gu keeps [gate; up] with the
    rank's MLP rows. The small tensors (norm weights) are shared. Concatenating the shards along the split
    dimensions gives back the full matrices."""
    check_tp(cfg, n)
    H, KV, HD, FF = cfg.H, cfg.KV, cfg.HD, cfg.FF
    hq, hk, fr = H // n * HD, KV // n * HD, FF // n
    q, k, v = torch.split(lw["qkv"], [H * HD, KV * HD, KV * HD])
    g, u = torch.split(lw["gu"], [FF, FF])
    out = dict(lw)
    out["qkv"] = torch.cat([q[rank * hq:(rank + 1) * hq], k[rank * hk:(rank + 1) * hk], v[rank * hk:(rank + 1) * hk]])
    out["o"] = lw["o"][:, rank * hq:(rank + 1) * hq].contiguous()
    out["gu"] = torch.cat([g[rank * fr:(rank + 1) * fr], u[rank * fr:(rank + 1) * fr]])
    out["down"] = lw["down"][:, rank * fr:(rank + 1) * fr].contiguous()
    return out


def save_checkpoint(path, cfg: Qwen3Config, weights: RandomWeights):
    """Write a random-init model as an HF folder (config.json + model.safetensors), unfused tensors."""
    os.makedirs(path, exist_ok=True)
    tensors = {"model.embed_tokens.weight": weights.embedding(), "model.norm.weight": weights.final_norm()}
    if not cfg.tied:
        tensors["lm_head.weight"] = weights.head()
    c = cfg
    for i in range(cfg.L):
        lw = weights.layer(i)
        n = layer_tensor_names(i)
        q, k, v = torch.split(lw["qkv"], [c.H * c.HD, c.KV * c.HD, c.KV * c.HD])
        g, u = torch.split(lw["gu"], [c.FF, c.FF])
        for key, val in (("q", q), ("k", k), ("v", v), ("o", lw["o"]), ("gate", g), ("up", u),
                         ("down", lw["down"]), ("ln1", lw["ln1"]), ("ln2", lw["ln2"]), ("qn", lw["qn"]),
                         ("kn", lw["kn"])):
            tensors[n[key]] = val.contiguous()
    header, blobs, off = {}, [], 0
    for k in sorted(tensors):
        b = tensors[k].contiguous().view(torch.uint16).numpy().tobytes() if tensors[k].dtype == torch.bfloat16 \
            else tensors[k].numpy().tobytes()
        dt = {torch.bfloat16: "BF16", torch.float32: "F32", torch.float16: "F16"}[tensors[k].dtype]
        header[k] = {"dtype": dt, "shape": list(tensors[k].shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(os.path.join(path, "model.safetensors"), "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)
    json.dump({"model_type": "qwen3", "num_hidden_layers": c.L, "hidden_size": c.D, "num_attention_heads": c.H,
               "num_key_value_heads": c.KV, "head_dim": c.HD, "intermediate_size": c.FF, "vocab_size": c.V,
               "rms_norm_eps": c.eps, "rope_theta": c.theta, "tie_word_embeddings": c.tied,
               "eos_token_id": list(c.eos)}, open(os.path.join(path, "config.json"), "w"))
