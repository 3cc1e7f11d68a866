"""Model configurations of the served decoder: Llama-style 8B and 70B, and a tiny one.

The reference serves Qwen3.8-27B-AWQ through sglang (docs/performance.md:3-5);
it ships no model code. These are the Llama-style dense shapes the B200 build
is measured on, with random-init weights N(0, 0.02)."""
import dataclasses


@dataclasses.dataclass(frozen=True)
class LlamaConfig:
    name: str = "llama-8b"
    hidden: int = 4096
    layers: int = 32
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    vocab: int = 128256
    rope_theta: float = 500000.0
    eps: float = 1e-5
    max_pos: int = 16384
    init_std: float = 0.02
    # RoPE frequency scaling as (key, value) pairs, e.g. Llama 3.1's
    # (("rope_type", "llama3"), ("factor", 8.0), ...); empty = plain RoPE
    rope_scaling: tuple = ()
    # per-head RMSNorm of q and k before RoPE (Qwen3); weights q_norm / k_norm [head_dim]
    qk_norm: bool = False
    # biases on the q, k and v projections (Qwen2); weight qkv_bias [(nq + 2 nkv) head_dim]
    qkv_bias: bool = False

    @classmethod
    def llama_8b(cls):
        return cls()

    @classmethod
    def llama_70b(cls):
        return cls(name="llama-70b", hidden=8192, layers=80, heads=64, kv_heads=8, ffn=28672)

    @classmethod
    def tiny(cls, layers: int = 2):
        """Small shapes with the same structure (tests / smoke)."""
        return cls(name="llama-tiny", hidden=512, layers=layers, heads=8, kv_heads=2, ffn=1024, vocab=4096,
                   max_pos=4096)

    @classmethod
    def by_name(cls, name: str):
        return {"llama-8b": cls.llama_8b, "8b": cls.llama_8b, "llama-70b": cls.llama_70b, "70b": cls.llama_70b,
                "tiny": cls.tiny, "llama-tiny": cls.tiny}[name]()

    def params(self) -> int:
        att = self.hidden * (self.heads + 2 * self.kv_heads) * self.head_dim + self.heads * self.head_dim * self.hidden
        mlp = 3 * self.hidden * self.ffn
        return self.layers * (att + mlp + 2 * self.hidden) + 2 * self.vocab * self.hidden + self.hidden

    def check_tp(self, tp: int):
        for what, v in (("heads", self.heads), ("kv_heads", self.kv_heads), ("ffn", self.ffn),
                        ("vocab", self.vocab)):
            if v % tp:
                raise ValueError(f"{self.name}: {what}={v} is not divisible by TP={tp}")
