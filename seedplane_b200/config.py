"""Qwen2 architecture descriptions used by the B200 engine, the tests and the benchmark.

The fields mirror the Hugging Face `config.json` keys that SeedPlane's engine reads
(`seedplane/qwen_engine.py:37-53`: layers, heads, kv heads, hidden, rope theta, eps) and the
`arch` block of a `seedplane-bundle/2` manifest (`seedplane/native_bundle.py:129-131`).
head_dim is derived as hidden // heads, exactly as `qwen_engine.py:48` does.
"""
from __future__ import annotations

from dataclasses import dataclass, asdict, replace


@dataclass(frozen=True)
class Qwen2Config:
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    intermediate: int
    vocab: int
    rope_theta: float = 1e6
    rms_norm_eps: float = 1e-6
    max_positions: int = 32768
    tied_embeddings: bool = True
    name: str = "qwen2"

    def __post_init__(self):
        if self.hidden % self.heads or self.heads % self.kv_heads:
            raise ValueError("invalid Qwen2 head configuration")

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def qkv_rows(self) -> int:
        return (self.heads + 2 * self.kv_heads) * self.head_dim

    @property
    def group(self) -> int:
        return self.heads // self.kv_heads

    def n_params(self) -> int:
        """Parameters streamed per decoded token (norm gains excluded, tied head counted once)."""
        H, I, V = self.hidden, self.intermediate, self.vocab
        per_layer = self.qkv_rows * H + self.qkv_rows + H * H + 2 * I * H + H * I
        head = 0 if self.tied_embeddings else V * H
        return self.layers * per_layer + V * H + head

    def weight_bytes_per_token(self, bytes_per_weight: float = 2.0) -> int:
        """Matrix bytes read by one decode step: every layer matrix, biases, and the LM head once.

        The embedding row gather (H elements) is negligible and is not counted; with tied
        embeddings the LM head *is* the embedding matrix, read once.
        """
        H, I, V = self.hidden, self.intermediate, self.vocab
        mats = self.layers * (self.qkv_rows * H + H * H + 2 * I * H + H * I) + V * H
        biases = self.layers * self.qkv_rows * 4
        norms = (2 * self.layers + 1) * H * 4
        return int(mats * bytes_per_weight) + biases + norms

    def kv_bytes_per_position(self, bytes_per_value: int = 2) -> int:
        return self.layers * 2 * self.kv_heads * self.head_dim * bytes_per_value

    def to_hf(self) -> dict:
        """An HF-style config.json that SeedPlane's own Qwen2Engine loads unmodified."""
        return {
            "model_type": "qwen2", "architectures": ["Qwen2ForCausalLM"],
            "num_hidden_layers": self.layers, "hidden_size": self.hidden,
            "num_attention_heads": self.heads, "num_key_value_heads": self.kv_heads,
            "intermediate_size": self.intermediate, "vocab_size": self.vocab,
            "rope_theta": self.rope_theta, "rms_norm_eps": self.rms_norm_eps,
            "max_position_embeddings": self.max_positions,
            "tie_word_embeddings": self.tied_embeddings,
        }

    @classmethod
    def from_hf(cls, cfg: dict, name: str = "qwen2") -> "Qwen2Config":
        if cfg.get("model_type") != "qwen2":
            raise ValueError("SeedPlane Qwen2 engine only supports model_type=qwen2")
        theta = cfg.get("rope_theta", cfg.get("rope_parameters", {}).get("rope_theta", 10000.0))
        return cls(layers=cfg["num_hidden_layers"], hidden=cfg["hidden_size"],
                   heads=cfg["num_attention_heads"], kv_heads=cfg["num_key_value_heads"],
                   intermediate=cfg["intermediate_size"], vocab=cfg["vocab_size"],
                   rope_theta=float(theta), rms_norm_eps=float(cfg.get("rms_norm_eps", 1e-6)),
                   max_positions=int(cfg.get("max_position_embeddings", 32768)),
                   tied_embeddings=bool(cfg.get("tie_word_embeddings", True)), name=name)

    @classmethod
    def from_bundle_arch(cls, arch: dict, name: str = "qwen2") -> "Qwen2Config":
        """Read the `arch` block of a seedplane-bundle/2 manifest (`native_bundle.py:129-131`)."""
        return cls(layers=arch["layers"], hidden=arch["hidden"], heads=arch["heads"],
                   kv_heads=arch["kv_heads"], intermediate=arch["intermediate"], vocab=arch["vocab"],
                   rope_theta=float(arch["rope_theta"]), rms_norm_eps=float(arch["rms_norm_eps"]),
                   max_positions=int(arch.get("max_positions", 32768)),
                   tied_embeddings=bool(arch.get("tied_embeddings", True)), name=name)

    def truncated(self, layers: int) -> "Qwen2Config":
        """Same model cut to its first `layers` layers (the speculative drafter of the verify configs)."""
        return replace(self, layers=layers, name=f"{self.name}-first{layers}")

    def as_dict(self) -> dict:
        return asdict(self)


# The architectures named by the benchmark configurations.
QWEN2_0_5B = Qwen2Config(layers=24, hidden=896, heads=14, kv_heads=2, intermediate=4864, vocab=151936,
                         name="qwen2-0.5b")
QWEN2_1_5B = Qwen2Config(layers=28, hidden=1536, heads=12, kv_heads=2, intermediate=8960, vocab=151936,
                         name="qwen2-1.5b")
# Qwen2.5-7B ships an untied LM head; the int8 configuration keeps it untied.
QWEN2_5_7B = Qwen2Config(layers=28, hidden=3584, heads=28, kv_heads=4, intermediate=18944, vocab=152064,
                         tied_embeddings=False, name="qwen2.5-7b")
# Small shapes for unit and parity tests: one head_dim-64 and one head_dim-128 variant.
TINY_HD64 = Qwen2Config(layers=2, hidden=256, heads=4, kv_heads=2, intermediate=512, vocab=1000,
                        max_positions=512, name="tiny-hd64")
TINY_HD128 = Qwen2Config(layers=2, hidden=256, heads=2, kv_heads=1, intermediate=768, vocab=1200,
                         max_positions=512, name="tiny-hd128")
TINY_UNTIED = replace(TINY_HD128, tied_embeddings=False, name="tiny-untied")

PRESETS = {c.name: c for c in (QWEN2_0_5B, QWEN2_1_5B, QWEN2_5_7B, TINY_HD64, TINY_HD128, TINY_UNTIED)}
