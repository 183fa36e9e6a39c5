"""Qwen3 model profiles (Fire's ``include/Fire/model/model_weights.h:64-121``).

A profile is data, not a class hierarchy: one Qwen3 decode engine serves every
dense size. The two reference profiles are reproduced with the same numbers;
``tiny`` profiles exist only to make small, fast parity cases.
"""
from __future__ import annotations

from dataclasses import dataclass, replace


@dataclass(frozen=True)
class Qwen3Profile:
    name: str
    vocab_size: int
    max_seq_len: int
    hidden_size: int
    intermediate_size: int
    num_layers: int
    num_attention_heads: int
    num_kv_heads: int
    head_dim: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    tie_word_embeddings: bool = False

    @property
    def q_dim(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def kv_groups(self) -> int:
        return self.num_attention_heads // self.num_kv_heads

    @property
    def tensor_count(self) -> int:
        # embedding + final norm + output, and eleven tensors per decoder layer
        return self.num_layers * 11 + 3

    def is_valid(self) -> bool:
        return (bool(self.name) and self.vocab_size > 0 and self.max_seq_len > 0
                and self.hidden_size > 0 and self.intermediate_size > 0 and self.num_layers > 0
                and self.num_attention_heads > 0 and self.num_kv_heads > 0 and self.head_dim > 0
                and self.num_attention_heads % self.num_kv_heads == 0 and self.head_dim % 2 == 0
                and self.rms_norm_eps > 0 and self.rope_theta > 0)

    def with_layers(self, n: int) -> "Qwen3Profile":
        return replace(self, num_layers=n)


QWEN3_0_6B = Qwen3Profile("Qwen/Qwen3-0.6B", 151936, 40960, 1024, 3072, 28, 16, 8, 128,
                          1e-6, 1_000_000.0, True)
QWEN3_8B = Qwen3Profile("Qwen/Qwen3-8B", 151936, 40960, 4096, 12288, 36, 32, 8, 128,
                        1e-6, 1_000_000.0, False)
# Small shapes with the same structure (GQA 2:1, head_dim 128, group-128 K).
TINY = Qwen3Profile("tiny-qwen3", 1000, 4096, 256, 512, 2, 4, 2, 128, 1e-6, 1_000_000.0)

PROFILES = {"qwen3-0.6b": QWEN3_0_6B, "qwen3-8b": QWEN3_8B, "tiny": TINY}
