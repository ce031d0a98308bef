"""Model configuration for the Qwen3-shaped W8A8 decode path.

Field names follow the reference ``ModelConfig`` (``superl8serve/models/config.py:91-226``)
so a config built for the reference engine carries over unchanged.
"""

from __future__ import annotations

from dataclasses import dataclass, replace


@dataclass
class ModelConfig:
    arch: str = "qwen3"
    vocab_size: int = 151936
    hidden_size: int = 4096
    num_hidden_layers: int = 36
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    intermediate_size: int = 12288
    max_position_embeddings: int = 40960
    head_dim: int | None = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    qk_norm: bool = True
    tie_word_embeddings: bool = False
    torch_dtype: str = "bfloat16"

    def resolved_head_dim(self) -> int:
        return self.head_dim if self.head_dim else self.hidden_size // self.num_attention_heads

    def act_dtype(self):
        import torch

        return torch.bfloat16 if str(self.torch_dtype).endswith("bfloat16") else torch.float16

    def with_(self, **kw) -> "ModelConfig":
        return replace(self, **kw)


def qwen3_0_6b(**kw) -> ModelConfig:
    """Qwen3-0.6B shape: 28 layers, hidden 1024, 16 q / 8 kv heads."""
    return ModelConfig(hidden_size=1024, num_hidden_layers=28, num_attention_heads=16,
                       num_key_value_heads=8, intermediate_size=3072,
                       tie_word_embeddings=True).with_(**kw)


def qwen3_8b(**kw) -> ModelConfig:
    """Qwen3-8B shape: 36 layers, hidden 4096, 32 q / 8 kv heads."""
    return ModelConfig().with_(**kw)


def qwen3_27b_dense(**kw) -> ModelConfig:
    """27B dense long-context shape: 64 layers, hidden 5120, 40/8 heads."""
    return ModelConfig(hidden_size=5120, num_hidden_layers=64, num_attention_heads=40,
                       num_key_value_heads=8, intermediate_size=17408).with_(**kw)


def tiny(**kw) -> ModelConfig:
    """Small Qwen3-shaped model for tests (head_dim stays 128, the kernels' head size)."""
    return ModelConfig(vocab_size=512, hidden_size=256, num_hidden_layers=4,
                       num_attention_heads=4, num_key_value_heads=2, intermediate_size=512,
                       max_position_embeddings=1024, tie_word_embeddings=True).with_(**kw)
