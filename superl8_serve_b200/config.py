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
    # sparse MoE FFN (Qwen3-MoE): 0 experts = dense model
    num_experts: int = 0
    num_experts_per_tok: int = 8
    moe_intermediate_size: int = 0
    norm_topk_prob: bool = True
    decoder_sparse_step: int = 1
    mlp_only_layers: tuple = ()

    def is_moe(self) -> bool:
        return self.num_experts > 0

    def layer_is_moe(self, layer_idx: int) -> bool:
        """``ModelConfig.layer_is_moe`` (``superl8serve/models/config.py:221-224``)."""
        if not self.is_moe() or layer_idx in self.mlp_only_layers:
            return False
        return (layer_idx + 1) % self.decoder_sparse_step == 0

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


def qwen3_30b_a3b(**kw) -> ModelConfig:
    """Qwen3-30B-A3B MoE shape: 48 layers, hidden 2048, 32 q / 4 kv heads,
    128 experts top-8 (softmax, renormalised), expert FFN 768."""
    return ModelConfig(hidden_size=2048, num_hidden_layers=48, num_attention_heads=32,
                       num_key_value_heads=4, intermediate_size=6144, num_experts=128,
                       num_experts_per_tok=8, moe_intermediate_size=768).with_(**kw)


def tiny_moe(**kw) -> ModelConfig:
    """Small Qwen3-MoE-shaped model for tests: 16 experts top-4, every layer sparse."""
    return tiny(num_experts=16, num_experts_per_tok=4, moe_intermediate_size=128).with_(**kw)


def tiny(**kw) -> ModelConfig:
    """Small Qwen3-shaped model for tests (head_dim stays 128, the kernels' head size)."""
    return ModelConfig(vocab_size=512, hidden_size=256, num_hidden_layers=4,
                       num_attention_heads=4, num_key_value_heads=2, intermediate_size=512,
                       max_position_embeddings=1024, tie_word_embeddings=True).with_(**kw)
