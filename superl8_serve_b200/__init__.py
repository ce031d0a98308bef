"""s8b: B200-native (sm_100a) pipeline-parallel W8A8 decode step for superl8-serve.

Kernels live in ``libs8b.so`` (built from ``csrc/`` for sm_100a, C ABI in ``include/s8b.h``);
this package is the host side: the reference-shaped layer / cache / transport / pipeline API,
the stage runtime that launches the kernels, prefill, the sparse-MoE layer, the sampler and
continuous batching.
"""

from .config import (ModelConfig, qwen3_0_6b, qwen3_8b, qwen3_27b_dense, qwen3_30b_a3b,  # noqa: F401
                     tiny, tiny_moe)
from .weights import QTensor, merge_qtensor, to_qtensor  # noqa: F401

__version__ = "0.1.0"
