"""CPU oracle for the s8b pipeline-parallel W8A8 decode step — TEST INFRASTRUCTURE ONLY.

This package is the checker, never the product. Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline / ``--impl reference`` legs may import it. The CUDA path in
``superl8_serve_b200`` never imports, links or falls back to anything here.

What it restates (all citations are paths inside the superl8-serve project):

* the per-token int8 activation quantizer and the per-row int8 weight quantizer
  (``superl8serve/layers/linear.py:1-13``, ``tests/test_layers.py:29-33``);
* the W8A8 linear: int8 x int8 -> int32 accumulate, dequant by token and row scale
  (``superl8serve/layers/linear.py:112-124``);
* RMSNorm with fused residual add (``superl8serve/layers/norm.py:38-58``), RoPE
  rotate-half (``superl8serve/layers/rotary.py:16-55``), SwiGLU
  (``superl8serve/layers/activation.py:20-26``);
* the Qwen3 decoder layer order (``superl8serve/models/qwen3.py:70-80``) and GQA split
  (``superl8serve/layers/gqa_attention.py:63-74``);
* the paged int8 KV write (Hadamard-rotated K, per-token RTN int8 + fp32 scale, row layout
  ``(block*Hkv+h)*block_size+off``; ``superl8serve/engine/kv_cache.py:570-604``) and the
  paged GQA decode attention (``superl8serve/engine/kv_cache.py:1148-1201``);
* the inter-stage activation codec (``superl8serve/dist/__init__.py:163-302``,
  ``superl8serve/dist/transfer_model.py:25-41``) and the stage split
  (``superl8serve/dist/pipeline.py:452``);
* the varlen prefill (``superl8serve/dist/pipeline.py:908-984``; ``model.OraclePipeline
  .prefill``);
* the sparse-MoE FFN of Qwen3-MoE (``superl8serve/models/moe.py:88-141``; ``moe``);
* the rANS entropy stage (``superl8serve/dist/entropy.py``; ``entropy``) and the sampling
  recipe that follows ``superl8serve/layers/sampler.py:22-156`` (``sampler``);
* the float contract the attention recipe approximates (``read_dense`` dequantization and
  an fp32 softmax, ``superl8serve/engine/kv_cache.py:1233-1299``; ``float_contract``).

The arithmetic kernels themselves live in the third-party ``superl8`` package, which is
not vendored in the reference and is not installed here (only its call sites are
visible). Bit-level recipes are therefore DEFINED here, following the documented
behaviour, and pinned by ``tests/golden/`` fixtures produced by running the reference's
own Python module graph with these restatements standing in for the absent kernels.
At the ``superl8`` kernel boundary itself parity is unpinned (no golden integer codes
exist in the reference); the composition around it is pinned.
"""

from . import numerics, kernels, codec, model, moe, entropy, sampler, float_contract  # noqa: F401
