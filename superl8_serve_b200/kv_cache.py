"""``PagedKVCache`` with the reference's interface, backed by the s8b paged int8 kernels.

Storage and addressing follow ``superl8serve/engine/kv_cache.py``: one pool of
``block_size``-token int8 blocks per layer ``[L, num_blocks, Hkv, block_size, D]`` plus fp32
per-token scales ``[L, num_blocks, Hkv, block_size]`` (``:484-512``); token ``(block, off)``
of head ``h`` is row ``(block*Hkv + h)*block_size + off`` (``:570-585``); a slot's blocks
come from a shared free list (``:703-749``). K is Hadamard-rotated before quantization.
Only the int8 V layout is on this path (K8V3 / eviction / prefix trie are not).
"""

from __future__ import annotations

import torch

from . import ops
from .engine import BlockAllocator
from .runtime import KVPool


class PagedKVCache:
    def __init__(self, num_layers, num_slots, num_kv_heads, max_len, head_dim, *, device,
                 block_size: int = 16, num_blocks: int | None = None):
        if head_dim != 128:
            raise ValueError("the s8b paged kernels handle head_dim 128")
        self.block_size = block_size
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.max_blocks_per_seq = (max_len + block_size - 1) // block_size
        self.num_blocks = num_blocks or num_slots * self.max_blocks_per_seq
        self.num_slots = num_slots
        self.max_len = max_len
        self.device = torch.device(device)
        self.pool = KVPool(num_layers, self.num_blocks, num_kv_heads, head_dim, block_size,
                           self.device)
        self.k_cache, self.k_scale = self.pool.kc, self.pool.ks
        self.v_cache, self.v_scale = self.pool.vc, self.pool.vs
        self._alloc = BlockAllocator(self.num_blocks, num_slots, block_size, self.max_blocks_per_seq)
        self._ws: torch.Tensor | None = None

    # ------------------------------------------------------------------ host side ----
    @property
    def _slot_blocks(self):
        return self._alloc._slot_blocks

    def alloc(self) -> int:
        return self._alloc.alloc()

    def free(self, slot: int):
        self._alloc.free(slot)

    def has_free_slot(self) -> bool:
        return bool(self._alloc._free_slots)

    def has_free_block(self) -> bool:
        return bool(self._alloc._free_blocks)

    @property
    def used_blocks(self) -> int:
        return self.num_blocks - len(self._alloc._free_blocks)

    def ensure_capacity(self, slots, lengths):
        self._alloc.ensure_capacity(slots, lengths)

    def _slot_mapping(self, slots, positions) -> torch.Tensor:
        bs = self.block_size
        flat = [self._slot_blocks[s][p // bs] * bs + p % bs for s, p in zip(slots, positions)]
        return torch.tensor(flat, dtype=torch.int32, device=self.device)

    slot_mapping_for = _slot_mapping

    def _flat_rows(self, slot_mapping: torch.Tensor) -> torch.Tensor:
        bs, nkv = self.block_size, self.num_kv_heads
        b = slot_mapping.shape[0]
        blk, off = slot_mapping // bs, slot_mapping % bs
        heads = torch.arange(nkv, device=slot_mapping.device)
        return (blk.repeat_interleave(nkv) * (nkv * bs) + heads.repeat(b) * bs
                + off.repeat_interleave(nkv)).long()

    def block_table(self, slots) -> torch.Tensor:
        return self._alloc.block_table(slots).to(self.device)

    def fill_block_table(self, dst: torch.Tensor, slots):
        dst[: len(slots)].copy_(self._alloc.block_table(slots), non_blocking=True)

    def fill_slot_mapping(self, dst: torch.Tensor, slots, positions):
        dst[: len(slots)].copy_(self._slot_mapping(slots, positions))

    # ----------------------------------------------------------------- device side ----
    def write_decode_static(self, layer: int, slot_mapping, k_new, v_new):
        """k_new, v_new [B, Hkv, D]: quantize-on-write at slot_mapping [B] int32."""
        ops.kv_write_paged(k_new.contiguous(), v_new.contiguous(), self.k_cache[layer],
                           self.k_scale[layer], self.v_cache[layer], self.v_scale[layer],
                           slot_mapping.to(torch.int32).contiguous())

    def write_decode(self, layer: int, slots, positions, k_new, v_new):
        self.write_decode_static(layer, self._slot_mapping(slots, positions), k_new, v_new)

    write_prefill_varlen = write_decode_static

    def decode_attn_static(self, layer: int, q, block_table, context_lens, max_context_len: int,
                           *, scale: float):
        """q [B, Hq, 1, D] -> [B, Hq, 1, D]; reads context_lens[b] tokens of row b."""
        B, Hq = q.shape[0], q.shape[1]
        need = ops.decode_workspace_bytes(B, Hq, self.head_dim, int(max_context_len), ref=True)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.zeros(need, dtype=torch.uint8, device=self.device)
        out = ops.paged_decode(q, self.k_cache[layer], self.k_scale[layer], self.v_cache[layer],
                               self.v_scale[layer], block_table.to(torch.int32).contiguous(),
                               context_lens.to(torch.int32).contiguous(), int(max_context_len),
                               scale, workspace=self._ws)
        return out.reshape(B, Hq, 1, self.head_dim)

    def decode_attn(self, layer: int, q, slots, lengths, *, scale: float):
        context_lens = torch.tensor([n + 1 for n in lengths], dtype=torch.int32, device=self.device)
        return self.decode_attn_static(layer, q, self.block_table(slots), context_lens,
                                       max(lengths) + 1, scale=scale)

    def read_dense(self, layer: int, slot: int, length: int, *, dtype=torch.bfloat16):
        """Dequantized [1, Hkv, N, D] K (un-rotated) and V of one sequence (debug / tests)."""
        blocks = self._slot_blocks[slot]
        pos = torch.arange(length)
        blk = torch.tensor([blocks[p // self.block_size] for p in range(length)], dtype=torch.long)
        off = pos % self.block_size
        k = self.k_cache[layer][blk, :, off, :].float() * self.k_scale[layer][blk, :, off].unsqueeze(-1)
        v = self.v_cache[layer][blk, :, off, :].float() * self.v_scale[layer][blk, :, off].unsqueeze(-1)
        i = torch.arange(128)
        pc = torch.zeros(128, 128, dtype=torch.int64)
        a = i[:, None] & i[None, :]
        while bool(a.any()):
            pc += a & 1
            a = a >> 1
        Hm = ((1 - 2 * (pc % 2)).float() / 128 ** 0.5).to(k.device)
        k = k @ Hm
        return k.permute(1, 0, 2).unsqueeze(0).to(dtype), v.permute(1, 0, 2).unsqueeze(0).to(dtype)
