"""Paged KV cache: device pool plus a host-side block allocator.

MLA layers cache one ``kv_lora + rope`` latent row per token
(``[L, blocks, block_size, 576]`` for DeepSeek); GQA layers cache K and V
(``[L, blocks, block_size, kv_heads, head_dim]`` each).  A token's slot is
``block_id * block_size + offset``.
"""

from __future__ import annotations

import torch

from afd_plugin_b200.models.configs import ModelArchConfig


class BlockAllocator:
    """LIFO free list of block ids (block 0 is kept as the padding block)."""

    def __init__(self, num_blocks: int):
        if num_blocks < 2:
            raise ValueError("need at least two KV blocks")
        self.num_blocks = num_blocks
        self._free = list(range(num_blocks - 1, 0, -1))

    @property
    def num_free(self) -> int:
        return len(self._free)

    def allocate(self, n: int) -> list[int]:
        if n > len(self._free):
            raise MemoryError(f"KV cache exhausted: want {n} blocks, {len(self._free)} free")
        out = self._free[-n:][::-1] if n else []
        del self._free[len(self._free) - n :]
        return out

    def free(self, blocks: list[int]) -> None:
        self._free.extend(reversed(blocks))


PAD_BLOCK = 0


class KVCache:
    def __init__(
        self,
        arch: ModelArchConfig,
        num_blocks: int,
        block_size: int,
        dtype: torch.dtype,
        device: torch.device | str,
    ):
        self.arch = arch
        self.num_blocks = num_blocks
        self.block_size = block_size
        L = arch.num_hidden_layers
        if arch.is_mla:
            self.kv = torch.zeros(L, num_blocks, block_size, arch.kv_lora_rank + arch.qk_rope_head_dim,
                                  dtype=dtype, device=device)
            self.k = self.v = None
        else:
            shape = (L, num_blocks, block_size, arch.num_key_value_heads, arch.head_dim)
            self.k = torch.zeros(shape, dtype=dtype, device=device)
            self.v = torch.zeros(shape, dtype=dtype, device=device)
            self.kv = None
        self.allocator = BlockAllocator(num_blocks)

    def layer(self, i: int):
        if self.kv is not None:
            return self.kv[i]
        return (self.k[i], self.v[i])

    @staticmethod
    def bytes_per_block(arch: ModelArchConfig, block_size: int, dtype: torch.dtype) -> int:
        elem = torch.empty((), dtype=dtype).element_size()
        return arch.num_hidden_layers * block_size * arch.kv_cache_width * elem

    def fill_random_(self, seed: int = 0, std: float = 1.0) -> None:
        """Synthetic cache contents for decode-only benchmarks (prefill skipped)."""
        g = torch.Generator(device=self.kv.device if self.kv is not None else self.k.device)
        g.manual_seed(seed)
        for t in (self.kv, self.k, self.v):
            if t is not None:
                t.normal_(0.0, std, generator=g)


__all__ = ["BlockAllocator", "KVCache", "PAD_BLOCK"]
