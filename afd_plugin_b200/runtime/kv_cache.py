"""Paged KV cache (plus linear-attention state): device pool and a host-side block allocator.

MLA layers cache one ``kv_lora + rope`` latent row per token
(``[L, blocks, block_size, 576]`` for DeepSeek), plus the sparse-attention
indexer's key row when the model has one (``index_k``, DeepSeek-V3.2 /
GLM-MoE-DSA); GQA layers cache K and V
(``[L, blocks, block_size, kv_heads, head_dim]`` each).  A token's slot is
``block_id * block_size + offset``.
"""

from __future__ import annotations

from collections import OrderedDict

import torch

from afd_plugin_b200.models.configs import ModelArchConfig


class BlockAllocator:
    """Block ids with reference counts (block 0 is kept as the padding block).

    With prefix caching, a full block of prompt tokens is registered under a
    hash of its tokens and of every token before it.  When its last user
    releases it, the block keeps its content on an LRU list; a later prompt
    with the same prefix takes it back (:meth:`lookup`) instead of computing
    it again, and allocation reuses such blocks only when no empty one is left.
    """

    def __init__(self, num_blocks: int):
        if num_blocks < 2:
            raise ValueError("need at least two KV blocks")
        self.num_blocks = num_blocks
        self._free = list(range(num_blocks - 1, 0, -1))
        self._ref = [0] * num_blocks
        self._hash_of: dict[int, int] = {}  # block -> content hash
        self._block_of: dict[int, int] = {}  # content hash -> block
        self._evictable: OrderedDict[int, None] = OrderedDict()  # cached, unreferenced, oldest first
        self.queries = 0
        self.hits = 0

    @property
    def num_free(self) -> int:
        return len(self._free) + len(self._evictable)

    @property
    def num_cached(self) -> int:
        return len(self._hash_of)

    def _forget(self, b: int) -> None:
        h = self._hash_of.pop(b, None)
        if h is not None and self._block_of.get(h) == b:
            del self._block_of[h]

    def allocate(self, n: int) -> list[int]:
        if n > self.num_free:
            raise MemoryError(f"KV cache exhausted: want {n} blocks, {self.num_free} free")
        out = []
        for _ in range(n):
            if self._free:
                b = self._free.pop()
            else:  # evict the least recently released cached block
                b, _ = self._evictable.popitem(last=False)
                self._forget(b)
            self._ref[b] = 1
            out.append(b)
        return out

    def free(self, blocks: list[int]) -> None:
        for b in reversed(blocks):
            self._ref[b] -= 1
            if self._ref[b] > 0:
                continue
            if b in self._hash_of:
                self._evictable[b] = None
            else:
                self._free.append(b)

    def lookup(self, hashes: list[int]) -> list[int]:
        """Blocks of the longest cached prefix of ``hashes``, each taken (reference added)."""
        out = []
        for h in hashes:
            self.queries += 1
            b = self._block_of.get(h)
            if b is None:
                break
            self.hits += 1
            if self._ref[b] == 0:
                self._evictable.pop(b, None)
            self._ref[b] += 1
            out.append(b)
        return out

    def register(self, block: int, h: int) -> None:
        """Mark ``block`` as holding the full block of tokens with prefix hash ``h``."""
        if h in self._block_of or block in self._hash_of:
            return
        self._hash_of[block] = h
        self._block_of[h] = block

    def reset_cache(self) -> int:
        """Forget every cached prefix; returns how many blocks were registered."""
        n = len(self._hash_of)
        for b in list(self._evictable):
            self._free.append(b)
        self._evictable.clear()
        self._hash_of.clear()
        self._block_of.clear()
        return n


def block_hashes(tokens: list[int], block_size: int) -> list[int]:
    """Chained hashes of the full blocks of ``tokens`` (each covers its block and all before it)."""
    out, h = [], 0
    for i in range(len(tokens) // block_size):
        h = hash((h, tuple(tokens[i * block_size : (i + 1) * block_size])))
        out.append(h)
    return out


PAD_BLOCK = 0


class KVCache:
    """Per-layer decode state.

    Full-attention layers get paged KV; Gated DeltaNet (linear attention)
    layers get per-sequence recurrent state instead: a conv state
    ``[max_seqs, conv_dim, K - 1]`` and an fp32 delta-rule state
    ``[max_seqs, nv, dk, dv]``, addressed by the sequence's state slot.
    """

    def __init__(
        self,
        arch: ModelArchConfig,
        num_blocks: int,
        block_size: int,
        dtype: torch.dtype,
        device: torch.device | str,
        *,
        max_seqs: int = 1,
    ):
        self.arch = arch
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.max_seqs = max_seqs
        attn_layers = arch.full_attention_layers
        self._kv_index = {layer: i for i, layer in enumerate(attn_layers)}
        L = len(attn_layers)
        self.index_k = None
        if arch.is_mla:
            self.kv = torch.zeros(L, num_blocks, block_size, arch.kv_lora_rank + arch.qk_rope_head_dim,
                                  dtype=dtype, device=device)
            self.k = self.v = None
            if arch.has_indexer:
                # DeepSeek sparse attention: the indexer's key row per position
                self.index_k = torch.zeros(L, num_blocks, block_size, arch.index_head_dim, dtype=dtype,
                                           device=device)
        else:
            shape = (L, num_blocks, block_size, arch.num_key_value_heads, arch.head_dim)
            self.k = torch.zeros(shape, dtype=dtype, device=device)
            self.v = torch.zeros(shape, dtype=dtype, device=device)
            self.kv = None
        lin = arch.linear_attention_layers
        self._state_index = {layer: i for i, layer in enumerate(lin)}
        self.conv_state = self.ssm_state = None
        if lin:
            self.conv_state = torch.zeros(len(lin), max_seqs, arch.linear_conv_dim, arch.linear_conv_kernel_dim - 1,
                                          dtype=dtype, device=device)
            self.ssm_state = torch.zeros(len(lin), max_seqs, arch.linear_num_value_heads, arch.linear_key_head_dim,
                                         arch.linear_value_head_dim, dtype=torch.float32, device=device)
        self.allocator = BlockAllocator(num_blocks)

    def layer(self, i: int):
        if i in self._state_index:
            j = self._state_index[i]
            return (self.conv_state[j], self.ssm_state[j])
        j = self._kv_index[i]
        if self.index_k is not None:
            return (self.kv[j], self.index_k[j])
        if self.kv is not None:
            return self.kv[j]
        return (self.k[j], self.v[j])

    @staticmethod
    def bytes_per_block(arch: ModelArchConfig, block_size: int, dtype: torch.dtype) -> int:
        elem = torch.empty((), dtype=dtype).element_size()
        return len(arch.full_attention_layers) * block_size * arch.kv_cache_width * elem

    @staticmethod
    def state_bytes_per_seq(arch: ModelArchConfig, dtype: torch.dtype) -> int:
        """Recurrent-state bytes one sequence holds over all linear-attention layers."""
        lin = len(arch.linear_attention_layers)
        if not lin:
            return 0
        elem = torch.empty((), dtype=dtype).element_size()
        conv = arch.linear_conv_dim * (arch.linear_conv_kernel_dim - 1) * elem
        ssm = arch.linear_num_value_heads * arch.linear_key_head_dim * arch.linear_value_head_dim * 4
        return lin * (conv + ssm)

    def fill_random_(self, seed: int = 0, std: float = 1.0) -> None:
        """Synthetic cache contents for decode-only benchmarks (prefill skipped)."""
        dev = next(t for t in (self.kv, self.k, self.conv_state) if t is not None).device
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        for t in (self.kv, self.index_k, self.k, self.v, self.conv_state):
            if t is not None:
                t.normal_(0.0, std, generator=g)
        if self.ssm_state is not None:
            self.ssm_state.normal_(0.0, 0.02, generator=g)


__all__ = ["BlockAllocator", "KVCache", "PAD_BLOCK", "block_hashes"]
