"""Paged Q4 KV cache: a device block pool addressed through per-layer block tables.

This is the B200-native replacement of the reference's block handling.  The reference
keeps 256-token Q4 blocks per layer (BlockPool, domain/services.py:31-450) but
concatenates them into contiguous left-padded tensors before every attention call
(mlx_cache_adapter.py:46-87, batch_engine.py:1745-1882, merge/extend at
mlx_quantized_extensions.py:77-435).  Here the blocks stay where they are: the append
kernel quantizes straight into pool rows and the attention kernels read through the block
table, so batch composition changes are table edits, not copies.

Device layout (one pool shared by every layer; a block id belongs to one layer):
  K codes  int32 [num_blocks, Hkv, block_tokens, Dk/8]   (8 x 4-bit codes per word)
  K scales f16/bf16 [num_blocks, Hkv, block_tokens, Dk/64], K biases likewise
  V codes / scales / biases with Dv.
A (block, head) slab is contiguous: 256 rows x (Dk/2 + Dk/16) bytes, streamed in 16-token
tiles by the decode kernel.
"""

from __future__ import annotations

import random
from typing import Sequence

import torch

from . import kernels
from .block_pool import BlockPool, KVBlock, ModelCacheSpec


class PagedQ4Pool:
    """Device storage for num_blocks Q4 blocks of one cache geometry."""

    def __init__(self, n_kv_heads: int, k_dim: int, v_dim: int | None, num_blocks: int,
                 block_tokens: int = 256, dtype: torch.dtype = torch.float16,
                 device: torch.device | str = "cuda"):
        v_dim = k_dim if v_dim is None else v_dim
        if k_dim % 64 or v_dim % 64:
            raise ValueError("head dims must be multiples of 64")
        if block_tokens % 16:
            raise ValueError("block_tokens must be a multiple of 16")
        self.n_kv_heads, self.k_dim, self.v_dim = n_kv_heads, k_dim, v_dim
        self.num_blocks, self.block_tokens, self.dtype = num_blocks, block_tokens, dtype
        dev = torch.device(device)
        shp = (num_blocks, n_kv_heads, block_tokens)
        self.k = (torch.zeros(*shp, k_dim // 8, dtype=torch.int32, device=dev),
                  torch.zeros(*shp, k_dim // 64, dtype=dtype, device=dev),
                  torch.zeros(*shp, k_dim // 64, dtype=dtype, device=dev))
        self.v = (torch.zeros(*shp, v_dim // 8, dtype=torch.int32, device=dev),
                  torch.zeros(*shp, v_dim // 64, dtype=dtype, device=dev),
                  torch.zeros(*shp, v_dim // 64, dtype=dtype, device=dev))
        self.device = dev

    @classmethod
    def for_spec(cls, spec: ModelCacheSpec, num_blocks: int, dtype=torch.float16, device="cuda"):
        return cls(spec.n_kv_heads, spec.head_dim, spec.effective_v_head_dim, num_blocks,
                   spec.block_tokens, dtype, device)

    @property
    def bytes_per_block(self) -> int:
        per_row = (self.k_dim // 2 + self.k_dim // 16) + (self.v_dim // 2 + self.v_dim // 16)
        return self.n_kv_heads * self.block_tokens * per_row

    @property
    def nbytes(self) -> int:
        return self.num_blocks * self.bytes_per_block

    def view(self, block_table: torch.Tensor) -> kernels.CacheView:
        return kernels.paged_view(self.k, self.v, block_table)


class PagedLayerCache:
    """One layer's view of a set of agents over a :class:`PagedQ4Pool`.

    Agents are rows of the block table; each has its own length (no left padding).
    Blocks come from the host :class:`BlockPool` (ids = pool rows).
    """

    bits = 4
    group_size = 64

    def __init__(self, pool: PagedQ4Pool, allocator: BlockPool, layer_id: int,
                 agent_ids: Sequence[str], max_tokens: int):
        self.pool, self.allocator, self.layer_id = pool, allocator, layer_id
        self.agent_ids = list(agent_ids)
        self.max_blocks = max(1, -(-max_tokens // pool.block_tokens))
        self.blocks: list[list[KVBlock]] = [[] for _ in self.agent_ids]
        self.lengths = [0] * len(self.agent_ids)
        self._table_host = torch.full((len(self.agent_ids), self.max_blocks), -1, dtype=torch.int32)
        self.table = self._table_host.to(pool.device)
        self.kv_len = torch.zeros(len(self.agent_ids), dtype=torch.int32, device=pool.device)

    # -------------------------------------------------------------- block management
    def reserve(self, row: int, n_tokens: int) -> None:
        """Make sure agent `row` has blocks for n_tokens tokens."""
        need = -(-n_tokens // self.pool.block_tokens)
        if need > self.max_blocks:
            raise ValueError(f"{n_tokens} tokens exceed the table width of {self.max_blocks} blocks")
        have = len(self.blocks[row])
        if need > have:
            new = self.allocator.allocate(need - have, self.layer_id, self.agent_ids[row])
            self.blocks[row].extend(new)
            for i, blk in enumerate(new, start=have):
                self._table_host[row, i] = blk.block_id
            self.table[row].copy_(self._table_host[row], non_blocking=True)

    def free(self, row: int) -> None:
        if self.blocks[row]:
            self.allocator.free(self.blocks[row], self.agent_ids[row])
        self.blocks[row] = []
        self.lengths[row] = 0
        self._table_host[row] = -1
        self.table[row].copy_(self._table_host[row])
        self.kv_len[row] = 0

    def set_lengths(self, lengths: Sequence[int]) -> None:
        self.lengths = list(int(x) for x in lengths)
        self.kv_len.copy_(torch.tensor(self.lengths, dtype=torch.int32))

    # -------------------------------------------------------------- data path
    def view(self) -> kernels.CacheView:
        return self.pool.view(self.table)

    def append(self, keys: torch.Tensor, values: torch.Tensor, positions: torch.Tensor | None = None,
               advance: bool = True) -> None:
        """Quantize keys/values [A, Hkv, L, D] into each agent's next positions."""
        A, _, L, _ = keys.shape
        if A != len(self.agent_ids):
            raise ValueError("append expects one row per agent")
        for r in range(A):
            self.reserve(r, self.lengths[r] + L)
        if positions is None:
            positions = torch.tensor(self.lengths, dtype=torch.int32, device=keys.device)
        kernels.append(self.view(), keys, values, positions)
        if advance:
            self.set_lengths([n + L for n in self.lengths])

    def update_and_fetch(self, keys: torch.Tensor, values: torch.Tensor) -> "PagedLayerCache":
        self.append(keys, values)
        return self

    def attention(self, queries: torch.Tensor, scale: float, *, window: int = 0,
                  causal: bool = True, out: torch.Tensor | None = None,
                  mode: str = "auto") -> torch.Tensor:
        """queries [A, Hq, L, Dk]; query l of agent a sits at position len[a] - L + l."""
        return kernels.attention(self.view(), queries, scale, self.kv_len, max(self.lengths or [0]),
                                 causal=causal and queries.shape[2] > 1, window=window, out=out,
                                 mode=mode)


def shuffled_allocator(spec: ModelCacheSpec, total_blocks: int, seed: int = 0) -> BlockPool:
    """BlockPool whose free list is a seeded permutation, so consecutive allocations land at
    random pool offsets (the multi-agent workload scatters blocks this way)."""
    pool = BlockPool(spec, total_blocks)
    rng = random.Random(seed)
    rng.shuffle(pool.free_list)
    return pool


def lpt_partition(lengths: Sequence[int], n_parts: int) -> list[list[int]]:
    """Greedy longest-processing-time partition of agents by token count: agents sorted by
    length (descending) go to the part with the fewest tokens so far.  Returns agent
    indices per part."""
    parts: list[list[int]] = [[] for _ in range(n_parts)]
    load = [0] * n_parts
    for i in sorted(range(len(lengths)), key=lambda i: (-lengths[i], i)):
        j = min(range(n_parts), key=lambda j: (load[j], j))
        parts[j].append(i)
        load[j] += lengths[i]
    return parts
