"""Paged BatchQuantizedKVCache: the reference's batch-cache lifecycle as block-table edits.

The reference keeps one left-padded contiguous Q4 tensor per layer
(BatchQuantizedKVCache, mlx_quantized_extensions.py:32-532) and copies it on merge,
extend, filter and extract and on every 256-token capacity growth (:234-271);
batch_engine.py:1745-2064 concatenates 256-token blocks into it and slices them back out.
Here one layer's batch is a block table over a shared :class:`PagedQ4Pool`:

==================  ===========================================================
merge / extend      concatenate table rows (no K/V copy)
filter              keep rows; the dropped rows' blocks go back to the free list
extract             detach one row's blocks into a single-sequence cache
trim                shorten every row; blocks past the new length are released
update_and_fetch    take blocks from the device free list, quantize the new tokens
                    straight into them, advance the lengths (no host sync)
==================  ===========================================================

Rows keep their own lengths instead of left padding: ``left_padding`` is zero, ``offset``
is the per-row length and ``_idx`` the longest row.  Block allocation runs on the device
(:class:`DeviceBlockPool`, the reference's BlockPool free list, services.py:111-223), so a
whole decode step -- growth into new blocks included -- can be captured in a CUDA graph.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import torch

from . import _lib, kernels
from .block_pool import (AgentBlocks, BlockOperationError, BlockPool, KVBlock,
                         PoolExhaustedError)
from .paged import PagedQ4Pool


class DeviceBlockPool:
    """BlockPool's LIFO free list held on the device (domain/services.py:111-223).

    ``free_ids[0:top]`` are the free block ids, the next one handed out last; the initial
    order is BlockPool's (``range(total_blocks)`` popped from the end).  :meth:`reserve`
    and :meth:`release` are device calls (no host sync); errors accumulate in a status
    word that :meth:`check` reads.
    """

    def __init__(self, total_blocks: int, device: torch.device | str = "cuda",
                 order: Sequence[int] | None = None):
        ids = list(range(total_blocks)) if order is None else [int(i) for i in order]
        if len(ids) > total_blocks or any(not 0 <= i < total_blocks for i in ids):
            raise ValueError("free order must list block ids of this pool")
        self.total_blocks = total_blocks
        dev = torch.device(device)
        self.free_ids = torch.full((total_blocks,), -1, dtype=torch.int32, device=dev)
        if ids:
            self.free_ids[:len(ids)] = torch.tensor(ids, dtype=torch.int32, device=dev)
        self.free_top = torch.tensor([len(ids)], dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.device = dev

    @classmethod
    def from_host(cls, pool: BlockPool, device: torch.device | str = "cuda") -> "DeviceBlockPool":
        """Mirror a host BlockPool's current free list (same order, same next block)."""
        return cls(pool.total_blocks, device, order=list(pool.free_list))

    def reserve(self, table: torch.Tensor, lengths: torch.Tensor, add: torch.Tensor,
                block_tokens: int) -> None:
        kernels.block_reserve(self.free_ids, self.free_top, table, lengths, add, block_tokens,
                              self.status)

    def release(self, table: torch.Tensor, keep_blocks: torch.Tensor) -> None:
        kernels.block_release(self.free_ids, self.free_top, table, keep_blocks, self.status)

    def allocate(self, n_blocks: int, layer_id: int = 0, agent_id: str = "") -> list[KVBlock]:
        """BlockPool.allocate (services.py:111-175) from the host: pops n ids (LIFO) and
        returns them as KVBlocks; PoolExhaustedError leaves the pool unchanged.  Syncs."""
        if n_blocks <= 0:
            raise BlockOperationError(f"n_blocks must be > 0, got {n_blocks}")
        tab = torch.full((1, n_blocks), -1, dtype=torch.int32, device=self.device)
        zero = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.reserve(tab, zero, torch.full((1,), n_blocks, dtype=torch.int32, device=self.device), 1)
        self.check()
        return [KVBlock(block_id=int(i), layer_id=layer_id, token_count=0, layer_data=None,
                        metadata={"agent_id": agent_id}) for i in tab[0].tolist()]

    def free(self, blocks: Sequence[KVBlock], agent_id: str = "") -> None:
        """BlockPool.free (services.py:177-223): the ids go back on the stack in order."""
        ids = [int(b.block_id) for b in blocks]
        if not ids:
            return
        tab = torch.tensor([ids], dtype=torch.int32, device=self.device)
        self.release(tab, torch.zeros(1, dtype=torch.int32, device=self.device))

    def available_blocks(self) -> int:
        return int(self.free_top.item())

    def allocated_block_count(self) -> int:
        return self.total_blocks - self.available_blocks()

    def free_list(self) -> list[int]:
        """The free ids in BlockPool order (next to be handed out last)."""
        return self.free_ids[: self.available_blocks()].tolist()

    def check(self) -> None:
        """Raise the domain error for any failed device call since the last check."""
        st = int(self.status.item())
        self.status.zero_()
        if st & _lib.STATUS_POOL_EXHAUSTED:
            raise PoolExhaustedError(
                f"device block pool exhausted ({self.available_blocks()} of {self.total_blocks} free)")
        if st & (_lib.STATUS_BAD_BLOCK | _lib.STATUS_BAD_POSITION):
            raise BlockOperationError(f"device block pool error (status {st:#x})")


@dataclass(frozen=True)
class PagedKV:
    """What update_and_fetch returns for keys and values: a handle on the paged batch
    (the drop-in attention op reads the pool through the cache's block table)."""

    cache: "PagedBatchQuantizedKVCache"
    part: str  # "k" or "v"


@dataclass(frozen=True)
class PagedMask:
    """make_mask() of a paged batch: N query rows at the end of each row's keys, causal,
    optionally within a sliding window (the rows' own lengths replace left padding)."""

    n_queries: int
    window_size: int | None = None


class PagedBatchQuantizedKVCache:
    """One layer's batch of sequences over a :class:`PagedQ4Pool` (see module docstring)."""

    bits = 4
    group_size = 64

    def __init__(self, pool: PagedQ4Pool, allocator: DeviceBlockPool, max_blocks: int,
                 rows: int = 0):
        self.pool, self.allocator = pool, allocator
        self.max_blocks = max(1, int(max_blocks))
        self.table = torch.full((rows, self.max_blocks), -1, dtype=torch.int32, device=pool.device)
        self.lengths: list[int] = [0] * rows
        self.kv_len = torch.zeros(rows, dtype=torch.int32, device=pool.device)

    # ------------------------------------------------------------------ bookkeeping
    @property
    def rows(self) -> int:
        return len(self.lengths)

    @property
    def offset(self) -> torch.Tensor:
        return self.kv_len

    @property
    def left_padding(self) -> torch.Tensor:
        return torch.zeros(self.rows, dtype=torch.int32, device=self.pool.device)

    @property
    def _idx(self) -> int:
        return max(self.lengths, default=0)

    def size(self) -> int:
        return self._idx

    def empty(self) -> bool:
        return self.rows == 0 or self._idx == 0

    def is_trimmable(self) -> bool:
        return True

    def view(self) -> kernels.CacheView:
        return self.pool.view(self.table)

    def _set_rows(self, table: torch.Tensor, lengths: list[int]) -> None:
        self.table = table.contiguous()
        self.lengths = [int(n) for n in lengths]
        self.kv_len = torch.tensor(self.lengths, dtype=torch.int32, device=self.pool.device)

    def _widen(self, width: int) -> None:
        if width > self.table.shape[1]:
            pad = torch.full((self.rows, width - self.table.shape[1]), -1, dtype=torch.int32,
                             device=self.pool.device)
            self.table = torch.cat([self.table, pad], dim=1).contiguous()
            self.max_blocks = width

    # ------------------------------------------------------------------ lifecycle
    @classmethod
    def merge(cls, caches: Sequence["PagedBatchQuantizedKVCache"]) -> "PagedBatchQuantizedKVCache":
        """One batch from several caches of the same pool (mlx_quantized_extensions.py:77-220):
        their rows, in order.  The inputs give up their rows (each block keeps one owner)."""
        if not caches:
            raise ValueError("merge needs at least one cache")
        pool, alloc = caches[0].pool, caches[0].allocator
        if any(c.pool is not pool or c.allocator is not alloc for c in caches):
            raise ValueError("merged caches must share one pool and allocator")
        width = max(c.table.shape[1] for c in caches)
        out = cls(pool, alloc, width)
        for c in caches:
            c._widen(width)
        out._set_rows(torch.cat([c.table for c in caches], dim=0),
                      [n for c in caches for n in c.lengths])
        for c in caches:
            c._set_rows(c.table[:0], [])
        return out

    def extend(self, other: "PagedBatchQuantizedKVCache") -> None:
        """Append other's rows (mlx_quantized_extensions.py:369-435); other gives them up."""
        if other.pool is not self.pool or other.allocator is not self.allocator:
            raise ValueError("extend needs a cache of the same pool and allocator")
        width = max(self.table.shape[1], other.table.shape[1])
        self._widen(width)
        other._widen(width)
        self._set_rows(torch.cat([self.table, other.table], dim=0), self.lengths + other.lengths)
        other._set_rows(other.table[:0], [])

    def filter(self, batch_indices: Sequence[int]) -> None:
        """Keep rows batch_indices (in that order); the other rows' blocks return to the
        free list (mlx_quantized_extensions.py:309-367)."""
        idx = [int(i) for i in batch_indices]
        if any(not 0 <= i < self.rows for i in idx) or len(set(idx)) != len(idx):
            raise IndexError(f"bad batch indices {idx} for {self.rows} rows")
        keep = torch.zeros(self.rows, dtype=torch.int32)
        keep[idx] = self.table.shape[1]
        if len(idx) < self.rows:
            self.allocator.release(self.table, keep.to(self.pool.device))
        sel = torch.tensor(idx, dtype=torch.long, device=self.pool.device)
        self._set_rows(self.table.index_select(0, sel), [self.lengths[i] for i in idx])

    def extract(self, idx: int) -> "PagedBatchQuantizedKVCache":
        """Row idx as a single-sequence cache (mlx_quantized_extensions.py:440-470).  The
        row's blocks move to the returned cache without a copy; the row here is left empty."""
        if not 0 <= idx < self.rows:
            raise IndexError(idx)
        one = type(self)(self.pool, self.allocator, self.table.shape[1])
        one._set_rows(self.table[idx:idx + 1].clone(), [self.lengths[idx]])
        self.table[idx].fill_(-1)
        self.lengths[idx] = 0
        self.kv_len[idx] = 0
        return one

    def trim(self, n: int) -> int:
        """Drop the last n tokens of every row (mlx_quantized_extensions.py:511-515); blocks
        past each row's new length return to the free list."""
        n = min(self._idx, max(0, int(n)))
        if n == 0:
            return 0
        bt = self.pool.block_tokens
        self.lengths = [max(0, L - n) for L in self.lengths]
        keep = torch.tensor([-(-L // bt) for L in self.lengths], dtype=torch.int32,
                            device=self.pool.device)
        self.allocator.release(self.table, keep)
        self.kv_len = torch.tensor(self.lengths, dtype=torch.int32, device=self.pool.device)
        return n

    def free(self) -> None:
        """Return every block to the free list."""
        if self.rows:
            self.allocator.release(self.table, torch.zeros(self.rows, dtype=torch.int32,
                                                           device=self.pool.device))
        self._set_rows(self.table[:0], [])

    # ------------------------------------------------------------------ data path
    def update_and_fetch(self, keys: torch.Tensor, values: torch.Tensor) -> tuple[PagedKV, PagedKV]:
        """Quantize keys/values [rows, Hkv, L, D] onto the end of each row
        (mlx_quantized_extensions.py:224-306): blocks come from the device free list, the
        append kernel writes straight into them, the lengths advance on the device."""
        B, _, L, _ = keys.shape
        if B != self.rows:
            raise ValueError(f"update has {B} rows, the cache has {self.rows}")
        need = -(-(self._idx + L) // self.pool.block_tokens)
        self._widen(need)
        add = torch.full((B,), L, dtype=torch.int32, device=self.pool.device)
        self.allocator.reserve(self.table, self.kv_len, add, self.pool.block_tokens)
        kernels.append(self.view(), keys, values, self.kv_len)
        self.kv_len.add_(L)
        self.lengths = [n + L for n in self.lengths]
        return PagedKV(self, "k"), PagedKV(self, "v")

    def make_mask(self, N: int = 1, return_array: bool = False, window_size: int | None = None,
                  **_: object):
        """Structured mask for N new query rows (mlx_quantized_extensions.py:475-498); with
        return_array, the dense boolean [rows, 1, N, _idx] keep-mask (keys of each row at
        positions [0, len))."""
        if not return_array:
            return PagedMask(N, window_size)
        dev = self.pool.device
        k = torch.arange(self._idx, device=dev)[None, None, :]
        lens = self.kv_len.long()[:, None, None]
        qpos = lens - N + torch.arange(N, device=dev)[None, :, None]
        keep = (k <= qpos) & (k < lens)
        if window_size:
            keep &= k > qpos - window_size
        return keep[:, None]

    @property
    def state(self):
        """Contiguous tuples for persistence (mlx_quantized_extensions.py:517-532): keys and
        values [rows, Hkv, _idx, .] with each row right-aligned (left padding = _idx - len),
        offsets and left padding.  A gather copy; not on the decode path."""
        N = self._idx
        bt = self.pool.block_tokens
        out = []
        for part in (self.pool.k, self.pool.v):
            arrs = []
            for t in part:
                full = torch.zeros((self.rows, t.shape[1], N, t.shape[-1]), dtype=t.dtype,
                                   device=t.device)
                for r, L in enumerate(self.lengths):
                    nb = -(-L // bt)
                    if nb == 0:
                        continue
                    blocks = self.table[r, :nb].long()
                    seq = t.index_select(0, blocks).permute(1, 0, 2, 3).reshape(t.shape[1], nb * bt, -1)
                    full[r, :, N - L:] = seq[:, :L]
                arrs.append(full)
            out.append(tuple(arrs))
        lp = torch.tensor([N - L for L in self.lengths], dtype=torch.int32, device=self.pool.device)
        return out[0], out[1], self.kv_len.clone(), lp


# ---------------------------------------------------------------------- engine glue


def reconstruct_cache(agent_blocks: AgentBlocks, pool: PagedQ4Pool, allocator: DeviceBlockPool,
                      n_layers: int, max_tokens: int | None = None) -> list[PagedBatchQuantizedKVCache]:
    """BatchEngine._reconstruct_cache (batch_engine.py:1745-1882) over pool blocks: one
    single-row cache per layer whose block table lists the agent's blocks -- no
    concatenation, no copy.  With max_tokens, blocks after the first max_tokens tokens are
    not loaded (the EXACT-match shortcut) and go back to the free list.  The caches take
    ownership of the blocks."""
    caches = []
    for layer in range(n_layers):
        blocks = agent_blocks.blocks_for_layer(layer)
        taken, loaded = [], 0
        for blk in blocks:
            if max_tokens is not None and loaded >= max_tokens:
                break
            taken.append(blk)
            loaded += blk.token_count
        rest = blocks[len(taken):]
        if rest:
            allocator.free(rest)
        length = loaded if max_tokens is not None else (agent_blocks.total_tokens if taken else 0)
        c = PagedBatchQuantizedKVCache(pool, allocator, max(1, len(taken)), rows=1)
        if taken:
            c.table[0, :len(taken)] = torch.tensor([b.block_id for b in taken], dtype=torch.int32,
                                                   device=pool.device)
        c._set_rows(c.table, [length])
        caches.append(c)
    return caches


def slice_cache_to_length(caches: Sequence[PagedBatchQuantizedKVCache], target_length: int) -> None:
    """BatchEngine._slice_cache_to_length (batch_engine.py:1690-1743): every row of every
    layer keeps its first target_length tokens; the blocks past them return to the free
    list (a table edit, no copy)."""
    for c in caches:
        if c.rows == 0:
            continue
        bt = c.pool.block_tokens
        c.lengths = [min(L, max(0, int(target_length))) for L in c.lengths]
        keep = torch.tensor([-(-L // bt) for L in c.lengths], dtype=torch.int32, device=c.pool.device)
        c.allocator.release(c.table, keep)
        c.kv_len = torch.tensor(c.lengths, dtype=torch.int32, device=c.pool.device)


def extract_agent_blocks(agent_id: str, caches: Sequence[PagedBatchQuantizedKVCache],
                         token_sequence: list[int] | None = None,
                         prompt_text: str = "") -> AgentBlocks:
    """BatchEngine._extract_cache (batch_engine.py:1884-2064) for single-row paged caches
    (one per layer, e.g. from PagedBatchQuantizedKVCache.extract): the row's block table is
    already the block list, so the AgentBlocks name those pool blocks (block_id = pool row,
    token_count = tokens held) without allocating or slicing anything."""
    blocks: dict[int, list[KVBlock]] = {}
    total = 0
    for layer, c in enumerate(caches):
        if c.rows != 1:
            raise ValueError("extract_agent_blocks takes single-sequence caches")
        n = c.lengths[0]
        if n == 0:
            continue
        bt = c.pool.block_tokens
        ids = c.table[0, :-(-n // bt)].tolist()
        blocks[layer] = [KVBlock(block_id=int(bid), layer_id=layer, token_count=min(bt, n - j * bt),
                                 layer_data=None, metadata={"agent_id": agent_id})
                         for j, bid in enumerate(ids)]
        total = max(total, n)
    return AgentBlocks(agent_id=agent_id, blocks=blocks, total_tokens=total,
                       token_sequence=list(token_sequence or []), prompt_text=prompt_text)
