"""Host-side block accounting for the Q4 block pool.

Mirrors the reference's domain layer so callers keep the same interface:
``ModelCacheSpec`` (domain/value_objects.py:24-132), ``KVBlock`` / ``AgentBlocks``
(domain/entities.py:20-248) and ``BlockPool`` (domain/services.py:31-450).  Block ids are
global across layers (a block belongs to one layer), 256 tokens per block
(entities.py:17).  On the GPU the ids index the rows of the device pool tensors; this
module only decides which ids are in use.
"""

from __future__ import annotations

import threading
from dataclasses import dataclass, field
from typing import Any

BLOCK_SIZE_TOKENS = 256


class AgentMemoryError(Exception):
    """Base class of the domain errors (domain/errors.py)."""


class PoolConfigurationError(AgentMemoryError):
    pass


class PoolExhaustedError(AgentMemoryError):
    pass


class BlockOperationError(AgentMemoryError):
    pass


class BlockValidationError(AgentMemoryError):
    pass


class AgentBlocksValidationError(AgentMemoryError):
    pass


class ModelSpecValidationError(AgentMemoryError):
    pass


@dataclass(frozen=True)
class ModelCacheSpec:
    """KV-cache geometry of a model (value_objects.py:24-132)."""

    n_layers: int
    n_kv_heads: int
    head_dim: int
    block_tokens: int
    layer_types: list[str]
    sliding_window_size: int | None = None
    kv_bits: int | None = 4
    kv_group_size: int = 64
    v_head_dim: int | None = None

    @property
    def effective_v_head_dim(self) -> int:
        return self.head_dim if self.v_head_dim is None else self.v_head_dim

    def __post_init__(self) -> None:
        checks = [
            (self.n_layers > 0, f"n_layers must be > 0, got {self.n_layers}"),
            (self.n_kv_heads > 0, f"n_kv_heads must be > 0, got {self.n_kv_heads}"),
            (self.head_dim > 0, f"head_dim must be > 0, got {self.head_dim}"),
            (self.v_head_dim is None or self.v_head_dim > 0,
             f"v_head_dim must be > 0, got {self.v_head_dim}"),
            (self.block_tokens > 0, f"block_tokens must be > 0, got {self.block_tokens}"),
            (len(self.layer_types) == self.n_layers,
             f"layer_types length ({len(self.layer_types)}) must equal n_layers ({self.n_layers})"),
            (self.kv_bits in (None, 4, 8, 16), f"kv_bits must be one of None/4/8/16, got {self.kv_bits}"),
            (self.kv_group_size > 0, f"kv_group_size must be > 0, got {self.kv_group_size}"),
            (self.kv_group_size & (self.kv_group_size - 1) == 0,
             f"kv_group_size must be a power of 2, got {self.kv_group_size}"),
        ]
        for ok, msg in checks:
            if not ok:
                raise ModelSpecValidationError(msg)

    def bytes_per_block_per_layer(self) -> int:
        """Bytes of one block at one layer: packed codes + 2-byte scale and bias per group."""
        k_el = self.n_kv_heads * self.head_dim * self.block_tokens
        v_el = self.n_kv_heads * self.effective_v_head_dim * self.block_tokens
        total = k_el + v_el
        if self.kv_bits is None or self.kv_bits == 16:
            return total * 2
        groups = -(-k_el // self.kv_group_size) + -(-v_el // self.kv_group_size)
        return (total * self.kv_bits) // 8 + groups * 4

    def max_blocks_for_layer(self, layer_type: str) -> int | None:
        if layer_type == "sliding_window" and self.sliding_window_size is not None:
            return -(-self.sliding_window_size // self.block_tokens)
        return None


@dataclass
class KVBlock:
    """One 256-token block of one layer (entities.py:20-80)."""

    block_id: int
    layer_id: int
    token_count: int
    layer_data: Any
    metadata: dict[str, Any] = field(default_factory=dict)

    def is_full(self) -> bool:
        return self.token_count == BLOCK_SIZE_TOKENS

    def is_empty(self) -> bool:
        return self.token_count == 0

    def __post_init__(self) -> None:
        if self.block_id < 0:
            raise BlockValidationError(f"block_id must be >= 0, got {self.block_id}")
        if self.layer_id < 0:
            raise BlockValidationError(f"layer_id must be >= 0, got {self.layer_id}")
        if not 0 <= self.token_count <= BLOCK_SIZE_TOKENS:
            raise BlockValidationError(
                f"token_count must be 0-{BLOCK_SIZE_TOKENS}, got {self.token_count}")


@dataclass
class AgentBlocks:
    """Blocks of one agent, per layer (entities.py:83-248)."""

    agent_id: str
    blocks: dict[int, list[KVBlock]]
    total_tokens: int
    token_sequence: list[int] = field(default_factory=list)
    prompt_text: str = ""
    metadata: dict[str, Any] = field(default_factory=dict)

    def num_blocks(self) -> int:
        return sum(len(v) for v in self.blocks.values())

    def num_layers(self) -> int:
        return len(self.blocks)

    def blocks_for_layer(self, layer_id: int) -> list[KVBlock]:
        return self.blocks.get(layer_id, [])

    def common_prefix_length(self, query_tokens: list[int]) -> int:
        n = 0
        for a, b in zip(self.token_sequence, query_tokens):
            if a != b:
                break
            n += 1
        return n

    def __post_init__(self) -> None:
        if not self.agent_id:
            raise AgentBlocksValidationError("agent_id must not be empty")
        if self.total_tokens < 0:
            raise AgentBlocksValidationError(f"total_tokens must be >= 0, got {self.total_tokens}")
        for layer_id, blocks in self.blocks.items():
            for blk in blocks:
                if blk.layer_id != layer_id:
                    raise AgentBlocksValidationError(
                        f"block {blk.block_id} has layer_id {blk.layer_id} but is stored under "
                        f"layer {layer_id}")


class BlockPool:
    """Free-list allocator of block ids with per-agent ownership (services.py:31-450).

    LIFO free list, all operations under one lock.  Allocation failures raise
    PoolExhaustedError without changing state.
    """

    def __init__(self, spec: ModelCacheSpec, total_blocks: int) -> None:
        if total_blocks <= 0:
            raise PoolConfigurationError(f"total_blocks must be > 0, got {total_blocks}")
        if spec.n_layers <= 0:
            raise PoolConfigurationError(f"spec.n_layers must be > 0, got {spec.n_layers}")
        self.spec = spec
        self.total_blocks = total_blocks
        self.block_tokens = spec.block_tokens
        self._lock = threading.Lock()
        self.free_list: list[int] = list(range(total_blocks))
        self.allocated_blocks: dict[int, KVBlock] = {}
        self.agent_allocations: dict[str, set[int]] = {}

    def allocate(self, n_blocks: int, layer_id: int, agent_id: str) -> list[KVBlock]:
        with self._lock:
            if n_blocks <= 0:
                raise BlockOperationError(f"n_blocks must be > 0, got {n_blocks}")
            if not 0 <= layer_id < self.spec.n_layers:
                raise BlockOperationError(
                    f"layer_id must be 0-{self.spec.n_layers - 1}, got {layer_id}")
            if len(self.free_list) < n_blocks:
                raise PoolExhaustedError(
                    f"Requested {n_blocks} blocks but only {len(self.free_list)} available. "
                    f"Total pool size: {self.total_blocks}, allocated: {len(self.allocated_blocks)}")
            out = []
            for _ in range(n_blocks):
                bid = self.free_list.pop()
                blk = KVBlock(block_id=bid, layer_id=layer_id, token_count=0, layer_data=None,
                              metadata={"agent_id": agent_id})
                self.allocated_blocks[bid] = blk
                out.append(blk)
            self.agent_allocations.setdefault(agent_id, set()).update(b.block_id for b in out)
            return out

    def free(self, blocks: list[KVBlock], agent_id: str) -> None:
        with self._lock:
            for blk in blocks:
                if blk.block_id not in self.allocated_blocks:
                    raise BlockOperationError(f"Block {blk.block_id} is not allocated (double-free?)")
                owned = self.agent_allocations.get(agent_id)
                if owned is None or blk.block_id not in owned:
                    raise BlockOperationError(f"Block {blk.block_id} does not belong to agent {agent_id}")
                blk.layer_data = None
                self.free_list.append(blk.block_id)
                del self.allocated_blocks[blk.block_id]
                owned.discard(blk.block_id)
            if agent_id in self.agent_allocations and not self.agent_allocations[agent_id]:
                del self.agent_allocations[agent_id]

    def free_agent_blocks(self, agent_id: str) -> int:
        with self._lock:
            ids = self.agent_allocations.pop(agent_id, None)
            if not ids:
                return 0
            n = 0
            for bid in ids:
                blk = self.allocated_blocks.pop(bid, None)
                if blk is not None:
                    blk.layer_data = None
                    self.free_list.append(bid)
                    n += 1
            return n

    def used_memory(self) -> int:
        with self._lock:
            return len(self.allocated_blocks) * self.spec.bytes_per_block_per_layer()

    def available_memory(self) -> int:
        with self._lock:
            return len(self.free_list) * self.spec.bytes_per_block_per_layer()

    def total_memory(self) -> int:
        return self.total_blocks * self.spec.bytes_per_block_per_layer()

    def available_blocks(self) -> int:
        with self._lock:
            return len(self.free_list)

    def allocated_block_count(self) -> int:
        with self._lock:
            return len(self.allocated_blocks)

    def reconfigure(self, new_spec: ModelCacheSpec) -> None:
        with self._lock:
            if self.allocated_blocks:
                raise PoolConfigurationError(
                    f"Cannot reconfigure pool with {len(self.allocated_blocks)} active "
                    "allocations. Drain all agents first.")
            self.spec = new_spec
            self.block_tokens = new_spec.block_tokens
            self.free_list = list(range(self.total_blocks))
            self.allocated_blocks.clear()
            self.agent_allocations.clear()

    def force_clear_all_allocations(self) -> int:
        with self._lock:
            n = len(self.agent_allocations)
            for blk in self.allocated_blocks.values():
                blk.layer_data = None
            self.free_list = list(range(self.total_blocks))
            self.allocated_blocks.clear()
            self.agent_allocations.clear()
            return n

    def max_batch_size(self, tokens_per_agent: int = 256) -> int:
        if tokens_per_agent <= 0:
            raise BlockOperationError(f"tokens_per_agent must be > 0, got {tokens_per_agent}")
        per_agent = -(-tokens_per_agent // self.block_tokens) * self.spec.n_layers
        return self.total_blocks if per_agent == 0 else self.total_blocks // per_agent
