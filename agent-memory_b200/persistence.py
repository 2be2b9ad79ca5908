"""Q4 block persistence: the reference's safetensors cache files, written from and read
straight into pool blocks.

File format (safetensors_cache_adapter.py:71-339): one ``{agent_id}.safetensors`` per
agent, tensors ``L{layer}_B{block}_{K,V}_{weights,scales,biases}`` of shape
``[1, n_kv_heads, tokens, cols]`` (weights uint32 with cols = head_dim/8; scales and
biases in the cache dtype with cols = head_dim/64), string-valued ``__metadata__``.  The
files are interchangeable with the reference's: same names, shapes, dtypes and metadata
rules, standard safetensors framing (8-byte little-endian header length, JSON header,
data section).

The reference builds one mx array per block tensor and lets mx.save_safetensors / mx.load
copy each one.  Here a save is one gather kernel (am_q4_blocks_pack) into a device staging
buffer laid out exactly as the file's data section, one device->host copy into pinned
memory and one file write; a load reads the data section into pinned memory, makes one
host->device copy and one scatter kernel (am_q4_blocks_unpack) places every tensor in its
pool block.  Tensor offsets come from the header, so files written by either
implementation load.
"""

from __future__ import annotations

import json
import logging
import re
import struct
from pathlib import Path
from typing import Any

import torch

from . import _lib, kernels
from .block_pool import AgentBlocks, AgentMemoryError, BlockPool, KVBlock
from .paged import PagedQ4Pool

logger = logging.getLogger(__name__)

_VALID_AGENT_ID = re.compile(r"^[a-zA-Z0-9_-]+$")  # safetensors_cache_adapter.py:26
_SECTIONS = ("K_weights", "K_scales", "K_biases", "V_weights", "V_scales", "V_biases")
_ST_DTYPE = {torch.float16: "F16", torch.bfloat16: "BF16"}


class CachePersistenceError(AgentMemoryError):
    """domain/errors.py CachePersistenceError."""


class AgentNotFoundError(AgentMemoryError):
    """domain/errors.py AgentNotFoundError."""


def _section_geometry(pool: PagedQ4Pool) -> list[tuple[str, int, int]]:
    """(safetensors dtype, cols, bytes per row) of the six tensors of a block."""
    sd = _ST_DTYPE[pool.dtype]
    kd, vd = pool.k_dim, pool.v_dim
    return [("U32", kd // 8, kd // 2), (sd, kd // 64, kd // 32), (sd, kd // 64, kd // 32),
            ("U32", vd // 8, vd // 2), (sd, vd // 64, vd // 32), (sd, vd // 64, vd // 32)]


def block_layout(pool: PagedQ4Pool, layers: dict[int, list[tuple[int, int]]]):
    """Header entries and packing plan for blocks {layer: [(block_id, tokens), ...]}.

    Returns (header dict, block ids, tokens, offsets [n, 6], data bytes); tensors are laid
    out layer by layer, block by block, in _SECTIONS order."""
    geo = _section_geometry(pool)
    H = pool.n_kv_heads
    header: dict[str, Any] = {}
    ids, toks, offs = [], [], []
    pos = 0
    for layer in sorted(layers):
        for b, (bid, T) in enumerate(layers[layer]):
            if not 0 <= T <= pool.block_tokens:
                raise CachePersistenceError(f"block L{layer}_B{b} has {T} tokens")
            row = []
            for name, (dt, cols, rb) in zip(_SECTIONS, geo):
                n = H * T * rb
                header[f"L{layer}_B{b}_{name}"] = {"dtype": dt, "shape": [1, H, T, cols],
                                                   "data_offsets": [pos, pos + n]}
                row.append(pos)
                pos += n
            ids.append(bid)
            toks.append(T)
            offs.append(row)
    return header, ids, toks, offs, pos


def _encode_header(header: dict[str, Any], metadata: dict[str, Any]) -> bytes:
    h = dict(header)
    if metadata:
        h["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    raw = json.dumps(h, separators=(",", ":")).encode("utf-8")
    raw += b" " * (-len(raw) % 8)  # the data section starts 8-byte aligned
    return struct.pack("<Q", len(raw)) + raw


def read_header(path: Path) -> tuple[dict[str, Any], dict[str, str], int]:
    """(tensor entries, metadata, byte offset of the data section) of a safetensors file."""
    try:
        with Path(path).open("rb") as f:
            head = f.read(8)
            if len(head) < 8:
                raise CachePersistenceError(f"Invalid cache file (truncated header): {path}")
            (n,) = struct.unpack("<Q", head)
            header = json.loads(f.read(n).decode("utf-8"))
    except json.JSONDecodeError as e:
        raise CachePersistenceError(f"Corrupted cache metadata for {path}: {e}") from e
    except OSError as e:
        raise CachePersistenceError(f"Failed to read cache file {path}: {e}") from e
    meta = header.pop("__metadata__", {}) or {}
    return header, meta, 8 + n


def save_blocks(path: Path, pool: PagedQ4Pool, layers: dict[int, list[tuple[int, int]]],
                metadata: dict[str, Any] | None = None) -> Path:
    """Write pool blocks {layer: [(block_id, tokens), ...]} to `path` (atomic rename)."""
    path = Path(path)
    header, ids, toks, offs, nbytes = block_layout(pool, layers)
    dev = pool.device
    host = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    if ids:
        staging = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        kernels.blocks_copy(pool.k, pool.v, torch.tensor(ids, dtype=torch.int32),
                            torch.tensor(toks, dtype=torch.int32),
                            torch.tensor(offs, dtype=torch.int64), staging, to_buffer=True,
                            status=status)
        host.copy_(staging)
        if int(status.item()) & _lib.STATUS_BAD_BLOCK:
            raise CachePersistenceError("a block id is outside the pool")
    tmp = path.with_name(path.stem + ".tmp.safetensors")
    try:
        with tmp.open("wb") as f:
            f.write(_encode_header(header, metadata or {}))
            f.write(memoryview(host.numpy()))
        tmp.replace(path)
    except OSError as e:
        raise CachePersistenceError(f"Failed to save cache {path}: {e}") from e
    finally:
        if tmp.exists():
            tmp.unlink()
    return path


def load_blocks(path: Path, pool: PagedQ4Pool, allocate) -> tuple[dict[int, list[tuple[int, int]]],
                                                                  dict[str, str]]:
    """Read a Q4 cache file into pool blocks.  `allocate(layer_id, n_blocks)` returns block
    ids.  Returns ({layer: [(block_id, tokens), ...]}, metadata)."""
    path = Path(path)
    if not path.exists():
        raise AgentNotFoundError(f"Cache not found: {path}")
    header, meta, data_start = read_header(path)
    nbytes = path.stat().st_size - data_start
    geo = _section_geometry(pool)
    H = pool.n_kv_heads
    found: dict[int, set[int]] = {}
    for key in header:
        m = re.match(r"^L(\d+)_B(\d+)_[KV]_", key)
        if m:
            found.setdefault(int(m.group(1)), set()).add(int(m.group(2)))
    # validate every tensor before any block is taken from the allocator
    plan: dict[int, list[tuple[int, list[int]]]] = {}
    for layer in sorted(found):
        blocks = sorted(found[layer])
        if blocks != list(range(len(blocks))):
            raise CachePersistenceError(f"layer {layer} has non-contiguous blocks {blocks}")
        plan[layer] = []
        for b in blocks:
            row, T = [], None
            for name, (dt, cols, rb) in zip(_SECTIONS, geo):
                e = header.get(f"L{layer}_B{b}_{name}")
                if e is None:
                    raise CachePersistenceError(f"L{layer}_B{b}_{name} missing (not a Q4 cache file)")
                shp = list(e["shape"])
                if e["dtype"] != dt or len(shp) != 4 or shp[0] != 1 or shp[1] != H or shp[3] != cols:
                    raise CachePersistenceError(
                        f"L{layer}_B{b}_{name}: {e['dtype']} {shp} does not fit this pool "
                        f"({dt} [1, {H}, T, {cols}])")
                T = shp[2] if T is None else T
                s0, s1 = (int(x) for x in e["data_offsets"])
                if (shp[2] != T or s1 - s0 != H * T * rb or not 0 <= T <= pool.block_tokens or s0 < 0
                        or s1 > nbytes):
                    raise CachePersistenceError(f"L{layer}_B{b}_{name}: inconsistent size or offsets")
                row.append(s0)
            plan[layer].append((T, row))
    layers: dict[int, list[tuple[int, int]]] = {}
    ids, toks, offs = [], [], []
    for layer, entries in plan.items():
        got = list(allocate(layer, len(entries)))
        if len(got) != len(entries):
            raise CachePersistenceError(f"allocator gave {len(got)} blocks for {len(entries)}")
        layers[layer] = []
        for bid, (T, row) in zip(got, entries):
            ids.append(bid)
            toks.append(T)
            offs.append(row)
            layers[layer].append((bid, T))
    if ids:
        host = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
        with path.open("rb") as f:
            f.seek(data_start)
            if f.readinto(memoryview(host.numpy())) != nbytes:
                raise CachePersistenceError(f"truncated data section in {path}")
        staging = host.to(pool.device, non_blocking=True)
        status = torch.zeros(1, dtype=torch.int32, device=pool.device)
        kernels.blocks_copy(pool.k, pool.v, torch.tensor(ids, dtype=torch.int32),
                            torch.tensor(toks, dtype=torch.int32),
                            torch.tensor(offs, dtype=torch.int64), staging, to_buffer=False,
                            status=status)
        if int(status.item()) & _lib.STATUS_BAD_BLOCK:
            raise CachePersistenceError("a block id is outside the pool")
    return layers, meta


class SafetensorsQ4Store:
    """SafetensorsCacheAdapter (safetensors_cache_adapter.py:29-345) over a device pool:
    save() writes an agent's pool blocks, load() reads a file into freshly allocated pool
    blocks.  KVBlock.block_id is the pool row; layer_data stays None (the data lives in the
    pool)."""

    def __init__(self, cache_dir: Path, pool: PagedQ4Pool, allocator: BlockPool) -> None:
        self.cache_dir = Path(cache_dir).expanduser().resolve()
        try:
            self.cache_dir.mkdir(parents=True, exist_ok=True)
        except OSError as e:
            raise CachePersistenceError(f"Failed to create cache directory {self.cache_dir}: {e}") from e
        for tmp in list(self.cache_dir.glob("*.tmp.safetensors")) + list(self.cache_dir.glob("*.safetensors.tmp")):
            try:
                tmp.unlink()
            except OSError:
                pass
        self.pool, self.allocator = pool, allocator

    @staticmethod
    def _validate_agent_id(agent_id: str) -> None:
        if not agent_id:
            raise CachePersistenceError("agent_id cannot be empty")
        if len(agent_id) > 256:
            raise CachePersistenceError(f"agent_id too long: {len(agent_id)} chars (max 256)")
        if not _VALID_AGENT_ID.match(agent_id):
            raise CachePersistenceError(
                f"Invalid agent_id '{agent_id}': must contain only alphanumeric characters, "
                "hyphens, and underscores")

    def path_for(self, agent_id: str) -> Path:
        self._validate_agent_id(agent_id)
        return self.cache_dir / f"{agent_id}.safetensors"

    def save(self, agent_id: str, blocks: AgentBlocks, metadata: dict[str, Any]) -> Path:
        """Write the agent's blocks (block_id = pool row, token_count = tokens held)."""
        path = self.path_for(agent_id)
        bt = metadata.get("block_tokens", self.pool.block_tokens)
        expected = (blocks.total_tokens + bt - 1) // bt
        for layer_id, lb in blocks.blocks.items():
            if len(lb) > expected * 2:  # the reference's corruption guard (:85-104)
                raise CachePersistenceError(
                    f"Cache corruption: layer {layer_id} has {len(lb)} blocks but expected "
                    f"~{expected} for {blocks.total_tokens} tokens")
        layers = {layer: [(blk.block_id, blk.token_count) for blk in lb]
                  for layer, lb in blocks.blocks.items()}
        return save_blocks(path, self.pool, layers, metadata)

    def load(self, cache_path: Path, agent_id: str | None = None):
        """-> ({layer: [KVBlock]}, metadata) with the data placed in newly allocated pool
        blocks owned by agent_id (default: the file's stem)."""
        owner = agent_id or Path(cache_path).stem

        def allocate(layer: int, n: int) -> list[int]:
            return [b.block_id for b in self.allocator.allocate(n, layer, owner)] if n else []

        layers, meta = load_blocks(Path(cache_path), self.pool, allocate)
        out = {layer: [KVBlock(block_id=bid, layer_id=layer, token_count=T, layer_data=None,
                               metadata={"agent_id": owner}) for bid, T in entries]
               for layer, entries in layers.items()}
        return out, meta

    def exists(self, agent_id: str) -> bool:
        return self.path_for(agent_id).exists()

    def delete(self, agent_id: str) -> None:
        p = self.path_for(agent_id)
        if p.exists():
            p.unlink()

    def list_cached_agents(self) -> list[str]:
        return sorted(p.stem for p in self.cache_dir.glob("*.safetensors")
                      if not p.name.endswith(".tmp.safetensors"))
