"""Q4 KV caches with the reference's interface, backed by CUDA tensors.

* :class:`QuantizedKVCache` — single-sequence Q4 cache with mlx-lm 0.30.4's
  ``QuantizedKVCache`` semantics (256-step capacity growth) plus the reference's patches:
  ``size()`` returns the offset, ``make_mask`` honours ``window_size`` and ``merge`` builds
  a :class:`BatchQuantizedKVCache` (mlx_quantized_extensions.py:575-630).
* :class:`BatchQuantizedKVCache` — batched, left-padded Q4 cache
  (mlx_quantized_extensions.py:32-532): ``merge``, ``prepare``/``finalize``,
  ``update_and_fetch``, ``filter``, ``extend``, ``extract``, ``make_mask``, ``trim``,
  ``state``.

``update_and_fetch`` quantizes the new tokens and scatters them into the capacity buffers
in ONE kernel (am_q4_append) instead of quantize + slice-update + eval.  Buffers are
allocated with their token capacity rounded up to 16 rows (tensors still report the
reference's shapes) so the attention kernels can stream whole 16-token tiles.
Offsets and left padding are host int64 tensors, as bookkeeping.
"""

from __future__ import annotations

from typing import Any, Sequence

import torch

from . import kernels
from .masks import CausalMask

Q4 = tuple  # (codes int32, scales, biases)


def _alloc(B: int, H: int, rows: int, width: int, dtype: torch.dtype,
           device: torch.device) -> torch.Tensor:
    """Zeroed [B, H, rows, width] view of a buffer with rows rounded up to 16."""
    rows16 = max(16, (rows + 15) // 16 * 16)
    return torch.zeros(B, H, rows16, width, dtype=dtype, device=device)[:, :, :rows, :]


def _alloc_q4(B: int, H: int, rows: int, dim: int, dtype: torch.dtype, device) -> Q4:
    return (_alloc(B, H, rows, dim // 8, torch.int32, device),
            _alloc(B, H, rows, dim // 64, dtype, device),
            _alloc(B, H, rows, dim // 64, dtype, device))


def _copy_rows(dst: Q4, src: Q4, b_dst: slice | int, b_src: slice | int, d0: int, s0: int, n: int):
    for d, s in zip(dst, src):
        d[b_dst, :, d0:d0 + n].copy_(s[b_src, :, s0:s0 + n])


def _view_desc(keys: Q4, values: Q4) -> kernels.CacheView:
    view, _ = kernels.contiguous_view(keys, values)
    return view


class QuantizedKVCache:
    """Single-sequence Q4 cache (mlx-lm QuantizedKVCache semantics + reference patches)."""

    step = 256

    def __init__(self, group_size: int = 64, bits: int = 4):
        kernels._check_params(group_size, bits)
        self.keys: Q4 | None = None
        self.values: Q4 | None = None
        self.offset = 0
        self.group_size = group_size
        self.bits = bits

    def update_and_fetch(self, keys: torch.Tensor, values: torch.Tensor):
        B, H, num_steps, kd = keys.shape
        vd = values.shape[-1]
        prev = self.offset
        if self.keys is None or prev + num_steps > self.keys[0].shape[-2]:
            new_steps = (self.step + num_steps - 1) // self.step * self.step
            if self.keys is not None:
                keep = prev if prev % self.step != 0 else self.keys[0].shape[-2]
                rows = keep + new_steps
                nk = _alloc_q4(B, H, rows, kd, keys.dtype, keys.device)
                nv = _alloc_q4(B, H, rows, vd, keys.dtype, keys.device)
                _copy_rows(nk, self.keys, slice(None), slice(None), 0, 0, keep)
                _copy_rows(nv, self.values, slice(None), slice(None), 0, 0, keep)
                self.keys, self.values = nk, nv
            else:
                self.keys = _alloc_q4(B, H, new_steps, kd, keys.dtype, keys.device)
                self.values = _alloc_q4(B, H, new_steps, vd, keys.dtype, keys.device)
        view = _view_desc(self.keys, self.values)
        pos = torch.full((B,), prev, dtype=torch.int32, device=keys.device)
        kernels.append(view, keys, values, pos)
        self.offset += num_steps
        return (tuple(x[..., :self.offset, :] for x in self.keys),
                tuple(x[..., :self.offset, :] for x in self.values))

    # reference patch: size() returns the offset (mlx_quantized_extensions.py:617-625)
    def size(self) -> int:
        return self.offset

    def empty(self) -> bool:
        return self.keys is None

    def is_trimmable(self) -> bool:
        return True

    def trim(self, n: int) -> int:
        n = min(self.offset, n)
        self.offset -= n
        return n

    # reference patch: window-aware mask (mlx_quantized_extensions.py:601-612)
    def make_mask(self, N: int = 1, return_array: bool = False, window_size: int | None = None,
                  **kwargs):
        if window_size is not None:
            if N == 1 and self.offset <= window_size:
                return None
            return CausalMask(N, self.offset, window_size)
        if N == 1:
            return None
        if return_array:
            return CausalMask(N, self.offset)
        return "causal"

    @property
    def state(self):
        if self.keys is not None and self.offset < self.keys[0].shape[-2]:
            return (tuple(x[..., :self.offset, :] for x in self.keys),
                    tuple(x[..., :self.offset, :] for x in self.values))
        return self.keys, self.values

    @state.setter
    def state(self, v):
        self.keys, self.values = v
        self.offset = 0 if self.keys is None else self.keys[0].shape[-2]

    @property
    def meta_state(self):
        return tuple(map(str, (self.step, self.offset, self.group_size, self.bits)))

    @meta_state.setter
    def meta_state(self, v):
        self.step, self.offset, self.group_size, self.bits = map(int, v)

    @classmethod
    def merge(cls, caches: Sequence[Any]) -> "BatchQuantizedKVCache":
        return BatchQuantizedKVCache.merge(caches)


class BatchQuantizedKVCache:
    """Batched left-padded Q4 cache (mlx_quantized_extensions.py:32-532)."""

    step = 256

    def __init__(self, left_padding: list[int] | None = None, group_size: int = 64, bits: int = 4,
                 n_q_heads: int | None = None, n_kv_heads: int | None = None):
        kernels._check_params(group_size, bits)
        self.keys: Q4 | None = None
        self.values: Q4 | None = None
        self.group_size = group_size
        self.bits = bits
        self._n_q_heads = n_q_heads
        self._n_kv_heads = n_kv_heads
        self._right_padding: torch.Tensor | None = None
        if left_padding:
            self.left_padding = torch.tensor(left_padding, dtype=torch.int64)
            self.offset = -self.left_padding.clone()
        else:
            self.left_padding = torch.tensor([0], dtype=torch.int64)
            self.offset = torch.tensor([0], dtype=torch.int64)
        self._idx = 0

    # -------------------------------------------------------------- merge
    @classmethod
    def merge(cls, caches: Sequence[Any]) -> "BatchQuantizedKVCache":
        if not caches:
            raise ValueError("Cannot merge empty cache list")
        src = next((c for c in caches if hasattr(c, "bits") and hasattr(c, "group_size")), None)
        if src is None:
            raise ValueError("No QuantizedKVCache found in merge list")
        kw = dict(group_size=src.group_size, bits=src.bits,
                  n_q_heads=getattr(src, "_n_q_heads", None),
                  n_kv_heads=getattr(src, "_n_kv_heads", None))
        lengths = [int(c.offset) for c in caches]
        max_length = max(lengths)
        lp = [max_length - n for n in lengths]
        B = len(caches)
        if max_length == 0:
            out = cls(**kw)
            out.left_padding = torch.zeros(B, dtype=torch.int64)
            out.offset = torch.zeros(B, dtype=torch.int64)
            return out
        sample = next(c for c in caches if c.keys is not None)
        kq, ks, _ = sample.keys
        vq, _, _ = sample.values
        H = kq.shape[1]
        dev, dt = kq.device, ks.dtype
        keys = _alloc_q4(B, H, max_length, kq.shape[-1] * 8, dt, dev)
        values = _alloc_q4(B, H, max_length, vq.shape[-1] * 8, dt, dev)
        for i, (p, c) in enumerate(zip(lp, caches)):
            if c.keys is None:
                continue
            src_len = c.keys[0].shape[-2]
            n = min(int(c.offset), src_len)
            if p + n > max_length:
                raise ValueError(f"Merge bounds error: cache {i} writes to {p + n} but "
                                 f"max_length={max_length}")
            _copy_rows(keys, c.keys, slice(i, i + 1), slice(0, 1), p, 0, n)
            _copy_rows(values, c.values, slice(i, i + 1), slice(0, 1), p, 0, n)
        out = cls(**kw)
        out.keys, out.values = keys, values
        out.offset = torch.tensor(lengths, dtype=torch.int64)
        out.left_padding = torch.tensor(lp, dtype=torch.int64)
        out._idx = max_length
        return out

    # -------------------------------------------------------------- prepare / finalize
    def prepare(self, *, left_padding: list[int] | None = None, lengths: list[int] | None = None,
                right_padding: list[int] | None = None) -> None:
        if left_padding is not None:
            if self.keys is not None:
                raise ValueError("Left padding can only be added to an empty BatchQuantizedKVCache")
            lp = torch.tensor(left_padding, dtype=torch.int64)
            self.left_padding = self.left_padding + lp
            self.offset = self.offset - lp
        if right_padding is not None and max(right_padding) > 0:
            self._right_padding = torch.tensor(right_padding, dtype=torch.int64)

    def finalize(self) -> None:
        if self._right_padding is None:
            return
        pad = self._right_padding
        if self.keys is not None:
            self.keys = _dynamic_roll(self.keys, pad)
            self.values = _dynamic_roll(self.values, pad)
        self.offset = self.offset - pad
        self.left_padding = self.left_padding + pad
        self._right_padding = None

    # -------------------------------------------------------------- update_and_fetch
    def update_and_fetch(self, keys: torch.Tensor, values: torch.Tensor):
        B, H, num_steps, kd = keys.shape
        vd = values.shape[-1]
        prev = self._idx
        required = prev + num_steps + 1
        if self.keys is None or required > self.keys[0].shape[-2]:
            new_capacity = (required + 256 + self.step - 1) // self.step * self.step
            if self.keys is not None:
                new_steps = new_capacity - prev
                keep = prev if prev % self.step != 0 else self.keys[0].shape[-2]
                rows = keep + new_steps
                nk = _alloc_q4(B, H, rows, kd, keys.dtype, keys.device)
                nv = _alloc_q4(B, H, rows, vd, keys.dtype, keys.device)
                _copy_rows(nk, self.keys, slice(None), slice(None), 0, 0, keep)
                _copy_rows(nv, self.values, slice(None), slice(None), 0, 0, keep)
                self.keys, self.values = nk, nv
            else:
                self.keys = _alloc_q4(B, H, new_capacity, kd, keys.dtype, keys.device)
                self.values = _alloc_q4(B, H, new_capacity, vd, keys.dtype, keys.device)
        cap = self.keys[0].shape[-2]
        n = min(num_steps, cap - prev)
        view = _view_desc(self.keys, self.values)
        pos = torch.full((B,), prev, dtype=torch.int32, device=keys.device)
        kernels.append(view, keys[:, :, :n], values[:, :, :n], pos)
        self._idx += n
        self.offset = self.offset + n
        return (tuple(x[..., :self._idx, :] for x in self.keys),
                tuple(x[..., :self._idx, :] for x in self.values))

    # -------------------------------------------------------------- filter / extend / extract
    def filter(self, batch_indices) -> None:
        if self.keys is None:
            return
        idx = torch.as_tensor(batch_indices, dtype=torch.int64)
        self.offset = self.offset[idx]
        self.left_padding = self.left_padding[idx]
        min_pad = int(self.left_padding.min().item())
        didx = idx.to(self.keys[0].device)
        cap = self.keys[0].shape[-2]
        rows = cap - min_pad
        B = idx.numel()
        H = self.keys[0].shape[1]

        def _take(q: Q4) -> Q4:
            out = _alloc_q4(B, H, rows, q[0].shape[-1] * 8, q[1].dtype, q[0].device)
            for d, s in zip(out, q):
                d.copy_(s.index_select(0, didx)[:, :, min_pad:])
            return out

        self.keys, self.values = _take(self.keys), _take(self.values)
        if min_pad > 0:
            self._idx -= min_pad
            self.left_padding = self.left_padding - min_pad

    def extend(self, other: "BatchQuantizedKVCache") -> None:
        if other.keys is None:
            self.offset = torch.cat([self.offset, other.offset])
            self.left_padding = torch.cat([self.left_padding, other.left_padding])
            return
        if self.keys is None:
            self.keys, self.values = other.keys, other.values
            self.offset = torch.cat([self.offset, other.offset])
            self.left_padding = torch.cat([self.left_padding, other.left_padding])
            self._idx = other._idx
            return
        max_idx = max(self._idx, other._idx)
        B1, B2 = self.keys[0].shape[0], other.keys[0].shape[0]
        H = self.keys[0].shape[1]
        dev, dt = self.keys[0].device, self.keys[1].dtype
        kd, vd = self.keys[0].shape[-1] * 8, self.values[0].shape[-1] * 8
        nk = _alloc_q4(B1 + B2, H, max_idx, kd, dt, dev)
        nv = _alloc_q4(B1 + B2, H, max_idx, vd, dt, dev)
        for c, b0 in ((self, 0), (other, B1)):
            left = max_idx - c._idx
            nb = c.keys[0].shape[0]
            _copy_rows(nk, c.keys, slice(b0, b0 + nb), slice(None), left, 0, c._idx)
            _copy_rows(nv, c.values, slice(b0, b0 + nb), slice(None), left, 0, c._idx)
        lp1 = self.left_padding + (max_idx - self._idx)
        lp2 = other.left_padding + (max_idx - other._idx)
        self.keys, self.values = nk, nv
        self.offset = torch.cat([self.offset, other.offset])
        self.left_padding = torch.cat([lp1, lp2])
        self._idx = max_idx

    def extract(self, idx: int) -> QuantizedKVCache:
        cache = QuantizedKVCache(group_size=self.group_size, bits=self.bits)
        if self.keys is not None:
            pad = int(self.left_padding[idx].item())
            end = self._idx
            H = self.keys[0].shape[1]
            dev, dt = self.keys[0].device, self.keys[1].dtype
            cache.keys = _alloc_q4(1, H, end - pad, self.keys[0].shape[-1] * 8, dt, dev)
            cache.values = _alloc_q4(1, H, end - pad, self.values[0].shape[-1] * 8, dt, dev)
            _copy_rows(cache.keys, self.keys, slice(0, 1), slice(idx, idx + 1), 0, pad, end - pad)
            _copy_rows(cache.values, self.values, slice(0, 1), slice(idx, idx + 1), 0, pad, end - pad)
            cache.offset = end - pad
        return cache

    # -------------------------------------------------------------- masks / bookkeeping
    def make_mask(self, N: int = 1, return_array: bool = False, **kwargs) -> CausalMask:
        """Structured stand-in for create_causal_mask(N, offset=_idx, left_padding, window)."""
        return CausalMask(N, self._idx, kwargs.get("window_size"), self.left_padding)

    def empty(self) -> bool:
        return self.keys is None

    def size(self) -> int:
        return self._idx

    def is_trimmable(self) -> bool:
        return True

    def trim(self, n: int) -> int:
        n = min(self._idx, n)
        self._idx -= n
        self.offset = self.offset - n
        return n

    @property
    def state(self):
        k, v = self.keys, self.values
        if k is not None and self._idx < k[0].shape[-2]:
            k = tuple(x[..., :self._idx, :] for x in k)
            v = tuple(x[..., :self._idx, :] for x in v)
        return k, v, self.offset, self.left_padding

    @state.setter
    def state(self, new_state) -> None:
        self.keys, self.values, self.offset, self.left_padding = new_state
        self._idx = 0 if self.keys is None else self.keys[0].shape[-2]


def _dynamic_roll(q4: Q4, shifts: torch.Tensor) -> Q4:
    """Roll each batch row along the token axis by its shift (right -> left padding)."""
    out = []
    for t in q4:
        B, H, rows, W = t.shape
        buf = _alloc(B, H, rows, W, t.dtype, t.device)
        for b in range(B):
            buf[b].copy_(torch.roll(t[b], shifts=int(shifts[b]), dims=1))
        out.append(buf)
    return tuple(out)


def validate_q4_pipeline() -> bool:
    """Startup self-check of the cache interface (mlx_quantized_extensions.py:761-836)."""
    c = QuantizedKVCache(group_size=64, bits=4)
    c.offset = 42
    if c.size() != 42:
        return False
    if not isinstance(QuantizedKVCache.merge([QuantizedKVCache()]), BatchQuantizedKVCache):
        return False
    c = QuantizedKVCache(group_size=64, bits=4)
    c.offset = 1000
    m = c.make_mask(N=512, window_size=256)
    if m is None or (isinstance(m, str) and m == "causal"):
        return False
    return True
