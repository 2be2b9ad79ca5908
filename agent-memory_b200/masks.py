"""Structured attention masks.

``create_causal_mask`` restates mlx-lm's mask builder (mlx-lm 0.30.4, third-party, called
by the reference at mlx_quantized_extensions.py:483 and :602-611): N query rows at
positions offset .. offset+N-1 over offset+N keys; query i sees key j when j <= i, and
additionally j > i - window_size with a window and j >= left_padding[b] with left
padding.

Instead of materialising that boolean array on every layer of every step, the caches
return a :class:`CausalMask` describing it; the attention op turns it into the kernels'
structured arguments (causal flag, window, kv_start) and never reads a dense mask.
``to_dense()`` gives the exact array for any other consumer.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class CausalMask:
    n_queries: int
    offset: int
    window_size: int | None = None
    left_padding: torch.Tensor | None = None  # int64 [B] (host or device)

    @property
    def n_keys(self) -> int:
        return self.offset + self.n_queries

    def to_dense(self, device: torch.device | str | None = None) -> torch.Tensor:
        return create_causal_mask(self.n_queries, self.offset, self.window_size,
                                  left_padding=self.left_padding, device=device)


def create_causal_mask(N: int, offset: int = 0, window_size: int | None = None,
                       right_padding: torch.Tensor | None = None,
                       left_padding: torch.Tensor | None = None,
                       device: torch.device | str | None = None) -> torch.Tensor:
    """Boolean keep-mask: [N, offset+N], or [B, 1, N, offset+N] with padding vectors."""
    dev = device if device is not None else (left_padding.device if left_padding is not None
                                             else None)
    rinds = torch.arange(offset + N, device=dev)
    linds = torch.arange(offset, offset + N, device=dev)[:, None]
    rinds = rinds[None]
    mask = linds >= rinds
    if window_size is not None:
        mask = mask & (linds < rinds + window_size)
    if right_padding is not None:
        rp = torch.as_tensor(right_padding, device=dev).reshape(-1, 1, 1, 1)
        mask = mask & (rinds < (offset + N) - rp)
    if left_padding is not None:
        lp = torch.as_tensor(left_padding, device=dev).reshape(-1, 1, 1, 1)
        mask = mask & (lp <= rinds)
    return mask
