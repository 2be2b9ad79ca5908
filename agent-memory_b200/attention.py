"""Drop-in quantized attention op and its patch installer.

``quantized_scaled_dot_product_attention`` keeps the signature and semantics of the
function agent-memory installs into ``mlx_lm.models.base``
(src/agent_memory/adapters/outbound/mlx_fused_attention.py:144-207, :462-484):

* ``queries`` [B, Hq, L, Dk] (float16/bfloat16), ``q_keys``/``q_values`` Q4 tuples
  ``(codes [B, Hkv, N, D/8], scales [B, Hkv, N, D/64], biases)``;
* ``mask``: None (every key visible), the string ``"causal"`` (query l at position
  N - L + l, mlx_fused_attention.py:156-161), a boolean keep-mask (masked scores take the
  dtype minimum, :95-98), an additive mask (:99-100), or a :class:`CausalMask` from the
  caches in this package;
* GQA maps query head h to KV head h // (Hq // Hkv) (:76-79);
* returns [B, Hq, L, Dv] in the query dtype.

All batch entries run in one launch (the reference splits the batch into B=1 calls,
:185-207).  L <= 64 / n_rep goes to the split-KV decode kernel; longer query blocks go to
the tcgen05 prefill kernel (head dims 64 and 128), or for head dims without a prefill
instantiation (Gemma-3 D256, MLA K192/V128) to the decode kernel in slices of 64 / n_rep
query positions.  Accumulation is fp32.  group_size/bits other than 64/4 have
no kernel and raise (the reference would call the original MLX op, :164-173).
"""

from __future__ import annotations

import os
from typing import Any

import torch

from . import kernels
from .masks import CausalMask
from .paged_cache import PagedKV, PagedMask

_dispatch_module: Any = None  # module patched by apply_fused_attention_patch


def _as_mask_args(mask, B: int, L: int, N: int, device: torch.device):
    """-> (causal, window, kv_start tensor | None, dense mask | None)."""
    if mask is None:
        return False, 0, None, None
    if isinstance(mask, str):
        if mask != "causal":
            raise ValueError(f"unknown mask string {mask!r}")
        return True, 0, None, None
    if isinstance(mask, CausalMask):
        if mask.n_keys != N or mask.n_queries != L:
            raise ValueError(f"mask covers {mask.n_queries}x{mask.n_keys}, attention is {L}x{N}")
        ks = None
        if mask.left_padding is not None:
            ks = torch.as_tensor(mask.left_padding).to(device=device, dtype=torch.int32)
            if ks.numel() == 1 and B > 1:
                ks = ks.expand(B).contiguous()
        return True, int(mask.window_size or 0), ks, None
    if not torch.is_tensor(mask):
        raise TypeError(f"unsupported mask type {type(mask)}")
    m = mask.to(device)
    while m.dim() < 4:
        m = m.unsqueeze(0)
    if m.shape[-1] != N or m.shape[-2] not in (1, L):
        raise ValueError(f"mask shape {tuple(mask.shape)} does not broadcast to [{B}, *, {L}, {N}]")
    return False, 0, None, m


def quantized_scaled_dot_product_attention(queries: torch.Tensor, q_keys, q_values, scale: float,
                                           mask=None, group_size: int = 64, bits: int = 4,
                                           sinks: torch.Tensor | None = None):
    """Q4 scaled dot-product attention on the GPU (see module docstring).

    ``sinks`` (optional [Hq] logits, scaled-score units) adds one value-less key per head to
    the softmax normaliser, as mx.fast.scaled_dot_product_attention(..., sinks=) does on
    the reference's dequantized fallback (mlx_sink_compat.py:46-69)."""
    kernels._check_params(group_size, bits)
    B, Hq, L, Dk = queries.shape
    if isinstance(q_keys, PagedKV):
        return _paged_attention(queries, q_keys.cache, scale, mask, sinks)
    view, N = kernels.contiguous_view(q_keys, q_values)
    if Hq % view.n_kv_heads:
        raise ValueError(f"{Hq} query heads is not a multiple of {view.n_kv_heads} KV heads")
    if view.desc.batch != B:
        raise ValueError(f"queries have batch {B}, cache has {view.desc.batch}")
    causal, window, kv_start, dense = _as_mask_args(mask, B, L, N, queries.device)
    kv_len = torch.full((B,), N, dtype=torch.int32, device=queries.device)
    return kernels.attention(view, queries, scale, kv_len, N, kv_start=kv_start, causal=causal,
                             window=window, mask=dense, out_dtype=queries.dtype, sinks=sinks)


def _paged_attention(queries, cache, scale, mask, sinks):
    """The drop-in op over a PagedBatchQuantizedKVCache (keys/values from its
    update_and_fetch): each row attends its own [0, len) keys through the block table;
    query l of row b sits at position len[b] - L + l."""
    B, Hq, L, _ = queries.shape
    if B != cache.rows:
        raise ValueError(f"queries have batch {B}, the paged cache has {cache.rows} rows")
    causal, window, dense = False, 0, None
    if isinstance(mask, str):
        if mask != "causal":
            raise ValueError(f"unknown mask string {mask!r}")
        causal = True
    elif isinstance(mask, (PagedMask, CausalMask)):
        causal, window = True, int(mask.window_size or 0)
    elif mask is not None:
        dense = mask.to(queries.device)
        while dense.dim() < 4:
            dense = dense.unsqueeze(0)
    return kernels.attention(cache.view(), queries, scale, cache.kv_len, cache._idx, causal=causal,
                             window=window, mask=dense, out_dtype=queries.dtype, sinks=sinks)


def scaled_dot_product_attention(queries: torch.Tensor, keys, values, cache, scale: float, mask,
                                 sinks: torch.Tensor | None = None):
    """Dispatch shim of mlx_sink_compat._patched_sdpa (mlx_sink_compat.py:36-89).

    With a quantized cache (an object with ``bits``) and no sinks, routes to the Q4 op that
    is currently installed on the patched module (dynamic lookup, :70-81).  With sinks
    (GPT-OSS), the reference dequantizes the Q4 tuples to fp16 and calls the fast SDPA
    (:46-69); here the Q4 kernels take the sinks directly, with no fp16 copy of the cache.
    Non-quantized caches use PyTorch math (not part of the Q4 hot path).
    """
    if hasattr(cache, "bits"):
        if sinks is not None:
            return quantized_scaled_dot_product_attention(
                queries, keys, values, scale, mask, group_size=cache.group_size, bits=cache.bits,
                sinks=sinks)
        op = getattr(_dispatch_module, "quantized_scaled_dot_product_attention",
                     quantized_scaled_dot_product_attention)
        return op(queries, keys, values, scale=scale, mask=mask, group_size=cache.group_size,
                  bits=cache.bits)
    import torch.nn.functional as F

    if sinks is not None:
        return _sdpa_with_sinks(queries, keys, values, scale, mask, sinks)

    attn_mask = mask
    is_causal = False
    if isinstance(mask, str):
        attn_mask, is_causal = None, mask == "causal"
    elif isinstance(mask, CausalMask):
        attn_mask = mask.to_dense(queries.device)
    n_rep = queries.shape[1] // keys.shape[1]
    if n_rep > 1:
        keys = keys.repeat_interleave(n_rep, dim=1)
        values = values.repeat_interleave(n_rep, dim=1)
    return F.scaled_dot_product_attention(queries, keys, values, attn_mask=attn_mask,
                                          is_causal=is_causal, scale=scale)


def _sdpa_with_sinks(queries, keys, values, scale, mask, sinks):
    """Dense attention with per-head sink logits (fp32 math; the non-Q4 fallback)."""
    B, Hq, L, _ = queries.shape
    n_rep = Hq // keys.shape[1]
    k = keys.repeat_interleave(n_rep, dim=1).float()
    v = values.repeat_interleave(n_rep, dim=1).float()
    s = (queries.float() * scale) @ k.transpose(-1, -2)
    N = s.shape[-1]
    if isinstance(mask, str):
        keep = torch.arange(N - L, N, device=s.device)[:, None] >= torch.arange(N, device=s.device)[None]
        s = s.masked_fill(~keep, float("-inf"))
    elif isinstance(mask, CausalMask):
        s = s.masked_fill(~mask.to_dense(s.device), float("-inf"))
    elif mask is not None:
        s = s.masked_fill(~mask, float("-inf")) if mask.dtype == torch.bool else s + mask.float()
    sk = sinks.to(device=s.device, dtype=torch.float32).view(1, Hq, 1, 1).expand(B, Hq, L, 1)
    p = torch.softmax(torch.cat([s, sk], dim=-1), dim=-1)[..., :N]
    return (p @ v).to(queries.dtype)


def apply_fused_attention_patch(base_module: Any) -> bool:
    """Install the Q4 op as ``base_module.quantized_scaled_dot_product_attention``.

    Mirrors apply_fused_attention_patch (mlx_fused_attention.py:27-528): idempotent,
    skipped when SEMANTIC_DISABLE_FUSED_ATTN=1 (returns False), returns True once installed.
    The previous attribute is kept as ``base_module._original_quantized_sdpa``.
    """
    global _dispatch_module
    if getattr(base_module, "_am_b200_patched", False):
        return True
    if os.environ.get("SEMANTIC_DISABLE_FUSED_ATTN", "") == "1":
        return False
    base_module._original_quantized_sdpa = getattr(base_module,
                                                   "quantized_scaled_dot_product_attention", None)
    base_module.quantized_scaled_dot_product_attention = quantized_scaled_dot_product_attention
    base_module._am_b200_patched = True
    _dispatch_module = base_module
    return True
