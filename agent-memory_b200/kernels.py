"""Tensor-level wrappers over the C ABI (PyTorch tensors carry the device memory).

Every function here launches a CUDA kernel from libamq4.so on the current stream of the
tensor's device; nothing runs on the CPU and nothing falls back.  Q4 tuples follow the
reference's ``mx.quantize`` output: ``(codes, scales, biases)`` with codes packed 8 per
32-bit word (held as ``torch.int32``, bit-identical to MLX's uint32) and scales/biases in
the input dtype, one per 64 elements.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Any, Sequence

import torch

from . import _lib
from ._lib import (AttnArgs, DTYPE_BF16, DTYPE_F16, DTYPE_F32, DTYPE_U8, LAYOUT_CONTIGUOUS,
                   LAYOUT_PAGED, MASK_ADDITIVE, MASK_BOOL, MASK_NONE, Q4CacheDesc, check)

GROUP_SIZE = 64
BITS = 4

_DT = {torch.float16: DTYPE_F16, torch.bfloat16: DTYPE_BF16, torch.float32: DTYPE_F32}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DT[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}; expected float16/bfloat16"
                        + (" or float32" if dt is torch.float32 else "")) from None


def _half_code(dt: torch.dtype) -> int:
    if dt not in (torch.float16, torch.bfloat16):
        raise TypeError(f"expected float16 or bfloat16, got {dt}")
    return _DT[dt]


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*ts: torch.Tensor) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("Q4 kernels run on CUDA tensors only (no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("all tensors must live on the same CUDA device")
    return dev


def _check_params(group_size: int, bits: int) -> None:
    if group_size != GROUP_SIZE or bits != BITS:
        raise NotImplementedError(
            f"only group_size=64, bits=4 is implemented (got group_size={group_size}, bits={bits})")


def as_codes(t: torch.Tensor) -> torch.Tensor:
    """View packed codes as int32 (uint32 tensors are reinterpreted bit-for-bit)."""
    if t.dtype == torch.int32:
        return t
    if t.dtype == torch.uint32:
        return t.view(torch.int32)
    raise TypeError(f"Q4 codes must be int32/uint32, got {t.dtype}")


# ----------------------------------------------------------------------------- quantize


def quantize(x: torch.Tensor, group_size: int = 64, bits: int = 4):
    """mx.quantize(x, group_size=64, bits=4) on the GPU.

    x: [..., D] float16/bfloat16 CUDA tensor, D % 64 == 0.  Returns (codes int32 [..., D/8],
    scales [..., D/64], biases [..., D/64]) with scales/biases in x's dtype.
    """
    _check_params(group_size, bits)
    dev = _require_cuda(x)
    dt = _half_code(x.dtype)
    d = x.shape[-1]
    if d % GROUP_SIZE:
        raise ValueError(f"last dimension {d} must be a multiple of {GROUP_SIZE}")
    xc = x.contiguous()
    rows = xc.numel() // d if d else 0
    codes = torch.empty(*x.shape[:-1], d // 8, dtype=torch.int32, device=dev)
    scales = torch.empty(*x.shape[:-1], d // GROUP_SIZE, dtype=x.dtype, device=dev)
    biases = torch.empty_like(scales)
    rc = _lib.load().am_q4_quantize(xc.data_ptr(), dt, rows, d, codes.data_ptr(),
                                    scales.data_ptr(), biases.data_ptr(), _stream(dev))
    check("am_q4_quantize", rc)
    return codes, scales, biases


def dequantize(codes: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
               group_size: int = 64, bits: int = 4, dtype: torch.dtype | None = None):
    """mx.dequantize on the GPU: code * scale + bias, as `dtype` (default: scales' dtype)."""
    _check_params(group_size, bits)
    dev = _require_cuda(codes, scales, biases)
    codes = as_codes(codes).contiguous()
    scales = scales.contiguous()
    biases = biases.contiguous()
    out_dt = scales.dtype if dtype is None else dtype
    d = codes.shape[-1] * 8
    rows = codes.numel() // codes.shape[-1] if codes.shape[-1] else 0
    out = torch.empty(*codes.shape[:-1], d, dtype=out_dt, device=dev)
    rc = _lib.load().am_q4_dequantize(codes.data_ptr(), scales.data_ptr(), biases.data_ptr(),
                                      _half_code(scales.dtype), rows, d, out.data_ptr(),
                                      dtype_code(out_dt), _stream(dev))
    check("am_q4_dequantize", rc)
    return out


# ----------------------------------------------------------------------------- cache views


@dataclass
class CacheView:
    """A Q4 K/V cache as the kernels address it (contiguous or paged), plus keep-alives."""

    desc: Q4CacheDesc
    device: torch.device
    keep: list = field(default_factory=list)

    @property
    def n_kv_heads(self) -> int:
        return self.desc.n_kv_heads

    @property
    def k_dim(self) -> int:
        return self.desc.k_dim

    @property
    def v_dim(self) -> int:
        return self.desc.v_dim

    @property
    def scale_dtype(self) -> torch.dtype:
        return torch.bfloat16 if self.desc.scale_dtype == DTYPE_BF16 else torch.float16


def _capacity_of(t: torch.Tensor) -> int | None:
    """Rows per (batch, head) plane of a [B, H, N, W] tensor that lives in a [B, H, cap, W]
    row-major buffer starting at its data pointer; None if it does not."""
    if t.dim() != 4:
        return None
    B, H, N, W = t.shape
    s0, s1, s2, s3 = t.stride()
    if s3 != 1 or s2 != W or s1 % W:
        return None
    cap = s1 // W
    if cap < N or (B > 1 and s0 != H * s1):
        return None
    if t.data_ptr() % 16:  # the decode kernel moves codes and scales with 16-byte bulk copies
        return None
    # the kernels stream whole 16-row tiles: rows up to ceil16(N) of every plane must exist
    end = t.storage_offset() + (B - 1) * s0 + (H - 1) * s1 + ((N + 15) // 16 * 16) * W
    if end * t.element_size() > t.untyped_storage().nbytes():
        return None
    return cap


def contiguous_view(keys: Sequence[torch.Tensor], values: Sequence[torch.Tensor]) -> tuple[CacheView, int]:
    """CacheView over reference-layout Q4 tuples ([B, Hkv, N, D/8] codes, [B, Hkv, N, D/64]
    scales/biases; N may be a prefix view of a larger capacity).  Returns (view, N).

    Tensors that are not row-major inside a [B, Hkv, cap, .] buffer with cap % 16 == 0 are
    copied (on the GPU) into one that is.
    """
    kc, ks, kb = keys
    vc, vs, vb = values
    dev = _require_cuda(kc, ks, kb, vc, vs, vb)
    kc, vc = as_codes(kc), as_codes(vc)
    if ks.dtype != kb.dtype or ks.dtype != vs.dtype or vs.dtype != vb.dtype:
        raise TypeError("all scales/biases must share one dtype")
    B, H, N, kw = kc.shape
    vw = vc.shape[-1]
    parts = [kc, ks, kb, vc, vs, vb]
    caps = [_capacity_of(t) for t in parts]
    if any(c is None for c in caps) or len(set(caps)) != 1 or caps[0] % 16:
        cap = max(16, (N + 15) // 16 * 16)
        new = []
        for t in parts:
            buf = torch.zeros(B, H, cap, t.shape[-1], dtype=t.dtype, device=dev)
            buf[:, :, :N].copy_(t)
            new.append(buf)
        parts = new
        caps = [cap] * 6
    kc, ks, kb, vc, vs, vb = parts
    d = Q4CacheDesc()
    d.k_codes, d.k_scales, d.k_biases = kc.data_ptr(), ks.data_ptr(), kb.data_ptr()
    d.v_codes, d.v_scales, d.v_biases = vc.data_ptr(), vs.data_ptr(), vb.data_ptr()
    d.scale_dtype = _half_code(ks.dtype)
    d.layout = LAYOUT_CONTIGUOUS
    d.n_kv_heads = H
    d.k_dim = kw * 8
    d.v_dim = vw * 8
    d.block_tokens = 0
    d.capacity = caps[0]
    d.batch = B
    d.block_table_stride = 0
    d.block_table = None
    return CacheView(d, dev, parts), N


def paged_view(k_pool: Sequence[torch.Tensor], v_pool: Sequence[torch.Tensor],
               block_table: torch.Tensor) -> CacheView:
    """CacheView over a block pool: codes [num_blocks, Hkv, block_tokens, D/8], scales and
    biases [num_blocks, Hkv, block_tokens, D/64]; block_table int32 [rows, max_blocks]."""
    kc, ks, kb = k_pool
    vc, vs, vb = v_pool
    dev = _require_cuda(kc, ks, kb, vc, vs, vb, block_table)
    kc, vc = as_codes(kc), as_codes(vc)
    for t in (kc, ks, kb, vc, vs, vb):
        if not t.is_contiguous():
            raise ValueError("pool tensors must be contiguous")
    if block_table.dtype != torch.int32 or block_table.dim() != 2 or not block_table.is_contiguous():
        raise ValueError("block_table must be a contiguous int32 [rows, max_blocks] tensor")
    nb, H, bt, kw = kc.shape
    d = Q4CacheDesc()
    d.k_codes, d.k_scales, d.k_biases = kc.data_ptr(), ks.data_ptr(), kb.data_ptr()
    d.v_codes, d.v_scales, d.v_biases = vc.data_ptr(), vs.data_ptr(), vb.data_ptr()
    d.scale_dtype = _half_code(ks.dtype)
    d.layout = LAYOUT_PAGED
    d.n_kv_heads = H
    d.k_dim = kw * 8
    d.v_dim = vc.shape[-1] * 8
    d.block_tokens = bt
    d.capacity = nb
    d.batch = block_table.shape[0]
    d.block_table_stride = block_table.shape[1]
    d.block_table = block_table.data_ptr()
    return CacheView(d, dev, [kc, ks, kb, vc, vs, vb, block_table])


# ----------------------------------------------------------------------------- append


def append(view: CacheView, keys: torch.Tensor, values: torch.Tensor, positions: torch.Tensor,
           status: torch.Tensor | None = None) -> None:
    """Quantize keys [B, Hkv, L, Dk] / values [B, Hkv, L, Dv] and write token l of sequence b
    at cache position positions[b] + l (through the block table for a paged view)."""
    dev = _require_cuda(keys, values, positions)
    if keys.dtype != view.scale_dtype or values.dtype != view.scale_dtype:
        raise TypeError(f"keys/values must be {view.scale_dtype} to match the cache scales")
    B, H, L, Dk = keys.shape
    if H != view.n_kv_heads or Dk != view.k_dim or values.shape[-1] != view.v_dim:
        raise ValueError(f"append shape {tuple(keys.shape)} does not match the cache geometry")

    def _prep(t):
        if t.stride(-1) != 1 or any(s % 8 for s in t.stride()[:-1]) or t.data_ptr() % 16:
            t = t.contiguous()
        return t

    keys, values = _prep(keys), _prep(values)
    positions = positions.to(device=dev, dtype=torch.int32).contiguous()
    st = status.data_ptr() if status is not None else None
    rc = _lib.load().am_q4_append(ctypes.byref(view.desc), keys.data_ptr(), values.data_ptr(),
                                  _half_code(keys.dtype), B, L, keys.stride(0), keys.stride(1),
                                  keys.stride(2), values.stride(0), values.stride(1),
                                  values.stride(2), positions.data_ptr(), st, _stream(dev))
    check("am_q4_append", rc)


# ----------------------------------------------------------------------------- attention


def _mask_args(args: AttnArgs, mask: torch.Tensor | None, keep: list) -> None:
    args.mask_kind = MASK_NONE
    args.mask = None
    args.mask_dtype = DTYPE_U8
    args.mask_stride_b = args.mask_stride_h = args.mask_stride_l = args.mask_stride_n = 0
    if mask is None:
        return
    m = mask
    if m.dtype == torch.bool:
        m = m.to(torch.uint8)
        args.mask_kind = MASK_BOOL
        args.mask_dtype = DTYPE_U8
    else:
        args.mask_kind = MASK_ADDITIVE
        args.mask_dtype = dtype_code(m.dtype)
    while m.dim() < 4:
        m = m.unsqueeze(0)
    strides = [0 if m.shape[i] == 1 else m.stride(i) for i in range(4)]
    keep.append(m)
    args.mask = m.data_ptr()
    (args.mask_stride_b, args.mask_stride_h, args.mask_stride_l, args.mask_stride_n) = strides


def decode_workspace_bytes(view: CacheView, batch: int, n_q_heads: int, q_len: int,
                           max_kv_len: int, *, window: int = 0) -> int:
    """Workspace bytes a decode call of this shape needs for split-KV partials: 0 when it
    runs as one launch (a single chunk per sequence, or chunks merged inside a thread-block
    cluster), else the partials that the second launch (the combine kernel) merges."""
    a = AttnArgs()
    a.batch, a.n_q_heads, a.q_len = int(batch), int(n_q_heads), int(q_len)
    a.max_kv_len = int(max_kv_len)
    a.window = int(window or 0)
    a.scale = 1.0
    return int(_lib.load().am_q4_attention_workspace_bytes(ctypes.byref(view.desc), ctypes.byref(a)))


def attention_args(view: CacheView, queries: torch.Tensor, scale: float, kv_len: torch.Tensor,
                   max_kv_len: int, *, kv_start: torch.Tensor | None = None, causal: bool = False,
                   window: int = 0, mask: torch.Tensor | None = None,
                   out_dtype: torch.dtype | None = None, out: torch.Tensor | None = None,
                   status: torch.Tensor | None = None, sinks: torch.Tensor | None = None):
    """The am_attn_args of an attention call (arguments as for `attention`) -> (args, keep,
    out): `keep` holds the tensors the args point into, which must outlive every call made
    with them.  Callers that issue the same call repeatedly build the args once."""
    dev = _require_cuda(queries, kv_len)
    B, Hq, L, Dk = queries.shape
    if Dk != view.k_dim:
        raise ValueError(f"query head dim {Dk} != cache k_dim {view.k_dim}")
    q = queries if (queries.stride(-1) == 1 and queries.data_ptr() % 16 == 0
                    and all(s % 8 == 0 for s in queries.stride()[:-1])) else queries.contiguous()
    odt = out_dtype or queries.dtype
    if out is None:
        out = torch.empty(B, Hq, L, view.v_dim, dtype=odt, device=dev)
    elif out.shape != (B, Hq, L, view.v_dim) or out.stride(-1) != 1:
        raise ValueError("out must be [B, Hq, L, Dv] with a contiguous last dim")
    keep = [q, out]
    kv_len = kv_len.to(device=dev, dtype=torch.int32).contiguous()
    keep.append(kv_len)
    a = AttnArgs()
    a.q = q.data_ptr()
    a.q_dtype = _half_code(q.dtype)
    a.batch, a.n_q_heads, a.q_len = B, Hq, L
    a.q_stride_b, a.q_stride_h, a.q_stride_l = q.stride(0), q.stride(1), q.stride(2)
    a.out = out.data_ptr()
    a.out_dtype = dtype_code(out.dtype)
    a.causal = 1 if causal else 0
    a.o_stride_b, a.o_stride_h, a.o_stride_l = out.stride(0), out.stride(1), out.stride(2)
    a.scale = float(scale)
    a.window = int(window or 0)
    a.kv_len = kv_len.data_ptr()
    if kv_start is not None:
        kv_start = kv_start.to(device=dev, dtype=torch.int32).contiguous()
        keep.append(kv_start)
        a.kv_start = kv_start.data_ptr()
    else:
        a.kv_start = None
    a.max_kv_len = int(max_kv_len)
    _mask_args(a, mask, keep)
    a.status = status.data_ptr() if status is not None else None
    if sinks is not None:
        sk = torch.as_tensor(sinks).to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
        if sk.numel() != Hq:
            raise ValueError(f"sinks must hold one logit per query head ({Hq}), got {sk.numel()}")
        keep.append(sk)
        a.sinks = sk.data_ptr()
    else:
        a.sinks = None
    return a, keep, out


def attention(view: CacheView, queries: torch.Tensor, scale: float, kv_len: torch.Tensor,
              max_kv_len: int, *, kv_start: torch.Tensor | None = None, causal: bool = False,
              window: int = 0, mask: torch.Tensor | None = None, out_dtype: torch.dtype | None = None,
              out: torch.Tensor | None = None, status: torch.Tensor | None = None,
              mode: str = "auto", sinks: torch.Tensor | None = None,
              workspace: torch.Tensor | None = None,
              stage_keys: tuple[int, int] | None = None) -> torch.Tensor:
    """Attention of queries [B, Hq, L, Dk] over the cache -> [B, Hq, L, Dv].

    kv_len/kv_start: int32 device tensors [B].  mode: "auto" (library dispatch), "decode"
    (split-KV kernel) or "prefill" (tcgen05 kernel); "prefill_stage" dequantizes only the
    keys at positions stage_keys = (lo, hi) (default: all) into `workspace`, and
    "prefill_attend" runs only the attention kernel over a workspace that stage calls have
    filled (am_q4_prefill_stage / am_q4_prefill_attend).  sinks: optional [Hq]
    attention-sink logits (scaled-score units).  workspace: a contiguous uint8 device tensor
    of at least the call's workspace bytes (256-byte aligned); by default the workspace the
    chosen kernel needs (split-KV partials, or the prefill kernel's fp16 rows of the visible
    keys and values) is allocated here from the caching allocator, on the call's stream.
    """
    a, keep, out = attention_args(view, queries, scale, kv_len, max_kv_len, kv_start=kv_start,
                                  causal=causal, window=window, mask=mask, out_dtype=out_dtype,
                                  out=out, status=status, sinks=sinks)
    dev = out.device
    L_ = _lib.load()
    fn = {"decode": "am_q4_decode", "prefill": "am_q4_prefill",
          "prefill_stage": "am_q4_prefill_stage",
          "prefill_attend": "am_q4_prefill_attend"}.get(mode, "am_q4_attention")
    sizing = {"am_q4_decode": L_.am_q4_decode_workspace_bytes,
              "am_q4_attention": L_.am_q4_attention_workspace_bytes}.get(
                  fn, L_.am_q4_prefill_workspace_bytes)
    ws_bytes = int(sizing(ctypes.byref(view.desc), ctypes.byref(a)))
    if workspace is not None:
        if (workspace.device != dev or workspace.dtype != torch.uint8
                or not workspace.is_contiguous() or workspace.numel() < ws_bytes):
            raise ValueError(f"workspace must be a contiguous uint8 tensor of at least {ws_bytes} "
                             f"bytes on {dev}")
        ws = workspace
    else:
        # the caching allocator's blocks are 512-byte aligned (the prefill workspace needs 256)
        ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev) if ws_bytes else None
    ws_ptr = ws.data_ptr() if ws is not None else None
    if fn == "am_q4_prefill_stage":
        lo, hi = stage_keys if stage_keys is not None else (0, 2 ** 31 - 1)
        rc = L_.am_q4_prefill_stage(ctypes.byref(view.desc), ctypes.byref(a), int(lo), int(hi),
                                    ws_ptr, ws.numel() if ws is not None else 0, _stream(dev))
    else:
        rc = getattr(L_, fn)(ctypes.byref(view.desc), ctypes.byref(a), ws_ptr,
                             ws.numel() if workspace is not None else ws_bytes, _stream(dev))
    check(fn, rc)
    return out


def prefill_workspace_bytes(view: CacheView, batch: int, n_q_heads: int, q_len: int,
                            max_kv_len: int, *, window: int = 0) -> int:
    """Workspace bytes of a prefill call of this shape (fp16 rows of the visible keys and
    values), for callers that keep their own workspaces (mode "prefill_stage" /
    "prefill_attend")."""
    a = AttnArgs()
    a.batch, a.n_q_heads, a.q_len = int(batch), int(n_q_heads), int(q_len)
    a.max_kv_len = int(max_kv_len)
    a.window = int(window or 0)
    a.scale = 1.0
    return int(_lib.load().am_q4_prefill_workspace_bytes(ctypes.byref(view.desc), ctypes.byref(a)))


# ----------------------------------------------------------------------------- pool blocks


def _pool_desc(k_pool: Sequence[torch.Tensor], v_pool: Sequence[torch.Tensor]) -> CacheView:
    """CacheView describing a paged pool without a block table (block-level calls)."""
    dummy = torch.full((1, 1), -1, dtype=torch.int32, device=k_pool[0].device)
    return paged_view(k_pool, v_pool, dummy)


def blocks_copy(k_pool, v_pool, block_ids: torch.Tensor, tokens: torch.Tensor,
                offsets: torch.Tensor, buffer: torch.Tensor, *, to_buffer: bool,
                status: torch.Tensor | None = None) -> None:
    """Copy whole pool blocks to (pack) or from (unpack) a packed uint8 device buffer: block i
    holds six tensors [1, Hkv, tokens[i], cols] (K weights, K scales, K biases, V weights, V
    scales, V biases) at byte offsets offsets[i, 0:6]."""
    view = _pool_desc(k_pool, v_pool)
    dev = _require_cuda(buffer)
    if dev != view.device:
        raise ValueError("buffer and pool must be on the same device")
    n = int(block_ids.numel())
    ids = block_ids.to(device=dev, dtype=torch.int32).contiguous()
    tok = tokens.to(device=dev, dtype=torch.int32).contiguous()
    off = offsets.to(device=dev, dtype=torch.int64).contiguous()
    if tok.numel() != n or off.numel() != 6 * n:
        raise ValueError("tokens must have n entries and offsets n x 6")
    if buffer.dtype != torch.uint8 or not buffer.is_contiguous():
        raise ValueError("buffer must be a contiguous uint8 tensor")
    st = status.data_ptr() if status is not None else None
    L = _lib.load()
    fn = L.am_q4_blocks_pack if to_buffer else L.am_q4_blocks_unpack
    rc = fn(ctypes.byref(view.desc), ids.data_ptr(), tok.data_ptr(), off.data_ptr(), n,
            buffer.data_ptr(), st, _stream(dev))
    check("am_q4_blocks_pack" if to_buffer else "am_q4_blocks_unpack", rc)


def block_reserve(free_ids: torch.Tensor, free_top: torch.Tensor, table: torch.Tensor,
                  lengths: torch.Tensor, add: torch.Tensor, block_tokens: int,
                  status: torch.Tensor | None = None) -> None:
    """Device free list: give each row of `table` blocks for lengths + add tokens."""
    dev = _require_cuda(free_ids, free_top, table, lengths, add)
    for t in (free_ids, free_top, table, lengths, add):
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise ValueError("free list, table, lengths and counts must be contiguous int32")
    rows, stride = table.shape
    rc = _lib.load().am_block_reserve(free_ids.data_ptr(), free_top.data_ptr(), free_ids.numel(),
                                      table.data_ptr(), stride, rows, lengths.data_ptr(),
                                      add.data_ptr(), int(block_tokens),
                                      status.data_ptr() if status is not None else None,
                                      _stream(dev))
    check("am_block_reserve", rc)


def block_release(free_ids: torch.Tensor, free_top: torch.Tensor, table: torch.Tensor,
                  keep_blocks: torch.Tensor, status: torch.Tensor | None = None) -> None:
    """Device free list: return each row's blocks past keep_blocks[r] to the free stack."""
    dev = _require_cuda(free_ids, free_top, table, keep_blocks)
    for t in (free_ids, free_top, table, keep_blocks):
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise ValueError("free list, table and counts must be contiguous int32")
    rows, stride = table.shape
    rc = _lib.load().am_block_release(free_ids.data_ptr(), free_top.data_ptr(), free_ids.numel(),
                                      table.data_ptr(), stride, rows, keep_blocks.data_ptr(),
                                      status.data_ptr() if status is not None else None,
                                      _stream(dev))
    check("am_block_release", rc)
