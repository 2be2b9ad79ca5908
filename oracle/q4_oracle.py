"""CPU oracle for the Q4 KV-cache attention path (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
import this module.  The product package never does: its kernels must run on the
GPU or fail loudly.

Two independent restatements live here:

* pure NumPy (:func:`quantize_np`, :func:`dequantize_np`, :func:`attention_np`,
  :func:`attention_mlx_fp16_np`) for small cases, and
* the C/OpenMP restatement in ``q4_oracle.c`` (:func:`quantize`,
  :func:`attention`), used for larger cases and as the timed CPU baseline.

Sources restated (reference paths are relative to the agent-memory repository):

* affine Q4 quantization, group 64: mlx 0.30.3 ``mx.quantize`` (third-party,
  pyproject.toml:33, not vendored; in the mlx sources mlx/backend/cpu/quantized.cpp and
  the Metal kernels' affine_quantize), called at
  src/agent_memory/adapters/outbound/mlx_quantized_extensions.py:273-274.  Ties round to
  the even code (rint); codes come from the fp32 scale/bias before their rounding to the
  storage dtype (the corner cases are listed in q4_oracle.c's header);
* dequantization ``code * scale + bias``: mlx_fused_attention.py:274-288;
* attention op order (scale q, q.k^T, bool mask -> dtype min / additive mask
  added, softmax in fp32, P.V) and GQA reshape: mlx_fused_attention.py:69-139;
* the structured mask (causal offset, window, left padding): mlx-lm's
  ``create_causal_mask`` as called at mlx_quantized_extensions.py:483, :601-615.

Parity status: there is no golden vector produced by mlx itself (mlx is not
installed here and the reference's tests hold no known-answer values), so the
bit-exactness of the quantizer against mlx is UNPINNED.  What the reference's
tests do pin (dtype rule, shapes, byte formula, persistence bit-identity,
batch-split consistency) is checked in tests/test_oracle.py, and the two
restatements below are checked against each other bit-for-bit.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

GROUP = 64
F16, BF16, F32 = 0, 1, 2
CONTIGUOUS, PAGED = 0, 1
MASK_NONE, MASK_BOOL, MASK_ADDITIVE = 0, 1, 2

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "libq4oracle.so"


# --------------------------------------------------------------------------------------
# 16-bit float helpers.  bf16 values are carried as uint16 bit patterns (NumPy has no bf16).
# --------------------------------------------------------------------------------------


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16).astype(np.uint16)
    r = np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)
    return r


def to_f32(x16: np.ndarray, dtype: int) -> np.ndarray:
    """uint16 bit patterns (or float16 array) of `dtype` -> float32."""
    if dtype == BF16:
        return bf16_bits_to_f32(x16)
    return np.asarray(x16).view(np.float16).astype(np.float32)


def from_f32(x: np.ndarray, dtype: int) -> np.ndarray:
    """float32 -> uint16 bit patterns of `dtype` (round to nearest even)."""
    if dtype == BF16:
        return f32_to_bf16_bits(x)
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


# --------------------------------------------------------------------------------------
# NumPy restatement
# --------------------------------------------------------------------------------------


def quantize_np(x16: np.ndarray, dtype: int = F16):
    """mx.quantize(x, group_size=64, bits=4) restated in NumPy float32 arithmetic.

    ``x16``: uint16 bit patterns (or float16 values) shaped [..., D], D % 64 == 0.
    Returns (codes uint32 [..., D/8], scales uint16-bits [..., D/64], biases [..., D/64]).
    """
    x16 = np.asarray(x16)
    shape = x16.shape
    d = shape[-1]
    if d % GROUP:
        raise ValueError(f"last dim {d} is not a multiple of {GROUP}")
    w = to_f32(x16.reshape(-1), dtype).reshape(-1, GROUP)
    f = np.float32
    w_max = w.max(axis=1)
    w_min = w.min(axis=1)
    side = np.abs(w_min) > np.abs(w_max)
    scale = np.maximum((w_max - w_min) / f(15.0), f(1e-7)).astype(f)
    scale = np.where(side, scale, -scale).astype(f)
    edge = np.where(side, w_min, w_max).astype(f)
    with np.errstate(divide="ignore", invalid="ignore"):
        q0 = np.rint(edge / scale).astype(f)
        nz = q0 != 0
        scale = np.where(nz, edge / np.where(nz, q0, f(1.0)), scale).astype(f)
    bias = np.where(nz, edge, f(0.0)).astype(f)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.rint((w - bias[:, None]) / scale[:, None])
    q = np.clip(q, 0.0, 15.0).astype(np.uint32)
    q = q.reshape(-1, 8)
    shifts = (np.arange(8, dtype=np.uint32) * 4)[None, :]
    codes = np.bitwise_or.reduce(q << shifts, axis=1).astype(np.uint32)
    codes = codes.reshape(*shape[:-1], d // 8)
    scales = from_f32(scale, dtype).reshape(*shape[:-1], d // GROUP)
    biases = from_f32(bias, dtype).reshape(*shape[:-1], d // GROUP)
    return codes, scales, biases


def dequantize_np(codes: np.ndarray, scales: np.ndarray, biases: np.ndarray, dtype: int = F16):
    """x = code * scale + bias (fp32), the reference's dequant4 (mlx_fused_attention.py:274-288)."""
    codes = np.asarray(codes, dtype=np.uint32)
    d = codes.shape[-1] * 8
    shifts = (np.arange(8, dtype=np.uint32) * 4)
    nib = ((codes[..., :, None] >> shifts) & 0xF).astype(np.float32).reshape(*codes.shape[:-1], d)
    s = np.repeat(to_f32(scales, dtype), GROUP, axis=-1)
    b = np.repeat(to_f32(biases, dtype), GROUP, axis=-1)
    return nib * s + b


def structured_keep(n: int, L: int, kv_start: int = 0, causal: bool = True, window: int = 0):
    """[L, n] boolean keep-mask of mlx-lm create_causal_mask (query l at position n-L+l)."""
    pos = np.arange(n - L, n)[:, None]
    r = np.arange(n)[None, :]
    keep = r >= kv_start
    if causal:
        keep = keep & (r <= pos)
    if window > 0:
        keep = keep & (r > pos - window)
    return keep


def attention_np(q, k_q4, v_q4, scale, *, sdtype=F16, kv_len=None, kv_start=None, causal=True,
                 window=0, mask=None, mask_kind=MASK_NONE, sinks=None, acc=np.float64):
    """Reference-order attention over contiguous Q4 tensors, in float64 (or `acc`).

    q: [B, Hq, L, Dk] float; k_q4/v_q4: (codes [B,Hkv,N,D/8], scales, biases).
    kv_len/kv_start: per-sequence valid length / left padding (default N / 0).
    mask: optional dense [B or 1, Hq or 1, L, N] array (bool keep-mask or additive).
    sinks: optional [Hq] sink logits appended to every row's scores before the softmax and
    dropped after it.
    Returns [B, Hq, L, Dv] in `acc` precision.
    """
    q = np.asarray(q, dtype=acc)
    B, Hq, L, Dk = q.shape
    kc = k_q4[0]
    Hkv, N = kc.shape[1], kc.shape[2]
    n_rep = Hq // Hkv
    k = dequantize_np(*k_q4, dtype=sdtype).astype(acc)
    v = dequantize_np(*v_q4, dtype=sdtype).astype(acc)
    Dv = v.shape[-1]
    out = np.zeros((B, Hq, L, Dv), dtype=acc)
    masked = acc(-65504.0)
    for b in range(B):
        n = N if kv_len is None else int(kv_len[b])
        st = 0 if kv_start is None else int(kv_start[b])
        keep = structured_keep(n, L, st, causal, window)
        for h in range(Hq):
            hk = h // n_rep
            s = (q[b, h] @ k[b, hk, :n].T) * acc(scale)
            kk = keep.copy()
            if mask is not None:
                m = np.asarray(mask)
                mb = m[min(b, m.shape[0] - 1), min(h, m.shape[1] - 1), :, :n]
                if mask_kind == MASK_BOOL:
                    kk = kk & mb.astype(bool)
                else:
                    s = s + mb.astype(acc)
            s = np.where(kk, s, masked)
            if sinks is not None:
                s = np.concatenate([s, np.full((L, 1), acc(sinks[h]))], axis=-1)
            s = s - s.max(axis=-1, keepdims=True)
            p = np.exp(s)
            p = p / p.sum(axis=-1, keepdims=True)
            out[b, h] = p[:, :n] @ v[b, hk, :n]
    return out


def attention_mlx_fp16_np(q16, k_q4, v_q4, scale, *, sdtype=F16, mask_keep=None):
    """The reference's compiled path with its fp16 intermediates (fp16 queries only).

    mlx_fused_attention.py:69-139: ``queries * scale`` in the query dtype, quantized_matmul
    returning the query dtype, where(mask, s, finfo.min), softmax(precise=True) computed in
    fp32 and returned in the query dtype, then the second quantized_matmul returning fp16.
    Used to bound the gap between the fp32-accumulating kernels and the reference's rounding.
    """
    f16 = np.float16
    q = np.asarray(q16, dtype=f16)
    B, Hq, L, Dk = q.shape
    Hkv = k_q4[0].shape[1]
    n_rep = Hq // Hkv
    k = dequantize_np(*k_q4, dtype=sdtype)
    v = dequantize_np(*v_q4, dtype=sdtype)
    qs = (q.astype(np.float32) * np.float32(f16(scale))).astype(f16)
    out = np.zeros((B, Hq, L, v.shape[-1]), dtype=f16)
    for b in range(B):
        for h in range(Hq):
            hk = h // n_rep
            s = (qs[b, h].astype(np.float32) @ k[b, hk].T).astype(f16)
            if mask_keep is not None:
                mk = mask_keep[min(b, mask_keep.shape[0] - 1), 0]
                s = np.where(mk, s, f16(-65504.0))
            sf = s.astype(np.float32)
            sf = np.exp(sf - sf.max(axis=-1, keepdims=True))
            p = (sf / sf.sum(axis=-1, keepdims=True)).astype(f16)
            out[b, h] = (p.astype(np.float32) @ v[b, hk]).astype(f16)
    return out


# --------------------------------------------------------------------------------------
# C restatement (ctypes)
# --------------------------------------------------------------------------------------


def build(force: bool = False) -> Path:
    """Compile q4_oracle.c into oracle/_build/libq4oracle.so (gcc, OpenMP)."""
    src = _HERE / "q4_oracle.c"
    if _LIB_PATH.exists() and not force and _LIB_PATH.stat().st_mtime >= src.stat().st_mtime:
        return _LIB_PATH
    _LIB_PATH.parent.mkdir(parents=True, exist_ok=True)
    cmd = ["gcc", "-O3", "-march=x86-64-v3", "-mtune=generic", "-fopenmp", "-fPIC", "-shared",
           "-Wall", "-o", str(_LIB_PATH), str(src), "-lm"]
    subprocess.run(cmd, check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _LIB_PATH if _LIB_PATH.exists() else build()
        L = ctypes.CDLL(str(path))
        p = ctypes.c_void_p
        i32, i64, f32 = ctypes.c_int, ctypes.c_int64, ctypes.c_float
        L.amo_quantize.argtypes = [p, i32, i64, i32, p, p, p]
        L.amo_quantize_f32.argtypes = [p, i32, i64, i32, p, p, p]
        L.amo_dequantize.argtypes = [p, p, p, i32, i64, i32, p]
        L.amo_attention.argtypes = [p, i32, i32, i32, i32, i32, i32, p, p, p, p, p, p, i32, i32,
                                    i64, i32, p, i32, p, p, i32, i32, i32, p, i64, i64, i64, i64,
                                    f32, p, p]
        L.amo_attention.restype = i32
        L.amo_num_threads.restype = i32
        L.amo_set_threads.argtypes = [i32]
        _lib = L
    return _lib


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def num_threads() -> int:
    return int(lib().amo_num_threads())


def set_threads(n: int) -> None:
    lib().amo_set_threads(int(n))


def quantize(x16: np.ndarray, dtype: int = F16):
    """C restatement of mx.quantize (group 64, 4 bits); same contract as quantize_np."""
    x16 = np.ascontiguousarray(np.asarray(x16).view(np.uint16))
    shape = x16.shape
    d = shape[-1]
    rows = x16.size // d
    codes = np.empty((rows, d // 8), np.uint32)
    scales = np.empty((rows, d // GROUP), np.uint16)
    biases = np.empty((rows, d // GROUP), np.uint16)
    lib().amo_quantize(_ptr(x16), dtype, rows, d, _ptr(codes), _ptr(scales), _ptr(biases))
    return (codes.reshape(*shape[:-1], d // 8), scales.reshape(*shape[:-1], d // GROUP),
            biases.reshape(*shape[:-1], d // GROUP))


def quantize_f32(x: np.ndarray, dtype: int = F16):
    """Quantize fp32 data with the same rule (scales/biases rounded to `dtype`)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    shape = x.shape
    d = shape[-1]
    rows = x.size // d
    codes = np.empty((rows, d // 8), np.uint32)
    scales = np.empty((rows, d // GROUP), np.uint16)
    biases = np.empty((rows, d // GROUP), np.uint16)
    lib().amo_quantize_f32(_ptr(x), dtype, rows, d, _ptr(codes), _ptr(scales), _ptr(biases))
    return (codes.reshape(*shape[:-1], d // 8), scales.reshape(*shape[:-1], d // GROUP),
            biases.reshape(*shape[:-1], d // GROUP))


def dequantize(codes, scales, biases, dtype: int = F16) -> np.ndarray:
    codes = np.ascontiguousarray(codes, dtype=np.uint32)
    scales = np.ascontiguousarray(np.asarray(scales).view(np.uint16))
    biases = np.ascontiguousarray(np.asarray(biases).view(np.uint16))
    d = codes.shape[-1] * 8
    rows = codes.size // (d // 8)
    out = np.empty((rows, d), np.float32)
    lib().amo_dequantize(_ptr(codes), _ptr(scales), _ptr(biases), dtype, rows, d, _ptr(out))
    return out.reshape(*codes.shape[:-1], d)


def attention(q, k_q4, v_q4, scale, *, sdtype=F16, n_kv_heads=None, layout=CONTIGUOUS,
              block_table=None, block_tokens=256, kv_len=None, kv_start=None, causal=True,
              window=0, mask=None, mask_kind=MASK_NONE, sinks=None):
    """C restatement of the attention path (fp32 accumulation, OpenMP).

    sinks: optional [Hq] attention-sink logits (in scaled-score units): each joins its
    head's softmax normaliser as one extra key with no value (mlx_sink_compat.py:46-69
    hands them to mx.fast.scaled_dot_product_attention).

    Contiguous: k_q4 = (codes [B,Hkv,cap,Dk/8], scales [B,Hkv,cap,Dk/64], biases).
    Paged:      k_q4 = (codes [num_blocks,Hkv,block_tokens,Dk/8], ...), with
                block_table [B, max_blocks] int32.
    q: [B, Hq, L, Dk] float32.  Returns float32 [B, Hq, L, Dv].
    """
    q = np.ascontiguousarray(q, dtype=np.float32)
    B, Hq, L, Dk = q.shape
    kc, ks, kb = (np.ascontiguousarray(np.asarray(a).view(np.uint32 if i == 0 else np.uint16))
                  for i, a in enumerate(k_q4))
    vc, vs, vb = (np.ascontiguousarray(np.asarray(a).view(np.uint32 if i == 0 else np.uint16))
                  for i, a in enumerate(v_q4))
    Hkv = kc.shape[1] if n_kv_heads is None else n_kv_heads
    Dv = vc.shape[-1] * 8
    if layout == CONTIGUOUS:
        cap = kc.shape[2]
        table = None
        tstride = 0
        if kv_len is None:
            kv_len = np.full(B, cap, np.int32)
    else:
        cap = kc.shape[0]
        table = np.ascontiguousarray(block_table, dtype=np.int32)
        tstride = table.shape[1]
        block_tokens = kc.shape[2]
    kv_len = np.ascontiguousarray(kv_len, dtype=np.int32)
    kv_start = None if kv_start is None else np.ascontiguousarray(kv_start, dtype=np.int32)
    mstr = (0, 0, 0, 0)
    if mask is not None:
        m = np.asarray(mask)
        if mask_kind == MASK_BOOL:
            m = m.astype(np.float32)
        m = np.ascontiguousarray(m, dtype=np.float32)
        while m.ndim < 4:
            m = m[None]
        st = [s // 4 if dim > 1 else 0 for s, dim in zip(m.strides, m.shape)]
        mstr = tuple(st)
        mask = m
    if sinks is not None:
        sinks = np.ascontiguousarray(np.asarray(sinks, dtype=np.float32).reshape(Hq))
    out = np.empty((B, Hq, L, Dv), np.float32)
    rc = lib().amo_attention(_ptr(q), B, Hq, L, Hkv, Dk, Dv, _ptr(kc), _ptr(ks), _ptr(kb),
                             _ptr(vc), _ptr(vs), _ptr(vb), sdtype, layout, cap, block_tokens,
                             _ptr(table), tstride, _ptr(kv_len), _ptr(kv_start), int(causal),
                             int(window), mask_kind, _ptr(mask), *mstr, float(scale), _ptr(sinks),
                             _ptr(out))
    if rc != 0:
        raise ValueError("block table entry out of range")
    return out


def q4_bytes_per_block_per_layer(n_kv_heads: int, head_dim: int, block_tokens: int,
                                 v_head_dim: int | None = None, bits: int = 4,
                                 group_size: int = GROUP) -> int:
    """ModelCacheSpec.bytes_per_block_per_layer (domain/value_objects.py:91-122), restated."""
    vd = head_dim if v_head_dim is None else v_head_dim
    k_el = n_kv_heads * head_dim * block_tokens
    v_el = n_kv_heads * vd * block_tokens
    total = k_el + v_el
    w = (total * bits) // 8
    groups = (k_el + group_size - 1) // group_size + (v_el + group_size - 1) // group_size
    return w + groups * 2 + groups * 2
