"""NumPy stand-in for the parts of ``mlx`` / ``mlx_lm`` that agent-memory's Q4 path calls.

Test infrastructure for tests/golden/make_golden.py only.  mlx (0.30.3) and mlx-lm
(0.30.4) are third-party dependencies of the reference that are not installed here; this
module lets the reference's OWN Python (mlx_quantized_extensions.py, mlx_fused_attention.py)
run in this container so its cache bookkeeping, padding, mask and dispatch logic produce
golden vectors.  Array values are NumPy arrays; the numeric primitives are the oracle's
restatements:

* ``quantize`` / ``dequantize``: oracle.q4_oracle (mlx's affine rule restated);
* ``quantized_matmul``: dequantize to fp32, matmul in fp32, result in the input dtype
  (mlx's qmm returns the activation dtype);
* ``softmax(precise=True)``: fp32 internally, result in the input dtype;
* mlx-lm's ``create_causal_mask`` and ``QuantizedKVCache`` (256-step growth) restated.

So the fixtures pin the reference's code paths; mlx's own kernels remain restated.
"""

from __future__ import annotations

import sys
import types

import numpy as np

from oracle import q4_oracle as orc


class _DType:
    def __init__(self, name: str, np_dtype):
        self.name = name
        self.dtype = np.dtype(np_dtype)
        self.size = self.dtype.itemsize

    def __eq__(self, other):
        try:
            return np.dtype(other) == self.dtype
        except TypeError:
            return False

    def __hash__(self):
        return hash(self.dtype)

    def __repr__(self):
        return f"mlx.core.{self.name}"


def _npdt(dt):
    return None if dt is None else np.dtype(dt)


def _tree_map(fn, tree, *rest):
    if isinstance(tree, (list, tuple)):
        out = [_tree_map(fn, t, *[r[i] for r in rest]) for i, t in enumerate(tree)]
        return type(tree)(out)
    if isinstance(tree, dict):
        return {k: _tree_map(fn, v, *[r[k] for r in rest]) for k, v in tree.items()}
    return fn(tree, *rest)


def _quantize(w, group_size=64, bits=4):
    assert group_size == 64 and bits == 4
    w = np.asarray(w)
    assert w.dtype == np.float16, "fixtures use float16 data"
    c, s, b = orc.quantize_np(w.view(np.uint16), orc.F16)
    return c, s.view(np.float16), b.view(np.float16)


def _dequantize(w, scales, biases, group_size=64, bits=4):
    assert group_size == 64 and bits == 4
    return orc.dequantize_np(w, np.asarray(scales).view(np.uint16), np.asarray(biases).view(np.uint16),
                             orc.F16).astype(np.asarray(scales).dtype)


def _quantized_matmul(x, w, scales, biases, transpose=True, group_size=64, bits=4):
    W = orc.dequantize_np(w, np.asarray(scales).view(np.uint16), np.asarray(biases).view(np.uint16),
                          orc.F16)
    xf = np.asarray(x).astype(np.float32)
    out = xf @ np.swapaxes(W, -1, -2) if transpose else xf @ W
    return out.astype(np.asarray(x).dtype)


def _softmax(x, axis=-1, precise=False):
    x = np.asarray(x)
    xf = x.astype(np.float32)
    xf = xf - xf.max(axis=axis, keepdims=True)
    e = np.exp(xf)
    return (e / e.sum(axis=axis, keepdims=True)).astype(x.dtype)


def create_causal_mask(N, offset=0, window_size=None, right_padding=None, left_padding=None):
    rinds = np.arange(offset + N)
    linds = np.arange(offset, offset + N) if offset else rinds
    linds = linds[:, None]
    rinds = rinds[None]
    mask = linds >= rinds
    if window_size is not None:
        mask = mask & (linds < rinds + window_size)
    if right_padding is not None:
        mask = mask & (rinds < np.expand_dims((offset + N) - np.asarray(right_padding), (1, 2, 3)))
    if left_padding is not None:
        mask = mask & (np.expand_dims(np.asarray(left_padding), (1, 2, 3)) <= rinds)
    return mask


class _BaseCache:
    pass


class QuantizedKVCache(_BaseCache):
    """mlx-lm QuantizedKVCache (256-step capacity growth), restated over NumPy."""

    step = 256

    def __init__(self, group_size: int = 64, bits: int = 8):
        self.keys = None
        self.values = None
        self.offset = 0
        self.group_size = group_size
        self.bits = bits

    def update_and_fetch(self, keys, values):
        B, H, num_steps, kd = keys.shape
        vd = values.shape[-1]
        prev = self.offset
        if self.keys is None or prev + num_steps > self.keys[0].shape[-2]:
            el_per_int = 8 * 4 // self.bits
            new_steps = (self.step + num_steps - 1) // self.step * self.step
            shape = (B, H, new_steps)

            def init_quant(dim):
                return (np.zeros((*shape, dim // el_per_int), np.uint32),
                        np.zeros((*shape, dim // self.group_size), keys.dtype),
                        np.zeros((*shape, dim // self.group_size), keys.dtype))

            def expand_quant(x):
                return np.concatenate([x, np.zeros((*shape, x.shape[-1]), x.dtype)], axis=-2)

            if self.keys is not None:
                if prev % self.step != 0:
                    self.keys, self.values = _tree_map(lambda x: x[..., :prev, :],
                                                       (self.keys, self.values))
                self.keys, self.values = _tree_map(expand_quant, (self.keys, self.values))
            else:
                self.keys, self.values = init_quant(kd), init_quant(vd)
        self.offset += num_steps
        qk = _quantize(keys, self.group_size, self.bits)
        qv = _quantize(values, self.group_size, self.bits)
        for i in range(3):
            self.keys[i][..., prev:self.offset, :] = qk[i]
            self.values[i][..., prev:self.offset, :] = qv[i]
        return _tree_map(lambda x: x[..., :self.offset, :], (self.keys, self.values))

    def size(self):
        return 0

    def make_mask(self, N=1, return_array=False, window_size=None, **kw):
        if N == 1:
            return None
        return "causal"

    def trim(self, n):
        n = min(self.offset, n)
        self.offset -= n
        return n


def _original_qsdpa(queries, q_keys, q_values, scale, mask, group_size=64, bits=4):
    B, Hq, L, D = queries.shape
    Hkv = q_keys[0].shape[-3]
    n_rep = Hq // Hkv
    queries = queries * np.asarray(scale, dtype=queries.dtype)
    if n_rep > 1:
        queries = queries.reshape(B, Hkv, n_rep, L, D)
        q_keys = _tree_map(lambda x: np.expand_dims(x, -3), q_keys)
        q_values = _tree_map(lambda x: np.expand_dims(x, -3), q_values)
    scores = _quantized_matmul(queries, *q_keys, transpose=True, group_size=group_size, bits=bits)
    if mask is not None:
        if isinstance(mask, str):
            qL, kL = scores.shape[-2:]
            mask = np.arange(kL - qL, kL)[:, None] >= np.arange(kL)[None]
        if mask.dtype == np.bool_:
            scores = np.where(mask, scores, np.finfo(scores.dtype).min)
        else:
            scores = scores + mask
    scores = _softmax(scores, axis=-1, precise=True)
    out = _quantized_matmul(scores, *q_values, transpose=False, group_size=group_size, bits=bits)
    if n_rep > 1:
        out = out.reshape(B, Hq, L, -1)
    return out


class _Array:
    """mx.array: a type (annotations such as ``mx.array | tuple`` are evaluated at import)
    whose construction returns a NumPy array."""

    def __new__(cls, x, dtype=None):
        return np.array(x, dtype=_npdt(dtype))


def _fast_sdpa(queries, keys, values, scale, mask=None, sinks=None):
    """mx.fast.scaled_dot_product_attention as documented: GQA by head repetition, boolean
    masks keep True, additive masks add, "causal" aligns the last query with the last key,
    and each head's sink logit joins the softmax as one extra column with no value.
    Computed in fp32, returned in the query dtype."""
    q = np.asarray(queries)
    B, Hq, L, _ = q.shape
    Hkv = np.asarray(keys).shape[1]
    n_rep = Hq // Hkv
    k = np.repeat(np.asarray(keys, dtype=np.float32), n_rep, axis=1)
    v = np.repeat(np.asarray(values, dtype=np.float32), n_rep, axis=1)
    s = (q.astype(np.float32) * np.float32(scale)) @ np.swapaxes(k, -1, -2)
    if mask is not None:
        if isinstance(mask, str):
            kL = s.shape[-1]
            mask = np.arange(kL - L, kL)[:, None] >= np.arange(kL)[None]
        mask = np.asarray(mask)
        if mask.dtype == np.bool_:
            s = np.where(mask, s, -np.inf)
        else:
            s = s + mask.astype(np.float32)
    if sinks is not None:
        sk = np.broadcast_to(np.asarray(sinks, dtype=np.float32).reshape(1, Hq, 1, 1), (B, Hq, L, 1))
        s = np.concatenate([s, sk], axis=-1)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(axis=-1, keepdims=True)
    if sinks is not None:
        p = p[..., :-1]
    return (p @ v).astype(q.dtype)


def install() -> types.SimpleNamespace:
    """Register the stand-in modules in sys.modules; returns the mlx_lm.models.base module."""
    core = types.ModuleType("mlx.core")
    core.uint32 = _DType("uint32", np.uint32)
    core.int32 = _DType("int32", np.int32)
    core.float16 = _DType("float16", np.float16)
    core.float32 = _DType("float32", np.float32)
    core.bfloat16 = _DType("bfloat16", np.float32)  # unused by the fixtures (no NumPy bf16)
    core.bool_ = _DType("bool_", np.bool_)
    core.array = _Array
    core.zeros = lambda shape, dtype=core.float32: np.zeros(shape, dtype=_npdt(dtype))
    core.concatenate = lambda arrs, axis=0: np.concatenate(arrs, axis=axis)
    core.eval = lambda *a, **k: None
    core.async_eval = core.eval
    core.synchronize = lambda *a, **k: None
    core.contiguous = lambda x: np.ascontiguousarray(x)
    core.arange = lambda *a, **k: np.arange(*a)
    core.where = np.where
    core.finfo = lambda dt: np.finfo(_npdt(dt))
    core.softmax = _softmax
    core.reshape = lambda x, shape: np.reshape(x, shape)
    core.expand_dims = lambda x, axis: np.expand_dims(x, axis)
    core.quantize = _quantize
    core.dequantize = _dequantize
    core.quantized_matmul = _quantized_matmul
    core.compile = lambda fn=None, shapeless=False: fn
    core.fast = types.SimpleNamespace(metal_kernel=None, scaled_dot_product_attention=_fast_sdpa)
    mlx = types.ModuleType("mlx")
    mlx.core = core
    utils = types.ModuleType("mlx.utils")
    utils.tree_map = _tree_map
    mlx.utils = utils
    mlx_lm = types.ModuleType("mlx_lm")
    models = types.ModuleType("mlx_lm.models")
    cache = types.ModuleType("mlx_lm.models.cache")
    cache._BaseCache = _BaseCache
    cache.QuantizedKVCache = QuantizedKVCache
    base = types.ModuleType("mlx_lm.models.base")
    base.create_causal_mask = create_causal_mask
    base.quantized_scaled_dot_product_attention = _original_qsdpa
    base.scaled_dot_product_attention = None  # replaced by the reference's sink patch
    mlx_lm.models = models
    models.cache = cache
    models.base = base
    sys.modules.update({"mlx": mlx, "mlx.core": core, "mlx.utils": utils, "mlx_lm": mlx_lm,
                        "mlx_lm.models": models, "mlx_lm.models.cache": cache,
                        "mlx_lm.models.base": base})
    return base
