"""Generate the golden fixtures in tests/golden/ (run in the build container only).

    python tests/golden/make_golden.py [--reference /path/to/agent-memory]

Three kinds of fixtures:

* ``quantize_*.npz``: oracle restatement of mx.quantize on seeded data (regression pins
  of the restatement; the GPU kernels are checked bit-for-bit against them).
* ``ref_*.npz`` / ``ref_block_pool.json``: outputs of the REFERENCE's own Python code run
  here: BatchQuantizedKVCache (mlx_quantized_extensions.py) driven through merge /
  update_and_fetch / make_mask / extend / filter / extract / trim, the patched
  quantized SDPA of mlx_fused_attention.py (op order, GQA reshape, mask handling, batch
  split), the sink shim of mlx_sink_compat.py, and BlockPool (domain/services.py).  mlx is not installed, so the reference runs
  over tests/golden/mlx_standin.py (NumPy arrays, oracle numerics).
* nothing here is read at test time except the .npz/.json files.
"""

from __future__ import annotations

import argparse
import importlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

from oracle import q4_oracle as orc  # noqa: E402


def f16(rng, *shape):
    return rng.standard_normal(shape).astype(np.float16)


def quantize_fixtures():
    rng = np.random.default_rng(2024)
    x = f16(rng, 64, 128) * np.float16(3)
    x[0] = 0
    x[1] = 1.5
    x[2, 5] = 60000
    c, s, b = orc.quantize(x.view(np.uint16), orc.F16)
    np.savez_compressed(HERE / "quantize_f16.npz", kind="quantize", dtype=orc.F16,
                        x=x.view(np.uint16), codes=c, scales=s, biases=b)
    xb = orc.f32_to_bf16_bits(rng.standard_normal((64, 192)).astype(np.float32) * 5)
    c, s, b = orc.quantize(xb, orc.BF16)
    np.savez_compressed(HERE / "quantize_bf16.npz", kind="quantize", dtype=orc.BF16, x=xb,
                        codes=c, scales=s, biases=b)


def _q4(a):
    return {"c": np.asarray(a[0], np.uint32), "s": np.asarray(a[1]).view(np.uint16),
            "b": np.asarray(a[2]).view(np.uint16)}


def cache_lifecycle(ext, cache_mod):
    """Drive the reference's BatchQuantizedKVCache and record every observable state."""
    rng = np.random.default_rng(7)
    H, D = 2, 128
    rec: dict[str, np.ndarray] = {}
    meta: list[dict] = []
    inputs: dict[str, np.ndarray] = {}

    def snap(tag, c):
        st = {"tag": tag, "idx": int(c._idx), "offset": np.asarray(c.offset).tolist(),
              "left_padding": np.asarray(c.left_padding).tolist(),
              "capacity": None if c.keys is None else int(c.keys[0].shape[-2])}
        meta.append(st)
        if c.keys is not None:
            k, v = c.state[0], c.state[1]
            for nm, q in (("k", k), ("v", v)):
                for part, arr in _q4(q).items():
                    rec[f"{tag}_{nm}{part}"] = arr

    def tok(name, b, n):
        k, v = f16(rng, b, H, n, D), f16(rng, b, H, n, D)
        inputs[f"in_{name}_k"] = k.view(np.uint16)
        inputs[f"in_{name}_v"] = v.view(np.uint16)
        return k, v

    # single-sequence caches (mlx-lm QuantizedKVCache, 4-bit)
    c1 = cache_mod.QuantizedKVCache(group_size=64, bits=4)
    c1.update_and_fetch(*tok("c1", 1, 5))
    c2 = cache_mod.QuantizedKVCache(group_size=64, bits=4)
    c2.update_and_fetch(*tok("c2", 1, 9))
    batch = ext.BatchQuantizedKVCache.merge([c1, c2])
    snap("merge", batch)
    mask = batch.make_mask(1)
    rec["mask_after_merge"] = np.asarray(mask)
    batch.update_and_fetch(*tok("u1", 2, 1))
    snap("update1", batch)
    mask = batch.make_mask(3, window_size=6)
    rec["mask_window"] = np.asarray(mask)
    batch.update_and_fetch(*tok("u2", 2, 3))
    snap("update2", batch)
    c4 = cache_mod.QuantizedKVCache(group_size=64, bits=4)
    c4.update_and_fetch(*tok("c4", 1, 20))
    other = ext.BatchQuantizedKVCache.merge([c4])
    snap("other", other)
    batch.extend(other)
    snap("extend", batch)
    batch.filter([0, 2])
    snap("filter", batch)
    e = batch.extract(1)
    rec["extract_kc"], rec["extract_ks"], rec["extract_kb"] = (_q4(e.keys)[p] for p in "csb")
    rec["extract_vc"], rec["extract_vs"], rec["extract_vb"] = (_q4(e.values)[p] for p in "csb")
    meta.append({"tag": "extract", "offset": int(e.offset)})
    batch.trim(2)
    snap("trim", batch)
    batch.update_and_fetch(*tok("u3", 2, 300))  # crosses the 256-step capacity growth
    snap("update3", batch)
    np.savez_compressed(HERE / "ref_cache_lifecycle.npz", kind="cache_lifecycle",
                        meta=json.dumps(meta), **rec, **inputs)


def sdpa_cases(fused, base, ext, cache_mod):
    """The reference's patched quantized SDPA on seeded inputs."""
    assert fused.apply_fused_attention_patch() is True
    sdpa = base.quantized_scaled_dot_product_attention
    rng = np.random.default_rng(11)
    cases = {}

    def q4(b, h, n, d):
        x = f16(rng, b, h, n, d)
        return orc.quantize_np(x.view(np.uint16), orc.F16)

    def as_mx(t):
        return (t[0], t[1].view(np.float16), t[2].view(np.float16))

    def run(name, B, Hq, Hkv, N, dk, dv, L, mask, scale):
        k, v = q4(B, Hkv, N, dk), q4(B, Hkv, N, dv)
        q = f16(rng, B, Hq, L, dk)
        out = sdpa(q, as_mx(k), as_mx(v), scale=scale, mask=mask)
        arrays = {"q": q.view(np.uint16), "kc": k[0], "ks": k[1], "kb": k[2], "vc": v[0],
                  "vs": v[1], "vb": v[2], "out": np.asarray(out).view(np.uint16),
                  "scale": np.float32(scale)}
        if isinstance(mask, str):
            arrays["mask_str"] = mask
        elif mask is not None:
            arrays["mask"] = np.asarray(mask)
        cases[name] = arrays

    run("gqa_decode", 2, 8, 2, 100, 128, 128, 1, None, 128 ** -0.5)
    run("mha_prefill_causal", 1, 4, 4, 80, 128, 128, 16, "causal", 0.09)
    run("mla_decode", 2, 4, 4, 70, 192, 128, 1, None, 192 ** -0.5)
    run("asym_k128_v64", 1, 4, 2, 50, 128, 64, 1, None, 0.1)
    bc = ext.BatchQuantizedKVCache(left_padding=[0, 7])
    bc._idx = 39
    run("leftpad_window_bool", 2, 8, 4, 40, 128, 128, 1, bc.make_mask(1, window_size=16), 0.088)
    add = (rng.standard_normal((1, 1, 4, 60)) * 2).astype(np.float16)
    run("additive_mask", 1, 4, 1, 60, 64, 64, 4, add, 0.125)
    for name, arrays in cases.items():
        np.savez_compressed(HERE / f"ref_sdpa_{name}.npz", kind="ref_sdpa", **arrays)


def sink_cases(base):
    """The reference's sink shim (mlx_sink_compat.py:36-69: dequantize the Q4 tuples, then
    fast SDPA with sinks) on seeded GPT-OSS-shaped inputs (head_dim 64, n_rep 8)."""
    importlib.import_module("agent_memory.adapters.outbound.mlx_sink_compat")  # patches on import
    sdpa = base.scaled_dot_product_attention
    rng = np.random.default_rng(23)
    cache = type("Q4Cache", (), {"bits": 4, "group_size": 64})()

    def run(name, B, Hq, Hkv, N, D, L, mask, scale):
        k = orc.quantize_np(f16(rng, B, Hkv, N, D).view(np.uint16), orc.F16)
        v = orc.quantize_np(f16(rng, B, Hkv, N, D).view(np.uint16), orc.F16)
        q = f16(rng, B, Hq, L, D)
        sinks = (rng.standard_normal(Hq) * 2).astype(np.float32)
        as_mx = lambda t: (t[0], t[1].view(np.float16), t[2].view(np.float16))  # noqa: E731
        out = sdpa(q, as_mx(k), as_mx(v), cache, scale=scale, mask=mask, sinks=sinks)
        arrays = {"q": q.view(np.uint16), "kc": k[0], "ks": k[1], "kb": k[2], "vc": v[0],
                  "vs": v[1], "vb": v[2], "out": np.asarray(out).view(np.uint16),
                  "scale": np.float32(scale), "sinks": sinks}
        if isinstance(mask, str):
            arrays["mask_str"] = mask
        elif mask is not None:
            arrays["mask"] = np.asarray(mask)
        np.savez_compressed(HERE / f"ref_sinks_{name}.npz", kind="ref_sinks", **arrays)

    run("decode", 2, 16, 2, 90, 64, 1, None, 0.125)
    run("prefill_causal", 1, 16, 2, 70, 64, 8, "causal", 0.125)
    keep = np.zeros((1, 1, 1, 100), dtype=bool)
    keep[..., 100 - 32:] = True  # a 32-key sliding window for the one query
    run("window_bool", 1, 8, 1, 100, 64, 1, keep, 0.125)


def block_pool_ops(services, vo):
    spec = vo.ModelCacheSpec(n_layers=4, n_kv_heads=8, head_dim=128, block_tokens=256,
                             layer_types=["global"] * 4)
    pool = services.BlockPool(spec=spec, total_blocks=32)
    log = []
    a = pool.allocate(3, 0, "a")
    log.append(["alloc", "a", 0, [blk.block_id for blk in a]])
    b = pool.allocate(5, 2, "b")
    log.append(["alloc", "b", 2, [blk.block_id for blk in b]])
    pool.free(a[1:2], "a")
    log.append(["free", "a", [a[1].block_id]])
    c = pool.allocate(2, 1, "c")
    log.append(["alloc", "c", 1, [blk.block_id for blk in c]])
    log.append(["free_agent", "b", pool.free_agent_blocks("b")])
    d = pool.allocate(4, 3, "d")
    log.append(["alloc", "d", 3, [blk.block_id for blk in d]])
    log.append(["state", pool.available_blocks(), pool.allocated_block_count(), pool.used_memory(),
                pool.max_batch_size(600)])
    (HERE / "ref_block_pool.json").write_text(json.dumps(log, indent=1))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="checkout of the agent-memory repository whose src/ is imported")
    args = ap.parse_args()
    quantize_fixtures()
    import mlx_standin

    base = mlx_standin.install()
    sys.path.insert(0, str(Path(args.reference) / "src"))
    ext = importlib.import_module("agent_memory.adapters.outbound.mlx_quantized_extensions")
    fused = importlib.import_module("agent_memory.adapters.outbound.mlx_fused_attention")
    services = importlib.import_module("agent_memory.domain.services")
    vo = importlib.import_module("agent_memory.domain.value_objects")
    cache_mod = sys.modules["mlx_lm.models.cache"]
    assert ext.validate_q4_pipeline() is True
    cache_lifecycle(ext, cache_mod)
    sdpa_cases(fused, base, ext, cache_mod)
    sink_cases(base)
    block_pool_ops(services, vo)
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
